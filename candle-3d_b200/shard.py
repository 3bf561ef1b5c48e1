"""Row sharding across ranks (one process per GPU).

Every per-token op is independent per row, so rank r of W owns the contiguous
row range `shard_range(n, W, r)` and runs the fused kernels on it with no
communication.  `gather_rows` is the optional final all-gather of the block
outputs (uneven shards are padded to the largest shard for the collective and
trimmed afterwards); it works with any torch.distributed backend (NCCL on the
GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's rows; the first n % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_rows(local: torch.Tensor, n: int, world: int, group=None) -> torch.Tensor:
    """All-gather row shards [rows_r, ...] into the full [n, ...] tensor on every rank."""
    if world == 1:
        return local
    cap = shard_range(n, world, 0)[1]  # the largest shard
    padded = local.new_zeros((cap,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    out = local.new_empty((world * cap,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, padded, group=group)
    parts = [out[r * cap: r * cap + (shard_range(n, world, r)[1] - shard_range(n, world, r)[0])]
             for r in range(world)]
    return torch.cat(parts, 0)


# ------------------------------------------------------ interleaved row blocks
def interleaved_block(chunk: int, world: int, rank: int, rows_per_chunk: int) -> tuple[int, int]:
    """Global [start, end) of rank's `chunk`-th block when ranks own row blocks
    round-robin: block c of rank r is global rows (c * world + r) * rows_per_chunk
    onward.  With this ownership the all-gather of every rank's chunk c fills
    one contiguous range of the global row order, so the final gather can run
    chunk by chunk, overlapped with the computation of the next chunk."""
    start = (chunk * world + rank) * rows_per_chunk
    return start, start + rows_per_chunk


def gather_chunk(out: torch.Tensor, local_chunk: torch.Tensor, chunk: int, world: int,
                 group=None) -> None:
    """All-gather every rank's block `chunk` ([rows_per_chunk, ...], contiguous)
    into its place in the global [world * chunks * rows_per_chunk, ...] output."""
    rc = local_chunk.shape[0]
    dist.all_gather_into_tensor(out[chunk * world * rc:(chunk + 1) * world * rc], local_chunk,
                                group=group)


# --------------------------------------------------- one scene across ranks
class SceneSplit:
    """One scene's tokens split across the ranks of a process group, for the
    attention layers that mix all tokens (VGGT global blocks,
    crate/runtime/vggt.rs:299-311).  Rank r owns a contiguous slab of the
    scene's token sequence (whole views: frame blocks need no communication).
    A global attention is computed head-parallel: each rank sends the q, k, v
    of its tokens for head group j (H / world heads) to rank j, attends over
    all tokens for its own head group, and sends each token slab's outputs back
    to its owner (two all-to-alls, about (3 + 1) / world of the layer's q/k/v/o
    bytes crossing NVLink per rank, instead of an all-gather of every rank's K
    and V)."""

    def __init__(self, group=None, world: int | None = None, rank: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if world is None else world
        self.rank = dist.get_rank(group) if rank is None else rank

    def all_to_all(self, send: torch.Tensor) -> torch.Tensor:
        """Block j of dim 0 goes to rank j; block j of the result came from rank j."""
        if self.world == 1:
            return send
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send.contiguous(), group=self.group)
        return recv

    def exchange_qkv(self, send: torch.Tensor):
        """send [world, L, 3, h, D]: this rank's L tokens, head group j at [j].
        Returns q, k, v as [1, h, world * L, D] views over all tokens of this
        rank's head group (token order = rank order = the scene's order)."""
        world, L, three, h, D = send.shape
        r = self.all_to_all(send).view(world * L, 3, h, D)
        return tuple(r[:, i].permute(1, 0, 2).unsqueeze(0) for i in range(3))

    def return_heads(self, out_tokens: torch.Tensor) -> torch.Tensor:
        """out_tokens [world * L, h, D] (this head group's output, token-major)
        -> [L, world * h * D] rows of this rank's tokens, channel = head * D + d."""
        Lall, h, D = out_tokens.shape
        L = Lall // self.world
        r = self.all_to_all(out_tokens).view(self.world, L, h, D)
        return r.permute(1, 0, 2, 3).reshape(L, self.world * h * D)

    # ---- slabs of unequal length (rank j owns counts[j] tokens)
    #
    # With `groups` = G < world head groups (H not divisible by the ranks; G
    # divides world), the ranks form world / G query blocks of G consecutive
    # ranks: rank r attends head group r % G for the queries of its block's
    # tokens (the slabs of ranks [b G, (b + 1) G), b = r // G) over all keys.
    # Each token's q / k / v of head group j then go to the world / G ranks
    # that attend group j, and each rank gets its tokens' outputs back from
    # the G ranks of its own block.  G = world is the plain head-parallel case.
    def _groups(self, groups):
        G = self.world if groups is None else int(groups)
        if G <= 0 or self.world % G:
            raise ValueError(f"{G} head groups do not tile {self.world} ranks")
        return G

    def query_block(self, counts, groups=None) -> tuple[int, int]:
        """Token range [start, end) of this rank's query block."""
        G = self._groups(groups)
        b = self.rank // G
        return int(sum(counts[:b * G])), int(sum(counts[:(b + 1) * G]))

    def exchange_qkv_uneven(self, send: torch.Tensor, counts, groups=None):
        """As exchange_qkv when the ranks' slabs differ in length: send
        [G, L, 3, h, D] with L = counts[rank] (head group j at [j]); returns
        q over this rank's query block [1, h, block tokens, D] and k, v over
        all tokens [1, h, sum(counts), D] (token order = rank order)."""
        G = self._groups(groups)
        g, L, three, h, D = send.shape
        total = int(sum(counts))
        if self.world == 1:
            r = send.view(L, 3, h, D)
        else:
            if G < self.world:  # head group r % G for every destination rank r
                idx = torch.arange(self.world, device=send.device) % G
                send = send.index_select(0, idx)
            r = send.new_empty((total, 3, h, D))
            dist.all_to_all_single(r, send.contiguous().view(self.world * L, 3, h, D),
                                   output_split_sizes=list(counts),
                                   input_split_sizes=[L] * self.world, group=self.group)
        q0, q1 = self.query_block(counts, G)
        q = r[q0:q1, 0].permute(1, 0, 2).unsqueeze(0)
        return (q,) + tuple(r[:, i].permute(1, 0, 2).unsqueeze(0) for i in (1, 2))

    def return_heads_uneven(self, out_tokens: torch.Tensor, counts, groups=None) -> torch.Tensor:
        """As return_heads for unequal slabs: out_tokens [block tokens, h, D]
        (this rank's head group over its query block) -> [counts[rank],
        G * h * D] rows of this rank's tokens, channel = head * D + d."""
        G = self._groups(groups)
        _, h, D = out_tokens.shape
        L = int(counts[self.rank])
        if self.world == 1:
            return out_tokens.reshape(L, h * D)
        b = self.rank // G
        mine = [i // G == b for i in range(self.world)]
        r = out_tokens.new_empty((G * L, h, D))
        dist.all_to_all_single(r, out_tokens.contiguous(),
                               output_split_sizes=[L if m else 0 for m in mine],
                               input_split_sizes=[int(counts[i]) if m else 0
                                                  for i, m in enumerate(mine)],
                               group=self.group)
        return r.view(G, L, h, D).permute(1, 0, 2, 3).reshape(L, G * h * D)

    def all_gather_rows(self, local: torch.Tensor) -> torch.Tensor:
        """[L, ...] slabs of every rank -> [world * L, ...] in rank order."""
        if self.world == 1:
            return local
        out = local.new_empty((self.world * local.shape[0],) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        return out


# ------------------------------------------- batch elements x token slabs
class BatchTokenSplit:
    """A batch of `batch` sequences, each `1 + L` tokens long (one prefix token,
    then L rows whose outputs are kept), spread over `world` ranks: batch
    element b goes to the `world / batch` consecutive ranks of group b, which
    split its token sequence into slabs (shard_range).  This is the TripoSG
    CFG split (crate/runtime/triposg_dit.rs:619-621: the [uncond, cond]
    batch of 2, each element an independent DiT forward) and, with more than
    one rank per element, the token split of each element.

    `rows(rank)` gives a rank's batch element and its slab of the L kept rows
    [lo, hi) (the slab of rank 0 of a group starts with the prefix token,
    which is not one of them); `counts` the slab lengths of the group's ranks
    (prefix included) for SceneSplit's uneven exchange."""

    def __init__(self, batch: int, L: int, world: int):
        if batch <= 0 or world <= 0 or world % batch:
            raise ValueError(f"{world} ranks do not split a batch of {batch}")
        self.batch, self.L, self.world = batch, L, world
        self.per = world // batch
        self.counts = [shard_range(1 + L, self.per, r)[1] - shard_range(1 + L, self.per, r)[0]
                       for r in range(self.per)]

    def rows(self, rank: int) -> tuple[int, int, int, bool]:
        """(batch element, lo, hi, holds the prefix token) of `rank`."""
        b, g = divmod(rank, self.per)
        a0, a1 = shard_range(1 + self.L, self.per, g)
        return b, max(a0 - 1, 0), a1 - 1, a0 == 0

    def groups(self):
        """The ranks of each batch element's group, in batch order."""
        return [list(range(b * self.per, (b + 1) * self.per)) for b in range(self.batch)]

    def gather(self, local: torch.Tensor, group=None) -> torch.Tensor:
        """local [hi - lo, F] rows of this rank -> [batch, L, F] on every rank
        (one all-gather of row blocks padded to the longest slab)."""
        F = local.shape[-1]
        if self.world == 1:
            return local.reshape(1, self.L, F)
        spans = [self.rows(r)[1:3] for r in range(self.world)]
        cap = max(hi - lo for lo, hi in spans)
        padded = local.new_zeros((cap, F))
        padded[: local.shape[0]] = local
        out = local.new_empty((self.world * cap, F))
        dist.all_gather_into_tensor(out, padded, group=group)
        parts = [out[r * cap: r * cap + hi - lo] for r, (lo, hi) in enumerate(spans)]
        return torch.cat(parts, 0).view(self.batch, self.L, F)


# ------------------------------------------ gather buffers in peer memory
class _CudaArray:
    """Raw device memory described through __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape),
                                         "typestr": typestr, "strides": None, "version": 3}


class PeerRows:
    """A [world * rows, C] gather buffer on every rank, each mapped into every
    other rank's address space with CUDA IPC, so a kernel on rank r can store
    its `rows` output rows straight into block r of every rank's buffer over
    NVLink (`dest(p)` is that block on rank p).  Collective: every rank of
    `group` constructs it together; `ok` is False on every rank when any rank
    could not map a peer's buffer.  `close()` (also collective) unmaps and
    frees."""

    def __init__(self, rows: int, C: int, dtype, device, group=None):
        from cuda.bindings import runtime as rt

        self.rt = rt
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.C, self.dtype = rows, C, dtype
        self.device = torch.device(device)
        esize = torch.empty((), dtype=dtype).element_size()
        self.nbytes = self.world * rows * C * esize

        def ok(res):
            err = res[0] if isinstance(res, tuple) else res
            if int(err) != 0:
                raise RuntimeError(f"CUDA runtime error {err}")
            return res[1] if isinstance(res, tuple) and len(res) > 1 else None

        self._ok = ok
        self.error = None
        self.base = None
        mine = None
        try:
            ok(rt.cudaSetDevice(self.device.index))
            self.base = ok(rt.cudaMalloc(self.nbytes))
            mine = bytes(ok(rt.cudaIpcGetMemHandle(self.base)).reserved)
        except RuntimeError as e:  # recorded; every rank learns of it below
            self.error = f"rank {self.rank} cannot export its buffer: {e}"
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self.ptrs = []
        for p in range(self.world):
            if p == self.rank:
                self.ptrs.append(None if self.base is None else int(self.base))
                continue
            if handles[p] is None or self.base is None:
                self.ptrs.append(None)
                continue
            try:
                h = rt.cudaIpcMemHandle_t()
                h.reserved = handles[p]
                self.ptrs.append(int(ok(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess))))
            except RuntimeError as e:  # recorded; every rank learns of it below
                self.error = f"rank {self.rank} cannot map rank {p}'s buffer: {e}"
                self.ptrs.append(None)
        # All ranks agree whether every mapping exists (a rank that failed
        # alone must not leave the others waiting in a later collective).
        good = self.error is None and all(h is not None for h in handles)
        flag = torch.tensor([1 if good else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        self.ok = bool(flag.item())
        self.local = None
        if self.ok:
            n16 = self.nbytes // 2
            raw = torch.as_tensor(_CudaArray(self.base, (n16,), "<i2"), device=self.device)
            self.local = raw.view(dtype).view(self.world * rows, C)  # this rank's gathered rows

    def dest(self, p: int):
        """(device pointer, element offset) of this rank's block in rank p's buffer."""
        return self.ptrs[p], self.rank * self.rows * self.C

    def close(self):
        dist.barrier(group=self.group)
        for p, ptr in enumerate(self.ptrs):
            if p != self.rank and ptr is not None:
                self._ok(self.rt.cudaIpcCloseMemHandle(ptr))
        dist.barrier(group=self.group)
        self.local = None
        if self.base is not None:
            self._ok(self.rt.cudaFree(self.base))
