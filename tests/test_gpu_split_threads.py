"""GPU parity of the multi-rank block-stack splits on ONE GPU: the W ranks run
as W host threads that share the device's default stream, and the collectives
that `shard.py` issues (all_to_all_single with even or uneven splits,
all_gather_into_tensor, per-group communicators) are served by an in-process
stand-in for torch.distributed that copies between the ranks' tensors after a
host barrier.  Every kernel is the one a real multi-GPU run launches; only the
transport differs.  Each split stack is compared with the same input run
unsplit (relative L2 below 2e-2, the stacks' bf16 tolerance), covering the
VGGT scene split (views, head-parallel global blocks), the TRELLIS.2
voxel-row split (uneven slabs, shared head groups) and the TripoSG CFG batch
split with token slabs inside each element (crate/runtime/vggt.rs:299-311,
crate/runtime/trellis2_dit.rs:549-574, crate/runtime/triposg_dit.rs:619-621).

The threads wait for one another only on the host (a barrier with a timeout
that raises), never inside a kernel."""
import threading

import pytest

pytestmark = pytest.mark.gpu


class _Hub:
    def __init__(self, n):
        self.slots = [None] * n
        self.bar = threading.Barrier(n, timeout=120)


class ThreadDist:
    """The torch.distributed calls shard.py makes, for ranks that are threads
    of one process on one GPU (one stream, so host order is device order)."""

    def __init__(self, world, device):
        self.world, self.device = world, device
        self.local = threading.local()
        self.hubs = {}
        self.lock = threading.Lock()

    def _members(self, group):
        return tuple(range(self.world)) if group is None else tuple(group)

    def _hub(self, group):
        m = self._members(group)
        with self.lock:
            if m not in self.hubs:
                self.hubs[m] = _Hub(len(m))
            return self.hubs[m], m.index(self.local.rank), len(m)

    def get_world_size(self, group=None):
        return len(self._members(group))

    def get_rank(self, group=None):
        return self._members(group).index(self.local.rank)

    def new_group(self, ranks):
        return tuple(ranks)

    def all_to_all_single(self, out, inp, output_split_sizes=None, input_split_sizes=None,
                          group=None):
        hub, me, n = self._hub(group)
        sizes = list(input_split_sizes) if input_split_sizes is not None else [inp.shape[0] // n] * n
        hub.slots[me] = (inp, sizes)
        hub.bar.wait()
        o = 0
        for src in range(n):
            t, s = hub.slots[src]
            off, ln = sum(s[:me]), s[me]
            out[o:o + ln].copy_(t[off:off + ln])
            o += ln
        assert o == out.shape[0]
        hub.bar.wait()

    def all_gather_into_tensor(self, out, inp, group=None):
        hub, me, n = self._hub(group)
        hub.slots[me] = (inp, None)
        hub.bar.wait()
        k = inp.shape[0]
        for src in range(n):
            out[src * k:(src + 1) * k].copy_(hub.slots[src][0])
        hub.bar.wait()


def run_ranks(fake, fn):
    """fn(rank) on `fake.world` threads; returns the results in rank order."""
    out, err = [None] * fake.world, []

    def body(r):
        import torch

        fake.local.rank = r
        try:
            torch.cuda.set_device(fake.device)  # the thread's CUDA context
            out[r] = fn(r)
        except BaseException as e:  # noqa: BLE001 - re-raised below
            err.append(e)
            for hub in list(fake.hubs.values()):
                hub.bar.abort()

    ts = [threading.Thread(target=body, args=(r,)) for r in range(fake.world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=600)
    if err:
        raise err[0]
    return out


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


@pytest.fixture
def shard_threads(pkg, dev, monkeypatch):
    """Installs ThreadDist in shard.py, and makes each C-ABI call submit its
    launches as one unit: a layer's cached workspace (the dequant-linear's
    staged activations) is shared by the threads that run the same layer, and
    on one stream a call whose launches are not interleaved with another
    thread's finishes with it before the next call starts."""
    from candle3d_b200 import ops, shard

    lock = threading.Lock()
    call = ops.call

    def locked_call(*args):
        with lock:
            return call(*args)

    monkeypatch.setattr(ops, "call", locked_call)

    def make(world):
        fake = ThreadDist(world, dev)
        monkeypatch.setattr(shard, "dist", fake)
        return fake
    return make


@pytest.mark.parametrize("world", [2, 4])
def test_vggt_scene_split_threads(pkg, dev, shard_threads, world):
    import torch

    from candle3d_b200 import blocks, shard

    agg = blocks.VggtAggregator(depth=2, device=dev, ls_init=1.0)
    S, ph, special = 4, 9, 5
    N = special + ph * ph
    g = torch.Generator().manual_seed(11)
    tok = torch.randn(S, N, 1024, generator=g).to(dev, torch.bfloat16)
    fpos = blocks.VggtAggregator.positions(1, S, ph, ph, special, dev)
    single = agg.forward(tok.clone(), fpos, fpos.reshape(1, S * N, 2), S)
    torch.cuda.synchronize()
    fake = shard_threads(world)
    sl = S // world

    def rank_fn(r):
        split = shard.SceneSplit()
        fp = blocks.VggtAggregator.positions(1, sl, ph, ph, special, dev)
        out = agg.forward(tok[r * sl:(r + 1) * sl].clone(), fp, fp.reshape(1, sl * N, 2), sl,
                          split=split)
        return split.all_gather_rows(out.view(sl * N, 1024))

    outs = run_ranks(fake, rank_fn)
    torch.cuda.synchronize()
    for o in outs:
        assert rel_l2(o.view(S, N, 1024), single) < 2e-2


@pytest.mark.parametrize("world,groups", [(2, None), (3, None), (4, 2), (4, 1)])
def test_trellis_voxel_split_threads(pkg, dev, shard_threads, world, groups):
    """Uneven voxel slabs; (4, 2) and (4, 1): each head group shared by 2 or 4
    ranks that split its queries (the layout 8 GPUs use for 12 heads)."""
    import torch

    from candle3d_b200 import blocks, shard

    m = blocks.Trellis2Slat(blocks=2, device=dev)
    g = torch.Generator().manual_seed(12)
    occ = torch.rand(16, 16, 16, generator=g) < 0.12
    coords = torch.nonzero(occ).to(torch.int32).to(dev)
    n = coords.shape[0]
    feats = torch.randn(n, 32, generator=g).to(dev, torch.bfloat16)
    cond = torch.randn(1, 40, 1024, generator=g).to(dev, torch.bfloat16)
    t = torch.tensor([650.0], device=dev)
    single = m.forward(feats, coords, t, cond)
    torch.cuda.synchronize()
    fake = shard_threads(world)
    counts = [shard.shard_range(n, world, r)[1] - shard.shard_range(n, world, r)[0]
              for r in range(world)]

    def rank_fn(r):
        a0, a1 = shard.shard_range(n, world, r)
        out = m.forward(feats[a0:a1].contiguous(), coords[a0:a1].contiguous(), t, cond,
                        split=shard.SceneSplit(), counts=counts, head_groups=groups)
        return shard.gather_rows(out, n, world)

    outs = run_ranks(fake, rank_fn)
    torch.cuda.synchronize()
    for o in outs:
        assert o.shape == single.shape
        assert rel_l2(o, single) < 2e-2


@pytest.mark.parametrize("world", [2, 4])
def test_triposg_cfg_split_threads(pkg, dev, shard_threads, world):
    """The [uncond, cond] batch split over 2 ranks, and at 4 ranks each
    element's 1 + L tokens split over its own group of 2 (the timestep token
    on the group's first rank)."""
    import torch

    from candle3d_b200 import blocks, shard

    m = blocks.TripoSgDit(layers=5, device=dev)
    g = torch.Generator().manual_seed(13)
    L = 64
    lat = torch.randn(2, L, 64, generator=g).to(dev, torch.bfloat16)
    cond = torch.randn(2, 37, 1024, generator=g).to(dev, torch.bfloat16)
    cond[0].zero_()
    t = torch.tensor([370.0], device=dev)
    single = m.forward(lat, t, cond)
    torch.cuda.synchronize()
    fake = shard_threads(world)
    bts = shard.BatchTokenSplit(2, L, world)

    def rank_fn(r):
        groups = [fake.new_group(x) for x in bts.groups()] if bts.per > 1 else None
        b, lo, hi, prefix = bts.rows(r)
        split = shard.SceneSplit(groups[b]) if groups else None
        out = m.forward(lat[b:b + 1, lo:hi].contiguous(), t, cond[b:b + 1].contiguous(),
                        split=split, counts=bts.counts, prefix=prefix)
        return bts.gather(out[0])

    outs = run_ranks(fake, rank_fn)
    torch.cuda.synchronize()
    for o in outs:
        assert o.shape == single.shape
        assert rel_l2(o, single) < 2e-2
