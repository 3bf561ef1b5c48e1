"""CPU, world size 2 over gloo: row sharding of the layer-op chain.  Each rank
runs the chain (CPU oracle standing in for the device kernels) on its own
rows, the final all-gather reassembles the rows, and the result must equal the
unsharded chain bit for bit (row ops are independent per row)."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, C, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist

    import __graft_entry__ as g
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g.load_package()
        from candle3d_b200 import shard

        r = np.random.default_rng(5)
        x = r.standard_normal((n, C)).astype(np.float32)
        sh, sc = (0.1 * r.standard_normal((2, C))).astype(np.float32)
        a, b = shard.shard_range(n, world, rank)
        y = orc.gelu_tanh(orc.layer_norm_modulate(x[a:b][None], shift=sh, scale=sc, eps=1e-6)[0])
        full = shard.gather_rows(torch.from_numpy(y), n, world).numpy()
        if rank == 0:
            ref = orc.gelu_tanh(orc.layer_norm_modulate(x[None], shift=sh, scale=sc, eps=1e-6)[0])
            q.put(bool(np.array_equal(full, ref)) and full.shape == (n, C))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [1000, 7])
def test_row_shards_gather_to_the_unsharded_result(n):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, 64, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=10) is True


def test_shard_ranges_cover_rows_exactly():
    import __graft_entry__ as g

    g.load_package()
    from candle3d_b200 import shard

    for n in [0, 1, 7, 1000, 1 << 20]:
        for w in [1, 2, 3, 4, 8]:
            ranges = [shard.shard_range(n, w, r) for r in range(w)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(w - 1))
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1


def _scene_worker(rank, world, port, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    import __graft_entry__ as g

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g.load_package()
        from candle3d_b200 import shard

        # One scene of S views x N tokens, H heads of D; rank r owns views
        # [r S / world, (r + 1) S / world) (a contiguous token slab).
        S, N, H, D = 4, 37, 4, 8
        L = S * N // world
        gen = torch.Generator().manual_seed(11)
        qkv = torch.randn(S * N, 3, H, D, generator=gen)
        full = F.scaled_dot_product_attention(*(qkv[:, i].transpose(0, 1)[None] for i in range(3)))
        full = full[0].transpose(0, 1).reshape(S * N, H * D)
        split = shard.SceneSplit()
        h = H // world
        mine = qkv[rank * L:(rank + 1) * L]                       # [L, 3, H, D]
        send = mine.view(L, 3, world, h, D).permute(2, 0, 1, 3, 4).contiguous()
        qh, kh, vh = split.exchange_qkv(send)                    # [1, h, S N, D]
        ok = qh.shape == (1, h, S * N, D)
        # this rank's head group over every token, as the unsplit layer sees it
        ref_heads = qkv[:, :, rank * h:(rank + 1) * h]
        ok = ok and torch.equal(kh[0].transpose(0, 1), ref_heads[:, 1])
        a = F.scaled_dot_product_attention(qh, kh, vh)[0].transpose(0, 1).contiguous()
        o = split.return_heads(a)                                 # [L, H D]
        ok = ok and torch.allclose(o, full[rank * L:(rank + 1) * L], atol=1e-6, rtol=1e-5)
        back = split.all_gather_rows(o)
        ok = ok and torch.allclose(back, full, atol=1e-6, rtol=1e-5)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_scene_split_head_exchange_matches_unsplit_attention():
    """The global-attention exchange of a scene split across 2 ranks (gloo):
    q/k/v of each rank's token slab sent head-parallel, attention over all
    tokens per head group, outputs returned to the token owners, equals the
    unsplit attention (crate/runtime/vggt.rs:299-311 global blocks)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_scene_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


def test_interleaved_blocks_tile_the_rows():
    import __graft_entry__ as g

    g.load_package()
    from candle3d_b200 import shard

    for world in [1, 2, 8]:
        rc, chunks = 5, 3
        seen = sorted(r for c in range(chunks) for k in range(world)
                      for r in range(*shard.interleaved_block(c, world, k, rc)))
        assert seen == list(range(chunks * world * rc))


def test_peer_rows_layout():
    """PeerRows.dest: rank r's block starts at row r * rows of every buffer."""
    import __graft_entry__ as g

    g.load_package()
    from candle3d_b200 import shard

    pr = shard.PeerRows.__new__(shard.PeerRows)
    pr.rank, pr.rows, pr.C, pr.ptrs = 2, 10, 4, [100, 200, 300]
    assert pr.dest(0) == (100, 80) and pr.dest(2) == (300, 80)


def _uneven_worker(rank, world, port, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    import __graft_entry__ as g

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g.load_package()
        from candle3d_b200 import shard

        # 61 voxel rows split 31 / 30 (shard_range), 6 heads of 8.
        Ntot, H, D = 61, 6, 8
        counts = [shard.shard_range(Ntot, world, r)[1] - shard.shard_range(Ntot, world, r)[0]
                  for r in range(world)]
        a0, a1 = shard.shard_range(Ntot, world, rank)
        gen = torch.Generator().manual_seed(12)
        qkv = torch.randn(Ntot, 3, H, D, generator=gen)
        full = F.scaled_dot_product_attention(*(qkv[:, i].transpose(0, 1)[None] for i in range(3)))
        full = full[0].transpose(0, 1).reshape(Ntot, H * D)
        split = shard.SceneSplit()
        h = H // world
        L = a1 - a0
        send = qkv[a0:a1].view(L, 3, world, h, D).permute(2, 0, 1, 3, 4).contiguous()
        qh, kh, vh = split.exchange_qkv_uneven(send, counts)
        ok = qh.shape == (1, h, Ntot, D)
        a = F.scaled_dot_product_attention(qh, kh, vh)[0].transpose(0, 1).contiguous()
        o = split.return_heads_uneven(a, counts)
        ok = ok and torch.allclose(o, full[a0:a1], atol=1e-6, rtol=1e-5)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_scene_split_uneven_slabs_match_unsplit_attention():
    """The head-parallel exchange with slabs of unequal length (61 voxel rows
    over 2 ranks, the TRELLIS.2 voxel-row split), gloo world size 2."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_uneven_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


def test_batch_token_split_layout():
    """The CFG batch x token slabs of BatchTokenSplit tile each element's L
    kept rows exactly once, only a group's first rank holds the prefix token,
    and the counts (prefix included) sum to 1 + L."""
    import __graft_entry__ as g

    g.load_package()
    from candle3d_b200 import shard

    for world in (1, 2, 4, 8):
        for L in (2048, 7):
            bts = shard.BatchTokenSplit(2, L, world) if world > 1 else None
            if bts is None:
                with pytest.raises(ValueError):
                    shard.BatchTokenSplit(2, L, world)
                continue
            assert sum(bts.counts) == 1 + L
            seen = {0: [], 1: []}
            for r in range(world):
                b, lo, hi, prefix = bts.rows(r)
                assert prefix == (r % bts.per == 0)
                assert hi - lo + int(prefix) == bts.counts[r % bts.per]
                seen[b].extend(range(lo, hi))
            assert seen[0] == list(range(L)) and seen[1] == list(range(L))


def _batch_token_worker(rank, world, port, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist

    import __graft_entry__ as g

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g.load_package()
        from candle3d_b200 import shard

        L, F = 37, 5
        full = torch.arange(2 * L * F, dtype=torch.float32).view(2, L, F)
        bts = shard.BatchTokenSplit(2, L, world)
        b, lo, hi, _ = bts.rows(rank)
        got = bts.gather(full[b, lo:hi].contiguous())
        q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_batch_token_split_gathers_every_row(world):
    """gloo world sizes 2, 4 and 8: each rank's slab of one batch element,
    gathered, rebuilds the [2, L, F] output exactly."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_token_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert res == {r: True for r in range(world)}


def _shared_groups_worker(rank, world, port, q, H, groups):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    import __graft_entry__ as g

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g.load_package()
        from candle3d_b200 import shard

        Ntot, D = 83, 8
        counts = [shard.shard_range(Ntot, world, r)[1] - shard.shard_range(Ntot, world, r)[0]
                  for r in range(world)]
        a0, a1 = shard.shard_range(Ntot, world, rank)
        gen = torch.Generator().manual_seed(13)
        qkv = torch.randn(Ntot, 3, H, D, generator=gen)
        full = F.scaled_dot_product_attention(*(qkv[:, i].transpose(0, 1)[None] for i in range(3)))
        full = full[0].transpose(0, 1).reshape(Ntot, H * D)
        split = shard.SceneSplit()
        h = H // groups
        L = a1 - a0
        send = qkv[a0:a1].view(L, 3, groups, h, D).permute(2, 0, 1, 3, 4).contiguous()
        qh, kh, vh = split.exchange_qkv_uneven(send, counts, groups)
        b0, b1 = split.query_block(counts, groups)
        ok = qh.shape == (1, h, b1 - b0, D) and kh.shape == (1, h, Ntot, D)
        a = F.scaled_dot_product_attention(qh, kh, vh)[0].transpose(0, 1).contiguous()
        o = split.return_heads_uneven(a, counts, groups)
        ok = ok and torch.allclose(o, full[a0:a1], atol=1e-6, rtol=1e-5)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,H,groups", [(4, 6, 2), (4, 12, 4), (4, 6, 1), (2, 3, 1),
                                            (8, 12, 4)])
def test_scene_split_shared_head_groups_match_unsplit_attention(world, H, groups):
    """Fewer head groups than ranks (the TRELLIS.2 split at 8 ranks: 12 heads
    in 4 groups, each shared by 2 ranks that split its queries): gloo world
    sizes 2, 4 and 8, 83 rows in uneven slabs, against the unsplit attention."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shared_groups_worker, args=(r, world, port, q, H, groups))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert res == {r: True for r in range(world)}
