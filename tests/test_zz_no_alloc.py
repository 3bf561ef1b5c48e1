"""GPU: the allocation-free neighbour-pair entry point.

Who needs it: callers that cannot give the library a workspace, such as a
Candle CustomOp whose cuda_fwd only allocates its output, a CUDA graph
replayed with buffers fixed at capture time, or a serving runtime that forbids
device allocation on its request path.  l3d_sparse_neighbor_pairs_noalloc
uses a fixed scratch array inside the library instead (at most 65536
coordinates).

The test calls it through the C ABI and checks that it returns exactly what
the workspace entry point returns (integer pair lists: bit-exact, the same
tolerance the sparse tests use), on two calls in a row with different
coordinate sets so a stale scratch table would show.  It also checks that
inputs beyond the limit are rejected on the host.  This file sorts last so a
stop-at-first-failure run has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _coords(seed, res, p):
    occ = np.random.default_rng(seed).random((res, res, res)) < p
    return np.argwhere(occ).astype(np.int32)


def _noalloc_pairs(pkg, coords):
    import torch

    from candle3d_b200._lib import call, desc, ref, stream_handle

    n = coords.shape[0]
    dest = torch.full((27, n), -1, dtype=torch.int32, device=coords.device)
    src = torch.full((27, n), -1, dtype=torch.int32, device=coords.device)
    counts = torch.zeros(27, dtype=torch.int32, device=coords.device)
    call("l3d_sparse_neighbor_pairs_noalloc", ref(desc(coords)), ref(desc(dest)), ref(desc(src)),
         ref(desc(counts)), stream_handle(coords.device))
    return dest, src, counts


def test_noalloc_matches_workspace_entry_twice(pkg, ops, dev):
    import torch

    # First call: the TRELLIS-sized grid (~31.5k voxels); second call: a
    # smaller, unsorted set with duplicates, after the first has filled the
    # scratch table; third: exactly the 65536-coordinate limit (the dense
    # 16 x 64 x 64 block, every table slot pair in use).
    first = _coords(20261201, 64, 0.12)
    second = np.random.default_rng(7).integers(0, 12, size=(900, 3)).astype(np.int32)
    third = np.argwhere(np.ones((16, 64, 64), bool)).astype(np.int32)
    assert third.shape[0] == 65536
    for c in (first, second, third):
        ct = torch.from_numpy(c).to(dev)
        d0, s0, n0 = ops.sparse_neighbor_pairs(ct)
        d1, s1, n1 = _noalloc_pairs(pkg, ct)
        torch.cuda.synchronize()
        assert torch.equal(n0, n1)
        for k in range(27):
            m = int(n0[k])
            assert torch.equal(d0[k, :m], d1[k, :m]), f"dest offset {k}"
            assert torch.equal(s0[k, :m], s1[k, :m]), f"src offset {k}"


def test_noalloc_rejects_inputs_beyond_its_limit(pkg, dev):
    import torch

    big = torch.zeros((65537, 3), dtype=torch.int32, device=dev)
    with pytest.raises(pkg._lib.L3dError) as e:
        _noalloc_pairs(pkg, big)
    assert e.value.status == 4  # L3D_E_UNSUPPORTED
    assert "65536" in str(e.value)
