"""Submanifold sparse conv 3x3x3 (SparseConv3d::forward,
crate/runtime/trellis2_sparse.rs:197-243).

CPU: the oracle against the reference's own two tests, restated
(crates/lux3d-core/tests/trellis2_sparse.rs:98-190 dense-grid parity with
pattern weights, max |diff| < 1e-4; :195-260 identity and +x shift kernels).
GPU: the neighbour map bit-exact against the oracle's pair lists, and the
tensor-core gather GEMM against the exact product of the same bf16 operands
(bound 2e-5 * sum |x||w|, f32 accumulation), plus the cost of the bf16
operands against the f32 oracle.
"""
import numpy as np
import pytest

from conftest import rng


def _pattern(i):
    return ((i % 23) - 11.0) * 0.1


def _offsets():
    return [(k // 9 - 1, (k % 9) // 3 - 1, k % 3 - 1) for k in range(27)]


def _dense_reference(coords, feats, w_okc, bias):
    """out[i, o] = bias[o] + sum_k sum_c w[o, k, c] * feats[nbr_k(i), c], f32
    accumulation in the reference test's loop order."""
    lookup = {tuple(c): i for i, c in enumerate(coords)}
    n, cin = feats.shape
    cout = w_okc.shape[0]
    out = np.zeros((n, cout), np.float32)
    for i, c in enumerate(coords):
        for o in range(cout):
            acc = np.float32(bias[o])
            for k, d in enumerate(_offsets()):
                j = lookup.get((c[0] + d[0], c[1] + d[1], c[2] + d[2]))
                if j is not None:
                    for ch in range(cin):
                        acc = np.float32(acc + np.float32(w_okc[o, k, ch] * feats[j, ch]))
            out[i, o] = acc
    return out


def test_sparse_conv_matches_dense_reference(orc):
    res, cin, cout = 4, 3, 5
    coords = np.array([(x, y, z) for x in range(res) for y in range(res) for z in range(res)
                       if (x * res * res + y * res + z) % 5 != 0], np.int32)
    assert len(coords) == 64 - 13
    feats = np.array([[_pattern(i * 13 + c * 7) for c in range(cin)] for i in range(len(coords))],
                     np.float32)
    w_okc = np.array([[[_pattern(o * 31 + k * 5 + c * 3) * 0.5 for c in range(cin)]
                       for k in range(27)] for o in range(cout)], np.float32)
    bias = np.array([((o * 3) % 7) * 0.02 - 0.06 for o in range(cout)], np.float32)
    got = orc.sparse_conv3d(coords, feats, w_okc.transpose(1, 0, 2), bias)
    ref = _dense_reference(coords, feats, w_okc, bias)
    assert np.abs(got - ref).max() < 1e-4


def test_sparse_conv_hand_picked_kernels(orc):
    cin = 2
    coords = np.array([[0, 0, 0], [1, 0, 0], [1, 1, 0], [3, 0, 0]], np.int32)
    feats = np.array([_pattern(i) for i in range(len(coords) * cin)], np.float32).reshape(-1, cin)
    # Identity: only the centre offset (k = 13) carries W = I.
    w = np.zeros((27, cin, cin), np.float32)
    w[13] = np.eye(cin)
    assert np.abs(orc.sparse_conv3d(coords, feats, w) - feats).max() < 1e-6
    # +x shift: k = 22 (kd = 2, kh = 1, kw = 1) carries W = I.
    w = np.zeros((27, cin, cin), np.float32)
    w[22] = np.eye(cin)
    got = orc.sparse_conv3d(coords, feats, w)
    lookup = {tuple(c): i for i, c in enumerate(coords)}
    for i, c in enumerate(coords):
        j = lookup.get((c[0] + 1, c[1], c[2]))
        expect = feats[j] if j is not None else np.zeros(cin, np.float32)
        assert np.abs(got[i] - expect).max() < 1e-6


def _coords(seed, res=24, p=0.3):
    occ = np.random.default_rng(seed).random((res, res, res)) < p
    return np.argwhere(occ).astype(np.int32)


@pytest.mark.gpu
def test_sparse_neighbor_map_matches_pairs(ops, orc, dev):
    import torch

    coords = _coords(5)
    n = len(coords)
    nbr = ops.sparse_neighbor_map(torch.from_numpy(coords).to(dev)).cpu().numpy()
    dest, src, counts = orc.neighbor_pairs(coords)
    ref = np.full((n, 27), -1, np.int32)
    for k in range(27):
        ref[dest[k, :counts[k]], k] = src[k, :counts[k]]
    assert np.array_equal(nbr, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("cin,cout,seed,ydt,method", [
    (64, 64, 11, "f32", "implicit"),    # last VAE stage width
    (128, 520, 12, "f32", "implicit"),  # several N tiles with a tail
    (40, 72, 13, "bf16", "implicit"),   # Cin padded to 64 inside the kernel; bf16 out
    (256, 256, 14, "f32", "implicit"),
    (64, 64, 11, "f32", "pairs"),
    (128, 520, 12, "bf16", "pairs"),    # N tiles with a tail, bf16 out
    (40, 70, 13, "f32", "pairs"),       # Cin padded; Cout not a multiple of 4
    (256, 256, 14, "f32", "pairs"),
])
def test_sparse_conv3d_gather_gemm(ops, orc, dev, cin, cout, seed, ydt, method):
    import torch

    coords = _coords(seed, res=20 if cin >= 256 else 24)
    n = len(coords)
    r = rng(seed)
    feats = r.standard_normal((n, cin)).astype(np.float32)
    w27 = (r.standard_normal((27, cout, cin)) / np.sqrt(27 * cin)).astype(np.float32)
    bias = (0.1 * r.standard_normal(cout)).astype(np.float32)
    fdev = torch.from_numpy(feats).to(dev).to(torch.bfloat16)
    conv = ops.SparseConv3d(torch.from_numpy(w27).to(dev), bias=torch.from_numpy(bias).to(dev))
    cd = torch.from_numpy(coords).to(dev)
    odt = torch.float32 if ydt == "f32" else torch.bfloat16
    if method == "implicit":
        y = conv(fdev, nbr=ops.sparse_neighbor_map(cd), out_dtype=odt)
    else:
        y = conv(fdev, coords=cd, out_dtype=odt)
    torch.cuda.synchronize()
    # The kernels' status word (workspace header): no bounded wait expired.
    assert conv._ws[:4].view(torch.int32).item() == 0
    got = y.float().cpu().numpy().astype(np.float64)
    # Exact product of the bf16 operands through the dense gathered form.
    nbr = ops.sparse_neighbor_map(cd).cpu().numpy()
    fb = fdev.float().cpu().numpy().astype(np.float64)
    wb = orc.round_bf16(w27).astype(np.float64)
    G = np.zeros((n, 27, cin))
    for k in range(27):
        m = nbr[:, k] >= 0
        G[m, k] = fb[nbr[m, k]]
    G = G.reshape(n, 27 * cin)
    W = wb.transpose(1, 0, 2).reshape(cout, 27 * cin)
    ref = G @ W.T + bias
    bound = 2e-5 * (np.abs(G) @ np.abs(W).T) + 1e-6
    if ydt == "bf16":
        bound = bound + np.abs(ref) * 2.0 ** -8
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    # bf16 operands against the f32 reference semantics.
    exact = orc.sparse_conv3d(coords, feats, w27, bias).astype(np.float64)
    assert np.linalg.norm(ref - exact) / np.linalg.norm(exact) < 1e-2


@pytest.mark.gpu
def test_sparse_conv3d_pairs_repeatable(ops, dev):
    """The pair-list conv accumulates offsets in a fixed order: two calls agree
    bit for bit."""
    import torch

    coords = torch.from_numpy(_coords(21)).to(dev)
    g = torch.Generator().manual_seed(4)
    feats = torch.randn(coords.shape[0], 128, generator=g).to(dev, torch.bfloat16)
    conv = ops.SparseConv3d((torch.randn(27, 96, 128, generator=g) * 0.02).to(dev))
    pairs = ops.sparse_neighbor_pairs(coords)
    a = conv(feats, pairs=pairs)
    b = conv(feats, pairs=pairs)
    assert torch.equal(a, b)
