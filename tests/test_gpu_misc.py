"""GPU parity: activations, timestep embeddings, small linears, patch
embedding, GGML block decoding and sparse voxel index build against the C
oracle."""
import numpy as np
import pytest

from conftest import assert_close, rng, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("kind", ["gelu_tanh", "gelu_erf", "silu"])
@pytest.mark.parametrize("shape", [(2, 4096, 4096), (1001,), (3, 5, 7)])
def test_activations(ops, orc, dev, dt, kind, shape):
    if shape == (2, 4096, 4096) and dt != "f32" and kind != "gelu_tanh":
        pytest.skip("large case covered by f32 and gelu_tanh")
    r = rng(20)
    x, xv = to_dev(3 * r.standard_normal(shape), dt, dev)
    fn = {"gelu_tanh": ops.gelu, "gelu_erf": ops.gelu_erf, "silu": ops.silu}[kind]
    y = fn(x)
    assert_close(y.float().cpu().numpy(), orc.activation(xv, kind), dt, kind)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_activation_strided_and_geglu(ops, orc, dev, dt):
    r = rng(21)
    x, xv = to_dev(r.standard_normal((4, 6, 64)), dt, dev)
    v = x[:, ::2, :]
    y = ops.gelu_erf(v)
    assert_close(y.float().cpu().numpy(), orc.gelu_erf(np.ascontiguousarray(xv[:, ::2, :])), dt, "strided")
    g, gv = to_dev(r.standard_normal((3, 9, 2 * 40)), dt, dev)
    yg = ops.geglu(g)
    assert_close(yg.float().cpu().numpy(), orc.geglu(gv), dt, "geglu")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("order,dim", [("cos_first", 256), ("sin_first", 2048), ("cos_first", 7),
                                       ("sin_first", 64)])
def test_timestep_embedding(ops, orc, dev, dt, order, dim):
    import torch

    t = np.array([0.0, 1.0, 500.0, 999.9, 1000.0 * 0.37], np.float32)
    out = ops.timestep_embedding(torch.from_numpy(t).to(dev), dim, order,
                                 dtype=getattr(torch, {"f32": "float32", "bf16": "bfloat16"}[dt]))
    code = 0 if order == "cos_first" else 1
    ref = orc.timestep_embedding(t, dim, code, 10000.0, rnd=1 if dt == "bf16" else 0)
    assert_close(out.float().cpu().numpy(), ref, dt, "timestep")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("B,K,N,ai,ao,addend", [(1, 1536, 9216, "silu", "none", True),
                                                (2, 256, 1536, "none", "silu", False),
                                                (2, 2048, 2048, "none", "gelu_erf", False),
                                                (3, 20, 7, "none", "none", True)])
def test_linear_small(ops, orc, dev, dt, B, K, N, ai, ao, addend):
    r = rng(22)
    x, xv = to_dev(r.standard_normal((B, K)), dt, dev)
    w, wv = to_dev(0.02 * r.standard_normal((N, K)), dt, dev)
    b, bv = to_dev(0.1 * r.standard_normal(N), dt, dev)
    a = av = None
    if addend:
        a, av = to_dev(0.1 * r.standard_normal(N), dt, dev)
    y = ops.linear_small(x, w, b, a, act_in=ai, act_out=ao)
    ref = orc.linear(xv, wv, bv, av, ai, ao)
    assert_close(y.float().cpu().numpy(), ref, dt, "linear_small")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("BS,HW,C,R", [(2, 28, 64, 4), (1, 518, 1024, 4), (3, 42, 96, 0)])
def test_patch_embed(ops, orc, dev, dt, BS, HW, C, R):
    r = rng(23)
    p = 14
    np_ = (HW // p) ** 2
    pix, pixv = to_dev(r.random((BS, 3, HW, HW)), dt, dev)
    w, wv = to_dev(0.02 * r.standard_normal((C, 3, p, p)), dt, dev)
    b, bv = to_dev(0.02 * r.standard_normal(C), dt, dev)
    pos, posv = to_dev(0.02 * r.standard_normal((1 + np_, C)), dt, dev)
    cls, clsv = to_dev(0.02 * r.standard_normal(C), dt, dev)
    reg = regv = None
    if R:
        reg, regv = to_dev(0.02 * r.standard_normal((R, C)), dt, dev)
    out = ops.patch_embed(pix, w, b, pos, cls, reg, p)
    ref = orc.patch_embed(pixv, wv, bv, posv, clsv, regv, p)
    assert_close(out.float().cpu().numpy(), ref, dt, "patch_embed")


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("n,k", [(256, 1024), (7, 32), (4608, 1536)])
def test_dequantize_bit_exact(ops, orc, dev, fmt, n, k):
    import torch

    w = (0.02 * rng(24).standard_normal((n, k))).astype(np.float32)
    q = orc.quantize(w, fmt)
    ref = orc.dequantize(q, fmt, n, k)
    got = ops.dequantize(torch.from_numpy(q).to(dev), fmt, n, k).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    gb = ops.dequantize(torch.from_numpy(q).to(dev), fmt, n, k, dtype=torch.bfloat16)
    assert torch.equal(gb.cpu(), torch.from_numpy(ref).to(torch.bfloat16))


def _pairs_equal(ops, orc, dev, coords):
    import torch

    d, s, c = ops.sparse_neighbor_pairs(torch.from_numpy(coords.astype(np.int32)).to(dev))
    rd, rs, rc = orc.neighbor_pairs(coords)
    c = c.cpu().numpy()
    assert np.array_equal(c, rc), "counts differ"
    d, s = d.cpu().numpy(), s.cpu().numpy()
    for k in range(27):
        assert np.array_equal(d[k, :c[k]], rd[k, :c[k]]), f"dest of offset {k}"
        assert np.array_equal(s[k, :c[k]], rs[k, :c[k]]), f"src of offset {k}"
    return d, s, c


def test_sparse_pairs_bernoulli_grid(ops, orc, dev):
    occ = np.random.default_rng(20261201).random((64, 64, 64)) < 0.12
    coords = np.argwhere(occ)  # sorted, ~31.5k voxels
    _pairs_equal(ops, orc, dev, coords)


def test_sparse_pairs_unsorted_duplicates_empty(ops, orc, dev):
    r = rng(25)
    coords = r.integers(0, 9, size=(700, 3))  # many duplicates, unsorted
    _pairs_equal(ops, orc, dev, coords)
    _pairs_equal(ops, orc, dev, np.zeros((0, 3), np.int64))
    _pairs_equal(ops, orc, dev, np.array([[0, 0, 0]]))


def test_sparse_pairs_drive_a_dense_equivalent_conv(ops, dev):
    """sparse_conv_matches_dense_reference (crates/lux3d-core/tests/trellis2_sparse.rs:98):
    4^3 grid with every 5th cell missing; conv through the device pair lists
    equals the dense per-voxel neighbour sum."""
    import torch

    res = 4
    coords = [(x, y, z) for x in range(res) for y in range(res) for z in range(res)
              if (x * 16 + y * 4 + z) % 5 != 0]
    coords = np.array(coords)
    assert len(coords) == 51
    Cin, Cout = 3, 5
    pat = lambda i: ((i % 23) - 11) * 0.1  # noqa: E731
    feats = np.array([[pat(i * 13 + c * 7) for c in range(Cin)] for i in range(len(coords))])
    W = np.array([[[pat(o * 31 + k * 5 + c * 3) * 0.5 for c in range(Cin)] for k in range(27)]
                  for o in range(Cout)])
    lookup = {tuple(c): i for i, c in enumerate(coords)}
    dense = np.zeros((len(coords), Cout))
    for i, c in enumerate(coords):
        for k in range(27):
            dlt = (k // 9 - 1, (k % 9) // 3 - 1, k % 3 - 1)
            j = lookup.get((c[0] + dlt[0], c[1] + dlt[1], c[2] + dlt[2]))
            if j is not None:
                dense[i] += W[:, k, :] @ feats[j]
    d, s, c = ops.sparse_neighbor_pairs(torch.from_numpy(coords.astype(np.int32)).to(dev))
    d, s, c = d.cpu().numpy(), s.cpu().numpy(), c.cpu().numpy()
    out = np.zeros_like(dense)
    for k in range(27):
        np.add.at(out, d[k, :c[k]], feats[s[k, :c[k]]] @ W[:, k, :].T)
    assert np.allclose(out, dense, atol=1e-12)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_index_select_rows(ops, dev, dt):
    import torch

    r = rng(26)
    feats, fv = to_dev(r.standard_normal((1000, 1536)), dt, dev)
    ids = r.integers(0, 1000, 5000)
    out = ops.index_select_rows(feats, torch.from_numpy(ids.astype(np.int32)).to(dev))
    assert np.array_equal(out.float().cpu().numpy(), fv[ids])
    out64 = ops.index_select_rows(feats, torch.from_numpy(ids).to(dev))
    assert torch.equal(out64, out)


def test_invalid_shapes_raise(ops, pkg, dev):
    import torch

    x = torch.randn(4, 64, device=dev)
    with pytest.raises(pkg._lib.L3dError) as e:
        ops.layer_norm(x, torch.ones(32, device=dev))
    assert e.value.status == 1
    with pytest.raises(pkg._lib.L3dError):
        ops.gated_residual(x, torch.randn(4, 64, device=dev, dtype=torch.bfloat16),
                           torch.ones(64, device=dev))
    q = torch.randn(1, 2, 3, 48, device=dev)  # head dim must be 64
    with pytest.raises(pkg._lib.L3dError):
        ops.rope_fused(q, torch.ones(1, 1, 3, 48, device=dev), torch.ones(1, 1, 3, 48, device=dev))


@pytest.mark.parametrize("dt", ["bf16", "f32"])
@pytest.mark.parametrize("act", ["gelu_tanh", "gelu_erf", "silu"])
def test_activation_scatter_matches_activation(ops, dev, dt, act):
    """l3d_activation_scatter (the last op fused with the final gather) stores
    exactly the bits of the plain activation to every output (here three
    buffers on this GPU; across GPUs they are peer-mapped blocks)."""
    import torch

    x = torch.randn(3000, 1024, device=dev).to(getattr(torch, {"bf16": "bfloat16", "f32": "float32"}[dt]))
    ref = {"gelu_tanh": ops.gelu, "gelu_erf": ops.gelu_erf, "silu": ops.silu}[act](x)
    bufs = [torch.zeros(4 * x.numel(), dtype=x.dtype, device=dev) for _ in range(3)]
    offs = [0, x.numel(), 3 * x.numel()]
    ops.activation_scatter(x, [(b.data_ptr(), o) for b, o in zip(bufs, offs)], act)
    torch.cuda.synchronize()
    for b, o in zip(bufs, offs):
        assert torch.equal(b[o:o + x.numel()].view_as(x), ref)
