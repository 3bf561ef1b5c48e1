"""GPU parity: QK-norm + RoPE entries (2D axial for VGGT/Pi3, 3D voxel for
TRELLIS.2) against the C oracle (crate/runtime/attention_math.rs:14-165,
crate/runtime/trellis2_blocks.rs:57-160,306-319).  Angles/indices are formed
bit-exactly; tables are compared to the oracle's f32 cos/sin."""
import numpy as np
import pytest

from conftest import assert_close, rng, to_dev

pytestmark = pytest.mark.gpu


def vggt_positions(B, ph, pw, special=5):
    """Positions of crate/runtime/vggt.rs:288-291: 0 for special tokens, (y+1, x+1)."""
    ys, xs = np.meshgrid(np.arange(1, ph + 1), np.arange(1, pw + 1), indexing="ij")
    grid = np.stack([ys, xs], -1).reshape(1, ph * pw, 2)
    pos = np.concatenate([np.zeros((1, special, 2), np.int64), grid], 1)
    return np.repeat(pos, B, 0).astype(np.int64)


def test_rope2d_tables(ops, orc, dev):
    import torch

    pos = vggt_positions(2, 37, 37)
    emb = ops.Rope2d(100.0).embeddings(torch.from_numpy(pos).to(dev), 64)
    c, s = emb.cos_full, emb.sin_alt_full
    cr, sr = orc.rope2d_tables(pos, 100.0, 64)
    assert np.max(np.abs(c.cpu().numpy()[:, 0] - cr)) <= 2e-7
    assert np.max(np.abs(s.cpu().numpy()[:, 0] - sr)) <= 2e-7


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("cfg", [(2, 16, 64, 64), (8, 16, 37, 37), (1, 3, 5, 7)])
@pytest.mark.parametrize("norm", [True, False])
def test_layernorm_rope2d_tables(ops, orc, dev, dt, cfg, norm):
    """layernorm_rope_fused / rope_fused on the strided q view of
    qkv.reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4)[0] (crate/runtime/vggt.rs:163-166)."""
    import torch

    B, H, ph, pw = cfg
    D = 64
    pos = vggt_positions(B, ph, pw)
    N = pos.shape[1]
    r = rng(10)
    qkv, qkvv = to_dev(r.standard_normal((B, N, 3, H, D)), dt, dev)
    q = qkv.permute(2, 0, 3, 1, 4)[0]
    w = b = wv = bv = None
    if norm:
        w, wv = to_dev(1 + 0.1 * r.standard_normal(D), dt, dev)
        b, bv = to_dev(0.1 * r.standard_normal(D), dt, dev)
    emb = ops.Rope2d(100.0).embeddings(torch.from_numpy(pos).to(dev), D)
    y = ops.layernorm_rope_fused(q, w, b, 1e-5, emb.cos_full, emb.sin_alt_full) if norm else \
        ops.rope_fused(q, emb.cos_full, emb.sin_alt_full)
    cs, sn = orc.rope2d_tables(pos, 100.0, D)
    qv = np.ascontiguousarray(qkvv.transpose(2, 0, 3, 1, 4)[0])
    ref = orc.layernorm_rope2d(qv, wv, bv, 1e-5, cs, sn)
    assert_close(y.float().cpu().numpy(), ref, dt, "ln+rope2d")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("cfg", [(2, 16, 64, 64), (1, 16, 37, 37 * 8), (3, 5, 4, 6)])
@pytest.mark.parametrize("out_layout", ["bhnd", "bnhd"])
def test_qk_layernorm_rope2d_positions(ops, orc, dev, dt, cfg, out_layout):
    """q and k in one launch, angles from integer positions (no tables);
    outputs contiguous [B, H, N, D] or token-major [B, N, H, D] memory."""
    import torch

    B, H, ph, pw = cfg
    D = 64
    pos = vggt_positions(B, ph, pw)
    N = pos.shape[1]
    r = rng(11)
    qkv, qkvv = to_dev(r.standard_normal((B, N, 3, H, D)), dt, dev)
    v = qkv.permute(2, 0, 3, 1, 4)
    wq, wqv = to_dev(1 + 0.1 * r.standard_normal(D), dt, dev)
    bq, bqv = to_dev(0.1 * r.standard_normal(D), dt, dev)
    wk, wkv = to_dev(1 + 0.1 * r.standard_normal(D), dt, dev)
    bk, bkv = to_dev(0.1 * r.standard_normal(D), dt, dev)
    outs = {}
    if out_layout == "bnhd":
        qk = torch.empty(2, B, N, H, D, dtype=qkv.dtype, device=dev).permute(0, 1, 3, 2, 4)
        outs = {"q_out": qk[0], "k_out": qk[1]}
    qo, ko = ops.qk_layernorm_rope2d(v[0], v[1], wq, bq, wk, bk, 1e-5,
                                     torch.from_numpy(pos).to(dev), 100.0, **outs)
    cs, sn = orc.rope2d_tables(pos, 100.0, D)
    vv = qkvv.transpose(2, 0, 3, 1, 4)
    assert_close(qo.float().cpu().numpy(),
                 orc.layernorm_rope2d(np.ascontiguousarray(vv[0]), wqv, bqv, 1e-5, cs, sn), dt, "q")
    assert_close(ko.float().cpu().numpy(),
                 orc.layernorm_rope2d(np.ascontiguousarray(vv[1]), wkv, bkv, 1e-5, cs, sn), dt, "k")


def bernoulli_coords(res, p, seed):
    occ = np.random.default_rng(seed).random((res, res, res)) < p
    return np.argwhere(occ).astype(np.int64)  # lexicographically sorted (x, y, z)


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("H,D", [(12, 128), (4, 64), (2, 12), (3, 6)])
@pytest.mark.parametrize("mode", ["norm+rope", "rope", "norm"])
def test_qk_l2norm_rope3d(ops, orc, dev, dt, H, D, mode):
    """q view of to_qkv(x).reshape(B, L, 3, H, D) (crate/runtime/trellis2_blocks.rs:397-409)."""
    import torch

    coords = bernoulli_coords(24, 0.12, 7)
    L = coords.shape[0]
    r = rng(12)
    qkv, qkvv = to_dev(r.standard_normal((1, L, 3, H, D)), dt, dev)
    q = qkv[:, :, 0]
    gamma = (1 + 0.1 * r.standard_normal((H, D))).astype(np.float32)
    g = torch.from_numpy(gamma).to(dev) if mode != "rope" else None
    cd = torch.from_numpy(coords).to(dev) if mode != "norm" else None
    y = ops.qk_l2norm_rope3d(q, g, cd, 10000.0)
    ref = orc.qk_l2norm_rope3d(np.ascontiguousarray(qkvv[:, :, 0]), gamma if mode != "rope" else None,
                               coords if mode != "norm" else None, 10000.0)
    assert_close(y.float().cpu().numpy(), ref, dt, f"l2norm+rope3d {mode}")


def test_rope3d_tables_and_apply(ops, orc, dev):
    import torch

    coords = bernoulli_coords(64, 0.05, 3)
    rope = ops.Trellis2Rope3d(128)
    c, s = rope.cos_sin(torch.from_numpy(coords).to(dev))
    cr, sr = orc.rope3d_tables(coords, 128, 10000.0)
    assert np.max(np.abs(c.cpu().numpy() - cr)) <= 2e-7
    assert np.max(np.abs(s.cpu().numpy() - sr)) <= 2e-7
    r = rng(13)
    x, xv = to_dev(r.standard_normal((2, coords.shape[0], 12, 128)), "f32", dev)
    y = rope.apply(x, c, s)
    assert_close(y.cpu().numpy(), orc.rope3d_apply(xv, cr, sr), "f32", "rope3d apply")


def test_rope3d_table_and_coord_paths_agree(ops, dev):
    """Rotation from coordinates in-kernel == rotation by the device tables."""
    import torch

    coords = torch.from_numpy(bernoulli_coords(32, 0.1, 5)).to(dev)
    x = torch.randn(1, coords.shape[0], 12, 128, device=dev)
    rope = ops.Trellis2Rope3d(128)
    c, s = rope.cos_sin(coords)
    a = rope.apply(x, c, s)
    b = ops.qk_l2norm_rope3d(x, None, coords)
    assert torch.allclose(a, b, rtol=1e-6, atol=1e-6)
