"""CPU: pin the oracle.  (1) The reference's own known-answer tests
(tests/golden/reference_kats.json, made by tests/golden/make_golden.py);
(2) an independent numpy restatement of each op at small sizes; (3) the GGML
block formats (round trip and the quant_probe methodology,
crates/lux3d-core/examples/quant_probe.rs:47-124)."""
import json
from math import erf
from pathlib import Path

import numpy as np
import pytest

from conftest import rng

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def test_kat_rope_tables(orc):
    k = KATS["rope_tables"]
    c, s = orc.rope3d_tables(np.array(k["coords"]), k["head_dim"], 10000.0)
    assert np.max(np.abs(c - np.array(k["cos"]))) < k["tol"]
    assert np.max(np.abs(s - np.array(k["sin"]))) < k["tol"]


def test_kat_rope_apply(orc):
    k = KATS["rope_apply"]
    c, s = orc.rope3d_tables(np.array(k["coords"]), k["head_dim"], 10000.0)
    x = np.array(k["x"], np.float32).reshape(1, 1, 1, 12)
    y = orc.rope3d_apply(x, c, s).reshape(-1)
    assert np.max(np.abs(y - np.array(k["expected"]))) < k["tol"]
    e_in = float(np.sum(x.astype(np.float64) ** 2))
    e_out = float(np.sum(y.astype(np.float64) ** 2))
    assert abs(e_in - e_out) < k["norm_tol"]
    # The fused norm+rope entry with gamma=None is the same rotation.
    y2 = orc.qk_l2norm_rope3d(x, None, np.array(k["coords"]), 10000.0).reshape(-1)
    assert np.array_equal(y, y2)


def test_kat_cubic_coords(pkg):
    import torch

    k = KATS["cubic_coords"]
    c = pkg.ops.cubic_token_coords(k["resolution"], device="cpu").numpy()
    assert c.size == k["len"]
    assert c[k["index_x1_y2_z0"]].tolist() == k["coord_at_index"]
    assert c[-1].tolist() == k["last"]
    del torch


def test_kat_qk_rms_norm(orc):
    k = KATS["qk_rms_norm"]
    x = np.array(k["x"], np.float32).reshape(1, 1, 1, 4)
    for case in k["cases"]:
        gamma = np.full((1, 4), case["gamma"], np.float32)
        y = orc.qk_l2norm_rope3d(x, gamma, None).reshape(-1)
        assert np.max(np.abs(y - np.array(case["expected"]))) < k["tol"]


def test_kat_timestep(orc):
    k = KATS["timestep"]
    y = orc.timestep_embedding([k["t"]], k["dim"], 0).reshape(-1)
    assert np.max(np.abs(y - np.array(k["expected"]))) < k["tol"]


def test_kat_ada_chunks(pkg):
    import torch

    k = KATS["ada_chunks"]
    mod = torch.tensor([k["mod_vec"]])
    chunks = pkg.ops.chunk_modulation(mod)
    assert [c.shape for c in chunks] == [(1, 1, 2)] * 6
    assert [c.reshape(-1).tolist() for c in chunks] == k["expected"]


def test_kat_coord_map_and_offsets(orc):
    """CoordMap lookups through the pair lists: a probe voxel placed at
    coord - delta_14 (delta_14 = (0, 0, 1)) finds map[coord] at offset 14."""
    k = KATS["coord_map"]
    coords = np.array(k["coords"])
    for coord, want in k["lookups"]:
        probe = np.array(coord) - np.array([0, 0, 1])
        d, s, c = orc.neighbor_pairs(np.concatenate([coords, [probe]]))
        hits = dict(zip(d[14, :c[14]].tolist(), s[14, :c[14]].tolist()))
        assert hits.get(3) == want
    for kk, delta in KATS["offsets"]["cases"]:
        assert list(orc.kernel_offset_delta(kk)) == delta
    assert len({orc.kernel_offset_delta(i) for i in range(27)}) == 27


# ---------------------------------------------------- numpy cross-restatement
def np_layer_norm(x, w, b, eps):
    m = x.mean(-1, keepdims=True, dtype=np.float64)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    y = (x - m) / np.sqrt(v + eps)
    return y * w + b if w is not None else y


def test_cross_layer_norm_modulate(orc):
    r = rng(30)
    x = r.standard_normal((2, 33, 96)).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal(96)).astype(np.float32)
    b = (0.02 * r.standard_normal(96)).astype(np.float32)
    sh, sc, g = (0.1 * r.standard_normal((3, 2, 96))).astype(np.float32)
    got = orc.layer_norm_modulate(x, w, b, sh, sc, g, add_input=True, eps=1e-6)
    ref = g[:, None] * (np_layer_norm(x, w, b, 1e-6) * (1 + sc[:, None]) + sh[:, None]) + x
    assert np.max(np.abs(got - ref)) < 2e-5


def np_rope2d(x, pos, theta):
    D = x.shape[-1]
    half, q = D // 2, D // 4
    inv = 1.0 / theta ** (np.arange(q) * 2.0 / half)
    out = np.empty_like(x, dtype=np.float64)
    for hf in range(2):
        ang = pos[:, None, :, hf, None] * inv  # [B,1,N,q]
        c, s = np.cos(ang), np.sin(ang)
        a = x[..., hf * half:hf * half + q]
        bb = x[..., hf * half + q:(hf + 1) * half]
        out[..., hf * half:hf * half + q] = a * c - bb * s
        out[..., hf * half + q:(hf + 1) * half] = bb * c + a * s
    return out


def test_cross_layernorm_rope2d(orc):
    r = rng(31)
    B, H, N, D = 2, 3, 20, 64
    x = r.standard_normal((B, H, N, D)).astype(np.float32)
    pos = r.integers(0, 40, (B, N, 2))
    cs, sn = orc.rope2d_tables(pos, 100.0, D)
    got = orc.layernorm_rope2d(x, None, None, 1e-5, cs, sn)
    assert np.max(np.abs(got - np_rope2d(x.astype(np.float64), pos, 100.0))) < 2e-5
    w = np.ones(D, np.float32)
    got2 = orc.layernorm_rope2d(x, w, 0 * w, 1e-5, cs, sn)
    ref2 = np_rope2d(np_layer_norm(x.astype(np.float64), None, None, 1e-5), pos, 100.0)
    assert np.max(np.abs(got2 - ref2)) < 2e-5


def test_cross_l2norm_rope3d(orc):
    r = rng(32)
    L, H, D = 30, 4, 128
    x = r.standard_normal((1, L, H, D)).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal((H, D))).astype(np.float32)
    coords = r.integers(0, 64, (L, 3))
    got = orc.qk_l2norm_rope3d(x, gamma, coords)
    xn = x / np.linalg.norm(x.astype(np.float64), axis=-1, keepdims=True) * gamma * np.sqrt(D)
    fd = D // 2 // 3
    freqs = 1.0 / 10000.0 ** (np.arange(fd) / fd)
    ang = np.zeros((L, D // 2))
    for a in range(3):
        ang[:, a * fd:(a + 1) * fd] = coords[:, a, None] * freqs
    z = (xn[..., 0::2] + 1j * xn[..., 1::2]) * np.exp(1j * ang)[None, :, None, :]
    ref = np.stack([z.real, z.imag], -1).reshape(x.shape)
    assert np.max(np.abs(got - ref)) < 5e-5


def test_cross_activations(orc):
    x = np.linspace(-8, 8, 4001).astype(np.float32)
    xd = x.astype(np.float64)
    assert np.max(np.abs(orc.silu(x) - xd / (1 + np.exp(-xd)))) < 1e-5
    ge = np.array([0.5 * v * (1 + erf(v / np.sqrt(2))) for v in xd])
    assert np.max(np.abs(orc.gelu_erf(x) - ge)) < 1e-5
    gt = 0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))
    assert np.max(np.abs(orc.gelu_tanh(x) - gt)) < 1e-5


def test_cross_timestep_orders(orc):
    t = np.array([0.0, 37.5, 999.0], np.float32)
    for order, dim in [(0, 256), (1, 64)]:
        half = dim // 2
        f = np.exp(-np.log(10000.0) * np.arange(half) / half)
        a = t[:, None].astype(np.float64) * f
        ref = np.concatenate([np.cos(a), np.sin(a)] if order == 0 else [np.sin(a), np.cos(a)], -1)
        got = orc.timestep_embedding(t, dim, order)
        assert np.max(np.abs(got - ref)) < 2e-4  # f32 argument rounding at t ~ 1e3


def test_cross_patch_embed(orc):
    r = rng(33)
    pix = r.random((2, 3, 28, 28)).astype(np.float32)
    w = (0.1 * r.standard_normal((8, 3, 14, 14))).astype(np.float32)
    b, cls = (0.1 * r.standard_normal((2, 8))).astype(np.float32)
    pos = (0.1 * r.standard_normal((5, 8))).astype(np.float32)
    reg = (0.1 * r.standard_normal((4, 8))).astype(np.float32)
    got = orc.patch_embed(pix, w, b, pos, cls, reg, 14)
    patches = pix.reshape(2, 3, 2, 14, 2, 14).transpose(0, 2, 4, 1, 3, 5).reshape(2, 4, -1)
    conv = patches @ w.reshape(8, -1).T + b
    tok = np.concatenate([np.broadcast_to(cls, (2, 1, 8)), conv], 1) + pos
    ref = np.concatenate([tok[:, :1], np.broadcast_to(reg, (2, 4, 8)), tok[:, 1:]], 1)
    assert np.max(np.abs(got - ref)) < 1e-5


@pytest.mark.parametrize("fmt,max_rel", [("q8_0", 0.01), ("q4_0", 0.12)])
def test_ggml_blocks_quant_probe(orc, fmt, max_rel):
    """quant_probe methodology: deterministic LCG [256, 1024] weight, decode
    error and matmul error vs the dequantized f32 weights."""
    n, k = 256, 1024
    state = 0x123456789ABCDEF0
    vals = np.empty(n * k, np.float32)
    for i in range(n * k):
        state = (state * 6364136223846793005 + 1) & (2 ** 64 - 1)
        vals[i] = ((state >> 33) / float(1 << 31) * 2.0 - 1.0) * 0.05
    w = vals.reshape(n, k)
    q = orc.quantize(w, fmt)
    assert q.size == n * (k // 32) * (34 if fmt == "q8_0" else 18)
    d = orc.dequantize(q, fmt, n, k)
    rel = np.linalg.norm(d - w) / np.linalg.norm(w)
    assert rel < max_rel
    act = np.sin(np.arange(4 * k, dtype=np.float32) * 0.001).reshape(4, k)
    y = orc.linear(act, d)
    assert np.linalg.norm(y - act.astype(np.float64) @ d.T.astype(np.float64)) / np.linalg.norm(y) < 1e-6
    # Re-quantising the decoded weights is a fixed point of the format.
    assert np.array_equal(orc.dequantize(orc.quantize(d, fmt), fmt, n, k), d)


def test_neighbor_pairs_ascending_and_symmetric(orc):
    occ = np.random.default_rng(20261201).random((16, 16, 16)) < 0.3
    coords = np.argwhere(occ)
    d, s, c = orc.neighbor_pairs(coords)
    assert c[13] == len(coords)  # the centre offset pairs every voxel with itself
    for k in range(27):
        assert np.all(np.diff(d[k, :c[k]]) > 0)
        assert c[k] == c[26 - k]  # delta and -delta pair the same voxel pairs


# --------------------------------------------------------------- torch CPU
# An implementation that is neither this build's nor the reference's: torch's
# CPU kernels compute the same textbook formulas Candle's ops are defined by
# (LayerNorm with biased variance, GELU tanh / erf, SiLU, RMSNorm).  These
# cases check the oracle against them in f32; they do not pin Candle's own
# rounding, which no reference test exposes.
def test_oracle_matches_torch_cpu_layer_ops(orc):
    import torch
    import torch.nn.functional as F

    r = np.random.default_rng(77)
    x = r.standard_normal((4, 96, 1024)).astype(np.float32) * 3 + 0.5
    w = (1 + 0.02 * r.standard_normal(1024)).astype(np.float32)
    b = (0.02 * r.standard_normal(1024)).astype(np.float32)
    tx = torch.from_numpy(x)
    ref = F.layer_norm(tx, (1024,), torch.from_numpy(w), torch.from_numpy(b), 1e-6).numpy()
    got = orc.layer_norm(x, w, b, 1e-6)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < 1e-5
    sc = (0.1 * r.standard_normal((4, 1024))).astype(np.float32)
    sh = (0.1 * r.standard_normal((4, 1024))).astype(np.float32)
    ln = F.layer_norm(tx, (1024,), eps=1e-6)
    ref = (ln * (1 + torch.from_numpy(sc)[:, None]) + torch.from_numpy(sh)[:, None]).numpy()
    got = orc.layer_norm_modulate(x, shift=sh, scale=sc, eps=1e-6)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < 1e-5
    for name, fn in (("gelu_tanh", lambda t: F.gelu(t, approximate="tanh")),
                     ("gelu_erf", F.gelu), ("silu", F.silu)):
        ref = fn(tx).numpy()
        got = getattr(orc, name)(x)
        assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < 1e-5, name
    q = r.standard_normal((2, 16, 50, 128)).astype(np.float32)
    wq = (1 + 0.05 * r.standard_normal(128)).astype(np.float32)
    tq = torch.from_numpy(q)
    ref = (tq * torch.rsqrt(tq.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(wq)).numpy()
    got = orc.rms_norm_heads(q, wq, 1e-6)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < 1e-5
