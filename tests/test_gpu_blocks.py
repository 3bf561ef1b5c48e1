"""GPU parity of the block stacks (fused ops + cuBLAS GEMMs + attention, both
torch SDPA and l3d_attention) against plain torch f32 restatements of the
reference blocks at reduced depth/size.

Stacks compound bf16 rounding across blocks, so the comparison is normwise:
relative L2 error of the stack output (and of the residual-stream update)
within 2e-2, the bf16 tolerance of the parity contract applied to the whole
block rather than to one op.
"""
import pytest

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


@pytest.fixture(params=["sdpa", "l3d"])
def attn(request, pkg):
    """The stacks' bf16 attention core: torch SDPA, or l3d_attention."""
    from candle3d_b200 import blocks

    blocks.set_attention(request.param)
    yield request.param
    blocks.set_attention("sdpa")


@pytest.mark.parametrize("fused_mlp", [False, True])
def test_vggt_stack_matches_reference(pkg, dev, attn, fused_mlp, monkeypatch):
    import torch

    from candle3d_b200 import blocks

    # fused_mlp: fc1 + GELU-erf as one tcgen05 GEMM at any size (normally from
    # 8192 rows).
    monkeypatch.setattr(blocks, "FUSED_MLP_MIN_ROWS", 0 if fused_mlp else 1 << 62)

    # LayerScale 1.0 instead of the 0.01 init: with 0.01 the per-block update
    # is far below one bf16 ulp of the residual stream and rounds away (in
    # Candle's bf16 path as well), leaving nothing to compare.
    agg = blocks.VggtAggregator(depth=2, device=dev, ls_init=1.0)
    B, S, ph, pw, special = 1, 2, 9, 9, 5
    N = special + ph * pw
    fpos = blocks.VggtAggregator.positions(B, S, ph, pw, special, dev)
    gpos = fpos.reshape(B, S * N, 2)
    g = torch.Generator().manual_seed(1)
    tok = torch.randn(B * S, N, 1024, generator=g).to(dev, torch.bfloat16)
    ref = blocks.vggt_reference(agg, tok, fpos, gpos, S)
    out = agg.forward(tok.clone(), fpos, gpos, S)
    assert rel_l2(out - tok, ref - tok.float()) < 2e-2
    assert rel_l2(out, ref) < 2e-2


def test_triposg_stack_matches_reference(pkg, dev, attn):
    import torch

    from candle3d_b200 import blocks

    m = blocks.TripoSgDit(layers=5, device=dev)
    g = torch.Generator().manual_seed(2)
    lat = torch.randn(2, 64, 64, generator=g).to(dev, torch.bfloat16)
    cond = torch.randn(2, 37, 1024, generator=g).to(dev, torch.bfloat16)
    cond[0].zero_()  # CFG batch [uncond (zeros), cond]
    t = torch.tensor([370.0], device=dev)
    out = m.forward(lat, t, cond)
    ref = blocks.triposg_reference(m, lat, t, cond)
    assert out.shape == (2, 64, 64)
    assert rel_l2(out, ref) < 2e-2


def test_trellis_slat_stack_matches_reference(pkg, ops, dev, attn):
    import torch
    import torch.nn.functional as F

    from candle3d_b200 import blocks

    m = blocks.Trellis2Slat(blocks=2, device=dev)
    g = torch.Generator().manual_seed(3)
    occ = torch.rand(16, 16, 16, generator=g) < 0.12
    coords = torch.nonzero(occ).to(torch.int32).to(dev)
    N = coords.shape[0]
    feats = torch.randn(N, 32, generator=g).to(dev, torch.bfloat16)
    cond = torch.randn(1, 40, 1024, generator=g).to(dev, torch.bfloat16)
    t = torch.tensor([650.0], device=dev)
    out = m.forward(feats, coords, t, cond)

    # torch f32 restatement of Trellis2SparseBlock / SLAT forward with the
    # dequantised weights (crate/runtime/trellis2_blocks.rs:609-646).
    f = lambda a: a.float()  # noqa: E731

    def lin(q, x):
        w = ops.dequantize(q.blocks, "q8_0", q.n, q.k)
        return F.linear(x, w, q.bias)

    C, H, D = m.C, m.H, m.D
    half = 128
    freqs = torch.exp(-torch.log(torch.tensor(10000.0)) * torch.arange(half) / half).to(dev)
    arg = t.float() * freqs
    tab = torch.cat([torch.cos(arg), torch.sin(arg)]).view(1, 256)
    th = F.linear(F.silu(F.linear(tab, f(m.t_fc1[0]), f(m.t_fc1[1]))), f(m.t_fc2[0]), f(m.t_fc2[1]))
    temb = F.linear(F.silu(th), f(m.ada[0]), f(m.ada[1]))
    cs, sn = ops.Trellis2Rope3d(D).cos_sin(coords)

    def qknorm(x, gamma):
        return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12) * gamma * D ** 0.5

    def rope(x):
        z = torch.view_as_complex(x.reshape(*x.shape[:-1], D // 2, 2).contiguous())
        rot = torch.polar(torch.ones_like(cs), torch.atan2(sn, cs))
        return torch.view_as_real(z * rot[None, :, None, :]).reshape(x.shape)

    x = F.linear(f(feats), f(m.input_layer[0]), f(m.input_layer[1])).view(1, N, C)
    for p in m.blocks:
        mv = f(p["modulation"]).unsqueeze(0) + temb
        sh1, sc1, g1, sh2, sc2, g2 = [c.unsqueeze(1) for c in mv.chunk(6, -1)]
        h = F.layer_norm(x, (C,), eps=1e-6) * (1 + sc1) + sh1
        qkv = lin(p["to_qkv"], h).view(1, N, 3, H, D)
        q = rope(qknorm(qkv[:, :, 0], p["qg"]))
        k = rope(qknorm(qkv[:, :, 1], p["kg"]))
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), qkv[:, :, 2].transpose(1, 2))
        x = x + g1 * lin(p["to_out"], a.transpose(1, 2).reshape(1, N, C))
        h = F.layer_norm(x, (C,), f(p["n2w"]), f(p["n2b"]), 1e-6)
        cq = qknorm(lin(p["c_q"], h).view(1, N, H, D), p["cqg"])
        kv = lin(p["c_kv"], f(cond)).view(1, -1, 2, H, D)
        ck = qknorm(kv[:, :, 0], p["ckg"])
        ca = F.scaled_dot_product_attention(cq.transpose(1, 2), ck.transpose(1, 2), kv[:, :, 1].transpose(1, 2))
        x = x + lin(p["c_out"], ca.transpose(1, 2).reshape(1, N, C))
        h = F.layer_norm(x, (C,), eps=1e-6) * (1 + sc2) + sh2
        x = x + g2 * lin(p["mlp2"], F.gelu(lin(p["mlp0"], h), approximate="tanh"))
    ref = F.linear(F.layer_norm(x, (C,), eps=1e-5).view(N, C), f(m.out_layer[0]), f(m.out_layer[1]))
    assert out.shape == (N, 32)
    assert rel_l2(out, ref) < 2e-2
