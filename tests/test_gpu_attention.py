"""GPU parity: tcgen05 flash attention (exact_sdpa_heads,
crate/runtime/attention_math.rs:199-259) against softmax(q k^T * scale) v in
torch f32 on the same bf16 inputs.

Numerics: S and the running O are f32 (tensor-core accumulation); P is
rounded to bf16 for the second product and the output to bf16, so the
bound is |err| <= 2e-2 * max(1, |ref|) (bf16 tolerance) with a relative-L2
check of 1e-2."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    return (s.softmax(-1) @ v.float())


@pytest.mark.parametrize("B,H,N,NK,D,layout", [
    (1, 2, 256, 256, 64, "bhnd"),       # whole tiles
    (2, 3, 200, 333, 64, "bhnd"),       # ragged q and kv tails, Nk != N
    (1, 16, 1374, 1374, 64, "qkv"),     # VGGT frame attention: views of [B, N, 3, H, D]
    (1, 4, 300, 300, 128, "bhnd"),      # D = 128 (TripoSG / TRELLIS heads)
    (1, 4, 190, 190, 64, "bnhd"),       # token-major q, k, v memory
    (1, 1, 5, 7, 64, "bhnd"),           # tiny
])
def test_attention_matches_torch(ops, dev, B, H, N, NK, D, layout):
    import torch

    g = torch.Generator().manual_seed(N * 7 + D)
    if layout == "qkv":
        qkv = torch.randn(B, N, 3, H, D, generator=g).to(dev, torch.bfloat16).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
    elif layout == "bnhd":
        q = torch.randn(B, N, H, D, generator=g).to(dev, torch.bfloat16).transpose(1, 2)
        k = torch.randn(B, NK, H, D, generator=g).to(dev, torch.bfloat16).transpose(1, 2)
        v = torch.randn(B, NK, H, D, generator=g).to(dev, torch.bfloat16).transpose(1, 2)
    else:
        q = torch.randn(B, H, N, D, generator=g).to(dev, torch.bfloat16)
        k = torch.randn(B, H, NK, D, generator=g).to(dev, torch.bfloat16)
        v = torch.randn(B, H, NK, D, generator=g).to(dev, torch.bfloat16)
    scale = D ** -0.5
    out = ops.attention(q, k, v, scale)
    torch.cuda.synchronize()
    ws = ops.attention_workspace(q.device)
    assert ws[:4].view(torch.int32).item() == 0  # no bounded wait expired
    ref = _ref(q, k, v, scale)
    got = out.float()
    err = (got - ref).abs()
    assert torch.all(err <= 2e-2 * torch.clamp(ref.abs(), min=1.0)), f"max err {err.max().item():.3e}"
    rel = (torch.linalg.norm(got - ref) / torch.linalg.norm(ref)).item()
    assert rel < 1e-2, rel


def test_attention_sharp_softmax(ops, dev):
    """Scores of large magnitude (max changes across tiles): the running max /
    rescale path."""
    import torch

    g = torch.Generator().manual_seed(5)
    B, H, N, D = 1, 2, 640, 64
    q = (4 * torch.randn(B, H, N, D, generator=g)).to(dev, torch.bfloat16)
    k = (4 * torch.randn(B, H, N, D, generator=g)).to(dev, torch.bfloat16)
    v = torch.randn(B, H, N, D, generator=g).to(dev, torch.bfloat16)
    out = ops.attention(q, k, v, D ** -0.5)
    ref = _ref(q, k, v, D ** -0.5)
    rel = (torch.linalg.norm(out.float() - ref) / torch.linalg.norm(ref)).item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("span", [12.0, 60.0])
def test_attention_rising_scores(ops, dev, D, span):
    """Scores that rise along the keys by `span` (natural-log units) over the
    sequence: the row max grows tile after tile, sometimes by less than the
    rescale threshold (O keeps the stale max) and sometimes by more."""
    import torch

    g = torch.Generator().manual_seed(D + int(span))
    B, H, N, NK = 1, 2, 300, 700
    u = torch.randn(D, generator=g)
    u = u / u.norm()
    q = (u * D ** 0.5).expand(B, H, N, D).contiguous()
    ramp = torch.linspace(0, span, NK)[:, None] * u + 0.05 * torch.randn(NK, D, generator=g)
    k = ramp.expand(B, H, NK, D).contiguous()
    v = torch.randn(B, H, NK, D, generator=g)
    q, k, v = (t.to(dev, torch.bfloat16) for t in (q, k, v))
    out = ops.attention(q, k, v, D ** -0.5)
    torch.cuda.synchronize()
    assert ops.attention_workspace(q.device)[:4].view(torch.int32).item() == 0
    ref = _ref(q, k, v, D ** -0.5)
    err = (out.float() - ref).abs()
    assert torch.all(err <= 2e-2 * torch.clamp(ref.abs(), min=1.0)), f"max err {err.max().item():.3e}"
    rel = (torch.linalg.norm(out.float() - ref) / torch.linalg.norm(ref)).item()
    assert rel < 1e-2, rel


def test_attention_rejects_bad_scale(ops, dev):
    import torch

    q = torch.zeros(1, 1, 8, 64, device=dev, dtype=torch.bfloat16)
    with pytest.raises(Exception, match="scale"):
        ops.attention(q, q, q, -1.0)


@pytest.mark.parametrize("D", [64, 128])
def test_attention_single_key_returns_v(ops, dev, D):
    """softmax over one key is 1: every output row is that key's v row."""
    import torch

    g = torch.Generator().manual_seed(D)
    q = torch.randn(2, 3, 300, D, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(2, 3, 1, D, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(2, 3, 1, D, generator=g).to(dev, torch.bfloat16)
    out = ops.attention(q, k, v, D ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(out, v.expand(2, 3, 300, D))


def test_attention_empty_keys_give_zeros(ops, dev):
    import torch

    q = torch.randn(1, 2, 40, 64, device=dev).to(torch.bfloat16)
    kv = torch.zeros(1, 2, 0, 64, device=dev, dtype=torch.bfloat16)
    out = ops.attention(q, kv, kv, 0.125, out=torch.full_like(q, 7.0))
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0


@pytest.mark.parametrize("D", [64, 128])
def test_attention_one_query_odd_heads_strided_out(ops, dev, D):
    """nq = 1 (one row in a 256-row block), B x H = 3 x 5, and an output that
    is a view into a wider buffer."""
    import torch

    g = torch.Generator().manual_seed(7 + D)
    B, H, NK = 3, 5, 517
    q = torch.randn(B, H, 1, D, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(B, H, NK, D, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(B, H, NK, D, generator=g).to(dev, torch.bfloat16)
    buf = torch.zeros(B, 1, H, 2 * D, device=dev, dtype=torch.bfloat16)
    out = buf[..., :D].transpose(1, 2)  # [B, H, 1, D] with strides (H*2D, 2D, H*2D, 1)
    ops.attention(q, k, v, D ** -0.5, out=out)
    torch.cuda.synchronize()
    assert torch.count_nonzero(buf[..., D:]).item() == 0  # nothing written past the view
    ref = _ref(q, k, v, D ** -0.5)
    err = (out.float() - ref).abs()
    assert torch.all(err <= 2e-2 * torch.clamp(ref.abs(), min=1.0)), f"max err {err.max().item():.3e}"


@pytest.mark.parametrize("D", [64, 128])
def test_attention_bounded_wait_runs_out(pkg, ops, dev, D):
    """Failure handling without a GPU fault: the self-test launch never loads
    the first key tile, so the kernel's waits (limited to 50 ms) run out.  It
    must record status 5 in its workspace, wait for what it started, free its
    tensor memory and return; the context stays usable, so a normal (checked)
    call afterwards is exact again."""
    import ctypes as C

    import torch

    from candle3d_b200._lib import desc, ref

    g = torch.Generator().manual_seed(5 + D)
    q, k, v = (torch.randn(1, 2, 256, D, generator=g).to(dev, torch.bfloat16) for _ in range(3))
    k2, v2 = (torch.randn(1, 2, 640, D, generator=g).to(dev, torch.bfloat16) for _ in range(2))
    out = torch.zeros_like(q)
    ws = torch.full((256,), 0xFF, dtype=torch.uint8, device=dev)
    lib = pkg._lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for kk, vv in ((k, v), (k2, v2)):
        rc = lib.l3d_attention_selftest_timeout(ref(desc(q)), ref(desc(kk)), ref(desc(vv)),
                                                C.c_float(D ** -0.5), ref(desc(out)),
                                                C.c_void_p(ws.data_ptr()), C.c_size_t(256),
                                                C.c_uint32(50), C.c_void_p(stream))
        assert rc == 0, lib.l3d_last_error()
        torch.cuda.synchronize()
        assert ws[:4].view(torch.int32).item() == 5
    assert lib.l3d_attention_selftest_timeout(ref(desc(q)), ref(desc(k)), ref(desc(v)),
                                              C.c_float(1.0), ref(desc(out)),
                                              C.c_void_p(ws.data_ptr()), C.c_size_t(256),
                                              C.c_uint32(0), C.c_void_p(stream)) == 4
    got = ops.attention(q, k2, v2, D ** -0.5, check=True)
    ref_ = _ref(q, k2, v2, D ** -0.5)
    assert (got.float() - ref_).abs().max().item() < 2e-2
