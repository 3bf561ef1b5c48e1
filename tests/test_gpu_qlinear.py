"""GPU parity: tcgen05 dequant-linear (QMatMul on GGML Q8_0 / Q4_0 blocks,
crate/runtime/nn_blocks.rs:80-95) against the oracle.

Numerics contract of the kernel: the activations are bf16, each weight is
decoded as d * q in f32 and rounded once to bf16 (the tensor-core operand),
products are accumulated in f32.  The test therefore compares against the
exact (f64) product of the same bf16 operands with a bound proportional to
sum_k |x_k| |w_k| (f32 accumulation), and separately checks that rounding the
weights to bf16 costs far less accuracy than the Q8_0 / Q4_0 format itself
(the quant_probe methodology, crates/lux3d-core/examples/quant_probe.rs:84-123).
"""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu


def _case(orc, M, N, K, fmt, seed, scale_rows=True):
    r = rng(seed)
    x = r.standard_normal((M, K)).astype(np.float32)
    # int8 per-output-channel symmetric weights with scales ~ U(0.001, 0.02),
    # encoded as GGML blocks (config 4).
    s = r.uniform(0.001, 0.02, size=(N, 1)).astype(np.float32) if scale_rows else 0.02
    w = (np.clip(np.round(r.standard_normal((N, K)) * 40), -127, 127) * s).astype(np.float32)
    q = orc.quantize(w, fmt)
    b = (0.1 * r.standard_normal(N)).astype(np.float32)
    return x, q, b


@pytest.mark.parametrize("M,N,K,fmt,ydt,bias", [
    (1000, 4608, 1536, "q8_0", "f32", True),     # to_qkv shape, TMA raw window path
    (257, 1536, 8192, "q8_0", "f32", True),      # mlp.2 shape, M tail
    (300, 300, 96, "q4_0", "f32", False),        # K % 256 != 0: direct-load path, N tail
    (4, 3072, 1024, "q4_0", "f32", True),        # to_kv, tiny M
    (513, 1536, 1536, "q8_0", "bf16", True),     # bf16 output
    (128, 256, 256, "q8_0", "f32", False),       # exactly one tile
    (64, 100, 256, "q8_0", "bf16", True),        # rows of 200 B: scalar stores (direct path)
    (700, 100, 512, "q8_0", "f32", True),        # rows of 400 B, decode-once mode
])
def test_dequant_linear_matches_oracle(ops, orc, dev, M, N, K, fmt, ydt, bias):
    import torch

    x, q, b = _case(orc, M, N, K, fmt, 40 + M)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    xv = xb.float().cpu().numpy().astype(np.float64)
    wdeq = orc.dequantize(q, fmt, N, K)
    wb = orc.round_bf16(wdeq).astype(np.float64)
    bt = torch.from_numpy(b).to(dev) if bias else None
    mm = ops.QMatMul(torch.from_numpy(q).to(dev), fmt, N, K, bias=bt)
    y = mm(xb, out_dtype=torch.float32 if ydt == "f32" else torch.bfloat16)
    torch.cuda.synchronize()
    ref = xv @ wb.T + (b if bias else 0.0)
    bound = 2e-5 * (np.abs(xv) @ np.abs(wb).T) + 1e-6
    if ydt == "bf16":
        bound = bound + np.abs(ref) * 2.0 ** -8
    err = np.abs(y.float().cpu().numpy() - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    # Rounding the decoded weights to bf16 is well inside the format's own error.
    exact = xv @ wdeq.astype(np.float64).T + (b if bias else 0.0)
    rel = np.linalg.norm(ref - exact) / np.linalg.norm(exact)
    assert rel < 4e-3


def test_dequant_linear_f32_input_and_strided_rows(ops, orc, dev):
    import torch

    M, N, K = 200, 512, 512
    x, q, b = _case(orc, M, N, K, "q8_0", 77)
    big = torch.zeros(M, K + 64, device=dev)
    big[:, :K] = torch.from_numpy(x).to(dev)
    xv = big[:, :K]  # row stride K + 64 (F32 -> converted in the workspace)
    mm = ops.QMatMul(torch.from_numpy(q).to(dev), "q8_0", N, K, bias=torch.from_numpy(b).to(dev))
    y = mm(xv, out_dtype=torch.float32)
    xr = torch.from_numpy(x).to(torch.bfloat16).float().numpy().astype(np.float64)
    wb = orc.round_bf16(orc.dequantize(q, "q8_0", N, K)).astype(np.float64)
    ref = xr @ wb.T + b
    bound = 2e-5 * (np.abs(xr) @ np.abs(wb).T) + 1e-6
    assert np.all(np.abs(y.cpu().numpy() - ref) <= bound)


def test_dequant_linear_repeated_calls_are_deterministic(ops, orc, dev):
    import torch

    M, N, K = 640, 1024, 1536
    x, q, b = _case(orc, M, N, K, "q8_0", 5)
    mm = ops.QMatMul(torch.from_numpy(q).to(dev), "q8_0", N, K)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    y1 = mm(xb, out_dtype=torch.float32)
    y2 = mm(xb, out_dtype=torch.float32)
    assert torch.equal(y1, y2)
    ws = mm.workspace(M)
    assert int(ws[:4].view(torch.int32).item()) == 0  # kernel status word: no timeouts


@pytest.mark.parametrize("fmt", ["q4_k", "q5_k", "q6_k"])
def test_dequantize_kquants_bit_exact(ops, orc, dev, fmt):
    """Device decode of K-quant super-blocks equals the oracle bit for bit
    (f32 out), and its bf16 output is the oracle rounded once."""
    import torch

    from conftest import random_kquant_blocks

    n, k = 96, 2048
    blk = random_kquant_blocks(rng(500 + len(fmt)), fmt, n, k)
    ref = orc.dequantize(blk, fmt, n, k)
    q = torch.from_numpy(blk).to(dev)
    got = ops.dequantize(q, fmt, n, k, dtype=torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    gb = ops.dequantize(q, fmt, n, k, dtype=torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(gb, orc.round_bf16(ref))


@pytest.mark.parametrize("M,N,K,fmt", [
    (37, 512, 1024, "q4_k"),     # small M: K-quants decode once as well
    (700, 1536, 1536, "q6_k"),   # TRELLIS to_out shape
    (300, 768, 2048, "q5_k"),
])
def test_dequant_linear_kquants(ops, orc, dev, M, N, K, fmt):
    import torch

    from conftest import random_kquant_blocks

    r = rng(600 + M)
    x = r.standard_normal((M, K)).astype(np.float32)
    blk = random_kquant_blocks(r, fmt, N, K)
    b = (0.1 * r.standard_normal(N)).astype(np.float32)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    xv = xb.float().cpu().numpy().astype(np.float64)
    wb = orc.round_bf16(orc.dequantize(blk, fmt, N, K)).astype(np.float64)
    mm = ops.QMatMul(torch.from_numpy(blk).to(dev), fmt, N, K, bias=torch.from_numpy(b).to(dev))
    y = mm(xb, out_dtype=torch.float32).cpu().numpy()
    ref = xv @ wb.T + b
    bound = 2e-5 * (np.abs(xv) @ np.abs(wb).T) + 1e-6
    err = np.abs(y - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"


def _act_ref(name, z):
    from math import sqrt

    from scipy.special import erf

    if name == "gelu":
        return 0.5 * z * (1.0 + np.tanh(sqrt(2.0 / np.pi) * (z + 0.044715 * z ** 3)))
    if name == "gelu_erf":
        return 0.5 * z * (1.0 + erf(z / sqrt(2.0)))
    if name == "silu":
        return z / (1.0 + np.exp(-z))
    return z


@pytest.mark.parametrize("M,N,K,act,res,gate,ydt", [
    (700, 1024, 1536, "gelu", False, False, "bf16"),       # mlp.0 + GELU-tanh, TMA-store epilogue
    (64, 512, 512, "gelu", False, False, "bf16"),          # small M: fused-decode mode, direct stores
    (600, 768, 512, "gelu_erf", False, False, "f32"),      # accurate activation for f32 output
    (700, 1536, 1024, None, True, True, "bf16"),           # x += gate * linear(h), in place
    (300, 300, 256, "silu", True, False, "f32"),           # N tail, residual without gate
    (37, 520, 1024, None, True, True, "bf16"),             # small M, N tail, gated residual
    (600, 300, 512, "gelu", True, True, "f32"),            # f32 residual tiles by TMA, N tail
])
def test_dequant_linear_fused_epilogue(ops, orc, dev, M, N, K, act, res, gate, ydt):
    """y = residual + gate * act(x . W^T + b) against the f64 product of the same
    bf16 operands; bounds: the GEMM's f32 accumulation (scaled by the largest
    derivative of the activation, < 1.13), one rounding to bf16, and the
    tanh.approx / ex2.approx forms used for 16-bit outputs (abs. error below
    3e-4 |z|)."""
    import torch

    x, q, b = _case(orc, M, N, K, "q8_0", 90 + M)
    r = rng(91 + M)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    xv = xb.float().cpu().numpy().astype(np.float64)
    wb = orc.round_bf16(orc.dequantize(q, "q8_0", N, K)).astype(np.float64)
    tdt = torch.float32 if ydt == "f32" else torch.bfloat16
    mm = ops.QMatMul(torch.from_numpy(q).to(dev), "q8_0", N, K, bias=torch.from_numpy(b).to(dev))
    z = xv @ wb.T + b
    bound = 1.2 * (2e-5 * (np.abs(xv) @ np.abs(wb).T)) + 1e-6
    ref = _act_ref(act, z)
    kw = {"act": act}
    if res:
        r0 = torch.from_numpy(r.standard_normal((M, N)).astype(np.float32)).to(dev).to(tdt)
        g = torch.from_numpy((0.5 + r.random(N)).astype(np.float32)).to(dev) if gate else None
        rv = r0.float().cpu().numpy().astype(np.float64)
        gv = g.cpu().numpy().astype(np.float64) if gate else 1.0
        ref = rv + gv * ref
        bound = bound * (np.max(np.abs(gv)) if gate else 1.0)
        kw.update(residual=r0, gate=g, out=r0)  # in place: x += gate * ...
    y = mm(xb, out_dtype=tdt, **kw)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    if ydt == "bf16":
        bound = bound + np.abs(ref) * 2.0 ** -8 + (3e-4 * np.abs(z) if act else 0.0)
    else:
        bound = bound + 1e-6 * np.abs(ref)
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    if res:
        assert y.data_ptr() == r0.data_ptr()
