"""GPU parity: the dense bf16 linear with its fused epilogue (l3d_linear_ex;
candle_nn::Linear::forward / ops::mul_mat_add, crate/runtime/nn_blocks.rs:
82,179-195, and the element-wise ops the blocks run after it) against the f64
product of the same bf16 operands.

Bounds as for the dequant-linear epilogue: the GEMM's f32 accumulation
(2e-5 * sum |x||w|, scaled by the largest derivative of the activation,
< 1.13), one rounding to bf16 (2^-8 relative) and the tanh.approx /
ex2.approx forms of the 16-bit activations (3e-4 |z|)."""
import numpy as np
import pytest

from conftest import rng
from test_gpu_qlinear import _act_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,act,res,gate,ydt,wview,bdt", [
    (700, 1024, 1536, "gelu_erf", False, False, "bf16", False, "f32"),  # VGGT fc1 + GELU-erf
    (600, 768, 512, "gelu", False, False, "f32", False, "f32"),
    (700, 1536, 1024, None, True, True, "bf16", False, "f32"),          # x += ls * proj(h), in place
    (300, 300, 256, "silu", True, False, "f32", False, "f32"),          # N tail
    (37, 520, 1000, None, True, True, "bf16", False, "f32"),            # small M, N and K tails
    (256, 384, 512, None, False, False, "bf16", True, "f32"),           # weight = rows of a wider matrix
    (700, 1024, 1024, "gelu_erf", False, False, "bf16", False, "bf16"),  # bf16 bias (the stacks' dtype)
    (300, 300, 256, None, False, False, "f32", False, "bf16"),          # bf16 bias with an N tail
])
def test_linear_fused_epilogue(ops, dev, M, N, K, act, res, gate, ydt, wview, bdt):
    import torch

    r = rng(300 + M + N)
    x = torch.from_numpy(r.standard_normal((M, K)).astype(np.float32)).to(dev).to(torch.bfloat16)
    wfull = torch.from_numpy((r.standard_normal((N, K + (64 if wview else 0))) / np.sqrt(K))
                             .astype(np.float32)).to(dev).to(torch.bfloat16)
    w = wfull[:, :K]
    b = torch.from_numpy((0.1 * r.standard_normal(N)).astype(np.float32)).to(dev)
    if bdt == "bf16":
        b = b.to(torch.bfloat16)
    xv = x.float().cpu().numpy().astype(np.float64)
    wv = w.float().cpu().numpy().astype(np.float64)
    tdt = torch.float32 if ydt == "f32" else torch.bfloat16
    z = xv @ wv.T + b.float().cpu().numpy()
    bound = 1.2 * (2e-5 * (np.abs(xv) @ np.abs(wv).T)) + 1e-6
    ref = _act_ref(act, z)
    kw = {"act": act}
    if res:
        r0 = torch.from_numpy(r.standard_normal((M, N)).astype(np.float32)).to(dev).to(tdt)
        g = torch.from_numpy((0.5 + r.random(N)).astype(np.float32)).to(dev) if gate else None
        rv = r0.float().cpu().numpy().astype(np.float64)
        gv = g.cpu().numpy().astype(np.float64) if gate else 1.0
        ref = rv + gv * ref
        bound = bound * (np.max(np.abs(gv)) if gate else 1.0)
        kw.update(residual=r0, gate=g, out=r0)
    y = ops.linear(x, w, bias=b, out_dtype=tdt, **kw)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    if ydt == "bf16":
        bound = bound + np.abs(ref) * 2.0 ** -8 + (3e-4 * np.abs(z) if act else 0.0)
    else:
        bound = bound + 1e-6 * np.abs(ref)
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    assert ops._LIN_WS[x.device][:4].view(torch.int32).item() == 0  # no bounded wait expired
    if res:
        assert y.data_ptr() == r0.data_ptr()


def test_linear_rejects_unaligned_weight(ops, dev):
    import torch

    x = torch.zeros(4, 12, device=dev, dtype=torch.bfloat16)
    w = torch.zeros(8, 12, device=dev, dtype=torch.bfloat16)  # k = 12: rows not 16-byte multiples
    with pytest.raises(Exception, match="multiple of 8"):
        ops.linear(x, w)
