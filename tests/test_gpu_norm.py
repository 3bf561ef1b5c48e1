"""GPU parity: LayerNorm / adaLN modulation / residual / RMSNorm entries of the
C ABI against the C oracle (crate/runtime/trellis2_blocks.rs:280-286,627-645,
crate/runtime/vggt.rs:104-123,392-437, crate/runtime/triposg_dit.rs:511-522)."""
import numpy as np
import pytest

from conftest import assert_close, rng, to_dev

pytestmark = pytest.mark.gpu
DTS = ["f32", "bf16", "f16"]


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(2, 4096, 1024), (3, 7, 12), (1, 1, 1), (5, 1536), (2, 33, 2048),
                                   (4, 3, 100), (2, 8192), (1, 2, 2049)])
@pytest.mark.parametrize("affine", [True, False])
def test_layer_norm(ops, orc, dev, dt, shape, affine):
    r = rng(1)
    C = shape[-1]
    x, xv = to_dev(r.standard_normal(shape), dt, dev)
    w = b = wv = bv = None
    if affine:
        w, wv = to_dev(1 + 0.02 * r.standard_normal(C), dt, dev)
        b, bv = to_dev(0.02 * r.standard_normal(C), dt, dev)
    y = ops.layer_norm(x, w, b, eps=1e-6)
    ref = orc.layer_norm(xv, wv, bv, 1e-6)
    assert_close(y.float().cpu().numpy(), ref, dt, "layer_norm")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_layer_norm_strided_views(ops, orc, dev, dt):
    """Non-contiguous leading dims (a token slice and a transposed view)."""
    r = rng(2)
    x, xv = to_dev(r.standard_normal((3, 40, 256)), dt, dev)
    v = x[:, 1::3, :]
    y = ops.layer_norm(v, None, None, eps=1e-5)
    assert_close(y.float().cpu().numpy(), orc.layer_norm(xv[:, 1::3, :], eps=1e-5), dt, "slice")
    x2, x2v = to_dev(r.standard_normal((6, 5, 128)), dt, dev)
    t = x2.transpose(0, 1)
    y2 = ops.layer_norm(t, None, None, eps=1e-5)
    assert_close(y2.float().cpu().numpy(), orc.layer_norm(x2v.transpose(1, 0, 2), eps=1e-5), dt, "T")


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(2, 4096, 1024), (1, 300, 1536), (3, 5, 24)])
def test_layer_norm_modulate_chunk_views(ops, orc, dev, dt, shape):
    """shift/scale/gate as chunk views of a [B, 6C] adaLN vector
    (chunk_modulation, crate/runtime/trellis2_blocks.rs:264-277)."""
    r = rng(3)
    B, C = shape[0], shape[-1]
    x, xv = to_dev(r.standard_normal(shape), dt, dev)
    mod, modv = to_dev(0.1 * r.standard_normal((B, 6 * C)), dt, dev)
    sh, sc, gt, *_ = ops.chunk_modulation(mod)
    y = ops.layer_norm_modulate(x, sh, sc, eps=1e-6)
    ref = orc.layer_norm_modulate(xv, shift=modv[:, :C], scale=modv[:, C:2 * C], eps=1e-6)
    assert_close(y.float().cpu().numpy(), ref, dt, "ln+modulate")
    # VGGT camera-head adaLN: gate * (LN(x) (1 + scale) + shift) + x
    y2 = ops.layer_norm_modulate(x, sh, sc, gate=gt, add_input=True, eps=1e-6)
    ref2 = orc.layer_norm_modulate(xv, shift=modv[:, :C], scale=modv[:, C:2 * C],
                                   gate=modv[:, 2 * C:3 * C], add_input=True, eps=1e-6)
    assert_close(y2.float().cpu().numpy(), ref2, dt, "adaLN gate+residual")


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(2, 4096, 1024), (1, 7, 20)])
def test_gated_and_layerscale_residual(ops, orc, dev, dt, shape):
    r = rng(4)
    B, C = shape[0], shape[-1]
    x, xv = to_dev(r.standard_normal(shape), dt, dev)
    h, hv = to_dev(r.standard_normal(shape), dt, dev)
    g, gv = to_dev(0.1 * r.standard_normal((B, C)), dt, dev)
    out = ops.gated_residual(x, h, g)
    assert_close(out.float().cpu().numpy(), orc.gated_residual(xv, hv, gv), dt, "gated residual")
    gam, gamv = to_dev(np.full(C, 0.01, np.float32) + 0.001 * r.standard_normal(C), dt, dev)
    out2 = ops.layerscale_residual(x, h, gam)
    assert_close(out2.float().cpu().numpy(), orc.layerscale_residual(xv, hv, gamv), dt, "layerscale")


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("inplace", [False, True])
def test_residual_layer_norm_modulate(ops, orc, dev, dt, inplace):
    """x += gate * h followed by the next modulated LN, one pass; y is computed
    from the residual as stored (rounded to the activation dtype)."""
    r = rng(5)
    B, N, C = 2, 513, 1536
    x, xv = to_dev(r.standard_normal((B, N, C)), dt, dev)
    h, hv = to_dev(r.standard_normal((B, N, C)), dt, dev)
    mod, modv = to_dev(0.1 * r.standard_normal((B, 6 * C)), dt, dev)
    ch = ops.chunk_modulation(mod)
    rr, y = ops.residual_layer_norm_modulate(x, h, gate=ch[2], shift=ch[3], scale=ch[4], eps=1e-6,
                                             inplace=inplace)
    rref = orc.gated_residual(xv, hv, modv[:, 2 * C:3 * C])
    assert_close(rr.float().cpu().numpy(), rref, dt, "residual")
    rstored = rr.float().cpu().numpy()
    yref = orc.layer_norm_modulate(rstored, shift=modv[:, 3 * C:4 * C], scale=modv[:, 4 * C:5 * C],
                                   eps=1e-6)
    assert_close(y.float().cpu().numpy(), yref, dt, "next norm")
    if inplace:
        assert rr.data_ptr() == x.data_ptr()


@pytest.mark.parametrize("dt", DTS)
def test_rms_norm_heads_triposg_views(ops, orc, dev, dt):
    """q/k/v split of cat([q, k, v]).reshape(B, L, H, 3D) (crate/runtime/triposg_dit.rs:436-454)."""
    import torch

    r = rng(6)
    B, L, H, D = 2, 257, 16, 128
    qkv, qkvv = to_dev(r.standard_normal((B, L, H, 3 * D)), dt, dev)
    wq, wqv = to_dev(1 + 0.05 * r.standard_normal(D), dt, dev)
    q = qkv.chunk(3, dim=-1)[0].transpose(1, 2)  # [B, H, L, D] strided view
    y = ops.rms_norm_heads(q, wq, eps=1e-6)
    qv = np.ascontiguousarray(qkvv[..., :D].transpose(0, 2, 1, 3))
    assert_close(y.float().cpu().numpy(), orc.rms_norm_heads(qv, wqv, 1e-6), dt, "rms heads")
    assert y.is_contiguous()
    k = qkv.chunk(3, dim=-1)[1].transpose(1, 2)
    yk = ops.rms_norm_heads(k, wq, eps=1e-6)
    kv = np.ascontiguousarray(qkvv[..., D:2 * D].transpose(0, 2, 1, 3))
    assert_close(yk.float().cpu().numpy(), orc.rms_norm_heads(kv, wqv, 1e-6), dt, "rms heads k")
    del torch


def test_empty_rows_are_noops(ops, dev):
    import torch

    x = torch.empty((0, 64), device=dev)
    assert ops.layer_norm(x).shape == (0, 64)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("C,affine", [(2048, False), (1536, True), (1024, True), (4096, False)])
def test_layer_norm_ring_path_rows(ops, orc, dev, dt, C, affine):
    """Inputs of at least 32768 rows of 2-8 KB take the shared-memory ring
    kernel (bulk copies of whole rows): with and without affine vectors,
    modulation and gate; the kernels' status word stays 0."""
    import ctypes

    if C * {"f32": 4, "bf16": 2, "f16": 2}[dt] > 8192:
        C = 2048
    r = rng(7)
    T = 32768 + 77
    x, xv = to_dev(r.standard_normal((T, C)), dt, dev)
    w = b = wv = bv = None
    if affine:
        w, wv = to_dev(1 + 0.02 * r.standard_normal(C), dt, dev)
        b, bv = to_dev(0.02 * r.standard_normal(C), dt, dev)
    y = ops.layer_norm(x, w, b, eps=1e-6)
    assert_close(y.float().cpu().numpy(), orc.layer_norm(xv, wv, bv, 1e-6), dt, "ring LN")
    g, gv = to_dev(0.1 * r.standard_normal(C), dt, dev)
    sh, shv = to_dev(0.1 * r.standard_normal(C), dt, dev)
    y2 = ops.layer_norm_modulate(x, sh, None, gate=g, add_input=True, eps=1e-6)
    ref2 = orc.layer_norm_modulate(xv.reshape(1, T, C), shift=shv, gate=gv, add_input=True,
                                   eps=1e-6).reshape(T, C)
    assert_close(y2.float().cpu().numpy(), ref2, dt, "ring LN+modulate+gate")
    import torch

    torch.cuda.synchronize()
    st = ctypes.c_int(-1)
    assert ops._lib.lib().l3d_kernel_status(ctypes.byref(st), 1) == 0
    assert st.value == 0


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_layer_norm_modulate_ring_per_batch_chunks(ops, orc, dev, dt):
    """The ring kernel with per-batch adaLN vectors: shift / scale / gate as
    chunk views of a [B, 6C] vector over 2 x 16401 rows of C = 1024 (one
    consumer's row pair then straddles the batch boundary, so the pair's
    coefficients differ)."""
    r = rng(8)
    B, N, C = 2, 16401, 1024
    x, xv = to_dev(r.standard_normal((B, N, C)), dt, dev)
    mod, modv = to_dev(0.1 * r.standard_normal((B, 6 * C)), dt, dev)
    sh, sc, gt, *_ = ops.chunk_modulation(mod)
    y = ops.layer_norm_modulate(x, sh, sc, gate=gt, eps=1e-6)
    ref = orc.layer_norm_modulate(xv, shift=modv[:, :C], scale=modv[:, C:2 * C],
                                  gate=modv[:, 2 * C:3 * C], eps=1e-6)
    assert_close(y.float().cpu().numpy(), ref, dt, "ring per-batch adaLN")
