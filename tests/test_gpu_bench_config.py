"""GPU parity at the exact shapes `bench.py` times:
LN + adaLN modulate with [C] shift/scale at C = 1536 / 2048, the TRELLIS
q/k L2-norm + 3D RoPE at 12 x 128 and 16 x 128 heads over voxel
coordinates spanning the whole 64^3 grid and the 1024^3 grid of the
TRELLIS.2 1024-resolution cascade, the VGGT per-head LN + 2D RoPE at the
bench's C = 1024 position grid, and the bench's own `Chain` end to end
against its CPU restatement (crate/runtime/trellis2_blocks.rs:106-160,
280-286,306-319,627-630; crate/runtime/attention_math.rs:127-150)."""
import numpy as np
import pytest

from conftest import assert_close, rng, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["bf16", "f32"])
@pytest.mark.parametrize("C", [1024, 1536, 2048])
def test_layer_norm_modulate_channel_vectors(ops, orc, dev, dt, C):
    """shift / scale as plain [C] vectors broadcast over 8192 token rows,
    the layout the bench passes (x ~ N(0, 1), shift / scale ~ N(0, 0.1))."""
    r = rng(40)
    T = 8192
    x, xv = to_dev(r.standard_normal((T, C)), dt, dev)
    sh, shv = to_dev(0.1 * r.standard_normal(C), dt, dev)
    sc, scv = to_dev(0.1 * r.standard_normal(C), dt, dev)
    y = ops.layer_norm_modulate(x, sh, sc, eps=1e-6)
    ref = orc.layer_norm_modulate(xv.reshape(1, T, C), shift=shv.reshape(1, C),
                                  scale=scv.reshape(1, C), eps=1e-6).reshape(T, C)
    assert_close(y.float().cpu().numpy(), ref, dt, f"ln+modulate C={C}")


def grid_coords(res, n, seed):
    """n voxel coordinates drawn uniformly from [0, res)^3 plus the grid's
    eight corners, row-sorted (x, y, z) as the reference sorts them."""
    r = np.random.default_rng(seed)
    c = r.integers(0, res, size=(n, 3))
    corners = np.array([[i, j, k] for i in (0, res - 1) for j in (0, res - 1) for k in (0, res - 1)])
    c = np.unique(np.concatenate([c, corners]), axis=0)
    return c.astype(np.int64)


@pytest.mark.parametrize("dt", ["bf16", "f32"])
@pytest.mark.parametrize("H", [12, 16])
@pytest.mark.parametrize("res,n", [(64, 16384), (1024, 8192)])
def test_qk_l2norm_rope3d_bench_heads(ops, orc, dev, dt, H, res, n):
    """D = 128 heads as the bench views a [T, C] row (C = 128 H), angles up to
    coordinate 1023 (each frequency-0 angle then reaches 1023 radians)."""
    import torch

    coords = grid_coords(res, n, 41 + res)
    T = coords.shape[0]
    r = rng(42)
    x, xv = to_dev(r.standard_normal((T, H * 128)), dt, dev)
    gamma = (1 + 0.02 * r.standard_normal((H, 128))).astype(np.float32)
    out = torch.empty_like(x)
    ops.qk_l2norm_rope3d(x.view(1, T, H, 128), torch.from_numpy(gamma).to(dev),
                         torch.from_numpy(coords.astype(np.int32)).to(dev), 10000.0,
                         out=out.view(1, T, H, 128))
    ref = orc.qk_l2norm_rope3d(xv.reshape(1, T, H, 128), gamma, coords, 10000.0)
    assert_close(out.float().cpu().numpy(), ref.reshape(T, H * 128), dt,
                 f"l2norm+rope3d H={H} res={res}")


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_qk_layernorm_rope2d_bench_grid(ops, orc, dev, dt):
    """The bench's C = 1024 second op: a [T, 1024] row viewed as 16 heads of 64,
    positions of a 64 x 64 grid repeated over the rows, q only, written into
    the permuted [1, H, T, D] view of a [T, C] buffer."""
    import torch

    T, H, D = 8192, 16, 64
    side = 64
    pos = np.stack([np.arange(T) // side % side + 1, np.arange(T) % side + 1], -1)
    pos = pos.reshape(1, T, 2).astype(np.int64)
    r = rng(43)
    x, xv = to_dev(r.standard_normal((T, H * D)), dt, dev)
    w, wv = to_dev(1 + 0.02 * r.standard_normal(D), dt, dev)
    b, bv = to_dev(0.02 * r.standard_normal(D), dt, dev)
    out = torch.empty_like(x)
    q = x.view(1, T, H, D).permute(0, 2, 1, 3)
    qo = out.view(1, T, H, D).permute(0, 2, 1, 3)
    ops.qk_layernorm_rope2d(q, None, w, b, None, None, 1e-5,
                            torch.from_numpy(pos.astype(np.int32)).to(dev), 100.0, q_out=qo)
    cs, sn = orc.rope2d_tables(pos, 100.0, D)
    qv = np.ascontiguousarray(xv.reshape(1, T, H, D).transpose(0, 2, 1, 3))
    ref = orc.layernorm_rope2d(qv, wv, bv, 1e-5, cs, sn)
    ref = ref.transpose(0, 2, 1, 3).reshape(T, H * D)
    assert_close(out.float().cpu().numpy(), ref, dt, "qk-ln+rope2d bench grid")


@pytest.mark.parametrize("C", [1024, 1536, 2048])
def test_bench_chain_matches_oracle(ops, orc, dev, C):
    """bench.py's timed Chain (the kernels and buffers it launches) on 8192
    rows of its own seeded inputs: each kernel against the oracle's op on the
    same input (the bench's own parity record), and the chain end to end
    against the oracle's chain within two bf16 ulps (one op's output may round
    to the other neighbour, which the next op carries on)."""
    import bench

    T = 8192
    host = bench.make_inputs(T, C, 20261201, None)
    inp = {k: (v.to(dev) if hasattr(v, "to") else tuple(p.to(dev) for p in v))
           for k, v in host.items()}
    chain = bench.Chain(ops, inp, T, C)
    stages = chain.stage_outputs(T)
    prev = None
    for i, got in enumerate(stages):
        assert_close(got, bench.chain_stage_reference(orc, host, C, i, prev), "bf16",
                     f"bench chain C={C} op {i}")
        prev = got
    assert bench.chain_parity(orc, host, C, stages)["ok"]
    ref = bench.chain_reference_cpu(orc, host, C)
    err = np.abs(stages[2] - ref)
    assert (err <= np.maximum(2e-2, np.abs(ref) * 2.0 ** -6)).all(), float(err.max())
