"""Candle-shaped front end of libl3dops for torch tensors on a CUDA device.

Each function mirrors the Candle op (or composed op chain) the Lux3D model
code calls, with the same argument meaning, and runs the sm_100a kernel
through the C ABI.  Like a Candle `CustomOp::cuda_fwd`, every op allocates its
output on the input's device and enqueues the kernel on the current stream.
Invalid inputs raise `L3dError` carrying the library's status and message.
("crate/" below = crates/lux3d-core/src/ of the reference.)
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import _lib
from ._lib import call, desc, ref, stream_handle

ACT = {"none": 0, "silu": 1, "gelu_erf": 2, "gelu_tanh": 3}


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libl3dops ops take CUDA tensors (no CPU implementation exists)")


def _s(t):
    return stream_handle(t.device)


# ------------------------------------------------------------- LayerNorm family
def layer_norm(x, weight=None, bias=None, eps=1e-5):
    """candle_nn::LayerNorm::forward / ops::layer_norm (crate/runtime/vggt.rs:104)."""
    _check_cuda(x, weight, bias)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call("l3d_layer_norm", ref(desc(x)), ref(desc(weight)), ref(desc(bias)), eps, ref(desc(y)),
         _s(x))
    return y


def layer_norm_no_affine(x, eps=1e-6):
    """layer_norm_no_affine (crate/runtime/trellis2_blocks.rs:280-286)."""
    return layer_norm(x, None, None, eps)


def layer_norm_modulate(x, shift=None, scale=None, gate=None, add_input=False, weight=None,
                        bias=None, eps=1e-6):
    """LN(x)[*w+b] * (1 + scale) + shift, then optional gate and + x.
    crate/runtime/trellis2_blocks.rs:627-630 (norm + modulate) and the VGGT camera
    head adaLN crate/runtime/vggt.rs:399-405 (gate * modulated + x)."""
    _check_cuda(x, shift, scale, gate, weight, bias)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call("l3d_layer_norm_modulate", ref(desc(x)), ref(desc(weight)), ref(desc(bias)),
         ref(desc(shift)), ref(desc(scale)), ref(desc(gate)), int(bool(add_input)), eps,
         ref(desc(y)), _s(x))
    return y


def gated_residual(x, h, gate=None):
    """x + h * gate (crate/runtime/trellis2_blocks.rs:632-633); gate None: x + h."""
    _check_cuda(x, h, gate)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call("l3d_gated_residual", ref(desc(x)), ref(desc(h)), ref(desc(gate)), ref(desc(out)), _s(x))
    return out


def layerscale_residual(x, h, gamma):
    """x + LayerScale(h) (crate/runtime/nn_blocks.rs:210-214, crate/runtime/vggt.rs:118)."""
    _check_cuda(x, h, gamma)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call("l3d_layerscale_residual", ref(desc(x)), ref(desc(h)), ref(desc(gamma)), ref(desc(out)),
         _s(x))
    return out


def residual_layer_norm_modulate(x, h, gate=None, weight=None, bias=None, shift=None, scale=None,
                                 eps=1e-6, inplace=False):
    """r = x + gate * h; y = LN(r)[*w+b][*(1+scale)+shift]; returns (r, y).
    With inplace=True the residual stream x is updated in place (r is x)."""
    _check_cuda(x, h, gate, weight, bias, shift, scale)
    r = x if inplace else torch.empty(x.shape, dtype=x.dtype, device=x.device)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call("l3d_residual_layer_norm_modulate", ref(desc(x)), ref(desc(h)), ref(desc(gate)),
         ref(desc(weight)), ref(desc(bias)), ref(desc(shift)), ref(desc(scale)), eps,
         ref(desc(r)), ref(desc(y)), _s(x))
    return r, y


def rms_norm_heads(x, weight, eps=1e-6, out=None):
    """RmsNormHeads::rms_norm_heads (crate/runtime/triposg_dit.rs:511-522).
    Output is contiguous in x's logical shape (strided chunk views accepted),
    or written into `out` (x's shape, rows strided, last dim contiguous)."""
    _check_cuda(x, weight)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device) if out is None else out
    call("l3d_rms_norm_heads", ref(desc(x)), ref(desc(weight)), eps, ref(desc(y)), _s(x))
    return y


# -------------------------------------------------------------------- 2D RoPE
class RopeEmbeddings:
    """cos_full / sin_alt_full tables [B, 1, N, D] (crate/runtime/attention_math.rs:88-95)."""

    def __init__(self, cos_full, sin_alt_full):
        self.cos_full = cos_full
        self.sin_alt_full = sin_alt_full


class Rope2d:
    """Rope2d (crate/runtime/attention_math.rs:4-85); tables built on the device."""

    def __init__(self, base: float = 100.0):
        self.base = float(base)

    def embeddings(self, positions, token_dim: int) -> RopeEmbeddings:
        _check_cuda(positions)
        B, N, _ = positions.shape
        c = torch.empty((B, 1, N, token_dim), dtype=torch.float32, device=positions.device)
        s = torch.empty_like(c)
        call("l3d_rope2d_tables", ref(desc(positions)), self.base, token_dim, ref(desc(c)),
             ref(desc(s)), _s(positions))
        return RopeEmbeddings(c, s)


def layernorm_rope_fused(q, weight, bias, eps, cos_full, sin_alt_full):
    """candle_nn::ops::layernorm_rope_fused (crate/runtime/attention_math.rs:139-146):
    per-head LN of the (possibly strided) [B, H, N, 64] view, then 2D RoPE;
    contiguous [B, H, N, 64] output."""
    _check_cuda(q, weight, bias, cos_full, sin_alt_full)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    call("l3d_layernorm_rope2d", ref(desc(q)), ref(desc(weight)), ref(desc(bias)), eps,
         ref(desc(cos_full)), ref(desc(sin_alt_full)), ref(desc(out)), _s(q))
    return out


def rope_fused(x, cos_full, sin_alt_full):
    """candle_nn::ops::rope_fused (crate/runtime/attention_math.rs:155-165)."""
    return layernorm_rope_fused(x, None, None, 0.0, cos_full, sin_alt_full)


def qk_layernorm_rope2d(q, k, q_weight, q_bias, k_weight, k_bias, eps, positions, theta=100.0,
                        q_out=None, k_out=None):
    """q and k of one attention in one launch, angles from integer positions
    (no table traffic).  Outputs default to contiguous [B, H, N, 64]."""
    _check_cuda(q, k, positions)
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device) if q_out is None else q_out
    if k is not None and k_out is None:
        k_out = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    call("l3d_qk_layernorm_rope2d_pos", ref(desc(q)), ref(desc(q_weight)), ref(desc(q_bias)),
         ref(desc(k)), ref(desc(k_weight)), ref(desc(k_bias)), eps, ref(desc(positions)),
         float(theta), ref(desc(q_out)), ref(desc(k_out)), _s(q))
    return q_out, k_out


def position_getter(batch: int, h: int, w: int, device) -> torch.Tensor:
    """position_getter (crate/runtime/attention_math.rs:167-183): (y + 1, x + 1)."""
    ys = torch.arange(1, h + 1, device=device, dtype=torch.int64)
    xs = torch.arange(1, w + 1, device=device, dtype=torch.int64)
    grid = torch.stack(torch.meshgrid(ys, xs, indexing="ij"), -1).reshape(1, h * w, 2)
    return grid.expand(batch, h * w, 2).contiguous()


# -------------------------------------------------------------------- 3D RoPE
def cubic_token_coords(resolution: int, device=None) -> torch.Tensor:
    """cubic_token_coords (crate/runtime/trellis2_blocks.rs:166-178): row-major
    x * res^2 + y * res + z."""
    r = torch.arange(resolution, device=device, dtype=torch.int64)
    g = torch.stack(torch.meshgrid(r, r, r, indexing="ij"), -1)
    return g.reshape(-1, 3).contiguous()


class Trellis2Rope3d:
    """Trellis2Rope3d (crate/runtime/trellis2_blocks.rs:85-161)."""

    def __init__(self, head_dim: int, rope_base: float = 10000.0):
        self.head_dim = head_dim
        self.rope_base = float(rope_base)

    def cos_sin(self, coords):
        _check_cuda(coords)
        L = coords.shape[0]
        c = torch.empty((L, self.head_dim // 2), dtype=torch.float32, device=coords.device)
        s = torch.empty_like(c)
        call("l3d_rope3d_tables", ref(desc(coords)), self.head_dim, self.rope_base, ref(desc(c)),
             ref(desc(s)), _s(coords))
        return c, s

    def apply(self, x, cos, sin):
        _check_cuda(x, cos, sin)
        y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        call("l3d_rope3d_apply", ref(desc(x)), ref(desc(cos)), ref(desc(sin)), ref(desc(y)), _s(x))
        return y


def qk_l2norm_rope3d(x, gamma, coords, theta=10000.0, out=None):
    """Trellis2QkRmsNorm::forward + Trellis2Rope3d::apply in one pass
    (crate/runtime/trellis2_blocks.rs:306-319, :139-160); coords None = norm only."""
    _check_cuda(x, gamma, coords)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device) if out is None else out
    call("l3d_qk_l2norm_rope3d", ref(desc(x)), ref(desc(gamma)), ref(desc(coords)), float(theta),
         ref(desc(out)), _s(x))
    return out


# ---------------------------------------------------------------- activations
def _unary(name, x):
    _check_cuda(x)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    call(name, ref(desc(x)), ref(desc(y)), _s(x))
    return y


def gelu(x):
    """Tensor::gelu, tanh form (crate/runtime/trellis2_blocks.rs:558-561)."""
    return _unary("l3d_gelu_tanh", x)


def gelu_erf(x):
    """Tensor::gelu_erf (crate/runtime/nn_blocks.rs:233)."""
    return _unary("l3d_gelu_erf", x)


def silu(x):
    """Tensor::silu (crate/runtime/trellis2_blocks.rs:236)."""
    return _unary("l3d_silu", x)


def geglu(x):
    """GeGlu::forward after the projection (crate/runtime/nn_blocks.rs:250-253)."""
    _check_cuda(x)
    y = torch.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=x.dtype, device=x.device)
    call("l3d_geglu", ref(desc(x)), ref(desc(y)), _s(x))
    return y


# ------------------------------------------------------- timestep / linears
def timestep_embedding(t, dim: int, order: str = "cos_first", max_period: float = 10000.0,
                       dtype=torch.float32):
    """TRELLIS.2 (`cos_first`, crate/runtime/trellis2_blocks.rs:184-204) or TripoSG
    (`sin_first`, crate/runtime/triposg_dit.rs:280-294) sinusoidal table, [B, dim]."""
    _check_cuda(t)
    t = t.reshape(-1).to(torch.float32)
    out = torch.empty((t.numel(), dim), dtype=dtype, device=t.device)
    code = {"cos_first": 0, "sin_first": 1}[order]
    call("l3d_timestep_embedding", ref(desc(t)), dim, code, float(max_period), ref(desc(out)),
         _s(t))
    return out


def linear_small(x, w, bias=None, addend=None, act_in="none", act_out="none", out_dtype=None):
    """act_out(act_in(x) @ w.T + bias + addend) for small batches (per-step vectors)."""
    _check_cuda(x, w, bias, addend)
    y = torch.empty((x.shape[0], w.shape[0]), dtype=out_dtype or x.dtype, device=x.device)
    call("l3d_linear_small", ref(desc(x)), ref(desc(w)), ref(desc(bias)), ref(desc(addend)),
         ACT[act_in], ACT[act_out], ref(desc(y)), _s(x))
    return y


def ada_ln(t_emb, weight, bias, block_modulation=None):
    """Trellis2AdaLn::forward (SiLU -> Linear(C, 6C), trellis2_blocks.rs:243-258),
    optionally + the block's `modulation` vector (:617)."""
    return linear_small(t_emb, weight, bias, block_modulation, act_in="silu")


def chunk_modulation(mod_vec, chunks: int = 6):
    """chunk_modulation (crate/runtime/trellis2_blocks.rs:264-277): views
    (shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp), each [B, 1, C]."""
    return [c.unsqueeze(1) for c in mod_vec.chunk(chunks, dim=-1)]


def patch_embed(pixels, weight, bias, pos, cls, reg, patch: int):
    """PatchEmbed + prepare_tokens (crate/runtime/pi3_encoder.rs:116-126,219-231)."""
    _check_cuda(pixels, weight, bias, pos, cls, reg)
    BS, _, H, W = pixels.shape
    R = 0 if reg is None else reg.shape[0]
    np_ = (H // patch) * (W // patch)
    out = torch.empty((BS, 1 + R + np_, weight.shape[0]), dtype=pixels.dtype, device=pixels.device)
    call("l3d_patch_embed", ref(desc(pixels)), ref(desc(weight)), ref(desc(bias)), ref(desc(pos)),
         ref(desc(cls)), ref(desc(reg)), patch, ref(desc(out)), _s(pixels))
    return out


# ------------------------------------------------------------- dequant-linear
QFMT = {"q8_0": _lib.Q8_0, "q4_0": _lib.Q4_0, "q4_k": _lib.Q4_K, "q5_k": _lib.Q5_K,
        "q6_k": _lib.Q6_K}
BLOCK_BYTES = {"q8_0": 34, "q4_0": 18, "q4_k": 144, "q5_k": 176, "q6_k": 210}
BLOCK_ELEMS = {"q8_0": 32, "q4_0": 32, "q4_k": 256, "q5_k": 256, "q6_k": 256}
ACT_CODES = {None: 0, "silu": 1, "gelu_erf": 2, "gelu": 3}


def dequantize(wq, fmt: str, n: int, k: int, dtype=torch.float32):
    """QTensor::dequantize of raw GGML blocks (uint8 CUDA tensor)."""
    _check_cuda(wq)
    out = torch.empty((n, k), dtype=dtype, device=wq.device)
    call("l3d_dequantize", wq.data_ptr(), QFMT[fmt], n, k, ref(desc(out)), _s(wq))
    return out


class QMatMul:
    """Quantized linear weight kept packed on the device
    (LinearInner::Quant, crate/runtime/nn_blocks.rs:51-56,80-95)."""

    def __init__(self, blocks, fmt: str, n: int, k: int, bias=None):
        _check_cuda(blocks, bias)
        if blocks.numel() != n * (k // BLOCK_ELEMS[fmt]) * BLOCK_BYTES[fmt]:
            raise ValueError("block buffer size does not match [n, k]")
        self.blocks, self.fmt, self.n, self.k, self.bias = blocks, fmt, n, k, bias
        self._ws = None

    def workspace(self, m: int):
        need = _lib.lib().l3d_dequant_linear_workspace_size(QFMT[self.fmt], m, self.n, self.k)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.blocks.device)
        return self._ws

    def forward(self, x, out_dtype=None, act=None, residual=None, gate=None, out=None):
        """y = x . deq(W)^T + bias; with `act` ("gelu", "gelu_erf", "silu") and/or
        `residual` (+ per-column `gate`) the block's next ops run in the GEMM
        epilogue: y = residual + gate * act(...).  `out` may be `residual`."""
        _check_cuda(x, residual, gate, out)
        x2 = x.reshape(-1, self.k)
        if out is not None:
            y = out.reshape(-1, self.n)
        else:
            y = torch.empty((x2.shape[0], self.n), dtype=out_dtype or x.dtype, device=x.device)
        ws = self.workspace(x2.shape[0])
        r2 = None if residual is None else residual.reshape(-1, self.n)
        if act is None and residual is None:
            call("l3d_dequant_linear", ref(desc(x2)), self.blocks.data_ptr(), QFMT[self.fmt], self.n,
                 self.k, ref(desc(self.bias)), ref(desc(y)), ws.data_ptr(), ws.numel(), _s(x))
        else:
            call("l3d_dequant_linear_ex", ref(desc(x2)), self.blocks.data_ptr(), QFMT[self.fmt],
                 self.n, self.k, ref(desc(self.bias)), ACT_CODES[act], ref(desc(r2)),
                 ref(desc(gate)), ref(desc(y)), ws.data_ptr(), ws.numel(), _s(x))
        return y.reshape(*x.shape[:-1], self.n)

    __call__ = forward


_LIN_WS = {}


def linear(x, weight, bias=None, act=None, residual=None, gate=None, out=None, out_dtype=None):
    """candle_nn::Linear::forward / ops::mul_mat_add on a bf16 [n, k] weight
    (crate/runtime/nn_blocks.rs:82,179-195) on the tensor cores, with the
    block's next element-wise ops in the GEMM epilogue:
    y = residual + gate * act(x . W^T + bias) (act "gelu" (tanh), "gelu_erf",
    "silu"; `out` may be `residual`)."""
    _check_cuda(x, weight, bias, residual, gate, out)
    n, k = weight.shape
    x2 = x.reshape(-1, k)
    if out is not None:
        y = out.reshape(-1, n)
    else:
        y = torch.empty((x2.shape[0], n), dtype=out_dtype or x.dtype, device=x.device)
    need = _lib.lib().l3d_linear_workspace_size(x2.shape[0], n, k)
    ws = _LIN_WS.get(x.device)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
        _LIN_WS[x.device] = ws
    r2 = None if residual is None else residual.reshape(-1, n)
    call("l3d_linear_ex", ref(desc(x2)), ref(desc(weight)), ref(desc(bias)), ACT_CODES[act],
         ref(desc(r2)), ref(desc(gate)), ref(desc(y)), ws.data_ptr(), ws.numel(), _s(x))
    return y.reshape(*x.shape[:-1], n)


# ------------------------------------------------------------------- sparse
def sparse_neighbor_pairs(coords):
    """CoordMap + 27 per-offset neighbour lists (crate/runtime/trellis2_sparse.rs:68-106,
    :211-236): returns (pair_dest [27, N], pair_src [27, N], counts [27]) int32;
    entries beyond counts[k] are unspecified."""
    _check_cuda(coords)
    coords = coords.to(torch.int32)
    n = coords.shape[0]
    dest = torch.empty((27, n), dtype=torch.int32, device=coords.device)
    src = torch.empty_like(dest)
    counts = torch.empty(27, dtype=torch.int32, device=coords.device)
    need = _lib.lib().l3d_sparse_neighbor_pairs_workspace_size(n)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=coords.device)
    call("l3d_sparse_neighbor_pairs", ref(desc(coords)), ref(desc(dest)), ref(desc(src)),
         ref(desc(counts)), ws.data_ptr(), ws.numel(), _s(coords))
    return dest, src, counts


def index_select_rows(feats, ids):
    """index_select_rows (crate/runtime/trellis2_sparse.rs:118-133)."""
    _check_cuda(feats, ids)
    out = torch.empty((ids.shape[0], feats.shape[1]), dtype=feats.dtype, device=feats.device)
    call("l3d_index_select_rows", ref(desc(feats)), ref(desc(ids)), ref(desc(out)), _s(feats))
    return out


def sparse_neighbor_map(coords):
    """[N, 27] int32 neighbour rows (-1 when absent) of a coordinate set, the
    dense form of the CoordMap lookups (crate/runtime/trellis2_sparse.rs:68-106)."""
    _check_cuda(coords)
    coords = coords.to(torch.int32)
    n = coords.shape[0]
    nbr = torch.empty((n, 27), dtype=torch.int32, device=coords.device)
    need = _lib.lib().l3d_sparse_neighbor_pairs_workspace_size(n)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=coords.device)
    call("l3d_sparse_neighbor_map", ref(desc(coords)), ref(desc(nbr)), ws.data_ptr(), ws.numel(),
         _s(coords))
    return nbr


class SparseConv3d:
    """SparseConv3d (crate/runtime/trellis2_sparse.rs:138-243): submanifold
    3x3x3 conv.  `weight` is the checkpoint layout [Cout, 3, 3, 3, Cin] or the
    transposed kernel [27, Cout, Cin]; it is kept on the device as bf16
    [27, Cout, Cin], the tensor-core operand."""

    def __init__(self, weight, bias=None):
        _check_cuda(weight, bias)
        if weight.dim() == 5:
            cout, cin = weight.shape[0], weight.shape[4]
            weight = weight.reshape(cout, 27, cin).permute(1, 0, 2)
        self.weight = weight.to(torch.bfloat16).contiguous()
        self.cout, self.cin = self.weight.shape[1], self.weight.shape[2]
        self.bias = bias
        self._ws = None

    def _workspace(self, need, device):
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        return self._ws

    def __call__(self, feats, pairs=None, coords=None, nbr=None, out_dtype=torch.float32):
        """Per-offset GEMMs over the neighbour pairs (`pairs` = the
        (pair_dest, pair_src, counts) of `sparse_neighbor_pairs`, built from
        `coords` when omitted); with `nbr` (a `sparse_neighbor_map`) instead,
        one implicit GEMM over all 27 offsets of every row, which pays when
        most neighbours exist."""
        _check_cuda(feats, coords, nbr)
        n = feats.shape[0]
        out = torch.empty((n, self.cout), dtype=out_dtype, device=feats.device)
        if nbr is not None:
            need = _lib.lib().l3d_sparse_conv3d_workspace_size(n, self.cin,
                                                               _lib._TORCH_TO_L3D[feats.dtype])
            ws = self._workspace(need, feats.device)
            call("l3d_sparse_conv3d", ref(desc(feats)), ref(desc(nbr)), ref(desc(self.weight)),
                 ref(desc(self.bias)), ref(desc(out)), ws.data_ptr(), ws.numel(), _s(feats))
            return out
        if pairs is None:
            pairs = sparse_neighbor_pairs(coords)
        dest, src, counts = pairs[:3]
        # The 27 counts on the host size the launch; pass them as a fourth
        # element of `pairs` to avoid reading them back on every call.
        counts_host = pairs[3] if len(pairs) > 3 else counts.cpu().numpy()
        counts_host = np.ascontiguousarray(counts_host, dtype=np.int32)
        chp = counts_host.ctypes.data
        need = _lib.lib().l3d_sparse_conv3d_pairs_workspace_size(n, self.cin, self.cout, chp)
        ws = self._workspace(need, feats.device)
        call("l3d_sparse_conv3d_pairs", ref(desc(feats)), ref(desc(src)), ref(desc(dest)),
             ref(desc(counts)), chp, ref(desc(self.weight)), ref(desc(self.bias)),
             ref(desc(out)), ws.data_ptr(), ws.numel(), _s(feats))
        return out


def activation_scatter(x, outs, act="gelu_tanh"):
    """act(x) stored to every output in one pass (l3d_activation_scatter):
    `outs` are (device pointer, element offset) pairs of contiguous buffers
    with x's dtype and element count, on this GPU or another GPU's memory
    mapped here (shard.PeerRows.dest) - the last op of a block fused with the
    final all-gather of the block outputs."""
    _check_cuda(x)
    arr = (_lib.L3dTensor * len(outs))()
    for d, (ptr, off) in zip(arr, outs):
        d.data = ptr
        d.dtype = _lib._TORCH_TO_L3D[x.dtype]
        d.ndim = 1
        d.dims[0] = x.numel()
        d.strides[0] = 1
        d.offset = off
    call("l3d_activation_scatter", ACT[act], ref(desc(x)), arr, len(outs), _s(x))


# Status-word workspaces of l3d_attention, one per (device, stream): calls on
# different streams then never clear or overwrite each other's status.
_ATTN_WS = {}
# Read the status word back after every attention call (synchronises the
# stream) and raise on a kernel-reported error; also on with L3D_CHECK_STATUS=1.
CHECK_STATUS = os.environ.get("L3D_CHECK_STATUS", "0") == "1"


def attention_workspace(device, stream=None):
    """The status-word workspace ops.attention uses on (device, stream)."""
    st = torch.cuda.current_stream(device) if stream is None else stream
    return _ATTN_WS.get((torch.device(device), st.cuda_stream))


def attention(q, k, v, scale=None, out=None, check=None):
    """exact_sdpa_heads (crate/runtime/attention_math.rs:199-259): softmax(q k^T
    * scale) v on [B, H, N, D] bf16 views (D = 64 or 128), tcgen05 flash
    attention.  `out` defaults to token-major [B, N, H, D] memory viewed as
    [B, H, N, D], so out.transpose(1, 2).reshape(B, N, H * D) is a view.
    With `check` (default CHECK_STATUS) the stream is synchronised and a
    non-zero status word (a bounded wait in the kernel ran out) raises
    L3dError(L3D_E_DEVICE)."""
    _check_cuda(q, k, v, out)
    B, H, N, D = q.shape
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty((B, N, H, D), dtype=q.dtype, device=q.device).transpose(1, 2)
    need = _lib.lib().l3d_attention_workspace_size(B, H, k.shape[2], D)
    stream = torch.cuda.current_stream(q.device)
    key = (q.device, stream.cuda_stream)
    ws = _ATTN_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
        _ATTN_WS[key] = ws
    call("l3d_attention", ref(desc(q)), ref(desc(k)), ref(desc(v)), float(scale), ref(desc(out)),
         ws.data_ptr(), ws.numel(), stream.cuda_stream)
    if CHECK_STATUS if check is None else check:
        stream.synchronize()
        st = int(ws[:4].view(torch.int32).item())
        if st != 0:
            raise _lib.L3dError(8, "l3d_attention", f"kernel status word {st} (bounded wait expired)")
    return out
