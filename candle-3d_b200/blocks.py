"""Block stacks of the three model families, assembled from the fused layer ops.

Each stack follows the reference block's op order exactly; between the GEMMs
(cuBLAS through torch, or the tcgen05 dequant-linear for GGML weights) and the
attention (torch SDPA by default; `set_attention("l3d")` routes the bf16
attention cores to this package's tcgen05 kernel, `ops.attention`) every
per-token op runs as one of this package's fused kernels, and every residual
add is fused with the norm that follows it:

  * VGGT aggregator (crate/runtime/vggt.rs:113-186,264-313): frame / global
    alternating blocks; LN -> qkv -> per-head LN + 2D RoPE (q and k, one launch)
    -> SDPA -> proj -> LayerScale residual + norm2 (one kernel) -> fc1 +
    GELU-erf (one tcgen05 GEMM at >= 8192 rows) -> fc2 -> LayerScale residual +
    next block's norm1 (one kernel).
  * TripoSG DiT (crate/runtime/triposg_dit.rs:217-276,346-506): sin-first
    timestep token, UViT long skips, RMSNorm-heads on the diffusers q/k/v
    split, bf16 flash cross attention, exact-GELU FFN.
  * TRELLIS.2 SLAT (crate/runtime/trellis2_blocks.rs:609-646,
    crate/runtime/trellis2_dit.rs:549-574): shared adaLN, modulated norms,
    L2-norm * gamma + 3D RoPE on integer voxel coordinates, Q8_0 weights through
    the dequant-linear, tanh-GELU FFN (the GELU runs in mlp.0's GEMM epilogue).

Weights are random (~N(0, 0.02)); there is no checkpoint loader here.
`*_reference` functions restate each block in plain torch f32 (used by the
parity tests at small sizes).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import ops

_ATTENTION = "sdpa"
# Rows from which the VGGT MLP's fc1 + GELU-erf runs as one tcgen05 GEMM with
# the activation in its epilogue (measured 94.6 vs 99.8 us for cuBLAS + the
# GELU kernel at 10,992 rows x 1024 -> 4096; slower below about 5,000 rows,
# where its 128-row tiles leave most SMs idle).
FUSED_MLP_MIN_ROWS = 8192


def set_attention(impl: str) -> None:
    """Selects the attention core of the stacks' bf16 attention: "sdpa" (torch
    scaled_dot_product_attention, cuDNN) or "l3d" (l3d_attention)."""
    global _ATTENTION
    if impl not in ("sdpa", "l3d"):
        raise ValueError(f"unknown attention implementation {impl!r}")
    _ATTENTION = impl


def _attend(q, k, v):
    """exact_sdpa_heads (crate/runtime/attention_math.rs:199-259) on [B, H, N, D]
    views, by the implementation set_attention selected."""
    if _ATTENTION == "l3d":
        return ops.attention(q, k, v)
    return F.scaled_dot_product_attention(q, k, v)


def _w(g, shape, std=0.02, dev=None, dtype=torch.bfloat16):
    return (std * torch.randn(shape, generator=g)).to(dev, dtype)


def _ln_params(g, C, dev, dtype):
    return ((1 + 0.02 * torch.randn(C, generator=g)).to(dev, dtype),
            (0.02 * torch.randn(C, generator=g)).to(dev, dtype))


# =============================================================== VGGT
class VggtAggregator:
    """24 frame + 24 global VGGT blocks (dim 1024, 16 heads of 64, MLP 4096,
    LayerScale init 0.01, LN eps 1e-5, RoPE theta 100)."""

    def __init__(self, depth=24, C=1024, H=16, mlp=4096, device="cuda", dtype=torch.bfloat16,
                 seed=20261201, ls_init=0.01):
        g = torch.Generator().manual_seed(seed)
        self.C, self.H, self.D, self.depth, self.dtype = C, H, C // H, depth, dtype
        self.blocks = []
        for _ in range(2 * depth):  # frame_blocks[r], global_blocks[r] interleaved
            p = {}
            p["n1w"], p["n1b"] = _ln_params(g, C, device, dtype)
            p["qkv_w"], p["qkv_b"] = _w(g, (3 * C, C), dev=device, dtype=dtype), _w(g, 3 * C, dev=device, dtype=dtype)
            p["qnw"], p["qnb"] = _ln_params(g, self.D, device, dtype)
            p["knw"], p["knb"] = _ln_params(g, self.D, device, dtype)
            p["proj_w"], p["proj_b"] = _w(g, (C, C), dev=device, dtype=dtype), _w(g, C, dev=device, dtype=dtype)
            p["ls1"] = torch.full((C,), ls_init, device=device, dtype=dtype)
            p["n2w"], p["n2b"] = _ln_params(g, C, device, dtype)
            p["fc1_w"], p["fc1_b"] = _w(g, (mlp, C), dev=device, dtype=dtype), _w(g, mlp, dev=device, dtype=dtype)
            p["fc2_w"], p["fc2_b"] = _w(g, (C, mlp), dev=device, dtype=dtype), _w(g, C, dev=device, dtype=dtype)
            p["ls2"] = torch.full((C,), ls_init, device=device, dtype=dtype)
            self.blocks.append(p)

    @staticmethod
    def positions(B, S, ph, pw, special, device):
        """crate/runtime/vggt.rs:288-291: 0 for special tokens, (y+1, x+1) for patches."""
        grid = ops.position_getter(B * S, ph, pw, device)
        zeros = torch.zeros((B * S, special, 2), dtype=torch.int64, device=device)
        return torch.cat([zeros, grid], 1).to(torch.int32)

    def _attn(self, p, y, pos):
        B, N, C = y.shape
        H, D = self.H, self.D
        qkv = F.linear(y, p["qkv_w"], p["qkv_b"]).view(B, N, 3, H, D).permute(2, 0, 3, 1, 4)
        # q / k written token-major ([B, N, H, D] memory seen as [B, H, N, D]),
        # the layout the attention kernel keeps for its output, so the
        # output's transpose-reshape below is a view, not a copy.
        qk = torch.empty(2, B, N, H, D, dtype=y.dtype, device=y.device).permute(0, 1, 3, 2, 4)
        q, k = ops.qk_layernorm_rope2d(qkv[0], qkv[1], p["qnw"], p["qnb"], p["knw"], p["knb"],
                                       1e-5, pos, 100.0, q_out=qk[0], k_out=qk[1])
        a = _attend(q, k, qkv[2])
        return F.linear(a.transpose(1, 2).reshape(B, N, C), p["proj_w"], p["proj_b"])

    def _attn_split(self, p, y, pos, split):
        """Global attention of one scene whose token slabs live on the ranks of
        `split` (shard.SceneSplit): y [1, L, C] and pos [1, L, 2] are this
        rank's slab.  q/k are normed and rotated on the local tokens straight
        into the head-group-major send buffer, exchanged head-parallel,
        attended over all tokens, and the outputs sent back to their owners."""
        _, L, C = y.shape
        H, D, world = self.H, self.D, split.world
        h = H // world
        qkv = F.linear(y, p["qkv_w"], p["qkv_b"]).view(L, 3, world, h, D)
        send = torch.empty(world, L, 3, h, D, dtype=y.dtype, device=y.device)
        # [world, h, L, D] views: head j * h + i of the layer is head i of group j;
        # the positions are shared by the groups (batch stride 0).
        qin, kin = (qkv[:, i].permute(1, 2, 0, 3) for i in range(2))
        qo, ko = (send[:, :, i].permute(0, 2, 1, 3) for i in range(2))
        ops.qk_layernorm_rope2d(qin, kin, p["qnw"], p["qnb"], p["knw"], p["knb"], 1e-5,
                                pos.expand(world, L, 2), 100.0, q_out=qo, k_out=ko)
        send[:, :, 2].copy_(qkv[:, 2].transpose(0, 1))
        q, k, v = split.exchange_qkv(send)
        if _ATTENTION == "l3d":
            a = torch.empty(world * L, h, D, dtype=y.dtype, device=y.device)
            ops.attention(q, k, v, out=a.permute(1, 0, 2).unsqueeze(0))
        else:
            a = F.scaled_dot_product_attention(q, k, v)[0].transpose(0, 1).contiguous()
        o = split.return_heads(a)
        return F.linear(o.view(1, L, C), p["proj_w"], p["proj_b"])

    def forward(self, tokens, frame_pos, global_pos, S, split=None):
        """tokens [B*S, N, C] -> final tokens [B*S, N, C] (residual stream updated in place).

        With `split` (shard.SceneSplit over W ranks, B = 1) the arguments are
        this rank's S views of a W * S-view scene (its frame positions and its
        slab of the global positions): frame blocks run locally and global
        blocks exchange q/k/v head-parallel across the ranks."""
        BS, N, C = tokens.shape
        B = BS // S
        if split is not None and split.world > 1:
            if B != 1 or self.H % split.world:
                raise ValueError("a split scene needs B = 1 and heads divisible by the ranks")
        else:
            split = None
        x = tokens.contiguous()
        y = ops.layer_norm(x, self.blocks[0]["n1w"], self.blocks[0]["n1b"], 1e-5)
        nb = len(self.blocks)
        for i, p in enumerate(self.blocks):
            is_global = i % 2 == 1
            shape = (B, S * N, C) if is_global else (BS, N, C)
            xv, yv = x.view(shape), y.view(shape)
            if is_global and split is not None:
                o = self._attn_split(p, yv, global_pos, split)
            else:
                o = self._attn(p, yv, global_pos if is_global else frame_pos)
            _, y2 = ops.residual_layer_norm_modulate(xv, o, gate=p["ls1"], weight=p["n2w"],
                                                     bias=p["n2b"], eps=1e-5, inplace=True)
            if y2.numel() // C >= FUSED_MLP_MIN_ROWS:
                # fc1 with GELU-erf in the tcgen05 GEMM epilogue (l3d_linear_ex)
                h = ops.linear(y2, p["fc1_w"], p["fc1_b"], act="gelu_erf")
            else:
                h = ops.gelu_erf(F.linear(y2, p["fc1_w"], p["fc1_b"]))
            m = F.linear(h, p["fc2_w"], p["fc2_b"])
            if i + 1 < nb:
                nxt = self.blocks[i + 1]
                _, y = ops.residual_layer_norm_modulate(xv, m, gate=p["ls2"], weight=nxt["n1w"],
                                                        bias=nxt["n1b"], eps=1e-5, inplace=True)
                y = y.view(BS, N, C)
            else:
                ops.residual_layer_norm_modulate(xv, m, gate=p["ls2"], eps=1e-5, inplace=True)
        return x


def rope2d_reference(t, pos, theta=100.0):
    """rope_apply (crate/runtime/attention_math.rs:104-118) in torch f32; t [B,H,N,D], pos [B,N,2]."""
    D = t.shape[-1]
    half, quarter = D // 2, D // 4
    inv = 1.0 / theta ** (torch.arange(quarter, device=t.device, dtype=torch.float32) * 2 / half)
    out = torch.empty_like(t)
    for hf in range(2):
        ang = pos[:, None, :, hf, None].float() * inv
        c, s = torch.cos(ang), torch.sin(ang)
        a = t[..., hf * half:hf * half + quarter]
        b = t[..., hf * half + quarter:(hf + 1) * half]
        out[..., hf * half:hf * half + quarter] = a * c - b * s
        out[..., hf * half + quarter:(hf + 1) * half] = b * c + a * s
    return out


def vggt_reference(agg: VggtAggregator, tokens, frame_pos, global_pos, S):
    """VggtBlock::forward x 2*depth in torch f32 (crate/runtime/vggt.rs:113-186)."""
    f = lambda t: t.float()  # noqa: E731
    BS, N, C = tokens.shape
    B = BS // S
    H, D = agg.H, agg.D
    x = tokens.float()
    for i, p in enumerate(agg.blocks):
        is_global = i % 2 == 1
        xv = x.view(B, S * N, C) if is_global else x.view(BS, N, C)
        pos = global_pos if is_global else frame_pos
        y = F.layer_norm(xv, (C,), f(p["n1w"]), f(p["n1b"]), 1e-5)
        qkv = F.linear(y, f(p["qkv_w"]), f(p["qkv_b"])).view(*y.shape[:2], 3, H, D).permute(2, 0, 3, 1, 4)
        q = rope2d_reference(F.layer_norm(qkv[0], (D,), f(p["qnw"]), f(p["qnb"]), 1e-5), pos)
        k = rope2d_reference(F.layer_norm(qkv[1], (D,), f(p["knw"]), f(p["knb"]), 1e-5), pos)
        a = F.scaled_dot_product_attention(q, k, qkv[2])
        o = F.linear(a.transpose(1, 2).reshape(y.shape), f(p["proj_w"]), f(p["proj_b"]))
        xv = xv + f(p["ls1"]) * o
        y2 = F.layer_norm(xv, (C,), f(p["n2w"]), f(p["n2b"]), 1e-5)
        m = F.linear(F.gelu(F.linear(y2, f(p["fc1_w"]), f(p["fc1_b"]))), f(p["fc2_w"]), f(p["fc2_b"]))
        x = (xv + f(p["ls2"]) * m).reshape(BS, N, C)
    return x


# ============================================================= TripoSG
class TripoSgDit:
    """TripoSG rectified-flow DiT: 21 blocks, width 2048, 16 heads of 128, FFN
    8192, cross attention to [B, S, 1024] encoder tokens, UViT long skips."""

    def __init__(self, layers=21, C=2048, H=16, ff=8192, cond_dim=1024, in_ch=64, device="cuda",
                 dtype=torch.bfloat16, seed=20261202):
        g = torch.Generator().manual_seed(seed)
        self.C, self.H, self.D, self.layers, self.dtype = C, H, C // H, layers, dtype
        dev = device
        self.proj_in = (_w(g, (C, in_ch), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype))
        # time_proj: Linear(width, 4 width) -> GELU-erf -> Linear(4 width, width)
        # (time_embed_dim, crate/runtime/triposg_dit.rs:156-160).
        self.t1 = (_w(g, (4 * C, C), dev=dev, dtype=dtype), _w(g, 4 * C, dev=dev, dtype=dtype))
        self.t2 = (_w(g, (C, 4 * C), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype))
        self.norm_out = _ln_params(g, C, dev, dtype)
        self.proj_out = (_w(g, (in_ch, C), dev=dev, dtype=dtype), _w(g, in_ch, dev=dev, dtype=dtype))
        self.blocks = []
        mid = layers // 2
        for i in range(layers):
            p = {}
            if i > mid:
                p["skip_w"], p["skip_b"] = _w(g, (C, 2 * C), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype)
                p["skn_w"], p["skn_b"] = _ln_params(g, C, dev, dtype)
            for n in ("n1", "n2", "n3"):
                p[n + "w"], p[n + "b"] = _ln_params(g, C, dev, dtype)
            p["qkv1_w"] = _w(g, (3 * C, C), dev=dev, dtype=dtype)  # cat([to_q, to_k, to_v])
            p["o1_w"], p["o1_b"] = _w(g, (C, C), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype)
            p["nq1"], p["nk1"] = (1 + 0.05 * torch.randn(self.D, generator=g)).to(dev, dtype), \
                (1 + 0.05 * torch.randn(self.D, generator=g)).to(dev, dtype)
            p["q2_w"] = _w(g, (C, C), dev=dev, dtype=dtype)
            p["kv2_w"] = _w(g, (2 * C, cond_dim), dev=dev, dtype=dtype)  # cat([to_k, to_v])
            p["o2_w"], p["o2_b"] = _w(g, (C, C), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype)
            p["nq2"], p["nk2"] = (1 + 0.05 * torch.randn(self.D, generator=g)).to(dev, dtype), \
                (1 + 0.05 * torch.randn(self.D, generator=g)).to(dev, dtype)
            p["ff1_w"], p["ff1_b"] = _w(g, (ff, C), dev=dev, dtype=dtype), _w(g, ff, dev=dev, dtype=dtype)
            p["ff2_w"], p["ff2_b"] = _w(g, (C, ff), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype)
            self.blocks.append(p)

    def _self_attn(self, p, y):
        B, L, C = y.shape
        H, D = self.H, self.D
        # cat([q, k, v]).reshape(B, L, H, 3D).chunk(3) (crate/runtime/triposg_dit.rs:436-454)
        qkv = F.linear(y, p["qkv1_w"]).view(B, L, H, 3 * D)
        q = ops.rms_norm_heads(qkv[..., :D].transpose(1, 2), p["nq1"], 1e-6)
        k = ops.rms_norm_heads(qkv[..., D:2 * D].transpose(1, 2), p["nk1"], 1e-6)
        v = qkv[..., 2 * D:].transpose(1, 2)
        a = _attend(q, k, v)
        return F.linear(a.transpose(1, 2).reshape(B, L, C), p["o1_w"], p["o1_b"])

    def _self_attn_split(self, p, y, split, counts):
        """Self-attention over one batch element's whole token sequence when
        its tokens are split across the ranks of `split` (shard.SceneSplit;
        rank r owns counts[r] consecutive tokens, y [1, L, C]): the RMS-normed
        q / k and v are written head-group-major into the send buffer,
        exchanged head-parallel, attended over all tokens and sent back."""
        _, L, C = y.shape
        H, D, world = self.H, self.D, split.world
        h = H // world
        qkv = F.linear(y, p["qkv1_w"]).view(L, world, h, 3 * D)
        send = torch.empty(world, L, 3, h, D, dtype=y.dtype, device=y.device)
        ops.rms_norm_heads(qkv[..., :D], p["nq1"], 1e-6, out=send[:, :, 0].transpose(0, 1))
        ops.rms_norm_heads(qkv[..., D:2 * D], p["nk1"], 1e-6, out=send[:, :, 1].transpose(0, 1))
        send[:, :, 2].copy_(qkv[..., 2 * D:].transpose(0, 1))
        q, k, v = split.exchange_qkv_uneven(send, counts)
        total = int(sum(counts))
        if _ATTENTION == "l3d":
            a = torch.empty(total, h, D, dtype=y.dtype, device=y.device)
            ops.attention(q, k, v, out=a.permute(1, 0, 2).unsqueeze(0))
        else:
            a = F.scaled_dot_product_attention(q, k, v)[0].transpose(0, 1).contiguous()
        o = split.return_heads_uneven(a, counts)
        return F.linear(o.view(1, L, C), p["o1_w"], p["o1_b"])

    def _cross_attn(self, p, y, cond):
        B, L, C = y.shape
        H, D = self.H, self.D
        q = ops.rms_norm_heads(F.linear(y, p["q2_w"]).view(B, L, H, D).transpose(1, 2), p["nq2"], 1e-6)
        kv = F.linear(cond, p["kv2_w"]).view(B, cond.shape[1], H, 2 * D)
        k = ops.rms_norm_heads(kv[..., :D].transpose(1, 2), p["nk2"], 1e-6)
        v = kv[..., D:].transpose(1, 2)
        # bf16 operands with f32 softmax / accumulation inside the flash kernel,
        # as for the self attention (the stack parity tests bound the result).
        a = _attend(q, k, v)
        return F.linear(a.transpose(1, 2).reshape(B, L, C), p["o2_w"], p["o2_b"])

    def timestep_token(self, t, B):
        temb = ops.timestep_embedding(t.reshape(1), self.C, "sin_first", dtype=self.dtype)
        h = ops.linear_small(temb, self.t1[0], self.t1[1], act_out="gelu_erf")
        h = ops.linear_small(h, self.t2[0], self.t2[1])
        return h.view(1, 1, self.C).expand(B, 1, self.C)

    def forward(self, latents, t, cond, split=None, counts=None, prefix=True):
        """latents [B, L, 64], cond [B, S, 1024] -> [B, L, 64].

        With `split` (shard.SceneSplit over W ranks, 16 heads divisible by W)
        and `counts` (tokens per rank of the 1 + L token sequence, the
        timestep token first), latents [1, l, 64] are this rank's latent rows
        of one batch element, cond that element's encoder tokens, `prefix`
        whether this rank's slab starts with the timestep token, and the
        result is those rows' output [1, l, 64]: every op is per token except
        the self-attention, which exchanges q/k/v head-parallel (the cross
        attention reads all of cond on every rank)."""
        B, L, _ = latents.shape
        C = self.C
        if split is not None and split.world > 1:
            if (B != 1 or self.H % split.world or counts is None
                    or int(counts[split.rank]) != L + int(prefix)):
                raise ValueError("a split needs one batch element, heads divisible by the ranks "
                                 "and this rank's token count")
        else:
            split, prefix = None, True
        x = F.linear(latents, *self.proj_in)
        if prefix:
            x = torch.cat([self.timestep_token(t, B), x], 1)
        x = x.contiguous()
        mid = self.layers // 2
        skips = []
        y = None  # norm1 output of the current block when fused upstream
        for i, p in enumerate(self.blocks):
            if i > mid:
                s = skips.pop()
                x = ops.layer_norm(F.linear(torch.cat([s, x], -1), p["skip_w"], p["skip_b"]),
                                   p["skn_w"], p["skn_b"], 1e-5)
                y = None
            if y is None:
                y = ops.layer_norm(x, p["n1w"], p["n1b"], 1e-5)
            a = self._self_attn(p, y) if split is None else self._self_attn_split(p, y, split, counts)
            x, y = ops.residual_layer_norm_modulate(x, a, weight=p["n2w"], bias=p["n2b"], eps=1e-5)
            x, y = ops.residual_layer_norm_modulate(x, self._cross_attn(p, y, cond),
                                                    weight=p["n3w"], bias=p["n3b"], eps=1e-5)
            ff = F.linear(ops.gelu_erf(F.linear(y, p["ff1_w"], p["ff1_b"])), p["ff2_w"], p["ff2_b"])
            nxt = self.blocks[i + 1] if i + 1 < self.layers else None
            if nxt is None:
                x, y = ops.residual_layer_norm_modulate(x, ff, weight=self.norm_out[0],
                                                        bias=self.norm_out[1], eps=1e-5)
            elif i + 1 <= mid:
                x, y = ops.residual_layer_norm_modulate(x, ff, weight=nxt["n1w"], bias=nxt["n1b"],
                                                        eps=1e-5)
            else:  # the next block first merges its long skip
                x, y = ops.gated_residual(x, ff), None
            if i < mid:
                skips.append(x)
        # norm_out over all tokens (y holds it after the last block), slice, proj_out.
        return F.linear(y[:, -L:], *self.proj_out)


def triposg_reference(m: TripoSgDit, latents, t, cond):
    """TripoSgDiT::forward (crate/runtime/triposg_dit.rs:217-276) in torch f32."""
    f = lambda a: a.float()  # noqa: E731
    B, L, _ = latents.shape
    C, H, D = m.C, m.H, m.D
    half = C // 2
    freq = torch.exp(-math.log(10000.0) * torch.arange(half, device=latents.device) / half)
    arg = (t.float().reshape(1) * freq).to(m.dtype).float()
    temb = torch.cat([torch.sin(arg), torch.cos(arg)]).view(1, C)
    h = F.linear(F.gelu(F.linear(temb, f(m.t1[0]), f(m.t1[1]))), f(m.t2[0]), f(m.t2[1]))
    x = torch.cat([h.view(1, 1, C).expand(B, 1, C), F.linear(f(latents), f(m.proj_in[0]), f(m.proj_in[1]))], 1)

    def rms(v, w):
        return v / torch.sqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6) * f(w)

    mid = m.layers // 2
    skips = []
    for i, p in enumerate(m.blocks):
        if i > mid:
            x = F.layer_norm(F.linear(torch.cat([skips.pop(), x], -1), f(p["skip_w"]), f(p["skip_b"])),
                             (C,), f(p["skn_w"]), f(p["skn_b"]), 1e-5)
        y = F.layer_norm(x, (C,), f(p["n1w"]), f(p["n1b"]), 1e-5)
        qkv = F.linear(y, f(p["qkv1_w"])).view(B, -1, H, 3 * D)
        q = rms(qkv[..., :D].transpose(1, 2), p["nq1"])
        k = rms(qkv[..., D:2 * D].transpose(1, 2), p["nk1"])
        a = F.scaled_dot_product_attention(q, k, qkv[..., 2 * D:].transpose(1, 2))
        x = x + F.linear(a.transpose(1, 2).reshape(B, -1, C), f(p["o1_w"]), f(p["o1_b"]))
        y = F.layer_norm(x, (C,), f(p["n2w"]), f(p["n2b"]), 1e-5)
        q = rms(F.linear(y, f(p["q2_w"])).view(B, -1, H, D).transpose(1, 2), p["nq2"])
        kv = F.linear(f(cond), f(p["kv2_w"])).view(B, cond.shape[1], H, 2 * D)
        k = rms(kv[..., :D].transpose(1, 2), p["nk2"])
        a = F.scaled_dot_product_attention(q, k, kv[..., D:].transpose(1, 2))
        x = x + F.linear(a.transpose(1, 2).reshape(B, -1, C), f(p["o2_w"]), f(p["o2_b"]))
        y = F.layer_norm(x, (C,), f(p["n3w"]), f(p["n3b"]), 1e-5)
        x = x + F.linear(F.gelu(F.linear(y, f(p["ff1_w"]), f(p["ff1_b"]))), f(p["ff2_w"]), f(p["ff2_b"]))
        if i < mid:
            skips.append(x)
    y = F.layer_norm(x, (C,), f(m.norm_out[0]), f(m.norm_out[1]), 1e-5)
    return F.linear(y[:, -L:], f(m.proj_out[0]), f(m.proj_out[1]))


# ============================================================ TRELLIS.2
def _q8_linear(g, n, k, dev, scale_lo=0.001, scale_hi=0.02):
    """Int8 per-output-channel symmetric weight (scales ~ U(lo, hi)) encoded as
    GGML Q8_0 blocks on the device, plus its f32 bias."""
    s = torch.empty(n, 1).uniform_(scale_lo, scale_hi, generator=g)
    q = torch.clamp(torch.round(torch.randn(n, k, generator=g) * 40), -127, 127)
    w = (q * s).float()
    blocks = quantize_q8_0_torch(w)
    b = (0.02 * torch.randn(n, generator=g)).float()
    return ops.QMatMul(blocks.to(dev), "q8_0", n, k, bias=b.to(dev))


KQ_BLOCK_BYTES = {"q4_k": 144, "q5_k": 176, "q6_k": 210}


def _kq_linear(g, fmt, n, k, dev):
    """Synthetic GGML K-quant weight ([n, k], k % 256 == 0): random quant bits
    and 6-bit scales / mins (Q6_K int8 scales in [-16, 16]), f16 super-block
    scales ~ U(1e-4, 1e-3); plus its f32 bias."""
    nsb = n * (k // 256)
    bb = KQ_BLOCK_BYTES[fmt]
    blk = torch.randint(0, 256, (nsb, bb), generator=g, dtype=torch.int32).to(torch.uint8)
    d = torch.empty(nsb).uniform_(1e-4, 1e-3, generator=g).to(torch.float16).view(torch.uint8)
    d = d.reshape(nsb, 2)
    if fmt == "q6_k":
        sc = torch.randint(-16, 17, (nsb, 16), generator=g, dtype=torch.int32).to(torch.int8)
        blk[:, 192:208] = sc.view(torch.uint8)
        blk[:, 208:210] = d
    else:
        dm = torch.empty(nsb).uniform_(1e-4, 1e-3, generator=g).to(torch.float16)
        blk[:, 0:2] = d
        blk[:, 2:4] = dm.view(torch.uint8).reshape(nsb, 2)
    b = (0.02 * torch.randn(n, generator=g)).float()
    return ops.QMatMul(blk.reshape(-1).contiguous().to(dev), fmt, n, k, bias=b.to(dev))


def quantize_q8_0_torch(w: torch.Tensor) -> torch.Tensor:
    """GGML quantize_row_q8_0 (d = amax / 127, q = round(w / d)) on the host."""
    n, k = w.shape
    blk = w.reshape(n, k // 32, 32)
    d = blk.abs().amax(-1, keepdim=True) / 127.0
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.round(blk * inv).to(torch.int8)
    dh = d.to(torch.float16).view(torch.uint8).reshape(n, k // 32, 2)
    return torch.cat([dh, q.view(torch.uint8)], -1).reshape(-1).contiguous()


class Trellis2Slat:
    """TRELLIS.2 sparse SLAT flow transformer on N voxel tokens: width 1536, 12
    heads of 128, MLP 8192 (tanh GELU), cross attention to [1, Lc, 1024],
    shared adaLN, Q8_0 weights for every block linear."""

    def __init__(self, blocks=24, C=1536, H=12, mlp=8192, cond_dim=1024, in_ch=32, device="cuda",
                 dtype=torch.bfloat16, seed=20261203):
        g = torch.Generator().manual_seed(seed)
        self.C, self.H, self.D, self.dtype = C, H, C // H, dtype
        dev = device
        self.input_layer = (_w(g, (C, in_ch), dev=dev, dtype=dtype), _w(g, C, dev=dev, dtype=dtype))
        self.t_fc1 = (_w(g, (C, 256), dev=dev), _w(g, C, dev=dev))
        self.t_fc2 = (_w(g, (C, C), dev=dev), _w(g, C, dev=dev))
        self.ada = (_w(g, (6 * C, C), dev=dev), _w(g, 6 * C, dev=dev))
        self.out_layer = (_w(g, (in_ch, C), dev=dev, dtype=dtype), _w(g, in_ch, dev=dev, dtype=dtype))
        self.blocks = []
        for _ in range(blocks):
            p = {"modulation": (0.1 * torch.randn(6 * C, generator=g)).to(dev, dtype)}
            p["to_qkv"] = _q8_linear(g, 3 * C, C, dev)
            p["to_out"] = _q8_linear(g, C, C, dev)
            p["qg"] = (1 + 0.05 * torch.randn(H, self.D, generator=g)).to(dev)
            p["kg"] = (1 + 0.05 * torch.randn(H, self.D, generator=g)).to(dev)
            p["n2w"], p["n2b"] = _ln_params(g, C, dev, dtype)
            p["c_q"] = _q8_linear(g, C, C, dev)
            p["c_kv"] = _q8_linear(g, 2 * C, cond_dim, dev)
            p["c_out"] = _q8_linear(g, C, C, dev)
            p["cqg"] = (1 + 0.05 * torch.randn(H, self.D, generator=g)).to(dev)
            p["ckg"] = (1 + 0.05 * torch.randn(H, self.D, generator=g)).to(dev)
            p["mlp0"] = _q8_linear(g, mlp, C, dev)
            p["mlp2"] = _q8_linear(g, C, mlp, dev)
            self.blocks.append(p)

    def t_emb(self, t_model):
        """Trellis2TimestepEmbedder + shared adaLN (trellis2_blocks.rs:209-258)."""
        tab = ops.timestep_embedding(t_model.reshape(1), 256, "cos_first", dtype=self.dtype)
        h = ops.linear_small(tab, *self.t_fc1, act_out="silu")
        h = ops.linear_small(h, *self.t_fc2)
        return ops.linear_small(h, *self.ada, act_in="silu")  # [1, 6C]

    def block_mods(self, temb):
        """(modulation + t_emb).chunk(6) per block (trellis2_blocks.rs:617-625)."""
        return [ops.chunk_modulation((p["modulation"].unsqueeze(0) + temb).contiguous())
                for p in self.blocks]

    def _self_attn_split(self, p, y, coords, split, counts, groups):
        """Self-attention over all voxels when the voxel rows are split across
        the ranks of `split` (shard.SceneSplit; rank r owns counts[r]
        consecutive rows of the sorted voxel list, y [1, L, C], coords [L, 3]):
        q / k are normed and rotated on the local rows per head group straight
        into the head-group-major send buffer, exchanged head-parallel (uneven
        slabs; with `groups` < world head groups each group is shared by
        world / groups ranks, which split its queries), attended over all
        voxels and sent back to their owners."""
        _, L, C = y.shape
        H, D = self.H, self.D
        h = H // groups
        qkv = p["to_qkv"](y).view(1, L, 3, H, D)
        send = torch.empty(groups, L, 3, h, D, dtype=y.dtype, device=y.device)
        for j in range(groups):
            hs = slice(j * h, (j + 1) * h)
            ops.qk_l2norm_rope3d(qkv[:, :, 0, hs], p["qg"][hs], coords, out=send[j:j + 1, :, 0])
            ops.qk_l2norm_rope3d(qkv[:, :, 1, hs], p["kg"][hs], coords, out=send[j:j + 1, :, 1])
        send[:, :, 2].copy_(qkv[0, :, 2].view(L, groups, h, D).transpose(0, 1))
        q, k, v = split.exchange_qkv_uneven(send, counts, groups)
        if _ATTENTION == "l3d":
            a = torch.empty(q.shape[2], h, D, dtype=y.dtype, device=y.device)
            ops.attention(q, k, v, out=a.permute(1, 0, 2).unsqueeze(0))
        else:
            a = F.scaled_dot_product_attention(q, k, v)[0].transpose(0, 1).contiguous()
        o = split.return_heads_uneven(a, counts, groups)
        return p["to_out"](o.view(1, L, C))

    def forward(self, feats, coords, t_model, cond, split=None, counts=None, head_groups=None):
        """feats [N, in_ch], coords [N, 3] int32, cond [1, Lc, cond_dim] -> [N, in_ch].

        With `split` (shard.SceneSplit over W ranks) and `counts` (rows per
        rank), feats / coords are this rank's consecutive rows of the sorted
        voxel list and the result is those rows' output: every op is per voxel
        except the self-attention, which exchanges q/k/v head-parallel across
        the ranks in `head_groups` groups (default gcd(12, W); each group is
        shared by W / head_groups ranks, which split its queries)."""
        N = feats.shape[0]
        C, H, D = self.C, self.H, self.D
        if split is not None and split.world > 1:
            G = math.gcd(H, split.world) if head_groups is None else int(head_groups)
            if (H % G or split.world % G or counts is None
                    or int(counts[split.rank]) != N):
                raise ValueError("a split needs head groups dividing the heads and the ranks, "
                                 "and this rank's count")
        else:
            split = None
        x = F.linear(feats, *self.input_layer).view(1, N, C).contiguous()
        mods = self.block_mods(self.t_emb(t_model))
        y = ops.layer_norm_modulate(x, mods[0][0], mods[0][1], eps=1e-6)
        Lc = cond.shape[1]
        for i, p in enumerate(self.blocks):
            sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = mods[i]
            if split is not None:
                o = self._self_attn_split(p, y, coords, split, counts, G)
            else:
                qkv = p["to_qkv"](y).view(1, N, 3, H, D)
                q = ops.qk_l2norm_rope3d(qkv[:, :, 0], p["qg"], coords)
                k = ops.qk_l2norm_rope3d(qkv[:, :, 1], p["kg"], coords)
                a = _attend(q.transpose(1, 2), k.transpose(1, 2), qkv[:, :, 2].transpose(1, 2))
                o = p["to_out"](a.transpose(1, 2).reshape(1, N, C))
            x, y = ops.residual_layer_norm_modulate(x, o, gate=g_msa, weight=p["n2w"], bias=p["n2b"],
                                                    eps=1e-6, inplace=True)
            cq = ops.qk_l2norm_rope3d(p["c_q"](y).view(1, N, H, D), p["cqg"], None)
            kv = p["c_kv"](cond).view(1, Lc, 2, H, D)
            ck = ops.qk_l2norm_rope3d(kv[:, :, 0], p["ckg"], None)
            ca = _attend(cq.transpose(1, 2), ck.transpose(1, 2), kv[:, :, 1].transpose(1, 2))
            co = p["c_out"](ca.transpose(1, 2).reshape(1, N, C))
            x, y = ops.residual_layer_norm_modulate(x, co, shift=sh_mlp, scale=sc_mlp, eps=1e-6,
                                                    inplace=True)
            h = p["mlp2"](p["mlp0"](y, act="gelu"))  # tanh-GELU in mlp.0's epilogue
            if i + 1 < len(self.blocks):
                x, y = ops.residual_layer_norm_modulate(x, h, gate=g_mlp, shift=mods[i + 1][0],
                                                        scale=mods[i + 1][1], eps=1e-6, inplace=True)
            else:
                # final non-affine LN eps 1e-5 (trellis2_dit.rs:572)
                x, y = ops.residual_layer_norm_modulate(x, h, gate=g_mlp, eps=1e-5, inplace=True)
        return F.linear(y.view(N, C), *self.out_layer)
