/*
 * l3d_ops.h — C ABI of the B200 (sm_100a) per-token layer-op library
 * (libl3dops.so).
 *
 * Every entry point replaces one Candle op (or one composed op chain) that the
 * Lux3D model code calls on its hot path; the reference call site is cited
 * beside each declaration as `crates/lux3d-core/src/<file>:<line>`
 * ("crate/" below abbreviates `crates/lux3d-core/src/`).
 *
 * Conventions shared by all entries
 * ---------------------------------
 *  - Tensors are passed as `l3d_tensor` descriptors: a DEVICE pointer to the
 *    storage base plus Candle's Layout triple (dims, strides in elements,
 *    start offset in elements).  Outputs are caller-allocated, exactly as a
 *    Candle `CustomOp::cuda_fwd` would allocate them before calling in.
 *  - Unless an entry says otherwise, the last dimension of every activation
 *    tensor must have stride 1; leading dimensions may have any strides
 *    (strided q/k/v head views of a fused qkv projection are accepted).
 *  - Floating dtypes: F32, F16, BF16.  Arithmetic is f32 internally and the
 *    result is rounded once to the output dtype.
 *  - Every entry validates shapes/dtypes/alignment on the host and returns a
 *    status (0 = ok).  On failure `l3d_last_error()` returns a thread-local
 *    message.  No entry synchronises the host; all work is enqueued on
 *    `stream`.  Entries are stateless and reentrant unless noted.
 *  - Scratch memory is caller-provided (`workspace` + size queried with the
 *    matching `*_workspace_size` function), with one exception:
 *    `l3d_sparse_neighbor_pairs_noalloc` keeps its scratch in a fixed
 *    in-library device array, for callers that cannot allocate.
 */
#ifndef L3D_OPS_H
#define L3D_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is
 * exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* l3d_stream;

#define L3D_ABI_VERSION 1
#define L3D_MAX_DIMS 6

typedef enum l3d_dtype {
  L3D_F32 = 0,
  L3D_F16 = 1,
  L3D_BF16 = 2,
  L3D_I32 = 3,
  L3D_I64 = 4,
  L3D_U32 = 5,
  L3D_U8 = 6
} l3d_dtype;

typedef enum l3d_status {
  L3D_OK = 0,
  L3D_E_SHAPE = 1,       /* shape / rank mismatch */
  L3D_E_DTYPE = 2,       /* unsupported or mismatched dtype */
  L3D_E_ALIGN = 3,       /* stride / alignment requirement violated */
  L3D_E_UNSUPPORTED = 4, /* valid request outside the implemented envelope */
  L3D_E_CUDA = 5,        /* a CUDA runtime call failed */
  L3D_E_NULL = 6,        /* a required pointer is null */
  L3D_E_WORKSPACE = 7,   /* workspace missing or too small */
  L3D_E_DEVICE = 8       /* a kernel reported an error through its status word */
} l3d_status;

/* Candle-style tensor view: storage base + Layout (shape, strides, offset). */
typedef struct l3d_tensor {
  void* data;                     /* device pointer to the storage base */
  int32_t dtype;                  /* l3d_dtype */
  int32_t ndim;                   /* 0 .. L3D_MAX_DIMS */
  int64_t dims[L3D_MAX_DIMS];
  int64_t strides[L3D_MAX_DIMS];  /* element strides */
  int64_t offset;                 /* start offset in elements */
} l3d_tensor;

/* ---- library -------------------------------------------------------------- */
int l3d_abi_version(void);
/* Thread-local message describing the last non-zero status on this thread. */
const char* l3d_last_error(void);

/* ---- a1/a2/a3: row normalisation + adaLN modulation + residual ------------- */

/* Affine or non-affine LayerNorm over the last dim (biased variance):
 *   y = (x - mean) / sqrt(var + eps) [* weight] [+ bias]
 * weight/bias: [C] or NULL.
 * Replaces candle_nn::LayerNorm::forward at crate/runtime/vggt.rs:104,107,
 * crate/runtime/pi3_encoder.rs:67,70,153, crate/runtime/triposg_dit.rs:199,323,
 * crate/runtime/trellis2_blocks.rs:587, and the composed non-affine
 * `layer_norm_no_affine` at crate/runtime/trellis2_blocks.rs:280-286. */
int l3d_layer_norm(const l3d_tensor* x, const l3d_tensor* weight, const l3d_tensor* bias,
                   float eps, const l3d_tensor* y, l3d_stream stream);

/* Status of the kernels that take no workspace, on the current device (no
 * counterpart in the reference: Candle ops report errors only on the host).
 * The row-norm entries stream long inputs through shared memory with bounded
 * waits; a wait that runs out (status 5) is recorded in a
 * per-device word, since these entries have no workspace to hold a status.
 * This call copies it to *status (synchronising with the device) and clears
 * it when reset != 0.  0 = no wait has expired. */
int l3d_kernel_status(int* status, int reset);

/* LayerNorm + adaLN modulation (+ optional gate and residual), one HBM pass:
 *   n = LN(x) [* weight + bias]
 *   m = n * (1 + scale) + shift           (scale/shift optional)
 *   y = [x +] [gate *] m                   (gate optional, add_input 0/1)
 * x: [B, N, C] (or [N, C], B = 1).  shift/scale/gate: [C], [B, C] or
 * [B, 1, C] (arbitrary batch stride, e.g. a chunk view of a [B, 6C] vector).
 * Replaces crate/runtime/trellis2_blocks.rs:627-630,703-706 (norm1/norm3 +
 * modulate) and the VGGT camera-head adaLN crate/runtime/vggt.rs:399-405,432-437. */
int l3d_layer_norm_modulate(const l3d_tensor* x, const l3d_tensor* weight,
                            const l3d_tensor* bias, const l3d_tensor* shift,
                            const l3d_tensor* scale, const l3d_tensor* gate, int add_input,
                            float eps, const l3d_tensor* y, l3d_stream stream);

/* Gated residual: out = x + gate * h, gate [B, C] / [B, 1, C] / [C], or NULL
 * for the plain residual add out = x + h.
 * Replaces `xs.add(h.broadcast_mul(gate))` crate/runtime/trellis2_blocks.rs:632-633,
 * 644-645,708-709,716-717. */
int l3d_gated_residual(const l3d_tensor* x, const l3d_tensor* h, const l3d_tensor* gate,
                       const l3d_tensor* out, l3d_stream stream);

/* LayerScale residual: out = x + gamma * h, gamma [C].
 * Replaces LayerScale::forward crate/runtime/nn_blocks.rs:210-214 followed by the
 * residual add crate/runtime/vggt.rs:115-123, crate/runtime/pi3_encoder.rs:77-90. */
int l3d_layerscale_residual(const l3d_tensor* x, const l3d_tensor* h,
                            const l3d_tensor* gamma, const l3d_tensor* out,
                            l3d_stream stream);

/* Fused block seam: residual then the next norm, one HBM pass.
 *   r     = x + [gate *] h                 (gate: [C] LayerScale or [B,C] adaLN gate)
 *   y     = LN(r) [* weight + bias] [* (1 + scale) + shift]
 *   r_out = r                              (may alias x)
 * Composes crate/runtime/vggt.rs:118-121 (ls1 + residual, then norm2) and
 * crate/runtime/trellis2_blocks.rs:632-642,708-714 (gate + residual, then the
 * next modulated norm) into one kernel. */
int l3d_residual_layer_norm_modulate(const l3d_tensor* x, const l3d_tensor* h,
                                     const l3d_tensor* gate, const l3d_tensor* weight,
                                     const l3d_tensor* bias, const l3d_tensor* shift,
                                     const l3d_tensor* scale, float eps,
                                     const l3d_tensor* r_out, const l3d_tensor* y,
                                     l3d_stream stream);

/* ---- a5/a6: VGGT / Pi3 per-head LayerNorm + 2D axial RoPE ------------------- */

/* Same semantics as candle_nn::ops::layernorm_rope_fused(q, w, b, eps, cos_full,
 * sin_alt_full) (crate/runtime/attention_math.rs:127-150): per-head affine
 * LayerNorm over D = 64 (weight/bias [64]; both NULL = RoPE only, i.e.
 * rope_fused, crate/runtime/attention_math.rs:155-165), then
 *   out[j] = y[j] * cos_full[j] + y[partner(j)] * sin_alt_full[j]
 * per 32-wide half (crate/runtime/attention_math.rs:104-118).
 * x: [B, H, N, 64] with any strides (last stride 1); cos_full/sin_alt_full:
 * [B, 1, N, 64] F32 (or [B, N, 64]); out: [B, H, N, 64], any strides. */
int l3d_layernorm_rope2d(const l3d_tensor* x, const l3d_tensor* weight,
                         const l3d_tensor* bias, float eps, const l3d_tensor* cos_full,
                         const l3d_tensor* sin_alt_full, const l3d_tensor* out,
                         l3d_stream stream);

/* As l3d_layernorm_rope2d, but the rotation angles are formed in-kernel from
 * integer positions [B, N, 2] (y, x; I32/I64/U32) and `theta` exactly as
 * Rope2d::embeddings does (crate/runtime/attention_math.rs:14-85): no table
 * traffic.  Two tensors (q and k) may be processed in one launch: pass k/k_out
 * (and k_weight/k_bias) or NULL. */
int l3d_qk_layernorm_rope2d_pos(const l3d_tensor* q, const l3d_tensor* q_weight,
                                const l3d_tensor* q_bias, const l3d_tensor* k,
                                const l3d_tensor* k_weight, const l3d_tensor* k_bias,
                                float eps, const l3d_tensor* positions, float theta,
                                const l3d_tensor* q_out, const l3d_tensor* k_out,
                                l3d_stream stream);

/* Rope2d::embeddings (crate/runtime/attention_math.rs:14-58) on the device:
 * positions [B, N, 2] -> cos_full, sin_alt_full [B, 1, N, head_dim] F32. */
int l3d_rope2d_tables(const l3d_tensor* positions, float theta, int head_dim,
                      const l3d_tensor* cos_full, const l3d_tensor* sin_alt_full,
                      l3d_stream stream);

/* ---- a7: TripoSG per-head RMSNorm --------------------------------------------- */

/* y = x / sqrt(mean(x^2) + eps) * weight, over the last dim (D <= 256),
 * weight [D].  Replaces RmsNormHeads::rms_norm_heads
 * crate/runtime/triposg_dit.rs:511-522 (input may be the strided chunk view of
 * cat([q,k,v]) at crate/runtime/triposg_dit.rs:436-454). */
int l3d_rms_norm_heads(const l3d_tensor* x, const l3d_tensor* weight, float eps,
                       const l3d_tensor* y, l3d_stream stream);

/* ---- a8/a9: TRELLIS.2 MultiHeadRMSNorm + 3D RoPE -------------------------------- */

/* y = rope3d( x / max(||x||_2, 1e-12) * gamma[h, :] * sqrt(D) )
 * x: [B, L, H, D] (any strides, last stride 1; D even, D/2 >= 3*(D/2/3));
 * gamma: [H, D] F32 or NULL (NULL = RoPE only); coords: [L, 3] I32/I64
 * integer voxel coordinates (x, y, z), or NULL = normalisation only
 * (Trellis2QkRmsNorm alone, as in the cross attention); angles coord[axis] * freq[i],
 * freq[i] = 1 / theta^(i / (D/2/3)), pad pairs at angle 0.
 * Replaces Trellis2QkRmsNorm::forward crate/runtime/trellis2_blocks.rs:306-319
 * followed by Trellis2Rope3d::{cos_sin,apply} :106-160. */
int l3d_qk_l2norm_rope3d(const l3d_tensor* x, const l3d_tensor* gamma,
                         const l3d_tensor* coords, float theta, const l3d_tensor* y,
                         l3d_stream stream);

/* Trellis2Rope3d::cos_sin (crate/runtime/trellis2_blocks.rs:106-134) on the
 * device: coords [L, 3] -> cos, sin [L, head_dim/2] F32. */
int l3d_rope3d_tables(const l3d_tensor* coords, int head_dim, float theta,
                      const l3d_tensor* cos_out, const l3d_tensor* sin_out,
                      l3d_stream stream);

/* Trellis2Rope3d::apply (crate/runtime/trellis2_blocks.rs:139-160): rotate
 * interleaved pairs of x [B, L, H, D] by tables cos/sin [L, D/2]. */
int l3d_rope3d_apply(const l3d_tensor* x, const l3d_tensor* cos_t, const l3d_tensor* sin_t,
                     const l3d_tensor* y, l3d_stream stream);

/* ---- a10: activations --------------------------------------------------------- */

/* Tensor::gelu (tanh form) crate/runtime/trellis2_blocks.rs:558-561. */
int l3d_gelu_tanh(const l3d_tensor* x, const l3d_tensor* y, l3d_stream stream);
/* Tensor::gelu_erf crate/runtime/nn_blocks.rs:233, crate/runtime/triposg_dit.rs:298,380. */
int l3d_gelu_erf(const l3d_tensor* x, const l3d_tensor* y, l3d_stream stream);
/* Tensor::silu crate/runtime/trellis2_blocks.rs:236,257, crate/runtime/vggt.rs:393. */
int l3d_silu(const l3d_tensor* x, const l3d_tensor* y, l3d_stream stream);
/* GeGlu::forward crate/runtime/nn_blocks.rs:250-253: x [.., 2F] -> y [.., F],
 * y = x[.., :F] * gelu_erf(x[.., F:]). */
int l3d_geglu(const l3d_tensor* x, const l3d_tensor* y, l3d_stream stream);

/* Activation with its result stored to several outputs in one pass: the last
 * op of a block fused with the final all-gather of the block outputs across
 * GPUs (no single counterpart in the reference, whose pipeline runs on one
 * device: it composes `Tensor::gelu` / `gelu_erf` / `silu`,
 * crate/runtime/trellis2_blocks.rs:558-561, crate/runtime/nn_blocks.rs:233,
 * with the gather of the row shards).  act: 1 SiLU, 2 GELU-erf, 3 GELU-tanh
 * (the arithmetic of l3d_silu / l3d_gelu_erf / l3d_gelu_tanh).  x and the
 * n_out (1..8) outputs are contiguous, 16-byte aligned, same dtype and
 * element count; an output may be another GPU's memory mapped into this
 * process (CUDA IPC / peer access), which the kernel writes over NVLink.
 * The caller orders the peers' later reads (e.g. a barrier after the kernel). */
int l3d_activation_scatter(int act, const l3d_tensor* x, const l3d_tensor* outs, int n_out,
                           l3d_stream stream);

/* ---- a4/a11: timestep embedding and the small (per-step) linears ---------------- */

/* Sinusoidal timestep table for t [B] (F32) -> out [B, dim] (F32/BF16/F16).
 * order 0 = cos first, freqs exp(-ln(max_period) * i / half) with the f64 log
 *   (TRELLIS.2, crate/runtime/trellis2_blocks.rs:184-204);
 * order 1 = sin first, f32 log, arguments rounded to the output dtype before
 *   sin/cos (TripoSG, crate/runtime/triposg_dit.rs:280-294). */
int l3d_timestep_embedding(const l3d_tensor* t, int dim, int order, float max_period,
                           const l3d_tensor* out, l3d_stream stream);

/* y[b, n] = act_out( sum_k act_in(x[b, k]) * w[n, k] + bias[n] + addend[n] )
 * for small B (<= 16): the memory-bound GEMV shape of the per-step vectors.
 * act codes: 0 none, 1 SiLU, 2 GELU-erf, 3 GELU-tanh.  bias/addend [N] or NULL.
 * Covers Trellis2AdaLn::forward (SiLU -> Linear(C, 6C)) and the per-block
 * `modulation + t_emb` crate/runtime/trellis2_blocks.rs:243-258,617, and the
 * timestep MLPs crate/runtime/trellis2_blocks.rs:209-238,
 * crate/runtime/triposg_dit.rs:295-299. */
int l3d_linear_small(const l3d_tensor* x, const l3d_tensor* w, const l3d_tensor* bias,
                     const l3d_tensor* addend, int act_in, int act_out, const l3d_tensor* y,
                     l3d_stream stream);

/* ---- a12: patch embedding ------------------------------------------------------ */

/* Pi3/DINOv2 prepare_tokens (crate/runtime/pi3_encoder.rs:116-126,219-231):
 *   pixels [BS, Cin, H, W]; weight [C, Cin, p, p]; bias [C];
 *   pos [1 + np, C] (row 0 = cls position, already interpolated);
 *   cls [C]; reg [R, C] (R may be 0); out [BS, 1 + R + np, C] with
 *   out[:, 0] = cls + pos[0], out[:, 1:1+R] = reg,
 *   out[:, 1+R+i] = conv_p/p(pixels)[i] + bias + pos[1+i].
 * All tensors contiguous; F32 or BF16 (one dtype for all). */
int l3d_patch_embed(const l3d_tensor* pixels, const l3d_tensor* weight,
                    const l3d_tensor* bias, const l3d_tensor* pos, const l3d_tensor* cls,
                    const l3d_tensor* reg, int patch, const l3d_tensor* out,
                    l3d_stream stream);

/* ---- a13: dequant-linear on GGML Q8_0 / Q4_0 / K-quant blocks ------------------ */

/* Values are the GGML type ids (GgmlDType in candle_core::quantized, the
 * dtypes crate/weights/quantize.rs:355-373 names). */
typedef enum l3d_qfmt {
  L3D_Q8_0 = 8, L3D_Q4_0 = 2,
  L3D_Q4_K = 12, L3D_Q5_K = 13, L3D_Q6_K = 14
} l3d_qfmt;

/* QTensor::dequantize for a [N, K] block matrix in the GGML public layouts:
 *  Q8_0 = {f16 d; int8 q[32]} 34 B, w = d*q;
 *  Q4_0 = {f16 d; u8 qs[16]} 18 B, w = d*((nibble) - 8), low nibbles hold
 *         elements 0..15, high 16..31;
 *  256-weight super-blocks (K % 256 == 0):
 *  Q4_K = {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]} 144 B, 8 sub-blocks of
 *         32 with 6-bit scale sc and min m, w = (d*sc)*q - dmin*m;
 *  Q5_K = {f16 d; f16 dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]} 176 B,
 *         as Q4_K with a fifth bit from qh;
 *  Q6_K = {u8 ql[128]; u8 qh[64]; int8 scales[16]; f16 d} 210 B,
 *         w = (d*sc)*(q - 32) with 6-bit q and 16 sub-blocks of 16.
 * out: [N, K] F32/BF16/F16 contiguous. */
int l3d_dequantize(const void* wq, int fmt, int64_t n, int64_t k, const l3d_tensor* out,
                   l3d_stream stream);

/* Workspace bytes l3d_dequant_linear needs for an [n, k] weight and m rows. */
size_t l3d_dequant_linear_workspace_size(int fmt, int64_t m, int64_t n, int64_t k);

/* y[M, N] = x[M, K] . deq(W)^T + bias  (Linear::forward / QMatMul::forward,
 * crate/runtime/nn_blocks.rs:80-95, weights from quantized_linear :123-152).
 * x: [.., K] BF16 (F32 accepted: rounded to BF16 on the way in), contiguous
 * rows; W: raw GGML blocks (n rows of k/32 blocks, or k/256 super-blocks for
 * the K-quants, which are always decoded once per call into the workspace);
 * bias [N] F32/BF16 or NULL;
 * y: [.., N] BF16 or F32 contiguous.  Tensor cores (tcgen05, TMEM
 * accumulators, f32 accumulate). */
int l3d_dequant_linear(const l3d_tensor* x, const void* wq, int fmt, int64_t n, int64_t k,
                       const l3d_tensor* bias, const l3d_tensor* y, void* workspace,
                       size_t workspace_bytes, l3d_stream stream);

/* As l3d_dequant_linear, with the element-wise ops that follow the linear in
 * the reference's blocks fused into the GEMM epilogue (no extra pass over y):
 *   y = residual + gate * act(x . deq(W)^T + bias)
 * act: 0 none, 1 SiLU, 2 GELU-erf, 3 GELU-tanh (computed in f32 before the
 * single rounding to y's dtype); residual: y's dtype and shape, row-major, or
 * NULL (it may be y itself, for an in-place x += ...; y must not overlap x);
 * gate: [N] F32/BF16, or NULL for 1 (only with a residual).  Replaces
 * Trellis2FeedForward's mlp.0 + gelu (crate/runtime/trellis2_blocks.rs:
 * 558-561) and the gated residuals xs + gate * h (:632-633, :644-645). */
int l3d_dequant_linear_ex(const l3d_tensor* x, const void* wq, int fmt, int64_t n, int64_t k,
                          const l3d_tensor* bias, int act, const l3d_tensor* residual,
                          const l3d_tensor* gate, const l3d_tensor* y, void* workspace,
                          size_t workspace_bytes, l3d_stream stream);

/* Workspace bytes for l3d_linear_ex with m rows. */
size_t l3d_linear_workspace_size(int64_t m, int64_t n, int64_t k);

/* Dense linear with the same fused epilogue as l3d_dequant_linear_ex:
 *   y = residual + gate * act(x . W^T + bias)
 * W: BF16 [n, k], row-major with 16-byte aligned rows (k a multiple of 8),
 * used as is (bf16 operands, f32 accumulation on the tensor cores).  Replaces
 * candle_nn::Linear::forward / ops::mul_mat_add on unquantised weights
 * (crate/runtime/nn_blocks.rs:82,179-195) followed by the element-wise ops of
 * the blocks: Mlp fc1 + gelu_erf (crate/runtime/nn_blocks.rs:219-236), the
 * LayerScale residual x + ls * proj(..) (crate/runtime/nn_blocks.rs:210-214,
 * crate/runtime/vggt.rs:118-121) as residual = x, gate = ls. */
int l3d_linear_ex(const l3d_tensor* x, const l3d_tensor* weight, const l3d_tensor* bias, int act,
                  const l3d_tensor* residual, const l3d_tensor* gate, const l3d_tensor* y,
                  void* workspace, size_t workspace_bytes, l3d_stream stream);

/* ---- next row: submanifold sparse conv 3x3x3 ------------------------------------ */

/* Dense neighbour table of a coordinate set: nbr[i, k] = row of coord_i +
 * delta_k (k = kd*9 + kh*3 + kw, delta = (kd-1, kh-1, kw-1)) or -1; the same
 * lookups as l3d_sparse_neighbor_pairs (CoordMap, later duplicates win,
 * crate/runtime/trellis2_sparse.rs:68-106), in [N, 27] I32 form.  Workspace:
 * l3d_sparse_neighbor_pairs_workspace_size(N) bytes, 256-byte aligned. */
int l3d_sparse_neighbor_map(const l3d_tensor* coords, const l3d_tensor* nbr, void* workspace,
                            size_t workspace_bytes, l3d_stream stream);

/* Workspace bytes for l3d_sparse_conv3d on n rows of cin channels. */
size_t l3d_sparse_conv3d_workspace_size(int64_t n, int64_t cin, int feats_dtype);

/* SparseConv3d::forward (crate/runtime/trellis2_sparse.rs:197-243):
 * out[i] = bias + sum_k W[k] . feats[nbr[i, k]] (missing neighbours add 0),
 * as one implicit GEMM on the tensor cores (tcgen05, f32 accumulate): the
 * neighbour rows are gathered into the operand tile in shared memory, never
 * materialised.  feats [N, Cin] BF16 (F32 accepted: rounded to BF16), Cin a
 * multiple of 8; nbr [N, 27] I32 from l3d_sparse_neighbor_map; weight
 * [27, Cout, Cin] BF16 contiguous (the reference's weight27 layout); bias
 * [Cout] F32/BF16 or NULL; out [N, Cout] F32/BF16. */
int l3d_sparse_conv3d(const l3d_tensor* feats, const l3d_tensor* nbr, const l3d_tensor* weight,
                      const l3d_tensor* bias, const l3d_tensor* out, void* workspace,
                      size_t workspace_bytes, l3d_stream stream);

/* Workspace bytes for l3d_sparse_conv3d_pairs (counts_host: the 27 pair
 * counts, as in `counts`, read on the host). */
size_t l3d_sparse_conv3d_pairs_workspace_size(int64_t n, int64_t cin, int64_t cout,
                                              const int32_t* counts_host);

/* SparseConv3d::forward as the reference computes it
 * (crate/runtime/trellis2_sparse.rs:211-241): for each kernel offset k, the
 * rows feats[pair_src[k, p]] of its pairs times W[k]^T, added into
 * out[pair_dest[k, p]] in ascending k (index_add), then + bias.  One
 * tensor-core launch multiplies the pairs of all offsets (each offset's pairs
 * a segment of 128-row tiles, so the work follows the neighbour count, not
 * 27 x N), storing f32 products; a second pass adds each output row's
 * products in ascending offset order, then the bias - the reference's
 * summation order, deterministic.  Pair lists and device counts as written by
 * l3d_sparse_neighbor_pairs; counts_host holds the same 27 counts in host
 * memory (they size the launch and the workspace); other arguments as for
 * l3d_sparse_conv3d. */
int l3d_sparse_conv3d_pairs(const l3d_tensor* feats, const l3d_tensor* pair_src,
                            const l3d_tensor* pair_dest, const l3d_tensor* counts,
                            const int32_t* counts_host, const l3d_tensor* weight,
                            const l3d_tensor* bias, const l3d_tensor* out, void* workspace,
                            size_t workspace_bytes, l3d_stream stream);

/* ---- next row: the attention core --------------------------------------------- */

/* Workspace bytes for l3d_attention (256: the status word). */
size_t l3d_attention_workspace_size(int64_t b, int64_t h, int64_t nk, int64_t d);

/* exact_sdpa_heads / exact_query_chunked_sdpa
 * (crate/runtime/attention_math.rs:199-259), non-causal: out = softmax(q k^T *
 * scale) v per (batch, head), on the tensor cores (tcgen05, TMEM, TMA; online
 * softmax in f32, P rounded to bf16 for the second product).  q [B, H, N, D],
 * k and v [B, H, Nk, D], out [B, H, N, D], BF16, D = 64 or 128, any strides
 * with the head dim contiguous and 16-byte multiples elsewhere (e.g. views of
 * a [B, N, 3, H, D] projection or token-major [B, N, H, D] memory), read in
 * place.  scale must be positive.  The workspace holds a status word (0 = ok;
 * non-zero = a bounded wait inside the kernel expired). */
int l3d_attention(const l3d_tensor* q, const l3d_tensor* k, const l3d_tensor* v, float scale,
                  const l3d_tensor* out, void* workspace, size_t workspace_bytes,
                  l3d_stream stream);

/* Failure-handling self-test of l3d_attention (no counterpart in the
 * reference): the same launch, except that the first key tile is never
 * loaded and every bounded wait gives up after wait_limit_ms (1 .. 2000).
 * The kernel must then record status 5 (timeout) in the workspace, wait for
 * the copies and tensor-core operations it started, free its tensor memory
 * and return, leaving the context usable; the caller reads the status word
 * after synchronising.  Needs at least one key. */
int l3d_attention_selftest_timeout(const l3d_tensor* q, const l3d_tensor* k,
                                   const l3d_tensor* v, float scale, const l3d_tensor* out,
                                   void* workspace, size_t workspace_bytes,
                                   uint32_t wait_limit_ms, l3d_stream stream);

/* ---- GGUF tensor index (the on-disk format feeding a13) ------------------------ */

/* One tensor of a GGUF file.  name points into the caller's buffer (not
 * NUL-terminated); dims are in row-major (Candle) order, dims[0] outermost,
 * unused trailing dims 1; offset is the byte offset of the data from the start
 * of the buffer; nbytes is 0 for a GGML type this library does not know. */
typedef struct l3d_gguf_tensor {
  const char* name;
  uint64_t name_len;
  int32_t type;      /* GGML type id: 0 F32, 1 F16, 30 BF16, 2 Q4_0, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K, ... */
  int32_t n_dims;
  int64_t dims[4];
  uint64_t offset;
  uint64_t nbytes;
} l3d_gguf_tensor;

/* gguf_file::Content::read (Candle, used at crate/weights/mod.rs:596-650 on
 * the file crate/weights/quantize.rs:255-295 writes): index a GGUF v2/v3
 * buffer (e.g. an mmap of model.gguf).  Fills up to max_tensors entries
 * (tensors may be NULL when max_tensors is 0) and stores the file's tensor
 * count in *n_tensors; version / alignment (general.alignment, default 32)
 * are optional outputs.  Host code only: no device work, no allocation;
 * malformed or truncated buffers return L3D_E_SHAPE. */
int l3d_gguf_index(const void* buf, uint64_t len, l3d_gguf_tensor* tensors,
                   int64_t max_tensors, int64_t* n_tensors, uint32_t* version,
                   uint64_t* alignment);

/* The string value of metadata `key` (e.g. "general.architecture",
 * "lux3d.family", "lux3d.resolved_config", crate/weights/mod.rs:26-28),
 * pointing into buf; L3D_E_SHAPE when absent or not a string. */
int l3d_gguf_metadata_string(const void* buf, uint64_t len, const char* key,
                             const char** value, uint64_t* value_len);

/* ---- a14: sparse voxel neighbour pairs and row gather ---------------------------- */

/* Workspace bytes for l3d_sparse_neighbor_pairs on n coordinates. */
size_t l3d_sparse_neighbor_pairs_workspace_size(int64_t n);

/* Submanifold 3x3x3 neighbour lists (CoordMap + kernel_offset_delta,
 * crate/runtime/trellis2_sparse.rs:68-106, pair build :211-236):
 * coords [N, 3] I32 unique (x, y, z) >= 0 (any order; later duplicates win);
 * for each offset k (delta = (k/9-1, (k%9)/3-1, k%3-1)) writes the pairs
 * (dest = i, src = map[coord_i + delta]) in ascending i into
 * pair_dest[k, 0:count[k]], pair_src[k, 0:count[k]] ([27, N] I32) and
 * counts [27] I32.  Bit-exact with the reference's host loop. */
int l3d_sparse_neighbor_pairs(const l3d_tensor* coords, const l3d_tensor* pair_dest,
                              const l3d_tensor* pair_src, const l3d_tensor* counts,
                              void* workspace, size_t workspace_bytes, l3d_stream stream);

/* Same result as l3d_sparse_neighbor_pairs, for callers that cannot allocate
 * device memory (a Candle CustomOp's cuda_fwd, a replayed CUDA graph, a host
 * runtime that forbids allocation while serving): takes no workspace and
 * allocates nothing.  No counterpart in the reference (its CoordMap is a
 * host HashMap).  Scratch is a file-scope device array of the library sized
 * for at most 65536 coordinates (about 1.6 MB, held on every GPU that loads
 * the library until the process exits); larger inputs are rejected with
 * L3D_E_UNSUPPORTED.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  All calls share the one array: calls that overlap on the
 * GPU (different streams, or different host threads) race and must be
 * serialised by the caller. */
int l3d_sparse_neighbor_pairs_noalloc(const l3d_tensor* coords, const l3d_tensor* pair_dest,
                                      const l3d_tensor* pair_src, const l3d_tensor* counts,
                                      l3d_stream stream);

/* index_select_rows crate/runtime/trellis2_sparse.rs:118-133:
 * out[j, :] = feats[ids[j], :]; ids I32/U32/I64; feats/out same dtype. */
int l3d_index_select_rows(const l3d_tensor* feats, const l3d_tensor* ids,
                          const l3d_tensor* out, l3d_stream stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* L3D_OPS_H */
