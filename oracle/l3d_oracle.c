/*
 * l3d_oracle.c — TEST INFRASTRUCTURE ONLY.  CPU restatement of the Lux3D
 * (FerrisMind/candle-3d) per-token layer-op path, used as the parity checker
 * for the CUDA kernels of libl3dops and as the timed CPU baseline.  Nothing in
 * the product path links or calls this file.
 *
 * Every function restates the reference's op order in f32 (the reference's
 * production compute dtype), citing the file:line it follows
 * ("crate/" = crates/lux3d-core/src/).  `rnd` selects Candle's per-op output
 * rounding for reduced-precision activations: 0 = f32 (no rounding),
 * 1 = round every op output to bf16, 2 = to f16 (each Candle op materialises
 * its output tensor in the activation dtype).
 *
 * Pinning: the RoPE tables and rotation, the q/k L2-norm, the cos-first
 * timestep table, the adaLN chunk order and the 3x3x3 offset order are
 * checked against the reference's own known-answer tests
 * (crates/lux3d-core/tests/trellis2_blocks.rs:43-225,
 * crates/lux3d-core/tests/trellis2_sparse.rs:68-98); Candle's internal
 * LayerNorm / GELU / SiLU arithmetic lives in the un-vendored Candle fork and
 * is restated from the formulas only (parity unpinned at the bit level for
 * those ops).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ rounding */
static inline float rbf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    if (u & 0x7fffffu) u |= 0x00400000u; /* quiet NaN */
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  float r;
  memcpy(&r, &u, 4);
  return r;
}
static inline float rf16(float f) { return (float)(_Float16)f; }
static inline float R(float f, int rnd) { return rnd == 1 ? rbf16(f) : rnd == 2 ? rf16(f) : f; }

int orc_round_array(float* x, int64_t n, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) x[i] = R(x[i], rnd);
  return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Use n host threads (launchers such as torchrun default OMP_NUM_THREADS to 1). */
int orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
  return 0;
}

/* ------------------------------------------------------ LayerNorm family */
/* Composed LayerNorm over one row, as layer_norm_no_affine
 * (crate/runtime/trellis2_blocks.rs:280-286): mean_keepdim, broadcast_sub,
 * sqr, mean_keepdim, affine(1, eps), sqrt, broadcast_div; then the affine
 * weight/bias of candle_nn::LayerNorm (crate/runtime/vggt.rs:104). */
static void ln_row(const float* x, int64_t C, const float* w, const float* b, float eps,
                   float* y, int rnd) {
  float s = 0.f;
  for (int64_t c = 0; c < C; ++c) s += x[c];
  const float mean = R(s / (float)C, rnd);
  float ss = 0.f;
  for (int64_t c = 0; c < C; ++c) {
    const float d = R(x[c] - mean, rnd);
    ss += R(d * d, rnd);
  }
  const float var = R(ss / (float)C, rnd);
  const float denom = R(sqrtf(R(var + eps, rnd)), rnd);
  for (int64_t c = 0; c < C; ++c) {
    float v = R(R(x[c] - mean, rnd) / denom, rnd);
    if (w) v = R(v * w[c], rnd);
    if (b) v = R(v + b[c], rnd);
    y[c] = v;
  }
}

int orc_layer_norm(const float* x, int64_t rows, int64_t C, const float* w, const float* b,
                   float eps, float* y, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) ln_row(x + r * C, C, w, b, eps, y + r * C, rnd);
  return 0;
}

/* LayerNorm + adaLN modulate + gate + residual:
 *   h = LN(x) [*w + b]; h = h * (1 + scale) + shift        trellis2_blocks.rs:627-630
 *   y = gate * h [+ x]                                       vggt.rs:399-405
 * shift/scale/gate are [B, C] (row r belongs to batch r / rows_per_batch). */
int orc_layer_norm_modulate(const float* x, int64_t rows, int64_t C, int64_t rows_per_batch,
                            const float* w, const float* b, const float* shift,
                            const float* scale, const float* gate, int add_input, float eps,
                            float* y, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t bb = r / rows_per_batch;
    float* yr = y + r * C;
    const float* xr = x + r * C;
    ln_row(xr, C, w, b, eps, yr, rnd);
    for (int64_t c = 0; c < C; ++c) {
      float v = yr[c];
      if (scale) v = R(v * R(1.f + scale[bb * C + c], rnd), rnd); /* scale.affine(1, 1) */
      if (shift) v = R(v + shift[bb * C + c], rnd);
      if (gate) v = R(gate[bb * C + c] * v, rnd);
      if (add_input) v = R(v + xr[c], rnd);
      yr[c] = v;
    }
  }
  return 0;
}

/* out = x + g * h; g is [B, C] (adaLN gate, trellis2_blocks.rs:632-633) or,
 * with rows_per_batch = rows, a LayerScale gamma [C] (nn_blocks.rs:210-214,
 * vggt.rs:118). */
int orc_gated_residual(const float* x, const float* h, const float* g, int64_t rows, int64_t C,
                       int64_t rows_per_batch, float* out, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t bb = r / rows_per_batch;
    for (int64_t c = 0; c < C; ++c) {
      const float gh = g ? R(h[r * C + c] * g[bb * C + c], rnd) : h[r * C + c];
      out[r * C + c] = R(x[r * C + c] + gh, rnd);
    }
  }
  return 0;
}

/* RMSNorm heads (crate/runtime/triposg_dit.rs:516-521):
 *   variance = mean(x^2); normed = x / sqrt(variance + eps); normed * weight */
int orc_rms_norm_heads(const float* x, int64_t rows, int64_t D, const float* w, float eps,
                       float* y, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * D;
    float ss = 0.f;
    for (int64_t d = 0; d < D; ++d) ss += R(xr[d] * xr[d], rnd);
    const float var = R(ss / (float)D, rnd);
    const float den = R(sqrtf(R(var + eps, rnd)), rnd);
    for (int64_t d = 0; d < D; ++d) {
      float v = R(xr[d] / den, rnd);
      if (w) v = R(v * w[d], rnd);
      y[r * D + d] = v;
    }
  }
  return 0;
}

/* --------------------------------------------------------------- 2D RoPE */
/* Rope2d::cos_sin + embeddings (crate/runtime/attention_math.rs:14-76):
 * inv_freq[f] = 1 / theta^(2f / dim) (dim = head_dim / 2), freqs = cat(f, f),
 * angle = (f32)pos * inv_freq (an outer product), tables gathered by the y
 * position for the first half and the x position for the second half,
 * sin_alt negated in the first quarter of each half (:36-50).
 * positions: [B, N, 2] int64; cos_full/sin_alt_full: [B, N, head_dim]. */
int orc_rope2d_tables(const int64_t* pos, int64_t B, int64_t N, float theta, int head_dim,
                      float* cos_full, float* sin_alt_full) {
  const int half = head_dim / 2, quarter = half / 2;
  float* inv = (float*)malloc(sizeof(float) * (size_t)quarter);
  for (int f = 0; f < quarter; ++f) inv[f] = 1.0f / powf(theta, (float)(2 * f) / (float)half);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < B * N; ++t) {
    for (int e = 0; e < head_dim; ++e) {
      const int hf = e / half, j = e % half, f = j % quarter;
      const float ang = (float)pos[t * 2 + hf] * inv[f];
      cos_full[t * head_dim + e] = cosf(ang);
      const float s = sinf(ang);
      sin_alt_full[t * head_dim + e] = j < quarter ? -s : s;
    }
  }
  free(inv);
  return 0;
}

/* apply_layernorm_rope composed path (crate/runtime/attention_math.rs:147-149):
 * q_norm.forward (per-head LayerNorm, affine) then rope_apply (:104-118):
 *   out = tokens * cos + cat(y2, y1, x2, x1) * sin_alt.
 * x: [B, H, N, D] contiguous; tables [B, N, D]; w/b NULL = rope only (:155-165).
 * For reduced precision the tables are cast to the activation dtype (:113-115). */
int orc_layernorm_rope2d(const float* x, int64_t B, int64_t H, int64_t N, int64_t D,
                         const float* w, const float* b, float eps, const float* cos_full,
                         const float* sin_alt_full, float* out, int rnd) {
  const int64_t half = D / 2, quarter = half / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < B * H * N; ++r) {
    const int64_t bb = r / (H * N), n = r % N;
    float y[1024];
    if (w || b) ln_row(x + r * D, D, w, b, eps, y, rnd);
    else memcpy(y, x + r * D, sizeof(float) * (size_t)D);
    const float* c = cos_full + (bb * N + n) * D;
    const float* s = sin_alt_full + (bb * N + n) * D;
    for (int64_t e = 0; e < D; ++e) {
      const int64_t j = e % half;
      const int64_t partner = (e - j) + (j < quarter ? j + quarter : j - quarter);
      const float a = R(y[e] * R(c[e], rnd), rnd);
      const float p = R(y[partner] * R(s[e], rnd), rnd);
      out[r * D + e] = R(a + p, rnd);
    }
  }
  return 0;
}

/* --------------------------------------------------------------- 3D RoPE */
/* rope_axis_frequencies (crate/runtime/trellis2_blocks.rs:57-75):
 * freq[i] = 1 / theta^(i / freq_dim), freq_dim = head_dim / 2 / 3.
 * Trellis2Rope3d::cos_sin (:106-134): angle[axis * freq_dim + i] =
 * (f32)coord[axis] * freq[i], zero (identity) pad to head_dim / 2.
 * coords: [L, 3] int64; cos/sin: [L, head_dim / 2]. */
int orc_rope3d_tables(const int64_t* coords, int64_t L, int head_dim, float theta, float* cosv,
                      float* sinv) {
  const int half = head_dim / 2, fd = head_dim / 2 / 3;
  if (fd == 0) return 1;
  float* fr = (float*)malloc(sizeof(float) * (size_t)fd);
  for (int i = 0; i < fd; ++i) fr[i] = 1.0f / powf(theta, (float)i / (float)fd);
#pragma omp parallel for schedule(static)
  for (int64_t l = 0; l < L; ++l) {
    for (int p = 0; p < half; ++p) {
      float ang = 0.f;
      if (p < 3 * fd) ang = (float)coords[l * 3 + p / fd] * fr[p % fd];
      cosv[l * half + p] = cosf(ang);
      sinv[l * half + p] = sinf(ang);
    }
  }
  free(fr);
  return 0;
}

/* Trellis2Rope3d::apply (crate/runtime/trellis2_blocks.rs:139-160):
 * out_re = re*cos - im*sin; out_im = re*sin + im*cos over interleaved pairs.
 * x: [B, L, H, D] contiguous; cos/sin: [L, D / 2]. */
int orc_rope3d_apply(const float* x, int64_t B, int64_t L, int64_t H, int64_t D,
                     const float* cosv, const float* sinv, float* y, int rnd) {
  const int64_t half = D / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < B * L * H; ++r) {
    const int64_t l = (r / H) % L;
    for (int64_t p = 0; p < half; ++p) {
      const float re = x[r * D + 2 * p], im = x[r * D + 2 * p + 1];
      const float c = R(cosv[l * half + p], rnd), s = R(sinv[l * half + p], rnd);
      y[r * D + 2 * p] = R(R(re * c, rnd) - R(im * s, rnd), rnd);
      y[r * D + 2 * p + 1] = R(R(re * s, rnd) + R(im * c, rnd), rnd);
    }
  }
  return 0;
}

/* Trellis2QkRmsNorm::forward (crate/runtime/trellis2_blocks.rs:306-319):
 * norm = clamp(sqrt(sum x^2), 1e-12, 1e30); x / norm * gamma[h, :] * sqrt(D),
 * computed in F32; then Rope3d (cos_sin + apply).  gamma NULL = rope only. */
int orc_qk_l2norm_rope3d(const float* x, int64_t B, int64_t L, int64_t H, int64_t D,
                         const float* gamma, const int64_t* coords, float theta, float* y,
                         int rnd) {
  const int64_t half = D / 2;
  float* cosv = (float*)malloc(sizeof(float) * (size_t)(L * half));
  float* sinv = (float*)malloc(sizeof(float) * (size_t)(L * half));
  float* nrm = (float*)malloc(sizeof(float) * (size_t)(B * L * H * D));
  if (!coords) {
    /* Normalisation only: identity rotation. */
    for (int64_t i = 0; i < L * half; ++i) { cosv[i] = 1.f; sinv[i] = 0.f; }
  } else if (orc_rope3d_tables(coords, L, (int)D, theta, cosv, sinv)) {
    free(cosv); free(sinv); free(nrm);
    return 1;
  }
  const float scale = sqrtf((float)D);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < B * L * H; ++r) {
    const int64_t h = r % H;
    const float* xr = x + r * D;
    if (!gamma) {
      memcpy(nrm + r * D, xr, sizeof(float) * (size_t)D);
      continue;
    }
    float ss = 0.f;
    for (int64_t d = 0; d < D; ++d) ss += xr[d] * xr[d];
    float n = sqrtf(ss);
    if (n < 1e-12f) n = 1e-12f;
    if (n > 1e30f) n = 1e30f;
    for (int64_t d = 0; d < D; ++d)
      nrm[r * D + d] = R(R(R(xr[d] / n, rnd) * gamma[h * D + d], rnd) * scale, rnd);
  }
  orc_rope3d_apply(nrm, B, L, H, D, cosv, sinv, y, rnd);
  free(cosv);
  free(sinv);
  free(nrm);
  return 0;
}

/* ------------------------------------------------------------ activations */
/* Tensor::gelu (tanh form, crate/runtime/trellis2_blocks.rs:558-561). */
static inline float gelu_tanh(float v) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * v * (1.0f + tanhf(k0 * v * (1.0f + k1 * v * v)));
}
/* Tensor::gelu_erf (crate/runtime/nn_blocks.rs:233). */
static inline float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f)); }
/* Tensor::silu (crate/runtime/trellis2_blocks.rs:236). */
static inline float silu(float v) { return v / (1.0f + expf(-v)); }
static inline float act(int a, float v) {
  return a == 1 ? silu(v) : a == 2 ? gelu_erf(v) : a == 3 ? gelu_tanh(v) : v;
}

int orc_activation(const float* x, int64_t n, int a, float* y, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) y[i] = R(act(a, x[i]), rnd);
  return 0;
}

/* GeGlu::forward (crate/runtime/nn_blocks.rs:250-253): x [rows, 2F]. */
int orc_geglu(const float* x, int64_t rows, int64_t F, float* y, int rnd) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < F; ++j)
      y[r * F + j] = R(x[r * 2 * F + j] * R(gelu_erf(x[r * 2 * F + F + j]), rnd), rnd);
  return 0;
}

/* ------------------------------------------------------------ timestep */
/* order 0: TRELLIS.2 timestep_embedding (crate/runtime/trellis2_blocks.rs:184-204):
 *   nlp = -(ln(max_period) in f64) as f32; freqs[i] = exp(nlp * i / half);
 *   args = freqs * t; [cos(args), sin(args)], odd dim zero-padded.
 * order 1: TripoSG (crate/runtime/triposg_dit.rs:280-294):
 *   lmp = -(ln(max_period) in f32); emb[i] = t * exp(lmp * i / half);
 *   emb cast to the activation dtype; [sin(emb), cos(emb)]. */
int orc_timestep_embedding(const float* t, int64_t B, int dim, int order, float max_period,
                           float* out, int rnd) {
  const int half = dim / 2;
  const float nlp = order == 0 ? (float)(-log((double)max_period)) : -logf(max_period);
  for (int64_t b = 0; b < B; ++b) {
    float* o = out + b * dim;
    for (int i = 0; i < half; ++i) {
      const float freq = expf(nlp * (float)i / (float)half);
      float arg = order == 0 ? freq * t[b] : t[b] * freq;
      if (order == 1) arg = R(arg, rnd);
      const float c = R(cosf(arg), rnd), s = R(sinf(arg), rnd);
      if (order == 0) { o[i] = c; o[half + i] = s; }
      else { o[i] = s; o[half + i] = c; }
    }
    if (dim % 2) o[dim - 1] = 0.f;
  }
  return 0;
}

/* ------------------------------------------------------------- linears */
/* y = act_out(act_in(x) . w^T + bias + addend), f64 accumulation (the exact
 * dot product the tolerance is measured against).  Linear::forward
 * (crate/runtime/nn_blocks.rs:80-95), Trellis2AdaLn (trellis2_blocks.rs:243-258),
 * the per-block modulation add (:617), timestep MLPs (:209-238). */
int orc_linear(const float* x, int64_t B, int64_t K, const float* w, int64_t N, const float* bias,
               const float* addend, int act_in, int act_out, float* y) {
  float* xa = (float*)malloc(sizeof(float) * (size_t)(B * K));
  for (int64_t i = 0; i < B * K; ++i) xa[i] = act(act_in, x[i]);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < B; ++b) {
      double acc = 0.0;
      const float* wr = w + n * K;
      const float* xr = xa + b * K;
      for (int64_t k = 0; k < K; ++k) acc += (double)xr[k] * (double)wr[k];
      float v = (float)acc;
      if (bias) v += bias[n];
      if (addend) v += addend[n];
      y[b * N + n] = act(act_out, v);
    }
  }
  free(xa);
  return 0;
}

/* Pi3 PatchEmbed + prepare_tokens (crate/runtime/pi3_encoder.rs:116-126,219-231):
 * conv2d(k = s = p) + bias, cat(cls, patches) + pos, then insert the register
 * tokens after cls.  pixels [BS, Cin, H, W]; weight [C, Cin, p, p];
 * pos [1 + np, C]; reg [R, C]; out [BS, 1 + R + np, C]. */
int orc_patch_embed(const float* pix, int64_t BS, int64_t Cin, int64_t H, int64_t W,
                    const float* wt, const float* bias, const float* pos, const float* cls,
                    const float* reg, int64_t R_, int p, int64_t C, float* out) {
  const int64_t ph = H / p, pw = W / p, np = ph * pw, K = Cin * p * p, T = 1 + R_ + np;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < BS * np; ++m) {
    const int64_t bs = m / np, t = m % np, py = t / pw, px = t % pw;
    for (int64_t n = 0; n < C; ++n) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        const int64_t c = k / (p * p), r = k % (p * p), ky = r / p, kx = r % p;
        acc += (double)pix[((bs * Cin + c) * H + py * p + ky) * W + px * p + kx] *
               (double)wt[n * K + k];
      }
      const float v = (float)acc + bias[n];
      out[(bs * T + 1 + R_ + t) * C + n] = v + pos[(1 + t) * C + n];
    }
  }
  for (int64_t bs = 0; bs < BS; ++bs) {
    for (int64_t n = 0; n < C; ++n) out[(bs * T) * C + n] = cls[n] + pos[n];
    for (int64_t r = 0; r < R_; ++r)
      for (int64_t n = 0; n < C; ++n) out[(bs * T + 1 + r) * C + n] = reg[r * C + n];
  }
  (void)K;
  return 0;
}

/* ------------------------------------------------------- GGML Q8_0 / Q4_0 */
static float h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}
static uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

/* GGML block decode (public format; QTensor::dequantize). */
/* GGML K-quant super-blocks (256 weights), public layouts and decode order
 * (dequantize_row_q4_K / _q5_K / _q6_K in ggml; Candle's k_quants follow
 * them): Q4_K {f16 d, f16 dmin, u8 scales[12], u8 qs[128]} 144 B; Q5_K adds
 * u8 qh[32] before qs, 176 B; Q6_K {u8 ql[128], u8 qh[64], i8 scales[16],
 * f16 d} 210 B.  The f32 products and differences are formed one at a time
 * (no contraction), in the order written here. */
static void kq_scale_min(const uint8_t* q, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

static void dequant_q45k_block(const uint8_t* blk, int q5, float* y) {
  const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
  const uint8_t* scales = blk + 4;
  const uint8_t* qh = blk + 16;
  const uint8_t* ql = blk + (q5 ? 48 : 16);
  int is = 0;
  for (int j = 0; j < 256; j += 64) {
    int sc, m;
    kq_scale_min(scales, is, &sc, &m);
    const float d1 = d * (float)sc, m1 = dmin * (float)m;
    kq_scale_min(scales, is + 1, &sc, &m);
    const float d2 = d * (float)sc, m2 = dmin * (float)m;
    const int b1 = is, b2 = is + 1; /* qh bit of the two sub-blocks */
    for (int l = 0; l < 32; ++l) {
      int q = ql[l] & 0xF;
      if (q5) q += ((qh[l] >> b1) & 1) << 4;
      *y++ = d1 * (float)q - m1;
    }
    for (int l = 0; l < 32; ++l) {
      int q = ql[l] >> 4;
      if (q5) q += ((qh[l] >> b2) & 1) << 4;
      *y++ = d2 * (float)q - m2;
    }
    ql += 32;
    is += 2;
  }
}

static void dequant_q6k_block(const uint8_t* blk, float* y) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const int8_t* sc = (const int8_t*)(blk + 192);
  const float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
  for (int n = 0; n < 256; n += 128) {
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
      const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * (float)sc[is + 0] * (float)q1;
      y[l + 32] = d * (float)sc[is + 2] * (float)q2;
      y[l + 64] = d * (float)sc[is + 4] * (float)q3;
      y[l + 96] = d * (float)sc[is + 6] * (float)q4;
    }
    y += 128;
    ql += 64;
    qh += 32;
    sc += 8;
  }
}

int orc_dequantize(const uint8_t* wq, int fmt, int64_t n, int64_t k, float* out) {
  if (fmt == 12 || fmt == 13 || fmt == 14) {
    const int bb = fmt == 12 ? 144 : fmt == 13 ? 176 : 210;
    if (k % 256) return 1;
    const int64_t nsb = n * (k / 256);
    for (int64_t b = 0; b < nsb; ++b) {
      if (fmt == 14) dequant_q6k_block(wq + b * bb, out + b * 256);
      else dequant_q45k_block(wq + b * bb, fmt == 13, out + b * 256);
    }
    return 0;
  }
  const int bb = fmt == 8 ? 34 : 18;
  const int64_t nblk = n * (k / 32);
  for (int64_t b = 0; b < nblk; ++b) {
    const uint8_t* blk = wq + b * bb;
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    float* o = out + b * 32;
    if (fmt == 8) {
      for (int j = 0; j < 32; ++j) o[j] = d * (float)(int8_t)blk[2 + j];
    } else {
      for (int j = 0; j < 16; ++j) {
        o[j] = d * (float)((int)(blk[2 + j] & 15) - 8);
        o[16 + j] = d * (float)((int)(blk[2 + j] >> 4) - 8);
      }
    }
  }
  return 0;
}

/* GGML reference quantisers (quantize_row_q8_0 / quantize_row_q4_0, public
 * algorithms): Q8_0 d = amax / 127, q = round(x / d); Q4_0 d = max / -8 with
 * max the signed value of largest magnitude, q = min(15, (int)(x / d + 8.5)). */
int orc_quantize(const float* w, int fmt, int64_t n, int64_t k, uint8_t* out) {
  const int bb = fmt == 8 ? 34 : 18;
  const int64_t nblk = n * (k / 32);
  for (int64_t b = 0; b < nblk; ++b) {
    const float* x = w + b * 32;
    uint8_t* blk = out + b * bb;
    if (fmt == 8) {
      float amax = 0.f;
      for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
      const float d = amax / 127.f;
      const float id = d != 0.f ? 1.f / d : 0.f;
      const uint16_t hd = f2h(d);
      blk[0] = (uint8_t)(hd & 0xff);
      blk[1] = (uint8_t)(hd >> 8);
      for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
    } else {
      float amax = 0.f, mx = 0.f;
      for (int j = 0; j < 32; ++j) {
        if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); mx = x[j]; }
      }
      const float d = mx / -8.f;
      const float id = d != 0.f ? 1.f / d : 0.f;
      const uint16_t hd = f2h(d);
      blk[0] = (uint8_t)(hd & 0xff);
      blk[1] = (uint8_t)(hd >> 8);
      for (int j = 0; j < 16; ++j) {
        const float x0 = x[j] * id, x1 = x[16 + j] * id;
        int q0 = (int)(x0 + 8.5f), q1 = (int)(x1 + 8.5f);
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------- sparse neighbours */
/* CoordMap (crate/runtime/trellis2_sparse.rs:68-94; HashMap insert, so a later
 * duplicate overwrites an earlier one), kernel_offset_delta (:99-106:
 * k = kd*9 + kh*3 + kw, delta = (kd-1, kh-1, kw-1)) and the per-offset pair
 * lists in ascending row order (:211-224).  Map: open addressing on the
 * packed coordinate.  pair_dest/pair_src: [27, N]; counts: [27]. */
typedef struct { uint64_t key; int32_t val; } orc_slot;

static uint64_t orc_mix(uint64_t k) {
  k ^= k >> 30; k *= 0xbf58476d1ce4e5b9ull;
  k ^= k >> 27; k *= 0x94d049bb133111ebull;
  k ^= k >> 31;
  return k;
}
static int orc_pack(int64_t x, int64_t y, int64_t z, uint64_t* key) {
  const int64_t lim = 1 << 20;
  if (x < -lim || x >= lim || y < -lim || y >= lim || z < -lim || z >= lim) return 0;
  *key = ((uint64_t)(x + lim) << 42) | ((uint64_t)(y + lim) << 21) | (uint64_t)(z + lim);
  return 1;
}

int orc_neighbor_pairs(const int32_t* coords, int64_t n, int32_t* pair_dest, int32_t* pair_src,
                       int32_t* counts) {
  uint64_t cap = 64;
  while (cap < (uint64_t)(2 * n)) cap <<= 1;
  orc_slot* tab = (orc_slot*)malloc(sizeof(orc_slot) * cap);
  for (uint64_t i = 0; i < cap; ++i) { tab[i].key = ~0ull; tab[i].val = -1; }
  for (int64_t i = 0; i < n; ++i) {
    uint64_t key;
    if (!orc_pack(coords[i * 3], coords[i * 3 + 1], coords[i * 3 + 2], &key)) continue;
    uint64_t s = orc_mix(key) & (cap - 1);
    while (tab[s].key != ~0ull && tab[s].key != key) s = (s + 1) & (cap - 1);
    tab[s].key = key;
    tab[s].val = (int32_t)i; /* later duplicates overwrite */
  }
  for (int k = 0; k < 27; ++k) {
    const int dx = k / 9 - 1, dy = (k % 9) / 3 - 1, dz = k % 3 - 1;
    int32_t c = 0;
    for (int64_t i = 0; i < n; ++i) {
      uint64_t key;
      if (!orc_pack(coords[i * 3], coords[i * 3 + 1], coords[i * 3 + 2], &key)) continue;
      if (!orc_pack((int64_t)coords[i * 3] + dx, (int64_t)coords[i * 3 + 1] + dy,
                    (int64_t)coords[i * 3 + 2] + dz, &key))
        continue;
      uint64_t s = orc_mix(key) & (cap - 1);
      int32_t found = -1;
      while (tab[s].key != ~0ull) {
        if (tab[s].key == key) { found = tab[s].val; break; }
        s = (s + 1) & (cap - 1);
      }
      if (found >= 0) {
        pair_dest[(int64_t)k * n + c] = (int32_t)i;
        pair_src[(int64_t)k * n + c] = found;
        ++c;
      }
    }
    counts[k] = c;
  }
  free(tab);
  return 0;
}

/* SparseConv3d::forward (crate/runtime/trellis2_sparse.rs:197-243): for each
 * kernel offset k in 0..26, the neighbour pairs (dest i, src j) in ascending i
 * (the lists orc_neighbor_pairs builds), product[p, o] = sum_c feats[j, c] *
 * w27[k, o, c] (f32, c ascending), then out[i, :] += product[p, :]
 * (index_add); finally + bias.  feats [n, cin], w27 [27, cout, cin], bias
 * [cout] or NULL, out [n, cout]. */
int orc_sparse_conv3d(const int32_t* coords, int64_t n, const float* feats, int64_t cin,
                      const float* w27, int64_t cout, const float* bias, float* out) {
  int32_t* dest = (int32_t*)malloc(sizeof(int32_t) * (size_t)(27 * (n > 0 ? n : 1)));
  int32_t* src = (int32_t*)malloc(sizeof(int32_t) * (size_t)(27 * (n > 0 ? n : 1)));
  int32_t counts[27];
  if (!dest || !src) { free(dest); free(src); return 1; }
  orc_neighbor_pairs(coords, n, dest, src, counts);
  for (int64_t i = 0; i < n * cout; ++i) out[i] = 0.f;
  for (int k = 0; k < 27; ++k) {
    const int32_t* dk = dest + (int64_t)k * n;
    const int32_t* sk = src + (int64_t)k * n;
    const float* wk = w27 + (int64_t)k * cout * cin;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < counts[k]; ++p) {
      const float* x = feats + (int64_t)sk[p] * cin;
      float* o = out + (int64_t)dk[p] * cout;
      for (int64_t oc = 0; oc < cout; ++oc) {
        const float* w = wk + oc * cin;
        float acc = 0.f;
        for (int64_t c = 0; c < cin; ++c) acc += x[c] * w[c];
        o[oc] += acc;
      }
    }
  }
  if (bias)
    for (int64_t i = 0; i < n; ++i)
      for (int64_t oc = 0; oc < cout; ++oc) out[i * cout + oc] += bias[oc];
  free(dest);
  free(src);
  return 0;
}
