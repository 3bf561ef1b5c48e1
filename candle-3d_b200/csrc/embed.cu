// Embeddings and the per-step small linears:
//   l3d_timestep_embedding  sinusoidal tables (TRELLIS.2 cos-first, TripoSG
//                           sin-first) formed on the device;
//   l3d_linear_small        memory-bound GEMV for [B <= 16, K] x [N, K]^T with
//                           fused input/output activations, bias and addend
//                           (adaLN modulation vectors, timestep MLPs);
//   l3d_patch_embed         Conv2d(k = s = p) patch projection as an implicit
//                           GEMM with cls / register / position tokens fused.
#include "act.cuh"
#include "common.cuh"

namespace l3d {

// ------------------------------------------------------------- timestep table
template <typename TO>
__global__ void timestep_kernel(const float* __restrict__ t, int64_t tstride, int64_t B, int dim,
                                int order, float neg_log_period, TO* __restrict__ out,
                                int64_t obstride) {
  const int half = dim / 2;
  const int64_t total = B * int64_t(dim);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = i / dim;
    const int j = int(i - b * dim);
    TO* o = out + b * obstride;
    if (j >= 2 * half) {  // odd dim: zero pad
      o[j] = from_f<TO>(0.f);
      continue;
    }
    const int f = j % half;
    // freq = exp(neg_log_period * f / half) in f32 steps; exp evaluated in
    // double and rounded once.
    const float e = __fdiv_rn(__fmul_rn(neg_log_period, float(f)), float(half));
    const float freq = static_cast<float>(exp(static_cast<double>(e)));
    float arg = __fmul_rn(t[b * tstride], freq);
    const bool first = j < half;
    float sv, cv;
    if (order == 1) {
      // TripoSG: the argument vector is cast to the activation dtype before
      // sin/cos; the table is [sin, cos].
      arg = to_f(from_f<TO>(arg));
      sincosf(arg, &sv, &cv);
      o[j] = from_f<TO>(first ? sv : cv);
    } else {
      sincosf(arg, &sv, &cv);
      o[j] = from_f<TO>(first ? cv : sv);
    }
  }
}

// -------------------------------------------------------------- small linear
constexpr int kLsBlock = 256;
constexpr int kLsMaxB = 16;

struct LinearSmallParams {
  const void* x; int xdt; int64_t xbase, xsb;   // [B, K]
  const void* w; int wdt; int64_t wbase, wsn;   // [N, K]
  ChanVec bias, addend;
  void* y; int ydt; int64_t ybase, ysb;         // [B, N]
  int64_t B, N, K;
  int act_in, act_out;
};

__device__ __forceinline__ float ld_any(const void* p, int dt, int64_t i) {
  if (dt == L3D_F32) return static_cast<const float*>(p)[i];
  if (dt == L3D_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void st_any(void* p, int dt, int64_t i, float v) {
  if (dt == L3D_F32) static_cast<float*>(p)[i] = v;
  else if (dt == L3D_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

// One warp per output feature n; x (after act_in) staged in shared memory as
// f32 for all batches of this block's batch chunk.  W is streamed once with
// 16-byte loads.
template <typename TW, int VEC>
__global__ void __launch_bounds__(kLsBlock) linear_small_kernel(const LinearSmallParams p,
                                                                int64_t b0, int nb) {
  extern __shared__ float xs[];  // [nb][K]
  for (int64_t i = threadIdx.x; i < int64_t(nb) * p.K; i += blockDim.x) {
    const int64_t b = i / p.K, k = i - b * p.K;
    xs[i] = act_dyn(p.act_in, ld_any(p.x, p.xdt, p.xbase + (b0 + b) * p.xsb + k));
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t n = warp; n < p.N; n += nwarps) {
    float acc[kLsMaxB];
#pragma unroll
    for (int b = 0; b < kLsMaxB; ++b) acc[b] = 0.f;
    const TW* wr = static_cast<const TW*>(p.w) + p.wbase + n * p.wsn;
    for (int64_t k = int64_t(lane) * VEC; k < p.K; k += 32 * VEC) {
      float wv[VEC];
      load_reuse<TW, VEC>(wr + k, wv);
#pragma unroll
      for (int b = 0; b < kLsMaxB; ++b) {
        if (b < nb) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[b] += wv[e] * xs[b * p.K + k + e];
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kLsMaxB; ++b) {
      if (b >= nb) break;
      float v = acc[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) {
        if (p.bias.ptr) v += ld_any(p.bias.ptr, p.bias.dtype, n);
        if (p.addend.ptr) v += ld_any(p.addend.ptr, p.addend.dtype, n);
        v = act_dyn(p.act_out, v);
        st_any(p.y, p.ydt, p.ybase + (b0 + b) * p.ysb + n, v);
      }
    }
  }
}

// -------------------------------------------------------------- patch embed
// Implicit-GEMM tile: 64 tokens x 64 channels per CTA, K (= Cin*p*p) in steps
// of 16 staged through shared memory; each thread owns a 4 x 4 output block.
constexpr int kPeTM = 64, kPeTN = 64, kPeTK = 16;

struct PatchParams {
  const void* pix; int64_t BS, Cin, H, W;      // [BS, Cin, H, W]
  const void* w;                               // [C, Cin*p*p]
  const void* bias;                            // [C]
  const void* pos;                             // [1 + np, C]
  const void* cls;                             // [C]
  const void* reg;                             // [R, C]
  void* out;                                   // [BS, 1 + R + np, C]
  int64_t C, R, np, pw, K;
  int p;
};

template <typename T>
__global__ void __launch_bounds__(256) patch_gemm_kernel(const PatchParams p) {
  __shared__ float As[kPeTK][kPeTM + 4];
  __shared__ float Bs[kPeTK][kPeTN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = int64_t(blockIdx.x) * kPeTM;   // token tile
  const int64_t n0 = int64_t(blockIdx.y) * kPeTN;   // channel tile
  const int64_t M = p.BS * p.np;
  const T* pix = static_cast<const T*>(p.pix);
  const T* w = static_cast<const T*>(p.w);
  const int pp = p.p * p.p;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.K; k0 += kPeTK) {
    // Stage A (im2col on the fly): 64 tokens x 16 k.
    for (int i = threadIdx.x; i < kPeTM * kPeTK; i += 256) {
      const int mm = i / kPeTK, kk = i % kPeTK;
      const int64_t m = m0 + mm, k = k0 + kk;
      float v = 0.f;
      if (m < M && k < p.K) {
        const int64_t bs = m / p.np, t = m - bs * p.np;
        const int64_t py = t / p.pw, px = t - py * p.pw;
        const int64_t c = k / pp;
        const int r = int(k - c * pp);
        const int ky = r / p.p, kx = r - ky * p.p;
        v = to_f(pix[((bs * p.Cin + c) * p.H + py * p.p + ky) * p.W + px * p.p + kx]);
      }
      As[kk][mm] = v;
    }
    for (int i = threadIdx.x; i < kPeTN * kPeTK; i += 256) {
      const int nn = i / kPeTK, kk = i % kPeTK;
      const int64_t n = n0 + nn, k = k0 + kk;
      Bs[kk][nn] = (n < p.C && k < p.K) ? to_f(w[n * p.K + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kPeTK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
  const T* bias = static_cast<const T*>(p.bias);
  const T* pos = static_cast<const T*>(p.pos);
  T* out = static_cast<T*>(p.out);
  const int64_t ntok = 1 + p.R + p.np;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
    const int64_t bs = m / p.np, t = m - bs * p.np;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n >= p.C) continue;
      float v = acc[i][j] + to_f(bias[n]);
      v = v + to_f(pos[(1 + t) * p.C + n]);
      out[(bs * ntok + 1 + p.R + t) * p.C + n] = from_f<T>(v);
    }
  }
}

template <typename T>
__global__ void patch_special_kernel(const PatchParams p) {
  // out[:, 0] = cls + pos[0]; out[:, 1 + r] = reg[r].
  const int64_t ntok = 1 + p.R + p.np;
  const int64_t total = p.BS * (1 + p.R) * p.C;
  const T* cls = static_cast<const T*>(p.cls);
  const T* reg = static_cast<const T*>(p.reg);
  const T* pos = static_cast<const T*>(p.pos);
  T* out = static_cast<T*>(p.out);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = i % p.C;
    const int64_t s = (i / p.C) % (1 + p.R);
    const int64_t bs = i / (p.C * (1 + p.R));
    float v = s == 0 ? to_f(cls[n]) + to_f(pos[n]) : to_f(reg[(s - 1) * p.C + n]);
    out[(bs * ntok + s) * p.C + n] = from_f<T>(v);
  }
}

static bool contiguous(const l3d_tensor* t) {
  int64_t st = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    if (t->dims[i] > 1 && t->strides[i] != st) return false;
    st *= t->dims[i];
  }
  return true;
}

}  // namespace l3d

using namespace l3d;

extern "C" int l3d_timestep_embedding(const l3d_tensor* t, int dim, int order, float max_period,
                                      const l3d_tensor* out, l3d_stream stream) {
  const char* op = "l3d_timestep_embedding";
  if (!t || !out || no_data(t) || no_data(out)) return fail(L3D_E_NULL, "%s: t and out required", op);
  if (t->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: t must be F32", op);
  if (!is_float_dtype(out->dtype)) return fail(L3D_E_DTYPE, "%s: out must be a float dtype", op);
  if (order != 0 && order != 1) return fail(L3D_E_UNSUPPORTED, "%s: order must be 0 or 1", op);
  if (dim < 2) return fail(L3D_E_SHAPE, "%s: dim must be >= 2", op);
  if (!(max_period > 0.f)) return fail(L3D_E_SHAPE, "%s: max_period must be positive", op);
  const int64_t B = numel(t);
  if (t->ndim > 1) return fail(L3D_E_SHAPE, "%s: t must be [B]", op);
  if (out->ndim != 2 || out->dims[0] != B || out->dims[1] != dim)
    return fail(L3D_E_SHAPE, "%s: out must be [B, dim]", op);
  if (dim > 1 && out->strides[1] != 1) return fail(L3D_E_ALIGN, "%s: out rows must be contiguous", op);
  if (B == 0) return L3D_OK;
  // -ln(max_period) in f32 (TRELLIS takes the f64 log and casts; TripoSG takes
  // the f32 log; both round the same real number once).
  const float nlp = -static_cast<float>(log(static_cast<double>(max_period)));
  const int64_t total = B * dim;
  const int blocks = int((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
  const float* tp = static_cast<const float*>(t->data) + t->offset;
  const int64_t ts = t->ndim == 1 ? t->strides[0] : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  L3D_DISPATCH_FLOAT(out->dtype, TO, {
    timestep_kernel<TO><<<blocks, 256, 0, s>>>(tp, ts, B, dim, order, nlp,
                                               static_cast<TO*>(out->data) + out->offset,
                                               out->strides[0]);
  });
  return check_launch(op);
}

extern "C" int l3d_linear_small(const l3d_tensor* x, const l3d_tensor* w, const l3d_tensor* bias,
                                const l3d_tensor* addend, int act_in, int act_out,
                                const l3d_tensor* y, l3d_stream stream) {
  const char* op = "l3d_linear_small";
  if (!x || !w || !y || no_data(x) || no_data(w) || no_data(y))
    return fail(L3D_E_NULL, "%s: x, w and y are required", op);
  if (!is_float_dtype(x->dtype) || !is_float_dtype(w->dtype) || !is_float_dtype(y->dtype))
    return fail(L3D_E_DTYPE, "%s: float dtypes required", op);
  if (act_in < 0 || act_in > 3 || act_out < 0 || act_out > 3)
    return fail(L3D_E_UNSUPPORTED, "%s: unknown activation code", op);
  if (x->ndim != 2 || w->ndim != 2 || y->ndim != 2)
    return fail(L3D_E_SHAPE, "%s: x [B, K], w [N, K], y [B, N] required", op);
  LinearSmallParams p{};
  p.B = x->dims[0]; p.K = x->dims[1]; p.N = w->dims[0];
  if (w->dims[1] != p.K || y->dims[0] != p.B || y->dims[1] != p.N)
    return fail(L3D_E_SHAPE, "%s: shape mismatch", op);
  if ((p.K > 1 && (x->strides[1] != 1 || w->strides[1] != 1)) || (p.N > 1 && y->strides[1] != 1))
    return fail(L3D_E_ALIGN, "%s: rows must be contiguous", op);
  bool al = true;
  int rc;
  if ((rc = make_chanvec(bias, "bias", p.N, 1, &p.bias, &al))) return rc;
  if ((rc = make_chanvec(addend, "addend", p.N, 1, &p.addend, &al))) return rc;
  if (p.B == 0 || p.N == 0) return L3D_OK;
  p.x = x->data; p.xdt = x->dtype; p.xbase = x->offset; p.xsb = x->strides[0];
  p.w = w->data; p.wdt = w->dtype; p.wbase = w->offset; p.wsn = w->strides[0];
  p.y = y->data; p.ydt = y->dtype; p.ybase = y->offset; p.ysb = y->strides[0];
  p.act_in = act_in; p.act_out = act_out;
  const int es = dtype_size(w->dtype);
  const int vec = 16 / es;
  const bool v = (p.K % vec == 0) && ((p.wsn * es) % 16 == 0) &&
                 ((reinterpret_cast<uintptr_t>(w->data) + w->offset * es) % 16 == 0);
  // Batches per block limited by the shared-memory staging (48 KB).
  int64_t nbmax = (48 * 1024 / 4) / (p.K > 0 ? p.K : 1);
  if (nbmax > kLsMaxB) nbmax = kLsMaxB;
  if (nbmax < 1) return fail(L3D_E_UNSUPPORTED, "%s: K = %lld too large", op, (long long)p.K);
  int64_t blocks = (p.N + 7) / 8;
  const int64_t cap = int64_t(sm_count()) * 4;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t b0 = 0; b0 < p.B; b0 += nbmax) {
    const int nb = int(p.B - b0 < nbmax ? p.B - b0 : nbmax);
    const size_t smem = size_t(nb) * p.K * sizeof(float);
    L3D_DISPATCH_FLOAT(w->dtype, TW, {
      if (v) linear_small_kernel<TW, Vec16<TW>::N><<<int(blocks), kLsBlock, smem, s>>>(p, b0, nb);
      else linear_small_kernel<TW, 1><<<int(blocks), kLsBlock, smem, s>>>(p, b0, nb);
    });
  }
  return check_launch(op);
}

extern "C" int l3d_patch_embed(const l3d_tensor* pixels, const l3d_tensor* weight,
                               const l3d_tensor* bias, const l3d_tensor* pos,
                               const l3d_tensor* cls, const l3d_tensor* reg, int patch,
                               const l3d_tensor* out, l3d_stream stream) {
  const char* op = "l3d_patch_embed";
  const l3d_tensor* req[] = {pixels, weight, bias, pos, cls, out};
  for (const l3d_tensor* t : req)
    if (!t || no_data(t)) return fail(L3D_E_NULL, "%s: pixels, weight, bias, pos, cls, out required", op);
  const int dt = pixels->dtype;
  if (dt != L3D_F32 && dt != L3D_BF16) return fail(L3D_E_DTYPE, "%s: F32 or BF16 required", op);
  for (const l3d_tensor* t : req)
    if (t->dtype != dt) return fail(L3D_E_DTYPE, "%s: all tensors must share one dtype", op);
  if (reg && reg->dtype != dt) return fail(L3D_E_DTYPE, "%s: reg dtype mismatch", op);
  for (const l3d_tensor* t : req)
    if (!contiguous(t) || t->offset != 0)
      return fail(L3D_E_ALIGN, "%s: tensors must be contiguous with zero offset", op);
  if (patch <= 0) return fail(L3D_E_SHAPE, "%s: patch must be positive", op);
  if (pixels->ndim != 4 || weight->ndim != 4 || out->ndim != 3)
    return fail(L3D_E_SHAPE, "%s: pixels [BS,Cin,H,W], weight [C,Cin,p,p], out [BS,T,C]", op);
  PatchParams p{};
  p.BS = pixels->dims[0]; p.Cin = pixels->dims[1]; p.H = pixels->dims[2]; p.W = pixels->dims[3];
  p.C = weight->dims[0]; p.p = patch;
  if (weight->dims[1] != p.Cin || weight->dims[2] != patch || weight->dims[3] != patch)
    return fail(L3D_E_SHAPE, "%s: weight must be [C, Cin, p, p]", op);
  if (p.H % patch || p.W % patch)
    return fail(L3D_E_SHAPE, "%s: image size must be divisible by patch size", op);
  p.pw = p.W / patch;
  p.np = (p.H / patch) * p.pw;
  p.R = reg ? (reg->ndim == 2 ? reg->dims[0] : 0) : 0;
  if (reg && (reg->ndim != 2 || reg->dims[1] != p.C)) return fail(L3D_E_SHAPE, "%s: reg [R, C]", op);
  if (numel(bias) != p.C || numel(cls) != p.C) return fail(L3D_E_SHAPE, "%s: bias/cls must be [C]", op);
  if (numel(pos) != (1 + p.np) * p.C) return fail(L3D_E_SHAPE, "%s: pos must be [1 + np, C]", op);
  if (out->dims[0] != p.BS || out->dims[1] != 1 + p.R + p.np || out->dims[2] != p.C)
    return fail(L3D_E_SHAPE, "%s: out must be [BS, 1 + R + np, C]", op);
  p.K = p.Cin * patch * patch;
  p.pix = pixels->data; p.w = weight->data; p.bias = bias->data; p.pos = pos->data;
  p.cls = cls->data; p.reg = reg ? reg->data : nullptr; p.out = out->data;
  if (p.BS == 0) return L3D_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned((p.BS * p.np + kPeTM - 1) / kPeTM), unsigned((p.C + kPeTN - 1) / kPeTN));
  const int64_t sp = p.BS * (1 + p.R) * p.C;
  const int sblocks = int((sp + 255) / 256 < 1024 ? (sp + 255) / 256 : 1024);
  if (dt == L3D_F32) {
    patch_gemm_kernel<float><<<grid, 256, 0, s>>>(p);
    patch_special_kernel<float><<<sblocks, 256, 0, s>>>(p);
  } else {
    patch_gemm_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(p);
    patch_special_kernel<__nv_bfloat16><<<sblocks, 256, 0, s>>>(p);
  }
  return check_launch(op);
}
