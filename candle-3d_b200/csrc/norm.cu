// Row-normalisation family: LayerNorm / RMSNorm fused with affine, adaLN
// modulation, gates and residuals.  One kernel template covers
//   l3d_layer_norm, l3d_layer_norm_modulate, l3d_gated_residual,
//   l3d_layerscale_residual, l3d_residual_layer_norm_modulate,
//   l3d_rms_norm_heads.
//
// Each row of C elements is owned by a group of G threads (G in 8..256); each
// thread keeps up to NV 16-byte vectors of the row in registers, so the row is
// read from HBM once and written once, with the reductions done by warp
// shuffles (G <= 32) or shuffles plus one shared-memory exchange (G > 32).
#include "common.cuh"
#include "ring.cuh"

namespace l3d {

enum NormKind { NORM_NONE = 0, NORM_LAYER = 1, NORM_RMS = 2 };

struct RowNormParams {
  int64_t rows;
  int64_t C;
  int64_t rows_per_batch;  // row -> batch index for per-batch vectors
  RowMap xm, hm, rm, ym;   // x, h (residual branch), r_out, y
  const void* x;
  const void* h;           // null: no residual branch
  void* r_out;             // null: residual sum not stored
  void* y;
  ChanVec g1;              // gate on h (residual branch)
  ChanVec w, b;            // affine
  ChanVec scale, shift;    // adaLN modulation
  ChanVec g2;              // gate on the normalised branch
  int add_input;           // y += r after the gate
  int norm;                // NormKind
  float eps;
  int nbatch;              // batches of the staged coefficients (1 = broadcast)
};

constexpr int kBlock = 256;
constexpr int64_t kWaves = 2;  // grid cap in resident waves (grid-stride beyond)

template <int G>
__device__ __forceinline__ float group_sum(float v, float* red) {
  if constexpr (G <= 32) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  } else {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    constexpr int W = G / 32;  // warps per row group
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int grp = threadIdx.x / G;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) s += red[grp * W + i];
    __syncthreads();
    return s;
  }
}

// A row vector kept in registers in its storage format (one 16-byte pack, or
// one float on the scalar path): half the registers of unpacked f32 for
// 16-bit activations, so more rows are in flight per SM.
template <typename T, int VEC> struct Packed { using S = uint4; };
template <typename T> struct Packed<T, 1> { using S = float; };

template <typename T, int VEC>
__device__ __forceinline__ typename Packed<T, VEC>::S ld_packed(const T* p) {
  if constexpr (VEC == 1) return to_f(p[0]);
  else return ld_act_raw(reinterpret_cast<const uint4*>(p));
}
template <typename T, int VEC>
__device__ __forceinline__ void unpack_v(const typename Packed<T, VEC>::S& s, float (&f)[VEC]) {
  if constexpr (VEC == 1) f[0] = s;
  else unpack(s, f, T());
}
// Pack (rounding to the activation dtype).
template <typename T, int VEC>
__device__ __forceinline__ typename Packed<T, VEC>::S pack_v(const float (&f)[VEC]) {
  if constexpr (VEC == 1) return to_f(from_f<T>(f[0]));
  else return pack(f, T());
}
template <typename T, int VEC>
__device__ __forceinline__ void st_packed(T* p, const typename Packed<T, VEC>::S& s) {
  if constexpr (VEC == 1) p[0] = from_f<T>(s);
  else st_act_raw(reinterpret_cast<uint4*>(p), s);
}

template <int VEC>
__device__ __forceinline__ void ld_smem_vec(const float* p, float (&f)[VEC]) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(p + i);
      f[i] = t.x; f[i + 1] = t.y; f[i + 2] = t.z; f[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = p[i];
  }
}

// RES: the residual branch is present (x and h both held in registers).
// STG: the per-channel vectors are folded once per block into shared memory,
//   A = w (1 + scale), Bc = b (1 + scale) + shift (and the output gate), so
//   the output costs one FFMA per element instead of several vector loads.
template <typename T, int VEC, int G, int kNV, bool RES, bool STG>
__global__ void __launch_bounds__(kBlock, (RES || kNV > 4) ? 2 : 3)
    rownorm_kernel(const RowNormParams p) {
  using S = typename Packed<T, VEC>::S;
  constexpr int P = VEC > 1 ? VEC / 2 : 1;  // float pairs per vector
  __shared__ float red[kBlock / 32];
  extern __shared__ float coef[];  // STG: [nbatch, C] A, [nbatch, C] Bc, [nbatch, C] gate
  if constexpr (STG) {
    const int64_t nc = int64_t(p.nbatch) * p.C;
    for (int64_t i = threadIdx.x; i < nc; i += blockDim.x) {
      const int64_t bb = i / p.C, c = i - bb * p.C;
      float w[1] = {1.f}, bi[1] = {0.f}, sc[1] = {0.f}, sh[1] = {0.f};
      if (p.w.ptr) load_chan<1>(p.w, 0, c, w);
      if (p.b.ptr) load_chan<1>(p.b, 0, c, bi);
      if (p.scale.ptr) load_chan<1>(p.scale, bb, c, sc);
      if (p.shift.ptr) load_chan<1>(p.shift, bb, c, sh);
      const float s1 = 1.f + sc[0];
      coef[i] = w[0] * s1;
      coef[nc + i] = bi[0] * s1 + sh[0];
      if (p.g2.ptr) {
        float g[1];
        load_chan<1>(p.g2, bb, c, g);
        coef[2 * nc + i] = g[0];
      }
    }
    __syncthreads();
  }
  constexpr int RPB = kBlock / G;  // rows per block
  const int tid = threadIdx.x % G;
  const int64_t nvec = p.C / VEC;
  const int64_t stride = int64_t(gridDim.x) * RPB;
  // Load row r's vectors of this thread (zeros past the row / past the end).
  auto load_x = [&](S (&dst)[kNV], int64_t r) {
    const bool ok = r < p.rows;
    const T* xr = static_cast<const T*>(p.x) + (ok ? row_offset(p.xm, r) : 0);
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      const int64_t vi = tid + int64_t(i) * G;
      if (ok && vi < nvec) dst[i] = ld_packed<T, VEC>(xr + vi * VEC);
      else dst[i] = S{};  // all-zero bits: 0.0 in every float dtype
    }
  };
  // Without a residual branch the next row of this thread group is prefetched
  // while the current one is reduced and written, so loads stay in flight.
  S pf[RES ? 1 : kNV];
  if constexpr (!RES) load_x(pf, int64_t(blockIdx.x) * RPB + threadIdx.x / G);
  // Grid-stride over groups of RPB rows; the trip count is uniform per block
  // (the cross-warp reductions synchronise the whole block).
  for (int64_t row0 = int64_t(blockIdx.x) * RPB; row0 < p.rows; row0 += stride) {
  const int64_t row = row0 + threadIdx.x / G;
  const bool valid = row < p.rows;
  const int64_t b = valid ? row / p.rows_per_batch : 0;

  S v[kNV];
  if constexpr (RES) {
    load_x(v, row);
  } else {
#pragma unroll
    for (int i = 0; i < kNV; ++i) v[i] = pf[i];
    if (row0 + stride < p.rows) load_x(pf, row + stride);
  }
  // Residual branch: r = x + g1 * h, rounded to the activation dtype exactly as
  // it is stored, so the norm sees the values a later reader of r sees.
  if constexpr (RES) {
    const T* hr = static_cast<const T*>(p.h) + (valid ? row_offset(p.hm, row) : 0);
    T* rr = p.r_out ? static_cast<T*>(p.r_out) + (valid ? row_offset(p.rm, row) : 0) : nullptr;
    S hp[kNV];
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      const int64_t vi = tid + int64_t(i) * G;
      if (valid && vi < nvec) hp[i] = ld_packed<T, VEC>(hr + vi * VEC);
    }
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      const int64_t vi = tid + int64_t(i) * G;
      if (valid && vi < nvec) {
        if constexpr (VEC == 1) {
          float a = v[i], hv = hp[i];
          if (p.g1.ptr) {
            float g[1];
            load_chan<1>(p.g1, b, vi, g);
            hv = hv * g[0];
          }
          float o[1] = {a + hv};
          v[i] = pack_v<T, 1>(o);
        } else {
          float2 a[P], hv[P];
          unpack2(v[i], a, T());
          unpack2(hp[i], hv, T());
          if (p.g1.ptr) {
            float g[VEC];
            load_chan<VEC>(p.g1, b, vi * VEC, g);
#pragma unroll
            for (int k = 0; k < P; ++k) a[k] = fma2(hv[k], make_float2(g[2 * k], g[2 * k + 1]), a[k]);
          } else {
#pragma unroll
            for (int k = 0; k < P; ++k) a[k] = add2(a[k], hv[k]);
          }
          v[i] = pack2(a, T());
        }
        if (rr) st_packed<T, VEC>(rr + vi * VEC, v[i]);
      }
    }
  }

  // Statistics: LayerNorm shifted moments in one pass (vector path, row within
  // one warp) or mean then centred sum of squares (two passes); RMSNorm sum of
  // squares.  Padding vectors are zero.
  float inv = 1.f, mean = 0.f;
  bool stats_done = false;
  if constexpr (G <= 32 && VEC > 1) {
    if (p.norm == NORM_LAYER) {
      stats_done = true;
      // One pass of shifted moments: with K the row's first element (from the
      // group's first thread), S1 = sum(x - K), S2 = sum((x - K)^2);
      // mean = K + S1 / C, var = S2 / C - (S1 / C)^2.  K lies within the row's
      // range, so the subtraction loses no more than the centred two-pass form
      // for ordinary rows.
      float2 a0[P];
      unpack2(v[0], a0, T());
      const int lane = threadIdx.x & 31;
      const float K = __shfl_sync(0xffffffffu, a0[0].x, lane & ~(G - 1));
      const float2 nk = f2(-K);
      float2 s1 = f2(0.f), s2 = f2(0.f);
#pragma unroll
      for (int i = 0; i < kNV; ++i) {
        const int64_t vi = tid + int64_t(i) * G;
        if (vi < nvec) {
          float2 a[P];
          unpack2(v[i], a, T());
#pragma unroll
          for (int k = 0; k < P; ++k) {
            const float2 d = add2(a[k], nk);
            s1 = add2(s1, d);
            s2 = fma2(d, d, s2);
          }
        }
      }
      float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
#pragma unroll
      for (int o = (G < 32 ? G : 32) / 2; o > 0; o >>= 1) {
        t1 += __shfl_xor_sync(0xffffffffu, t1, o);
        t2 += __shfl_xor_sync(0xffffffffu, t2, o);
      }
      const float m1 = t1 / float(p.C);
      mean = K + m1;
      inv = 1.f / sqrtf(fmaxf(t2 / float(p.C) - m1 * m1, 0.f) + p.eps);
    }
  }
  if (stats_done) {
  } else if (p.norm == NORM_LAYER) {
    float2 acc = f2(0.f);
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      if constexpr (VEC == 1) {
        acc.x += v[i];
      } else {
        float2 a[P];
        unpack2(v[i], a, T());
#pragma unroll
        for (int k = 0; k < P; ++k) acc = add2(acc, a[k]);
      }
    }
    const float s = group_sum<G>(acc.x + acc.y, red);
    mean = s / float(p.C);
    const float2 nm = f2(-mean);
    acc = f2(0.f);
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      const int64_t vi = tid + int64_t(i) * G;
      if (vi < nvec) {
        if constexpr (VEC == 1) {
          const float d = v[i] - mean;
          acc.x += d * d;
        } else {
          float2 a[P];
          unpack2(v[i], a, T());
#pragma unroll
          for (int k = 0; k < P; ++k) {
            const float2 d = add2(a[k], nm);
            acc = fma2(d, d, acc);
          }
        }
      }
    }
    const float ss = group_sum<G>(acc.x + acc.y, red);
    inv = 1.f / sqrtf(ss / float(p.C) + p.eps);
  } else if (p.norm == NORM_RMS) {
    float2 acc = f2(0.f);
#pragma unroll
    for (int i = 0; i < kNV; ++i) {
      if constexpr (VEC == 1) {
        acc.x += v[i] * v[i];
      } else {
        float2 a[P];
        unpack2(v[i], a, T());
#pragma unroll
        for (int k = 0; k < P; ++k) acc = fma2(a[k], a[k], acc);
      }
    }
    const float ss = group_sum<G>(acc.x + acc.y, red);
    inv = 1.f / sqrtf(ss / float(p.C) + p.eps);
  }
  if (!valid) continue;

  T* yr = static_cast<T*>(p.y) + row_offset(p.ym, row);
  const float2 nm = f2(-mean), inv2 = f2(inv);
#pragma unroll
  for (int i = 0; i < kNV; ++i) {
    const int64_t vi = tid + int64_t(i) * G;
    if (vi >= nvec) continue;
    if (p.norm == NORM_NONE) {
      st_packed<T, VEC>(yr + vi * VEC, v[i]);
      continue;
    }
    const int64_t c0 = vi * VEC;
    if constexpr (STG && VEC > 1) {
      // Folded per-channel coefficients: n * A + Bc [then gate, + input].
      float2 a[P], o[P], fa[P], fb[P];
      unpack2(v[i], a, T());
#pragma unroll
      for (int k = 0; k < P; ++k) o[k] = mul2(add2(a[k], nm), inv2);
      const float* ca = coef + (p.nbatch > 1 ? b : 0) * p.C + c0;
      const float* cb = ca + p.nbatch * p.C;
      ld_pairs<P>(ca, fa);
      ld_pairs<P>(cb, fb);
#pragma unroll
      for (int k = 0; k < P; ++k) o[k] = fma2(o[k], fa[k], fb[k]);
      if (p.g2.ptr) {
        ld_pairs<P>(cb + p.nbatch * p.C, fa);
#pragma unroll
        for (int k = 0; k < P; ++k) o[k] = mul2(fa[k], o[k]);
      }
      if (p.add_input) {
#pragma unroll
        for (int k = 0; k < P; ++k) o[k] = add2(o[k], a[k]);
      }
      st_packed<T, VEC>(yr + c0, pack2(o, T()));
      continue;
    }
    float a[VEC], o[VEC], t[VEC];
    unpack_v<T, VEC>(v[i], a);
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = (a[e] - mean) * inv;
    if constexpr (STG) {
      const float* ca = coef + (p.nbatch > 1 ? b : 0) * p.C + c0;
      const float* cb = ca + p.nbatch * p.C;
      float fa[VEC], fb[VEC];
      ld_smem_vec<VEC>(ca, fa);
      ld_smem_vec<VEC>(cb, fb);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] * fa[e] + fb[e];
      if (p.g2.ptr) {
        ld_smem_vec<VEC>(cb + p.nbatch * p.C, t);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = t[e] * o[e];
      }
      if (p.add_input) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = o[e] + a[e];
      }
      st_packed<T, VEC>(yr + c0, pack_v<T, VEC>(o));
      continue;
    }
    if (p.w.ptr) {
      load_chan<VEC>(p.w, 0, c0, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] * t[e];
    }
    if (p.b.ptr) {
      load_chan<VEC>(p.b, 0, c0, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] + t[e];
    }
    if (p.scale.ptr) {
      load_chan<VEC>(p.scale, b, c0, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] * (1.f + t[e]);
    }
    if (p.shift.ptr) {
      load_chan<VEC>(p.shift, b, c0, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] + t[e];
    }
    if (p.g2.ptr) {
      load_chan<VEC>(p.g2, b, c0, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = t[e] * o[e];
    }
    if (p.add_input) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = o[e] + a[e];
    }
    st_packed<T, VEC>(yr + c0, pack_v<T, VEC>(o));
  }
  }
}

// ------------------------------------------------------------ ring variant
// Rows of 2-8 KB without a residual branch, long inputs: one CTA per SM streams
// its contiguous block of rows through a ring of shared-memory slots filled by
// bulk copies (cp.async.bulk, one per row, issued by eight producer lanes of
// warp 0, so the rows in flight per SM are not held in registers); consumer
// warps each take R rows at a time: copy them from their slots into
// registers, release the slots, reduce with shuffles and store the
// normalised, modulated rows directly.  The arithmetic and its order are
// those of the register kernel above when it also gives a row one warp
// (G = 32, e.g. 2048 bf16 elements), so both give identical bits there.  Every mbarrier wait is bounded; on expiry the block
// records status 5 in g_norm_status, waits (bounded) for the copies it
// issued and returns.
constexpr int kRingProducers = 8;
constexpr int kRingMaxSlots = 96;
constexpr size_t kRingSmem = 200 * 1024;  // coefficients + slots + barriers
__device__ int g_norm_status;

struct RingCfg {
  int nslot;             // multiple of kRingProducers and of the consumer warps
  uint32_t row_bytes;    // C * element size (a multiple of 16)
  size_t coef_bytes;     // 128-aligned
  uint64_t wait_ns;
};

// SIMPLE: LayerNorm with one set of per-channel coefficients, no output gate,
// no added input (the common case, with the branches compiled out).
template <typename T, int NV, int NW, int R, bool SIMPLE>
__global__ void __launch_bounds__(32 * (NW + 1), 1)
    rowring_kernel(const RowNormParams p, const RingCfg rc) {
  constexpr int VEC = 16 / int(sizeof(T));
  constexpr int P = VEC / 2;
  extern __shared__ __align__(128) unsigned char ring_smem[];
  const int64_t C = p.C;
  const int64_t nc = int64_t(p.nbatch) * C;
  float* coef = reinterpret_cast<float*>(ring_smem);  // A [nc], Bc [nc] (, gate [nc])
  unsigned char* slots = ring_smem + rc.coef_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(slots + size_t(rc.nslot) * rc.row_bytes);
  uint64_t* empty = full + rc.nslot;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + rc.nslot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < rc.nslot; ++s) {
      ring_bar_init(&full[s], 1);
      ring_bar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    ring_init_fence();
  }
  __syncthreads();
  const int64_t per = (p.rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = int64_t(blockIdx.x) * per;
  const int64_t n = r0 < p.rows ? (p.rows - r0 < per ? p.rows - r0 : per) : 0;
  // Producer lane L issues rows L, L + 8, ...; row k lives in slot k % nslot,
  // so lane L alone fills the slots s = L (mod 8).
  int64_t last = -1;  // the last row this producer lane issued
  auto issue = [&](int64_t k) {
    const int s = int(k % rc.nslot);
    const T* src = static_cast<const T*>(p.x) + row_offset(p.xm, r0 + k);
    ring_load(slots + size_t(s) * rc.row_bytes, src, rc.row_bytes, &full[s]);
    last = k;
  };
  const int64_t first = n < rc.nslot ? n : rc.nslot;
  if (warp == 0 && lane < kRingProducers)
    for (int64_t k = lane; k < first; k += kRingProducers) issue(k);
  // The coefficients are folded while the first rows are in flight.
  for (int64_t i = threadIdx.x; i < nc; i += blockDim.x) {
    const int64_t bb = i / C, c = i - bb * C;
    float w[1] = {1.f}, bi[1] = {0.f}, sc[1] = {0.f}, sh[1] = {0.f};
    if (p.w.ptr) load_chan<1>(p.w, 0, c, w);
    if (p.b.ptr) load_chan<1>(p.b, 0, c, bi);
    if (p.scale.ptr) load_chan<1>(p.scale, bb, c, sc);
    if (p.shift.ptr) load_chan<1>(p.shift, bb, c, sh);
    const float s1 = 1.f + sc[0];
    coef[i] = w[0] * s1;
    coef[nc + i] = bi[0] * s1 + sh[0];
    if (p.g2.ptr) {
      float g[1];
      load_chan<1>(p.g2, bb, c, g);
      coef[2 * nc + i] = g[0];
    }
  }
  __syncthreads();
  const int64_t nvec = C / VEC;
  if (warp == 0) {
    if (lane < kRingProducers) {
      int64_t k = lane;
      while (k < first) k += kRingProducers;
      for (; k < n && !*abort_flag; k += kRingProducers) {
        const int s = int(k % rc.nslot);
        const uint32_t u = uint32_t(k / rc.nslot);  // >= 1: the slot's previous row is k - nslot
        if (!ring_wait(&empty[s], (u - 1) & 1u, abort_flag, rc.wait_ns, false, &g_norm_status)) break;
        issue(k);
      }
    }
  } else {
    // Consumer warp w takes R consecutive rows at a time, k = R (w - 1) +
    // R NW m: they share the coefficient loads of the output pass, and their
    // reductions interleave.
    for (int64_t k = int64_t(R) * (warp - 1); k < n; k += int64_t(R) * NW) {
      const int nr = n - k < R ? int(n - k) : R;  // rows of this step (the last may be short)
      uint4 v[R][NV];
      bool ok = true;
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (q >= nr) {
#pragma unroll
          for (int i = 0; i < NV; ++i) v[q][i] = make_uint4(0, 0, 0, 0);
          continue;
        }
        const int s = int((k + q) % rc.nslot);
        const uint32_t u = uint32_t((k + q) / rc.nslot);
        if (!ring_wait(&full[s], u & 1u, abort_flag, rc.wait_ns, false, &g_norm_status)) {
          ok = false;
          break;
        }
        const uint4* src = reinterpret_cast<const uint4*>(slots + size_t(s) * rc.row_bytes);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int64_t vi = lane + 32 * i;
          v[q][i] = vi < nvec ? src[vi] : make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        if (lane == 0) ring_arrive(&empty[s]);
      }
      if (!ok) break;
      float mean[R], inv[R];
      if (SIMPLE || p.norm == NORM_LAYER) {
        // Shifted one-pass moments (shift = the row's first element), as in
        // rownorm_kernel.
        float K[R];
        float2 s1[R], s2[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
          float2 a0[P];
          unpack2(v[q][0], a0, T());
          K[q] = __shfl_sync(0xffffffffu, a0[0].x, 0);
          s1[q] = f2(0.f);
          s2[q] = f2(0.f);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          if (lane + 32 * i < nvec) {
#pragma unroll
            for (int q = 0; q < R; ++q) {
              float2 a[P];
              unpack2(v[q][i], a, T());
              const float2 nk = f2(-K[q]);
#pragma unroll
              for (int e = 0; e < P; ++e) {
                const float2 d = add2(a[e], nk);
                s1[q] = add2(s1[q], d);
                s2[q] = fma2(d, d, s2[q]);
              }
            }
          }
        }
        float t1[R], t2[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
          t1[q] = s1[q].x + s1[q].y;
          t2[q] = s2[q].x + s2[q].y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
          for (int q = 0; q < R; ++q) {
            t1[q] += __shfl_xor_sync(0xffffffffu, t1[q], o);
            t2[q] += __shfl_xor_sync(0xffffffffu, t2[q], o);
          }
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
          const float m1 = t1[q] / float(C);
          mean[q] = K[q] + m1;
          inv[q] = 1.f / sqrtf(fmaxf(t2[q] / float(C) - m1 * m1, 0.f) + p.eps);
        }
      } else {
        float t[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
          float2 acc = f2(0.f);
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            float2 a[P];
            unpack2(v[q][i], a, T());
#pragma unroll
            for (int e = 0; e < P; ++e) acc = fma2(a[e], a[e], acc);
          }
          t[q] = acc.x + acc.y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
          for (int q = 0; q < R; ++q) t[q] += __shfl_xor_sync(0xffffffffu, t[q], o);
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
          mean[q] = 0.f;
          inv[q] = 1.f / sqrtf(t[q] / float(C) + p.eps);
        }
      }
      T* yr[R];
      int64_t bb[R];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const int64_t row = r0 + k + (q < nr ? q : 0);
        bb[q] = (!SIMPLE && p.nbatch > 1) ? row / p.rows_per_batch : 0;
        yr[q] = static_cast<T*>(p.y) + row_offset(p.ym, row);
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t vi = lane + 32 * i;
        if (vi >= nvec) continue;
        const int64_t c0 = vi * VEC;
        float2 fa[P], fb[P], fg[P];
#pragma unroll
        for (int q = 0; q < R; ++q) {
          if (q >= nr) break;
          // The coefficients are loaded once for rows of the same batch.
          if (q == 0 || (!SIMPLE && bb[q] != bb[q - 1])) {
            const float* ca = coef + bb[q] * C + c0;
            ld_pairs<P>(ca, fa);
            ld_pairs<P>(ca + nc, fb);
            if (!SIMPLE && p.g2.ptr) ld_pairs<P>(ca + 2 * nc, fg);
          }
          float2 a[P], o[P];
          unpack2(v[q][i], a, T());
          const float2 nm = f2(-mean[q]), inv2 = f2(inv[q]);
#pragma unroll
          for (int e = 0; e < P; ++e) o[e] = fma2(mul2(add2(a[e], nm), inv2), fa[e], fb[e]);
          if (!SIMPLE && p.g2.ptr) {
#pragma unroll
            for (int e = 0; e < P; ++e) o[e] = mul2(fg[e], o[e]);
          }
          if (!SIMPLE && p.add_input) {
#pragma unroll
            for (int e = 0; e < P; ++e) o[e] = add2(o[e], a[e]);
          }
          st_act_raw(reinterpret_cast<uint4*>(yr[q] + c0), pack2(o, T()));
        }
      }
    }
  }
  __syncthreads();
  // After an abort no copy into shared memory may still be in flight when the
  // block exits: each producer lane waits (bounded) for the last row it
  // issued into each of its slots.
  if (*abort_flag && warp == 0 && lane < kRingProducers && last >= 0) {
    for (int s = lane; s < rc.nslot; s += kRingProducers) {
      if (last < s) continue;
      const int64_t ks = last - ((last - s) % rc.nslot);  // newest row of slot s
      ring_wait(&full[s], uint32_t(ks / rc.nslot) & 1u, abort_flag, rc.wait_ns, true, &g_norm_status);
    }
  }
}

// Resident blocks of one kernel instance on the whole device (one full wave).
constexpr size_t kStageMax = 48 * 1024;  // shared-memory budget of the folded coefficients

template <typename T, int VEC, int G, int NV, bool RES, bool STG>
static int64_t rownorm_wave() {
  static const int64_t wave = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rownorm_kernel<T, VEC, G, NV, RES, STG>,
                                                      kBlock, STG ? kStageMax : 0) != cudaSuccess ||
        n < 1)
      n = 1;
    return int64_t(n) * sm_count();
  }();
  return wave;
}

template <typename T, int VEC, int G, int NV, bool RES, bool STG>
static void launch_rownorm_k(const RowNormParams& p, size_t smem, cudaStream_t s) {
  constexpr int rpb = kBlock / G;
  int64_t blocks = (p.rows + rpb - 1) / rpb;
  // Persistent: at most kWaves resident waves of blocks, each block striding
  // over row groups.
  const int64_t cap = kWaves * rownorm_wave<T, VEC, G, NV, RES, STG>();
  if (blocks > cap) blocks = cap;
  rownorm_kernel<T, VEC, G, NV, RES, STG><<<dim3(unsigned(blocks)), kBlock, smem, s>>>(p);
}

template <typename T, int VEC, int NV>
static void launch_rownorm_g(const RowNormParams& p, int G, size_t smem, cudaStream_t s) {
  switch (G) {
#define L3D_CASE(GG)                                                          \
  case GG:                                                                    \
    if (p.h) {                                                                \
      if (smem) launch_rownorm_k<T, VEC, GG, NV, true, true>(p, smem, s);     \
      else launch_rownorm_k<T, VEC, GG, NV, true, false>(p, 0, s);            \
    } else {                                                                  \
      if (smem) launch_rownorm_k<T, VEC, GG, NV, false, true>(p, smem, s);    \
      else launch_rownorm_k<T, VEC, GG, NV, false, false>(p, 0, s);           \
    }                                                                         \
    break;
    L3D_CASE(8) L3D_CASE(16) L3D_CASE(32) L3D_CASE(64) L3D_CASE(128) L3D_CASE(256)
#undef L3D_CASE
    default: break;
  }
}

template <typename T, int VEC>
static void launch_rownorm(const RowNormParams& p, int G, int NV, size_t smem, cudaStream_t s) {
  if constexpr (VEC == 1) {
    launch_rownorm_g<T, VEC, 16>(p, G, smem, s);
  } else {
    if (NV <= 2) launch_rownorm_g<T, VEC, 2>(p, G, smem, s);
    else if (NV <= 4) launch_rownorm_g<T, VEC, 4>(p, G, smem, s);
    else launch_rownorm_g<T, VEC, 8>(p, G, smem, s);
  }
}

// Pick threads-per-row G and vectors-per-thread NV for a row of nvec vectors:
// the smallest group that holds the row in at most eight 16-byte vectors per
// thread, so each thread has all its loads in flight at once.
static bool pick_geometry(int64_t nvec, bool scalar, int* G, int* NV) {
  if (scalar) {  // ragged rows: up to 256 threads x 16 elements
    int g = 8;
    while (g < 256 && (nvec + g - 1) / g > 16) g *= 2;
    *G = g;
    *NV = 16;
    return (nvec + g - 1) / g <= 16;
  }
  // Up to eight 16-byte vectors per thread: a whole 2048-element bf16 (or
  // 1024-element f32) row per warp, reduced with shuffles only.
  int g = 8;
  while (g < 256 && g * 8 < nvec) g *= 2;
  int64_t nv = (nvec + g - 1) / g;
  int n = 2;
  while (n < nv) n *= 2;
  *G = g;
  *NV = n;
  return n <= 8;
}

// Ring path selection (rowring_kernel): LN / RMS without a residual branch,
// 16-byte vectors, rows of 2 to 8 KB, enough rows to keep every SM's ring
// busy (shorter rows or inputs run faster in the register kernel, which
// packs several rows per warp and fills the device sooner).
constexpr int64_t kRingMinRows = 32768;
constexpr uint32_t kRingMinRowBytes = 2048;

template <typename T, int NV, int NW, int R>
static int launch_ring(const RowNormParams& p, const RingCfg& rc, size_t smem, cudaStream_t s) {
  const bool simple = p.norm == NORM_LAYER && !p.g2.ptr && !p.add_input && p.nbatch == 1;
  auto k = simple ? rowring_kernel<T, NV, NW, R, true> : rowring_kernel<T, NV, NW, R, false>;
  // The limit is set once per device to the most any launch of it uses.
  if (set_smem_limit(reinterpret_cast<const void*>(k), int(kRingSmem)) != cudaSuccess) return -1;
  int64_t grid = (p.rows + NW - 1) / NW;
  if (grid > sm_count()) grid = sm_count();
  k<<<dim3(unsigned(grid)), 32 * (NW + 1), smem, s>>>(p, rc);
  return 0;
}

// Returns 1 when the ring kernel was launched, 0 when the request is outside
// its envelope, -1 on a CUDA error.
template <typename T>
static int try_ring(const RowNormParams& p, cudaStream_t s) {
  const int es = int(sizeof(T));
  const int vec = 16 / es;
  const uint32_t row_bytes = uint32_t(p.C * es);
  if (p.rows < kRingMinRows || row_bytes < kRingMinRowBytes || row_bytes > 8192 || p.C % vec)
    return 0;
  const int64_t nv = (p.C / vec + 31) / 32;
  RingCfg rc{};
  rc.row_bytes = row_bytes;
  rc.coef_bytes = (size_t(p.nbatch) * size_t(p.C) * 4 * (p.g2.ptr ? 3 : 2) + 127) & ~size_t(127);
  if (rc.coef_bytes > 64 * 1024) return 0;
  // Rows up to 4 KB: 12 consumer warps taking row pairs; 8 KB rows: 16
  // warps taking single rows (a pair would not fit the registers).  Slot s
  // belongs to consumer warp (s / R) % NW and to producer lane s % 8 (row k
  // goes to slot k % nslot), so nslot is a multiple of R NW and of 8: each
  // slot's owner consumes its rows in order and no wait on a slot barrier is
  // ever more than one phase ahead of it, so the parity of the phase waited
  // for is never ambiguous.  Measured at 1M x 2048 bf16: one pair of slots
  // per warp (24 slots) is fastest; shorter rows get more.
  const bool pair = nv <= 8;
  const int64_t unit = pair ? 24 : 16;  // lcm(R NW, kRingProducers)
  const size_t bar_bytes = size_t(2) * kRingMaxSlots * 8 + 16;
  int64_t ns = int64_t((kRingSmem - rc.coef_bytes - bar_bytes) / row_bytes);
  if (pair) {
    const int64_t want = unit * (4096 / row_bytes);
    if (ns > want) ns = want;
  }
  if (ns > kRingMaxSlots) ns = kRingMaxSlots;
  ns -= ns % unit;
  if (ns < unit) return 0;
  rc.nslot = int(ns);
  rc.wait_ns = 2000000000ull;
  const size_t smem = rc.coef_bytes + size_t(rc.nslot) * row_bytes + size_t(2) * rc.nslot * 8 + 16;
  int rcode;
  if (nv <= 4) rcode = launch_ring<T, 4, 12, 2>(p, rc, smem, s);
  else if (nv <= 8) rcode = launch_ring<T, 8, 12, 2>(p, rc, smem, s);
  else rcode = launch_ring<T, 16, 16, 1>(p, rc, smem, s);
  static_assert(kRingMaxSlots % 24 == 0 && kRingMaxSlots % 16 == 0, "slot ownership");
  return rcode == 0 ? 1 : -1;
}

struct RowNormArgs {
  const l3d_tensor *x, *h, *g1, *w, *b, *scale, *shift, *g2, *r_out, *y;
  int add_input;
  int norm;
  float eps;
  const char* op;
  int batch_dims;  // leading dims of x that form the batch of per-batch vectors (0 or 1)
};

static bool same_shape(const l3d_tensor* a, const l3d_tensor* b) {
  if (a->ndim != b->ndim) return false;
  for (int i = 0; i < a->ndim; ++i)
    if (a->dims[i] != b->dims[i]) return false;
  return true;
}

static int check_act(const l3d_tensor* t, const l3d_tensor* x, const char* op,
                     const char* name) {
  if (no_data(t)) return fail(L3D_E_NULL, "%s: %s has a null data pointer", op, name);
  if (t->dtype != x->dtype)
    return fail(L3D_E_DTYPE, "%s: %s dtype %s != x dtype %s", op, name, dtype_name(t->dtype),
                dtype_name(x->dtype));
  if (!same_shape(t, x)) return fail(L3D_E_SHAPE, "%s: %s shape differs from x", op, name);
  if (t->dims[t->ndim - 1] > 1 && t->strides[t->ndim - 1] != 1)
    return fail(L3D_E_ALIGN, "%s: %s last dim must be contiguous", op, name);
  return L3D_OK;
}

static int run_rownorm(const RowNormArgs& a, cudaStream_t stream) {
  const char* op = a.op;
  if (!a.x || !a.y) return fail(L3D_E_NULL, "%s: x and y are required", op);
  if (no_data(a.x)) return fail(L3D_E_NULL, "%s: x has a null data pointer", op);
  if (!is_float_dtype(a.x->dtype)) return fail(L3D_E_DTYPE, "%s: x must be F32/F16/BF16", op);
  if (a.x->ndim < 1 || a.x->ndim > L3D_MAX_DIMS) return fail(L3D_E_SHAPE, "%s: bad rank", op);
  int rc;
  if ((rc = check_act(a.y, a.x, op, "y"))) return rc;
  if (a.h && (rc = check_act(a.h, a.x, op, "h"))) return rc;
  if (a.r_out && (rc = check_act(a.r_out, a.x, op, "r_out"))) return rc;
  if (a.x->dims[a.x->ndim - 1] > 1 && a.x->strides[a.x->ndim - 1] != 1)
    return fail(L3D_E_ALIGN, "%s: x last dim must be contiguous", op);

  RowNormParams p{};
  p.C = a.x->dims[a.x->ndim - 1];
  p.rows = 1;
  for (int i = 0; i < a.x->ndim - 1; ++i) p.rows *= a.x->dims[i];
  if (p.C <= 0) return fail(L3D_E_SHAPE, "%s: empty rows (C = 0)", op);
  if (p.rows == 0) return L3D_OK;
  int64_t B = 1;
  if (a.batch_dims == 1 && a.x->ndim >= 3) B = a.x->dims[0];
  p.rows_per_batch = p.rows / B;
  const int lead = a.x->ndim - 1;
  if (!make_rowmap(a.x, lead, &p.xm) || !make_rowmap(a.y, lead, &p.ym) ||
      (a.h && !make_rowmap(a.h, lead, &p.hm)) || (a.r_out && !make_rowmap(a.r_out, lead, &p.rm)))
    return fail(L3D_E_UNSUPPORTED, "%s: more than 5 non-collapsible leading dims", op);

  bool al = true;
  if ((rc = make_chanvec(a.g1, "gate", p.C, B, &p.g1, &al))) return rc;
  if ((rc = make_chanvec(a.w, "weight", p.C, 1, &p.w, &al))) return rc;
  if ((rc = make_chanvec(a.b, "bias", p.C, 1, &p.b, &al))) return rc;
  if ((rc = make_chanvec(a.scale, "scale", p.C, B, &p.scale, &al))) return rc;
  if ((rc = make_chanvec(a.shift, "shift", p.C, B, &p.shift, &al))) return rc;
  if ((rc = make_chanvec(a.g2, "gate", p.C, B, &p.g2, &al))) return rc;
  p.y = a.y->data;
  p.h = a.h ? a.h->data : nullptr;
  p.r_out = a.r_out ? a.r_out->data : nullptr;
  p.x = a.x->data;
  p.add_input = a.add_input;
  p.norm = a.norm;
  p.eps = a.eps;

  const int es = dtype_size(a.x->dtype);
  const int vec = 16 / es;
  bool vec_ok = al && (p.C % vec == 0);
  auto ptr_ok = [&](const l3d_tensor* t, const RowMap& m) {
    return !t || ((reinterpret_cast<uintptr_t>(t->data) % 16) == 0 && rowmap_aligned(m, vec));
  };
  vec_ok = vec_ok && ptr_ok(a.x, p.xm) && ptr_ok(a.y, p.ym) && ptr_ok(a.h, p.hm) &&
           ptr_ok(a.r_out, p.rm);
  const int64_t vlen = vec_ok ? vec : 1;
  const int64_t nvec = p.C / vlen;
  int G = 8, NV = 8;
  if (!pick_geometry(nvec, !vec_ok, &G, &NV))
    return fail(L3D_E_UNSUPPORTED, "%s: row length %lld exceeds the per-row limit", op,
                (long long)p.C);
  // Fold the per-channel vectors into shared memory when they fit.
  p.nbatch = (p.scale.bstride || p.shift.bstride || p.g2.bstride) ? int(B) : 1;
  size_t smem = 0;
  if (p.norm != NORM_NONE) {
    const size_t need = size_t(p.nbatch) * size_t(p.C) * sizeof(float) * (p.g2.ptr ? 3 : 2);
    if (need <= kStageMax) smem = need;
  }
  int ring = 0;
  if (vec_ok && !a.h && !a.r_out && p.norm != NORM_NONE && smem) {
    L3D_DISPATCH_FLOAT(a.x->dtype, T, { ring = try_ring<T>(p, stream); });
    if (ring < 0) return fail(L3D_E_CUDA, "%s: cannot reserve the ring kernel's shared memory", op);
  }
  if (!ring) {
    L3D_DISPATCH_FLOAT(a.x->dtype, T, {
      if (vec_ok) launch_rownorm<T, Vec16<T>::N>(p, G, NV, smem, stream);
      else launch_rownorm<T, 1>(p, G, NV, smem, stream);
    });
  }
  return check_launch(op);
}

}  // namespace l3d

using namespace l3d;

extern "C" int l3d_layer_norm(const l3d_tensor* x, const l3d_tensor* weight,
                              const l3d_tensor* bias, float eps, const l3d_tensor* y,
                              l3d_stream stream) {
  RowNormArgs a{};
  a.x = x; a.w = weight; a.b = bias; a.y = y; a.eps = eps;
  a.norm = NORM_LAYER; a.op = "l3d_layer_norm"; a.batch_dims = 0;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_layer_norm_modulate(const l3d_tensor* x, const l3d_tensor* weight,
                                       const l3d_tensor* bias, const l3d_tensor* shift,
                                       const l3d_tensor* scale, const l3d_tensor* gate,
                                       int add_input, float eps, const l3d_tensor* y,
                                       l3d_stream stream) {
  RowNormArgs a{};
  a.x = x; a.w = weight; a.b = bias; a.shift = shift; a.scale = scale; a.g2 = gate;
  a.add_input = add_input ? 1 : 0; a.y = y; a.eps = eps;
  a.norm = NORM_LAYER; a.op = "l3d_layer_norm_modulate"; a.batch_dims = 1;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_gated_residual(const l3d_tensor* x, const l3d_tensor* h,
                                  const l3d_tensor* gate, const l3d_tensor* out,
                                  l3d_stream stream) {
  if (!h) return fail(L3D_E_NULL, "l3d_gated_residual: h is required");  // gate NULL: x + h
  RowNormArgs a{};
  a.x = x; a.h = h; a.g1 = gate; a.y = out;
  a.norm = NORM_NONE; a.op = "l3d_gated_residual"; a.batch_dims = 1;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_layerscale_residual(const l3d_tensor* x, const l3d_tensor* h,
                                       const l3d_tensor* gamma, const l3d_tensor* out,
                                       l3d_stream stream) {
  if (!h || !gamma) return fail(L3D_E_NULL, "l3d_layerscale_residual: h and gamma are required");
  if (gamma->ndim != 1)
    return fail(L3D_E_SHAPE, "l3d_layerscale_residual: gamma must be [C]");
  RowNormArgs a{};
  a.x = x; a.h = h; a.g1 = gamma; a.y = out;
  a.norm = NORM_NONE; a.op = "l3d_layerscale_residual"; a.batch_dims = 0;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_residual_layer_norm_modulate(
    const l3d_tensor* x, const l3d_tensor* h, const l3d_tensor* gate, const l3d_tensor* weight,
    const l3d_tensor* bias, const l3d_tensor* shift, const l3d_tensor* scale, float eps,
    const l3d_tensor* r_out, const l3d_tensor* y, l3d_stream stream) {
  if (!h) return fail(L3D_E_NULL, "l3d_residual_layer_norm_modulate: h is required");
  RowNormArgs a{};
  a.x = x; a.h = h; a.g1 = gate; a.w = weight; a.b = bias; a.shift = shift; a.scale = scale;
  a.r_out = r_out; a.y = y; a.eps = eps;
  a.norm = NORM_LAYER; a.op = "l3d_residual_layer_norm_modulate"; a.batch_dims = 1;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_rms_norm_heads(const l3d_tensor* x, const l3d_tensor* weight, float eps,
                                  const l3d_tensor* y, l3d_stream stream) {
  RowNormArgs a{};
  a.x = x; a.w = weight; a.y = y; a.eps = eps;
  a.norm = NORM_RMS; a.op = "l3d_rms_norm_heads"; a.batch_dims = 0;
  return run_rownorm(a, reinterpret_cast<cudaStream_t>(stream));
}

namespace l3d {
cudaError_t norm_status_read(int* status, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_norm_status, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_norm_status, &zero, sizeof(int));
  }
  return e;
}
}  // namespace l3d
