// Per-head normalisation fused with rotary position embedding.
//
//  * rope2d: VGGT / Pi3 per-head affine LayerNorm (D = 64) + 2D axial RoPE
//    (rotate-half within each 32-wide half; y half uses the y position, x half
//    the x position).  One warp owns one token and walks all heads of q (and
//    optionally k) with 8 lanes per head, so the 32 distinct (half, frequency)
//    angles of a token are formed once (one sincosf per lane) and shuffled to
//    the lanes that need them; no cos/sin table is read in positions mode.
//    Each lane holds both rotate-half partners, so the rotation is local, and
//    the LayerNorm affine is folded into the rotation coefficients.
//  * rope3d: TRELLIS.2 MultiHeadRMSNorm (x / ||x|| * gamma * sqrt(D)) + 3D RoPE
//    over interleaved (re, im) pairs with angles coord[axis] * freq[i].  One
//    warp owns one token; each lane keeps the angles of its own pairs for all
//    heads of that token.
//
// Angles are formed bit-exactly as the reference forms them: inverse
// frequencies 1 / theta^(e) with e an f32 quotient, the power evaluated in
// double and rounded once (the correctly rounded f32 result), and the angle a
// single f32 product of the integer position and the frequency.
#include <type_traits>

#include "common.cuh"

namespace l3d {

// --------------------------------------------------------------------- helpers
__device__ __forceinline__ float inv_freq_f32(float theta, float num, float den) {
  const float e = __fdiv_rn(num, den);
  const float p = static_cast<float>(pow(static_cast<double>(theta), static_cast<double>(e)));
  return __fdiv_rn(1.0f, p);
}

// sin / cos of an exactly formed angle: the accurate libm form for f32
// activations; for 16-bit activations the hardware approximation after a
// Cody-Waite reduction by 2*pi (two-constant split: the f32 value of 2*pi and
// its f32 rounding error), so the error stays at the [-pi, pi] level (a few
// 1e-7) for any coordinate: TRELLIS.2 voxel coordinates reach 1023 and the
// unreduced hardware form loses accuracy in proportion to |angle|.
template <typename T>
__device__ __forceinline__ void sincos_t(float a, float* s, float* c) {
  if constexpr (sizeof(T) == 2) {
    const float k = rintf(a * 0.159154943091895336f);  // a / (2 pi), nearest
    float r = fmaf(-k, 6.28318548202514648f, a);        // f32(2 pi) = 2 pi + 1.7484555e-7
    r = fmaf(k, 1.74845553e-7f, r);
    __sincosf(r, s, c);
  } else {
    sincosf(a, s, c);
  }
}

__device__ __forceinline__ float load_index_f(const void* p, int dtype, int64_t off) {
  if (dtype == L3D_I64) return static_cast<float>(static_cast<const int64_t*>(p)[off]);
  if (dtype == L3D_U32) return static_cast<float>(static_cast<const uint32_t*>(p)[off]);
  return static_cast<float>(static_cast<const int32_t*>(p)[off]);
}

// 8 consecutive elements as floats (one 16-byte access for 16-bit types, two
// for f32).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    float a[4], b[4];
    load_act<T, 4>(p, a);
    load_act<T, 4>(p + 4, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[i] = a[i]; f[4 + i] = b[i]; }
  } else {
    load_act<T, 8>(p, f);
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    float a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) { a[i] = f[i]; b[i] = f[4 + i]; }
    store_act<T, 4>(p, a);
    store_act<T, 4>(p + 4, b);
  } else {
    store_act<T, 8>(p, f);
  }
}

// ======================================================================= 2D
struct HeadView {            // [B, H, N, D] view (element strides)
  void* data;
  int64_t base, sb, sh, sn;
};

struct Rope2dParams {
  int64_t B, N;
  int H;
  int ntensor;               // 1 (q) or 2 (q and k)
  HeadView in[2], out[2];
  ChanVec w[2], b[2];        // per-tensor LayerNorm affine ([64]) or null
  int do_norm;
  float eps;
  // table mode: cos_full / sin_alt_full [B, N, 64] F32 views
  int use_table;
  const float* cosp;
  const float* sinp;
  int64_t cbase, csb, csn, sbase, ssb, ssn;
  // positions mode: positions [B, N, 2]
  const void* pos;
  int pos_dtype;
  int64_t pbase, psb, psn, psc;
  float theta;
};

// 4 consecutive elements kept packed in registers (8 bytes for 16-bit types,
// 16 for f32) until they are used.
template <typename T>
struct Raw4 {
  using type = typename std::conditional<sizeof(T) == 4, float4, uint2>::type;
};
// Evict-first loads: measured about 3% faster than plain loads for this
// kernel's 8-byte accesses (the other kernels see no difference or lose).
template <typename T>
__device__ __forceinline__ typename Raw4<T>::type load_raw4(const T* p) {
  return __ldcs(reinterpret_cast<const typename Raw4<T>::type*>(p));
}
// Elements 2 pr and 2 pr + 1 of a 4-element array as a float pair.
__device__ __forceinline__ float2 as_f2(const float (&f)[4], int pr) {
  return make_float2(f[2 * pr], f[2 * pr + 1]);
}

// Rotation coefficients of one tensor for this lane's chunks A and B with the
// LayerNorm affine folded in.  With cos c and sin s of the chunk's four
// frequencies, rotate_half gives
//   out_A = (n_A w_A + b_A) c - (n_B w_B + b_B) s = n_A k1a + n_B k2a + k0a
//   out_B = (n_B w_B + b_B) c + (n_A w_A + b_A) s = n_B k1b + n_A k2b + k0b
// for normalised inputs n (w = 1, b = 0 without the norm).
struct Rope2dCoef {
  float2 k1a[2], k2a[2], k0a[2], k1b[2], k2b[2], k0b[2];
};
__device__ __forceinline__ void rope2d_coef(const float (*aff)[64], int ea, const float (&c)[4],
                                            const float (&sn)[4], Rope2dCoef& k) {
  const float4 wa4 = *reinterpret_cast<const float4*>(&aff[0][ea]);
  const float4 wb4 = *reinterpret_cast<const float4*>(&aff[0][ea + 16]);
  const float4 ba4 = *reinterpret_cast<const float4*>(&aff[1][ea]);
  const float4 bb4 = *reinterpret_cast<const float4*>(&aff[1][ea + 16]);
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    const float2 wa = pr ? make_float2(wa4.z, wa4.w) : make_float2(wa4.x, wa4.y);
    const float2 wb = pr ? make_float2(wb4.z, wb4.w) : make_float2(wb4.x, wb4.y);
    const float2 ba = pr ? make_float2(ba4.z, ba4.w) : make_float2(ba4.x, ba4.y);
    const float2 bb = pr ? make_float2(bb4.z, bb4.w) : make_float2(bb4.x, bb4.y);
    const float2 cc = as_f2(c, pr), ss = as_f2(sn, pr);
    const float2 ns = make_float2(-ss.x, -ss.y);
    k.k1a[pr] = __fmul2_rn(wa, cc);
    k.k2a[pr] = __fmul2_rn(wb, ns);
    k.k0a[pr] = __ffma2_rn(ba, cc, __fmul2_rn(bb, ns));
    k.k1b[pr] = __fmul2_rn(wb, cc);
    k.k2b[pr] = __fmul2_rn(wa, ss);
    k.k0b[pr] = __ffma2_rn(bb, cc, __fmul2_rn(ba, ss));
  }
}

// 4 packed elements -> two f32 pairs.
template <typename T>
__device__ __forceinline__ void unpack4x2(const typename Raw4<T>::type& u, float2 (&v)[2]) {
  if constexpr (sizeof(T) == 4) {
    v[0] = make_float2(u.x, u.y);
    v[1] = make_float2(u.z, u.w);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    v[0] = make_float2(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u));
    v[1] = make_float2(__uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  } else {
    v[0] = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    v[1] = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  }
}
template <typename T>
__device__ __forceinline__ void store4x2(T* p, const float2 (&v)[2]) {
  if constexpr (sizeof(T) == 4) {
    st_act_raw(reinterpret_cast<float4*>(p), make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
  } else {
    uint32_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[i].x, v[i].y);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[i].x, v[i].y);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    st_act_raw(reinterpret_cast<uint2*>(p), make_uint2(w[0], w[1]));
  }
}

// One lane's two quarter-chunks of a head (A = 4 elements at 32h + 4k, B =
// A + 16, packed) through the per-head LayerNorm (the head's 8 lanes reduce
// together, xor shuffles 1, 2, 4: mean, then the centred sum of squares) and
// the rotation with the folded coefficients `k`.  All lanes of the warp call
// it together.
template <typename T>
__device__ __forceinline__ void rope2d_chunks(const typename Raw4<T>::type& ra,
                                              const typename Raw4<T>::type& rb,
                                              const Rope2dCoef& k, int do_norm, float eps,
                                              float2 (&oa)[2], float2 (&ob)[2]) {
  float2 a[2], bv[2];
  unpack4x2<T>(ra, a);
  unpack4x2<T>(rb, bv);
  if (do_norm) {
    const float2 s2 = __fadd2_rn(__fadd2_rn(a[0], a[1]), __fadd2_rn(bv[0], bv[1]));
    float sum = s2.x + s2.y;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    const float2 nm = f2(-sum * (1.0f / 64.0f));
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      a[pr] = __fadd2_rn(a[pr], nm);
      bv[pr] = __fadd2_rn(bv[pr], nm);
    }
    float2 q2 = __fmul2_rn(a[0], a[0]);
    q2 = __ffma2_rn(a[1], a[1], q2);
    q2 = __ffma2_rn(bv[0], bv[0], q2);
    q2 = __ffma2_rn(bv[1], bv[1], q2);
    float ss = q2.x + q2.y;
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    const float var = ss * (1.0f / 64.0f) + eps;
    const float2 inv = f2(sizeof(T) == 2 ? rsqrtf(var) : 1.f / sqrtf(var));
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      a[pr] = __fmul2_rn(a[pr], inv);
      bv[pr] = __fmul2_rn(bv[pr], inv);
    }
  }
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    oa[pr] = __ffma2_rn(a[pr], k.k1a[pr], __ffma2_rn(bv[pr], k.k2a[pr], k.k0a[pr]));
    ob[pr] = __ffma2_rn(bv[pr], k.k1b[pr], __ffma2_rn(a[pr], k.k2b[pr], k.k0b[pr]));
  }
}

// One warp per token; 8 lanes per 64-wide head row, 4 heads per iteration.
// Lane j (0..7) of a head owns the two quarter-chunks that rotate into each
// other: elements A = 32h + 4k + t and B = A + 16 (h = j / 4, k = j % 4,
// t = 0..3), so rotate_half needs no data exchange.  Its four angles
// (half h, frequency 4k + t) are formed by lanes 4j + t of the warp (lane L
// forms half L / 16, frequency L % 16) and fetched with one shuffle each.
// The per-head LayerNorm reduces over the head's 8 lanes (xor shuffles 1, 2,
// 4; two passes: mean, then the centred sum of squares).  Element arithmetic
// is packed f32x2.  Launched with 256 threads per block; 16-bit variants are
// held to 4 blocks per SM (a few registers spill), which measured faster than
// 3 blocks without spills.
template <typename T>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? 4 : 2) rope2d_kernel(const Rope2dParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int j = lane & 7;     // lane within the head row
  const int hg = lane >> 3;   // head slot within an iteration of 4 heads
  const int ea = 32 * (j >> 2) + 4 * (j & 3);  // first element of chunk A (B = ea + 16)
  const int64_t tokens = p.B * p.N;

  // Lane `lane` forms the angle of (half = lane / 16, freq = lane % 16):
  // inv_freq[f] = 1 / theta^(2f / 32), Rope2d::cos_sin with dim = 32.
  const float invf = inv_freq_f32(p.theta, float(2 * (lane & 15)), 32.0f);

  // LayerNorm affine per tensor, staged in shared memory as [tensor][w|b][64]
  // (absent weight = 1, absent bias = 0; without the norm, 1 and 0).
  __shared__ __align__(16) float aff[2][2][64];
  {
    const int t = threadIdx.x >> 7, wb = (threadIdx.x >> 6) & 1, e = threadIdx.x & 63;
    float v = wb ? 0.f : 1.f;
    if (t < p.ntensor && p.do_norm) {
      const ChanVec& cv = wb ? p.b[t] : p.w[t];
      if (cv.ptr) {
        float one[1];
        load_chan<1>(cv, 0, e, one);
        v = one[0];
      }
    }
    aff[t][wb][e] = v;
  }
  __syncthreads();

  // Heads in groups of 4 iterations x 4 heads: the group's loads are all
  // issued before any arithmetic; the first group of q goes out before the
  // token's positions are read, so the two latencies overlap.
  constexpr int MAXIT = 4;
  for (int64_t tok = warp0; tok < tokens; tok += nwarps) {
    const int64_t b = tok / p.N;
    const int64_t n = tok - b * p.N;
    typename Raw4<T>::type ra[MAXIT], rb[MAXIT];
    auto load_group = [&](const HeadView& iv, int hb) {
      const T* src0 = static_cast<const T*>(iv.data) + iv.base + b * iv.sb + n * iv.sn + ea;
#pragma unroll
      for (int it = 0; it < MAXIT; ++it) {
        const int h = hb + it * 4 + hg;
        if (h < p.H) {
          const T* src = src0 + int64_t(h) * iv.sh;
          ra[it] = load_raw4<T>(src);
          rb[it] = load_raw4<T>(src + 16);
        } else {
          ra[it] = rb[it] = {};
        }
      }
    };
    load_group(p.in[0], 0);
    // cos c and sin s of this lane's four frequencies.
    float c[4], sn[4];
    if (p.use_table) {
      // cos_full / sin_alt_full: chunk A holds cos and -sin.
      const float* cp = p.cosp + p.cbase + b * p.csb + n * p.csn + ea;
      const float* sp = p.sinp + p.sbase + b * p.ssb + n * p.ssn + ea;
#pragma unroll
      for (int i = 0; i < 4; ++i) { c[i] = __ldg(cp + i); sn[i] = -__ldg(sp + i); }
    } else {
      const float pos = load_index_f(p.pos, p.pos_dtype,
                                     p.pbase + b * p.psb + n * p.psn + (lane >> 4) * p.psc);
      float sv, cv;
      sincos_t<T>(__fmul_rn(pos, invf), &sv, &cv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        c[i] = __shfl_sync(0xffffffffu, cv, 4 * j + i);
        sn[i] = __shfl_sync(0xffffffffu, sv, 4 * j + i);
      }
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t >= p.ntensor) break;
      const HeadView& iv = p.in[t];
      const HeadView& ov = p.out[t];
      T* dst0 = static_cast<T*>(ov.data) + ov.base + b * ov.sb + n * ov.sn + ea;
      Rope2dCoef k;
      rope2d_coef(aff[t], ea, c, sn, k);
      for (int hb = 0; hb < p.H; hb += 4 * MAXIT) {
        if (t > 0 || hb > 0) load_group(iv, hb);
#pragma unroll
        for (int it = 0; it < MAXIT; ++it) {
          if (hb + it * 4 >= p.H) break;  // warp-uniform
          const int h = hb + it * 4 + hg;
          float2 oa[2], ob[2];
          rope2d_chunks<T>(ra[it], rb[it], k, p.do_norm, p.eps, oa, ob);
          if (h < p.H) {
            T* dst = dst0 + int64_t(h) * ov.sh;
            store4x2<T>(dst, oa);
            store4x2<T>(dst + 16, ob);
          }
        }
      }
    }
  }
}

__global__ void rope2d_tables_kernel(int64_t B, int64_t N, const void* pos, int pos_dtype,
                                     int64_t pbase, int64_t psb, int64_t psn, int64_t psc,
                                     float theta, int D, float* cosp, float* sinp) {
  // cos_full / sin_alt_full [B, N, D] contiguous.
  const int64_t total = B * N * D;
  const int half = D / 2, quarter = D / 4;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int e = int(i % D);
    const int64_t tok = i / D;
    const int64_t b = tok / N, n = tok - b * N;
    const int hf = e / half;      // 0: y half, 1: x half
    const int j = e % half;
    const int f = j % quarter;    // freqs = cat(f, f)
    const float invf = inv_freq_f32(theta, float(2 * f), float(half));
    const float ps = load_index_f(pos, pos_dtype, pbase + b * psb + n * psn + hf * psc);
    float sv, cv;
    sincosf(__fmul_rn(ps, invf), &sv, &cv);
    cosp[i] = cv;
    sinp[i] = j < quarter ? -sv : sv;
  }
}

// ======================================================================= 3D
struct Rope3dParams {
  int64_t B, L;
  int H, D;
  const void* x;
  int64_t xbase, xsb, xsl, xsh;    // x [B, L, H, D]
  void* y;
  int64_t ybase, ysb, ysl, ysh;
  const float* gamma;              // [H, D] contiguous F32 or null
  int64_t gsh;
  float scale;                     // sqrt(D)
  // angles from coords [L, 3] ...
  const void* coords;
  int coord_dtype;
  int64_t cbase, csl, csa;
  float theta;
  int freq_dim;
  // ... or from tables cos/sin [L, D/2] F32
  int use_table;
  const float* cost;
  const float* sint;
  int64_t tcbase, tcsl, tsbase, tssl;
};

// 8 consecutive elements in their storage format (16 B for 16-bit types,
// 32 B for f32), unpacked only where the arithmetic needs them.
template <typename T>
struct Pack8 {
  uint4 u[sizeof(T) == 4 ? 2 : 1];
};
template <typename T>
__device__ __forceinline__ Pack8<T> ld_pack8(const T* p) {
  Pack8<T> r;
  r.u[0] = ld_act_raw(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) r.u[1] = ld_act_raw(reinterpret_cast<const uint4*>(p) + 1);
  return r;
}
template <typename T>
__device__ __forceinline__ void unpack8(const Pack8<T>& r, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    float a[4], b[4];
    unpack(r.u[0], a, float());
    unpack(r.u[1], b, float());
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[i] = a[i]; f[4 + i] = b[i]; }
  } else {
    unpack(r.u[0], f, T());
  }
}

// One 128-bit lane chunk of a head in the packed 16-bit path: four rotation
// pairs (re_k, im_k) of `u`, worked on as (re, re) / (im, im) float pairs.
// With `g` (gamma * sqrt(D) staged de-interleaved, this lane's 8 values) the
// head is L2-normalised first: the sum of squares is reduced over the LPH
// lanes of the head (all lanes of the warp call this together).  `valid`:
// the lane holds a real chunk.  Returns the rotated chunk, rounded to T.
template <typename T, int LPH>
__device__ __forceinline__ uint4 rope3d_pk_chunk(const uint4& u, const float (&cs)[4],
                                                 const float (&sn)[4], const float* g,
                                                 bool valid) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float2 re2[2], im2[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      re2[q] = make_float2(__uint_as_float(w[2 * q] << 16), __uint_as_float(w[2 * q + 1] << 16));
      im2[q] = make_float2(__uint_as_float(w[2 * q] & 0xffff0000u),
                           __uint_as_float(w[2 * q + 1] & 0xffff0000u));
    } else {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * q]));
      const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&w[2 * q + 1]));
      re2[q] = make_float2(a.x, c.x);
      im2[q] = make_float2(a.y, c.y);
    }
  }
  if (g) {
    float2 acc = mul2(re2[0], re2[0]);
    acc = fma2(im2[0], im2[0], acc);
    acc = fma2(re2[1], re2[1], acc);
    acc = fma2(im2[1], im2[1], acc);
    float ss = acc.x + acc.y;
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    // 1 / clamp(||x||, 1e-12, 1e30) = rsqrt(clamp(||x||^2, 1e-24, 1e60)).
    const float2 rn = f2(rsqrtf(fminf(fmaxf(ss, 1e-24f), 1e30f * 1e30f)));
    if (valid) {
      const float4* gp = reinterpret_cast<const float4*>(g);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float4 gq = gp[q];
        re2[q] = mul2(re2[q], mul2(make_float2(gq.x, gq.y), rn));
        im2[q] = mul2(im2[q], mul2(make_float2(gq.z, gq.w), rn));
      }
    }
  }
  // (re, im) -> (re c - im s, re s + im c).
  uint32_t ow[4];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const float2 c2 = make_float2(cs[2 * q], cs[2 * q + 1]);
    const float2 s2 = make_float2(sn[2 * q], sn[2 * q + 1]);
    const float2 ore = fma2(re2[q], c2, mul2(im2[q], make_float2(-s2.x, -s2.y)));
    const float2 oim = fma2(re2[q], s2, mul2(im2[q], c2));
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      __nv_bfloat162 h0 = __floats2bfloat162_rn(ore.x, oim.x);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(ore.y, oim.y);
      ow[2 * q] = *reinterpret_cast<uint32_t*>(&h0);
      ow[2 * q + 1] = *reinterpret_cast<uint32_t*>(&h1);
    } else {
      __half2 h0 = __floats2half2_rn(ore.x, oim.x);
      __half2 h1 = __floats2half2_rn(ore.y, oim.y);
      ow[2 * q] = *reinterpret_cast<uint32_t*>(&h0);
      ow[2 * q + 1] = *reinterpret_cast<uint32_t*>(&h1);
    }
  }
  return make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// EPL elements per lane (8: 16-byte path; 2: one pair per lane), LPH lanes per
// head row (D / EPL rounded up to a power of two).  gamma * sqrt(D) is staged
// once per block in shared memory (dynamic, H * D floats) when present.
template <typename T, int EPL, int LPH>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? 4 : 2) rope3d_kernel(const Rope3dParams p) {
  extern __shared__ float gsm[];  // [H, D] gamma * sqrt(D)
  constexpr int NP = EPL / 2;     // pairs per lane
  constexpr int HPI = 32 / LPH;   // heads per warp iteration
  const int lane = threadIdx.x & 31;
  const int m = lane % LPH;
  const int hg = lane / LPH;
  const int64_t warp0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t tokens = p.B * p.L;
  const int half = p.D / 2;
  const bool lane_on = m * EPL < p.D;

  // The packed 16-bit path (PK) works on (re, re) and (im, im) pairs of two
  // neighbouring rotation pairs, so gamma is staged in that order: each group
  // of 4 elements (re0, im0, re1, im1) is stored as (re0, re1, im0, im1).
  constexpr bool PK = EPL == 8 && sizeof(T) == 2;
  if (p.gamma) {
    for (int i = threadIdx.x; i < p.H * p.D; i += blockDim.x) {
      const int h = i / p.D, d = i - h * p.D;
      int dst = i;
      if constexpr (PK) dst = h * p.D + (d & ~3) + ((d & 1) << 1) + ((d >> 1) & 1);
      gsm[dst] = p.gamma[int64_t(h) * p.gsh + d] * p.scale;
    }
    __syncthreads();
  }

  // Frequencies of this lane's pairs (constant across tokens).
  float fr[NP];
  int axis[NP];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int pr = m * NP + k;
    const int a = p.freq_dim > 0 ? pr / p.freq_dim : 3;
    // -1: pad pair (or no coordinates given: normalisation only), angle 0.
    axis[k] = (p.coords && pr < half && a < 3) ? a : -1;
    fr[k] = axis[k] >= 0 ? inv_freq_f32(p.theta, float(pr - a * p.freq_dim), float(p.freq_dim))
                         : 0.f;
  }

  // Heads in groups of MAXIT warp iterations: the group's loads are all
  // issued (kept packed) before any arithmetic; the first group's loads go
  // out before the token's coordinates are read, so the two latencies
  // overlap.
  constexpr int MAXIT = 4;
  for (int64_t tok = warp0; tok < tokens; tok += nwarps) {
    const int64_t b = tok / p.L;
    const int64_t l = tok - b * p.L;
    const T* xt = static_cast<const T*>(p.x) + p.xbase + b * p.xsb + l * p.xsl + m * EPL;
    T* yt = static_cast<T*>(p.y) + p.ybase + b * p.ysb + l * p.ysl + m * EPL;
    Pack8<T> pk[EPL == 8 ? MAXIT : 1];
    float sv[EPL == 8 ? 1 : MAXIT][2];
    auto load_group = [&](int hb) {
#pragma unroll
      for (int it = 0; it < MAXIT; ++it) {
        const int h = hb + it * HPI + hg;
        const T* src = xt + int64_t(h) * p.xsh;
        const bool on = h < p.H && lane_on;
        if constexpr (EPL == 8) {
          if (on) pk[it] = ld_pack8<T>(src);
          else pk[it] = Pack8<T>{};
        } else {
          sv[it][0] = on ? to_f(src[0]) : 0.f;
          sv[it][1] = on ? to_f(src[1]) : 0.f;
        }
      }
    };
    load_group(0);
    float cs[NP], sn[NP];
    if (p.use_table) {
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int pr = m * NP + k;
        const bool ok = lane_on && pr < half;
        cs[k] = ok ? __ldg(p.cost + p.tcbase + l * p.tcsl + pr) : 1.f;
        sn[k] = ok ? __ldg(p.sint + p.tsbase + l * p.tssl + pr) : 0.f;
      }
    } else {
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        if (lane_on && axis[k] >= 0) {
          const float cv = load_index_f(p.coords, p.coord_dtype,
                                        p.cbase + l * p.csl + axis[k] * p.csa);
          sincos_t<T>(__fmul_rn(cv, fr[k]), &sn[k], &cs[k]);
        } else {
          cs[k] = 1.f;
          sn[k] = 0.f;
        }
      }
    }
    for (int hb = 0; hb < p.H; hb += HPI * MAXIT) {
      if (hb > 0) load_group(hb);
#pragma unroll
      for (int it = 0; it < MAXIT; ++it) {
        if (hb + it * HPI >= p.H) break;  // warp-uniform
        const int h = hb + it * HPI + hg;
        const bool valid = h < p.H && lane_on;
        if constexpr (PK) {
          float c4[4], s4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) { c4[k] = cs[k]; s4[k] = sn[k]; }
          const uint4 o = rope3d_pk_chunk<T, LPH>(pk[it].u[0], c4, s4,
                                                  p.gamma ? gsm + h * p.D + m * EPL : nullptr, valid);
          if (valid) st_act_raw(reinterpret_cast<uint4*>(yt + int64_t(h) * p.ysh), o);
          continue;
        }
        float v[EPL];
        if constexpr (EPL == 8) unpack8<T>(pk[it], v);
        else { v[0] = sv[it][0]; v[1] = sv[it][1]; }
        if (p.gamma) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < EPL; ++i) ss += v[i] * v[i];
#pragma unroll
          for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          // 1 / clamp(||x||, 1e-12, 1e30) = rsqrt(clamp(||x||^2, 1e-24, 1e60)).
          const float rn = rsqrtf(fminf(fmaxf(ss, 1e-24f), 1e30f * 1e30f));
          if (valid) {
            const float* g = gsm + h * p.D + m * EPL;
            float gv[EPL];
            if constexpr (EPL == 8) {
              const float4 g0 = reinterpret_cast<const float4*>(g)[0];
              const float4 g1 = reinterpret_cast<const float4*>(g)[1];
              gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
              gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
            } else {
              gv[0] = g[0]; gv[1] = g[1];
            }
#pragma unroll
            for (int i = 0; i < EPL; ++i) v[i] = v[i] * rn * gv[i];
          }
        }
        float o[EPL];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const float re = v[2 * k], im = v[2 * k + 1];
          o[2 * k] = re * cs[k] - im * sn[k];
          o[2 * k + 1] = re * sn[k] + im * cs[k];
        }
        if (valid) {
          T* dst = yt + int64_t(h) * p.ysh;
          if constexpr (EPL == 8) store8<T>(dst, o);
          else { dst[0] = from_f<T>(o[0]); dst[1] = from_f<T>(o[1]); }
        }
      }
    }
  }
}

__global__ void rope3d_tables_kernel(int64_t L, const void* coords, int cdt, int64_t cbase,
                                     int64_t csl, int64_t csa, int half, int fd, float theta,
                                     float* cosp, float* sinp) {
  const int64_t total = L * half;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int pr = int(i % half);
    const int64_t l = i / half;
    const int a = fd > 0 ? pr / fd : 3;
    float cv = 1.f, sv = 0.f;
    if (a < 3) {
      const float f = inv_freq_f32(theta, float(pr - a * fd), float(fd));
      const float c = load_index_f(coords, cdt, cbase + l * csl + a * csa);
      sincosf(__fmul_rn(c, f), &sv, &cv);
    }
    cosp[i] = cv;
    sinp[i] = sv;
  }
}

// ================================================================== host side
static int head_view(const l3d_tensor* t, const char* op, const char* name, int64_t D,
                     HeadView* v) {
  if (!t || no_data(t)) return fail(L3D_E_NULL, "%s: %s is required", op, name);
  if (t->ndim != 4) return fail(L3D_E_SHAPE, "%s: %s must be rank 4", op, name);
  if (t->dims[3] != D) return fail(L3D_E_SHAPE, "%s: %s last dim must be %lld", op, name,
                                   (long long)D);
  if (t->strides[3] != 1) return fail(L3D_E_ALIGN, "%s: %s last dim must be contiguous", op, name);
  v->data = t->data;
  v->base = t->offset;
  return L3D_OK;
}

static bool aligned_view16(const l3d_tensor* t) {
  const int es = dtype_size(t->dtype);
  if ((reinterpret_cast<uintptr_t>(t->data) % 16) || ((t->offset * es) % 16)) return false;
  for (int i = 0; i < t->ndim - 1; ++i)
    if (t->dims[i] > 1 && (t->strides[i] * es) % 16) return false;
  return true;
}

static int launch_grid_warps(int64_t warps_needed) {
  const int64_t cap = int64_t(sm_count()) * 8 * 8;  // 8 blocks of 8 warps per SM
  int64_t blocks = (warps_needed + 7) / 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return int(blocks);
}

static int run_rope2d(const l3d_tensor* const* xs, const l3d_tensor* const* ws,
                      const l3d_tensor* const* bs, const l3d_tensor* const* outs, int ntensor,
                      float eps, int do_norm, const l3d_tensor* cosf_t, const l3d_tensor* sinf_t,
                      const l3d_tensor* positions, float theta, const char* op,
                      cudaStream_t stream) {
  Rope2dParams p{};
  const int dt = xs[0] ? xs[0]->dtype : -1;
  if (!xs[0]) return fail(L3D_E_NULL, "%s: x is required", op);
  if (!is_float_dtype(dt)) return fail(L3D_E_DTYPE, "%s: x must be F32/F16/BF16", op);
  p.B = xs[0]->dims[0];
  p.H = int(xs[0]->dims[1]);
  p.N = xs[0]->dims[2];
  p.ntensor = ntensor;
  p.do_norm = do_norm;
  p.eps = eps;
  int rc;
  for (int t = 0; t < ntensor; ++t) {
    if ((rc = head_view(xs[t], op, t ? "k" : "x", 64, &p.in[t]))) return rc;
    if ((rc = head_view(outs[t], op, t ? "k_out" : "out", 64, &p.out[t]))) return rc;
    for (int i = 0; i < 3; ++i)
      if (xs[t]->dims[i] != xs[0]->dims[i] || outs[t]->dims[i] != xs[0]->dims[i])
        return fail(L3D_E_SHAPE, "%s: q/k/out shapes differ", op);
    if (xs[t]->dtype != dt || outs[t]->dtype != dt)
      return fail(L3D_E_DTYPE, "%s: activation dtypes differ", op);
    if (!aligned_view16(xs[t]) || !aligned_view16(outs[t]))
      return fail(L3D_E_ALIGN, "%s: views must be 16-byte aligned", op);
    p.in[t].sb = xs[t]->strides[0]; p.in[t].sh = xs[t]->strides[1]; p.in[t].sn = xs[t]->strides[2];
    p.out[t].sb = outs[t]->strides[0]; p.out[t].sh = outs[t]->strides[1];
    p.out[t].sn = outs[t]->strides[2];
    bool al = true;
    if (do_norm) {
      if ((rc = make_chanvec(ws[t], "weight", 64, 1, &p.w[t], &al))) return rc;
      if ((rc = make_chanvec(bs[t], "bias", 64, 1, &p.b[t], &al))) return rc;
      if (!al) return fail(L3D_E_ALIGN, "%s: weight/bias must be 16-byte aligned", op);
    }
  }
  if (p.H > 4096) return fail(L3D_E_UNSUPPORTED, "%s: too many heads", op);
  if (p.B * p.N == 0 || p.H == 0) return L3D_OK;
  if (positions) {
    if (no_data(positions)) return fail(L3D_E_NULL, "%s: positions has no data", op);
    if (!is_index_dtype(positions->dtype))
      return fail(L3D_E_DTYPE, "%s: positions must be I32/I64/U32", op);
    if (positions->ndim != 3 || positions->dims[0] != p.B || positions->dims[1] != p.N ||
        positions->dims[2] != 2)
      return fail(L3D_E_SHAPE, "%s: positions must be [B, N, 2]", op);
    p.use_table = 0;
    p.pos = positions->data;
    p.pos_dtype = positions->dtype;
    p.pbase = positions->offset;
    p.psb = positions->strides[0];
    p.psn = positions->strides[1];
    p.psc = positions->strides[2];
    p.theta = theta;
  } else {
    const l3d_tensor* tabs[2] = {cosf_t, sinf_t};
    int64_t* bases[2] = {&p.cbase, &p.sbase};
    int64_t* sbs[2] = {&p.csb, &p.ssb};
    int64_t* sns[2] = {&p.csn, &p.ssn};
    for (int i = 0; i < 2; ++i) {
      const l3d_tensor* tb = tabs[i];
      if (!tb || no_data(tb)) return fail(L3D_E_NULL, "%s: cos/sin tables are required", op);
      if (tb->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: rope tables must be F32", op);
      // Accept [B, 1, N, 64] or [B, N, 64].
      int64_t tb_b, tb_n, tb_d, s_b, s_n, s_d;
      if (tb->ndim == 4 && tb->dims[1] == 1) {
        tb_b = tb->dims[0]; tb_n = tb->dims[2]; tb_d = tb->dims[3];
        s_b = tb->strides[0]; s_n = tb->strides[2]; s_d = tb->strides[3];
      } else if (tb->ndim == 3) {
        tb_b = tb->dims[0]; tb_n = tb->dims[1]; tb_d = tb->dims[2];
        s_b = tb->strides[0]; s_n = tb->strides[1]; s_d = tb->strides[2];
      } else {
        return fail(L3D_E_SHAPE, "%s: rope tables must be [B, 1, N, 64]", op);
      }
      if ((tb_b != p.B && tb_b != 1) || tb_n != p.N || tb_d != 64)
        return fail(L3D_E_SHAPE, "%s: rope table shape does not match x", op);
      if (s_d != 1) return fail(L3D_E_ALIGN, "%s: rope table last dim must be contiguous", op);
      *bases[i] = tb->offset;
      *sbs[i] = tb_b == 1 ? 0 : s_b;
      *sns[i] = s_n;
    }
    p.use_table = 1;
    p.cosp = static_cast<const float*>(cosf_t->data);
    p.sinp = static_cast<const float*>(sinf_t->data);
  }
  const int blocks = launch_grid_warps(p.B * p.N);
  L3D_DISPATCH_FLOAT(dt, T, { rope2d_kernel<T><<<blocks, 256, 0, stream>>>(p); });
  return check_launch(op);
}

}  // namespace l3d

using namespace l3d;

extern "C" int l3d_layernorm_rope2d(const l3d_tensor* x, const l3d_tensor* weight,
                                    const l3d_tensor* bias, float eps,
                                    const l3d_tensor* cos_full, const l3d_tensor* sin_alt_full,
                                    const l3d_tensor* out, l3d_stream stream) {
  const l3d_tensor* xs[2] = {x, nullptr};
  const l3d_tensor* ws[2] = {weight, nullptr};
  const l3d_tensor* bs[2] = {bias, nullptr};
  const l3d_tensor* os[2] = {out, nullptr};
  const int do_norm = (weight || bias) ? 1 : 0;
  return run_rope2d(xs, ws, bs, os, 1, eps, do_norm, cos_full, sin_alt_full, nullptr, 0.f,
                    "l3d_layernorm_rope2d", reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_qk_layernorm_rope2d_pos(const l3d_tensor* q, const l3d_tensor* q_weight,
                                           const l3d_tensor* q_bias, const l3d_tensor* k,
                                           const l3d_tensor* k_weight,
                                           const l3d_tensor* k_bias, float eps,
                                           const l3d_tensor* positions, float theta,
                                           const l3d_tensor* q_out, const l3d_tensor* k_out,
                                           l3d_stream stream) {
  const l3d_tensor* xs[2] = {q, k};
  const l3d_tensor* ws[2] = {q_weight, k_weight};
  const l3d_tensor* bs[2] = {q_bias, k_bias};
  const l3d_tensor* os[2] = {q_out, k_out};
  const int nt = k ? 2 : 1;
  if (k && !k_out) return fail(L3D_E_NULL, "l3d_qk_layernorm_rope2d_pos: k_out is required");
  if (!positions) return fail(L3D_E_NULL, "l3d_qk_layernorm_rope2d_pos: positions is required");
  const int do_norm = (q_weight || q_bias) ? 1 : 0;
  if (nt == 2 && do_norm != ((k_weight || k_bias) ? 1 : 0))
    return fail(L3D_E_UNSUPPORTED, "l3d_qk_layernorm_rope2d_pos: q and k must both be normed");
  return run_rope2d(xs, ws, bs, os, nt, eps, do_norm, nullptr, nullptr, positions, theta,
                    "l3d_qk_layernorm_rope2d_pos", reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_rope2d_tables(const l3d_tensor* positions, float theta, int head_dim,
                                 const l3d_tensor* cos_full, const l3d_tensor* sin_alt_full,
                                 l3d_stream stream) {
  const char* op = "l3d_rope2d_tables";
  if (!positions || !cos_full || !sin_alt_full || no_data(positions) || no_data(cos_full) ||
      no_data(sin_alt_full))
    return fail(L3D_E_NULL, "%s: positions, cos_full and sin_alt_full are required", op);
  if (head_dim <= 0 || head_dim % 4) return fail(L3D_E_SHAPE, "%s: head_dim must be a multiple of 4", op);
  if (!is_index_dtype(positions->dtype)) return fail(L3D_E_DTYPE, "%s: positions must be integer", op);
  if (positions->ndim != 3 || positions->dims[2] != 2)
    return fail(L3D_E_SHAPE, "%s: positions must be [B, N, 2]", op);
  const int64_t B = positions->dims[0], N = positions->dims[1];
  for (const l3d_tensor* t : {cos_full, sin_alt_full}) {
    if (t->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: tables must be F32", op);
    if (numel(t) != B * N * head_dim) return fail(L3D_E_SHAPE, "%s: table size mismatch", op);
    // Contiguity: strides must be the row-major strides of the dims.
    int64_t st = 1;
    for (int i = t->ndim - 1; i >= 0; --i) {
      if (t->dims[i] > 1 && t->strides[i] != st)
        return fail(L3D_E_ALIGN, "%s: tables must be contiguous", op);
      st *= t->dims[i];
    }
  }
  if (B * N == 0) return L3D_OK;
  const int64_t total = B * N * head_dim;
  int64_t blocks = (total + 255) / 256;
  if (blocks > int64_t(sm_count()) * 32) blocks = int64_t(sm_count()) * 32;
  rope2d_tables_kernel<<<int(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      B, N, positions->data, positions->dtype, positions->offset, positions->strides[0],
      positions->strides[1], positions->strides[2], theta, head_dim,
      static_cast<float*>(cos_full->data) + cos_full->offset,
      static_cast<float*>(sin_alt_full->data) + sin_alt_full->offset);
  return check_launch(op);
}

// --------------------------------------------------------------------- 3D host
static int run_rope3d(const l3d_tensor* x, const l3d_tensor* gamma, const l3d_tensor* coords,
                      float theta, const l3d_tensor* cos_t, const l3d_tensor* sin_t,
                      const l3d_tensor* y, const char* op, cudaStream_t stream) {
  if (!x || !y || no_data(x) || no_data(y)) return fail(L3D_E_NULL, "%s: x and y are required", op);
  if (!is_float_dtype(x->dtype) || y->dtype != x->dtype)
    return fail(L3D_E_DTYPE, "%s: x/y must share a float dtype", op);
  if (x->ndim != 4 || y->ndim != 4) return fail(L3D_E_SHAPE, "%s: x/y must be [B, L, H, D]", op);
  for (int i = 0; i < 4; ++i)
    if (x->dims[i] != y->dims[i]) return fail(L3D_E_SHAPE, "%s: x/y shapes differ", op);
  if (x->strides[3] != 1 || y->strides[3] != 1)
    return fail(L3D_E_ALIGN, "%s: last dim must be contiguous", op);
  Rope3dParams p{};
  p.B = x->dims[0]; p.L = x->dims[1]; p.H = int(x->dims[2]); p.D = int(x->dims[3]);
  if (p.D % 2) return fail(L3D_E_SHAPE, "%s: head dim must be even", op);
  p.x = x->data; p.xbase = x->offset;
  p.xsb = x->strides[0]; p.xsl = x->strides[1]; p.xsh = x->strides[2];
  p.y = y->data; p.ybase = y->offset;
  p.ysb = y->strides[0]; p.ysl = y->strides[1]; p.ysh = y->strides[2];
  p.freq_dim = p.D / 2 / 3;
  p.theta = theta;
  p.scale = sqrtf(float(p.D));
  if (gamma) {
    if (no_data(gamma)) return fail(L3D_E_NULL, "%s: gamma has no data", op);
    if (gamma->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: gamma must be F32", op);
    if (gamma->ndim != 2 || gamma->dims[0] != p.H || gamma->dims[1] != p.D)
      return fail(L3D_E_SHAPE, "%s: gamma must be [H, D]", op);
    if (gamma->strides[1] != 1) return fail(L3D_E_ALIGN, "%s: gamma must be contiguous", op);
    p.gamma = static_cast<const float*>(gamma->data) + gamma->offset;
    p.gsh = gamma->strides[0];
  }
  if (coords) {
    if (no_data(coords)) return fail(L3D_E_NULL, "%s: coords has no data", op);
    if (coords->dtype != L3D_I32 && coords->dtype != L3D_I64)
      return fail(L3D_E_DTYPE, "%s: coords must be I32/I64", op);
    if (coords->ndim != 2 || coords->dims[0] != p.L || coords->dims[1] != 3)
      return fail(L3D_E_SHAPE, "%s: coords must be [L, 3]", op);
    if (p.freq_dim == 0) return fail(L3D_E_SHAPE, "%s: head dim too small for 3-axis RoPE", op);
    p.coords = coords->data; p.coord_dtype = coords->dtype; p.cbase = coords->offset;
    p.csl = coords->strides[0]; p.csa = coords->strides[1];
  } else if (!cos_t && !sin_t) {
    // Normalisation only (Trellis2QkRmsNorm without the rotation).
    if (!gamma) return fail(L3D_E_NULL, "%s: nothing to do without gamma and coords", op);
  } else {
    for (const l3d_tensor* t : {cos_t, sin_t}) {
      if (!t || no_data(t)) return fail(L3D_E_NULL, "%s: cos/sin tables are required", op);
      if (t->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: tables must be F32", op);
      if (t->ndim != 2 || t->dims[0] != p.L || t->dims[1] != p.D / 2)
        return fail(L3D_E_SHAPE, "%s: tables must be [L, D/2]", op);
      if (t->strides[1] != 1) return fail(L3D_E_ALIGN, "%s: tables must be contiguous rows", op);
    }
    p.use_table = 1;
    p.cost = static_cast<const float*>(cos_t->data); p.tcbase = cos_t->offset;
    p.tcsl = cos_t->strides[0];
    p.sint = static_cast<const float*>(sin_t->data); p.tsbase = sin_t->offset;
    p.tssl = sin_t->strides[0];
  }
  if (p.B * p.L == 0 || p.H == 0) return L3D_OK;
  const bool fast = (p.D % 8 == 0) && p.D <= 256 && aligned_view16(x) && aligned_view16(y);
  const size_t smem = p.gamma ? size_t(p.H) * size_t(p.D) * sizeof(float) : 0;
  if (smem > 48 * 1024) return fail(L3D_E_UNSUPPORTED, "%s: gamma [H, D] above 12288 values", op);
  const int blocks = launch_grid_warps(p.B * p.L);
  if (fast) {
    const int lph = p.D / 8 <= 4 ? 4 : p.D / 8 <= 8 ? 8 : p.D / 8 <= 16 ? 16 : 32;
    L3D_DISPATCH_FLOAT(x->dtype, T, {
      switch (lph) {
        case 4: rope3d_kernel<T, 8, 4><<<blocks, 256, smem, stream>>>(p); break;
        case 8: rope3d_kernel<T, 8, 8><<<blocks, 256, smem, stream>>>(p); break;
        case 16: rope3d_kernel<T, 8, 16><<<blocks, 256, smem, stream>>>(p); break;
        default: rope3d_kernel<T, 8, 32><<<blocks, 256, smem, stream>>>(p); break;
      }
    });
  } else {
    if (p.D > 64) return fail(L3D_E_UNSUPPORTED, "%s: unaligned head dim > 64", op);
    const int pairs = p.D / 2;
    const int lph = pairs <= 4 ? 4 : pairs <= 8 ? 8 : pairs <= 16 ? 16 : 32;
    L3D_DISPATCH_FLOAT(x->dtype, T, {
      switch (lph) {
        case 4: rope3d_kernel<T, 2, 4><<<blocks, 256, smem, stream>>>(p); break;
        case 8: rope3d_kernel<T, 2, 8><<<blocks, 256, smem, stream>>>(p); break;
        case 16: rope3d_kernel<T, 2, 16><<<blocks, 256, smem, stream>>>(p); break;
        default: rope3d_kernel<T, 2, 32><<<blocks, 256, smem, stream>>>(p); break;
      }
    });
  }
  return check_launch(op);
}

extern "C" int l3d_qk_l2norm_rope3d(const l3d_tensor* x, const l3d_tensor* gamma,
                                    const l3d_tensor* coords, float theta, const l3d_tensor* y,
                                    l3d_stream stream) {
  return run_rope3d(x, gamma, coords, theta, nullptr, nullptr, y, "l3d_qk_l2norm_rope3d",
                    reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_rope3d_apply(const l3d_tensor* x, const l3d_tensor* cos_t,
                                const l3d_tensor* sin_t, const l3d_tensor* y,
                                l3d_stream stream) {
  return run_rope3d(x, nullptr, nullptr, 0.f, cos_t, sin_t, y, "l3d_rope3d_apply",
                    reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int l3d_rope3d_tables(const l3d_tensor* coords, int head_dim, float theta,
                                 const l3d_tensor* cos_out, const l3d_tensor* sin_out,
                                 l3d_stream stream) {
  const char* op = "l3d_rope3d_tables";
  if (!coords || !cos_out || !sin_out || no_data(coords) || no_data(cos_out) || no_data(sin_out))
    return fail(L3D_E_NULL, "%s: coords, cos and sin are required", op);
  if (head_dim <= 0 || head_dim % 2) return fail(L3D_E_SHAPE, "%s: head_dim must be even", op);
  const int fd = head_dim / 2 / 3;
  if (fd == 0) return fail(L3D_E_SHAPE, "%s: head_dim too small for 3-axis RoPE", op);
  if (coords->dtype != L3D_I32 && coords->dtype != L3D_I64)
    return fail(L3D_E_DTYPE, "%s: coords must be I32/I64", op);
  if (coords->ndim != 2 || coords->dims[1] != 3) return fail(L3D_E_SHAPE, "%s: coords [L, 3]", op);
  const int64_t L = coords->dims[0];
  const int half = head_dim / 2;
  for (const l3d_tensor* t : {cos_out, sin_out}) {
    if (t->dtype != L3D_F32) return fail(L3D_E_DTYPE, "%s: tables must be F32", op);
    if (t->ndim != 2 || t->dims[0] != L || t->dims[1] != half)
      return fail(L3D_E_SHAPE, "%s: tables must be [L, head_dim/2]", op);
    if ((half > 1 && t->strides[1] != 1) || (L > 1 && t->strides[0] != half))
      return fail(L3D_E_ALIGN, "%s: tables must be contiguous", op);
  }
  if (L == 0) return L3D_OK;
  int64_t blocks = (L * half + 255) / 256;
  if (blocks > int64_t(sm_count()) * 32) blocks = int64_t(sm_count()) * 32;
  rope3d_tables_kernel<<<int(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      L, coords->data, coords->dtype, coords->offset, coords->strides[0], coords->strides[1],
      half, fd, theta, static_cast<float*>(cos_out->data) + cos_out->offset,
      static_cast<float*>(sin_out->data) + sin_out->offset);
  return check_launch(op);
}
