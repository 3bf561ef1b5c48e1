// GGML block decoding (l3d_dequantize) for the dequant-linear path.
//
// Block layouts (GGML public format), 32 weights per block:
//   Q8_0: { f16 d; int8 q[32]; }        34 bytes, w[j] = d * q[j]
//   Q4_0: { f16 d; uint8 qs[16]; }      18 bytes, w[j] = d * ((qs[j] & 15) - 8),
//                                                  w[16 + j] = d * ((qs[j] >> 4) - 8)
// and 256 weights per super-block (the K-quants):
//   Q4_K: { f16 d; f16 dmin; u8 scales[12]; u8 qs[128]; }            144 bytes
//   Q5_K: { f16 d; f16 dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]; } 176 bytes
//   Q6_K: { u8 ql[128]; u8 qh[64]; int8 scales[16]; f16 d; }        210 bytes
// Q4_K / Q5_K: the super-block is 4 chunks of 64 weights; chunk c holds
// sub-blocks 2c (low nibbles of qs[32c .. 32c+31]) and 2c+1 (high nibbles);
// Q5_K adds bit (2c + half) of qh[l] as the fifth bit (+16).  Sub-block j has
// a 6-bit scale sc and min m packed in scales[12]: for j < 4, sc = s[j] & 63,
// m = s[j+4] & 63; else sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,
// m = (s[j+4] >> 4) | (s[j] >> 6) << 4.  w = (d * sc) * q - (dmin * m).
// Q6_K: two halves of 128; in half n, element 32g + l (g = 0..3, l < 32) is
// q = (nibble | (bits 2g, 2g+1 of qh[32n + l]) << 4) - 32, the nibble being
// the low (g < 2) or high (g >= 2) one of ql[64n + l + 32 (g & 1)], with scale
// scales[8n + l/16 + 2g]; w = (d * sc) * q.
// The f32 operations are done in that order without contraction, so the
// decoded values equal the CPU decode of the same bytes.
#include "common.cuh"
#include "qlinear.cuh"

namespace l3d {

__device__ __forceinline__ float half_bits_to_f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// Decode one 32-weight block into f32 (unaligned byte source: blocks are 34 /
// 18 bytes, so only 2-byte alignment is guaranteed).
__device__ __forceinline__ void decode_block(const uint8_t* blk, int fmt, float (&w)[32]) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(blk);  // 2-byte aligned
  const float d = half_bits_to_f(__ldg(h));
  if (fmt == L3D_Q8_0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint16_t v = __ldg(h + 1 + j);
      w[2 * j] = d * float(int8_t(v & 0xff));
      w[2 * j + 1] = d * float(int8_t(v >> 8));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint16_t v = __ldg(h + 1 + j);
      const uint8_t q0 = v & 0xff, q1 = v >> 8;
      w[2 * j] = d * float(int(q0 & 15) - 8);
      w[2 * j + 1] = d * float(int(q1 & 15) - 8);
      w[16 + 2 * j] = d * float(int(q0 >> 4) - 8);
      w[16 + 2 * j + 1] = d * float(int(q1 >> 4) - 8);
    }
  }
}

template <typename TO>
__global__ void dequantize_kernel(const uint8_t* __restrict__ wq, int fmt, int64_t n, int64_t k,
                                  TO* __restrict__ out) {
  const int bb = block_bytes(fmt);
  const int64_t kb = k / 32;
  const int64_t nblk = n * kb;
  for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nblk;
       b += int64_t(gridDim.x) * blockDim.x) {
    float w[32];
    decode_block(wq + b * bb, fmt, w);
    // Row-major [n, k]: block b is the 32 consecutive elements at b * 32,
    // written as 16-byte vectors (the output is 16-byte aligned).
    TO* o = out + b * 32;
    constexpr int V = Vec16<TO>::N;
#pragma unroll
    for (int j = 0; j < 32; j += V) {
      float f[V];
#pragma unroll
      for (int e = 0; e < V; ++e) f[e] = w[j + e];
      *reinterpret_cast<uint4*>(o + j) = pack(f, TO());
    }
  }
}

// ------------------------------------------------------------------ K-quants
__device__ __forceinline__ uint8_t ldb(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ float ld_half_f(const uint8_t* p) {
  return half_bits_to_f(uint16_t(ldb(p)) | uint16_t(ldb(p + 1)) << 8);
}
// 6-bit scale and min of sub-block j (0..7) of a Q4_K / Q5_K super-block.
__device__ __forceinline__ void kq_scale_min(const uint8_t* sc, int j, int& s, int& m) {
  if (j < 4) {
    s = ldb(sc + j) & 63;
    m = ldb(sc + j + 4) & 63;
  } else {
    s = (ldb(sc + j + 4) & 15) | ((ldb(sc + j - 4) >> 6) << 4);
    m = (ldb(sc + j + 4) >> 4) | ((ldb(sc + j) >> 6) << 4);
  }
}

// Weights 8L .. 8L+7 of one super-block (lane L of a warp).
__device__ __forceinline__ void decode_kq8(const uint8_t* sb, int fmt, int L, float (&w)[8]) {
  if (fmt == L3D_Q6_K) {
    const int base = 8 * L;
    const int n = base >> 7, r = base & 127, g = r >> 5, l0 = r & 31;
    const uint8_t* ql = sb + 64 * n + l0 + ((g & 1) ? 32 : 0);
    const uint8_t* qh = sb + 128 + 32 * n + l0;
    const float sc = float(int8_t(ldb(sb + 192 + 8 * n + (l0 >> 4) + 2 * g)));
    const float d = ld_half_f(sb + 208);
    const float ds = __fmul_rn(d, sc);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int lo = g < 2 ? (ldb(ql + t) & 15) : (ldb(ql + t) >> 4);
      const int hi = (ldb(qh + t) >> (2 * g)) & 3;
      w[t] = __fmul_rn(ds, float((lo | (hi << 4)) - 32));
    }
    return;
  }
  // Q4_K / Q5_K
  const int c = L >> 3, p = (8 * L) & 63, half = p >> 5, off = p & 31;
  int sc, mn;
  kq_scale_min(sb + 4, 2 * c + half, sc, mn);
  const float d1 = __fmul_rn(ld_half_f(sb), float(sc));
  const float m1 = __fmul_rn(ld_half_f(sb + 2), float(mn));
  const bool q5 = fmt == L3D_Q5_K;
  const uint8_t* qs = sb + (q5 ? 48 : 16) + 32 * c + off;
  const uint8_t* qh = sb + 16 + off;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    int q = half ? (ldb(qs + t) >> 4) : (ldb(qs + t) & 15);
    if (q5) q += ((ldb(qh + t) >> (2 * c + half)) & 1) << 4;
    w[t] = __fsub_rn(__fmul_rn(d1, float(q)), m1);
  }
}

// One warp per super-block; each lane writes 8 consecutive outputs.
template <typename TO>
__global__ void dequantize_kq_kernel(const uint8_t* __restrict__ wq, int fmt, int64_t nsb,
                                     TO* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int bb = block_bytes(fmt);
  for (int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; b < nsb;
       b += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    float w[8];
    decode_kq8(wq + b * bb, fmt, lane, w);
    TO* o = out + b * 256 + 8 * lane;
    if constexpr (sizeof(TO) == 2) {
      *reinterpret_cast<uint4*>(o) = pack(w, TO());
    } else {
      float a[4] = {w[0], w[1], w[2], w[3]}, c[4] = {w[4], w[5], w[6], w[7]};
      reinterpret_cast<uint4*>(o)[0] = pack(a, TO());
      reinterpret_cast<uint4*>(o)[1] = pack(c, TO());
    }
  }
}

int launch_dequantize(const void* wq, int fmt, int64_t n, int64_t k, int out_dtype, void* out,
                      cudaStream_t s) {
  if (is_kquant(fmt)) {
    const int64_t nsb = n * (k / 256);
    if (nsb == 0) return L3D_OK;
    int64_t blocks = (nsb + 7) / 8;  // 8 warps per block
    if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
    const uint8_t* q = static_cast<const uint8_t*>(wq);
    L3D_DISPATCH_FLOAT(out_dtype, TO, {
      dequantize_kq_kernel<TO><<<int(blocks), 256, 0, s>>>(q, fmt, nsb, static_cast<TO*>(out));
    });
    return check_launch("dequantize");
  }
  const int64_t nblk = n * (k / 32);
  if (nblk == 0) return L3D_OK;
  int64_t blocks = (nblk + 255) / 256;
  if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
  const uint8_t* q = static_cast<const uint8_t*>(wq);
  L3D_DISPATCH_FLOAT(out_dtype, TO, {
    dequantize_kernel<TO><<<int(blocks), 256, 0, s>>>(q, fmt, n, k, static_cast<TO*>(out));
  });
  return check_launch("dequantize");
}

}  // namespace l3d

using namespace l3d;

extern "C" int l3d_dequantize(const void* wq, int fmt, int64_t n, int64_t k,
                              const l3d_tensor* out, l3d_stream stream) {
  const char* op = "l3d_dequantize";
  if (!wq || !out || no_data(out)) return fail(L3D_E_NULL, "%s: wq and out are required", op);
  if (!qfmt_known(fmt)) return fail(L3D_E_UNSUPPORTED, "%s: unknown format", op);
  if (n < 0 || k < 0 || k % block_elems(fmt))
    return fail(L3D_E_SHAPE, "%s: k must be a multiple of %d", op, block_elems(fmt));
  if (!is_float_dtype(out->dtype)) return fail(L3D_E_DTYPE, "%s: out must be a float dtype", op);
  if (out->ndim != 2 || out->dims[0] != n || out->dims[1] != k)
    return fail(L3D_E_SHAPE, "%s: out must be [n, k]", op);
  if ((k > 1 && out->strides[1] != 1) || (n > 1 && out->strides[0] != k))
    return fail(L3D_E_ALIGN, "%s: out must be contiguous", op);
  if (reinterpret_cast<uintptr_t>(wq) % 2) return fail(L3D_E_ALIGN, "%s: wq must be 2-byte aligned", op);
  if (reinterpret_cast<uintptr_t>(elem_ptr(out)) % 16)
    return fail(L3D_E_ALIGN, "%s: out must be 16-byte aligned", op);
  return launch_dequantize(wq, fmt, n, k, out->dtype,
                           const_cast<char*>(elem_ptr(out)), reinterpret_cast<cudaStream_t>(stream));
}
