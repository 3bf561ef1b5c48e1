// GGML Q8_0 / Q4_0 block decoding (l3d_dequantize) and the dequant-linear
// entry point.
//
// Block layouts (GGML public format, 32 weights per block):
//   Q8_0: { f16 d; int8 q[32]; }        34 bytes, w[j] = d * q[j]
//   Q4_0: { f16 d; uint8 qs[16]; }      18 bytes, w[j] = d * ((qs[j] & 15) - 8),
//                                                  w[16 + j] = d * ((qs[j] >> 4) - 8)
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

int launch_dequantize(const void* wq, int fmt, int64_t n, int64_t k, int out_dtype, void* out,
                      cudaStream_t s) {
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
  if (fmt != L3D_Q8_0 && fmt != L3D_Q4_0) return fail(L3D_E_UNSUPPORTED, "%s: unknown format", op);
  if (n < 0 || k < 0 || k % 32) return fail(L3D_E_SHAPE, "%s: k must be a multiple of 32", op);
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
