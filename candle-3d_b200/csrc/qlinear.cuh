// Shared declarations of the dequant-linear path (block decoding + tensor-core
// GEMM).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "l3d_ops.h"

namespace l3d {

// Bytes and weights per block of each GGML format (0 for an unknown format).
__host__ __device__ inline int block_bytes(int fmt) {
  switch (fmt) {
    case L3D_Q8_0: return 34;
    case L3D_Q4_0: return 18;
    case L3D_Q4_K: return 144;
    case L3D_Q5_K: return 176;
    case L3D_Q6_K: return 210;
    default: return 0;
  }
}
__host__ __device__ inline int block_elems(int fmt) {
  return (fmt == L3D_Q4_K || fmt == L3D_Q5_K || fmt == L3D_Q6_K) ? 256 : 32;
}
__host__ __device__ inline bool is_kquant(int fmt) { return block_elems(fmt) == 256; }
__host__ __device__ inline bool qfmt_known(int fmt) { return block_bytes(fmt) != 0; }

// Decode an [n, k] block matrix into a contiguous [n, k] tensor of out_dtype.
int launch_dequantize(const void* wq, int fmt, int64_t n, int64_t k, int out_dtype, void* out,
                      cudaStream_t s);

}  // namespace l3d
