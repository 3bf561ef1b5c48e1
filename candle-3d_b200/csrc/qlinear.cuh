// Shared declarations of the dequant-linear path (block decoding + tensor-core
// GEMM).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "l3d_ops.h"

namespace l3d {

__host__ __device__ inline int block_bytes(int fmt) { return fmt == L3D_Q8_0 ? 34 : 18; }

// Decode an [n, k] block matrix into a contiguous [n, k] tensor of out_dtype.
int launch_dequantize(const void* wq, int fmt, int64_t n, int64_t k, int out_dtype, void* out,
                      cudaStream_t s);

}  // namespace l3d
