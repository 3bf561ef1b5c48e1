// Shared device/host helpers for libl3dops: dtype handling, 16-byte vector
// I/O, row addressing for Candle-style strided layouts, status plumbing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "l3d_ops.h"

namespace l3d {

// ---------------------------------------------------------------- host status
// Set the thread-local error message and return `code`.
int fail(int code, const char* fmt, ...);
// Map a CUDA error from a launch to L3D_E_CUDA (or L3D_OK).
int check_launch(const char* what);

inline bool is_float_dtype(int dt) { return dt == L3D_F32 || dt == L3D_F16 || dt == L3D_BF16; }
inline bool is_index_dtype(int dt) { return dt == L3D_I32 || dt == L3D_I64 || dt == L3D_U32; }
inline int dtype_size(int dt) {
  switch (dt) {
    case L3D_F32: case L3D_I32: case L3D_U32: return 4;
    case L3D_F16: case L3D_BF16: return 2;
    case L3D_I64: return 8;
    case L3D_U8: return 1;
    default: return 0;
  }
}
const char* dtype_name(int dt);

// Number of SMs of the current device (cached per device).
int sm_count();
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (device, kernel): the attribute belongs to the device
// context, so a process that drives several GPUs sets it on each.  Returns
// the result of the first attempt on this device.
cudaError_t set_smem_limit(const void* kernel, int bytes);
// Per-device status word of the kernels that take no workspace (the
// row-norm ring kernel): copy to *status, clear when reset != 0.
cudaError_t norm_status_read(int* status, int reset);

// Byte address of the first element of a view.
inline const char* elem_ptr(const l3d_tensor* t) {
  return static_cast<const char*>(t->data) + t->offset * dtype_size(t->dtype);
}
inline int64_t numel(const l3d_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->dims[i];
  return n;
}
// A view that holds elements but no storage pointer (empty views may carry
// a null pointer, as torch / Candle empty tensors do).
inline bool no_data(const l3d_tensor* t) { return !t->data && numel(t) != 0; }

// --------------------------------------------------------------- row mapping
// Maps a flat row index over the leading dims of a view to an element offset.
// Leading dims are collapsed on the host wherever strides allow, so the common
// contiguous case costs one multiply per row.
struct RowMap {
  int nd;               // number of (collapsed) leading dims, 1..5
  int64_t dims[5];      // outermost first
  int64_t strides[5];   // element strides
  int64_t base;         // element offset of row 0
};

// Build a RowMap over dims [0, lead) of `t`.  Returns false when lead > 5
// after collapsing.
bool make_rowmap(const l3d_tensor* t, int lead, RowMap* m);
// True when every leading stride and the base offset are multiples of `elems`.
bool rowmap_aligned(const RowMap& m, int64_t elems);

__device__ __forceinline__ int64_t row_offset(const RowMap& m, int64_t r) {
  int64_t off = m.base;
#pragma unroll
  for (int i = 4; i >= 1; --i) {
    if (i < m.nd) {
      const int64_t d = m.dims[i];
      const int64_t q = r / d;
      off += (r - q * d) * m.strides[i];
      r = q;
    }
  }
  return off + r * m.strides[0];
}

// -------------------------------------------------------------- dtype traits
template <typename T> struct Vec16;
template <> struct Vec16<float> { static constexpr int N = 4; };
template <> struct Vec16<__nv_bfloat16> { static constexpr int N = 8; };
template <> struct Vec16<__half> { static constexpr int N = 8; };

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Unpack a 16-byte pack into floats.
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[4], float) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[8], __nv_bfloat16) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[8], __half) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x; f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack(const float (&f)[4], float) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
__device__ __forceinline__ uint4 pack(const float (&f)[8], __nv_bfloat16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint4 pack(const float (&f)[8], __half) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Activation loads and stores of the streaming kernels: plain cached
// accesses.  The evict-first (.cs) hints were measured slower on B200 for
// these read-once / write-once sweeps (GELU 5.9 -> 6.3 TB/s without them).
template <typename V>
__device__ __forceinline__ V ld_act_raw(const V* p) { return *p; }
template <typename V>
__device__ __forceinline__ void st_act_raw(V* p, const V& v) { *p = v; }

// Packed f32x2 arithmetic (FADD2 / FMUL2 / FFMA2 on sm_100): two independent
// IEEE round-to-nearest operations per instruction, so element-wise work in
// the HBM-bound kernels costs half the issue slots.
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// A 16-byte pack as float pairs (2 pairs of f32, or 4 pairs of 16-bit).
__device__ __forceinline__ void unpack2(const uint4& u, float2 (&f)[2], float) {
  f[0] = make_float2(__uint_as_float(u.x), __uint_as_float(u.y));
  f[1] = make_float2(__uint_as_float(u.z), __uint_as_float(u.w));
}
__device__ __forceinline__ void unpack2(const uint4& u, float2 (&f)[4], __nv_bfloat16) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    f[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
}
__device__ __forceinline__ void unpack2(const uint4& u, float2 (&f)[4], __half) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
}
__device__ __forceinline__ uint4 pack2(const float2 (&f)[2], float) {
  return make_uint4(__float_as_uint(f[0].x), __float_as_uint(f[0].y), __float_as_uint(f[1].x),
                    __float_as_uint(f[1].y));
}
__device__ __forceinline__ uint4 pack2(const float2 (&f)[4], __nv_bfloat16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __float22bfloat162_rn(f[i]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint4 pack2(const float2 (&f)[4], __half) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __float22half2_rn(f[i]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
// P consecutive float pairs of an f32 array in shared or global memory
// (16-byte aligned).
template <int P>
__device__ __forceinline__ void ld_pairs(const float* p, float2 (&f)[P]) {
#pragma unroll
  for (int i = 0; i < P; i += 2) {
    const float4 t = *reinterpret_cast<const float4*>(p + 2 * i);
    f[i] = make_float2(t.x, t.y);
    f[i + 1] = make_float2(t.z, t.w);
  }
}

// Load / store VEC consecutive elements as floats.  VEC == Vec16<T>::N uses a
// single 16-byte access; VEC == 1 is the scalar path for ragged shapes.
template <typename T, int VEC>
__device__ __forceinline__ void load_act(const T* p, float (&f)[VEC]) {
  if constexpr (VEC == Vec16<T>::N) {
    uint4 u = ld_act_raw(reinterpret_cast<const uint4*>(p));
    unpack(u, f, T());
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f(p[i]);
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void load_reuse(const T* p, float (&f)[VEC]) {
  if constexpr (VEC == Vec16<T>::N) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    unpack(u, f, T());
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f(p[i]);
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void store_act(T* p, const float (&f)[VEC]) {
  if constexpr (VEC == Vec16<T>::N) {
    st_act_raw(reinterpret_cast<uint4*>(p), pack(f, T()));
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = from_f<T>(f[i]);
  }
}

// Per-channel parameter vector of any float dtype: [C], [B, C] or [B, 1, C]
// (batch stride 0 = broadcast over batches).  Loaded VEC elements at a time.
struct ChanVec {
  const void* ptr;      // address of element (batch 0, channel 0); null = absent
  int64_t bstride;      // element stride between batches
  int dtype;
};

template <int VEC>
__device__ __forceinline__ void load_chan(const ChanVec& v, int64_t b, int64_t c0,
                                          float (&f)[VEC]) {
  const int64_t off = b * v.bstride + c0;
  if (v.dtype == L3D_F32) {
    const float* p = static_cast<const float*>(v.ptr) + off;
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int i = 0; i < VEC; i += 4) {
        float4 t = __ldg(reinterpret_cast<const float4*>(p + i));
        f[i] = t.x; f[i + 1] = t.y; f[i + 2] = t.z; f[i + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) f[i] = __ldg(p + i);
    }
  } else if (v.dtype == L3D_BF16) {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(v.ptr) + off;
    if constexpr (VEC == 8) {
      unpack(__ldg(reinterpret_cast<const uint4*>(p)), f, __nv_bfloat16());
    } else if constexpr (VEC == 4) {
      uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
      f[0] = __uint_as_float(u.x << 16); f[1] = __uint_as_float(u.x & 0xffff0000u);
      f[2] = __uint_as_float(u.y << 16); f[3] = __uint_as_float(u.y & 0xffff0000u);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) f[i] = __bfloat162float(p[i]);
    }
  } else {
    const __half* p = static_cast<const __half*>(v.ptr) + off;
    if constexpr (VEC == 8) {
      unpack(__ldg(reinterpret_cast<const uint4*>(p)), f, __half());
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) f[i] = __half2float(p[i]);
    }
  }
}

// Builds a ChanVec from a [C], [B, C] or [B, 1, C] view (last stride 1).
// Returns 0 or an error status; `vec_elems` is the access width the kernel
// will use (alignment checked against it).
int make_chanvec(const l3d_tensor* t, const char* name, int64_t C, int64_t B, ChanVec* out,
                 bool* aligned16);

}  // namespace l3d

// Dispatch helper over float activation dtypes.
#define L3D_DISPATCH_FLOAT(DT, T, ...)                                  \
  do {                                                                  \
    if ((DT) == L3D_F32) { using T = float; __VA_ARGS__; }              \
    else if ((DT) == L3D_BF16) { using T = __nv_bfloat16; __VA_ARGS__; } \
    else { using T = __half; __VA_ARGS__; }                             \
  } while (0)
