// Activation functions shared by the elementwise kernels and the GEMV /
// patch-embedding epilogues.
#pragma once
#include <cuda_runtime.h>

namespace l3d {

enum Act { ACT_NONE = 0, ACT_SILU = 1, ACT_GELU_ERF = 2, ACT_GELU_TANH = 3 };

// GELU tanh approximation (Hendrycks & Gimpel 2016): the published constants
// sqrt(2/pi) and 0.044715, evaluated in f32 like Candle's unary `gelu`.
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}
// Exact GELU: x * Phi(x) = 0.5 x (1 + erf(x / sqrt(2))).
__device__ __forceinline__ float gelu_erf_f(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}
// SiLU: x * sigmoid(x) = x / (1 + exp(-x)).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <int A>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (A == ACT_SILU) return silu_f(x);
  else if constexpr (A == ACT_GELU_ERF) return gelu_erf_f(x);
  else if constexpr (A == ACT_GELU_TANH) return gelu_tanh_f(x);
  else return x;
}
__device__ __forceinline__ float act_dyn(int a, float x) {
  switch (a) {
    case ACT_SILU: return silu_f(x);
    case ACT_GELU_ERF: return gelu_erf_f(x);
    case ACT_GELU_TANH: return gelu_tanh_f(x);
    default: return x;
  }
}

}  // namespace l3d
