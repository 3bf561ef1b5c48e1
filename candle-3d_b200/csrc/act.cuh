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

// ---- reduced-cost forms for 16-bit outputs ---------------------------------
// Their absolute errors (below ~2e-6 relative to |x| for GELU, ~5e-4 relative
// for tanh) are far inside half an ulp of bf16 / f16, so the rounded output is
// the same as (or one ulp from) the accurate form's.
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ex2_hw(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_hw(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanh_hw(k0 * x * (1.0f + k1 * x * x)));
}
// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.26 (|error| <= 1.5e-7): erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^{-z^2},
// t = 1 / (1 + p z), z >= 0, odd extension for z < 0.
__device__ __forceinline__ float erf_as(float z) {
  const float a = fabsf(z);
  const float t = rcp_hw(1.0f + 0.3275911f * a);
  const float poly =
      t * (0.254829592f +
           t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  const float e = ex2_hw(-a * a * 1.4426950408889634f);  // e^{-a^2}
  return copysignf(1.0f - poly * e, z);
}
__device__ __forceinline__ float gelu_erf_fast(float x) {
  return 0.5f * x * (1.0f + erf_as(x * 0.7071067811865476f));
}
__device__ __forceinline__ float silu_fast(float x) {
  return x * rcp_hw(1.0f + ex2_hw(-x * 1.4426950408889634f));
}

template <int A>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (A == ACT_SILU) return silu_f(x);
  else if constexpr (A == ACT_GELU_ERF) return gelu_erf_f(x);
  else if constexpr (A == ACT_GELU_TANH) return gelu_tanh_f(x);
  else return x;
}
// FAST selects the reduced-cost forms (used when the output is 16-bit).
template <int A, bool FAST>
__device__ __forceinline__ float act_t(float x) {
  if constexpr (!FAST) return act_f<A>(x);
  else if constexpr (A == ACT_SILU) return silu_fast(x);
  else if constexpr (A == ACT_GELU_ERF) return gelu_erf_fast(x);
  else if constexpr (A == ACT_GELU_TANH) return gelu_tanh_fast(x);
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
__device__ __forceinline__ float act_dyn_fast(int a, float x) {
  switch (a) {
    case ACT_SILU: return silu_fast(x);
    case ACT_GELU_ERF: return gelu_erf_fast(x);
    case ACT_GELU_TANH: return gelu_tanh_fast(x);
    default: return x;
  }
}

}  // namespace l3d
