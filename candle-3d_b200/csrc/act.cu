// Elementwise activations: GELU (tanh form), GELU (erf form), SiLU, GeGLU.
// Contiguous tensors run a flat, 16-byte vectorised grid-stride loop with
// several independent vectors per thread in flight; strided views and GeGLU
// run a row kernel over the Candle layout.
#include "act.cuh"
#include "common.cuh"

namespace l3d {

constexpr int kUnroll = 4;

// Flat contiguous kernel: n elements, vectorised when VEC > 1.
template <typename T, int VEC, int A>
__global__ void __launch_bounds__(256) act_flat_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                       int64_t n) {
  const int64_t nvec = n / VEC;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
    float v[kUnroll][VEC];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) load_act<T, VEC>(x + (i + u * stride) * VEC, v[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) v[u][e] = act_t<A, (sizeof(T) == 2)>(v[u][e]);
      store_act<T, VEC>(y + (i + u * stride) * VEC, v[u]);
    }
  }
  for (; i < nvec; i += stride) {
    float v[VEC];
    load_act<T, VEC>(x + i * VEC, v);
#pragma unroll
    for (int e = 0; e < VEC; ++e) v[e] = act_t<A, (sizeof(T) == 2)>(v[e]);
    store_act<T, VEC>(y + i * VEC, v);
  }
  // Scalar tail (n not a multiple of VEC).
  if (VEC > 1 && blockIdx.x == 0) {
    for (int64_t j = nvec * VEC + threadIdx.x; j < n; j += blockDim.x)
      y[j] = from_f<T>(act_t<A, (sizeof(T) == 2)>(to_f(x[j])));
  }
}

// Row kernel over strided views; GATED = GeGLU (y = a * gelu_erf(b) with a, b
// the two halves of each input row).
template <typename T, int VEC, int A, bool GATED>
__global__ void __launch_bounds__(256) act_rows_kernel(const T* __restrict__ x, RowMap xm,
                                                       T* __restrict__ y, RowMap ym, int64_t rows,
                                                       int64_t F) {
  const int64_t nv = F / VEC;
  const int64_t total = rows * nv;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv;
    const int64_t c = (i - r * nv) * VEC;
    const T* xr = x + row_offset(xm, r);
    float a[VEC];
    load_act<T, VEC>(xr + c, a);
    if constexpr (GATED) {
      float g[VEC];
      load_act<T, VEC>(xr + F + c, g);
#pragma unroll
      for (int e = 0; e < VEC; ++e) a[e] = a[e] * act_t<ACT_GELU_ERF, (sizeof(T) == 2)>(g[e]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) a[e] = act_t<A, (sizeof(T) == 2)>(a[e]);
    }
    store_act<T, VEC>(y + row_offset(ym, r) + c, a);
  }
}

// Activation whose result goes to several outputs: the local one and the
// gather buffers of other GPUs mapped into this process (peer memory), so
// the last op of the chain and the final all-gather are one pass.  Each
// thread keeps kUnroll vectors in flight; the stores of a vector go to the
// outputs in an order rotated by the block index, so concurrent blocks
// write to different peers.
constexpr int kMaxScatter = 8;
struct ScatterOut {
  void* p[kMaxScatter];
  int n;
};

template <typename T, int A>
__global__ void __launch_bounds__(256) act_scatter_kernel(const T* __restrict__ x, ScatterOut out,
                                                          int64_t nvec) {
  constexpr int VEC = Vec16<T>::N;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int rot = int(blockIdx.x % unsigned(out.n));
  for (; i < nvec; i += kUnroll * stride) {
    uint4 w[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = i + u * stride;
      float f[VEC];
      if (v < nvec) {
        load_act<T, VEC>(x + v * VEC, f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) f[e] = act_t<A, (sizeof(T) == 2)>(f[e]);
        w[u] = pack(f, T());
      }
    }
    for (int k = 0; k < out.n; ++k) {
      int o = k + rot;
      if (o >= out.n) o -= out.n;
      uint4* dst = static_cast<uint4*>(out.p[o]);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = i + u * stride;
        if (v < nvec) st_act_raw(dst + v, w[u]);
      }
    }
  }
}

static bool is_contiguous(const l3d_tensor* t) {
  int64_t st = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    if (t->dims[i] > 1 && t->strides[i] != st) return false;
    st *= t->dims[i];
  }
  return true;
}

static int grid_for(int64_t work) {
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  return int(blocks < 1 ? 1 : blocks);
}

template <int A, bool GATED>
static int run_act(const l3d_tensor* x, const l3d_tensor* y, const char* op,
                   cudaStream_t stream) {
  if (!x || !y || no_data(x) || no_data(y)) return fail(L3D_E_NULL, "%s: x and y are required", op);
  if (!is_float_dtype(x->dtype) || x->dtype != y->dtype)
    return fail(L3D_E_DTYPE, "%s: x/y must share a float dtype", op);
  if (x->ndim < 1 || x->ndim != y->ndim) return fail(L3D_E_SHAPE, "%s: rank mismatch", op);
  const int last = x->ndim - 1;
  for (int i = 0; i < last; ++i)
    if (x->dims[i] != y->dims[i]) return fail(L3D_E_SHAPE, "%s: x/y shapes differ", op);
  const int64_t F = y->dims[last];
  if (x->dims[last] != (GATED ? 2 * F : F))
    return fail(L3D_E_SHAPE, "%s: last dim mismatch (GeGLU input must be 2F)", op);
  if ((x->dims[last] > 1 && x->strides[last] != 1) || (F > 1 && y->strides[last] != 1))
    return fail(L3D_E_ALIGN, "%s: last dim must be contiguous", op);
  const int64_t n = numel(y);
  if (n == 0) return L3D_OK;
  const int es = dtype_size(x->dtype);
  const int vec = 16 / es;
  if (!GATED && is_contiguous(x) && is_contiguous(y)) {
    const char* xp = elem_ptr(x);
    char* yp = const_cast<char*>(elem_ptr(y));
    const bool v = (reinterpret_cast<uintptr_t>(xp) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(yp) % 16 == 0);
    L3D_DISPATCH_FLOAT(x->dtype, T, {
      if (v) {
        constexpr int V = Vec16<T>::N;
        const int g = grid_for(n / V / kUnroll);
        act_flat_kernel<T, V, A><<<g, 256, 0, stream>>>(reinterpret_cast<const T*>(xp),
                                                        reinterpret_cast<T*>(yp), n);
      } else {
        act_flat_kernel<T, 1, A><<<grid_for(n / kUnroll), 256, 0, stream>>>(
            reinterpret_cast<const T*>(xp), reinterpret_cast<T*>(yp), n);
      }
    });
    return check_launch(op);
  }
  RowMap xm, ym;
  if (!make_rowmap(x, last, &xm) || !make_rowmap(y, last, &ym))
    return fail(L3D_E_UNSUPPORTED, "%s: too many non-collapsible dims", op);
  const int64_t rows = n / F;
  const bool v = (F % vec == 0) && (reinterpret_cast<uintptr_t>(x->data) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(y->data) % 16 == 0) && rowmap_aligned(xm, vec) &&
                 rowmap_aligned(ym, vec);
  L3D_DISPATCH_FLOAT(x->dtype, T, {
    const T* xp = static_cast<const T*>(x->data);
    T* yp = static_cast<T*>(y->data);
    if (v) {
      constexpr int V = Vec16<T>::N;
      act_rows_kernel<T, V, A, GATED><<<grid_for(rows * F / V), 256, 0, stream>>>(xp, xm, yp, ym,
                                                                                  rows, F);
    } else {
      act_rows_kernel<T, 1, A, GATED><<<grid_for(rows * F), 256, 0, stream>>>(xp, xm, yp, ym,
                                                                              rows, F);
    }
  });
  return check_launch(op);
}

}  // namespace l3d

using namespace l3d;

extern "C" int l3d_gelu_tanh(const l3d_tensor* x, const l3d_tensor* y, l3d_stream s) {
  return run_act<ACT_GELU_TANH, false>(x, y, "l3d_gelu_tanh", reinterpret_cast<cudaStream_t>(s));
}
extern "C" int l3d_gelu_erf(const l3d_tensor* x, const l3d_tensor* y, l3d_stream s) {
  return run_act<ACT_GELU_ERF, false>(x, y, "l3d_gelu_erf", reinterpret_cast<cudaStream_t>(s));
}
extern "C" int l3d_silu(const l3d_tensor* x, const l3d_tensor* y, l3d_stream s) {
  return run_act<ACT_SILU, false>(x, y, "l3d_silu", reinterpret_cast<cudaStream_t>(s));
}
extern "C" int l3d_geglu(const l3d_tensor* x, const l3d_tensor* y, l3d_stream s) {
  return run_act<ACT_GELU_ERF, true>(x, y, "l3d_geglu", reinterpret_cast<cudaStream_t>(s));
}

extern "C" int l3d_activation_scatter(int act, const l3d_tensor* x, const l3d_tensor* outs,
                                      int n_out, l3d_stream stream) {
  const char* op = "l3d_activation_scatter";
  if (!x || no_data(x) || !outs) return fail(L3D_E_NULL, "%s: x and outs are required", op);
  if (n_out < 1 || n_out > kMaxScatter)
    return fail(L3D_E_UNSUPPORTED, "%s: 1 to %d outputs", op, kMaxScatter);
  if (act != ACT_SILU && act != ACT_GELU_ERF && act != ACT_GELU_TANH)
    return fail(L3D_E_UNSUPPORTED, "%s: act must be 1 (SiLU), 2 (GELU-erf) or 3 (GELU-tanh)", op);
  if (!is_float_dtype(x->dtype)) return fail(L3D_E_DTYPE, "%s: x must be F32/F16/BF16", op);
  if (!is_contiguous(x)) return fail(L3D_E_ALIGN, "%s: x must be contiguous", op);
  const int64_t n = numel(x);
  const int vec = 16 / dtype_size(x->dtype);
  if (n % vec || reinterpret_cast<uintptr_t>(elem_ptr(x)) % 16)
    return fail(L3D_E_ALIGN, "%s: x must be 16-byte aligned with a multiple of 16 bytes", op);
  ScatterOut so{};
  so.n = n_out;
  for (int k = 0; k < n_out; ++k) {
    const l3d_tensor* o = &outs[k];
    if (no_data(o)) return fail(L3D_E_NULL, "%s: output %d has no data", op, k);
    if (o->dtype != x->dtype) return fail(L3D_E_DTYPE, "%s: output %d dtype differs", op, k);
    if (numel(o) != n || !is_contiguous(o))
      return fail(L3D_E_SHAPE, "%s: output %d must be contiguous with x's element count", op, k);
    if (reinterpret_cast<uintptr_t>(elem_ptr(o)) % 16)
      return fail(L3D_E_ALIGN, "%s: output %d must be 16-byte aligned", op, k);
    so.p[k] = const_cast<char*>(elem_ptr(o));
  }
  if (n == 0) return L3D_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t nvec = n / vec;
  L3D_DISPATCH_FLOAT(x->dtype, T, {
    const T* xp = reinterpret_cast<const T*>(elem_ptr(x));
    const int g = grid_for(nvec / kUnroll);
    if (act == ACT_SILU) act_scatter_kernel<T, ACT_SILU><<<g, 256, 0, s>>>(xp, so, nvec);
    else if (act == ACT_GELU_ERF) act_scatter_kernel<T, ACT_GELU_ERF><<<g, 256, 0, s>>>(xp, so, nvec);
    else act_scatter_kernel<T, ACT_GELU_TANH><<<g, 256, 0, s>>>(xp, so, nvec);
  });
  return check_launch(op);
}
