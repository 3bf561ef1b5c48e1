// Host-side helpers of libl3dops: thread-local status, layout collapsing,
// device properties.
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace l3d {

static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(L3D_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return L3D_OK;
}

const char* dtype_name(int dt) {
  switch (dt) {
    case L3D_F32: return "F32";
    case L3D_F16: return "F16";
    case L3D_BF16: return "BF16";
    case L3D_I32: return "I32";
    case L3D_I64: return "I64";
    case L3D_U32: return "U32";
    case L3D_U8: return "U8";
    default: return "?";
  }
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> g(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

cudaError_t set_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, cudaError_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_pair(dev, kernel);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  done[key] = e;
  return e;
}

bool make_rowmap(const l3d_tensor* t, int lead, RowMap* m) {
  // Collect non-unit leading dims, outermost first.
  int64_t d[L3D_MAX_DIMS], s[L3D_MAX_DIMS];
  int n = 0;
  for (int i = 0; i < lead; ++i) {
    if (t->dims[i] == 1) continue;
    d[n] = t->dims[i];
    s[n] = t->strides[i];
    ++n;
  }
  // Merge adjacent dims whose strides nest (outer == inner * inner_dim).
  int64_t cd[L3D_MAX_DIMS], cs[L3D_MAX_DIMS];
  int c = 0;
  for (int i = 0; i < n; ++i) {
    if (c > 0 && cs[c - 1] == s[i] * d[i]) {
      cd[c - 1] *= d[i];
      cs[c - 1] = s[i];
    } else {
      cd[c] = d[i];
      cs[c] = s[i];
      ++c;
    }
  }
  if (c == 0) {
    cd[0] = 1;
    cs[0] = 0;
    c = 1;
  }
  if (c > 5) return false;
  m->nd = c;
  for (int i = 0; i < 5; ++i) {
    m->dims[i] = i < c ? cd[i] : 1;
    m->strides[i] = i < c ? cs[i] : 0;
  }
  m->base = t->offset;
  return true;
}

bool rowmap_aligned(const RowMap& m, int64_t elems) {
  if (m.base % elems) return false;
  for (int i = 0; i < m.nd; ++i)
    if (m.dims[i] > 1 && (m.strides[i] % elems)) return false;
  return true;
}

int make_chanvec(const l3d_tensor* t, const char* name, int64_t C, int64_t B, ChanVec* out,
                 bool* aligned16) {
  out->ptr = nullptr;
  out->bstride = 0;
  out->dtype = L3D_F32;
  if (!t) return L3D_OK;
  if (no_data(t)) return fail(L3D_E_NULL, "%s: null data pointer", name);
  if (!is_float_dtype(t->dtype)) return fail(L3D_E_DTYPE, "%s: float dtype required", name);
  if (t->ndim < 1 || t->dims[t->ndim - 1] != C)
    return fail(L3D_E_SHAPE, "%s: last dim must be %lld", name, (long long)C);
  if (C > 1 && t->strides[t->ndim - 1] != 1)
    return fail(L3D_E_ALIGN, "%s: last dim must be contiguous", name);
  int64_t tb = 1, bs = 0;
  if (t->ndim == 2) {
    tb = t->dims[0];
    bs = t->strides[0];
  } else if (t->ndim == 3) {
    if (t->dims[1] != 1) return fail(L3D_E_SHAPE, "%s: expected [B, 1, C]", name);
    tb = t->dims[0];
    bs = t->strides[0];
  } else if (t->ndim != 1) {
    return fail(L3D_E_SHAPE, "%s: expected [C], [B, C] or [B, 1, C]", name);
  }
  if (tb != 1 && tb != B)
    return fail(L3D_E_SHAPE, "%s: batch %lld does not match %lld", name, (long long)tb,
                (long long)B);
  if (tb == 1) bs = 0;
  out->ptr = elem_ptr(t);
  out->bstride = bs;
  out->dtype = t->dtype;
  const int es = dtype_size(t->dtype);
  const uintptr_t a = reinterpret_cast<uintptr_t>(out->ptr);
  if ((a % 16) != 0 || ((bs * es) % 16) != 0) *aligned16 = false;
  return L3D_OK;
}

}  // namespace l3d

extern "C" int l3d_abi_version(void) { return L3D_ABI_VERSION; }
extern "C" const char* l3d_last_error(void) { return l3d::g_last_error.c_str(); }

extern "C" int l3d_kernel_status(int* status, int reset) {
  using namespace l3d;
  if (!status) return fail(L3D_E_NULL, "l3d_kernel_status: status is required");
  if (norm_status_read(status, reset) != cudaSuccess)
    return fail(L3D_E_CUDA, "l3d_kernel_status: cannot read the status word");
  return L3D_OK;
}
