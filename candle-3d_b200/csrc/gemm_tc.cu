// Dequant-linear on the tensor cores (in progress).
#include "common.cuh"
#include "qlinear.cuh"

using namespace l3d;

extern "C" size_t l3d_dequant_linear_workspace_size(int fmt, int64_t m, int64_t n, int64_t k) {
  (void)fmt; (void)m;
  return size_t(n) * size_t(k) * 2 + 256;
}

extern "C" int l3d_dequant_linear(const l3d_tensor* x, const void* wq, int fmt, int64_t n,
                                  int64_t k, const l3d_tensor* bias, const l3d_tensor* y,
                                  void* workspace, size_t workspace_bytes, l3d_stream stream) {
  (void)x; (void)wq; (void)fmt; (void)n; (void)k; (void)bias; (void)y; (void)workspace;
  (void)workspace_bytes; (void)stream;
  return fail(L3D_E_UNSUPPORTED, "l3d_dequant_linear: not built yet");
}
