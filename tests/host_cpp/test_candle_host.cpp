// CPU checks of the C++ host layer (candle-3d_b200/host/candle_l3d.hpp): the
// Layout algebra of the strided head views, the C ABI descriptors, the host
// checks that throw before any allocation, and the C ABI's own status codes
// surfacing as l3d::candle::Error.  Runs without a GPU; the parts that pass
// made-up device pointers to the library run only where no CUDA device is
// visible, so nothing is ever dereferenced.
#include <cstdio>
#include <cstring>
#include <string>

#include "candle_l3d.hpp"

using namespace l3d::candle;

static int failures = 0;
#define EXPECT(c)                                                          \
  do {                                                                     \
    if (!(c)) {                                                            \
      std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #c);             \
      ++failures;                                                          \
    }                                                                      \
  } while (0)

template <class F>
static void expect_error(F&& f, int code, const char* needle, int line) {
  try {
    f();
    std::printf("FAIL line %d: no error thrown\n", line);
    ++failures;
  } catch (const Error& e) {
    if (e.code() != code || (needle && !std::strstr(e.what(), needle))) {
      std::printf("FAIL line %d: code %d (want %d), message '%s' (want '%s')\n", line, e.code(),
                  code, e.what(), needle ? needle : "");
      ++failures;
    }
  }
}
#define EXPECT_ERROR(expr, code, needle) expect_error([&] { (void)(expr); }, code, needle, __LINE__)

static void* const kFake = reinterpret_cast<void*>(uintptr_t(1) << 40);  // never dereferenced

static Tensor fake(const std::vector<int64_t>& dims, DType t, const Device& d = Device{}) {
  return Tensor::from_device_ptr(kFake, Layout::contiguous(dims), t, d);
}

static void layout_algebra() {
  Layout c = Layout::contiguous({2, 3, 4});
  EXPECT((c.stride == std::vector<int64_t>{12, 4, 1}) && c.is_contiguous() && c.elem_count() == 24);
  // qkv [B, N, 3 H D] -> reshape (B, N, 3, H, D) -> permute(2, 0, 3, 1, 4) -> [i]:
  // the q / k / v head views of crate/runtime/attention_math.rs:127-150.
  const int64_t B = 2, N = 5, H = 4, D = 8;
  Tensor qkv = fake({B, N, 3 * H * D}, DType::BF16);
  Tensor heads = qkv.reshape({B, N, 3, H, D}).permute({2, 0, 3, 1, 4});
  Tensor q = heads.get(0), k = heads.get(1);
  EXPECT((q.dims() == std::vector<int64_t>{B, H, N, D}));
  EXPECT((q.layout().stride == std::vector<int64_t>{N * 3 * H * D, D, 3 * H * D, 1}));
  EXPECT(q.layout().start_offset == 0 && k.layout().start_offset == H * D);
  EXPECT(!q.is_contiguous());
  // chunk of a [B, 6C] adaLN vector into six [B, C] views (chunk_modulation).
  Tensor mod = fake({B, 6 * 16}, DType::F32);
  auto parts = mod.chunk(6, 1);
  EXPECT(parts.size() == 6 && (parts[2].dims() == std::vector<int64_t>{B, 16}));
  EXPECT(parts[2].layout().start_offset == 32 && parts[2].layout().stride[0] == 96);
  // descriptor of a strided, offset view
  const l3d_tensor d = k.desc();
  EXPECT(d.data == kFake && d.dtype == L3D_BF16 && d.ndim == 4 && d.offset == H * D);
  EXPECT(d.dims[2] == N && d.strides[2] == 3 * H * D && d.strides[3] == 1);
  // transpose / narrow
  Layout t = c.transpose(0, 2);
  EXPECT((t.dims == std::vector<int64_t>{4, 3, 2}) && (t.stride == std::vector<int64_t>{1, 4, 12}));
  Layout n = c.narrow(-1, 1, 2);
  EXPECT(n.start_offset == 1 && n.dims[2] == 2 && !n.is_contiguous());
  EXPECT_ERROR(c.narrow(1, 2, 2), L3D_E_SHAPE, "narrow");
  EXPECT_ERROR(c.permute({0, 0, 1}), L3D_E_SHAPE, "repeated");
  EXPECT_ERROR(q.reshape({B * H * N * D}), L3D_E_UNSUPPORTED, "not contiguous");
  EXPECT_ERROR(qkv.reshape({7}), L3D_E_SHAPE, "element count");
  EXPECT_ERROR(mod.chunk(5, 1), L3D_E_SHAPE, "chunk");
}

// Host checks that throw before any allocation or device call.
static void host_checks() {
  Tensor x = fake({2, 7, 64}, DType::BF16);
  EXPECT_ERROR(nn::ops::layer_norm(x, fake({63}, DType::BF16), fake({64}, DType::BF16), 1e-5f),
               L3D_E_SHAPE, "alpha");
  EXPECT_ERROR(fake({4, 8}, DType::I32).gelu(), L3D_E_DTYPE, "gelu");
  Tensor q32 = fake({1, 4, 9, 32}, DType::BF16);
  Tensor tab = fake({1, 1, 9, 32}, DType::F32);
  EXPECT_ERROR(nn::ops::rope_fused(q32, tab, tab), L3D_E_SHAPE, "head dim 32");
  Tensor q = fake({1, 4, 9, 64}, DType::BF16);
  EXPECT_ERROR(nn::ops::layernorm_rope_fused(q, fake({64}, DType::BF16), fake({64}, DType::BF16),
                                             1e-5f, fake({1, 1, 9, 64}, DType::BF16),
                                             fake({1, 1, 9, 64}, DType::BF16)),
               L3D_E_DTYPE, "f32");
  Tensor xt = fake({1, 11, 12, 128}, DType::BF16);
  EXPECT_ERROR(runtime::qk_rms_norm_rope3d(xt, fake({12, 64}, DType::F32), std::nullopt),
               L3D_E_SHAPE, "gamma");
  EXPECT_ERROR(runtime::qk_rms_norm_rope3d(xt, fake({12, 128}, DType::F32),
                                           fake({11, 3}, DType::F32)),
               L3D_E_DTYPE, "coords");
  EXPECT_ERROR(runtime::rms_norm_heads(x, fake({32}, DType::BF16), 1e-6f), L3D_E_SHAPE, "w");
  EXPECT_ERROR(runtime::timestep_embedding(fake({2}, DType::BF16), 256,
                                           runtime::TimestepOrder::CosFirst, DType::BF16),
               L3D_E_DTYPE, "t is f32");
  using quantized::GgmlDType;
  using quantized::QMatMul;
  EXPECT_ERROR(QMatMul(kFake, GgmlDType::Q8_0, 64, 48), L3D_E_SHAPE, "whole blocks");
  EXPECT_ERROR(QMatMul(nullptr, GgmlDType::Q8_0, 64, 64), L3D_E_NULL, "null");
  QMatMul qm(kFake, GgmlDType::Q8_0, 64, 128);
  EXPECT(qm.weight_bytes() == 64 * 4 * 34);
  EXPECT_ERROR(qm.forward(fake({3, 96}, DType::BF16)), L3D_E_SHAPE, "last dim must be 128");
  EXPECT(QMatMul(kFake, GgmlDType::Q4K, 8, 256).weight_bytes() == 8 * 144);
  EXPECT_ERROR(qm.forward_ex(fake({3, 128}, DType::BF16), nn::Act::GeluTanh, std::nullopt,
                             fake({64}, DType::F32)),
               L3D_E_SHAPE, "gate needs a residual");
  EXPECT_ERROR(fake({2, 7}, DType::BF16).geglu(), L3D_E_SHAPE, "not even");
  Tensor qa = fake({1, 4, 16, 64}, DType::BF16), ka = fake({1, 4, 32, 64}, DType::BF16);
  EXPECT_ERROR(nn::ops::sdpa(fake({1, 4, 16, 64}, DType::F32), ka, ka, 0.125f), L3D_E_DTYPE, "bf16");
  EXPECT_ERROR(nn::ops::sdpa(qa, fake({1, 2, 32, 64}, DType::BF16), fake({1, 2, 32, 64}, DType::BF16),
                             0.125f),
               L3D_E_SHAPE, "differ");
  EXPECT_ERROR(nn::ops::sdpa(qa, ka, ka, 0.f), L3D_E_SHAPE, "positive");
  EXPECT_ERROR((nn::Linear{fake({32, 64}, DType::F32), std::nullopt}.forward(fake({4, 64}, DType::BF16))),
               L3D_E_DTYPE, "weight is bf16");
  EXPECT_ERROR((nn::Linear{fake({32, 64}, DType::BF16), std::nullopt}.forward(fake({4, 48}, DType::BF16))),
               L3D_E_SHAPE, "against weight");
  EXPECT_ERROR(runtime::linear_small(fake({2, 64}, DType::BF16), fake({96, 32}, DType::BF16),
                                     std::nullopt, std::nullopt, nn::Act::Silu, nn::Act::None),
               L3D_E_SHAPE, "against w");
  EXPECT_ERROR(runtime::patch_embed(fake({2, 3, 30, 28}, DType::BF16), fake({16, 3, 14, 14}, DType::BF16),
                                    fake({16}, DType::BF16), fake({5, 16}, DType::BF16),
                                    fake({16}, DType::BF16), std::nullopt, 14),
               L3D_E_SHAPE, "whole patches");
  EXPECT_ERROR(runtime::neighbor_pairs(fake({10, 3}, DType::I64)), L3D_E_SHAPE, "i32");
}

// Without a device: allocation fails with a CUDA error; and with a host
// allocator that hands out made-up pointers, the C ABI's own checks reject
// requests on the host and their status surfaces as an Error.
static void without_device() {
  Device plain;
  EXPECT_ERROR(Tensor::empty({4, 4}, DType::F32, plain), L3D_E_CUDA, "alloc");
  Device d;
  d.allocator = [](size_t bytes) {
    auto st = std::make_shared<Storage>();
    st->ptr = kFake;
    st->bytes = bytes;
    return st;
  };
  Tensor x = Tensor::from_device_ptr(kFake, Layout::contiguous({4, 64}), DType::BF16, d);
  Tensor xs = x.transpose(0, 1);  // last dim strided
  EXPECT_ERROR(nn::ops::layer_norm(xs, fake({4}, DType::BF16), fake({4}, DType::BF16), 1e-5f),
               L3D_E_ALIGN, "l3d_layer_norm: ");
  EXPECT_ERROR(runtime::layer_norm_modulate(x, fake({72}, DType::BF16), fake({72}, DType::BF16),
                                            1e-6f),
               L3D_E_SHAPE, "l3d_layer_norm_modulate: ");
  EXPECT_ERROR(runtime::gated_residual(x, x, fake({3, 64}, DType::BF16)), L3D_E_SHAPE,
               "l3d_gated_residual: ");
  // the attention's own envelope (head dim 64 or 128) and the seam's gate batch
  Tensor q96 = Tensor::from_device_ptr(kFake, Layout::contiguous({1, 2, 16, 96}), DType::BF16, d);
  EXPECT_ERROR(nn::ops::sdpa(q96, q96, q96, 0.1f), L3D_E_UNSUPPORTED, "head dim must be 64 or 128");
  EXPECT_ERROR(runtime::residual_layer_norm_modulate(x, x, fake({5, 64}, DType::BF16), std::nullopt,
                                                     std::nullopt, std::nullopt, std::nullopt, 1e-5f),
               L3D_E_SHAPE, "l3d_residual_layer_norm_modulate: ");
}

int main() {
  layout_algebra();
  host_checks();
  int n = 0;
  const bool no_device = cudaGetDeviceCount(&n) != cudaSuccess || n == 0;
  cudaGetLastError();
  if (no_device) without_device();
  if (failures) {
    std::printf("%d FAILED\n", failures);
    return 1;
  }
  std::printf("ALL OK%s\n", no_device ? "" : " (device present: no-device checks skipped)");
  return 0;
}
