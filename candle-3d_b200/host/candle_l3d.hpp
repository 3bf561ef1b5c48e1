// C++ host layer over libl3dops: the Candle-shaped tensor and op interface of
// the per-token layer-op path, for a compiled host (the reference is Rust on
// Candle; a C++ caller gets the same op names, argument meaning and error
// behaviour through this header).
//
//   * Tensor = shared storage + Layout (dims, element strides, start offset)
//     + DType + Device, as candle_core::Tensor; narrow / transpose / permute /
//     chunk / reshape produce views without copies, so the strided head views
//     the models build (`qkv.reshape(B,N,3,H,D).permute(2,0,3,1,4)` and its
//     chunks, crate/runtime/attention_math.rs:127-150) go to the kernels as
//     they are.
//   * Errors are thrown as l3d::candle::Error (Candle's Result<_, Error> with
//     `?`): shape and dtype checks run on the host before any allocation, and
//     a non-zero status of the C ABI carries its code and l3d_last_error().
//   * Each op allocates its contiguous output on the input's device and
//     stream, as a Candle CustomOp's cuda_fwd does, and never synchronises.
//
// Header-only; link libl3dops.so and libcudart.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <optional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "l3d_ops.h"

namespace l3d {
namespace candle {

// ----------------------------------------------------------------- errors
class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }  // an l3d_status value

 private:
  int code_;
};

inline std::string dims_str(const std::vector<int64_t>& d) {
  std::ostringstream s;
  s << "[";
  for (size_t i = 0; i < d.size(); ++i) s << (i ? ", " : "") << d[i];
  s << "]";
  return s.str();
}

// Throws the C ABI's status as an Error (candle_core::Error::Msg in the
// reference's shim).
inline void check(int rc, const char* op) {
  if (rc != L3D_OK) throw Error(rc, std::string(op) + ": " + l3d_last_error());
}

// ------------------------------------------------------------------ dtypes
enum class DType { F32, F16, BF16, I32, I64, U32, U8 };

inline int to_abi(DType t) {
  switch (t) {
    case DType::F32: return L3D_F32;
    case DType::F16: return L3D_F16;
    case DType::BF16: return L3D_BF16;
    case DType::I32: return L3D_I32;
    case DType::I64: return L3D_I64;
    case DType::U32: return L3D_U32;
    default: return L3D_U8;
  }
}

inline size_t size_in_bytes(DType t) {
  switch (t) {
    case DType::F32: case DType::I32: case DType::U32: return 4;
    case DType::F16: case DType::BF16: return 2;
    case DType::I64: return 8;
    default: return 1;
  }
}

inline bool is_float(DType t) { return t == DType::F32 || t == DType::F16 || t == DType::BF16; }

inline const char* as_str(DType t) {
  switch (t) {
    case DType::F32: return "f32";
    case DType::F16: return "f16";
    case DType::BF16: return "bf16";
    case DType::I32: return "i32";
    case DType::I64: return "i64";
    case DType::U32: return "u32";
    default: return "u8";
  }
}

// ------------------------------------------------------------------ layout
// candle_core::Layout: shape, element strides and the start offset into the
// storage.
struct Layout {
  std::vector<int64_t> dims, stride;
  int64_t start_offset = 0;

  static Layout contiguous(const std::vector<int64_t>& dims, int64_t offset = 0) {
    Layout l;
    l.dims = dims;
    l.stride.assign(dims.size(), 1);
    for (int i = int(dims.size()) - 2; i >= 0; --i) l.stride[i] = l.stride[i + 1] * dims[i + 1];
    l.start_offset = offset;
    return l;
  }
  size_t rank() const { return dims.size(); }
  int64_t elem_count() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
  bool is_contiguous() const {
    int64_t s = 1;
    for (int i = int(dims.size()) - 1; i >= 0; --i) {
      if (dims[i] > 1 && stride[i] != s) return false;
      s *= dims[i];
    }
    return true;
  }
  size_t dim_index(int64_t d, const char* op) const {
    const int64_t r = int64_t(rank());
    if (d < -r || d >= r)
      throw Error(L3D_E_SHAPE, std::string(op) + ": dim " + std::to_string(d) +
                                   " out of range for rank " + std::to_string(r));
    return size_t(d < 0 ? d + r : d);
  }
  Layout narrow(int64_t dim, int64_t start, int64_t len) const {
    const size_t d = dim_index(dim, "narrow");
    if (start < 0 || len < 0 || start + len > dims[d])
      throw Error(L3D_E_SHAPE, "narrow: [" + std::to_string(start) + ", " +
                                   std::to_string(start + len) + ") outside dim of size " +
                                   std::to_string(dims[d]));
    Layout l = *this;
    l.dims[d] = len;
    l.start_offset += start * stride[d];
    return l;
  }
  Layout transpose(int64_t d0, int64_t d1) const {
    Layout l = *this;
    const size_t a = dim_index(d0, "transpose"), b = dim_index(d1, "transpose");
    std::swap(l.dims[a], l.dims[b]);
    std::swap(l.stride[a], l.stride[b]);
    return l;
  }
  Layout permute(const std::vector<int64_t>& order) const {
    if (order.size() != rank()) throw Error(L3D_E_SHAPE, "permute: order has the wrong rank");
    std::vector<bool> seen(rank(), false);
    Layout l;
    l.start_offset = start_offset;
    for (int64_t o : order) {
      const size_t i = dim_index(o, "permute");
      if (seen[i]) throw Error(L3D_E_SHAPE, "permute: repeated dim");
      seen[i] = true;
      l.dims.push_back(dims[i]);
      l.stride.push_back(stride[i]);
    }
    return l;
  }
  // Index `i` of dim 0 (Tensor::i / get): drops that dim.
  Layout get(int64_t i) const {
    if (rank() == 0 || i < 0 || i >= dims[0]) throw Error(L3D_E_SHAPE, "get: index out of range");
    Layout l;
    l.dims.assign(dims.begin() + 1, dims.end());
    l.stride.assign(stride.begin() + 1, stride.end());
    l.start_offset = start_offset + i * stride[0];
    return l;
  }
};

// ----------------------------------------------------------------- device
// One stream per device, as candle_core::CudaDevice.  Storage comes from the
// allocator (stream-ordered cudaMallocAsync by default); a host that owns a
// pool passes its own.  As with Candle's CudaDevice, the device must be the
// calling thread's current one (cudaSetDevice) while its ops are issued: the
// kernels go to `stream`, which belongs to it.
struct Storage {
  void* ptr = nullptr;
  size_t bytes = 0;
  std::function<void(void*)> release;
  ~Storage() {
    if (release && ptr) release(ptr);
  }
};

struct Device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  std::function<std::shared_ptr<Storage>(size_t)> allocator;

  std::shared_ptr<Storage> alloc(size_t bytes) const {
    if (allocator) return allocator(bytes);
    auto st = std::make_shared<Storage>();
    st->bytes = bytes;
    if (bytes == 0) return st;
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess && cur != ordinal)
      throw Error(L3D_E_CUDA, "alloc on cuda:" + std::to_string(ordinal) + ": the thread's current "
                              "device is cuda:" + std::to_string(cur) + " (cudaSetDevice first)");
    if (e == cudaSuccess) e = cudaMallocAsync(&st->ptr, bytes, stream);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Error(L3D_E_CUDA, std::string("alloc of ") + std::to_string(bytes) +
                                  " bytes on cuda:" + std::to_string(ordinal) + ": " +
                                  cudaGetErrorString(e));
    }
    const cudaStream_t s = stream;
    st->release = [s](void* p) { cudaFreeAsync(p, s); };
    return st;
  }
};

// ----------------------------------------------------------------- tensor
class Tensor {
 public:
  Tensor() = default;
  Tensor(std::shared_ptr<Storage> st, Layout l, DType t, Device d)
      : st_(std::move(st)), layout_(std::move(l)), dtype_(t), dev_(std::move(d)) {}

  // Contiguous, uninitialised.
  static Tensor empty(const std::vector<int64_t>& dims, DType t, const Device& d) {
    Layout l = Layout::contiguous(dims);
    for (int64_t x : dims)
      if (x < 0) throw Error(L3D_E_SHAPE, "empty: negative dim in " + dims_str(dims));
    return Tensor(d.alloc(size_t(l.elem_count()) * size_in_bytes(t)), l, t, d);
  }
  // A view of memory the caller owns (CudaStorage handed in by the host).
  static Tensor from_device_ptr(void* ptr, const Layout& l, DType t, const Device& d) {
    auto st = std::make_shared<Storage>();
    st->ptr = ptr;
    return Tensor(st, l, t, d);
  }

  const Layout& layout() const { return layout_; }
  const std::vector<int64_t>& dims() const { return layout_.dims; }
  int64_t dim(int64_t d) const { return layout_.dims[layout_.dim_index(d, "dim")]; }
  size_t rank() const { return layout_.rank(); }
  int64_t elem_count() const { return layout_.elem_count(); }
  DType dtype() const { return dtype_; }
  const Device& device() const { return dev_; }
  bool is_contiguous() const { return layout_.is_contiguous(); }
  void* storage_ptr() const { return st_ ? st_->ptr : nullptr; }

  Tensor narrow(int64_t d, int64_t start, int64_t len) const { return view(layout_.narrow(d, start, len)); }
  Tensor transpose(int64_t a, int64_t b) const { return view(layout_.transpose(a, b)); }
  Tensor permute(const std::vector<int64_t>& o) const { return view(layout_.permute(o)); }
  Tensor get(int64_t i) const { return view(layout_.get(i)); }
  // Tensor::chunk: n equal pieces of dim d (the size must divide).
  std::vector<Tensor> chunk(int64_t n, int64_t d) const {
    const size_t i = layout_.dim_index(d, "chunk");
    if (n <= 0 || layout_.dims[i] % n)
      throw Error(L3D_E_SHAPE, "chunk: " + std::to_string(n) + " pieces of a dim of size " +
                                   std::to_string(layout_.dims[i]));
    std::vector<Tensor> out;
    const int64_t len = layout_.dims[i] / n;
    for (int64_t k = 0; k < n; ++k) out.push_back(narrow(int64_t(i), k * len, len));
    return out;
  }
  // Tensor::reshape of a contiguous tensor (a view; Candle copies otherwise).
  Tensor reshape(const std::vector<int64_t>& dims) const {
    Layout l = Layout::contiguous(dims, layout_.start_offset);
    if (l.elem_count() != elem_count())
      throw Error(L3D_E_SHAPE, "reshape: " + dims_str(layout_.dims) + " -> " + dims_str(dims) +
                                   " changes the element count");
    if (!is_contiguous())
      throw Error(L3D_E_UNSUPPORTED, "reshape: the view is not contiguous (copy it first)");
    return view(l);
  }

  // The C ABI descriptor of this view.
  l3d_tensor desc() const {
    if (rank() > L3D_MAX_DIMS)
      throw Error(L3D_E_SHAPE, "rank " + std::to_string(rank()) + " above " +
                                   std::to_string(L3D_MAX_DIMS));
    l3d_tensor t{};
    t.data = storage_ptr();
    t.dtype = to_abi(dtype_);
    t.ndim = int32_t(rank());
    for (size_t i = 0; i < rank(); ++i) {
      t.dims[i] = layout_.dims[i];
      t.strides[i] = layout_.stride[i];
    }
    t.offset = layout_.start_offset;
    return t;
  }

  // A new contiguous tensor of this one's dims and dtype (or `t`) on its device.
  Tensor empty_like(std::optional<DType> t = std::nullopt) const {
    return empty(layout_.dims, t ? *t : dtype_, dev_);
  }

  // Tensor::gelu / gelu_erf / silu (crate/runtime/trellis2_blocks.rs:558-561,
  // crate/runtime/nn_blocks.rs:233, crate/runtime/trellis2_blocks.rs:236).
  Tensor gelu() const { return unary(l3d_gelu_tanh, "gelu"); }
  Tensor gelu_erf() const { return unary(l3d_gelu_erf, "gelu_erf"); }
  Tensor silu() const { return unary(l3d_silu, "silu"); }
  // GeGlu::forward (crate/runtime/nn_blocks.rs:250-253): x [.., 2F] ->
  // x[.., :F] * gelu_erf(x[.., F:]).
  Tensor geglu() const {
    if (!is_float(dtype_)) throw Error(L3D_E_DTYPE, std::string("geglu: unsupported dtype ") + as_str(dtype_));
    if (rank() == 0 || layout_.dims.back() % 2)
      throw Error(L3D_E_SHAPE, "geglu: last dim of " + dims_str(layout_.dims) + " is not even");
    std::vector<int64_t> od = layout_.dims;
    od.back() /= 2;
    Tensor y = empty(od, dtype_, dev_);
    const l3d_tensor xd = desc(), yd = y.desc();
    check(l3d_geglu(&xd, &yd, dev_.stream), "l3d_geglu");
    return y;
  }

 private:
  Tensor view(Layout l) const { return Tensor(st_, std::move(l), dtype_, dev_); }
  Tensor unary(int (*fn)(const l3d_tensor*, const l3d_tensor*, l3d_stream), const char* op) const {
    if (!is_float(dtype_))
      throw Error(L3D_E_DTYPE, std::string(op) + ": unsupported dtype " + as_str(dtype_));
    Tensor y = empty_like();
    const l3d_tensor xd = desc(), yd = y.desc();
    check(fn(&xd, &yd, dev_.stream), op);
    return y;
  }

  std::shared_ptr<Storage> st_;
  Layout layout_;
  DType dtype_ = DType::F32;
  Device dev_;
};

namespace detail {
inline void require_float(const Tensor& t, const char* op, const char* what) {
  if (!is_float(t.dtype()))
    throw Error(L3D_E_DTYPE, std::string(op) + ": " + what + " has dtype " + as_str(t.dtype()));
}
inline void require_same_dtype(const Tensor& a, const Tensor& b, const char* op) {
  if (a.dtype() != b.dtype())
    throw Error(L3D_E_DTYPE, std::string(op) + ": dtype mismatch " + as_str(a.dtype()) + " vs " +
                                 as_str(b.dtype()));
}
inline void require_dims(const Tensor& t, const std::vector<int64_t>& want, const char* op,
                         const char* what) {
  if (t.dims() != want)
    throw Error(L3D_E_SHAPE, std::string(op) + ": " + what + " has shape " + dims_str(t.dims()) +
                                 ", expected " + dims_str(want));
}
inline void require_rank(const Tensor& t, size_t r, const char* op, const char* what) {
  if (t.rank() != r)
    throw Error(L3D_E_SHAPE, std::string(op) + ": " + what + " has rank " +
                                 std::to_string(t.rank()) + ", expected " + std::to_string(r));
}
inline int64_t last_dim(const Tensor& x, const char* op) {
  if (x.rank() == 0) throw Error(L3D_E_SHAPE, std::string(op) + ": rank-0 input");
  return x.dims().back();
}
// Pointer to an optional descriptor kept alive by `slot`.
inline const l3d_tensor* opt_desc(const std::optional<Tensor>& t, l3d_tensor& slot) {
  if (!t) return nullptr;
  slot = t->desc();
  return &slot;
}
}  // namespace detail

// ================================================================ candle_nn
namespace nn {
namespace ops {

// candle_nn::ops::layer_norm(x, alpha, beta, eps): LayerNorm over the last dim
// with biased variance (crate/runtime/vggt.rs:104,107; pi3_encoder.rs:67,70).
inline Tensor layer_norm(const Tensor& x, const Tensor& alpha, const Tensor& beta, float eps) {
  const char* op = "layer-norm";
  detail::require_float(x, op, "x");
  const int64_t C = detail::last_dim(x, op);
  detail::require_dims(alpha, {C}, op, "alpha");
  detail::require_dims(beta, {C}, op, "beta");
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), ad = alpha.desc(), bd = beta.desc(), yd = y.desc();
  check(l3d_layer_norm(&xd, &ad, &bd, eps, &yd, x.device().stream), "l3d_layer_norm");
  return y;
}

namespace detail_rope {
inline void check_rope_tables(const Tensor& x, const Tensor& cos_full, const Tensor& sin_alt_full,
                              const char* op) {
  using namespace ::l3d::candle::detail;
  require_rank(x, 4, op, "x");
  if (x.dim(3) != 64)
    throw Error(L3D_E_SHAPE, std::string(op) + ": head dim " + std::to_string(x.dim(3)) +
                                 ", the fused op takes 64");
  const std::vector<int64_t> tab = {x.dim(0), 1, x.dim(2), 64};
  require_dims(cos_full, tab, op, "cos_full");
  require_dims(sin_alt_full, tab, op, "sin_alt_full");
  if (cos_full.dtype() != DType::F32 || sin_alt_full.dtype() != DType::F32)
    throw Error(L3D_E_DTYPE, std::string(op) + ": the tables are f32");
}
}  // namespace detail_rope

// candle_nn::ops::layernorm_rope_fused(q, w, b, eps, cos_full, sin_alt_full)
// (crate/runtime/attention_math.rs:127-150): per-head affine LayerNorm over
// D = 64, then the 2D RoPE of rope_apply (:104-118).  q [B, H, N, 64], any
// strides with the last one 1 (a head view of the fused qkv projection);
// cos_full / sin_alt_full [B, 1, N, 64] f32 (Rope2d::embeddings).
inline Tensor layernorm_rope_fused(const Tensor& q, const Tensor& w, const Tensor& b, float eps,
                                   const Tensor& cos_full, const Tensor& sin_alt_full) {
  const char* op = "layernorm-rope-fused";
  detail::require_float(q, op, "q");
  detail_rope::check_rope_tables(q, cos_full, sin_alt_full, op);
  detail::require_dims(w, {64}, op, "w");
  detail::require_dims(b, {64}, op, "b");
  Tensor y = q.empty_like();
  const l3d_tensor qd = q.desc(), wd = w.desc(), bd = b.desc(), cd = cos_full.desc(),
                   sd = sin_alt_full.desc(), yd = y.desc();
  check(l3d_layernorm_rope2d(&qd, &wd, &bd, eps, &cd, &sd, &yd, q.device().stream),
        "l3d_layernorm_rope2d");
  return y;
}

// candle_nn::ops::rope_fused(x, cos_full, sin_alt_full)
// (crate/runtime/attention_math.rs:155-165): the rotation alone.
inline Tensor rope_fused(const Tensor& x, const Tensor& cos_full, const Tensor& sin_alt_full) {
  const char* op = "rope-fused";
  detail::require_float(x, op, "x");
  detail_rope::check_rope_tables(x, cos_full, sin_alt_full, op);
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), cd = cos_full.desc(), sd = sin_alt_full.desc(), yd = y.desc();
  check(l3d_layernorm_rope2d(&xd, nullptr, nullptr, 0.f, &cd, &sd, &yd, x.device().stream),
        "l3d_layernorm_rope2d");
  return y;
}

// exact_sdpa_heads (crate/runtime/attention_math.rs:199-259), non-causal:
// softmax(q k^T * scale) v per (batch, head) on the tensor cores.  q [B, H, N,
// D], k / v [B, H, Nk, D] bf16 views with the head dim contiguous (D = 64 or
// 128), read in place.  `status`, when given, receives the kernel's status
// word storage (4 bytes at its start; 0 = every bounded wait completed),
// readable after the stream is synchronised.
inline Tensor sdpa(const Tensor& q, const Tensor& k, const Tensor& v, float scale,
                   std::shared_ptr<Storage>* status = nullptr) {
  const char* op = "sdpa";
  using namespace ::l3d::candle::detail;
  require_rank(q, 4, op, "q");
  require_rank(k, 4, op, "k");
  require_dims(v, k.dims(), op, "v");
  if (q.dtype() != DType::BF16 || k.dtype() != DType::BF16 || v.dtype() != DType::BF16)
    throw Error(L3D_E_DTYPE, "sdpa: q, k and v are bf16");
  if (k.dim(0) != q.dim(0) || k.dim(1) != q.dim(1) || k.dim(3) != q.dim(3))
    throw Error(L3D_E_SHAPE, "sdpa: q " + dims_str(q.dims()) + " and k " + dims_str(k.dims()) +
                                 " differ in batch, heads or head dim");
  if (!(scale > 0.f)) throw Error(L3D_E_SHAPE, "sdpa: scale must be positive");
  Tensor y = q.empty_like();
  const size_t need = l3d_attention_workspace_size(k.dim(0), k.dim(1), k.dim(2), k.dim(3));
  std::shared_ptr<Storage> ws = q.device().alloc(need);
  const l3d_tensor qd = q.desc(), kd = k.desc(), vd = v.desc(), yd = y.desc();
  check(l3d_attention(&qd, &kd, &vd, scale, &yd, ws->ptr, ws->bytes, q.device().stream),
        "l3d_attention");
  if (status) *status = ws;
  return y;
}

}  // namespace ops

// candle_nn::Linear::forward / ops::mul_mat_add on an unquantised bf16 weight
// [n, k] (crate/runtime/nn_blocks.rs:82,179-195), with the element-wise ops
// the blocks apply next fused into the GEMM epilogue:
//   y = residual + gate * act(x . W^T + bias)
// (Mlp fc1 + gelu_erf, crate/runtime/nn_blocks.rs:219-236; the LayerScale
// residual x + ls * proj(..), crate/runtime/vggt.rs:118-121).
enum class Act { None = 0, Silu = 1, GeluErf = 2, GeluTanh = 3 };

struct Linear {
  Tensor weight;
  std::optional<Tensor> bias;

  Tensor forward(const Tensor& x, Act act = Act::None, const std::optional<Tensor>& residual = {},
                 const std::optional<Tensor>& gate = {}) const {
    const char* op = "linear";
    using namespace ::l3d::candle::detail;
    require_rank(weight, 2, op, "weight");
    if (weight.dtype() != DType::BF16) throw Error(L3D_E_DTYPE, "linear: weight is bf16");
    const int64_t n = weight.dim(0), k = weight.dim(1);
    if (last_dim(x, op) != k)
      throw Error(L3D_E_SHAPE, "linear: x " + dims_str(x.dims()) + " against weight " +
                                   dims_str(weight.dims()));
    if (bias) require_dims(*bias, {n}, op, "bias");
    std::vector<int64_t> od = x.dims();
    od.back() = n;
    if (residual) require_dims(*residual, od, op, "residual");
    if (gate && !residual) throw Error(L3D_E_SHAPE, "linear: a gate needs a residual");
    Tensor y = Tensor::empty(od, DType::BF16, x.device());
    const int64_t m = x.elem_count() / k;
    std::shared_ptr<Storage> ws = x.device().alloc(l3d_linear_workspace_size(m, n, k));
    l3d_tensor bs{}, rs{}, gs{};
    const l3d_tensor xd = x.desc(), wd = weight.desc(), yd = y.desc();
    check(l3d_linear_ex(&xd, &wd, opt_desc(bias, bs), int(act), opt_desc(residual, rs),
                        opt_desc(gate, gs), &yd, ws->ptr, ws->bytes, x.device().stream),
          "l3d_linear_ex");
    return y;
  }
};

// candle_nn::LayerNorm { weight, bias, eps } (affine or not).
struct LayerNorm {
  std::optional<Tensor> weight, bias;
  float eps = 1e-5f;

  Tensor forward(const Tensor& x) const {
    const char* op = "layer-norm";
    candle::detail::require_float(x, op, "x");
    const int64_t C = candle::detail::last_dim(x, op);
    if (weight) candle::detail::require_dims(*weight, {C}, op, "weight");
    if (bias) candle::detail::require_dims(*bias, {C}, op, "bias");
    Tensor y = x.empty_like();
    l3d_tensor ws{}, bs{};
    const l3d_tensor xd = x.desc(), yd = y.desc();
    check(l3d_layer_norm(&xd, candle::detail::opt_desc(weight, ws),
                         candle::detail::opt_desc(bias, bs), eps, &yd, x.device().stream),
          "l3d_layer_norm");
    return y;
  }
};

// Rope2d::embeddings (crate/runtime/attention_math.rs:14-58): integer
// positions [B, N, 2] (y, x) -> cos_full, sin_alt_full [B, 1, N, head_dim] f32.
struct Rope2d {
  float theta = 100.f;

  std::pair<Tensor, Tensor> embeddings(const Tensor& positions, int64_t head_dim) const {
    const char* op = "rope2d-embeddings";
    candle::detail::require_rank(positions, 3, op, "positions");
    if (positions.dim(2) != 2) throw Error(L3D_E_SHAPE, "rope2d-embeddings: positions [B, N, 2]");
    if (is_float(positions.dtype()))
      throw Error(L3D_E_DTYPE, "rope2d-embeddings: positions are integers");
    const std::vector<int64_t> tab = {positions.dim(0), 1, positions.dim(1), head_dim};
    Tensor c = Tensor::empty(tab, DType::F32, positions.device());
    Tensor s = Tensor::empty(tab, DType::F32, positions.device());
    const l3d_tensor pd = positions.desc(), cd = c.desc(), sd = s.desc();
    check(l3d_rope2d_tables(&pd, theta, int(head_dim), &cd, &sd, positions.device().stream),
          "l3d_rope2d_tables");
    return {c, s};
  }
};

}  // namespace nn

// ================================================================ runtime
// The model-side compositions the reference builds from Candle primitives.
namespace runtime {

// layer_norm_no_affine (crate/runtime/trellis2_blocks.rs:280-286).
inline Tensor layer_norm_no_affine(const Tensor& x, float eps) {
  return nn::LayerNorm{std::nullopt, std::nullopt, eps}.forward(x);
}

// layer_norm_no_affine(x) * (1 + scale) + shift, the adaLN modulation of the
// TRELLIS.2 blocks (crate/runtime/trellis2_blocks.rs:627-630): x [B, N, C],
// shift / scale [B, 1, C], [B, C] or [C] (chunks of the [B, 6C] vector).
inline Tensor layer_norm_modulate(const Tensor& x, const Tensor& shift, const Tensor& scale,
                                  float eps) {
  const char* op = "layer-norm-modulate";
  detail::require_float(x, op, "x");
  detail::require_same_dtype(shift, scale, op);
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), sh = shift.desc(), sc = scale.desc(), yd = y.desc();
  check(l3d_layer_norm_modulate(&xd, nullptr, nullptr, &sh, &sc, nullptr, 0, eps, &yd,
                                x.device().stream),
        "l3d_layer_norm_modulate");
  return y;
}

// xs.add(h.broadcast_mul(gate)) (crate/runtime/trellis2_blocks.rs:632-633).
inline Tensor gated_residual(const Tensor& x, const Tensor& h, const Tensor& gate) {
  const char* op = "gated-residual";
  detail::require_float(x, op, "x");
  detail::require_dims(h, x.dims(), op, "h");
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), hd = h.desc(), gd = gate.desc(), yd = y.desc();
  check(l3d_gated_residual(&xd, &hd, &gd, &yd, x.device().stream), "l3d_gated_residual");
  return y;
}

// LayerScale::forward + residual (crate/runtime/nn_blocks.rs:210-214,
// crate/runtime/vggt.rs:115-123): x + gamma * h, gamma [C].
inline Tensor layerscale_residual(const Tensor& x, const Tensor& h, const Tensor& gamma) {
  const char* op = "layerscale-residual";
  detail::require_float(x, op, "x");
  detail::require_dims(h, x.dims(), op, "h");
  detail::require_dims(gamma, {detail::last_dim(x, op)}, op, "gamma");
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), hd = h.desc(), gd = gamma.desc(), yd = y.desc();
  check(l3d_layerscale_residual(&xd, &hd, &gd, &yd, x.device().stream),
        "l3d_layerscale_residual");
  return y;
}

// RmsNormHeads::rms_norm_heads (crate/runtime/triposg_dit.rs:511-522):
// x / sqrt(mean(x^2) + eps) * w over the last dim; x may be a strided chunk
// view of the fused qkv projection (:436-454).
inline Tensor rms_norm_heads(const Tensor& x, const Tensor& w, float eps) {
  const char* op = "rms-norm-heads";
  detail::require_float(x, op, "x");
  detail::require_dims(w, {detail::last_dim(x, op)}, op, "w");
  Tensor y = x.empty_like();
  const l3d_tensor xd = x.desc(), wd = w.desc(), yd = y.desc();
  check(l3d_rms_norm_heads(&xd, &wd, eps, &yd, x.device().stream), "l3d_rms_norm_heads");
  return y;
}

// Trellis2QkRmsNorm::forward then Trellis2Rope3d::apply
// (crate/runtime/trellis2_blocks.rs:306-319, :106-160) in one pass: x [B, L, H,
// D], gamma [H, D] f32, coords [L, 3] integer voxel coordinates, or none for
// the norm alone (the cross attention).
inline Tensor qk_rms_norm_rope3d(const Tensor& x, const Tensor& gamma,
                                 const std::optional<Tensor>& coords, float theta = 10000.f) {
  const char* op = "qk-rms-norm-rope3d";
  detail::require_float(x, op, "x");
  detail::require_rank(x, 4, op, "x");
  detail::require_dims(gamma, {x.dim(2), x.dim(3)}, op, "gamma");
  if (coords) {
    detail::require_dims(*coords, {x.dim(1), 3}, op, "coords");
    if (is_float(coords->dtype())) throw Error(L3D_E_DTYPE, "qk-rms-norm-rope3d: coords are integers");
  }
  Tensor y = x.empty_like();
  l3d_tensor cs{};
  const l3d_tensor xd = x.desc(), gd = gamma.desc(), yd = y.desc();
  check(l3d_qk_l2norm_rope3d(&xd, &gd, detail::opt_desc(coords, cs), theta, &yd,
                             x.device().stream),
        "l3d_qk_l2norm_rope3d");
  return y;
}

// timestep_embedding: TRELLIS.2 (cos first, crate/runtime/trellis2_blocks.rs:
// 184-204) or TripoSG (sin first, crate/runtime/triposg_dit.rs:280-294).
enum class TimestepOrder { CosFirst = 0, SinFirst = 1 };
inline Tensor timestep_embedding(const Tensor& t, int64_t dim, TimestepOrder order, DType out,
                                 float max_period = 10000.f) {
  const char* op = "timestep-embedding";
  detail::require_rank(t, 1, op, "t");
  if (t.dtype() != DType::F32) throw Error(L3D_E_DTYPE, "timestep-embedding: t is f32");
  Tensor y = Tensor::empty({t.dim(0), dim}, out, t.device());
  const l3d_tensor td = t.desc(), yd = y.desc();
  check(l3d_timestep_embedding(&td, int(dim), int(order), max_period, &yd, t.device().stream),
        "l3d_timestep_embedding");
  return y;
}

// The block seam: residual, then the next (modulated) norm, one pass
// (crate/runtime/vggt.rs:118-121; crate/runtime/trellis2_blocks.rs:632-642):
//   r = x + [gate *] h;  y = LN(r) [* w + b] [* (1 + scale) + shift].
// Returns (r, y).
inline std::pair<Tensor, Tensor> residual_layer_norm_modulate(
    const Tensor& x, const Tensor& h, const std::optional<Tensor>& gate,
    const std::optional<Tensor>& weight, const std::optional<Tensor>& bias,
    const std::optional<Tensor>& shift, const std::optional<Tensor>& scale, float eps) {
  const char* op = "residual-layer-norm-modulate";
  detail::require_float(x, op, "x");
  detail::require_dims(h, x.dims(), op, "h");
  Tensor r = x.empty_like(), y = x.empty_like();
  l3d_tensor gs{}, ws{}, bs{}, shs{}, scs{};
  const l3d_tensor xd = x.desc(), hd = h.desc(), rd = r.desc(), yd = y.desc();
  check(l3d_residual_layer_norm_modulate(
            &xd, &hd, detail::opt_desc(gate, gs), detail::opt_desc(weight, ws),
            detail::opt_desc(bias, bs), detail::opt_desc(shift, shs), detail::opt_desc(scale, scs),
            eps, &rd, &yd, x.device().stream),
        "l3d_residual_layer_norm_modulate");
  return {r, y};
}

// The small per-step linears (Trellis2AdaLn, the timestep MLPs, modulation +
// t_emb; crate/runtime/trellis2_blocks.rs:209-258,617,
// crate/runtime/triposg_dit.rs:295-299): y = act_out(act_in(x) . w^T + bias +
// addend), x [B, K] with B <= 16, w [N, K].
inline Tensor linear_small(const Tensor& x, const Tensor& w, const std::optional<Tensor>& bias,
                           const std::optional<Tensor>& addend, nn::Act act_in, nn::Act act_out) {
  const char* op = "linear-small";
  detail::require_rank(x, 2, op, "x");
  detail::require_rank(w, 2, op, "w");
  if (w.dim(1) != x.dim(1))
    throw Error(L3D_E_SHAPE, "linear-small: x " + dims_str(x.dims()) + " against w " +
                                 dims_str(w.dims()));
  Tensor y = Tensor::empty({x.dim(0), w.dim(0)}, x.dtype(), x.device());
  l3d_tensor bs{}, as{};
  const l3d_tensor xd = x.desc(), wd = w.desc(), yd = y.desc();
  check(l3d_linear_small(&xd, &wd, detail::opt_desc(bias, bs), detail::opt_desc(addend, as),
                         int(act_in), int(act_out), &yd, x.device().stream),
        "l3d_linear_small");
  return y;
}

// PatchEmbed + prepare_tokens (crate/runtime/pi3_encoder.rs:116-126,219-231):
// pixels [BS, Cin, H, W], weight [C, Cin, p, p], bias [C], pos [1 + np, C],
// cls [C], reg [R, C] or none -> [BS, 1 + R + np, C].
inline Tensor patch_embed(const Tensor& pixels, const Tensor& weight, const Tensor& bias,
                          const Tensor& pos, const Tensor& cls, const std::optional<Tensor>& reg,
                          int64_t patch) {
  const char* op = "patch-embed";
  detail::require_rank(pixels, 4, op, "pixels");
  detail::require_rank(weight, 4, op, "weight");
  if (patch <= 0 || pixels.dim(2) % patch || pixels.dim(3) % patch)
    throw Error(L3D_E_SHAPE, "patch-embed: image " + dims_str(pixels.dims()) +
                                 " is not whole patches of " + std::to_string(patch));
  const int64_t np = (pixels.dim(2) / patch) * (pixels.dim(3) / patch);
  const int64_t R = reg ? reg->dim(0) : 0;
  Tensor y = Tensor::empty({pixels.dim(0), 1 + R + np, weight.dim(0)}, pixels.dtype(),
                           pixels.device());
  l3d_tensor rs{};
  const l3d_tensor px = pixels.desc(), wd = weight.desc(), bd = bias.desc(), pd = pos.desc(),
                   cd = cls.desc(), yd = y.desc();
  check(l3d_patch_embed(&px, &wd, &bd, &pd, &cd, detail::opt_desc(reg, rs), int(patch), &yd,
                        pixels.device().stream),
        "l3d_patch_embed");
  return y;
}

// CoordMap + the per-offset pair loops (crate/runtime/trellis2_sparse.rs:
// 68-106,211-236): coords [N, 3] i32 -> pair_dest, pair_src [27, N] and counts
// [27] (i32), offset k's pairs in ascending destination order.
struct NeighborPairs {
  Tensor pair_dest, pair_src, counts;
};
inline NeighborPairs neighbor_pairs(const Tensor& coords) {
  const char* op = "neighbor-pairs";
  detail::require_rank(coords, 2, op, "coords");
  if (coords.dim(1) != 3 || coords.dtype() != DType::I32)
    throw Error(L3D_E_SHAPE, "neighbor-pairs: coords are [N, 3] i32");
  const int64_t n = coords.dim(0);
  const Device& d = coords.device();
  NeighborPairs p{Tensor::empty({27, n}, DType::I32, d), Tensor::empty({27, n}, DType::I32, d),
                  Tensor::empty({27}, DType::I32, d)};
  std::shared_ptr<Storage> ws = d.alloc(l3d_sparse_neighbor_pairs_workspace_size(n));
  const l3d_tensor cd = coords.desc(), dd = p.pair_dest.desc(), sd = p.pair_src.desc(),
                   nd = p.counts.desc();
  check(l3d_sparse_neighbor_pairs(&cd, &dd, &sd, &nd, ws->ptr, ws->bytes, d.stream),
        "l3d_sparse_neighbor_pairs");
  return p;
}

// index_select_rows (crate/runtime/trellis2_sparse.rs:118-133).
inline Tensor index_select_rows(const Tensor& feats, const Tensor& ids) {
  const char* op = "index-select-rows";
  detail::require_rank(feats, 2, op, "feats");
  detail::require_rank(ids, 1, op, "ids");
  Tensor y = Tensor::empty({ids.dim(0), feats.dim(1)}, feats.dtype(), feats.device());
  const l3d_tensor fd = feats.desc(), id = ids.desc(), yd = y.desc();
  check(l3d_index_select_rows(&fd, &id, &yd, feats.device().stream), "l3d_index_select_rows");
  return y;
}

}  // namespace runtime

// ================================================================ quantized
namespace quantized {

enum class GgmlDType { Q4_0 = L3D_Q4_0, Q8_0 = L3D_Q8_0, Q4K = L3D_Q4_K, Q5K = L3D_Q5_K,
                       Q6K = L3D_Q6_K };

inline int64_t block_elems(GgmlDType f) {
  return (f == GgmlDType::Q4_0 || f == GgmlDType::Q8_0) ? 32 : 256;
}
inline int64_t block_bytes(GgmlDType f) {
  switch (f) {
    case GgmlDType::Q8_0: return 34;
    case GgmlDType::Q4_0: return 18;
    case GgmlDType::Q4K: return 144;
    case GgmlDType::Q5K: return 176;
    default: return 210;
  }
}

// QMatMul::forward on a GGML block matrix kept packed on the device
// (LinearInner::Quant, crate/runtime/nn_blocks.rs:51-56,80-95): y = x .
// deq(W)^T [+ bias].  The workspace the kernel needs is kept with the weight
// and grown on demand (stream-ordered, on the input's device).
class QMatMul {
 public:
  QMatMul(void* blocks, GgmlDType fmt, int64_t n, int64_t k, std::optional<Tensor> bias = {})
      : blocks_(blocks), fmt_(fmt), n_(n), k_(k), bias_(std::move(bias)) {
    if (!blocks_) throw Error(L3D_E_NULL, "qmatmul: null weight blocks");
    if (n_ <= 0 || k_ <= 0 || k_ % block_elems(fmt_))
      throw Error(L3D_E_SHAPE, "qmatmul: [" + std::to_string(n_) + ", " + std::to_string(k_) +
                                   "] is not whole blocks of " + std::to_string(block_elems(fmt_)));
    if (bias_) candle::detail::require_dims(*bias_, {n_}, "qmatmul", "bias");
  }
  int64_t n() const { return n_; }
  int64_t k() const { return k_; }
  size_t weight_bytes() const { return size_t(n_ * (k_ / block_elems(fmt_)) * block_bytes(fmt_)); }

  Tensor forward(const Tensor& x) const { return forward_ex(x, nn::Act::None, {}, {}); }

  // With the block's next element-wise ops in the GEMM epilogue:
  // y = residual + gate * act(x . deq(W)^T + bias) (Trellis2FeedForward's
  // mlp.0 + gelu, crate/runtime/trellis2_blocks.rs:558-561; the gated
  // residuals :632-633, :644-645).
  Tensor forward_ex(const Tensor& x, nn::Act act, const std::optional<Tensor>& residual,
                    const std::optional<Tensor>& gate) const {
    const char* op = "qmatmul";
    candle::detail::require_float(x, op, "x");
    if (candle::detail::last_dim(x, op) != k_)
      throw Error(L3D_E_SHAPE, "qmatmul: x has shape " + dims_str(x.dims()) + ", last dim must be " +
                                   std::to_string(k_));
    std::vector<int64_t> od = x.dims();
    od.back() = n_;
    if (residual) candle::detail::require_dims(*residual, od, op, "residual");
    if (gate && !residual) throw Error(L3D_E_SHAPE, "qmatmul: a gate needs a residual");
    const DType yt = residual ? residual->dtype() : (x.dtype() == DType::F32 ? DType::F32 : DType::BF16);
    Tensor y = Tensor::empty(od, yt, x.device());
    const int64_t m = x.elem_count() / k_;
    const size_t need = l3d_dequant_linear_workspace_size(int(fmt_), m, n_, k_);
    if (!ws_ || ws_->bytes < need) ws_ = x.device().alloc(need);
    l3d_tensor bs{}, rs{}, gs{};
    const l3d_tensor xd = x.desc(), yd = y.desc();
    if (act == nn::Act::None && !residual) {
      check(l3d_dequant_linear(&xd, blocks_, int(fmt_), n_, k_,
                               candle::detail::opt_desc(bias_, bs), &yd, ws_->ptr, ws_->bytes,
                               x.device().stream),
            "l3d_dequant_linear");
    } else {
      check(l3d_dequant_linear_ex(&xd, blocks_, int(fmt_), n_, k_,
                                  candle::detail::opt_desc(bias_, bs), int(act),
                                  candle::detail::opt_desc(residual, rs),
                                  candle::detail::opt_desc(gate, gs), &yd, ws_->ptr, ws_->bytes,
                                  x.device().stream),
            "l3d_dequant_linear_ex");
    }
    return y;
  }

 private:
  void* blocks_;
  GgmlDType fmt_;
  int64_t n_, k_;
  std::optional<Tensor> bias_;
  mutable std::shared_ptr<Storage> ws_;
};

}  // namespace quantized

}  // namespace candle
}  // namespace l3d
