// GGUF tensor index: the on-disk format whose tensors feed l3d_dequant_linear.
//
// The reference reads `model.gguf` with Candle's gguf_file::Content::read
// (crate/weights/mod.rs:596-650, written by crate/weights/quantize.rs:
// 255-295) and hands each quantized `*.weight` to QMatMul
// (crate/runtime/nn_blocks.rs:123-152).  This is host code over a byte buffer
// the caller provides (typically an mmap of the file): it reads the header,
// the metadata key/values and the tensor infos of the public GGUF layout
// (versions 2 and 3, little-endian) and reports, per tensor, its GGML type,
// its dims in row-major order (GGUF stores them fastest-first) and the byte
// range of its data.  No file I/O, no allocation, every read bounds-checked.
#include <string.h>

#include "common.cuh"
#include "qlinear.cuh"

namespace l3d {
namespace gguf {

enum ValueType {
  GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6,
  GT_BOOL = 7, GT_STRING = 8, GT_ARRAY = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};

// Size in bytes of a fixed-size metadata value type (0: not fixed-size).
static uint64_t scalar_size(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
  }
}

// (weights per block, bytes per block) of a GGML type id; (0, 0) if unknown.
static void type_block(int32_t type, int64_t* elems, int64_t* bytes) {
  switch (type) {
    case 0: *elems = 1; *bytes = 4; return;     // F32
    case 1: *elems = 1; *bytes = 2; return;     // F16
    case 30: *elems = 1; *bytes = 2; return;    // BF16
    case 2: *elems = 32; *bytes = 18; return;   // Q4_0
    case 3: *elems = 32; *bytes = 20; return;   // Q4_1
    case 6: *elems = 32; *bytes = 22; return;   // Q5_0
    case 7: *elems = 32; *bytes = 24; return;   // Q5_1
    case 8: *elems = 32; *bytes = 34; return;   // Q8_0
    case 9: *elems = 32; *bytes = 36; return;   // Q8_1
    case 10: *elems = 256; *bytes = 84; return;   // Q2_K
    case 11: *elems = 256; *bytes = 110; return;  // Q3_K
    case 12: *elems = 256; *bytes = 144; return;  // Q4_K
    case 13: *elems = 256; *bytes = 176; return;  // Q5_K
    case 14: *elems = 256; *bytes = 210; return;  // Q6_K
    case 15: *elems = 256; *bytes = 292; return;  // Q8_K
    default: *elems = 0; *bytes = 0; return;
  }
}

struct Reader {
  const uint8_t* p;
  uint64_t len, pos;
  bool ok = true;

  bool need(uint64_t n) {
    if (!ok || n > len - pos) ok = false;
    return ok;
  }
  template <typename V>
  V get() {
    V v{};
    if (need(sizeof(V))) {
      memcpy(&v, p + pos, sizeof(V));
      pos += sizeof(V);
    }
    return v;
  }
  // A GGUF string: u64 length + bytes (no terminator).
  bool str(const char** s, uint64_t* n) {
    const uint64_t l = get<uint64_t>();
    if (!need(l)) return false;
    *s = reinterpret_cast<const char*>(p + pos);
    *n = l;
    pos += l;
    return true;
  }
  bool skip(uint64_t n) {
    if (!need(n)) return false;
    pos += n;
    return true;
  }
  // Skips one metadata value of type t (arrays of arrays included).
  bool skip_value(uint32_t t, int depth = 0) {
    if (depth > 4) return ok = false;
    if (const uint64_t s = scalar_size(t)) return skip(s);
    if (t == GT_STRING) {
      const char* s;
      uint64_t n;
      return str(&s, &n);
    }
    if (t == GT_ARRAY) {
      const uint32_t et = get<uint32_t>();
      const uint64_t count = get<uint64_t>();
      if (!ok) return false;
      if (const uint64_t s = scalar_size(et)) {
        if (count > (len - pos) / s) return ok = false;
        return skip(count * s);
      }
      for (uint64_t i = 0; i < count && ok; ++i) skip_value(et, depth + 1);
      return ok;
    }
    return ok = false;
  }
};

struct Header {
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0, alignment = 32;
  uint64_t infos_pos = 0;  // first tensor info
};

// Parses the header and walks the metadata; optionally finds a string key.
static int read_header(Reader& r, Header& h, const char* op, const char* key = nullptr,
                       const char** kval = nullptr, uint64_t* kval_len = nullptr, bool* found = nullptr) {
  const uint32_t magic = r.get<uint32_t>();
  if (!r.ok || magic != 0x46554747u) return fail(L3D_E_SHAPE, "%s: not a GGUF buffer (bad magic)", op);
  h.version = r.get<uint32_t>();
  if (h.version != 2 && h.version != 3)
    return fail(L3D_E_UNSUPPORTED, "%s: GGUF version %u is not supported", op, h.version);
  h.n_tensors = r.get<uint64_t>();
  h.n_kv = r.get<uint64_t>();
  if (!r.ok) return fail(L3D_E_SHAPE, "%s: truncated header", op);
  const size_t klen = key ? strlen(key) : 0;
  for (uint64_t i = 0; i < h.n_kv; ++i) {
    const char* name;
    uint64_t nl;
    if (!r.str(&name, &nl)) return fail(L3D_E_SHAPE, "%s: truncated metadata key %llu", op, (unsigned long long)i);
    const uint32_t t = r.get<uint32_t>();
    if (!r.ok) return fail(L3D_E_SHAPE, "%s: truncated metadata", op);
    if (nl == 17 && memcmp(name, "general.alignment", 17) == 0 && t == GT_U32) {
      const uint32_t a = r.get<uint32_t>();
      if (!r.ok || a == 0 || (a & (a - 1)))
        return fail(L3D_E_SHAPE, "%s: general.alignment must be a power of two", op);
      h.alignment = a;
      continue;
    }
    if (key && found && t == GT_STRING && nl == klen && memcmp(name, key, klen) == 0) {
      if (!r.str(kval, kval_len)) return fail(L3D_E_SHAPE, "%s: truncated metadata value", op);
      *found = true;
      continue;
    }
    if (!r.skip_value(t)) return fail(L3D_E_SHAPE, "%s: malformed metadata value (key %llu)", op,
                                      (unsigned long long)i);
  }
  h.infos_pos = r.pos;
  return L3D_OK;
}

}  // namespace gguf
}  // namespace l3d

using namespace l3d;

extern "C" int l3d_gguf_index(const void* buf, uint64_t len, l3d_gguf_tensor* tensors,
                              int64_t max_tensors, int64_t* n_tensors, uint32_t* version,
                              uint64_t* alignment) {
  const char* op = "l3d_gguf_index";
  if (!buf || !n_tensors) return fail(L3D_E_NULL, "%s: buf and n_tensors are required", op);
  if (max_tensors > 0 && !tensors) return fail(L3D_E_NULL, "%s: tensors is required", op);
  gguf::Reader r{static_cast<const uint8_t*>(buf), len, 0};
  gguf::Header h;
  if (int rc = gguf::read_header(r, h, op)) return rc;
  if (h.n_tensors > (uint64_t(1) << 40)) return fail(L3D_E_SHAPE, "%s: implausible tensor count", op);
  // Tensor infos: name, n_dims, dims (fastest first), type, offset.  Every
  // tensor's data range is checked, also the ones not returned.
  int64_t filled = 0;
  uint64_t end_rel = 0;  // largest offset + nbytes, relative to the data section
  for (uint64_t i = 0; i < h.n_tensors; ++i) {
    const char* name;
    uint64_t nl;
    if (!r.str(&name, &nl)) return fail(L3D_E_SHAPE, "%s: truncated tensor info %llu", op, (unsigned long long)i);
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd == 0 || nd > 4)
      return fail(L3D_E_SHAPE, "%s: tensor %llu has %u dims (1..4 supported)", op, (unsigned long long)i, nd);
    uint64_t ne[4] = {1, 1, 1, 1};
    for (uint32_t d = 0; d < nd; ++d) ne[d] = r.get<uint64_t>();
    const int32_t type = static_cast<int32_t>(r.get<uint32_t>());
    const uint64_t off = r.get<uint64_t>();
    if (!r.ok) return fail(L3D_E_SHAPE, "%s: truncated tensor info %llu", op, (unsigned long long)i);
    if (off % h.alignment)
      return fail(L3D_E_SHAPE, "%s: tensor %llu data is not aligned to %llu", op,
                  (unsigned long long)i, (unsigned long long)h.alignment);
    int64_t be, bb;
    gguf::type_block(type, &be, &bb);
    uint64_t nbytes = 0;
    if (be > 0 && ne[0] % uint64_t(be) == 0) {
      uint64_t rows = 1;
      for (uint32_t d = 1; d < nd; ++d) {
        if (ne[d] != 0 && rows > (uint64_t(1) << 62) / ne[d])
          return fail(L3D_E_SHAPE, "%s: tensor %llu is implausibly large", op, (unsigned long long)i);
        rows *= ne[d];
      }
      nbytes = (ne[0] / uint64_t(be)) * uint64_t(bb);
      if (rows != 0 && nbytes > (uint64_t(1) << 62) / rows)
        return fail(L3D_E_SHAPE, "%s: tensor %llu is implausibly large", op, (unsigned long long)i);
      nbytes *= rows;
    }
    if (off > len || nbytes > len - off)
      return fail(L3D_E_SHAPE, "%s: tensor %llu data runs past the buffer (truncated file)", op,
                  (unsigned long long)i);
    if (off + nbytes > end_rel) end_rel = off + nbytes;
    if (filled < max_tensors) {
      l3d_gguf_tensor& t = tensors[filled++];
      t.name = name;
      t.name_len = nl;
      t.type = type;
      t.n_dims = int32_t(nd);
      for (int d = 0; d < 4; ++d) t.dims[d] = d < int(nd) ? int64_t(ne[nd - 1 - d]) : 1;
      t.offset = off;  // relative for now; made absolute below
      t.nbytes = nbytes;
    }
  }
  // Data section: the tensor infos end, rounded up to the alignment.
  const uint64_t data_start = (r.pos + h.alignment - 1) / h.alignment * h.alignment;
  if (data_start > len || end_rel > len - data_start)
    return fail(L3D_E_SHAPE, "%s: tensor data runs past the buffer (truncated file)", op);
  for (int64_t i = 0; i < filled; ++i) tensors[i].offset += data_start;
  *n_tensors = int64_t(h.n_tensors);
  if (version) *version = h.version;
  if (alignment) *alignment = h.alignment;
  return L3D_OK;
}

extern "C" int l3d_gguf_metadata_string(const void* buf, uint64_t len, const char* key,
                                        const char** value, uint64_t* value_len) {
  const char* op = "l3d_gguf_metadata_string";
  if (!buf || !key || !value || !value_len)
    return fail(L3D_E_NULL, "%s: buf, key, value and value_len are required", op);
  gguf::Reader r{static_cast<const uint8_t*>(buf), len, 0};
  gguf::Header h;
  bool found = false;
  *value = nullptr;
  *value_len = 0;
  if (int rc = gguf::read_header(r, h, op, key, value, value_len, &found)) return rc;
  if (!found) return fail(L3D_E_SHAPE, "%s: no string metadata `%s`", op, key);
  return L3D_OK;
}
