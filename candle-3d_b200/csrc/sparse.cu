// Sparse voxel index build and row gather (TRELLIS.2 submanifold conv plumbing).
//
// l3d_sparse_neighbor_pairs replaces the reference's host HashMap + 27 host
// loops + 27 host->device index uploads with four device passes over a
// caller-provided workspace:
//   1. insert every coordinate into an open-addressing hash table
//      (key = packed (x, y, z), value = row; duplicate keys keep the largest
//      row, i.e. the later one, as HashMap::insert does);
//   2. per (offset k, tile of 1024 rows) count the rows whose neighbour
//      coord + delta_k is present;
//   3. exclusive scan of the tile counts per offset (also yields counts[k]);
//   4. recompute the lookups and write (dest, src) pairs at their scanned
//      positions, so each offset's pairs come out in ascending dest order,
//      bit-identical to the reference loop.
#include <mutex>

#include "common.cuh"

namespace l3d {

constexpr int kTile = 1024;
constexpr uint64_t kEmpty = ~0ull;
constexpr int kCoordBits = 21;
constexpr int32_t kCoordMax = 1 << 20;  // valid coordinates: [-2^20, 2^20)

__device__ __forceinline__ bool pack_coord(int32_t x, int32_t y, int32_t z, uint64_t* key) {
  if (x < -kCoordMax || x >= kCoordMax || y < -kCoordMax || y >= kCoordMax || z < -kCoordMax ||
      z >= kCoordMax)
    return false;
  const uint64_t ux = uint64_t(x + kCoordMax), uy = uint64_t(y + kCoordMax),
                 uz = uint64_t(z + kCoordMax);
  *key = (ux << (2 * kCoordBits)) | (uy << kCoordBits) | uz;
  return true;
}

// 64-bit finaliser (SplitMix64 / MurmurHash3 fmix style mixing).
__device__ __forceinline__ uint64_t mix64(uint64_t k) {
  k ^= k >> 30;
  k *= 0xbf58476d1ce4e5b9ull;
  k ^= k >> 27;
  k *= 0x94d049bb133111ebull;
  k ^= k >> 31;
  return k;
}

struct SparseWs {
  unsigned long long* keys;  // [cap]
  int32_t* vals;             // [cap]
  int32_t* tile_counts;      // [27][tiles]
  uint64_t cap;              // power of two
  int64_t tiles;
};

__global__ void hash_insert_kernel(const int32_t* __restrict__ coords, int64_t cs0, int64_t cs1,
                                   int64_t n, SparseWs ws) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int32_t* c = coords + i * cs0;
    uint64_t key;
    if (!pack_coord(c[0], c[cs1], c[2 * cs1], &key)) continue;
    uint64_t slot = mix64(key) & (ws.cap - 1);
    for (uint64_t probe = 0; probe < ws.cap; ++probe) {
      const unsigned long long prev = atomicCAS(&ws.keys[slot], kEmpty, key);
      if (prev == kEmpty || prev == key) {
        atomicMax(&ws.vals[slot], int32_t(i));
        break;
      }
      slot = (slot + 1) & (ws.cap - 1);
    }
  }
}

__device__ __forceinline__ int32_t hash_find(const SparseWs& ws, uint64_t key) {
  uint64_t slot = mix64(key) & (ws.cap - 1);
  for (uint64_t probe = 0; probe < ws.cap; ++probe) {
    const uint64_t k = ws.keys[slot];
    if (k == key) return ws.vals[slot];
    if (k == kEmpty) return -1;
    slot = (slot + 1) & (ws.cap - 1);
  }
  return -1;
}

__device__ __forceinline__ int32_t neighbour(const int32_t* __restrict__ coords, int64_t cs0,
                                             int64_t cs1, int64_t i, int k, const SparseWs& ws) {
  const int32_t* c = coords + i * cs0;
  const int dx = k / 9 - 1, dy = (k % 9) / 3 - 1, dz = k % 3 - 1;
  uint64_t key;
  // Coordinates outside the packable range are never present.
  if (!pack_coord(c[0], c[cs1], c[2 * cs1], &key)) return -1;
  if (!pack_coord(c[0] + dx, c[cs1] + dy, c[2 * cs1] + dz, &key)) return -1;
  return hash_find(ws, key);
}

// grid (tiles, 27): count hits per (offset, tile).
__global__ void __launch_bounds__(kTile) pair_count_kernel(const int32_t* __restrict__ coords,
                                                           int64_t cs0, int64_t cs1, int64_t n,
                                                           SparseWs ws) {
  __shared__ int32_t warp_sum[kTile / 32];
  const int k = blockIdx.y;
  const int64_t i = int64_t(blockIdx.x) * kTile + threadIdx.x;
  const int hit = (i < n && neighbour(coords, cs0, cs1, i, k, ws) >= 0) ? 1 : 0;
  const int c = __popc(__ballot_sync(0xffffffffu, hit));
  if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = warp_sum[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) ws.tile_counts[int64_t(k) * ws.tiles + blockIdx.x] = v;
  }
}

// One block per offset: exclusive scan over the tile counts (in place) and the
// total into counts[k].
__global__ void __launch_bounds__(1024) pair_scan_kernel(SparseWs ws, int32_t* counts) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  const int k = blockIdx.x;
  int32_t* tc = ws.tile_counts + int64_t(k) * ws.tiles;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < ws.tiles; base += 1024) {
    const int64_t t = base + threadIdx.x;
    const int32_t v = t < ws.tiles ? tc[t] : 0;
    // Inclusive warp scan.
    int32_t x = v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int32_t before = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + x - v;
    if (t < ws.tiles) tc[t] = before;
    __syncthreads();
    if (threadIdx.x == 1023) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[k] = carry;
}

// grid (tiles, 27): write pairs at tile offset + in-tile exclusive rank.
__global__ void __launch_bounds__(kTile) pair_write_kernel(const int32_t* __restrict__ coords,
                                                           int64_t cs0, int64_t cs1, int64_t n,
                                                           SparseWs ws, int32_t* dest,
                                                           int32_t* src, int64_t row_stride) {
  __shared__ int32_t warp_sum[kTile / 32];
  const int k = blockIdx.y;
  const int64_t i = int64_t(blockIdx.x) * kTile + threadIdx.x;
  const int32_t s = i < n ? neighbour(coords, cs0, cs1, i, k, ws) : -1;
  const int hit = s >= 0 ? 1 : 0;
  const unsigned mask = __ballot_sync(0xffffffffu, hit);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_sum[warp] = __popc(mask);
  __syncthreads();
  if (threadIdx.x < 32) {
    int32_t x = warp_sum[lane];
    const int32_t v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    warp_sum[lane] = x - v;  // exclusive
  }
  __syncthreads();
  if (hit) {
    const int32_t pos = ws.tile_counts[int64_t(k) * ws.tiles + blockIdx.x] + warp_sum[warp] +
                        __popc(mask & ((1u << lane) - 1u));
    dest[int64_t(k) * row_stride + pos] = int32_t(i);
    src[int64_t(k) * row_stride + pos] = s;
  }
}

// nbr[i, k] = row of coord_i + delta_k, or -1 (the dense form of the pair
// lists, consumed by the sparse-conv gather GEMM).
__global__ void neighbor_map_kernel(const int32_t* __restrict__ coords, int64_t cs0, int64_t cs1,
                                    int64_t n, SparseWs ws, int32_t* __restrict__ nbr,
                                    int64_t ns0) {
  const int64_t total = n * 27;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = t / 27;
    const int k = int(t - i * 27);
    nbr[i * ns0 + k] = neighbour(coords, cs0, cs1, i, k, ws);
  }
}

template <typename T, typename I>
__global__ void index_select_kernel(const T* __restrict__ feats, int64_t fs0, int64_t nrows,
                                    const I* __restrict__ ids, int64_t is0, T* __restrict__ out,
                                    int64_t os0, int64_t n, int64_t C) {
  // One warp per output row, 16-byte accesses when the row allows.
  constexpr int V = Vec16<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const bool vec = (C % V == 0) && (fs0 % V == 0) && (os0 % V == 0) &&
                   (reinterpret_cast<uintptr_t>(feats) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  for (int64_t j = warp0; j < n; j += nw) {
    const int64_t r = int64_t(ids[j * is0]);
    const bool ok = r >= 0 && r < nrows;  // out-of-range ids produce zero rows
    T* o = out + j * os0;
    const T* f = feats + (ok ? r : 0) * fs0;
    if (vec) {
      for (int64_t c = int64_t(lane) * V; c < C; c += 32 * V) {
        uint4 u = ok ? __ldg(reinterpret_cast<const uint4*>(f + c)) : make_uint4(0, 0, 0, 0);
        st_act_raw(reinterpret_cast<uint4*>(o + c), u);
      }
    } else {
      for (int64_t c = lane; c < C; c += 32) o[c] = ok ? f[c] : from_f<T>(0.f);
    }
  }
}

static constexpr uint64_t table_cap(int64_t n) {
  uint64_t cap = 64;
  while (cap < uint64_t(2 * n)) cap <<= 1;
  return cap;
}

static constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static constexpr size_t sparse_ws_bytes(int64_t n) {
  const uint64_t cap = table_cap(n);
  const int64_t tiles = (n + kTile - 1) / kTile;
  return align256(cap * 8) + align256(cap * 4) + align256(size_t(27) * (tiles > 0 ? tiles : 1) * 4);
}

}  // namespace l3d

using namespace l3d;

extern "C" size_t l3d_sparse_neighbor_pairs_workspace_size(int64_t n) {
  return n < 0 ? 0 : sparse_ws_bytes(n);
}

extern "C" int l3d_sparse_neighbor_pairs(const l3d_tensor* coords, const l3d_tensor* pair_dest,
                                         const l3d_tensor* pair_src, const l3d_tensor* counts,
                                         void* workspace, size_t workspace_bytes,
                                         l3d_stream stream) {
  const char* op = "l3d_sparse_neighbor_pairs";
  const l3d_tensor* req[] = {coords, pair_dest, pair_src, counts};
  for (const l3d_tensor* t : req)
    if (!t) return fail(L3D_E_NULL, "%s: coords, pair_dest, pair_src, counts required", op);
  for (const l3d_tensor* t : req)
    if (t->dtype != L3D_I32) return fail(L3D_E_DTYPE, "%s: all index tensors must be I32", op);
  if (coords->ndim != 2 || coords->dims[1] != 3) return fail(L3D_E_SHAPE, "%s: coords [N, 3]", op);
  const int64_t n = coords->dims[0];
  // Empty coordinate lists (CoordMap::new(&[])) are valid; their views may
  // carry no storage.  counts always needs storage.
  if (no_data(counts) || (n > 0 && (no_data(coords) || no_data(pair_dest) || no_data(pair_src))))
    return fail(L3D_E_NULL, "%s: null data pointer", op);
  if (n >= (int64_t(1) << 31)) return fail(L3D_E_UNSUPPORTED, "%s: N must fit in I32", op);
  for (const l3d_tensor* t : {pair_dest, pair_src}) {
    if (t->ndim != 2 || t->dims[0] != 27 || t->dims[1] != n)
      return fail(L3D_E_SHAPE, "%s: pair_dest/pair_src must be [27, N]", op);
    if (n > 0 && ((n > 1 && t->strides[1] != 1) || t->strides[0] != n))
      return fail(L3D_E_ALIGN, "%s: pair tensors must be contiguous", op);
  }
  if (counts->ndim != 1 || counts->dims[0] != 27 || counts->strides[0] != 1)
    return fail(L3D_E_SHAPE, "%s: counts must be contiguous [27]", op);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t* cnt = static_cast<int32_t*>(counts->data) + counts->offset;
  if (n == 0) {
    if (cudaMemsetAsync(cnt, 0, 27 * sizeof(int32_t), s) != cudaSuccess)
      return fail(L3D_E_CUDA, "%s: memset failed", op);
    return L3D_OK;
  }
  const size_t need = sparse_ws_bytes(n);
  if (!workspace || workspace_bytes < need)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  SparseWs ws;
  ws.cap = table_cap(n);
  ws.tiles = (n + kTile - 1) / kTile;
  char* base = static_cast<char*>(workspace);
  ws.keys = reinterpret_cast<unsigned long long*>(base);
  base += align256(ws.cap * 8);
  ws.vals = reinterpret_cast<int32_t*>(base);
  base += align256(ws.cap * 4);
  ws.tile_counts = reinterpret_cast<int32_t*>(base);
  if (cudaMemsetAsync(ws.keys, 0xff, ws.cap * 8, s) != cudaSuccess ||
      cudaMemsetAsync(ws.vals, 0xff, ws.cap * 4, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: workspace clear failed", op);
  const int32_t* cp = static_cast<const int32_t*>(coords->data) + coords->offset;
  const int64_t cs0 = coords->strides[0], cs1 = coords->strides[1];
  int blocks = int((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  hash_insert_kernel<<<blocks, 256, 0, s>>>(cp, cs0, cs1, n, ws);
  const dim3 grid(unsigned(ws.tiles), 27);
  pair_count_kernel<<<grid, kTile, 0, s>>>(cp, cs0, cs1, n, ws);
  pair_scan_kernel<<<27, 1024, 0, s>>>(ws, cnt);
  pair_write_kernel<<<grid, kTile, 0, s>>>(cp, cs0, cs1, n, ws,
                                           static_cast<int32_t*>(pair_dest->data) + pair_dest->offset,
                                           static_cast<int32_t*>(pair_src->data) + pair_src->offset,
                                           n);
  return check_launch(op);
}

extern "C" int l3d_index_select_rows(const l3d_tensor* feats, const l3d_tensor* ids,
                                     const l3d_tensor* out, l3d_stream stream) {
  const char* op = "l3d_index_select_rows";
  if (!feats || !ids || !out || no_data(feats) || no_data(ids) || no_data(out))
    return fail(L3D_E_NULL, "%s: feats, ids, out required", op);
  if (!is_float_dtype(feats->dtype) || out->dtype != feats->dtype)
    return fail(L3D_E_DTYPE, "%s: feats/out must share a float dtype", op);
  if (!is_index_dtype(ids->dtype)) return fail(L3D_E_DTYPE, "%s: ids must be I32/U32/I64", op);
  if (feats->ndim != 2 || out->ndim != 2 || ids->ndim != 1)
    return fail(L3D_E_SHAPE, "%s: feats [N, C], ids [n], out [n, C]", op);
  const int64_t C = feats->dims[1], n = ids->dims[0];
  if (out->dims[0] != n || out->dims[1] != C) return fail(L3D_E_SHAPE, "%s: out must be [n, C]", op);
  if ((C > 1 && (feats->strides[1] != 1 || out->strides[1] != 1)))
    return fail(L3D_E_ALIGN, "%s: rows must be contiguous", op);
  if (n == 0 || C == 0) return L3D_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int64_t blocks = (n + 7) / 8;
  if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
  L3D_DISPATCH_FLOAT(feats->dtype, T, {
    const T* f = static_cast<const T*>(feats->data) + feats->offset;
    T* o = static_cast<T*>(out->data) + out->offset;
    if (ids->dtype == L3D_I64)
      index_select_kernel<T, int64_t><<<int(blocks), 256, 0, s>>>(
          f, feats->strides[0], feats->dims[0],
          static_cast<const int64_t*>(ids->data) + ids->offset, ids->strides[0], o,
          out->strides[0], n, C);
    else if (ids->dtype == L3D_U32)
      index_select_kernel<T, uint32_t><<<int(blocks), 256, 0, s>>>(
          f, feats->strides[0], feats->dims[0],
          static_cast<const uint32_t*>(ids->data) + ids->offset, ids->strides[0], o,
          out->strides[0], n, C);
    else
      index_select_kernel<T, int32_t><<<int(blocks), 256, 0, s>>>(
          f, feats->strides[0], feats->dims[0],
          static_cast<const int32_t*>(ids->data) + ids->offset, ids->strides[0], o,
          out->strides[0], n, C);
  });
  return check_launch(op);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of l3d_sparse_neighbor_pairs.
//
// Some callers cannot hand the library a workspace: a Candle `CustomOp`
// whose `cuda_fwd` only receives the input storages and returns one output
// allocation, a CUDA-graph replay whose buffers were fixed at capture, or a
// host runtime that forbids device allocation on its inference path.  For
// them the hash table and tile counts live in this file-scope device array,
// sized for at most kNoAllocMaxCoords coordinates.  Every GPU that loads the
// library holds the array until the process exits.
namespace l3d {
constexpr int64_t kNoAllocMaxCoords = 65536;
constexpr size_t kNoAllocCap = 131072;  // table slots for the maximum (>= 2N, power of two)
constexpr size_t kNoAllocTiles = (kNoAllocMaxCoords + kTile - 1) / kTile;
constexpr size_t kNoAllocBytes = ((kNoAllocCap * 8 + 255) & ~size_t(255)) +
                                 ((kNoAllocCap * 4 + 255) & ~size_t(255)) +
                                 ((27 * kNoAllocTiles * 4 + 255) & ~size_t(255));
// The fixed array must hold the workspace layout of the largest input.
static_assert(kNoAllocCap >= 2 * kNoAllocMaxCoords, "table needs two slots per coordinate");
static_assert((kNoAllocCap & (kNoAllocCap - 1)) == 0, "table size is a power of two");
static_assert(table_cap(kNoAllocMaxCoords) <= kNoAllocCap, "table of the largest input fits");
static_assert(kNoAllocBytes == sparse_ws_bytes(kNoAllocMaxCoords),
              "scratch bytes equal the workspace layout of the largest input");
static __device__ __align__(256) unsigned char g_pairs_scratch[kNoAllocBytes];

// Device address of g_pairs_scratch on the current device.  The host-side name
// of the array is only a stand-in for it, so the address is looked up once per
// device (with that device current) and cached.
static int pairs_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(L3D_E_CUDA, "l3d_sparse_neighbor_pairs_noalloc: no current device");
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_pairs_scratch);
    if (e != cudaSuccess || !p)
      return fail(L3D_E_CUDA, "l3d_sparse_neighbor_pairs_noalloc: cudaGetSymbolAddress: %s",
                  cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return L3D_OK;
}
}  // namespace l3d

extern "C" int l3d_sparse_neighbor_pairs_noalloc(const l3d_tensor* coords,
                                                 const l3d_tensor* pair_dest,
                                                 const l3d_tensor* pair_src,
                                                 const l3d_tensor* counts, l3d_stream stream) {
  const char* op = "l3d_sparse_neighbor_pairs_noalloc";
  const l3d_tensor* req[] = {coords, pair_dest, pair_src, counts};
  for (const l3d_tensor* t : req)
    if (!t) return fail(L3D_E_NULL, "%s: coords, pair_dest, pair_src, counts required", op);
  for (const l3d_tensor* t : req)
    if (t->dtype != L3D_I32) return fail(L3D_E_DTYPE, "%s: all index tensors must be I32", op);
  if (coords->ndim != 2 || coords->dims[1] != 3) return fail(L3D_E_SHAPE, "%s: coords [N, 3]", op);
  const int64_t n = coords->dims[0];
  if (n > kNoAllocMaxCoords)
    return fail(L3D_E_UNSUPPORTED,
                "%s: %lld coordinates exceed the fixed scratch limit of %lld; use "
                "l3d_sparse_neighbor_pairs with a workspace",
                op, (long long)n, (long long)kNoAllocMaxCoords);
  if (no_data(counts) || (n > 0 && (no_data(coords) || no_data(pair_dest) || no_data(pair_src))))
    return fail(L3D_E_NULL, "%s: null data pointer", op);
  for (const l3d_tensor* t : {pair_dest, pair_src}) {
    if (t->ndim != 2 || t->dims[0] != 27 || t->dims[1] != n)
      return fail(L3D_E_SHAPE, "%s: pair_dest/pair_src must be [27, N]", op);
    if (n > 0 && ((n > 1 && t->strides[1] != 1) || t->strides[0] != n))
      return fail(L3D_E_ALIGN, "%s: pair tensors must be contiguous", op);
  }
  if (counts->ndim != 1 || counts->dims[0] != 27 || counts->strides[0] != 1)
    return fail(L3D_E_SHAPE, "%s: counts must be contiguous [27]", op);
  void* scratch = nullptr;
  int rc = pairs_scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t* cnt = static_cast<int32_t*>(counts->data) + counts->offset;
  if (n == 0) {
    if (cudaMemsetAsync(cnt, 0, 27 * sizeof(int32_t), s) != cudaSuccess)
      return fail(L3D_E_CUDA, "%s: memset failed", op);
    return L3D_OK;
  }
  // Same passes as l3d_sparse_neighbor_pairs, over the fixed scratch array.
  // The table is cleared on every call (the array keeps the previous call's
  // contents); the tile counts are fully rewritten by the count pass.
  SparseWs ws;
  ws.cap = table_cap(n);
  ws.tiles = (n + kTile - 1) / kTile;
  if (sparse_ws_bytes(n) > kNoAllocBytes || ws.cap > kNoAllocCap)
    return fail(L3D_E_UNSUPPORTED, "%s: scratch layout of %lld coordinates exceeds the array", op,
                (long long)n);
  char* base = static_cast<char*>(scratch);
  ws.keys = reinterpret_cast<unsigned long long*>(base);
  base += align256(ws.cap * 8);
  ws.vals = reinterpret_cast<int32_t*>(base);
  base += align256(ws.cap * 4);
  ws.tile_counts = reinterpret_cast<int32_t*>(base);
  if (cudaMemsetAsync(ws.keys, 0xff, ws.cap * 8, s) != cudaSuccess ||
      cudaMemsetAsync(ws.vals, 0xff, ws.cap * 4, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: scratch clear failed", op);
  const int32_t* cp = static_cast<const int32_t*>(coords->data) + coords->offset;
  const int64_t cs0 = coords->strides[0], cs1 = coords->strides[1];
  const int blocks = int((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  hash_insert_kernel<<<blocks, 256, 0, s>>>(cp, cs0, cs1, n, ws);
  const dim3 grid(unsigned(ws.tiles), 27);
  pair_count_kernel<<<grid, kTile, 0, s>>>(cp, cs0, cs1, n, ws);
  pair_scan_kernel<<<27, 1024, 0, s>>>(ws, cnt);
  pair_write_kernel<<<grid, kTile, 0, s>>>(cp, cs0, cs1, n, ws,
                                           static_cast<int32_t*>(pair_dest->data) + pair_dest->offset,
                                           static_cast<int32_t*>(pair_src->data) + pair_src->offset,
                                           n);
  return check_launch(op);
}

extern "C" int l3d_sparse_neighbor_map(const l3d_tensor* coords, const l3d_tensor* nbr,
                                       void* workspace, size_t workspace_bytes,
                                       l3d_stream stream) {
  const char* op = "l3d_sparse_neighbor_map";
  if (!coords || !nbr) return fail(L3D_E_NULL, "%s: coords and nbr are required", op);
  if (coords->dtype != L3D_I32 || nbr->dtype != L3D_I32)
    return fail(L3D_E_DTYPE, "%s: coords and nbr must be I32", op);
  if (coords->ndim != 2 || coords->dims[1] != 3) return fail(L3D_E_SHAPE, "%s: coords [N, 3]", op);
  const int64_t n = coords->dims[0];
  if (nbr->ndim != 2 || nbr->dims[0] != n || nbr->dims[1] != 27)
    return fail(L3D_E_SHAPE, "%s: nbr must be [N, 27]", op);
  if (n == 0) return L3D_OK;
  if (no_data(coords) || no_data(nbr)) return fail(L3D_E_NULL, "%s: null data pointer", op);
  if (n >= (int64_t(1) << 31)) return fail(L3D_E_UNSUPPORTED, "%s: N must fit in I32", op);
  if (nbr->strides[1] != 1) return fail(L3D_E_ALIGN, "%s: nbr rows must be contiguous", op);
  const size_t need = sparse_ws_bytes(n);
  if (!workspace || workspace_bytes < need)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SparseWs ws;
  ws.cap = table_cap(n);
  ws.tiles = (n + kTile - 1) / kTile;
  char* base = static_cast<char*>(workspace);
  ws.keys = reinterpret_cast<unsigned long long*>(base);
  base += align256(ws.cap * 8);
  ws.vals = reinterpret_cast<int32_t*>(base);
  ws.tile_counts = nullptr;
  if (cudaMemsetAsync(ws.keys, 0xff, ws.cap * 8, s) != cudaSuccess ||
      cudaMemsetAsync(ws.vals, 0xff, ws.cap * 4, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: workspace clear failed", op);
  const int32_t* cp = static_cast<const int32_t*>(coords->data) + coords->offset;
  const int64_t cs0 = coords->strides[0], cs1 = coords->strides[1];
  int blocks = int((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  hash_insert_kernel<<<blocks, 256, 0, s>>>(cp, cs0, cs1, n, ws);
  const int64_t total = n * 27;
  const int64_t cap = int64_t(sm_count()) * 32;
  blocks = int((total + 255) / 256 < cap ? (total + 255) / 256 : cap);
  neighbor_map_kernel<<<blocks, 256, 0, s>>>(cp, cs0, cs1, n, ws,
                                             static_cast<int32_t*>(nbr->data) + nbr->offset,
                                             nbr->strides[0]);
  return check_launch(op);
}
