// Dequant-linear on the 5th-generation tensor cores (sm_100a).
//
//   y[M, N] = x[M, K] . deq(W)[N, K]^T (+ bias)   bf16 operands, f32 accumulate
//
// W arrives as raw GGML Q8_0 / Q4_0 blocks and is dequantised inside the
// kernel, in the operand prologue, never materialised in HBM.  Persistent,
// warp-specialised kernel, one CTA per SM, 128 x 256 output tiles, K in steps
// of 64, a 3-stage shared-memory ring:
//   warp 0       producer: one thread issues cp.async.bulk.tensor loads of the
//                x tile (128 x 64 bf16, 128B swizzle) and of the raw block
//                window of the W tile (256 rows x 96 B: the 16-byte-aligned
//                window holding the two GGML blocks of this K step);
//   warps 6..13  dequantisers: decode the raw window (f16 scale x int8 /
//                nibble), round to bf16 and write the K-major 128B-swizzled B
//                operand; fence.proxy.async, then arrive on the stage barrier;
//   warp 1       MMA issuer: one thread issues tcgen05.mma kind::f16
//                (M 128, N 256, K 16) into a double-buffered TMEM accumulator
//                (2 x 256 f32 columns) and commits stage / tile barriers;
//   warps 2..5   epilogue: tcgen05.ld of their TMEM lane quarter, + bias,
//                convert, store; overlaps the next tile's MMA.
// Weights whose rows are not 16-byte aligned (K % 256 != 0) are read by the
// dequantisers straight from global memory instead of the TMA window.
// Every mbarrier wait is bounded (wall-clock limit from %globaltimer); on
// expiry the CTA records an error in the status word, stops issuing work and
// still releases its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "act.cuh"
#include "common.cuh"
#include "qlinear.cuh"
#include "tc.cuh"

namespace l3d {
namespace gemm {

using namespace l3d::tc;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int RAW_ROW = 96;                 // bytes of the raw window per W row
constexpr int A_BYTES = BM * BK * 2;        // 16 KB
constexpr int B_BYTES = BN * BK * 2;        // 32 KB
constexpr int RAW_BYTES = BN * RAW_ROW;     // 24 KB
constexpr int TMEM_COLS = 512;              // two 256-column accumulators
constexpr int N_DQ_WARPS = 8;
constexpr int THREADS = (6 + N_DQ_WARPS) * 32;
// Epilogue staging (decode-once mode): per epilogue warp 32 rows x 64 columns
// in 128B-swizzled boxes of 128 bytes per row (one box of 64 bf16, or two of
// 32 f32), written by TMA stores whole 128-byte lines at a time.
constexpr int EPI_COLS = 64;
constexpr int EPI_WARP_BYTES = 32 * EPI_COLS * 4;  // 8 KB

// Operand modes.  MODE_RAW_TMA / MODE_RAW_LDG decode GGML blocks in the
// prologue (3 stages of x + B + raw window); MODE_BF16 streams a bf16 copy of
// the decoded weights with TMA (4 stages of x + B), used when the M dimension
// is large enough that decoding per 128-row tile would repeat the work
// hundreds of times.  MODE_GATHER is the submanifold sparse conv: the worker
// warps gather the A tile (the 27 neighbour rows of each output row, one
// kernel offset per Cin-wide stretch of K) and TMA streams the bf16
// [27, Cout, Cin] weights.
// MODE_PAIRS is the same conv over the compacted neighbour pairs of all 27
// offsets in one launch: offset k's pairs form a segment of whole 128-row
// tiles; a tile gathers its rows through the pair sources, multiplies by
// W[k] and stores the f32 products (a later pass adds them per output row in
// offset order).
// MODE_BF16_EPI8 is MODE_BF16 with eight epilogue warps (see EPI_WARPS).
enum { MODE_RAW_TMA = 0, MODE_RAW_LDG = 1, MODE_BF16 = 2, MODE_GATHER = 3, MODE_PAIRS = 4,
       MODE_BF16_EPI8 = 5 };
template <int MODE>
struct ModeCfg {
  static constexpr bool FUSED = MODE == MODE_RAW_TMA || MODE == MODE_RAW_LDG;  // decode W
  static constexpr bool PAIRS = MODE == MODE_PAIRS;
  static constexpr bool GATHER = MODE == MODE_GATHER || PAIRS;                 // gather A
  static constexpr bool WORKERS = FUSED || GATHER;  // warps 6.. build an operand
  static constexpr bool BF16W = MODE == MODE_BF16 || MODE == MODE_BF16_EPI8;  // bf16 W by TMA
  // MODE_BF16_EPI8 gives the idle worker warps 6-9 to the epilogue: eight
  // epilogue warps, each on half of the tile's columns, for one pipeline
  // stage less.  It pays when an activation runs in the epilogue (the
  // epilogue then bounds the kernel at small K); a plain GEMM keeps the
  // fourth stage.
  static constexpr int EPI_WARPS = MODE == MODE_BF16_EPI8 ? 8 : 4;
  static constexpr int NST = FUSED ? 3 : MODE == MODE_BF16_EPI8 ? 3 : 4;
  static constexpr int RAW = FUSED ? RAW_BYTES : 0;
  static constexpr int EPI = FUSED ? 0 : EPI_WARPS * EPI_WARP_BYTES;  // fused modes store directly
  static constexpr int SMEM = NST * (A_BYTES + B_BYTES + RAW) + EPI + 1024 + 512;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(3 * NST + 7 + 2 * EPI_WARPS <= 512 / 8, "barrier area");
};
// Status word codes written by the kernel into the workspace header.
constexpr int ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_TIMEOUT_TMEM = 3, ST_TIMEOUT_RAW = 4;

// kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = 256.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) |
                           (uint32_t(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(IDESC), "r"(accumulate)
      : "memory");
}
struct Params {
  int M, N, K;
  const void* bias;   // [N] or null
  int bias_dtype;
  void* y;            // [M, N] rows of y_ld elements
  int64_t y_ld;
  int y_dtype;
  int* status;        // workspace header
  const uint8_t* wq;  // raw GGML blocks, rows of row_bytes
  int64_t row_bytes;
  int fmt;
  int bpt;            // raw bytes per 64-wide K step (2 blocks)
  int tma_store;      // epilogue writes y through the map_y tensor map
  int y_vec;          // y's base and row stride are 16-byte aligned (vector stores)
  int bias_vec;       // bias is 16-byte aligned (vector loads)
  // Fused epilogue: y = res + gate * act(acc + bias).
  int act;            // Act code (0: none)
  const void* res;    // [M, N] rows of res_ld elements, y's dtype; null: none
  int64_t res_ld;
  int res_vec;        // res rows are 16-byte aligned (vector loads)
  int res_tma;        // TMA-store epilogue: res tiles arrive by TMA (map_r)
  const void* gate;   // [N] or null (= 1)
  int gate_dtype;
  // Sparse conv (MODE_GATHER): A[m, k * cin_pad + c] = feats[nbr[m, k], c]
  // (0 for nbr < 0 or c >= cin).
  const int32_t* nbr;              // [M, 27]
  const __nv_bfloat16* feats;      // rows of feats_ld elements
  int64_t feats_ld;
  int cin, cin_pad;                // cin_pad = cin rounded up to BK
  // MODE_PAIRS: segment k = tiles [seg_tile[k], seg_tile[k + 1]) holds the
  // seg_count[k] pairs of offset k, A rows feats[psrc[k * pstride + j]].
  const int32_t* psrc;
  int64_t pstride;
  int seg_tile[28];
  int seg_count[27];
};

// The fused epilogue ops on NC consecutive columns [col0, col0 + NC) of one
// row, after the bias: the activation (the reduced-cost forms for 16-bit
// outputs), then the gated residual, 8 columns at a time.  Columns past N are
// left alone.
template <int A, bool FAST, int NC>
__device__ __forceinline__ void act_chunk(float (&v)[NC]) {
#pragma unroll
  for (int i = 0; i < NC; ++i) v[i] = act_t<A, FAST>(v[i]);
}
// One dispatch per chunk, so each variant's loop is contiguous code.
template <int NC>
__device__ __forceinline__ void epi_act(int act, bool fast, float (&v)[NC]) {
  if (fast) {
    switch (act) {
      case ACT_SILU: act_chunk<ACT_SILU, true>(v); break;
      case ACT_GELU_ERF: act_chunk<ACT_GELU_ERF, true>(v); break;
      case ACT_GELU_TANH: act_chunk<ACT_GELU_TANH, true>(v); break;
      default: break;
    }
  } else {
    switch (act) {
      case ACT_SILU: act_chunk<ACT_SILU, false>(v); break;
      case ACT_GELU_ERF: act_chunk<ACT_GELU_ERF, false>(v); break;
      case ACT_GELU_TANH: act_chunk<ACT_GELU_TANH, false>(v); break;
      default: break;
    }
  }
}

template <int NC>
__device__ __forceinline__ void epi_post(const Params& p, int row, int col0, float (&v)[NC]) {
  if (p.act) epi_act<NC>(p.act, p.y_dtype != L3D_F32, v);
  if (!p.res || row >= p.M) return;
  const bool bf = p.y_dtype == L3D_BF16;
  const char* rrow = static_cast<const char*>(p.res) + (int64_t(row) * p.res_ld + col0) * (bf ? 2 : 4);
#pragma unroll
  for (int q = 0; q < NC / 8; ++q) {
    const int c = col0 + 8 * q;
    if (c >= p.N) break;
    float r[8], g[8];
    if (c + 8 <= p.N && p.res_vec) {
      if (bf) {
        unpack(__ldg(reinterpret_cast<const uint4*>(rrow) + q), r, __nv_bfloat16());
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(rrow) + 2 * q);
        const float4 b = __ldg(reinterpret_cast<const float4*>(rrow) + 2 * q + 1);
        r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w; r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c + e < p.N ? 8 * q + e : 8 * q;  // clamp to a valid column
        r[e] = bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(rrow)[i])
                  : __ldg(reinterpret_cast<const float*>(rrow) + i);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = c + e < p.N ? c + e : p.N - 1;
      g[e] = !p.gate ? 1.f
             : p.gate_dtype == L3D_F32 ? __ldg(static_cast<const float*>(p.gate) + col)
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(p.gate)[col]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (c + e < p.N) v[8 * q + e] = fmaf(g[e], v[8 * q + e], r[e]);
  }
}

// int8 -> f32 exactly: place (q ^ 0x80) = q + 128 in the mantissa of 2^23.
__device__ __forceinline__ float i8_to_f(uint32_t byte) {
  return __uint_as_float(0x4B000000u | (byte ^ 0x80u)) - 8388736.0f;
}
// 4-bit GGML code -> (code - 8) as f32.
__device__ __forceinline__ float q4_to_f(uint32_t nib) {
  return __uint_as_float(0x4B000000u | nib) - 8388616.0f;
}

// Decode one 32-weight block (2-byte aligned; src is smem or global) into
// floats, w = d * q.
template <bool GLOBAL>
__device__ __forceinline__ void decode32(const uint8_t* blk, int fmt, float (&w)[32]) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(blk);
  auto ld = [&](int i) -> uint32_t {
    if constexpr (GLOBAL) return __ldg(h + i);
    else return h[i];
  };
  const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(ld(0))));
  if (fmt == L3D_Q8_0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t v = ld(1 + j);
      w[2 * j] = d * i8_to_f(v & 0xffu);
      w[2 * j + 1] = d * i8_to_f(v >> 8);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t v = ld(1 + j);
      w[2 * j] = d * q4_to_f(v & 15u);
      w[2 * j + 1] = d * q4_to_f((v >> 8) & 15u);
      w[16 + 2 * j] = d * q4_to_f((v >> 4) & 15u);
      w[16 + 2 * j + 1] = d * q4_to_f(v >> 12);
    }
  }
}

// Dequantise the 256 x 64 W tile of (n0, kb) into the K-major SW128 layout:
// row r occupies 128 B at (r / 8) * 1024 + (r % 8) * 128; its 16-byte chunk c
// is stored at chunk (c ^ (r % 8)).  256 threads, 512 block jobs.
template <bool RAW_TMA>
__device__ __forceinline__ void dequant_tile(const Params& p, const uint8_t* raw, uint8_t* tile,
                                             int n0, int kb, int t) {
  const int bb = p.fmt == L3D_Q8_0 ? 34 : 18;
  const int win_off = (kb * p.bpt) & 15;  // offset of the K step inside the 16-byte aligned window
#pragma unroll 1
  for (int job = t; job < BN * 2; job += N_DQ_WARPS * 32) {
    const int r = job >> 1;      // tile row
    const int half = job & 1;    // which 32-element block of the 64
    const int n = n0 + r;
    const int kblk = kb * 2 + half;
    float w[32];
    if (n < p.N && kblk * 32 < p.K) {
      if constexpr (RAW_TMA) {
        decode32<false>(raw + r * RAW_ROW + win_off + half * bb, p.fmt, w);
      } else {
        decode32<true>(p.wq + int64_t(n) * p.row_bytes + int64_t(kblk) * bb, p.fmt, w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = 0.f;
    }
    uint8_t* row = tile + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = w[c * 8 + e];
      const int chunk = half * 4 + c;
      *reinterpret_cast<uint4*>(row + ((chunk ^ (r & 7)) << 4)) = pack(f, __nv_bfloat16());
    }
  }
}

// v[i] += bias[col0 + i] for NC columns: 16-byte loads through the read-only
// path when the chunk lies inside N and the bias is 16-byte aligned (f32 or
// bf16), else one element at a time (columns past N are left alone).
template <int NC>
__device__ __forceinline__ void add_bias(const Params& p, int col0, float (&v)[NC]) {
  if (col0 + NC <= p.N && p.bias_vec) {
    if (p.bias_dtype == L3D_F32) {
      const float4* b4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + col0);
#pragma unroll
      for (int q = 0; q < NC / 4; ++q) {
        const float4 t = __ldg(b4 + q);
        v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
      }
    } else {
      const uint4* b8 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.bias) + col0);
#pragma unroll
      for (int q = 0; q < NC / 8; ++q) {
        const uint4 t = __ldg(b8 + q);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[8 * q + 2 * e] += __uint_as_float(w[e] << 16);
          v[8 * q + 2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
        }
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int col = col0 + i;
    if (col < p.N)
      v[i] += p.bias_dtype == L3D_F32
                  ? __ldg(static_cast<const float*>(p.bias) + col)
                  : __uint_as_float(uint32_t(__ldg(static_cast<const unsigned short*>(p.bias) + col)) << 16);
  }
}

// Gather the 128 x 64 A tile of (m0, kb) into the K-major SW128 layout (row r
// at r * 128 bytes, its 16-byte chunk j at chunk j ^ (r % 8)).  256 threads,
// 4 chunks each: thread t takes chunk t % 8 of rows t / 8 + 32 i; src[] holds
// the rows' neighbours for the current kernel offset and is reloaded only
// when the offset changes.
// PAIRS: m0 is the tile's first row within its segment, `rows` the
// segment's pair count and `psrc` its pair sources.
template <bool PAIRS>
__device__ __forceinline__ void gather_tile(const Params& p, uint8_t* tile, int m0, int kb, int t,
                                            int rows, const int32_t* psrc, int& cur_off,
                                            int32_t (&src)[4]) {
  const int kk = kb * BK;
  const int off = PAIRS ? 0 : kk / p.cin_pad, c0 = kk - off * p.cin_pad;
  if (off != cur_off) {
    cur_off = off;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = m0 + (t >> 3) + 32 * i;
      if constexpr (PAIRS) src[i] = row < rows ? __ldg(psrc + row) : -1;
      else src[i] = row < rows ? __ldg(p.nbr + int64_t(row) * 27 + off) : -1;
    }
  }
  const int j = t & 7;
  const int c = c0 + 8 * j;
  // 16-byte asynchronous copies straight into the swizzled tile; a missing
  // neighbour (or a channel past cin) copies 0 source bytes and zero-fills.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (t >> 3) + 32 * i;
    const bool ok = src[i] >= 0 && c < p.cin;
    const __nv_bfloat16* g = ok ? p.feats + int64_t(src[i]) * p.feats_ld + c : p.feats;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     smem_u32(tile + r * 128 + ((j ^ (r & 7)) << 4))),
                 "l"(g), "r"(ok ? 16u : 0u)
                 : "memory");
  }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                 const __grid_constant__ CUtensorMap map_y, const __grid_constant__ CUtensorMap map_r,
                 const Params p) {
  constexpr bool RAW_TMA = MODE == MODE_RAW_TMA;
  constexpr bool FUSED = ModeCfg<MODE>::FUSED;
  constexpr bool GATHER = ModeCfg<MODE>::GATHER;
  constexpr bool PAIRS = ModeCfg<MODE>::PAIRS;
  constexpr bool WORKERS = ModeCfg<MODE>::WORKERS;
  constexpr int STAGES = ModeCfg<MODE>::NST;
  constexpr int RAWB = ModeCfg<MODE>::RAW;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sa = smem;                              // [STAGES][A_BYTES]
  uint8_t* sb = smem + STAGES * A_BYTES;           // [STAGES][B_BYTES]
  uint8_t* sr = sb + STAGES * B_BYTES;             // [STAGES][RAWB] (fused modes)
  uint8_t* se = sr + STAGES * RAWB;                // [4 warps][8 KB] epilogue staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(se + ModeCfg<MODE>::EPI);
  uint64_t* lfull = bars;                          // [STAGES] TMA -> dequant/MMA
  uint64_t* bfull = bars + STAGES;                 // [STAGES] dequant -> MMA
  uint64_t* empty = bars + 2 * STAGES;             // [STAGES] MMA -> producer
  uint64_t* tfull = bars + 3 * STAGES;             // [2] MMA -> epilogue
  uint64_t* tempty = bars + 3 * STAGES + 2;        // [2] epilogue -> MMA
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 5);
  uint64_t* rbars = bars + 3 * STAGES + 7;         // [EPI_WARPS][2] residual TMA -> epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // MODE_PAIRS: segment boundaries (in tiles) and pair counts per offset.
  __shared__ int s_seg[28], s_cnt[27];
  if constexpr (PAIRS) {
    if (threadIdx.x < 28) s_seg[threadIdx.x] = p.seg_tile[threadIdx.x];
    if (threadIdx.x < 27) s_cnt[threadIdx.x] = p.seg_count[threadIdx.x];
  }
  auto seg_of = [&](int mt) {  // offset whose segment holds row tile mt
    int k = 0;
    while (k < 26 && mt >= s_seg[k + 1]) ++k;
    return k;
  };
  const int rows_m = p.M;
  const int num_m = (rows_m + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&lfull[s], 1);
      mbar_init(&bfull[s], N_DQ_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], ModeCfg<MODE>::EPI_WARPS);
    }
    for (int w = 0; w < 2 * ModeCfg<MODE>::EPI_WARPS; ++w) mbar_init(&rbars[w], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, ST_TIMEOUT_EMPTY)) break;
          mbar_expect_tx(&lfull[stage], MODE == MODE_RAW_TMA ? A_BYTES + RAW_BYTES
                                        : ModeCfg<MODE>::BF16W ? A_BYTES + B_BYTES
                                        : GATHER             ? B_BYTES  // gather / pairs
                                                             : A_BYTES);
          if constexpr (GATHER) {
            // Weights [27, Cout, Cin]: box of 64 channels x 256 outputs of one offset.
            const int kk = kb * BK, off = PAIRS ? 0 : kk / p.cin_pad;
            tma_load_3d(sb + stage * B_BYTES, &map_w, &lfull[stage], kk - off * p.cin_pad, n0,
                        PAIRS ? seg_of(m0 / BM) : off);
          } else {
            tma_load_2d(sa + stage * A_BYTES, &map_x, &lfull[stage], kb * BK, m0);
          }
          if constexpr (RAW_TMA) {
            // 16-byte aligned window (in 2-byte elements) holding this K step.
            const int c0 = ((kb * p.bpt) >> 4) << 3;
            tma_load_2d(sr + stage * RAWB, &map_w, &lfull[stage], c0, n0);
          }
          if constexpr (ModeCfg<MODE>::BF16W) {
            tma_load_2d(sb + stage * B_BYTES, &map_w, &lfull[stage], kb * BK, n0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status, ST_TIMEOUT_TMEM)) break;
        tc_fence_after();
        const uint32_t dtm = tmem_base + uint32_t(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&lfull[stage], phase, abort_flag, p.status, ST_TIMEOUT_RAW) ||
              (WORKERS && !mbar_wait(&bfull[stage], phase, abort_flag, p.status, ST_TIMEOUT_FULL))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(sa + stage * A_BYTES);
          const uint64_t db = smem_desc_sw128(sb + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 B per K step inside the 128 B swizzle atom (encoded >> 4).
            umma_bf16(dtm, da + uint64_t(2 * k), db + uint64_t(2 * k), (kb | k) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
    }
  } else if (warp < 2 + ModeCfg<MODE>::EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    // Columns [c_lo, c_hi) of each tile: all of them with four epilogue
    // warps; with eight, warps 2-5 take the first half and 6-9 the second.
    constexpr int EPI_SPAN = ModeCfg<MODE>::EPI_WARPS == 8 ? BN / 2 : BN;
    const int c_lo = ((warp - 2) >> 2) * EPI_SPAN, c_hi = c_lo + EPI_SPAN;
    const int ci_end = c_hi / EPI_COLS;  // chunk index past this warp's columns
    int local = 0;
    // TMA-store epilogue staging, 8 KB per epilogue warp.  Without a residual,
    // bf16 chunks (32 x 64 = 4 KB) alternate between its two halves (a store
    // can still be reading one while the next chunk is written) and f32
    // chunks use all of it.  With a residual, bf16: the first half receives
    // the residual chunks by TMA and the second half stages the output, so
    // the next residual load starts as soon as the current one is consumed;
    // f32: the residual chunk arrives in the staging and is updated in place.
    const bool f32o = p.y_dtype == L3D_F32;
    uint8_t* stg = se + (warp - 2) * EPI_WARP_BYTES;
    uint64_t* rbar = &rbars[(warp - 2) * 2];
    uint32_t rph = 0;  // parity of this warp's residual barrier
    int last_b = -1;   // staging half of the most recent store (bf16, no residual)
    // Residual chunk ci (64 columns) of the tile at (m0, n0) by TMA into stg.
    auto issue_res = [&](int m0, int n0, int ci) {
      const int col0 = n0 + ci * EPI_COLS;
      if (col0 >= p.N) return;
      // The warp's generic reads of the staging come before the async write.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const bool two = f32o && col0 + 32 < p.N;
      mbar_expect_tx(rbar, two ? 8192u : 4096u);
      tma_load_2d(stg, &map_r, rbar, col0, m0 + quarter * 32);
      if (two) tma_load_2d(stg + 4096, &map_r, rbar, col0 + 32, m0 + quarter * 32);
    };
    for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, ++local) {
      const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if constexpr (!FUSED) {
        // The tile's first residual chunk loads while the MMA still works.
        if (p.tma_store && p.res && p.res_tma && lane == 0) {
          if (f32o) bulk_wait_read0();  // in-place staging: the last store has read it
          issue_res(m0, n0, c_lo / EPI_COLS);
        }
      }
      if (!mbar_wait_idle(&tfull[acc], acc_phase, abort_flag, p.status, ST_TIMEOUT_TMEM)) break;
      tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
      if constexpr (!FUSED) if (p.tma_store) {
        // 32 rows x 64 columns per step: TMEM -> registers (+ bias, act,
        // residual) -> staging (128B-swizzled boxes of 128 bytes per row) ->
        // TMA stores of whole 128-byte lines; rows / columns past the matrix
        // are clipped by the tensor maps.
        const bool f32 = f32o;
        const bool tres = p.res && p.res_tma;
        bool eok = true;
#pragma unroll 1
        for (int c = c_lo; c < c_hi; c += EPI_COLS) {
          const int col0 = n0 + c;
          if (col0 >= p.N) break;  // warp-uniform; later chunks are past N too
          const int ci = c / EPI_COLS;
          // Output staging of this chunk.
          const int b = tres ? 1 : (f32 ? 0 : (ci & 1));
          uint8_t* obuf = f32 ? stg : stg + b * 4096;
          float v[EPI_COLS];
          {
            float a[32], b2[32];
            tmem_ld32(taddr + uint32_t(c), a);
            tmem_ld32(taddr + uint32_t(c + 32), b2);
#pragma unroll
            for (int i = 0; i < 32; ++i) { v[i] = a[i]; v[32 + i] = b2[i]; }
          }
          if (p.bias) add_bias<EPI_COLS>(p, col0, v);
          if (tres) {
            if (p.act) {
              // In two halves of 32 columns (fewer live temporaries).
              epi_act<32>(p.act, !f32, *reinterpret_cast<float(*)[32]>(&v[0]));
              epi_act<32>(p.act, !f32, *reinterpret_cast<float(*)[32]>(&v[32]));
            }
          } else if (p.act || p.res) {
            epi_post<32>(p, row, col0, *reinterpret_cast<float(*)[32]>(&v[0]));
            epi_post<32>(p, row, col0 + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
          }
          // Row `lane` of a box is 128 bytes = 8 chunks of 16 B; chunk j lives
          // at chunk j ^ (lane % 8) (the SWIZZLE_128B pattern of the maps).
          if (tres) {
            if (!mbar_wait(rbar, rph, abort_flag, p.status, ST_TIMEOUT_RAW)) {
              eok = false;
              break;
            }
            rph ^= 1u;
            // y = r + g * v, with r read from the staged residual chunk.
            const uint8_t* rrow = stg + lane * 128;
            auto gate_at = [&](int i) {
              if (!p.gate) return 1.f;
              const int col = col0 + i < p.N ? col0 + i : p.N - 1;
              return p.gate_dtype == L3D_F32
                         ? __ldg(static_cast<const float*>(p.gate) + col)
                         : __bfloat162float(static_cast<const __nv_bfloat16*>(p.gate)[col]);
            };
            if (f32) {
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const int bx = q >> 3, j = q & 7;
                const float4 r = *reinterpret_cast<const float4*>(rrow + bx * 4096 + ((j ^ (lane & 7)) << 4));
                v[4 * q] = fmaf(gate_at(4 * q), v[4 * q], r.x);
                v[4 * q + 1] = fmaf(gate_at(4 * q + 1), v[4 * q + 1], r.y);
                v[4 * q + 2] = fmaf(gate_at(4 * q + 2), v[4 * q + 2], r.z);
                v[4 * q + 3] = fmaf(gate_at(4 * q + 3), v[4 * q + 3], r.w);
              }
            } else {
              const bool gvec = p.gate && p.gate_dtype == L3D_F32 && col0 + EPI_COLS <= p.N &&
                                (reinterpret_cast<uintptr_t>(p.gate) & 15) == 0;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float r[8], g[8];
                unpack(*reinterpret_cast<const uint4*>(rrow + ((j ^ (lane & 7)) << 4)), r,
                       __nv_bfloat16());
                if (gvec) {
                  const float4* g4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.gate) + col0 + 8 * j);
                  const float4 ga = __ldg(g4), gb = __ldg(g4 + 1);
                  g[0] = ga.x; g[1] = ga.y; g[2] = ga.z; g[3] = ga.w;
                  g[4] = gb.x; g[5] = gb.y; g[6] = gb.z; g[7] = gb.w;
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e) g[e] = gate_at(8 * j + e);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) v[8 * j + e] = fmaf(g[e], v[8 * j + e], r[e]);
              }
              // Every lane has read the residual half: load the next chunk.
              __syncwarp();
              if (lane == 0 && ci + 1 < ci_end) issue_res(m0, n0, ci + 1);
            }
          }
          if (f32 && !tres) {
            // f32 without a residual: each 32-column half is its own store
            // from its own 4 KB staging half, so one half is written while
            // the other's store is still reading.
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (col0 + 32 * h >= p.N) break;  // warp-uniform
              uint8_t* hbuf = stg + h * 4096;
              if (lane == 0) {
                if (last_b != h) bulk_wait_read1();
                else bulk_wait_read0();
              }
              __syncwarp();
              uint8_t* rowp = hbuf + lane * 128;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int q = 8 * h + j;
                *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              }
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&map_y, hbuf, col0 + 32 * h, m0 + quarter * 32);
                bulk_commit();
              }
              last_b = h;
            }
            continue;
          }
          if (lane == 0) {
            // The store that last read this staging has finished reading it
            // (bf16 without residual: the newest store may still be reading
            // the other half).
            if (!tres && !f32 && last_b != b) bulk_wait_read1();
            else if (!(tres && f32)) bulk_wait_read0();
          }
          __syncwarp();
          uint8_t* rowp = obuf + lane * 128;
          if (f32) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {  // two boxes of 32 columns
              const int bx = q >> 3, j = q & 7;
              *reinterpret_cast<float4*>(rowp + bx * 4096 + ((j ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = v[8 * j + e];
              *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) = pack(f, __nv_bfloat16());
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_y, obuf, col0, m0 + quarter * 32);
            if (f32 && col0 + 32 < p.N) tma_store_2d(&map_y, obuf + 4096, col0 + 32, m0 + quarter * 32);
            bulk_commit();
            if (tres && f32 && ci + 1 < ci_end) {
              bulk_wait_read0();  // in place: this store has read the staging
              issue_res(m0, n0, ci + 1);
            }
          }
          last_b = b;
        }
        if (!eok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c = c_lo; c < c_hi; c += 32) {
        float v[32];
        tmem_ld32(taddr + uint32_t(c), v);
        const int col0 = n0 + c;
        if (row < rows_m && col0 < p.N) {
          if (p.bias) add_bias<32>(p, col0, v);
          if (p.act || p.res) epi_post<32>(p, row, col0, v);
          if (p.y_dtype == L3D_BF16) {
            __nv_bfloat16* yr = static_cast<__nv_bfloat16*>(p.y) + int64_t(row) * p.y_ld + col0;
            if (col0 + 32 <= p.N && p.y_vec) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[q * 8 + e];
                *reinterpret_cast<uint4*>(yr + q * 8) = pack(f, __nv_bfloat16());
              }
            } else {
              for (int i = 0; i < 32 && col0 + i < p.N; ++i) yr[i] = __float2bfloat16_rn(v[i]);
            }
          } else {
            float* yr = static_cast<float*>(p.y) + int64_t(row) * p.y_ld + col0;
            if (col0 + 32 <= p.N && p.y_vec) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                *reinterpret_cast<float4*>(yr + q * 4) =
                    make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
            } else {
              for (int i = 0; i < 32 && col0 + i < p.N; ++i) yr[i] = v[i];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (p.tma_store && lane == 0) bulk_wait0();  // stores complete before teardown
  } else if constexpr (WORKERS) {
    // ------------------------------------- dequantisers / neighbour gatherers
    const int t = threadIdx.x - 6 * 32;  // 0 .. 255
    int stage = 0;
    uint32_t phase = 0;
    // Gather modes keep up to kGatherDepth stages of cp.async copies in
    // flight; a stage is signalled to the MMA once its copies have landed
    // (cp.async.wait_group) and a proxy fence has made them visible to the
    // tensor core.  The oldest stage is signalled as soon as kGatherDepth are
    // pending, before the gatherers wait for the next stage to be released,
    // so the MMA can always release the stage they wait on.
    constexpr int kGatherDepth = 3;
    int pend = 0, arr_stage = 0;
    auto retire_oldest = [&](bool all) {
      if (all) asm volatile("cp.async.wait_group 0;" ::: "memory");
      else asm volatile("cp.async.wait_group %0;" ::"n"(kGatherDepth - 1) : "memory");
      do {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[arr_stage]);
        if (++arr_stage == STAGES) arr_stage = 0;
        --pend;
      } while (all && pend > 0);
    };
    for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
      const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
      int cur_off = -1;
      int32_t src[4];
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        // Gatherers write only the A tile: they start once the MMA has
        // released the stage, in parallel with the weight TMA of the same
        // stage (the MMA waits for both).  Dequantisers read the stage's raw
        // TMA load, so they wait for it to land (which also means the MMA has
        // released the stage's buffers).
        const bool ready =
            GATHER ? mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, ST_TIMEOUT_EMPTY)
                   : mbar_wait(&lfull[stage], phase, abort_flag, p.status, ST_TIMEOUT_RAW);
        if (!ready) {
          ok = false;
          break;
        }
        if constexpr (GATHER) {
          if constexpr (PAIRS) {
            const int k = seg_of(m0 / BM);
            gather_tile<true>(p, sa + stage * A_BYTES, m0 - s_seg[k] * BM, kb, t, s_cnt[k],
                              p.psrc + int64_t(k) * p.pstride, cur_off, src);
          } else {
            gather_tile<false>(p, sa + stage * A_BYTES, m0, kb, t, rows_m, nullptr, cur_off, src);
          }
          asm volatile("cp.async.commit_group;" ::: "memory");
          if (++pend == kGatherDepth) retire_oldest(false);
        } else {
          (void)m0;
          dequant_tile<RAW_TMA>(p, sr + stage * RAWB, sb + stage * B_BYTES, n0, kb, t);
          // Generic-proxy smem writes must be visible to the tensor core.
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&bfull[stage]);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
    // Copies still in flight land before teardown (and their stages are
    // signalled, for an MMA that may still be waiting on them).
    if constexpr (GATHER) {
      if (pend > 0) retire_oldest(true);
    }
  }

  // Teardown: every role has left its loop (normally or on abort).
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 32) {
    // Drain before releasing TMEM and shared memory: wait (bounded) for every
    // MMA this thread issued, then for every TMA load still in flight.
    uint64_t* drain = bars + 3 * STAGES + 6;
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    umma_commit(drain);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < WAIT_LIMIT_NS) {
    }
    // TMA loads land within microseconds; give any still in flight 1 ms.
    const uint64_t t1 = globaltimer();
    while (globaltimer() - t1 < 1000000ull) {
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

// ------------------------------------------------------------------- host
// x: bf16 [rows, cols] with row stride ld elements; box rows x 64, 128B swizzle.
static bool make_map_x(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                       uint64_t ld, uint32_t box_rows = BM) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {uint32_t(BK), box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output y [rows, cols] (bf16 or f32, row stride ld elements); box 32 rows x
// EPI_COLS columns, unswizzled, for the epilogue's TMA stores.
static bool make_map_y(CUtensorMap* m, void* base, int dtype, uint64_t rows, uint64_t cols,
                       uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  const uint64_t es = dtype == L3D_F32 ? 4 : 2;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * es};
  const cuuint32_t box[2] = {uint32_t(128 / es), 32u};  // 128-byte rows
  const cuuint32_t el[2] = {1, 1};
  return fn(m, dtype == L3D_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
            2, base, dims, strides, box, el, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw blocks viewed as uint16 [n, row_bytes / 2]; box 256 rows x 48 elements (96 B).
static bool make_map_w(CUtensorMap* m, const void* base, uint64_t n, uint64_t row_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {row_bytes / 2, n};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {uint32_t(RAW_ROW / 2), uint32_t(BN)};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Sparse-conv weights [27, cout, cin] bf16 (contiguous): box 64 channels x 256
// outputs x 1 offset, 128B swizzle; channels past cin / outputs past cout read
// as zero.
static bool make_map_w27(CUtensorMap* m, const void* base, uint64_t cout, uint64_t cin) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {cin, cout, 27};
  const cuuint64_t strides[2] = {cin * 2, cout * cin * 2};
  const cuuint32_t box[3] = {uint32_t(BK), uint32_t(BN), 1u};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gemm

// Convert f32 activations to bf16 (rows of ld elements -> contiguous [M, K]).
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, int64_t ld, int64_t M, int64_t K,
                                   __nv_bfloat16* __restrict__ out) {
  const int64_t total = M * K;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / K, c = i - r * K;
    out[i] = __float2bfloat16_rn(x[r * ld + c]);
  }
}

}  // namespace l3d

using namespace l3d;

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Above this many rows the weights are decoded once per call into the
// workspace instead of once per 128-row tile.
constexpr int64_t kDecodeOnceRows = 512;

// Workspace: [0, 256) status word; a bf16 copy of the activations (used when
// x is F32 or its rows are not 16-byte aligned); for m > kDecodeOnceRows, and
// always for the K-quants (256-weight super-blocks), the decoded bf16 weights
// [n, k].
static bool decode_once(int fmt, int64_t m) { return m > kDecodeOnceRows || is_kquant(fmt); }

extern "C" size_t l3d_linear_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || k < 0 || n < 0) return 0;
  return 256 + align256(size_t(m) * size_t(k) * 2);  // status word + activation copy
}

extern "C" size_t l3d_dequant_linear_workspace_size(int fmt, int64_t m, int64_t n, int64_t k) {
  if (m < 0 || k < 0 || n < 0) return 0;
  size_t bytes = 256 + align256(size_t(m) * size_t(k) * 2);
  if (decode_once(fmt, m)) bytes += align256(size_t(n) * size_t(k) * 2);
  return bytes;
}

// wdense: a bf16 [n, k] weight used as is (l3d_linear_ex; wq and fmt unused),
// or NULL for GGML blocks at wq in format fmt.
static int run_dequant_linear(const l3d_tensor* x, const void* wq, int fmt, int64_t n, int64_t k,
                              const l3d_tensor* bias, int act, const l3d_tensor* residual,
                              const l3d_tensor* gate, const l3d_tensor* y, void* workspace,
                              size_t workspace_bytes, l3d_stream stream, const char* op,
                              const l3d_tensor* wdense = nullptr) {
  using namespace l3d::gemm;
  int64_t w_ld = 0;
  if (wdense) {
    if (no_data(wdense)) return fail(L3D_E_NULL, "%s: weight has no data", op);
    if (wdense->dtype != L3D_BF16) return fail(L3D_E_DTYPE, "%s: weight must be BF16", op);
    if (wdense->ndim != 2) return fail(L3D_E_SHAPE, "%s: weight must be [n, k]", op);
    n = wdense->dims[0];
    k = wdense->dims[1];
    w_ld = n > 1 ? wdense->strides[0] : k;
    if (k > 1 && wdense->strides[1] != 1) return fail(L3D_E_ALIGN, "%s: weight rows must be contiguous", op);
    wq = elem_ptr(wdense);
    if (k % 8 || (w_ld * 2) % 16 || reinterpret_cast<uintptr_t>(wq) % 16)
      return fail(L3D_E_ALIGN, "%s: k must be a multiple of 8 and weight rows 16-byte aligned", op);
  }
  if (!x || !y || !wq || no_data(x) || no_data(y))
    return fail(L3D_E_NULL, "%s: x, wq and y are required", op);
  if (!wdense && !qfmt_known(fmt)) return fail(L3D_E_UNSUPPORTED, "%s: unknown format", op);
  if (x->dtype != L3D_BF16 && x->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: x must be BF16 or F32", op);
  if (y->dtype != L3D_BF16 && y->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: y must be BF16 or F32", op);
  if (!wdense && (k <= 0 || k % block_elems(fmt) || n <= 0))
    return fail(L3D_E_SHAPE, "%s: k must be a positive multiple of %d", op, block_elems(fmt));
  if (wdense && (k <= 0 || n <= 0)) return fail(L3D_E_SHAPE, "%s: empty weight", op);
  if (x->ndim < 1 || x->dims[x->ndim - 1] != k) return fail(L3D_E_SHAPE, "%s: x last dim != k", op);
  if (y->ndim != x->ndim || y->dims[y->ndim - 1] != n) return fail(L3D_E_SHAPE, "%s: y last dim != n", op);
  int64_t M = 1;
  for (int i = 0; i < x->ndim - 1; ++i) {
    if (x->dims[i] != y->dims[i]) return fail(L3D_E_SHAPE, "%s: x/y leading dims differ", op);
    M *= x->dims[i];
  }
  if (M > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return fail(L3D_E_UNSUPPORTED, "%s: dimensions exceed 2^31", op);
  RowMap xm, ym;
  if (!make_rowmap(x, x->ndim - 1, &xm) || !make_rowmap(y, y->ndim - 1, &ym) || xm.nd != 1 ||
      ym.nd != 1)
    return fail(L3D_E_ALIGN, "%s: x and y must be row-major matrices (one row stride)", op);
  if ((k > 1 && x->strides[x->ndim - 1] != 1) || (n > 1 && y->strides[y->ndim - 1] != 1))
    return fail(L3D_E_ALIGN, "%s: last dims must be contiguous", op);
  const int64_t x_ld = M > 1 ? xm.strides[0] : k;
  const int64_t y_ld = M > 1 ? ym.strides[0] : n;
  if (bias) {
    if (no_data(bias)) return fail(L3D_E_NULL, "%s: bias has no data", op);
    if (bias->dtype != L3D_F32 && bias->dtype != L3D_BF16)
      return fail(L3D_E_DTYPE, "%s: bias must be F32 or BF16", op);
    if (numel(bias) != n || (bias->ndim >= 1 && n > 1 && bias->strides[bias->ndim - 1] != 1))
      return fail(L3D_E_SHAPE, "%s: bias must be contiguous [n]", op);
  }
  if (reinterpret_cast<uintptr_t>(wq) % 2) return fail(L3D_E_ALIGN, "%s: wq must be 2-byte aligned", op);
  if (act < ACT_NONE || act > ACT_GELU_TANH) return fail(L3D_E_UNSUPPORTED, "%s: unknown activation", op);
  const void* res_ptr = nullptr;
  int64_t res_ld = 0;
  int res_vec = 0;
  if (residual) {
    if (no_data(residual)) return fail(L3D_E_NULL, "%s: residual has no data", op);
    if (residual->dtype != y->dtype) return fail(L3D_E_DTYPE, "%s: residual must have y's dtype", op);
    if (residual->ndim != y->ndim) return fail(L3D_E_SHAPE, "%s: residual must have y's shape", op);
    for (int i = 0; i < y->ndim; ++i)
      if (residual->dims[i] != y->dims[i]) return fail(L3D_E_SHAPE, "%s: residual must have y's shape", op);
    RowMap rm;
    if (!make_rowmap(residual, residual->ndim - 1, &rm) || rm.nd != 1 ||
        (n > 1 && residual->strides[residual->ndim - 1] != 1))
      return fail(L3D_E_ALIGN, "%s: residual must be a row-major matrix", op);
    res_ptr = elem_ptr(residual);
    res_ld = M > 1 ? rm.strides[0] : n;
    const int res_es = residual->dtype == L3D_F32 ? 4 : 2;
    res_vec = (reinterpret_cast<uintptr_t>(res_ptr) % 16 == 0) && ((res_ld * res_es) % 16 == 0);
  }
  if (gate) {
    if (!residual) return fail(L3D_E_SHAPE, "%s: gate needs a residual", op);
    if (no_data(gate)) return fail(L3D_E_NULL, "%s: gate has no data", op);
    if (gate->dtype != L3D_F32 && gate->dtype != L3D_BF16)
      return fail(L3D_E_DTYPE, "%s: gate must be F32 or BF16", op);
    if (numel(gate) != n || (gate->ndim >= 1 && n > 1 && gate->strides[gate->ndim - 1] != 1))
      return fail(L3D_E_SHAPE, "%s: gate must be contiguous [n]", op);
  }
  const size_t need = wdense ? l3d_linear_workspace_size(M, n, k)
                             : l3d_dequant_linear_workspace_size(fmt, M, n, k);
  if (!workspace || workspace_bytes < need)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  if (M == 0) return L3D_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(status, 0, 256, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: status clear failed", op);

  // Activations as a bf16 [M, K] matrix with a 16-byte-aligned row stride.
  const void* xa = elem_ptr(x);
  int64_t lda = x_ld;
  if (x->dtype == L3D_F32 || (lda * 2) % 16 || reinterpret_cast<uintptr_t>(xa) % 16) {
    __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(ws + 256);
    if (x->dtype == L3D_F32) {
      int64_t blocks = (M * k + 255) / 256;
      if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
      f32_to_bf16_kernel<<<int(blocks), 256, 0, s>>>(static_cast<const float*>(xa), x_ld, M, k, xb);
    } else {
      if (cudaMemcpy2DAsync(xb, size_t(k) * 2, xa, size_t(x_ld) * 2, size_t(k) * 2, size_t(M),
                            cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return fail(L3D_E_CUDA, "%s: activation copy failed", op);
    }
    xa = xb;
    lda = k;
  }
  Params p{};
  p.M = int(M); p.N = int(n); p.K = int(k);
  p.bias = bias ? elem_ptr(bias) : nullptr;
  p.bias_dtype = bias ? bias->dtype : L3D_F32;
  p.y = const_cast<char*>(elem_ptr(y));
  p.y_ld = y_ld;
  p.y_dtype = y->dtype;
  p.y_vec = (reinterpret_cast<uintptr_t>(p.y) % 16 == 0) &&
            ((y_ld * (y->dtype == L3D_F32 ? 4 : 2)) % 16 == 0);
  p.bias_vec = bias ? (reinterpret_cast<uintptr_t>(elem_ptr(bias)) % 16 == 0) : 0;
  p.status = status;
  p.wq = static_cast<const uint8_t*>(wq);
  p.fmt = fmt;
  p.row_bytes = wdense ? 0 : (k / block_elems(fmt)) * block_bytes(fmt);
  p.bpt = wdense ? 0 : 2 * block_bytes(fmt);
  p.act = act;
  p.res = res_ptr;
  p.res_ld = res_ld;
  p.res_vec = res_vec;
  p.gate = gate ? elem_ptr(gate) : nullptr;
  p.gate_dtype = gate ? gate->dtype : L3D_F32;
  CUtensorMap map_x, map_w, map_y;
  if (!make_map_x(&map_x, xa, uint64_t(M), uint64_t(k), uint64_t(lda)))
    return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed for x", op);
  // TMA-store epilogue when y's base and row stride are 16-byte aligned;
  // otherwise the epilogue stores directly.
  const int yes = y->dtype == L3D_F32 ? 4 : 2;
  p.tma_store = (reinterpret_cast<uintptr_t>(p.y) % 16 == 0) && ((y_ld * yes) % 16 == 0) &&
                        make_map_y(&map_y, p.y, y->dtype, uint64_t(M), uint64_t(n), uint64_t(y_ld))
                    ? 1
                    : 0;
  if (!p.tma_store) map_y = map_x;  // unused
  int mode;
  if (wdense) {
    // Dense bf16 weights: streamed by TMA as they are.
    if (!make_map_x(&map_w, wq, uint64_t(n), uint64_t(k), uint64_t(w_ld), BN))
      return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed for the weights", op);
    mode = act != ACT_NONE ? MODE_BF16_EPI8 : MODE_BF16;
  } else if (decode_once(fmt, M)) {
    // Decode the weights once into the workspace (bf16 [n, k]), then stream
    // them with TMA like the activations.
    char* wb = ws + 256 + align256(size_t(M) * size_t(k) * 2);
    int rc = launch_dequantize(wq, fmt, n, k, L3D_BF16, wb, s);
    if (rc) return rc;
    if (!make_map_x(&map_w, wb, uint64_t(n), uint64_t(k), uint64_t(k), BN))
      return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed for the decoded weights", op);
    mode = act != ACT_NONE ? MODE_BF16_EPI8 : MODE_BF16;
  } else {
    // The TMA window needs 16-byte aligned weight rows (k % 256 == 0).
    const bool raw_tma = (reinterpret_cast<uintptr_t>(wq) % 16 == 0) && (p.row_bytes % 16 == 0) &&
                         make_map_w(&map_w, wq, uint64_t(n), uint64_t(p.row_bytes));
    if (!raw_tma) map_w = map_x;  // unused
    mode = raw_tma ? MODE_RAW_TMA : MODE_RAW_LDG;
    p.tma_store = 0;  // no shared memory left for staging: direct stores
  }
  // Residual tiles by TMA (into the store staging) when the epilogue stores by
  // TMA and the residual rows are 16-byte aligned; otherwise direct loads.
  CUtensorMap map_r = map_y;  // unused unless res_tma
  p.res_tma = (p.tma_store && res_ptr && res_vec &&
               make_map_y(&map_r, const_cast<void*>(res_ptr), y->dtype, uint64_t(M), uint64_t(n),
                          uint64_t(res_ld)))
                  ? 1
                  : 0;
  cudaError_t attr_err =
      set_smem_limit(reinterpret_cast<const void*>(qgemm_kernel<MODE_RAW_TMA>),
                     ModeCfg<MODE_RAW_TMA>::SMEM);
  if (attr_err == cudaSuccess)
    attr_err = set_smem_limit(reinterpret_cast<const void*>(qgemm_kernel<MODE_RAW_LDG>),
                              ModeCfg<MODE_RAW_LDG>::SMEM);
  if (attr_err == cudaSuccess)
    attr_err = set_smem_limit(reinterpret_cast<const void*>(qgemm_kernel<MODE_BF16>),
                              ModeCfg<MODE_BF16>::SMEM);
  if (attr_err == cudaSuccess)
    attr_err = set_smem_limit(reinterpret_cast<const void*>(qgemm_kernel<MODE_BF16_EPI8>),
                              ModeCfg<MODE_BF16_EPI8>::SMEM);
  if (attr_err != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: cannot reserve the kernel's shared memory", op);
  const int tiles = int(((M + BM - 1) / BM) * ((n + BN - 1) / BN));
  const int grid = tiles < sm_count() ? tiles : sm_count();
  switch (mode) {
    case MODE_RAW_TMA:
      qgemm_kernel<MODE_RAW_TMA><<<grid, THREADS, ModeCfg<MODE_RAW_TMA>::SMEM, s>>>(map_x, map_w, map_y, map_r, p);
      break;
    case MODE_RAW_LDG:
      qgemm_kernel<MODE_RAW_LDG><<<grid, THREADS, ModeCfg<MODE_RAW_LDG>::SMEM, s>>>(map_x, map_w, map_y, map_r, p);
      break;
    case MODE_BF16_EPI8:
      qgemm_kernel<MODE_BF16_EPI8><<<grid, THREADS, ModeCfg<MODE_BF16_EPI8>::SMEM, s>>>(map_x, map_w, map_y, map_r, p);
      break;
    default:
      qgemm_kernel<MODE_BF16><<<grid, THREADS, ModeCfg<MODE_BF16>::SMEM, s>>>(map_x, map_w, map_y, map_r, p);
      break;
  }
  return check_launch(op);
}

extern "C" int l3d_dequant_linear(const l3d_tensor* x, const void* wq, int fmt, int64_t n,
                                  int64_t k, const l3d_tensor* bias, const l3d_tensor* y,
                                  void* workspace, size_t workspace_bytes, l3d_stream stream) {
  return run_dequant_linear(x, wq, fmt, n, k, bias, ACT_NONE, nullptr, nullptr, y, workspace,
                            workspace_bytes, stream, "l3d_dequant_linear");
}

extern "C" int l3d_dequant_linear_ex(const l3d_tensor* x, const void* wq, int fmt, int64_t n,
                                     int64_t k, const l3d_tensor* bias, int act,
                                     const l3d_tensor* residual, const l3d_tensor* gate,
                                     const l3d_tensor* y, void* workspace, size_t workspace_bytes,
                                     l3d_stream stream) {
  return run_dequant_linear(x, wq, fmt, n, k, bias, act, residual, gate, y, workspace,
                            workspace_bytes, stream, "l3d_dequant_linear_ex");
}

// ------------------------------------------------------------- sparse conv
// Workspace: [0, 256) status word, then room for a contiguous bf16 copy of
// feats (used when they are F32 or their rows are not 16-byte aligned).
extern "C" size_t l3d_sparse_conv3d_workspace_size(int64_t n, int64_t cin, int feats_dtype) {
  (void)feats_dtype;
  if (n < 0 || cin < 0) return 0;
  return 256 + align256(size_t(n) * size_t(cin) * 2);
}

extern "C" int l3d_sparse_conv3d(const l3d_tensor* feats, const l3d_tensor* nbr,
                                 const l3d_tensor* weight, const l3d_tensor* bias,
                                 const l3d_tensor* out, void* workspace, size_t workspace_bytes,
                                 l3d_stream stream) {
  const char* op = "l3d_sparse_conv3d";
  using namespace l3d::gemm;
  if (!feats || !nbr || !weight || !out) return fail(L3D_E_NULL, "%s: feats, nbr, weight, out required", op);
  if (feats->dtype != L3D_BF16 && feats->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: feats must be BF16 or F32", op);
  if (weight->dtype != L3D_BF16) return fail(L3D_E_DTYPE, "%s: weight must be BF16 [27, Cout, Cin]", op);
  if (nbr->dtype != L3D_I32) return fail(L3D_E_DTYPE, "%s: nbr must be I32", op);
  if (out->dtype != L3D_BF16 && out->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: out must be BF16 or F32", op);
  if (feats->ndim != 2 || weight->ndim != 3 || weight->dims[0] != 27 || nbr->ndim != 2 ||
      out->ndim != 2)
    return fail(L3D_E_SHAPE, "%s: feats [N, Cin], nbr [N, 27], weight [27, Cout, Cin], out [N, Cout]", op);
  const int64_t n = feats->dims[0], cin = feats->dims[1], cout = weight->dims[1];
  if (weight->dims[2] != cin || nbr->dims[0] != n || nbr->dims[1] != 27 || out->dims[0] != n ||
      out->dims[1] != cout)
    return fail(L3D_E_SHAPE, "%s: shapes do not agree", op);
  if (cin <= 0 || cin % 8 || cout <= 0)
    return fail(L3D_E_UNSUPPORTED, "%s: Cin must be a positive multiple of 8", op);
  if (n > INT32_MAX || cout > INT32_MAX || 27 * ((cin + BK - 1) / BK * BK) > INT32_MAX)
    return fail(L3D_E_UNSUPPORTED, "%s: dimensions exceed 2^31", op);
  if (bias) {
    if (no_data(bias)) return fail(L3D_E_NULL, "%s: bias has no data", op);
    if (bias->dtype != L3D_F32 && bias->dtype != L3D_BF16)
      return fail(L3D_E_DTYPE, "%s: bias must be F32 or BF16", op);
    if (numel(bias) != cout || (bias->ndim >= 1 && cout > 1 && bias->strides[bias->ndim - 1] != 1))
      return fail(L3D_E_SHAPE, "%s: bias must be contiguous [Cout]", op);
  }
  const size_t need = l3d_sparse_conv3d_workspace_size(n, cin, feats->dtype);
  if (!workspace || workspace_bytes < need)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  if (n == 0) return L3D_OK;
  if (no_data(feats) || no_data(nbr) || no_data(weight) || no_data(out))
    return fail(L3D_E_NULL, "%s: null data pointer", op);
  if ((cin > 1 && feats->strides[1] != 1) || (cout > 1 && out->strides[1] != 1) ||
      nbr->strides[1] != 1 || (n > 1 && nbr->strides[0] != 27))
    return fail(L3D_E_ALIGN, "%s: feats/out rows and nbr must be contiguous", op);
  if (weight->strides[2] != 1 || weight->strides[1] != cin || weight->strides[0] != cout * cin)
    return fail(L3D_E_ALIGN, "%s: weight must be contiguous [27, Cout, Cin]", op);
  const void* wp = elem_ptr(weight);
  if (reinterpret_cast<uintptr_t>(wp) % 16) return fail(L3D_E_ALIGN, "%s: weight must be 16-byte aligned", op);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(status, 0, 256, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: status clear failed", op);
  // feats as bf16 rows with a 16-byte aligned stride.
  const void* fa = elem_ptr(feats);
  int64_t fld = n > 1 ? feats->strides[0] : cin;
  if (feats->dtype == L3D_F32 || (fld * 2) % 16 || reinterpret_cast<uintptr_t>(fa) % 16) {
    __nv_bfloat16* fb = reinterpret_cast<__nv_bfloat16*>(ws + 256);
    if (feats->dtype == L3D_F32) {
      int64_t blocks = (n * cin + 255) / 256;
      if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
      f32_to_bf16_kernel<<<int(blocks), 256, 0, s>>>(static_cast<const float*>(fa), fld, n, cin, fb);
    } else if (cudaMemcpy2DAsync(fb, size_t(cin) * 2, fa, size_t(fld) * 2, size_t(cin) * 2, size_t(n),
                                 cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      return fail(L3D_E_CUDA, "%s: feats copy failed", op);
    }
    fa = fb;
    fld = cin;
  }
  Params p{};
  p.M = int(n);
  p.N = int(cout);
  p.cin = int(cin);
  p.cin_pad = int((cin + BK - 1) / BK * BK);
  p.K = 27 * p.cin_pad;
  p.bias = bias ? elem_ptr(bias) : nullptr;
  p.bias_dtype = bias ? bias->dtype : L3D_F32;
  p.y = const_cast<char*>(elem_ptr(out));
  p.y_ld = n > 1 ? out->strides[0] : cout;
  p.y_dtype = out->dtype;
  p.y_vec = (reinterpret_cast<uintptr_t>(p.y) % 16 == 0) &&
            ((p.y_ld * (out->dtype == L3D_F32 ? 4 : 2)) % 16 == 0);
  p.bias_vec = bias ? (reinterpret_cast<uintptr_t>(elem_ptr(bias)) % 16 == 0) : 0;
  p.status = status;
  p.nbr = static_cast<const int32_t*>(static_cast<const void*>(elem_ptr(nbr)));
  p.feats = static_cast<const __nv_bfloat16*>(fa);
  p.feats_ld = fld;
  CUtensorMap map_w, map_y;
  if (!make_map_w27(&map_w, wp, uint64_t(cout), uint64_t(cin)))
    return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed for the weights", op);
  const int yes = out->dtype == L3D_F32 ? 4 : 2;
  p.tma_store = (reinterpret_cast<uintptr_t>(p.y) % 16 == 0) && ((p.y_ld * yes) % 16 == 0) &&
                        make_map_y(&map_y, p.y, out->dtype, uint64_t(n), uint64_t(cout), uint64_t(p.y_ld))
                    ? 1
                    : 0;
  if (!p.tma_store) map_y = map_w;  // unused
  const cudaError_t attr_err = set_smem_limit(
      reinterpret_cast<const void*>(qgemm_kernel<MODE_GATHER>), ModeCfg<MODE_GATHER>::SMEM);
  if (attr_err != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: cannot reserve the kernel's shared memory", op);
  const int tiles = int(((n + BM - 1) / BM) * ((cout + BN - 1) / BN));
  const int grid = tiles < sm_count() ? tiles : sm_count();
  qgemm_kernel<MODE_GATHER><<<grid, THREADS, ModeCfg<MODE_GATHER>::SMEM, s>>>(map_w, map_w, map_y, map_w, p);
  return check_launch(op);
}

// ------------------------------------------------- sparse conv over pair lists
// pos[dest_k[j] * 27 + k] = j: where row i's product for offset k sits in
// offset k's pair list (-1 when i has no neighbour at k; cleared before).
__global__ void pair_pos_kernel(const int32_t* __restrict__ dest, int64_t dstride,
                                const int32_t* __restrict__ counts, int64_t n,
                                int32_t* __restrict__ pos) {
  const int k = blockIdx.y;
  const int64_t cnt = __ldg(counts + k) < n ? __ldg(counts + k) : n;
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < cnt;
       j += int64_t(gridDim.x) * blockDim.x)
    pos[int64_t(__ldg(dest + k * dstride + j)) * 27 + k] = int32_t(j);
}

// out[i, c] = ((0 + prod_0) + prod_1) + ... + prod_26 + bias[c]: each row's
// products added in ascending offset order (the reference's index_add
// order), then the bias; f32, rounded once to out's dtype.  One warp per row:
// lane k < 27 reads the row's position in offset k's segment once, and the
// lanes sum 4 columns each per 128-column step.
__global__ void pair_reduce_kernel(const float* __restrict__ prod, int64_t pld,
                                   const int32_t* __restrict__ pos, const int64_t* __restrict__ seg_row,
                                   int64_t n, int64_t cout, const void* bias, int bias_dtype,
                                   void* out, int64_t old_, int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t srow = lane < 27 ? __ldg(seg_row + lane) : 0;
  for (int64_t i = warp0; i < n; i += nwarps) {
    const int32_t j = lane < 27 ? __ldg(pos + i * 27 + lane) : -1;
    const int64_t prow = j >= 0 ? srow + j : -1;  // product row of offset `lane`
    const unsigned have = __ballot_sync(0xffffffffu, j >= 0);
    // Warp-uniform column loop (every lane takes part in the shuffles).
    for (int64_t cb = 0; cb < cout; cb += 128) {
      const int64_t c = cb + 4 * lane;
      const bool active = c < cout;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      const bool full = c + 4 <= cout;
      unsigned m = have;
      while (m) {  // offsets with a neighbour, ascending, up to 4 loads in flight
        int64_t r[4];
        int cnt = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          r[q] = -1;
          if (m) {
            const int k = __ffs(m) - 1;
            m &= m - 1;
            r[q] = __shfl_sync(0xffffffffu, prow, k);
            ++cnt;
          }
        }
        if (!active) continue;
        float4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (q < cnt) {
            const float* src = prod + r[q] * pld + c;
            if (full) {
              v[q] = __ldg(reinterpret_cast<const float4*>(src));
            } else {
              v[q].x = __ldg(src);
              if (c + 1 < cout) v[q].y = __ldg(src + 1);
              if (c + 2 < cout) v[q].z = __ldg(src + 2);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q < cnt) {
            acc.x += v[q].x; acc.y += v[q].y; acc.z += v[q].z; acc.w += v[q].w;
          }
        }
      }
      if (!active) continue;
      const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t col = c + e;
        if (col >= cout) break;
        float v = vals[e];
        if (bias)
          v += bias_dtype == L3D_F32 ? static_cast<const float*>(bias)[col]
                                     : __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[col]);
        if (out_dtype == L3D_F32) static_cast<float*>(out)[i * old_ + col] = v;
        else static_cast<__nv_bfloat16*>(out)[i * old_ + col] = __float2bfloat16_rn(v);
      }
    }
  }
}

namespace {
struct PairsLayout {
  int seg_tile[28];     // prefix of ceil(count_k / 128), in 128-row tiles
  int64_t rows;         // padded product rows
  int64_t ld;           // product row stride (floats, multiple of 4)
  size_t feats_off, prod_off, pos_off, seg_off, total;
};
PairsLayout pairs_layout(int64_t n, int64_t cin, int64_t cout, const int32_t* counts_host) {
  PairsLayout L{};
  int64_t t = 0;
  for (int k = 0; k < 27; ++k) {
    L.seg_tile[k] = int(t);
    const int64_t c = counts_host[k] < 0 ? 0 : (counts_host[k] > n ? n : counts_host[k]);
    t += (c + l3d::gemm::BM - 1) / l3d::gemm::BM;
  }
  L.seg_tile[27] = int(t);
  L.rows = t * l3d::gemm::BM;
  L.ld = (cout + 3) / 4 * 4;
  L.feats_off = 256;
  L.prod_off = L.feats_off + align256(size_t(n) * size_t(cin) * 2);
  L.pos_off = L.prod_off + align256(size_t(L.rows) * size_t(L.ld) * 4);
  L.seg_off = L.pos_off + align256(size_t(n) * 27 * 4);
  L.total = L.seg_off + 256;
  return L;
}
}  // namespace

// Workspace: status word, a bf16 copy of feats (F32 or unaligned rows), the
// f32 products of every pair (segments padded to 128 rows), the [N, 27]
// position table and the segment row offsets.
extern "C" size_t l3d_sparse_conv3d_pairs_workspace_size(int64_t n, int64_t cin, int64_t cout,
                                                         const int32_t* counts_host) {
  if (n < 0 || cin < 0 || cout < 0 || !counts_host) return 0;
  return pairs_layout(n, cin, cout, counts_host).total;
}

extern "C" int l3d_sparse_conv3d_pairs(const l3d_tensor* feats, const l3d_tensor* pair_src,
                                       const l3d_tensor* pair_dest, const l3d_tensor* counts,
                                       const int32_t* counts_host, const l3d_tensor* weight,
                                       const l3d_tensor* bias, const l3d_tensor* out,
                                       void* workspace, size_t workspace_bytes,
                                       l3d_stream stream) {
  const char* op = "l3d_sparse_conv3d_pairs";
  using namespace l3d::gemm;
  if (!feats || !pair_src || !pair_dest || !counts || !counts_host || !weight || !out)
    return fail(L3D_E_NULL, "%s: feats, pair lists, counts (device and host), weight and out are required", op);
  if (feats->dtype != L3D_BF16 && feats->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: feats must be BF16 or F32", op);
  if (weight->dtype != L3D_BF16) return fail(L3D_E_DTYPE, "%s: weight must be BF16 [27, Cout, Cin]", op);
  if (pair_src->dtype != L3D_I32 || pair_dest->dtype != L3D_I32 || counts->dtype != L3D_I32)
    return fail(L3D_E_DTYPE, "%s: pair lists and counts must be I32", op);
  if (out->dtype != L3D_BF16 && out->dtype != L3D_F32)
    return fail(L3D_E_DTYPE, "%s: out must be BF16 or F32", op);
  if (feats->ndim != 2 || weight->ndim != 3 || weight->dims[0] != 27 || out->ndim != 2)
    return fail(L3D_E_SHAPE, "%s: feats [N, Cin], weight [27, Cout, Cin], out [N, Cout]", op);
  const int64_t n = feats->dims[0], cin = feats->dims[1], cout = weight->dims[1];
  if (weight->dims[2] != cin || out->dims[0] != n || out->dims[1] != cout)
    return fail(L3D_E_SHAPE, "%s: shapes do not agree", op);
  for (const l3d_tensor* t : {pair_src, pair_dest})
    if (t->ndim != 2 || t->dims[0] != 27 || t->dims[1] != n)
      return fail(L3D_E_SHAPE, "%s: pair lists must be [27, N]", op);
  if (counts->ndim != 1 || counts->dims[0] != 27) return fail(L3D_E_SHAPE, "%s: counts must be [27]", op);
  for (int k = 0; k < 27; ++k)
    if (counts_host[k] < 0 || counts_host[k] > n)
      return fail(L3D_E_SHAPE, "%s: counts_host[%d] out of range", op, k);
  if (cin <= 0 || cin % 8 || cout <= 0)
    return fail(L3D_E_UNSUPPORTED, "%s: Cin must be a positive multiple of 8", op);
  if (n > INT32_MAX || cout > INT32_MAX) return fail(L3D_E_UNSUPPORTED, "%s: dimensions exceed 2^31", op);
  if (bias) {
    if (no_data(bias)) return fail(L3D_E_NULL, "%s: bias has no data", op);
    if (bias->dtype != L3D_F32 && bias->dtype != L3D_BF16)
      return fail(L3D_E_DTYPE, "%s: bias must be F32 or BF16", op);
    if (numel(bias) != cout || (bias->ndim >= 1 && cout > 1 && bias->strides[bias->ndim - 1] != 1))
      return fail(L3D_E_SHAPE, "%s: bias must be contiguous [Cout]", op);
  }
  const PairsLayout L = pairs_layout(n, cin, cout, counts_host);
  if (L.rows > INT32_MAX) return fail(L3D_E_UNSUPPORTED, "%s: too many pairs", op);
  if (!workspace || workspace_bytes < L.total)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, L.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  if (n == 0) return L3D_OK;
  if (no_data(feats) || no_data(pair_src) || no_data(pair_dest) || no_data(counts) ||
      no_data(weight) || no_data(out))
    return fail(L3D_E_NULL, "%s: null data pointer", op);
  if ((cin > 1 && feats->strides[1] != 1) || (cout > 1 && out->strides[1] != 1) ||
      (n > 1 && (pair_src->strides[1] != 1 || pair_dest->strides[1] != 1)) ||
      counts->strides[0] != 1)
    return fail(L3D_E_ALIGN, "%s: feats/out rows, pair lists and counts must be contiguous", op);
  if (weight->strides[2] != 1 || weight->strides[1] != cin || weight->strides[0] != cout * cin)
    return fail(L3D_E_ALIGN, "%s: weight must be contiguous [27, Cout, Cin]", op);
  const void* wp = elem_ptr(weight);
  if (reinterpret_cast<uintptr_t>(wp) % 16) return fail(L3D_E_ALIGN, "%s: weight must be 16-byte aligned", op);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(status, 0, 256, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: status clear failed", op);
  const void* fa = elem_ptr(feats);
  int64_t fld = n > 1 ? feats->strides[0] : cin;
  if (feats->dtype == L3D_F32 || (fld * 2) % 16 || reinterpret_cast<uintptr_t>(fa) % 16) {
    __nv_bfloat16* fb = reinterpret_cast<__nv_bfloat16*>(ws + L.feats_off);
    if (feats->dtype == L3D_F32) {
      int64_t blocks = (n * cin + 255) / 256;
      if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
      f32_to_bf16_kernel<<<int(blocks), 256, 0, s>>>(static_cast<const float*>(fa), fld, n, cin, fb);
    } else if (cudaMemcpy2DAsync(fb, size_t(cin) * 2, fa, size_t(fld) * 2, size_t(cin) * 2, size_t(n),
                                 cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      return fail(L3D_E_CUDA, "%s: feats copy failed", op);
    }
    fa = fb;
    fld = cin;
  }
  float* prod = reinterpret_cast<float*>(ws + L.prod_off);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + L.pos_off);
  int64_t* segrow = reinterpret_cast<int64_t*>(ws + L.seg_off);
  const int32_t* src0 = static_cast<const int32_t*>(static_cast<const void*>(elem_ptr(pair_src)));
  const int32_t* dst0 = static_cast<const int32_t*>(static_cast<const void*>(elem_ptr(pair_dest)));
  const int32_t* cnt = static_cast<const int32_t*>(static_cast<const void*>(elem_ptr(counts)));
  // Position table and segment row offsets.
  int64_t seg_rows_host[27];
  for (int k = 0; k < 27; ++k) seg_rows_host[k] = int64_t(L.seg_tile[k]) * BM;
  if (cudaMemsetAsync(pos, 0xff, size_t(n) * 27 * 4, s) != cudaSuccess ||
      cudaMemcpyAsync(segrow, seg_rows_host, sizeof(seg_rows_host), cudaMemcpyHostToDevice, s) !=
          cudaSuccess)
    return fail(L3D_E_CUDA, "%s: workspace set-up failed", op);
  {
    const int64_t bx = (n + 255) / 256 < 64 ? (n + 255) / 256 : 64;
    pair_pos_kernel<<<dim3(unsigned(bx), 27), 256, 0, s>>>(dst0, pair_dest->strides[0], cnt, n, pos);
  }
  // One tensor-core launch over every offset's pair segment.
  if (L.rows > 0) {
    Params p{};
    p.M = int(L.rows);
    p.N = int(cout);
    p.cin = int(cin);
    p.cin_pad = int((cin + BK - 1) / BK * BK);
    p.K = p.cin_pad;
    p.y = prod;
    p.y_ld = L.ld;
    p.y_dtype = L3D_F32;
    p.y_vec = 1;
    p.status = status;
    p.feats = static_cast<const __nv_bfloat16*>(fa);
    p.feats_ld = fld;
    p.psrc = src0;
    p.pstride = pair_src->strides[0];
    for (int k = 0; k < 28; ++k) p.seg_tile[k] = L.seg_tile[k];
    for (int k = 0; k < 27; ++k) p.seg_count[k] = counts_host[k];
    CUtensorMap map_w, map_y;
    if (!make_map_w27(&map_w, wp, uint64_t(cout), uint64_t(cin)))
      return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed for the weights", op);
    p.tma_store = make_map_y(&map_y, prod, L3D_F32, uint64_t(L.rows), uint64_t(cout), uint64_t(L.ld)) ? 1 : 0;
    if (!p.tma_store) map_y = map_w;  // unused
    const cudaError_t attr_err = set_smem_limit(
        reinterpret_cast<const void*>(qgemm_kernel<MODE_PAIRS>), ModeCfg<MODE_PAIRS>::SMEM);
    if (attr_err != cudaSuccess)
      return fail(L3D_E_CUDA, "%s: cannot reserve the kernel's shared memory", op);
    const int tiles = int((L.rows / BM) * ((cout + BN - 1) / BN));
    const int grid = tiles < sm_count() ? tiles : sm_count();
    qgemm_kernel<MODE_PAIRS><<<grid, THREADS, ModeCfg<MODE_PAIRS>::SMEM, s>>>(map_w, map_w, map_y,
                                                                              map_w, p);
  }
  {
    int64_t blocks = (n + 7) / 8;  // a warp per row, 8 warps per block
    if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
    pair_reduce_kernel<<<int(blocks), 256, 0, s>>>(prod, L.ld, pos, segrow, n, cout,
                                                   bias ? elem_ptr(bias) : nullptr,
                                                   bias ? bias->dtype : L3D_F32,
                                                   const_cast<char*>(elem_ptr(out)),
                                                   n > 1 ? out->strides[0] : cout, out->dtype);
  }
  return check_launch(op);
}

extern "C" int l3d_linear_ex(const l3d_tensor* x, const l3d_tensor* weight, const l3d_tensor* bias,
                             int act, const l3d_tensor* residual, const l3d_tensor* gate,
                             const l3d_tensor* y, void* workspace, size_t workspace_bytes,
                             l3d_stream stream) {
  if (!weight) return fail(L3D_E_NULL, "l3d_linear_ex: weight is required");
  return run_dequant_linear(x, nullptr, 0, 0, 0, bias, act, residual, gate, y, workspace,
                            workspace_bytes, stream, "l3d_linear_ex", weight);
}
