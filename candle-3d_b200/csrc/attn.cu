// Scaled dot-product attention (the attention core of the block stacks,
// exact_sdpa_heads / exact_query_chunked_sdpa, crate/runtime/
// attention_math.rs:199-259) on the 5th-generation tensor cores.
//
//   out[b, h, i, :] = softmax_j(q[b,h,i,:] . k[b,h,j,:] * scale) v[b,h,j,:]
//
// One CTA per (256 queries = two 128-row tiles, head, batch), one CTA per SM:
//   warp 0     TMA producer: both Q tiles once, then a ring of K and V tiles
//              (128 keys x D each, 128B-swizzled boxes of 64 columns), read
//              in place from the caller's (possibly strided) views;
//   MMA warps  S_t(j) = Q_t K(j)^T (M 128, N 128, K D, operands in shared
//              memory) and O_t += P_t(j) V(j) (M 128, N D, K 128, P_t read
//              from tensor memory, V as an MN-major operand: D contiguous).  The two query tiles share each K / V
//              load; while one tile's softmax runs, the tensor core works for
//              the other.
//              D = 128: one MMA warp; TMEM is full, so P_t lies over the first
//              half of S_t and per key tile the order is O_0 += P_0 V, S_0(j+1),
//              O_1 += P_1 V, S_1(j+1).  Each tcgen05.commit tracks every MMA
//              issued before it and one thread's MMAs run in issue order, so
//              "S_t(j+1) complete" also means that P_t(j) has been consumed
//              and O_t is stable: the softmax warps wait on one barrier per
//              key tile.
//              D = 64: one MMA warp per query tile and P_t in columns of its
//              own, so S_t(j+1) is issued as soon as the softmax warps have
//              copied S_t(j) to registers (it overlaps their exponentials),
//              and O_t += P_t(j) V^T once P_t(j) is written;
//   softmax    four warps per query tile, one query row per thread (its TMEM
//              lane): the row of S_t(j) is copied to registers, the running
//              O_t is rescaled in TMEM when the max grows past the threshold,
//              P = exp2(S * scale * log2 e - m) is stored to TMEM as packed
//              bf16 and the row sum accumulated (at D = 64 a quarter of the
//              exponentials on the FMA pipe); after the last tile O / l is
//              stored.
// TMEM (512 columns): S_0, S_1 (128 each), O_0, O_1 (D each), and for D = 64
// P_0, P_1 (64 each).
// Every mbarrier wait is bounded (%globaltimer, 2 s); on expiry the CTA
// records an error in the workspace status word and stops.
#include "common.cuh"
#include "tc.cuh"

namespace l3d {
namespace attn {

using namespace l3d::tc;

constexpr int BQ = 128;               // rows of one query tile
constexpr int NT = 2;                  // query tiles per CTA
constexpr int TMEM_COLS = 512;
constexpr int ST_TIMEOUT = 5;
constexpr int ST_MISALIGNED = 6;
// The running max moves only when a row's max grows by more than 2^8 (log2
// units): until then exp2(s - m) <= 256, and O and l share the stale max, so
// the result is unchanged while most O rescales are skipped.
constexpr float RESCALE_LOG2 = 8.f;

// exp2 on the FMA pipe, for part of the elements, so that the MUFU unit (16
// exp2 per clock per SM) is not the only one doing them: Cody-Waite style
// range reduction x = j + f with j = round(x) (the 1.5 * 2^23 shifter) and f
// in [-1/2, 1/2], 2^f by a degree-3 minimax polynomial (Remez fit made for
// this kernel, relative error 7.5e-5, far below the bf16 rounding of P), and
// 2^j added to the exponent field.  x is clamped to -126 so that the exponent
// stays in range; the inputs here are <= 2^8 (the rescale threshold).
constexpr float EX2_C0 = 0.99992806f, EX2_C1 = 0.69326097f, EX2_C2 = 0.24261113f,
                EX2_C3 = 0.05517167f;
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x = make_float2(fmaxf(x.x, -126.f), fmaxf(x.y, -126.f));
  const float2 t = add2(x, f2(12582912.f));          // low mantissa bits = round(x)
  const float2 r = add2(t, f2(-12582912.f));
  const float2 f = add2(x, make_float2(-r.x, -r.y));
  float2 q = fma2(f, f2(EX2_C3), f2(EX2_C2));
  q = fma2(q, f, f2(EX2_C1));
  q = fma2(q, f, f2(EX2_C0));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}
// Of every 8 pairs of P at D = 64, this many take ex2_poly2, the rest the MUFU.
#ifndef L3D_ATTN_POLY_PAIRS
#define L3D_ATTN_POLY_PAIRS 2
#endif
constexpr int POLY_PAIRS = L3D_ATTN_POLY_PAIRS;

template <int D>
struct Cfg {
  static constexpr int BKV = 128;
  static constexpr int DC = D / 64;                   // 64-wide K atoms of Q / K
  static constexpr int Q_BYTES = BQ * D * 2;          // one query tile
  static constexpr int K_BYTES = BKV * D * 2;
  static constexpr int V_BYTES = BKV * D * 2;         // V tile: BKV keys x D
  static constexpr int STAGES = D == 64 ? 4 : 2;
  // No alignment slack: with no static shared memory the dynamic window
  // starts 1024-byte aligned (checked at run time).
  static constexpr int SMEM = NT * Q_BYTES + STAGES * (K_BYTES + V_BYTES) + 256;
  // The 256 bytes after the tiles: 1 + 2 STAGES + 4 NT + NMMA mbarriers, the
  // abort flag and the TMEM address (checked below, once NMMA is known).
  static constexpr uint32_t IDESC_S = make_idesc(128, BKV);
  static constexpr uint32_t IDESC_O = make_idesc(128, D) | (1u << 16);  // B (V) MN-major
  // TMEM columns.  For D = 64, P_t has columns of its own (SEP_P), so that
  // S_t(j+1) can be computed while the softmax of tile j still runs; for
  // D = 128 TMEM is full and P_t goes over the first half of S_t.
  static constexpr uint32_t COL_S = 0, COL_O = 2 * BKV;
  static constexpr bool SEP_P = COL_O + 2 * D + 2 * (BKV / 2) <= TMEM_COLS;
  static constexpr uint32_t COL_P = SEP_P ? COL_O + 2 * D : COL_S;
  static constexpr uint32_t P_STRIDE = SEP_P ? BKV / 2 : BKV;  // between P_0 and P_1
  static_assert(COL_O + 2 * D <= TMEM_COLS, "TMEM budget");
  // MMA warps: with SEP_P one per query tile, so that the two tiles' issue
  // chains do not wait on each other; without it one warp issues both tiles
  // in a fixed interleave (P_0 V, S_0, P_1 V, S_1), which measured faster.
  static constexpr int NMMA = SEP_P ? NT : 1;
  static constexpr int THREADS = (1 + NMMA + 4 * NT) * 32;  // producer, MMA, softmax
  static_assert((1 + 2 * STAGES + 4 * NT + NMMA) * 8 + 8 <= 256, "barrier area");
  // Of every 8 pairs of P, this many take ex2_poly2 (D = 64 is bound by the
  // MUFU; at D = 128 the MUFU has room).
  static constexpr int POLY = D == 64 ? POLY_PAIRS : 0;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct Params {
  int64_t nq, nk;       // query / key lengths
  int q_hn, k_hn, v_hn; // the q / k / v maps list heads before rows (token-major memory)
  float scale_log2;     // softmax scale * log2(e), > 0
  void* out;            // [B, H, nq, D] bf16
  int64_t ob, oh, on;   // out strides (elements)
  int* status;
  uint64_t wait_ns;     // limit of every mbarrier wait
  int hold_kv;          // failure self-test: this key tile is never loaded (-1: none)
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// MN-major, 128B-swizzled operand tile (B = V: N = D contiguous in rows of 128
// B, one row per K index): 8-row K groups 1024 B apart (SBO), 64-wide N blocks
// `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(const void* tile, uint32_t lbo) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3fffull;
  d |= uint64_t((lbo >> 4) & 0x3fff) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (M 128 x K 16, bf16 pairs packed in 32-bit
// columns, rows = TMEM lanes) from tensor memory, B from a shared-memory
// descriptor.
template <uint32_t IDESC_>
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(IDESC_), "r"(accumulate));
}

// 64 consecutive f32 TMEM columns of this thread's lane -> registers; the
// wait is inside the same statement, so no use can move above it.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, "
      "%45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, "
      "%62, %63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
        "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
        "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]),
        "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]),
        "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive 32-bit TMEM columns of this thread's lane <- registers.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats -> packed bf16 pair (lo = a, the lower K index).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int D>
__global__ void __launch_bounds__(Cfg<D>::THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Params p) {
  using C = Cfg<D>;
  constexpr int BKV = C::BKV;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The swizzled tiles need 1024-byte alignment; report and stop otherwise.
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, ST_MISALIGNED);
    return;
  }
  uint8_t* sq = smem_raw;                              // [NT][DC][128 x 64]
  uint8_t* sk = sq + NT * C::Q_BYTES;                  // [STAGES][DC][BKV x 64]
  uint8_t* sv = sk + C::STAGES * C::K_BYTES;           // [STAGES][DC][BKV x 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + C::STAGES * C::V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                        // [STAGES]
  uint64_t* kv_empty = kv_full + C::STAGES;            // [STAGES]
  uint64_t* s_full = kv_empty + C::STAGES;             // [NT]
  uint64_t* p_full = s_full + NT;                      // [NT]
  uint64_t* pv_done = p_full + NT;                     // [NT] (SEP_P: every P V^T; else the last)
  uint64_t* s_free = pv_done + NT;                     // [NT] (SEP_P only)
  uint64_t* mma_drain = s_free + NT;                   // [NMMA] abort teardown only
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_drain + C::NMMA);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + C::NMMA + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (NT * BQ), h = blockIdx.y, b = blockIdx.z;
  const int nkv = int((p.nk + BKV - 1) / BKV);
  // Query tiles of this CTA that hold rows (the second one can lie wholly
  // past nq in the last block); empty tiles are skipped by every role.
  const int ntv = int((p.nq - q0 + BQ - 1) / BQ) < NT ? int((p.nq - q0 + BQ - 1) / BQ) : NT;
  // MMA warps with work: each commits the release of every K / V stage.
  const int nmma = C::SEP_P ? ntv : 1;
  // Loads thread 0 issued into each ring stage: an aborting CTA waits for
  // the last of them before it exits.
  int nload[C::STAGES];
#pragma unroll
  for (int s = 0; s < C::STAGES; ++s) nload[s] = 0;
  // Key tile j (K and V, 128 keys) into ring stage j % STAGES (thread 0).
  auto load_kv = [&](int j) {
    const int s = j % C::STAGES;
    if (j == p.hold_kv) return;  // self-test: the stage never fills
    ++nload[s];
    mbar_expect_tx(&kv_full[s], C::K_BYTES + C::V_BYTES);
    uint8_t* kt = sk + s * C::K_BYTES;
    for (int dc = 0; dc < C::DC; ++dc)
      tma_load_4d(kt + dc * (BKV * 128), &map_k, &kv_full[s], dc * 64, p.k_hn ? h : j * BKV,
                  p.k_hn ? j * BKV : h, b);
    uint8_t* vt = sv + s * C::V_BYTES;
    for (int dc = 0; dc < C::DC; ++dc)
      tma_load_4d(vt + dc * (BKV * 128), &map_v, &kv_full[s], dc * 64, p.v_hn ? h : j * BKV,
                  p.v_hn ? j * BKV : h, b);
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], nmma);  // one commit per MMA warp with work
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&s_free[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    for (int w = 0; w < C::NMMA; ++w) mbar_init(&mma_drain[w], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // The Q tiles and the first key tiles start loading before the TMEM
    // allocation and the block barrier (the producer issues the rest).
    mbar_expect_tx(q_full, ntv * C::Q_BYTES);
    for (int t = 0; t < ntv; ++t)
      for (int dc = 0; dc < C::DC; ++dc) {
        const int row = q0 + t * BQ;
        tma_load_4d(sq + t * C::Q_BYTES + dc * (BQ * 128), &map_q, q_full, dc * 64,
                    p.q_hn ? h : row, p.q_hn ? row : h, b);
      }
    for (int j = 0; j < nkv && j < C::STAGES; ++j) load_kv(j);
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
    // (the Q tiles and the first STAGES key tiles were issued at set-up)
    if (lane == 0) {
      for (int j = C::STAGES; j < nkv && !*abort_flag; ++j) {
        const int s = j % C::STAGES;
        if (!mbar_wait(&kv_empty[s], ((j / C::STAGES) - 1) & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns))
          break;
        load_kv(j);
      }
    }
  } else if (warp <= C::NMMA) {
    // ------------------------------------------------------------------ MMA
    // Each MMA warp issues for its query tiles (t0 .. t0 + NT / NMMA); all
    // read the same K / V stages and each commits the stage's release once
    // its products are issued.
    constexpr int TPW = NT / C::NMMA;
    const int t0 = (warp - 1) * TPW;
    const int t1 = min(t0 + TPW, ntv);  // this warp's tiles with rows: t0 .. t1 - 1
    if (lane == 0 && t0 < t1) {
      auto issue_s = [&](int t, int j) {
        const uint8_t* kt = sk + (j % C::STAGES) * C::K_BYTES;
        const uint8_t* qt = sq + t * C::Q_BYTES;
#pragma unroll
        for (int dc = 0; dc < C::DC; ++dc) {
          const uint64_t da = smem_desc_sw128(qt + dc * (BQ * 128));
          const uint64_t db = smem_desc_sw128(kt + dc * (BKV * 128));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16<C::IDESC_S>(tmem_base + C::COL_S + t * BKV, da + uint64_t(2 * k),
                                 db + uint64_t(2 * k), (dc | k) ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint8_t* vt = sv + (j % C::STAGES) * C::V_BYTES;
        const uint32_t ta = tmem_base + C::COL_P + t * C::P_STRIDE;
        // K step of 16 keys = 16 rows of 128 B; P advances 8 columns.
        const uint64_t db = smem_desc_sw128_mn(vt, BKV * 128);
#pragma unroll
        for (int ks = 0; ks < BKV / 16; ++ks)
          umma_f16_ts<C::IDESC_O>(tmem_base + C::COL_O + t * D, ta + uint32_t(ks * 8),
                                  db + uint64_t(ks * (16 * 128 >> 4)), (j | ks) ? 1u : 0u);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, ST_TIMEOUT, p.wait_ns) &&
                mbar_wait(&kv_full[0], 0, abort_flag, p.status, ST_TIMEOUT, p.wait_ns);
      if (ok) {
        tc_fence_after();
        for (int t = t0; t < t1; ++t) issue_s(t, 0);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const bool more = j + 1 < nkv;
        bool kv_ready = !more;
        auto wait_kv = [&]() {
          if (!kv_ready)
            kv_ready = mbar_wait(&kv_full[(j + 1) % C::STAGES], ((j + 1) / C::STAGES) & 1,
                                 abort_flag, p.status, ST_TIMEOUT, p.wait_ns);
          return kv_ready;
        };
        for (int t = t0; ok && t < t1; ++t) {
          if constexpr (C::SEP_P) {
            // S_t(j+1) as soon as the softmax warps have copied S_t(j) to
            // registers, then O_t += P_t(j) V(j)^T once P_t(j) is written.
            if (more) {
              if (!wait_kv() || !mbar_wait(&s_free[t], j & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(t, j + 1);
            }
            if (!mbar_wait(&p_full[t], j & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, j);
            umma_commit(&pv_done[t]);
            if (t == t1 - 1) umma_commit(&kv_empty[j % C::STAGES]);
          } else {
            // O_t += P_t(j) V(j)^T, then S_t(j+1) over the consumed P_t(j).
            if (!mbar_wait(&p_full[t], j & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, j);
            if (t == t1 - 1) umma_commit(&kv_empty[j % C::STAGES]);
            if (more) {
              if (!wait_kv()) { ok = false; break; }
              tc_fence_after();
              issue_s(t, j + 1);
            } else {
              umma_commit(&pv_done[t]);
            }
          }
        }
      }
    }
  } else if ((warp - 1 - C::NMMA) >> 2 < ntv) {
    // ------------------------------------------------------ softmax / epilogue
    const int t = (warp - 1 - C::NMMA) >> 2;     // query tile of this warp
    const int quarter = warp & 3;                // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;           // query row within the tile
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t t_s = tmem_base + C::COL_S + t * BKV + lane_off;
    const uint32_t t_o = tmem_base + C::COL_O + t * D + lane_off;
    const uint32_t t_p = tmem_base + C::COL_P + t * C::P_STRIDE + lane_off;
    const float2 sc2 = f2(p.scale_log2);
    float m = -INFINITY;                         // running max, log2 units
    float2 l2 = f2(0.f);                         // running row sum (two halves)
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) { ok = false; break; }
      tc_fence_after();
      // The row's scores into registers; S is then free for S(j + 1).
      float sv[BKV];
#pragma unroll
      for (int c = 0; c < BKV; c += 64) tmem_ld64(t_s + uint32_t(c), sv + c);
      if constexpr (C::SEP_P) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);
      }
      const int kvalid = int(p.nk - int64_t(j) * BKV);  // keys of this tile (may exceed BKV)
      if (kvalid < BKV) {
#pragma unroll
        for (int e = 0; e < BKV; ++e)
          if (e >= kvalid) sv[e] = -INFINITY;
      }
      float mx0 = sv[0], mx1 = sv[1];
#pragma unroll
      for (int e = 2; e < BKV; e += 2) {
        mx0 = fmaxf(mx0, sv[e]);
        mx1 = fmaxf(mx1, sv[e + 1]);
      }
      const float mxs = fmaxf(mx0, mx1) * p.scale_log2;  // scale > 0
      const bool grow = mxs > m + RESCALE_LOG2;          // always on the first tile
      const float m_new = grow ? mxs : m;
      const float alpha = grow ? ex2f(m - m_new) : 1.f;  // 0 on the first tile
      // Without SEP_P, S_t(j) complete implies P_t(j-1) V^T complete: O_t is
      // stable and P_t free.  With SEP_P that is waited for here, before a
      // rescale, or else just before P is stored.
      bool pv_waited = !C::SEP_P || j == 0;
      if (j > 0) {
        if (__any_sync(0xffffffffu, grow)) {
          if (!pv_waited) {
            if (!mbar_wait(&pv_done[t], (j - 1) & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) { ok = false; break; }
            tc_fence_after();
            pv_waited = true;
          }
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(t_o + uint32_t(c), o);
            uint32_t u[32];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 v = mul2(make_float2(o[e], o[e + 1]), f2(alpha));
              u[e] = __float_as_uint(v.x);
              u[e + 1] = __float_as_uint(v.y);
            }
            tmem_st32u(t_o + uint32_t(c), u);
          }
        }
      }
      // P = exp2(s * scale * log2 e - m) as packed bf16 pairs into the P
      // columns of this row, and the row sum.
      const float2 nm2 = f2(-m_new);
      l2 = mul2(l2, f2(alpha));
      uint32_t u[BKV / 2];
#pragma unroll
      for (int e = 0; e < BKV; e += 2) {
        const float2 x = fma2(make_float2(sv[e], sv[e + 1]), sc2, nm2);
        const float2 f = ((e >> 1) & 7) < C::POLY ? ex2_poly2(x)
                                                      : make_float2(ex2f(x.x), ex2f(x.y));
        l2 = add2(l2, f);
        u[e >> 1] = pack_bf16x2(f.x, f.y);
      }
      if (!pv_waited) {  // P_t(j-1) V^T has read P_t
        if (!mbar_wait(&pv_done[t], (j - 1) & 1, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < BKV / 2; c += 32) tmem_st32u(t_p + uint32_t(c), u + c);
      tmem_wait_st();
      m = m_new;
      // P is in TMEM and O is rescaled.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // Epilogue: O / l, bf16, after the last P V^T.
    if (ok && nkv > 0 &&
        mbar_wait_idle(&pv_done[t], C::SEP_P ? (nkv - 1) & 1 : 0, abort_flag, p.status, ST_TIMEOUT, p.wait_ns)) {
      tc_fence_after();
      const float l = l2.x + l2.y;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t qi = int64_t(q0) + t * BQ + r;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + int64_t(b) * p.ob +
                            int64_t(h) * p.oh + qi * p.on;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(t_o + uint32_t(c), o);
        if (qi < p.nq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = o[8 * q + e] * inv;
            *reinterpret_cast<uint4*>(orow + c + 8 * q) = pack(f, __nv_bfloat16());
          }
        }
      }
    }
  }

  // Teardown.  After an abort nothing the CTA started may still be running
  // when it frees TMEM and exits: each MMA-issuing thread commits its issued
  // MMAs to a drain barrier and waits for it, and thread 0 waits for the last
  // TMA load it issued into the Q tiles and into each K / V stage (all
  // bounded).  The normal path needs neither: every MMA was waited for
  // through pv_done and every load consumed.
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    if (warp >= 1 && warp <= C::NMMA && lane == 0) {
      umma_commit(&mma_drain[warp - 1]);
      mbar_drain(&mma_drain[warp - 1], 0, p.wait_ns);
    }
    if (threadIdx.x == 0) {
      if (ntv > 0) mbar_drain(q_full, 0, p.wait_ns);
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s)
        if (nload[s] > 0) mbar_drain(&kv_full[s], uint32_t(nload[s] - 1) & 1u, p.wait_ns);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

// 4-D bf16 view [B, H, rows, cols] (cols contiguous) as a TMA map with a box
// of 64 columns x box_rows rows, 128B swizzle.  The map's dimensions are
// ordered by stride: (cols, rows, H, B), or (cols, H, rows, B) when heads are
// closer in memory than rows (*hn = 1; the kernel swaps those coordinates).
// Strides of size-1 dimensions are replaced by packed ones.
static bool make_map4(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t rows,
                      int64_t cols, int64_t s_row, int64_t s_h, int64_t s_b, uint32_t box_rows,
                      int* hn) {
  auto fn = encode_fn();
  if (!fn) return false;
  if (rows <= 1) s_row = cols;
  if (H <= 1) s_h = s_row * rows;
  if (B <= 1) s_b = (s_h > s_row ? s_h * H : s_row * rows);
  *hn = s_h < s_row ? 1 : 0;
  const cuuint64_t dims[4] = {uint64_t(cols), uint64_t(*hn ? H : rows), uint64_t(*hn ? rows : H),
                              uint64_t(B)};
  const cuuint64_t strides[3] = {uint64_t(*hn ? s_h : s_row) * 2, uint64_t(*hn ? s_row : s_h) * 2,
                                 uint64_t(s_b) * 2};
  const cuuint32_t box[4] = {64u, *hn ? 1u : box_rows, *hn ? box_rows : 1u, 1u};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace attn
}  // namespace l3d

using namespace l3d;

extern "C" size_t l3d_attention_workspace_size(int64_t b, int64_t h, int64_t nk, int64_t d) {
  if (b < 0 || h < 0 || nk < 0 || d < 0) return 0;
  return 256;  // the status word; q, k and v are read in place
}

static int run_attention(const l3d_tensor* q, const l3d_tensor* k, const l3d_tensor* v,
                         float scale, const l3d_tensor* out, void* workspace,
                         size_t workspace_bytes, l3d_stream stream, uint64_t wait_ns, int hold_kv,
                         const char* op) {
  using namespace l3d::attn;
  const l3d_tensor* all[] = {q, k, v, out};
  for (const l3d_tensor* t : all) {
    if (!t) return fail(L3D_E_NULL, "%s: q, k, v and out are required", op);
    if (t->dtype != L3D_BF16) return fail(L3D_E_DTYPE, "%s: q, k, v, out must be BF16", op);
    if (t->ndim != 4) return fail(L3D_E_SHAPE, "%s: tensors must be [B, H, N, D]", op);
    if (t->strides[3] != 1) return fail(L3D_E_ALIGN, "%s: the head dim must be contiguous", op);
  }
  const int64_t B = q->dims[0], H = q->dims[1], nq = q->dims[2], D = q->dims[3];
  const int64_t nk = k->dims[2];
  if (k->dims[0] != B || k->dims[1] != H || k->dims[3] != D || v->dims[0] != B ||
      v->dims[1] != H || v->dims[2] != nk || v->dims[3] != D || out->dims[0] != B ||
      out->dims[1] != H || out->dims[2] != nq || out->dims[3] != D)
    return fail(L3D_E_SHAPE, "%s: q [B,H,N,D], k and v [B,H,Nk,D], out [B,H,N,D]", op);
  if (D != 64 && D != 128) return fail(L3D_E_UNSUPPORTED, "%s: head dim must be 64 or 128", op);
  if (!(scale > 0.f) || !(scale < 3.0e38f))
    return fail(L3D_E_UNSUPPORTED, "%s: scale must be positive and finite", op);
  if (B > 65535 || H > 65535 || nq > (int64_t(1) << 30) || nk > (int64_t(1) << 30))
    return fail(L3D_E_UNSUPPORTED, "%s: dimensions too large", op);
  const size_t need = l3d_attention_workspace_size(B, H, nk, D);
  if (!workspace || workspace_bytes < need)
    return fail(L3D_E_WORKSPACE, "%s: workspace of %zu bytes required", op, need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(L3D_E_ALIGN, "%s: workspace must be 256-byte aligned", op);
  if (B * H * nq == 0) return L3D_OK;
  for (const l3d_tensor* t : all) {
    if (no_data(t)) return fail(L3D_E_NULL, "%s: null data pointer", op);
    if (reinterpret_cast<uintptr_t>(elem_ptr(t)) % 16)
      return fail(L3D_E_ALIGN, "%s: tensors must be 16-byte aligned", op);
    for (int i = 0; i < 3; ++i)
      if (t->dims[i] > 1 && (t->strides[i] * 2) % 16)
        return fail(L3D_E_ALIGN, "%s: strides must be multiples of 16 bytes", op);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(status, 0, 256, s) != cudaSuccess)
    return fail(L3D_E_CUDA, "%s: status clear failed", op);
  if (nk == 0) {
    // softmax over no keys: zeros, as an empty sum.
    const int64_t on = out->strides[2];
    if (on == D && out->strides[1] == nq * D && out->strides[0] == H * nq * D) {
      if (cudaMemsetAsync(const_cast<char*>(elem_ptr(out)), 0, size_t(B * H * nq * D) * 2, s) !=
          cudaSuccess)
        return fail(L3D_E_CUDA, "%s: memset failed", op);
      return L3D_OK;
    }
    return fail(L3D_E_UNSUPPORTED, "%s: empty keys need a contiguous out", op);
  }
  CUtensorMap map_q, map_k, map_v;
  int q_hn = 0, k_hn = 0, v_hn = 0;
  if (!make_map4(&map_q, elem_ptr(q), B, H, nq, D, q->strides[2], q->strides[1], q->strides[0], BQ,
                 &q_hn) ||
      !make_map4(&map_k, elem_ptr(k), B, H, nk, D, k->strides[2], k->strides[1], k->strides[0],
                 uint32_t(D == 64 ? Cfg<64>::BKV : Cfg<128>::BKV), &k_hn) ||
      !make_map4(&map_v, elem_ptr(v), B, H, nk, D, v->strides[2], v->strides[1], v->strides[0],
                 uint32_t(Cfg<64>::BKV), &v_hn))
    return fail(L3D_E_CUDA, "%s: cuTensorMapEncodeTiled failed", op);
  Params p{};
  p.q_hn = q_hn;
  p.k_hn = k_hn;
  p.v_hn = v_hn;
  p.nq = nq;
  p.nk = nk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = const_cast<char*>(elem_ptr(out));
  p.ob = out->strides[0];
  p.oh = out->strides[1];
  p.on = out->strides[2];
  p.status = status;
  p.wait_ns = wait_ns;
  p.hold_kv = hold_kv;
  const dim3 grid(unsigned((nq + NT * BQ - 1) / (NT * BQ)), unsigned(H), unsigned(B));
  const cudaError_t attr =
      D == 64 ? set_smem_limit(reinterpret_cast<const void*>(attn_kernel<64>), Cfg<64>::SMEM)
              : set_smem_limit(reinterpret_cast<const void*>(attn_kernel<128>), Cfg<128>::SMEM);
  if (attr != cudaSuccess) return fail(L3D_E_CUDA, "%s: cannot reserve shared memory", op);
  if (D == 64) attn_kernel<64><<<grid, Cfg<64>::THREADS, Cfg<64>::SMEM, s>>>(map_q, map_k, map_v, p);
  else attn_kernel<128><<<grid, Cfg<128>::THREADS, Cfg<128>::SMEM, s>>>(map_q, map_k, map_v, p);
  return check_launch(op);
}

extern "C" int l3d_attention(const l3d_tensor* q, const l3d_tensor* k, const l3d_tensor* v,
                             float scale, const l3d_tensor* out, void* workspace,
                             size_t workspace_bytes, l3d_stream stream) {
  return run_attention(q, k, v, scale, out, workspace, workspace_bytes, stream,
                       l3d::tc::WAIT_LIMIT_NS, -1, "l3d_attention");
}

extern "C" int l3d_attention_selftest_timeout(const l3d_tensor* q, const l3d_tensor* k,
                                              const l3d_tensor* v, float scale,
                                              const l3d_tensor* out, void* workspace,
                                              size_t workspace_bytes, uint32_t wait_limit_ms,
                                              l3d_stream stream) {
  const char* op = "l3d_attention_selftest_timeout";
  if (wait_limit_ms == 0 || wait_limit_ms > 2000)
    return fail(L3D_E_UNSUPPORTED, "%s: wait_limit_ms must be in [1, 2000]", op);
  if (k && k->ndim == 4 && k->dims[2] == 0)
    return fail(L3D_E_UNSUPPORTED, "%s: needs at least one key", op);
  return run_attention(q, k, v, scale, out, workspace, workspace_bytes, stream,
                       uint64_t(wait_limit_ms) * 1000000ull, 0, op);
}
