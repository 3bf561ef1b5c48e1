// Shared-memory ring of bulk-copied rows: the mbarrier helpers of the
// kernels that stream whole rows through shared memory (the row-norm ring).  A producer issues one cp.async.bulk per row into a slot and the
// slot's `full` barrier completes when the bytes land; the consumer warp
// arrives on the slot's `empty` barrier once it holds the row in registers.
#pragma once
#include <cstdint>

namespace l3d {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ring_bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void ring_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool ring_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t ring_clock_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// One row (bytes: a multiple of 16, both addresses 16-byte aligned) from
// global memory into a slot; completes `full`.
__device__ __forceinline__ void ring_load(void* slot, const void* src, uint32_t bytes,
                                          uint64_t* full) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(full)),
               "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(slot)),
      "l"(src), "r"(bytes), "r"(smem_addr(full))
      : "memory");
}
__device__ __forceinline__ void ring_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Bounded wait.  Normal mode: false when another warp of the block has
// aborted, or on expiry (then the abort flag is raised and status 5 recorded
// in *status).  Drain mode (teardown after an abort): ignores the flag and
// records nothing.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t limit_ns, bool drain, int* status) {
  if (ring_try_wait(bar, parity)) return true;
  const uint64_t t0 = ring_clock_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (ring_try_wait(bar, parity)) return true;
    if (!drain && *abort_flag) return false;
    if (ring_clock_ns() - t0 > limit_ns) {
      if (!drain) {
        *abort_flag = 1;
        atomicCAS(status, 0, 5);
      }
      return false;
    }
  }
}

}  // namespace l3d
