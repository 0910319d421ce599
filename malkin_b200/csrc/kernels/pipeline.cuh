// Shared-memory pipeline primitives for sm_100a: mbarriers and TMA bulk copies (cp.async.bulk) with
// bounded waits. A wait that runs out records an error code in a global status word and returns false, so a
// kernel whose copies never land returns instead of hanging the GPU.
#pragma once
#include <cstdint>

namespace mkb {

// Iterations of try_wait (each suspends for a hardware-chosen interval) before a wait gives up: far above any
// legitimate wait (a few microseconds), far below a hang (the loop ends within about a second).
constexpr uint32_t kWaitLimit = 1u << 20;

// Error codes in the status word.
constexpr int kErrWaitFull = 1;   // consumer waited for a stage that never filled
constexpr int kErrWaitEmpty = 2;  // producer waited for a stage that was never released

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false (and *status = code) if it never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (status) atomicCAS(status, 0, code);
  return false;
}

// mbar_wait by a whole warp with one outcome for every lane (true only if every lane saw the phase complete), so
// the warp stays converged for the .sync.aligned instructions that follow.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_wait(bar, parity, status, code);
  return __all_sync(0xffffffffu, ok) != 0;
}

// mbar_wait_warp for a warp in which only lane 0 acts on the guarded data (an MMA issuer): lane 0 alone polls, so
// the wait costs one shared-memory access per poll instead of 32, and the outcome is broadcast to the warp.
__device__ __forceinline__ bool mbar_wait_lane0(uint64_t* bar, uint32_t parity, int* status, int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, status, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// mbar_wait_warp for waits that are long or off the critical path: the warp sleeps about sleep_ns between polls,
// leaving its issue slots and the shared-memory pipe to the warps doing the work (the bound grows to
// kWaitLimit * sleep_ns).
__device__ __forceinline__ bool mbar_wait_warp_sleep(uint64_t* bar, uint32_t parity, int* status, int code,
                                                     uint32_t sleep_ns) {
  bool ok = false;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) {
      ok = true;
      break;
    }
    __nanosleep(sleep_ns);
  }
  if (!ok && status) atomicCAS(status, 0, code);
  return __all_sync(0xffffffffu, ok) != 0;
}

// 1-D bulk copy global -> shared, completion counted in bytes on bar. dst, src 16-byte aligned; bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace mkb
