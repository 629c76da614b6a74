// ptx.cuh -- thin wrappers over the sm_100a PTX used by the pipelined kernels:
// shared-memory addresses, the global timer, mbarriers with bounded waits,
// proxy fences.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gb {

// A bounded mbarrier wait gives up after this long (a normal wait is microseconds).
constexpr unsigned long long kMbarWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// Arrive without release semantics: the arriving thread's earlier global
// stores need not have completed (used where the waiter reads none of them).
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* b) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}

// A thread whose phase is not complete is suspended (not spinning, so it
// takes no issue slots from the warps doing work) until the phase completes
// or kMbarSuspendNs pass.
constexpr uint32_t kMbarSuspendNs = 1000000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(kMbarSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait (limit_ns, default kMbarWaitNs).  Returns false if the CTA is
// aborting or the wait ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                          int* err, uint64_t limit_ns = kMbarWaitNs) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(b, parity)) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicOr(err, 2);
      return false;
    }
  }
  return true;
}

// Programmatic dependent launch.  pdl_wait: wait until the grids this one
// depends on have completed and their writes are visible (returns at once for
// an ordinary launch); every kernel launched with launch_pdl calls it before
// its first global-memory access.  pdl_trigger: let the next grid on the
// stream begin launching (it still waits in its own pdl_wait).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}


// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace gb
