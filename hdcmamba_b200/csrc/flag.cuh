// System-scope flags between GPUs (sequence-parallel exchange over NVLink peer memory):
// acquire / release accesses and the bounded wait every consumer uses.
#pragma once
#include "tc.cuh"

namespace hdc {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// orders this thread's generic-proxy view (an acquired flag) before its later async-proxy
// global reads (bulk / TMA copies of the data the flag guards)
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// generation g has been reached (wrap-safe): a fast rank may already have written g + 1
__device__ __forceinline__ bool reached(uint32_t v, uint32_t g) { return (int32_t)(v - g) >= 0; }

constexpr uint64_t kPeerWaitNs = 2000000000ull;  // default limit of every flag wait (2 s)

// bounded spin until *flag has reached generation want; false (and the error code) after
// limit_ns nanoseconds of %globaltimer
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t want, int code,
                                          uint64_t limit_ns = kPeerWaitNs) {
  if (reached(ld_acquire_sys(flag), want)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!reached(ld_acquire_sys(flag), want)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicCAS(&g_dev_error, 0, code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// every flag s with bit s of mask set (s < 32) reaches *gen; false if a wait timed out
__device__ __forceinline__ bool wait_flags(const uint32_t* flags, uint32_t mask, const uint32_t* gen, int code) {
  const uint32_t g = *gen;
  bool ok = true;
#pragma unroll 1
  for (uint32_t m = mask; m != 0; m &= m - 1) ok = wait_flag(flags + (__ffs(m) - 1), g, code) && ok;
  return ok;
}

// After a wait that another thread finished: this thread acquires every flag of mask itself,
// so its later loads of the guarded data are ordered after the producer's stores.
__device__ __forceinline__ void acquire_flags(const uint32_t* flags, uint32_t mask) {
#pragma unroll 1
  for (uint32_t m = mask; m != 0; m &= m - 1) (void)ld_acquire_sys(flags + (__ffs(m) - 1));
}

// CTA-wide wait: thread 0 waits (bounded) for every flag of mask to reach *gen, the CTA
// synchronises, and every thread acquires the flags.  All threads of the CTA call it.
__device__ __forceinline__ void cta_wait_flags(const uint32_t* flags, uint32_t mask, const uint32_t* gen, int code) {
  if (threadIdx.x == 0) wait_flags(flags, mask, gen, code);
  __syncthreads();
  acquire_flags(flags, mask);
}

}  // namespace hdc
