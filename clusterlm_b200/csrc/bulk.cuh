// bulk.cuh — Blackwell bulk-copy staging: mbarrier + cp.async.bulk (global -> this CTA's shared memory).
//
// No multicast form is used anywhere (every copy lands in the issuing CTA's own shared memory).  Every wait is
// bounded: after kSpinLimit polls it records an error code in the caller's flag and returns false, so a copy that
// never completes ends the kernel with a host-visible error instead of a hang.
#pragma once
#include <stdint.h>

namespace clm {

constexpr uint32_t kSpinLimit = 1u << 20;  // polls of mbarrier.try_wait (each suspends the thread briefly)
constexpr int kErrWaitTimeout = 2;         // error-flag value: a bounded wait gave up
constexpr int kErrPartialSlots = 3;        // error-flag value: a split reduction had more segments than slots

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async proxy; follow with __syncthreads().
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Same with an L2 eviction-first hint (data read exactly once).
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Plain arrival (no transaction bytes), e.g. a consumer warp releasing a ring slot.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Waits for phase `parity` of the barrier; false (and *err = kErrWaitTimeout) after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  if (err != nullptr) atomicExch(err, kErrWaitTimeout);
  return false;
}

// L2 prefetch of global bytes (no shared memory, no completion to wait for): src 16-byte aligned, bytes a multiple
// of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Prefetches into L2 the first `cap` bytes of share c of [base, base + total) split into G contiguous shares (the
// way a G-CTA stream-K kernel splits its operand), in pieces of at most 32 KB.
__device__ __forceinline__ void l2_prefetch_share(const uint8_t* base, unsigned long long total, int c, int G,
                                                  unsigned long long cap) {
  if (base == nullptr || G <= 0) return;
  const unsigned long long lo = (total * (unsigned long long)c / G) & ~15ull;
  unsigned long long hi = (total * (unsigned long long)(c + 1) / G) & ~15ull;
  if (hi > lo + cap) hi = lo + (cap & ~15ull);
  for (unsigned long long o = lo; o < hi; o += 32768ull) {
    const unsigned long long n = hi - o < 32768ull ? hi - o : 32768ull;
    bulk_prefetch_l2(base + o, (uint32_t)n);
  }
}

// mbar_wait for a thread that can afford a little latency (a producer waiting for a ring slot): sleeps `ns`
// nanoseconds between polls, so the spin does not take issue slots from the warps doing the work.  Bounded like
// mbar_wait (kSpinLimit polls).
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* err, uint32_t ns) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    __nanosleep(ns);
  }
  if (err != nullptr) atomicExch(err, kErrWaitTimeout);
  return false;
}

// Release-add on a global counter (gpu scope): makes this thread's earlier writes, and those ordered before it by a
// CTA barrier, visible to a reader that acquires the counter.
__device__ __forceinline__ void red_release_add(int* ctr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(ctr), "r"(v) : "memory");
}

// Waits until *ctr >= target with acquire loads (gpu scope); false (and *err = kErrWaitTimeout) after kSpinLimit
// polls.
__device__ __forceinline__ bool wait_count(const int* ctr, int target, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if (i >= 64) __nanosleep(64);
  }
  if (err != nullptr) atomicExch(err, kErrWaitTimeout);
  return false;
}

// ---- dataflow between CTAs (and between the overlapping launches of a window chain)

constexpr unsigned long long kDepWaitNs = 1000000000ull;  // a cross-CTA wait gives up after 1 s without progress

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool dep_failed(const int* err) { return *reinterpret_cast<const volatile int*>(err) != 0; }

__device__ __forceinline__ void dep_raise(int* err) { atomicCAS(err, 0, kErrWaitTimeout); }

// Waits until *ctr >= target (acquire, gpu scope); false when the error flag is (or gets) raised, or after
// kDepWaitNs without reaching the target (then it raises the flag itself), so every wait ends.
__device__ inline bool dep_wait(const int* ctr, int target, int* err) {
  if (ld_acquire(ctr) >= target) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire(ctr) >= target) return true;
    if ((i & 63) == 63) {
      if (dep_failed(err)) return false;
      if (globaltimer() - t0 > kDepWaitNs) {
        dep_raise(err);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// Removes `bytes` of expected transactions from the current phase of a barrier (copies that will not be issued).
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// Bulk copies issued after this read global memory written by other CTAs' ordinary stores.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

}  // namespace clm
