// PTX helpers shared by the TMA / tcgen05 kernels and the bulk-copy streaming kernels:
// shared-memory addresses, mbarriers with bounded waits, and 1-D bulk copies.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace dsmz {

constexpr uint64_t kTimeoutNs = 1000000000ull;   // a wait gives up after ~1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One arrival that also raises the phase's expected transaction bytes.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Plain arrival (release at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or the
// hint runs out) instead of spinning, so waiting warps leave the issue slots to the warps
// doing the work.
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after kTimeoutNs (error word set) or when another role failed.
// The error word is one global address shared by every waiting thread of the grid, so it
// is read only every kPollNs of waiting: polled on every spin it turns into an L2 hot
// spot that slows the very copies being waited for.
constexpr uint64_t kPollNs = 20000;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  uint64_t tchk = t0;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    const uint64_t t = gtimer();
    if (t - tchk > kPollNs) {
      tchk = t;
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (t - t0 > kTimeoutNs) {
        atomicExch(err, 1);
        return false;
      }
    }
  }
}
// Wait for copies already issued to land before the CTA may exit: ignores the error word,
// gives up after kTimeoutNs.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity)) {
    if (gtimer() - t0 > kTimeoutNs) return;
  }
}
// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// 16-byte asynchronous copy global -> shared (L2 only), both addresses 16-byte aligned.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// One arrival on `bar` once every cp.async this thread issued so far has landed (the
// barrier's expected count includes it).
__device__ __forceinline__ void cp16_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// D += A B on the fp64 tensor path (m8n8k4): per thread one element of A (row lane/4,
// column lane%4), one of B (row lane%4, column lane/4) and two of D (row lane/4, columns
// 2(lane%4) and 2(lane%4)+1).
// Not volatile: a pure register computation, so loads may be scheduled across it.
__device__ __forceinline__ void dmma8x8x4(double& d0, double& d1, double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
      : "+d"(d0), "+d"(d1)
      : "d"(a), "d"(b));
}
__device__ __forceinline__ void tmap_acquire(const CUtensorMap* m) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(m) : "memory");
}
// 2-D TMA load into this CTA's own shared memory, completing on `bar`; x is the
// innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// L2 eviction policies for the cache_hint forms of the TMA loads (createpolicy).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// tma_load_2d with an L2 cache policy (no cluster multicast).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* m, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Acquire load of a counter another CTA advances with release semantics.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Orders this thread's generic-proxy global accesses with the async proxy (TMA) accesses
// that follow (or that other threads make after synchronising with it).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bounded wait until *p >= target (another CTA's release-ordered counter): false after
// kTimeoutNs (error word set) or when another role failed.
__device__ __forceinline__ bool spin_geq(const int* p, int target, int* err) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = gtimer();
  uint64_t tchk = t0;
  while (true) {
    __nanosleep(256);
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t = gtimer();
    if (t - tchk > kPollNs) {
      tchk = t;
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (t - t0 > kTimeoutNs) {
        atomicExch(err, 1);
        return false;
      }
    }
  }
}

// Barrier over the `n` threads of the consumer warps (id 1; warp-multiple n).
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

}  // namespace dsmz
