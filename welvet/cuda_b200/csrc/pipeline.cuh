// pipeline.cuh -- mbarrier / bulk-copy helpers shared by the TMA-fed kernels (sm_100a).
//
// Every wait is bounded by %globaltimer (kWaitNs): on expiry the waiting thread records an
// error code in the launch's error word and returns false, so a kernel whose producer or
// consumer went missing winds down instead of spinning forever.
#pragma once

#include <cstdint>

namespace wb {
namespace pipe {

constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the error word set) once kWaitNs of wall time has passed.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// A wait with its own limit (ns) on the same terms.
static __device__ __noinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int code, uint64_t ns) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > ns) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}

// The common case (phase already complete) stays inline; the bounded loop is out of line.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err, code);
}

// ---- CTA pairs (clusters of 2): barriers that the other CTA of the pair arrives on.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the object at `p`'s offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}

// Arrive on a barrier of either CTA of the pair (default semantics: release at CTA scope). A
// cluster-scope release here fenced every converter warp on every stage; what the even CTA's
// MMA needs from the odd CTA is ordered by tcgen05.wait::st and tcgen05.fence before the
// arrive, and its x bytes by the barrier's transaction count.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

// Every thread of both CTAs: arrivals before it are visible to the other CTA after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Ring position without divisions: slot and phase bit advance together.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void step(int n) {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Contiguous global -> shared copy (16-byte aligned, size a multiple of 16), no tensor map.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Lane 0 of the warp waits (bounded), the rest of the warp waits at __syncwarp: a few
// threads polling an mbarrier instead of whole warps.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, code);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

} // namespace pipe
} // namespace wb
