// TMA bulk copies (cp.async.bulk, never with cluster multicast) completing on shared-memory
// mbarriers, with bounded waits, plus small synchronisation helpers shared by the kernels.
#pragma once
#include "common.cuh"

namespace wisp {

__host__ __device__ inline int64_t ru16(int64_t v) { return (v + 15) & ~int64_t(15); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

constexpr unsigned WAIT_LIMIT = 1u << 24;  // bounded polling; a copy that never lands sets WAIT_TIMEOUT

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
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
// bounded wait on the given phase parity; flags and returns false if it gave up
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (unsigned it = 0; it < WAIT_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  flag(WISP_STATUS_WAIT_TIMEOUT);
  return false;
}
// TMA bulk copy global -> shared (no multicast), completing on an mbarrier
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// 16-byte aligned window [start, start+bytes) covering [off, off+len); skip = off - start
struct Win {
  int64_t start;
  uint32_t bytes, skip;
};
__device__ __forceinline__ Win window(int64_t off, int64_t len) {
  Win w;
  w.start = off & ~int64_t(15);
  w.bytes = uint32_t(ru16(off + len) - w.start);
  w.skip = uint32_t(off - w.start);
  return w;
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// pull [src, src + bytes) into L2 (16-byte aligned address, size a multiple of 16)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

}  // namespace wisp
