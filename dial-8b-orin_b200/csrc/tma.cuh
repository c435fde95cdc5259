// mbarrier / TMA helpers shared by the pipelined kernels (sm_100a).
//
// Every wait is bounded: it gives up after kWaitNs on %globaltimer (or as soon
// as another thread has flagged an error), records DIAL_ERR_TIMEOUT in the
// device error flag and returns false, so a kernel can drain and exit instead
// of hanging the GPU.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace dial {
namespace tma {

constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*(volatile int*)err != 0) return false;
      if (global_ns() - t0 > kWaitNs) {
        atomicCAS(err, 0, (int)DIAL_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Error path: waits for a copy still in flight, ignoring the error flag, until
// `deadline` (%globaltimer ns).  Lets a kernel that gives up keep no TMA writes
// pending into shared memory it is about to release.
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity, unsigned long long deadline) {
  while (!mbar_try(bar, parity))
    if (global_ns() > deadline) return false;
  return true;
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// 2D tiled TMA load (no multicast) completing `bytes` on `bar`.
__device__ __forceinline__ void load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                        int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Starts fetching a tensor map (a __grid_constant__ kernel parameter) into the
// TMA unit's descriptor cache, so the first copy does not wait for it.
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 1D bulk copy (16-byte aligned addresses, size a multiple of 16), no multicast.
__device__ __forceinline__ void load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---------------------------------------------------------------- host side
// 2D tensor map over a row-major [rows, row_bytes] byte matrix with a
// {box_bytes, box_rows} box; swizzle_bytes 0 (none), 64 or 128 (SWIZZLE_64B /
// SWIZZLE_128B, which need box_bytes == swizzle_bytes).
dial_status make_byte_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                          int box_bytes, int box_rows, int swizzle_bytes);

}  // namespace tma
}  // namespace dial
