// Shared helpers for the DIAL B200 kernels: status plumbing, launch counting,
// activation dtype traits and small PTX wrappers.  sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "dial_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a (B200) only"
#endif

namespace dial {

// ---------------------------------------------------------------- host side
// Records a formatted message in the calling thread's error slot and returns s.
dial_status fail(dial_status s, const char* fmt, ...);
// Maps a CUDA error (from the call named `what`) to DIAL_ERR_CUDA.
dial_status cuda_fail(cudaError_t e, const char* what);
// Checks the launch that was just made; counts it on success.
dial_status check_launch(const char* kernel_name);
void clear_error();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(dial_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

// Raises KERN's dynamic shared-memory limit to `bytes` once per device (the
// attribute belongs to the device's context, so every device needs its own call).
template <auto KERN>
cudaError_t ensure_smem(int bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(KERN, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  // the largest shared-memory carveout, so that two such CTAs can share an SM
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(KERN, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: the decode-chain kernels are launched with
// programmatic stream serialization, so a kernel's CTAs may be scheduled while
// its predecessor in the stream is still running.  Every such kernel calls
// pdl_trigger() (let the next kernel be scheduled) and pdl_wait() (block until
// the predecessor grid has completed and its memory is visible) before it
// touches any global data another kernel writes, and before any early return,
// so completion stays transitive along the stream.  Work that reads only
// constant data (weights) may run between the two.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_begin() {
  pdl_trigger();
  pdl_wait();
}

// DIAL_PDL=0 in the environment turns the attribute off (kernels then start
// only after their predecessor ends; pdl_wait() returns at once).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
dial_status launch_pdl(const char* name, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_fail(e, name);
  }
  return check_launch(name);
}

// ---------------------------------------------------------------- device side
template <typename T>
struct Act;
template <>
struct Act<float> {
  static __device__ __forceinline__ float to_f32(float v) { return v; }
  static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <>
struct Act<__half> {
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};
template <>
struct Act<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};

// Streaming 128-bit load: read-only path, do not keep the line in L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Read-only 128-bit load that may stay in L1 (activations reused across warps).
__device__ __forceinline__ uint4 ld_ro16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Greedy-sampling key of a logit: the order of the keys is the order of
// (value, -index), so the largest key is the first index of the maximum, as
// argmax_kernel picks it (NaN never wins: it maps to the smallest key; -0 and
// +0 compare equal, as floats do).
__device__ __forceinline__ unsigned long long argmax_key(float v, long long idx) {
  uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
  const uint32_t ord = v != v ? 0u : (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

}  // namespace dial
