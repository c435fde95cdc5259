// dial_gguf_linear_noalloc: the GGUF integer-path linear without a caller
// workspace.
//
// dial_gguf_linear needs scratch memory for the activations it quantises to
// Q8_0 (the workspace argument).  Some callers cannot provide it: code that may
// not call cudaMalloc or an allocating library routine at that point (a custom
// allocator that is not re-entrant from the worker's request loop, a host
// runtime that forbids device allocation after load, an FFI caller with no
// device allocator of its own).  This entry point keeps that scratch in a
// file-scope __device__ array of fixed size instead, so it allocates nothing.
//
// Limits and rules:
//  * K <= kNoAllocMaxK (16384); larger K is rejected with DIAL_ERR_SHAPE.  Any
//    M is accepted and processed 32 activation rows per pass, always on the
//    integer (Q8_0-activation) path, passes running one after another on the
//    caller's stream.  The GEMV is the in-CTA K-split kernel
//    (gguf_skinny_kernel: plain 16-byte loads, the K groups of a tile split
//    over a CTA's warps and reduced in shared memory), not the TMA-fed
//    stream-K kernel dial_gguf_linear runs: that one needs a workspace for its
//    split-tile partials.  Same arithmetic, so the outputs agree within the
//    integer path's tolerance; its speed is not tuned.
//  * The array (640 KiB) lives on every GPU that loads the library until the
//    process exits.
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it with the
//    device's current context; make that first call before any stream capture
//    on that device.  After cudaDeviceReset the context differs, and the next
//    call looks the address up again (again outside a capture).
//  * Every call shares the one array.  Calls whose kernels overlap on the GPU
//    (different streams, or different host threads, without ordering between
//    them) race on it and give wrong results; order them on one stream.
//  * The array keeps the last call's contents.  Nothing in it has to start at
//    zero: each pass writes every quantised activation and block scale it later
//    reads.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "layout.cuh"
#include "quant.cuh"

namespace dial {

namespace {

constexpr int64_t kNoAllocMaxK = 16384;
constexpr int64_t kNoAllocRows = kSkinnyMaxM;  // activation rows per pass
// xq: 32 rows x 128 groups x 128 B, then xs: 128 groups x 4 blocks x 32 rows x 8 B
constexpr size_t kNoAllocBytes = 32 * 128 * 128 + 128 * 4 * 32 * 8;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
void* g_scratch_ptr[64] = {nullptr};
CUcontext g_scratch_ctx[64] = {nullptr};  // the context each cached address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (no -lcuda).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

// Device address of g_noalloc_scratch for the current device (set-up on the
// first use in the device's current context).
dial_status scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(DIAL_ERR_INVALID_ARG, "device ordinal %d out of range", dev);
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return fail(DIAL_ERR_CUDA, "cuCtxGetCurrent is unavailable");
  CUcontext ctx = nullptr;  // null until the runtime has made a context current on this thread
  if (get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev] || !ctx || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // sets up the primary context if needed
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return fail(DIAL_ERR_CUDA, "no current CUDA context");
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return DIAL_OK;
}

}  // namespace

}  // namespace dial

using namespace dial;

extern "C" dial_status dial_gguf_linear_noalloc(const void* x, dial_dtype xdt, const void* qs,
                                                const uint16_t* d, dial_ggml_type type, void* y,
                                                int64_t M, int64_t K, int64_t N,
                                                dial_stream stream) {
  clear_error();
  if (!x || !qs || !d || !y) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (type != DIAL_GGML_Q4_0 && type != DIAL_GGML_Q8_0)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "ggml type %d is not Q4_0 (2) or Q8_0 (8)", (int)type);
  if (M <= 0 || K <= 0 || N <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (N > (1ll << 31) - 1 || M > (1ll << 31) - 1) return fail(DIAL_ERR_SHAPE, "dimension exceeds 2^31-1");
  if (xdt != DIAL_F32 && xdt != DIAL_F16 && xdt != DIAL_BF16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "activation dtype must be f32/f16/bf16");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  if (K > kNoAllocMaxK)
    return fail(DIAL_ERR_SHAPE,
                "dial_gguf_linear_noalloc takes K <= %lld (got K=%lld): its fixed scratch array "
                "holds %zu bytes; use dial_gguf_linear with a workspace",
                (long long)kNoAllocMaxK, (long long)K, kNoAllocBytes);
  if (!aligned16(qs) || !aligned16(d) || !aligned16(x))
    return fail(DIAL_ERR_MISALIGNED, "x, qs and d must be 16-byte aligned");
  if (gguf_skinny_workspace_bytes(kNoAllocRows, K) > kNoAllocBytes)
    return fail(DIAL_ERR_SHAPE, "scratch sizing error");
  void* scratch = nullptr;
  dial_status s = scratch_for_current_device(&scratch);
  if (s != DIAL_OK) return s;
  const size_t xsz = xdt == DIAL_F32 ? 4 : 2;
  cudaStream_t st = as_stream(stream);
  for (int64_t m0 = 0; m0 < M; m0 += kNoAllocRows) {
    const int64_t mc = M - m0 < kNoAllocRows ? M - m0 : kNoAllocRows;
    s = launch_gguf_skinny(static_cast<const uint8_t*>(x) + m0 * K * xsz, xdt, qs, d, type,
                           static_cast<uint8_t*>(y) + m0 * N * xsz, mc, K, N, scratch, st,
                           /*sk_ws=*/nullptr);
    if (s != DIAL_OK) return s;
  }
  return DIAL_OK;
}
