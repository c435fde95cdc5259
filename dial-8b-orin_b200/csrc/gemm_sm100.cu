// Prefill dequant-GEMM (tcgen05).  Not yet enabled: every M goes to the skinny kernel.
#include "gemm_sm100.cuh"

namespace dial {

bool gemm_sm100_supported(int64_t, int64_t, int64_t) { return false; }
size_t gemm_sm100_gguf_workspace_bytes(int64_t, int64_t) { return 0; }
dial_status launch_w8a16_gemm_sm100(const void*, dial_dtype, const int8_t*, const void*,
                                    dial_dtype, void*, int64_t, int64_t, int64_t, cudaStream_t) {
  return fail(DIAL_ERR_SHAPE, "tcgen05 GEMM not available");
}
dial_status launch_gguf_gemm_sm100(const void*, dial_dtype, const void*, const uint16_t*, int,
                                   void*, int64_t, int64_t, int64_t, void*, cudaStream_t) {
  return fail(DIAL_ERR_SHAPE, "tcgen05 GEMM not available");
}

}  // namespace dial
