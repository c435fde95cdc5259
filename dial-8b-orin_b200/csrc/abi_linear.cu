// extern "C" entry points for the W8A16 and GGUF linears (include/dial_cuda.h).
//
// Argument checks mirror the reference's error returns (worker_w8a16.rs:369-378
// dtype / last-dim checks, :410-416 contiguity and divisibility; worker_gguf.rs
// :489-494 shape checks) and add what the 128-bit loads need (16-byte
// alignment).  Nothing here allocates.
#include <algorithm>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "layout.cuh"
#include "quant.cuh"

using namespace dial;

namespace {

dial_status check_dims(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0)
    return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive (M=%lld K=%lld N=%lld)",
                (long long)M, (long long)K, (long long)N);
  if (N > (1ll << 31) - 1 || K > (1ll << 31) - 1 || M > (1ll << 31) - 1)
    return fail(DIAL_ERR_SHAPE, "dimension exceeds 2^31-1");
  return DIAL_OK;
}

bool is_half(dial_dtype t) { return t == DIAL_F16 || t == DIAL_BF16; }
bool is_act(dial_dtype t) { return t == DIAL_F32 || t == DIAL_F16 || t == DIAL_BF16; }

dial_status check_type(dial_ggml_type t) {
  if (t != DIAL_GGML_Q4_0 && t != DIAL_GGML_Q8_0)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "ggml type %d is not Q4_0 (2) or Q8_0 (8)", (int)t);
  return DIAL_OK;
}

}  // namespace

extern "C" {

dial_status dial_w8a16_quantize(const void* w, dial_dtype wdt, int64_t N, int64_t K, int8_t* q,
                                void* scale, dial_dtype sdt, dial_stream stream) {
  clear_error();
  if (!w || !q || !scale) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (wdt != DIAL_F32 && wdt != DIAL_F16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "W8A16 quantiser takes f32 or f16 weights");
  if (sdt != DIAL_F32 && sdt != DIAL_F16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "W8A16 scale must be f32 or f16");
  if (N > (1ll << 31) - 1) return fail(DIAL_ERR_SHAPE, "N exceeds 2^31-1");
  return launch_w8a16_quantize(w, wdt, N, K, q, scale, sdt, as_stream(stream));
}

dial_status dial_w8a16_dequantize(const int8_t* q, const void* scale, dial_dtype sdt, int64_t N,
                                  int64_t K, void* w, dial_dtype wdt, dial_stream stream) {
  clear_error();
  if (!w || !q || !scale) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (sdt != DIAL_F32 && sdt != DIAL_F16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "W8A16 scale must be f32 or f16");
  if (!is_act(wdt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad output dtype");
  return launch_w8a16_dequantize(q, scale, sdt, N, K, w, wdt, as_stream(stream));
}

size_t dial_w8a16_linear_workspace_bytes(int64_t N) {
  if (N <= 0) return 0;
  return gemv_workspace_bytes(N);
}

dial_status dial_w8a16_linear(const void* x, dial_dtype xdt, const int8_t* q, const void* scale,
                              dial_dtype sdt, void* y, int64_t M, int64_t K, int64_t N,
                              void* workspace, size_t workspace_bytes, dial_stream stream) {
  clear_error();
  if (!x || !q || !scale || !y) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_dims(M, K, N);
  if (s != DIAL_OK) return s;
  if (!is_half(xdt))
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "W8A16 expects f16 or bf16 activations, got dtype %d",
                (int)xdt);
  if (sdt != DIAL_F32 && sdt != DIAL_F16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "W8A16 scale must be f32 or f16");
  if (K % 16) return fail(DIAL_ERR_SHAPE, "W8A16 needs K %% 16 == 0 (K=%lld)", (long long)K);
  if (!aligned16(x) || !aligned16(q))
    return fail(DIAL_ERR_MISALIGNED, "x and q must be 16-byte aligned");
  if (workspace) {
    const size_t need = dial_w8a16_linear_workspace_bytes(N);
    if (workspace_bytes < need || !aligned16(workspace))
      return fail(DIAL_ERR_INVALID_ARG, "workspace must be 16-byte aligned and hold %zu bytes", need);
  }
  cudaStream_t st = as_stream(stream);
  if (M > kSkinnyMaxM && gemm_sm100_supported(M, K, N))
    return launch_w8a16_gemm_sm100(x, xdt, q, scale, sdt, y, M, K, N, st);
  // Small M (and any shape the tensor-memory GEMM does not take): the skinny
  // kernel in chunks of at most kSkinnyMaxM activation rows.
  for (int64_t m0 = 0; m0 < M; m0 += kSkinnyMaxM) {
    const int64_t mc = std::min<int64_t>(kSkinnyMaxM, M - m0);
    s = launch_w8a16_skinny(static_cast<const uint16_t*>(x) + m0 * K, xdt, q, scale, sdt,
                            static_cast<uint16_t*>(y) + m0 * N, mc, K, N, st, workspace);
    if (s != DIAL_OK) return s;
  }
  return DIAL_OK;
}

dial_status dial_gguf_repack(const void* blocks, dial_ggml_type type, int64_t N, int64_t K,
                             void* qs, uint16_t* d, dial_stream stream) {
  clear_error();
  if (!blocks || !qs || !d) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_type(type);
  if (s != DIAL_OK) return s;
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  return launch_gguf_repack(blocks, type, N, K, qs, d, as_stream(stream));
}

dial_status dial_gguf_unpack(const void* qs, const uint16_t* d, dial_ggml_type type, int64_t N,
                             int64_t K, void* blocks, dial_stream stream) {
  clear_error();
  if (!blocks || !qs || !d) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_type(type);
  if (s != DIAL_OK) return s;
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  return launch_gguf_unpack(qs, d, type, N, K, blocks, as_stream(stream));
}

dial_status dial_gguf_quantize(const float* w, dial_ggml_type type, int64_t N, int64_t K, void* qs,
                               uint16_t* d, dial_stream stream) {
  clear_error();
  if (!w || !qs || !d) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_type(type);
  if (s != DIAL_OK) return s;
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  return launch_gguf_quantize(w, type, N, K, qs, d, as_stream(stream));
}

dial_status dial_gguf_dequantize(const void* qs, const uint16_t* d, dial_ggml_type type,
                                 int64_t N, int64_t K, void* w, dial_dtype wdt,
                                 dial_stream stream) {
  clear_error();
  if (!w || !qs || !d) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_type(type);
  if (s != DIAL_OK) return s;
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  if (!is_act(wdt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad output dtype");
  return launch_gguf_dequantize(qs, d, type, N, K, w, wdt, as_stream(stream));
}

// [stream-K scratch (fixed size for N)][Q8_0 activations of one <=32-row pass,
// or the tcgen05 path's f16 copy of f32 activations].  The stream-K counters
// sit at a fixed place, so one workspace serves calls with any M.
size_t dial_gguf_linear_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  const size_t act = std::max(gguf_skinny_workspace_bytes(std::min<int64_t>(kSkinnyMaxM, M), K),
                              gemm_sm100_gguf_workspace_bytes(M, K));
  return gemv_workspace_bytes(N) + act;
}

dial_status dial_gguf_linear(const void* x, dial_dtype xdt, const void* qs, const uint16_t* d,
                             dial_ggml_type type, void* y, int64_t M, int64_t K, int64_t N,
                             void* workspace, size_t workspace_bytes, dial_stream stream) {
  clear_error();
  if (!x || !qs || !d || !y) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  dial_status s = check_type(type);
  if (s != DIAL_OK) return s;
  s = check_dims(M, K, N);
  if (s != DIAL_OK) return s;
  if (!is_act(xdt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "activation dtype must be f32/f16/bf16");
  if (K % kQK) return fail(DIAL_ERR_SHAPE, "GGUF needs K %% 32 == 0 (K=%lld)", (long long)K);
  if (!aligned16(qs) || !aligned16(d) || !aligned16(x))
    return fail(DIAL_ERR_MISALIGNED, "x, qs and d must be 16-byte aligned");
  const size_t need = dial_gguf_linear_workspace_bytes(M, K, N);
  if (need && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    return fail(DIAL_ERR_INVALID_ARG, "workspace must be 16-byte aligned and hold %zu bytes", need);
  cudaStream_t st = as_stream(stream);
  void* sk = workspace;
  void* act = static_cast<uint8_t*>(workspace) + gemv_workspace_bytes(N);
  if (gemm_sm100_supported(M, K, N))
    return launch_gguf_gemm_sm100(x, xdt, qs, d, type, y, M, K, N, act, st);
  const size_t xsz = xdt == DIAL_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += kSkinnyMaxM) {
    const int64_t mc = std::min<int64_t>(kSkinnyMaxM, M - m0);
    s = launch_gguf_skinny(static_cast<const uint8_t*>(x) + m0 * K * xsz, xdt, qs, d, type,
                           static_cast<uint8_t*>(y) + m0 * N * xsz, mc, K, N, act, st, sk);
    if (s != DIAL_OK) return s;
  }
  return DIAL_OK;
}

}  // extern "C"

extern "C" {

size_t dial_gguf_qs_bytes(dial_ggml_type type, int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || (type != DIAL_GGML_Q4_0 && type != DIAL_GGML_Q8_0)) return 0;
  return (size_t)N * (size_t)gguf_groups(K) * (size_t)group_bytes(type);
}

size_t dial_gguf_d_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return (size_t)gguf_d_elems(N, K) * sizeof(uint16_t);  // rows padded to a multiple of 16
}

}  // extern "C"
