// Prefill dequant-GEMM on the sm_100a tensor cores (tcgen05 + TMEM), gemm_sm100.cu.
#pragma once

#include "common.cuh"

namespace dial {

// Fewest activation rows for the tcgen05 GEMM.  GGUF linears take it from 17
// rows (32-row token tiles: the integer GEMV re-reads its quantised
// activations per 16-row unit, which dominates at 32 rows); W8A16 linears
// from kSkinnyMaxM + 1.
constexpr int64_t kGemmMinRows = 17;
// True when the tcgen05 GEMM takes this shape (else the caller uses the skinny kernel).
bool gemm_sm100_supported(int64_t M, int64_t K, int64_t N);
size_t gemm_sm100_gguf_workspace_bytes(int64_t M, int64_t K);
dial_status launch_w8a16_gemm_sm100(const void* x, dial_dtype xdt, const int8_t* q,
                                    const void* scale, dial_dtype sdt, void* y, int64_t M,
                                    int64_t K, int64_t N, cudaStream_t st);
dial_status launch_gguf_gemm_sm100(const void* x, dial_dtype xdt, const void* qs,
                                   const uint16_t* d, int type, void* y, int64_t M, int64_t K,
                                   int64_t N, void* ws, cudaStream_t st);

// Q4_K / Q6_K super-blocks as the file holds them ([N, K / 256] x 144 / 210
// bytes, 16-byte aligned), f16/bf16 activations, K % 256 == 0 (Q6_K: K % 2048
// == 0, so that a row is a 16-byte multiple): each weight group is one
// super-block, dequantised as GGML does and rounded to the activation dtype.
dial_status launch_kquant_gemm_sm100(const void* x, dial_dtype xdt, const void* blocks, int type,
                                     void* y, int64_t M, int64_t K, int64_t N, cudaStream_t st);

}  // namespace dial
