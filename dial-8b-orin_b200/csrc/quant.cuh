// Launchers implemented in quant.cu, skinny.cu and gemm_sm100.cu.
#pragma once

#include "common.cuh"

namespace dial {

dial_status launch_w8a16_quantize(const void* w, dial_dtype wdt, int64_t N, int64_t K, int8_t* q,
                                  void* scale, dial_dtype sdt, cudaStream_t st);
dial_status launch_w8a16_dequantize(const int8_t* q, const void* scale, dial_dtype sdt, int64_t N,
                                    int64_t K, void* w, dial_dtype wdt, cudaStream_t st);
dial_status launch_gguf_repack(const void* blocks, int type, int64_t N, int64_t K, void* qs,
                               uint16_t* d, cudaStream_t st);
dial_status launch_gguf_unpack(const void* qs, const uint16_t* d, int type, int64_t N, int64_t K,
                               void* blocks, cudaStream_t st);
dial_status launch_gguf_quantize(const float* w, int type, int64_t N, int64_t K, void* qs,
                                 uint16_t* d, cudaStream_t st);
dial_status launch_gguf_dequantize(const void* qs, const uint16_t* d, int type, int64_t N,
                                   int64_t K, void* w, dial_dtype wdt, cudaStream_t st);

// Skinny (small-M) dequant tensor-core kernels, skinny.cu.
constexpr int kSkinnyMaxM = 32;
// GEMV scratch (partial-chunk slots, chunk and per-tile counters) for M-row
// (M <= 32) passes over N output rows, any K.  The counter part must be zero
// before the first call; every call leaves it zero.  sk_ws == NULL selects the
// in-CTA K split instead (no scratch).
size_t gemv_workspace_bytes(int64_t N);

// Decode-path prologue of the W8A16 GEMV: its activation staging computes the
// linear's input instead of reading it (the separate rmsnorm / swiglu kernels
// then need not run).  kProRms: input = rmsnorm(x + res) * w, and x + res
// (rounded) is written to h_out, which must not alias x or res.  kProSwiglu:
// x is gate_up [M, 2K] and input = swiglu(gate, up).  Needs the staged path
// (M * K * 2 <= 32 KiB, a workspace, 16-byte aligned pointers).
enum { kProX = 0, kProRms = 1, kProSwiglu = 2 };
struct ActPrologue {
  int mode;
  const uint16_t* res;
  uint16_t* h_out;
  const uint16_t* w;
  float eps;
};
bool w8a16_prologue_ok(int64_t M, int64_t K);

// keys (optional): the whole-tile decode GEMV then also writes each tile's
// greedy key per token (argmax_key of the rounded outputs, rows numbered from
// key_off) to keys[token * ceil(N / 16) + tile], and *keyed reports whether it
// did (other paths leave that to the caller); y may then be NULL.
dial_status launch_w8a16_skinny(const void* x, dial_dtype xdt, const int8_t* q, const void* scale,
                                dial_dtype sdt, void* y, int64_t M, int64_t K, int64_t N,
                                cudaStream_t st, void* sk_ws, const ActPrologue* pro = nullptr,
                                unsigned long long* keys = nullptr, int64_t key_off = 0,
                                bool* keyed = nullptr);
// Q4_K decode GEMV on tensor cores (M <= 8 tokens, f16/bf16 activations, K a
// multiple of 256 with at least 8 super-blocks, 16-byte aligned x and blocks).
bool kq4_gemv_ok(int64_t M, int64_t K, int64_t N, dial_dtype xdt, const void* x, const void* blocks);
dial_status launch_kq4_gemv(const void* x, dial_dtype xdt, const void* blocks, void* y, int64_t M,
                            int64_t K, int64_t N, cudaStream_t st);
// Q6_K decode GEMV on tensor cores (as the Q4_K one; K a multiple of 2048, so
// that a row of 210-byte super-blocks is a 16-byte multiple).
bool kq6_gemv_ok(int64_t M, int64_t K, int64_t N, dial_dtype xdt, const void* x, const void* blocks);
dial_status launch_kq6_gemv(const void* x, dial_dtype xdt, const void* blocks, void* y, int64_t M,
                            int64_t K, int64_t N, cudaStream_t st);
// GGUF integer path: activations quantised to Q8_0 in `ws` first.
size_t gguf_skinny_workspace_bytes(int64_t M, int64_t K);
dial_status launch_gguf_skinny(const void* x, dial_dtype xdt, const void* qs, const uint16_t* d,
                               int type, void* y, int64_t M, int64_t K, int64_t N, void* ws,
                               cudaStream_t st, void* sk_ws);

}  // namespace dial
