// Launchers of the decoder glue kernels (glue.cu).
#pragma once

#include "common.cuh"

namespace dial {

// Device flag that kernels set on a detected error (bounded wait expired,
// out-of-range token id); defined in gemm_sm100.cu.
int* device_error_ptr();

dial_status launch_rmsnorm(const void* x, const void* res, void* h_out, const void* w, void* y,
                           dial_dtype dt, int64_t rows, int64_t dim, float eps, cudaStream_t st);
dial_status launch_qk_rope_kv(const void* qkv, const void* qn, const void* kn, const void* cos_t,
                              const void* sin_t, const int32_t* pos, const int32_t* slot,
                              void* q_out, void* kc, void* vc, dial_dtype dt, int64_t tokens,
                              int hq, int hkv, int64_t max_seq, float eps, int qk_norm,
                              cudaStream_t st);
size_t attention_workspace_bytes(int64_t tokens, int hq, int64_t max_len);
dial_status launch_attention(const void* q, const void* kc, const void* vc, const int32_t* pos,
                             const int32_t* slot, void* out, void* ws, dial_dtype dt,
                             int64_t tokens, int hq, int hkv, int64_t max_seq, int64_t max_len,
                             cudaStream_t st);
// Decode attention for one token (tokens == 1): QK-norm + RoPE of the raw
// qkv row, the K/V cache append and the attention in one launch (the
// arithmetic of launch_qk_rope_kv followed by launch_attention).  `ws` holds
// the split partials (attention_workspace_bytes(1, hq, max_len)); `ctr` hkv
// ints, zero before the launch and zero again after it.
size_t attention_decode_workspace_bytes(int hq, int64_t max_len);
dial_status launch_attention_decode(const void* qkv, const void* qn, const void* kn,
                                    const void* cos_t, const void* sin_t, const int32_t* pos,
                                    const int32_t* slot, void* kc, void* vc, void* out, void* ws,
                                    int* ctr, dial_dtype dt, int64_t tokens, int hq, int hkv,
                                    int64_t max_seq, int64_t max_len, float eps, int qk_norm,
                                    cudaStream_t st);
dial_status launch_swiglu(const void* gu, void* out, dial_dtype dt, int64_t tokens, int64_t inter,
                          cudaStream_t st);
dial_status launch_gather_rows(const void* src, const int32_t* idx, void* dst, dial_dtype dt,
                               int64_t rows, int64_t dim, cudaStream_t st);
// out = round(a + b) elementwise; out may alias a.
dial_status launch_add(void* out, const void* a, const void* b, dial_dtype dt, int64_t n,
                       cudaStream_t st);
dial_status launch_embedding(const void* table, const int32_t* ids, void* out, dial_dtype dt,
                             int64_t tokens, int64_t vocab, int64_t dim, cudaStream_t st);
dial_status launch_argmax(const void* x, int32_t* out, dial_dtype dt, int64_t rows, int64_t n,
                          cudaStream_t st);
// keys[r] = the greedy key (argmax_key) of row r of x [rows, n], indices from offset.
dial_status launch_argmax_keys(const void* x, unsigned long long* keys, dial_dtype dt, int64_t rows,
                               int64_t n, int64_t offset, cudaStream_t st);
// Per row r: the largest of keys[r * row_stride + i * elem_stride], i < n, into
// keys_out[r] and/or its index into ids[r] (either may be NULL).
dial_status launch_key_reduce(const unsigned long long* keys, int64_t n, int64_t elem_stride,
                              int64_t row_stride, int64_t rows, unsigned long long* keys_out,
                              int32_t* ids, cudaStream_t st);
dial_status launch_rope_tables(void* cos_t, void* sin_t, dial_dtype dt, int64_t max_pos,
                               int head_dim, float theta, cudaStream_t st);

}  // namespace dial
