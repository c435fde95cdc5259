// extern "C" entry points for the decoder glue (include/dial_cuda.h).
#include "common.cuh"
#include "glue.cuh"

using namespace dial;

namespace {

bool is_act(dial_dtype t) { return t == DIAL_F32 || t == DIAL_F16 || t == DIAL_BF16; }

dial_status check_heads(int hq, int hkv, int head_dim) {
  if (head_dim != 128) return fail(DIAL_ERR_SHAPE, "head_dim must be 128 (got %d)", head_dim);
  if (hq <= 0 || hkv <= 0 || hq % hkv || hq / hkv > 8)
    return fail(DIAL_ERR_SHAPE, "heads must satisfy Hq %% Hkv == 0 and Hq/Hkv <= 8 (%d, %d)", hq, hkv);
  return DIAL_OK;
}

}  // namespace

extern "C" {

dial_status dial_rmsnorm(const void* x, const void* residual, void* h_out, const void* w, void* y,
                         dial_dtype dt, int64_t rows, int64_t dim, float eps, dial_stream stream) {
  clear_error();
  if (!x || !w || !y) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (rows <= 0 || dim <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (!is_act(dt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad dtype");
  return launch_rmsnorm(x, residual, h_out, w, y, dt, rows, dim, eps, as_stream(stream));
}

dial_status dial_rope_tables(void* cos_t, void* sin_t, dial_dtype dt, int64_t max_pos,
                             int head_dim, float theta, dial_stream stream) {
  clear_error();
  if (!cos_t || !sin_t) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (max_pos <= 0 || head_dim <= 0 || head_dim % 2)
    return fail(DIAL_ERR_INVALID_ARG, "bad sizes");
  if (!is_act(dt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad dtype");
  return launch_rope_tables(cos_t, sin_t, dt, max_pos, head_dim, theta, as_stream(stream));
}

dial_status dial_qk_norm_rope_kv_append(const void* qkv, const void* q_norm_w,
                                        const void* k_norm_w, const void* cos_t,
                                        const void* sin_t, const int32_t* positions,
                                        const int32_t* slots, void* q_out, void* k_cache,
                                        void* v_cache, dial_dtype dt, int64_t tokens, int n_heads,
                                        int n_kv_heads, int head_dim, int64_t max_seq, float eps,
                                        int qk_norm, dial_stream stream) {
  clear_error();
  if (!qkv || !cos_t || !sin_t || !positions || !slots || !q_out || !k_cache || !v_cache)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (qk_norm && (!q_norm_w || !k_norm_w)) return fail(DIAL_ERR_INVALID_ARG, "null norm weight");
  if (tokens <= 0 || max_seq <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (dt != DIAL_F16 && dt != DIAL_BF16) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "f16/bf16 only");
  dial_status s = check_heads(n_heads, n_kv_heads, head_dim);
  if (s != DIAL_OK) return s;
  return launch_qk_rope_kv(qkv, q_norm_w, k_norm_w, cos_t, sin_t, positions, slots, q_out, k_cache,
                           v_cache, dt, tokens, n_heads, n_kv_heads, max_seq, eps, qk_norm,
                           as_stream(stream));
}

size_t dial_attention_workspace_bytes(int64_t tokens, int n_heads, int64_t max_len) {
  if (tokens <= 0 || n_heads <= 0 || max_len <= 0) return 0;
  return attention_workspace_bytes(tokens, n_heads, max_len);
}

dial_status dial_attention(const void* q, const void* k_cache, const void* v_cache,
                           const int32_t* positions, const int32_t* slots, void* out,
                           void* workspace, size_t workspace_bytes, dial_dtype dt, int64_t tokens,
                           int n_heads, int n_kv_heads, int head_dim, int64_t max_seq,
                           int64_t max_len, dial_stream stream) {
  clear_error();
  if (!q || !k_cache || !v_cache || !positions || !slots || !out)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (tokens <= 0 || max_seq <= 0 || max_len <= 0 || max_len > max_seq)
    return fail(DIAL_ERR_INVALID_ARG, "bad sizes (need 0 < max_len <= max_seq)");
  if (dt != DIAL_F16 && dt != DIAL_BF16) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "f16/bf16 only");
  dial_status s = check_heads(n_heads, n_kv_heads, head_dim);
  if (s != DIAL_OK) return s;
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(DIAL_ERR_MISALIGNED, "caches must be 16-byte aligned");
  const size_t need = attention_workspace_bytes(tokens, n_heads, max_len);
  if (need && (!workspace || workspace_bytes < need))
    return fail(DIAL_ERR_INVALID_ARG, "attention workspace must hold %zu bytes", need);
  return launch_attention(q, k_cache, v_cache, positions, slots, out, workspace, dt, tokens,
                          n_heads, n_kv_heads, max_seq, max_len, as_stream(stream));
}

size_t dial_decode_attention_workspace_bytes(int n_heads, int64_t max_len) {
  if (n_heads <= 0 || max_len <= 0) return 0;
  return attention_decode_workspace_bytes(n_heads, max_len);
}

dial_status dial_decode_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                  const void* cos_t, const void* sin_t, const int32_t* positions,
                                  const int32_t* slots, void* k_cache, void* v_cache, void* out,
                                  void* workspace, size_t workspace_bytes, dial_dtype dt,
                                  int n_heads, int n_kv_heads, int head_dim, int64_t max_seq,
                                  int64_t max_len, float eps, int qk_norm, dial_stream stream) {
  clear_error();
  if (!qkv || !cos_t || !sin_t || !positions || !slots || !k_cache || !v_cache || !out || !workspace)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (qk_norm && (!q_norm_w || !k_norm_w)) return fail(DIAL_ERR_INVALID_ARG, "null norm weight");
  if (max_seq <= 0 || max_len <= 0 || max_len > max_seq)
    return fail(DIAL_ERR_INVALID_ARG, "bad sizes (need 0 < max_len <= max_seq)");
  if (dt != DIAL_F16 && dt != DIAL_BF16) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "f16/bf16 only");
  dial_status s = check_heads(n_heads, n_kv_heads, head_dim);
  if (s != DIAL_OK) return s;
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(DIAL_ERR_MISALIGNED, "caches must be 16-byte aligned");
  const size_t need = attention_decode_workspace_bytes(n_heads, max_len);
  if (workspace_bytes < need)
    return fail(DIAL_ERR_INVALID_ARG, "decode attention workspace must hold %zu bytes", need);
  if (!aligned16(workspace)) return fail(DIAL_ERR_MISALIGNED, "workspace must be 16-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* ctr = reinterpret_cast<int*>(ws + need - (size_t)n_heads * sizeof(int));
  return launch_attention_decode(qkv, q_norm_w, k_norm_w, cos_t, sin_t, positions, slots, k_cache,
                                 v_cache, out, ws, ctr, dt, 1, n_heads, n_kv_heads, max_seq,
                                 max_len, eps, qk_norm, as_stream(stream));
}

dial_status dial_swiglu(const void* gate_up, void* out, dial_dtype dt, int64_t tokens,
                        int64_t intermediate, dial_stream stream) {
  clear_error();
  if (!gate_up || !out) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (tokens <= 0 || intermediate <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (!is_act(dt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad dtype");
  return launch_swiglu(gate_up, out, dt, tokens, intermediate, as_stream(stream));
}

dial_status dial_embedding(const void* table, const int32_t* ids, void* out, dial_dtype dt,
                           int64_t tokens, int64_t vocab, int64_t dim, dial_stream stream) {
  clear_error();
  if (!table || !ids || !out) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (tokens <= 0 || vocab <= 0 || dim <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (!is_act(dt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad dtype");
  return launch_embedding(table, ids, out, dt, tokens, vocab, dim, as_stream(stream));
}

dial_status dial_argmax(const void* x, int32_t* out, dial_dtype dt, int64_t rows, int64_t n,
                        dial_stream stream) {
  clear_error();
  if (!x || !out) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (rows <= 0 || n <= 0 || n > (1ll << 31) - 1) return fail(DIAL_ERR_INVALID_ARG, "bad sizes");
  if (!is_act(dt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad dtype");
  return launch_argmax(x, out, dt, rows, n, as_stream(stream));
}

}  // extern "C"
