// Decoder stage: a run of Qwen3 / Llama decoder layers over the quantised
// linears, plus the greedy output head (C ABI in include/dial_cuda.h).
//
// Layer order (Transformer::forward text.rs:1636-1688, QwenAttention::forward
// text.rs:1478-1596, Mlp text.rs:816-829):
//   x1 = rms_1(h)                     (fused with the previous layer's MLP residual)
//   qkv = Wqkv x1 ; q,k = qk_norm ; rope ; k,v -> cache ; a = attention(q, cache)
//   o = Wo a ; h = h + o ; x2 = rms_2(h)          (one fused kernel)
//   gu = Wgate_up x2 ; m = silu(g) * u ; d = Wdown m ; h = h + d
// Every linear goes through the same launchers as dial_w8a16_linear /
// dial_gguf_linear (skinny tensor-core kernels for small T, tcgen05 GEMM for
// large T).  Nothing here allocates: scratch comes from the caller's workspace.
#include <algorithm>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "glue.cuh"
#include "layout.cuh"
#include "quant.cuh"

namespace dial {

namespace {

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

struct Ws {
  uint8_t* sk;      // stream-K scratch shared by every linear (zero counters between calls)
  int* actr;        // decode attention split counters (zero between calls)
  uint8_t* x1;      // [T, H]
  uint8_t* qkv;     // [T, (Hq+2Hkv)D]
  uint8_t* q;       // [T, Hq D]
  uint8_t* attn;    // [T, Hq D]
  uint8_t* delta;   // [T, H]  (o, then down output)
  uint8_t* h2;      // [T, H]  second residual buffer of the fused decode path
  uint8_t* gu;      // [T, 2I]
  uint8_t* mid;     // [T, I]
  uint8_t* attn_ws; // attention partials
  uint8_t* lin_ws;  // GGUF activation scratch
  uint8_t* logits;  // [T, V] for the head
  unsigned long long* keys;  // [T, ceil(V / 16)] per-tile greedy keys of the head
  size_t total;
};

Ws layout(const dial_decoder_dims& d, int64_t T, int64_t max_len, uint8_t* base) {
  const size_t e = d.act_dtype == DIAL_F32 ? 4 : 2;
  const int64_t H = d.hidden, I = d.intermediate, D = d.head_dim;
  const int64_t QKV = (int64_t)(d.n_heads + 2 * d.n_kv_heads) * D, QD = (int64_t)d.n_heads * D;
  Ws w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += al256(bytes);
    return p;
  };
  const int64_t nmax = std::max<int64_t>(std::max<int64_t>(QKV, 2 * I), std::max<int64_t>(H, d.vocab));
  w.sk = take(gemv_workspace_bytes(nmax));  // first, so its place does not depend on T
  w.actr = reinterpret_cast<int*>(take((size_t)d.n_heads * sizeof(int)));  // as fixed
  w.x1 = take(T * H * e);
  w.qkv = take(T * QKV * e);
  w.q = take(T * QD * e);
  w.attn = take(T * QD * e);
  w.delta = take(T * H * e);
  w.h2 = take(T * H * e);
  w.gu = take(T * 2 * I * e);
  w.mid = take(T * I * e);
  w.attn_ws = take(attention_workspace_bytes(T, d.n_heads, max_len));
  const int64_t kmax = std::max<int64_t>(std::max<int64_t>(H, I), QD);
  w.lin_ws = take(std::max(gguf_skinny_workspace_bytes(std::min<int64_t>(T, kSkinnyMaxM), kmax),
                           gemm_sm100_gguf_workspace_bytes(T, kmax)));
  w.logits = take(T * (int64_t)d.vocab * e);
  w.keys = reinterpret_cast<unsigned long long*>(take(T * ((d.vocab + 15) / 16) * 8));
  w.total = off;
  return w;
}

// One quantised linear y[T, N] = x[T, K] W^T in the stage's weight format.
// `pro` (W8A16 decode only, see fused_decode_ok) makes the GEMV compute its own
// input from x (rmsnorm / swiglu prologue).
dial_status linear(const dial_decoder_dims& d, int fmt, dial_linear_ref W, const void* x, void* y,
                   int64_t T, int64_t K, int64_t N, void* lin_ws, void* sk_ws, cudaStream_t st,
                   const ActPrologue* pro = nullptr) {
  const dial_dtype xdt = (dial_dtype)d.act_dtype;
  if (fmt == DIAL_WFMT_W8A16 || fmt == DIAL_WFMT_W8A16_F16S) {
    const dial_dtype sdt = fmt == DIAL_WFMT_W8A16 ? DIAL_F32 : DIAL_F16;
    if (pro)
      return launch_w8a16_skinny(x, xdt, static_cast<const int8_t*>(W.w), W.s, sdt, y, T, K, N, st,
                                 sk_ws, pro);
    if (T > kSkinnyMaxM && gemm_sm100_supported(T, K, N))
      return launch_w8a16_gemm_sm100(x, xdt, static_cast<const int8_t*>(W.w), W.s, sdt, y, T, K, N,
                                     st);
    for (int64_t m0 = 0; m0 < T; m0 += kSkinnyMaxM) {
      const int64_t mc = std::min<int64_t>(kSkinnyMaxM, T - m0);
      dial_status s = launch_w8a16_skinny(static_cast<const uint16_t*>(x) + m0 * K, xdt,
                                          static_cast<const int8_t*>(W.w), W.s, sdt,
                                          static_cast<uint16_t*>(y) + m0 * N, mc, K, N, st, sk_ws);
      if (s != DIAL_OK) return s;
    }
    return DIAL_OK;
  }
  const uint16_t* dd = static_cast<const uint16_t*>(W.s);
  if (gemm_sm100_supported(T, K, N))
    return launch_gguf_gemm_sm100(x, xdt, W.w, dd, fmt, y, T, K, N, lin_ws, st);
  const size_t e = xdt == DIAL_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < T; m0 += kSkinnyMaxM) {
    const int64_t mc = std::min<int64_t>(kSkinnyMaxM, T - m0);
    dial_status s = launch_gguf_skinny(static_cast<const uint8_t*>(x) + m0 * K * e, xdt, W.w, dd,
                                       fmt, static_cast<uint8_t*>(y) + m0 * N * e, mc, K, N,
                                       lin_ws, st, sk_ws);
    if (s != DIAL_OK) return s;
  }
  return DIAL_OK;
}

// Decode fast path: W8A16 layers and T rows small enough for the GEMV's staged
// prologue at every input width; rmsnorm and swiglu then run inside the GEMVs.
bool fused_decode_ok(const dial_decoder_dims& d, int64_t T) {
  const bool w8 = d.weight_format == DIAL_WFMT_W8A16 || d.weight_format == DIAL_WFMT_W8A16_F16S;
  const int64_t QD = (int64_t)d.n_heads * d.head_dim;
  return w8 && d.act_dtype != DIAL_F32 && T <= kSkinnyMaxM && w8a16_prologue_ok(T, d.hidden) &&
         w8a16_prologue_ok(T, d.intermediate) && w8a16_prologue_ok(T, QD);
}

dial_status check_dims(const dial_decoder_dims* d) {
  if (!d) return fail(DIAL_ERR_INVALID_ARG, "null dims");
  if (d->hidden <= 0 || d->intermediate <= 0 || d->vocab <= 0 || d->max_seq <= 0 || d->n_slots <= 0)
    return fail(DIAL_ERR_INVALID_ARG, "decoder dims must be positive");
  if (d->head_dim != 128) return fail(DIAL_ERR_SHAPE, "head_dim must be 128");
  if (d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads ||
      d->n_heads / d->n_kv_heads > 8)
    return fail(DIAL_ERR_SHAPE, "bad head counts");
  if (d->act_dtype != DIAL_F16 && d->act_dtype != DIAL_BF16)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "decoder activations must be f16 or bf16");
  auto fmt_ok = [](int f) {
    return f == DIAL_WFMT_W8A16 || f == DIAL_WFMT_W8A16_F16S || f == DIAL_WFMT_Q4_0 || f == DIAL_WFMT_Q8_0;
  };
  if (!fmt_ok(d->weight_format) || !fmt_ok(d->head_format))
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad weight format");
  const int mult = (d->weight_format == DIAL_WFMT_Q4_0 || d->weight_format == DIAL_WFMT_Q8_0) ? 32 : 16;
  if (d->hidden % mult || d->intermediate % mult)
    return fail(DIAL_ERR_SHAPE, "hidden/intermediate must be multiples of %d", mult);
  return DIAL_OK;
}

}  // namespace

}  // namespace dial

using namespace dial;

extern "C" {

size_t dial_decoder_workspace_bytes(const dial_decoder_dims* dims, int64_t tokens,
                                    int64_t max_len) {
  if (!dims || tokens <= 0 || max_len <= 0) return 0;
  return layout(*dims, tokens, max_len, nullptr).total;
}

dial_status dial_decoder_layers(const dial_decoder_dims* dims, const dial_layer_weights* layers,
                                int n_layers, void* hidden, const int32_t* positions,
                                const int32_t* slots, int64_t tokens, int64_t max_len,
                                const void* cos_t, const void* sin_t, void* workspace,
                                size_t workspace_bytes, dial_stream stream) {
  clear_error();
  dial_status s = check_dims(dims);
  if (s != DIAL_OK) return s;
  const dial_decoder_dims& d = *dims;
  if (!layers || n_layers <= 0 || !hidden || !positions || !slots || !cos_t || !sin_t || !workspace)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (tokens <= 0 || max_len <= 0 || max_len > d.max_seq)
    return fail(DIAL_ERR_INVALID_ARG, "need tokens > 0 and 0 < max_len <= max_seq");
  Ws w = layout(d, tokens, max_len, static_cast<uint8_t*>(workspace));
  if (workspace_bytes < w.total)
    return fail(DIAL_ERR_INVALID_ARG, "decoder workspace must hold %zu bytes", w.total);
  cudaStream_t st = as_stream(stream);
  const dial_dtype dt = (dial_dtype)d.act_dtype;
  const int64_t H = d.hidden, I = d.intermediate, D = d.head_dim, T = tokens;
  const int64_t QKV = (int64_t)(d.n_heads + 2 * d.n_kv_heads) * D, QD = (int64_t)d.n_heads * D;
  if (fused_decode_ok(d, T)) {
    // residual stream in two buffers: the rmsnorm prologue writes x + res to
    // the buffer that is not an input, so no GEMV CTA reads what another writes
    void* h_cur = hidden;
    void* h_buf[2] = {hidden, w.h2};
    for (int li = 0; li < n_layers; ++li) {
      const dial_layer_weights& L = layers[li];
      void* h_next = h_cur == h_buf[0] ? h_buf[1] : h_buf[0];
      const ActPrologue rms1{kProRms, li ? static_cast<const uint16_t*>(h_cur) : nullptr,
                             li ? static_cast<uint16_t*>(h_next) : nullptr,
                             static_cast<const uint16_t*>(L.input_norm), d.rms_eps};
      if ((s = linear(d, d.weight_format, L.qkv, li ? w.delta : h_cur, w.qkv, T, H, QKV, w.lin_ws, w.sk,
                      st, &rms1)) != DIAL_OK)
        return s;
      if (li) h_cur = h_next, h_next = h_cur == h_buf[0] ? h_buf[1] : h_buf[0];
      if (T == 1) {  // one sequence's next token: QK-norm, RoPE, append and attention in one launch
        if ((s = launch_attention_decode(w.qkv, L.q_norm, L.k_norm, cos_t, sin_t, positions, slots,
                                         L.k_cache, L.v_cache, w.attn, w.attn_ws, w.actr, dt, T,
                                         d.n_heads, d.n_kv_heads, d.max_seq, max_len, d.rms_eps,
                                         d.qk_norm, st)) != DIAL_OK)
          return s;
      } else {
        if ((s = launch_qk_rope_kv(w.qkv, L.q_norm, L.k_norm, cos_t, sin_t, positions, slots, w.q,
                                   L.k_cache, L.v_cache, dt, T, d.n_heads, d.n_kv_heads, d.max_seq,
                                   d.rms_eps, d.qk_norm, st)) != DIAL_OK)
          return s;
        if ((s = launch_attention(w.q, L.k_cache, L.v_cache, positions, slots, w.attn, w.attn_ws, dt,
                                  T, d.n_heads, d.n_kv_heads, d.max_seq, max_len, st)) != DIAL_OK)
          return s;
      }
      if ((s = linear(d, d.weight_format, L.o, w.attn, w.delta, T, QD, H, w.lin_ws, w.sk, st)) != DIAL_OK)
        return s;
      const ActPrologue rms2{kProRms, static_cast<const uint16_t*>(h_cur), static_cast<uint16_t*>(h_next),
                             static_cast<const uint16_t*>(L.post_norm), d.rms_eps};
      if ((s = linear(d, d.weight_format, L.gate_up, w.delta, w.gu, T, H, 2 * I, w.lin_ws, w.sk, st,
                      &rms2)) != DIAL_OK)
        return s;
      h_cur = h_next;
      const ActPrologue glu{kProSwiglu, nullptr, nullptr, nullptr, 0.0f};
      if ((s = linear(d, d.weight_format, L.down, w.gu, w.delta, T, I, H, w.lin_ws, w.sk, st, &glu)) !=
          DIAL_OK)
        return s;
    }
    return launch_add(hidden, h_cur, w.delta, dt, T * H, st);  // h = h + d of the last layer
  }
  for (int li = 0; li < n_layers; ++li) {
    const dial_layer_weights& L = layers[li];
    // x1 = rms_1(h + pending delta of the previous layer)
    if (li == 0) s = launch_rmsnorm(hidden, nullptr, nullptr, L.input_norm, w.x1, dt, T, H, d.rms_eps, st);
    else s = launch_rmsnorm(w.delta, hidden, hidden, L.input_norm, w.x1, dt, T, H, d.rms_eps, st);
    if (s != DIAL_OK) return s;
    if ((s = linear(d, d.weight_format, L.qkv, w.x1, w.qkv, T, H, QKV, w.lin_ws, w.sk, st)) != DIAL_OK) return s;
    if ((s = launch_qk_rope_kv(w.qkv, L.q_norm, L.k_norm, cos_t, sin_t, positions, slots, w.q,
                               L.k_cache, L.v_cache, dt, T, d.n_heads, d.n_kv_heads, d.max_seq,
                               d.rms_eps, d.qk_norm, st)) != DIAL_OK)
      return s;
    if ((s = launch_attention(w.q, L.k_cache, L.v_cache, positions, slots, w.attn, w.attn_ws, dt, T,
                              d.n_heads, d.n_kv_heads, d.max_seq, max_len, st)) != DIAL_OK)
      return s;
    if ((s = linear(d, d.weight_format, L.o, w.attn, w.delta, T, QD, H, w.lin_ws, w.sk, st)) != DIAL_OK) return s;
    // h = h + o ; x2 = rms_2(h)
    if ((s = launch_rmsnorm(w.delta, hidden, hidden, L.post_norm, w.x1, dt, T, H, d.rms_eps, st)) != DIAL_OK)
      return s;
    if ((s = linear(d, d.weight_format, L.gate_up, w.x1, w.gu, T, H, 2 * I, w.lin_ws, w.sk, st)) != DIAL_OK) return s;
    if ((s = launch_swiglu(w.gu, w.mid, dt, T, I, st)) != DIAL_OK) return s;
    if ((s = linear(d, d.weight_format, L.down, w.mid, w.delta, T, I, H, w.lin_ws, w.sk, st)) != DIAL_OK) return s;
  }
  return launch_add(hidden, hidden, w.delta, dt, T * H, st);  // h = h + d of the last layer
}

namespace {

// The head over vocabulary rows [v0, v0 + n) (the full head: v0 = 0, n = vocab):
// y = head(rmsnorm(hidden[rows])) into lg, and per row either the index of
// its maximum (ids) or its greedy key (keys, indices from v0).  The W8A16
// decode GEMV writes each tile's key in its epilogue (one small reduction
// follows); other paths take argmax over the logits.
dial_status head_rows(const dial_decoder_dims& d, const void* final_norm, dial_linear_ref head,
                      int64_t v0, int64_t n, const void* hidden, const int32_t* row_index,
                      int64_t rows, int32_t* ids, unsigned long long* keys, void* logits,
                      const Ws& w, cudaStream_t st) {
  dial_status s;
  const dial_dtype dt = (dial_dtype)d.act_dtype;
  const int64_t H = d.hidden, tiles = (n + 15) / 16;
  void* lg = logits ? logits : w.logits;
  const bool w8head = d.head_format == DIAL_WFMT_W8A16 || d.head_format == DIAL_WFMT_W8A16_F16S;
  if (!row_index && w8head && d.act_dtype != DIAL_F32 && rows <= kSkinnyMaxM && w8a16_prologue_ok(rows, H)) {
    const ActPrologue fin{kProRms, nullptr, nullptr, static_cast<const uint16_t*>(final_norm), d.rms_eps};
    const dial_dtype sdt = d.head_format == DIAL_WFMT_W8A16 ? DIAL_F32 : DIAL_F16;
    bool keyed = false;
    if ((s = launch_w8a16_skinny(hidden, dt, static_cast<const int8_t*>(head.w), head.s, sdt, lg, rows,
                                 H, n, st, w.sk, &fin, w.keys, v0, &keyed)) != DIAL_OK)
      return s;
    if (keyed) return launch_key_reduce(w.keys, tiles, 1, tiles, rows, keys, ids, st);
  } else {
    const void* src = hidden;
    if (row_index) {
      if ((s = launch_gather_rows(hidden, row_index, w.delta, dt, rows, H, st)) != DIAL_OK) return s;
      src = w.delta;
    }
    if ((s = launch_rmsnorm(src, nullptr, nullptr, final_norm, w.x1, dt, rows, H, d.rms_eps, st)) != DIAL_OK)
      return s;
    if ((s = linear(d, d.head_format, head, w.x1, lg, rows, H, n, w.lin_ws, w.sk, st)) != DIAL_OK) return s;
  }
  if (keys) return launch_argmax_keys(lg, keys, dt, rows, n, v0, st);
  return launch_argmax(lg, ids, dt, rows, n, st);
}

}  // namespace

dial_status dial_decoder_head(const dial_decoder_dims* dims, const void* final_norm,
                              dial_linear_ref head, const void* hidden, const int32_t* row_index,
                              int64_t rows, int32_t* out_ids, void* logits, void* workspace,
                              size_t workspace_bytes, dial_stream stream) {
  clear_error();
  dial_status s = check_dims(dims);
  if (s != DIAL_OK) return s;
  const dial_decoder_dims& d = *dims;
  if (!final_norm || !head.w || !head.s || !hidden || !out_ids || !workspace)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (rows <= 0) return fail(DIAL_ERR_INVALID_ARG, "rows must be positive");
  Ws w = layout(d, rows, 1, static_cast<uint8_t*>(workspace));
  if (workspace_bytes < w.total)
    return fail(DIAL_ERR_INVALID_ARG, "head workspace must hold %zu bytes", w.total);
  return head_rows(d, final_norm, head, 0, d.vocab, hidden, row_index, rows, out_ids, nullptr, logits,
                   w, as_stream(stream));
}

dial_status dial_decoder_head_shard(const dial_decoder_dims* dims, const void* final_norm,
                                    dial_linear_ref head_shard, int64_t vocab_offset,
                                    int64_t shard_rows, const void* hidden, const int32_t* row_index,
                                    int64_t rows, uint64_t* out_keys, void* logits, void* workspace,
                                    size_t workspace_bytes, dial_stream stream) {
  clear_error();
  dial_status s = check_dims(dims);
  if (s != DIAL_OK) return s;
  const dial_decoder_dims& d = *dims;
  if (!final_norm || !head_shard.w || !head_shard.s || !hidden || !out_keys || !workspace)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (rows <= 0) return fail(DIAL_ERR_INVALID_ARG, "rows must be positive");
  if (vocab_offset < 0 || shard_rows <= 0 || vocab_offset + shard_rows > d.vocab)
    return fail(DIAL_ERR_INVALID_ARG, "shard rows [%lld, %lld) outside the vocabulary of %lld",
                (long long)vocab_offset, (long long)(vocab_offset + shard_rows), (long long)d.vocab);
  Ws w = layout(d, rows, 1, static_cast<uint8_t*>(workspace));
  if (workspace_bytes < w.total)
    return fail(DIAL_ERR_INVALID_ARG, "head workspace must hold %zu bytes", w.total);
  return head_rows(d, final_norm, head_shard, vocab_offset, shard_rows, hidden, row_index, rows, nullptr,
                   reinterpret_cast<unsigned long long*>(out_keys), logits, w, as_stream(stream));
}

dial_status dial_head_merge(const uint64_t* keys, int n_shards, int64_t rows, int32_t* out_ids,
                            dial_stream stream) {
  clear_error();
  if (!keys || !out_ids) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (n_shards <= 0 || rows <= 0) return fail(DIAL_ERR_INVALID_ARG, "n_shards and rows must be positive");
  return launch_key_reduce(reinterpret_cast<const unsigned long long*>(keys), n_shards, rows, 1, rows,
                           nullptr, out_ids, as_stream(stream));
}

}  // extern "C"
