/*
 * dial_cuda.h -- C ABI of the B200 (sm_100a) quantized-linear hot path of DIAL.
 *
 * Plain pointers and sizes only.  All tensor pointers are DEVICE pointers
 * unless a comment says otherwise; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  No entry point allocates device memory: outputs and
 * workspaces come from the caller, which matches the reference's ownership
 * (the linear owns its device weights, activations are borrowed and
 * contiguous, the output is allocated by the caller side).
 *
 * Every entry point returns a dial_status and never throws or aborts across
 * the boundary; `dial_last_error()` gives a thread-local message for the last
 * failure on the calling thread.  Launch errors are checked right after each
 * launch.
 *
 * Reference interfaces replaced (paths inside lisa301/DIAL-8B-orin):
 *   TextLinear::{from_dense, forward}          dial-core/src/models/qwen3_vl/worker_w8a16.rs:65-121
 *   CudaW8A16Linear::{from_linear, forward}     worker_w8a16.rs:301-386
 *   CustomOp1::cuda_fwd (NVRTC kernels)         worker_w8a16.rs:402-475 (kernels :146-224)
 *   load_worker_gguf_linear / forward_worker_gguf
 *                                               dial-core/src/models/qwen3_vl/worker_gguf.rs:462-522, :574-611
 *   QTensor::dequantize / dequantize_f16        worker_gguf.rs:56-63, worker_w8a16.rs:123-128
 */
#ifndef DIAL_CUDA_H_
#define DIAL_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DIAL_ABI_VERSION 1

#if defined(__GNUC__)
#define DIAL_API __attribute__((visibility("default")))
#else
#define DIAL_API
#endif

typedef int dial_status;
enum {
  DIAL_OK = 0,
  DIAL_ERR_INVALID_ARG = 1,       /* null pointer, non-positive size, bad enum */
  DIAL_ERR_UNSUPPORTED_DTYPE = 2, /* dtype combination the op does not support */
  DIAL_ERR_MISALIGNED = 3,        /* pointer or row stride breaks the 16-byte rule */
  DIAL_ERR_SHAPE = 4,             /* K not a multiple of the block / vector width */
  DIAL_ERR_CUDA = 5,              /* CUDA runtime error (message in dial_last_error) */
  DIAL_ERR_NCCL = 6,              /* NCCL error in the stage pipe */
  DIAL_ERR_TIMEOUT = 7,           /* bounded wait ran out (device flag or host deadline) */
  DIAL_ERR_NO_DEVICE = 8          /* no sm_100 device visible */
};

typedef enum { DIAL_F32 = 0, DIAL_F16 = 1, DIAL_BF16 = 2 } dial_dtype;

/* GGML type codes, as in the GGUF file format. */
typedef enum {
  DIAL_GGML_Q4_0 = 2,
  DIAL_GGML_Q8_0 = 8,
  DIAL_GGML_Q4_K = 12, /* dial_gguf_k_* only */
  DIAL_GGML_Q6_K = 14  /* dial_gguf_k_* only */
} dial_ggml_type;

typedef void* dial_stream; /* cudaStream_t */

/* ------------------------------------------------------------------ misc */
DIAL_API const char* dial_status_string(dial_status s);
/* Thread-local description of the last failure on this thread ("" if none). */
DIAL_API const char* dial_last_error(void);
DIAL_API int dial_abi_version(void);
/* Number of kernels launched by this library in this process (all threads). */
DIAL_API uint64_t dial_launch_count(void);
/* Synchronising check of the device error flag that kernels with bounded
 * waits set when a wait expires (DIAL_ERR_TIMEOUT); `clear` resets it. */
DIAL_API dial_status dial_device_error(int clear);

/* Self-test of the bounded-wait error path (no reference counterpart): one
 * CTA starts a 256-byte bulk copy from `src` (device, 16-byte aligned) into
 * shared memory, waits on an mbarrier that nothing signals until the wait
 * limit (1 s) expires -- which records DIAL_ERR_TIMEOUT in the device error
 * flag -- then drains the copy and writes result[0..2] (device int[3]):
 * {wait succeeded (0 expected), copy drained (1), word 12 of src as read}.
 * Clear the flag with dial_device_error(1) before and after. */
DIAL_API dial_status dial_check_bounded_wait(const void* src, int* result, dial_stream stream);

/* ------------------------------------------------------------------ W8A16
 * Layout: q int8 [N, K] row-major (K contiguous), scale [N] (f32 as in the
 * reference, or f16).  K must be a multiple of 16 and q 16-byte aligned.
 */

/* Per-output-row symmetric quantiser, bit-exact with worker_w8a16.rs:322-341:
 * scale = absmax/127 (1.0 for an all-zero row), q = clamp(round(w * (1/scale)),
 * -127, 127) with round-half-away-from-zero.  w is [N, K] f32 or f16 (f16 is
 * widened to f32 first, as the reference does).  With sdt == DIAL_F16 the int8
 * values are those of the f32 scale and the stored scale is its f16 rounding. */
DIAL_API dial_status dial_w8a16_quantize(const void* w, dial_dtype wdt, int64_t N, int64_t K, int8_t* q,
                                void* scale, dial_dtype sdt, dial_stream stream);

/* w[n, k] = q[n, k] * scale[n], one f32 rounding, then converted to wdt. */
DIAL_API dial_status dial_w8a16_dequantize(const int8_t* q, const void* scale, dial_dtype sdt, int64_t N,
                                  int64_t K, void* w, dial_dtype wdt, dial_stream stream);

/* y[m, n] = round_ydt( (sum_k f32(q[n,k]) * f32(x[m,k])) * scale[n] ), f32
 * accumulation (worker_w8a16.rs:158-181).  x is [M, K] f16 or bf16, y is
 * [M, N] in the same dtype (the reference is f16 in / f16 out).  Any M >= 1;
 * the kernel is picked by M (decode GEMV, small-M tensor-core tile, or the
 * tcgen05 dequant-GEMM).
 * `workspace` (optional, dial_w8a16_linear_workspace_bytes(N) bytes, about
 * 10 MiB on a 148-SM B200, 16-byte aligned) lets the small-M kernel give every
 * warp of the GPU an equal share of the weight bytes (stream-K); it must be
 * zero-filled before its first use and every call leaves it zero-filled (a
 * call that reported a device error may not: zero it again).  Calls that share
 * a workspace must not overlap on the GPU.  One workspace sized for the largest
 * N serves every linear.  NULL: no workspace (same results, slower small M). */
DIAL_API size_t dial_w8a16_linear_workspace_bytes(int64_t N);
DIAL_API dial_status dial_w8a16_linear(const void* x, dial_dtype xdt, const int8_t* q, const void* scale,
                              dial_dtype sdt, void* y, int64_t M, int64_t K, int64_t N,
                              void* workspace, size_t workspace_bytes, dial_stream stream);

/* ------------------------------------------------------------------ GGUF
 * Native block layout (what a GGUF file holds and candle uploads):
 *   Q4_0: 18-byte blocks {f16 d; u8 qs[16]} per 32 weights, element j in the
 *         low nibble of qs[j], element j+16 in the high nibble;
 *   Q8_0: 34-byte blocks {f16 d; i8 qs[32]}.
 * Blocks are row-major over [N, K/32].  On the device the linear keeps a
 * split layout made once at load by dial_gguf_repack, in groups of 4 blocks
 * (G = ceil(K/128) groups per row, missing blocks zero-padded):
 *   d  : f16 [ceil(N/16), G, 16, 4]        (dial_gguf_d_bytes): the scales of
 *        one 16-row x 4-block unit are 128 contiguous bytes; rows past N are
 *        padding (allocate the array zero-filled)
 *   qs : u8  [N, G*64] (Q4_0) or [N, G*128] (Q8_0)   (dial_gguf_qs_bytes)
 * with the bytes of a group interleaved so that each 16-byte load is one
 * lane's slice of an int8 tensor-core fragment (dial-8b-orin_b200/csrc/layout.cuh
 * gives the byte map).  Values and scales are unchanged, so dequantised
 * weights stay bit-exact.  K must be a multiple of 32.
 */
DIAL_API size_t dial_gguf_qs_bytes(dial_ggml_type type, int64_t N, int64_t K);
DIAL_API size_t dial_gguf_d_bytes(int64_t N, int64_t K);

/* Native blocks -> split (qs, d) device layout.  `blocks` is a device pointer. */
DIAL_API dial_status dial_gguf_repack(const void* blocks, dial_ggml_type type, int64_t N, int64_t K,
                             void* qs, uint16_t* d, dial_stream stream);

/* Split layout -> native blocks (inverse of dial_gguf_repack). */
DIAL_API dial_status dial_gguf_unpack(const void* qs, const uint16_t* d, dial_ggml_type type, int64_t N,
                             int64_t K, void* blocks, dial_stream stream);

/* GGML reference quantiser (quantize_row_q4_0_ref / quantize_row_q8_0_ref,
 * which candle's QTensor::quantize restates), w [N, K] f32 -> split layout. */
DIAL_API dial_status dial_gguf_quantize(const float* w, dial_ggml_type type, int64_t N, int64_t K,
                               void* qs, uint16_t* d, dial_stream stream);

/* w[n, k] = f32(d) * q, bit-exact with GGML dequantize_row_*, then to wdt. */
DIAL_API dial_status dial_gguf_dequantize(const void* qs, const uint16_t* d, dial_ggml_type type,
                                 int64_t N, int64_t K, void* w, dial_dtype wdt,
                                 dial_stream stream);

/* y = x . deq(W)^T.  x [M, K] f32/f16/bf16, y [M, N] in the same dtype
 * (forward_worker_gguf keeps the activation dtype, worker_gguf.rs:589-605).
 * Small M (<= 32 rows per pass): activations are quantised to Q8_0 blocks and
 * every block is an exact integer dot scaled in f32 (candle's CPU QMatMul
 * arithmetic).  Larger M: weights are dequantised to f16/bf16 tiles feeding
 * tensor-core MMAs with f32 accumulation.  K % 32 == 0.  `workspace` must hold
 * dial_gguf_linear_workspace_bytes(M, K, N) bytes, 16-byte aligned, zero-filled
 * before its first use (every call leaves its counters zero again, unless it
 * reported a device error); calls that share a workspace must not overlap on
 * the GPU. */
DIAL_API size_t dial_gguf_linear_workspace_bytes(int64_t M, int64_t K, int64_t N);
DIAL_API dial_status dial_gguf_linear(const void* x, dial_dtype xdt, const void* qs, const uint16_t* d,
                             dial_ggml_type type, void* y, int64_t M, int64_t K, int64_t N,
                             void* workspace, size_t workspace_bytes, dial_stream stream);

/* The same GGUF linear (integer path: activations quantised to Q8_0, exact
 * block dots) for callers that cannot allocate device memory when they run it
 * -- e.g. a worker loop whose allocator is not re-entrant, or an FFI caller
 * with no device allocator.  No counterpart in the reference: its scratch
 * lives in a fixed 640 KiB __device__ array inside this library instead of a
 * caller workspace, so the call allocates nothing.  K <= 16384 (larger K
 * returns DIAL_ERR_SHAPE); any M, 32 rows per pass, on the in-CTA K-split GEMV
 * (plain loads; not the TMA stream-K kernel of dial_gguf_linear, which needs
 * the workspace; speed not tuned).  The first call on a device looks up the
 * array's address (make it before any stream capture); after cudaDeviceReset
 * the next call looks it up again.  All calls share the array: calls that
 * overlap on the GPU race on it, so order them on one stream. */
DIAL_API dial_status dial_gguf_linear_noalloc(const void* x, dial_dtype xdt, const void* qs,
                                              const uint16_t* d, dial_ggml_type type, void* y,
                                              int64_t M, int64_t K, int64_t N, dial_stream stream);

/* ------------------------------------------------------------------ GGUF K-quants
 * Q4_K and Q6_K super-blocks of 256 weights in their native GGML layout, as a
 * GGUF file holds them and candle's QMatMul loads them (load_worker_gguf_linear,
 * worker_gguf.rs:462-522; the reference's deployed files are Q4_K_M):
 *   Q4_K: 144 bytes {f16 d; f16 dmin; u8 scales[12] (6-bit scale and min of each
 *         32-weight sub-block); u8 qs[128] (4-bit)};  value = d*sc*q - dmin*m
 *   Q6_K: 210 bytes {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d};
 *         value = d*scale*(q - 32), q 6-bit
 * Blocks are row-major over [N, K/256]; K must be a multiple of 256.  Q4_K
 * blocks must be 16-byte aligned, Q6_K blocks 2-byte aligned.  Unlike Q4_0 and
 * Q8_0 there is no repacked device layout: the kernels read the file's blocks.
 */
/* Bytes of one row of K weights (0 for a bad type or K). */
DIAL_API size_t dial_gguf_k_row_bytes(dial_ggml_type type, int64_t K);

/* w[n, k] in wdt: the GGML reference dequantisers' f32 values bit for bit
 * (each product and the Q4_K difference rounded on its own), then to wdt. */
DIAL_API dial_status dial_gguf_k_dequantize(const void* blocks, dial_ggml_type type, int64_t N,
                                            int64_t K, void* w, dial_dtype wdt, dial_stream stream);

/* y = x . deq(W)^T for decode-sized M: x [M, K] f32/f16/bf16 (16-byte aligned),
 * y [M, N] in the same dtype (forward_worker_gguf keeps the activation dtype,
 * worker_gguf.rs:589-605), f32 accumulation of f32 activations times the
 * dequantised f32 weights, one rounding to the output dtype.  Rows are handled
 * 8 per pass; for prefill the reference dequantises once to f16 and runs a
 * dense GEMM (worker_gguf.rs:399-460), which dial_gguf_k_dequantize serves.
 * Needs no workspace. */
DIAL_API dial_status dial_gguf_k_linear(const void* x, dial_dtype xdt, const void* blocks,
                                        dial_ggml_type type, void* y, int64_t M, int64_t K, int64_t N,
                                        dial_stream stream);

/* ------------------------------------------------------------------ decoder glue
 * Activations are row-major [tokens, ...] in `dt` (f16 as the reference's
 * --dtype f16, or bf16); all arithmetic is f32.  head_dim must be 128.
 * KV caches are [slots, n_kv_heads, max_seq, head_dim]: one slot per sequence,
 * the preallocated decode storage of llama3/cache.rs:149-217.
 */

/* RMSNorm with an optional fused residual add (candle_nn::RmsNorm at
 * text.rs:1620-1626, 1649-1674; ln_f qwen3_vl.rs:2425-2429):
 *   h = residual ? round_dt(x + residual) : x;   if h_out: h_out = h
 *   y = round_dt(h * rsqrt(mean(h^2) + eps) * w)          w: [dim]
 * h_out may alias x or residual. */
DIAL_API dial_status dial_rmsnorm(const void* x, const void* residual, void* h_out, const void* w,
                                  void* y, dial_dtype dt, int64_t rows, int64_t dim, float eps,
                                  dial_stream stream);

/* RoPE tables of llama3/cache.rs:24-64: angle[p, i] = p * (1 / theta^(2i/D)),
 * cos/sin [max_pos, D/2] in dt. */
DIAL_API dial_status dial_rope_tables(void* cos_t, void* sin_t, dial_dtype dt, int64_t max_pos,
                                      int head_dim, float theta, dial_stream stream);

/* Post-QKV step of QwenAttention::forward (text.rs:1485-1531): split the fused
 * qkv [T, (Hq + 2*Hkv) * D]; per-head RMSNorm of q and k with q_norm_w / k_norm_w
 * [D] when qk_norm != 0 (Qwen3; Llama has none); RoPE at positions[t]; q goes to
 * q_out [T, Hq, D], k and v to row positions[t] of cache slot slots[t]. */
DIAL_API dial_status dial_qk_norm_rope_kv_append(
    const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_t,
    const void* sin_t, const int32_t* positions, const int32_t* slots, void* q_out,
    void* k_cache, void* v_cache, dial_dtype dt, int64_t tokens, int n_heads, int n_kv_heads,
    int head_dim, int64_t max_seq, float eps, int qk_norm, dial_stream stream);

/* GQA attention over the cache (text.rs:1258-1327): query t (q [T, Hq, D]) attends
 * rows 0..positions[t] of slot slots[t]; out [T, Hq*D] = softmax(q.K^T/sqrt(D)) V.
 * Decode passes one token per sequence, prefill a run of tokens (causal through
 * positions).  max_len >= max(positions)+1 sizes the key split; `workspace` holds
 * dial_attention_workspace_bytes(T, Hq, max_len) bytes (NULL when 0). */
DIAL_API size_t dial_attention_workspace_bytes(int64_t tokens, int n_heads, int64_t max_len);
DIAL_API dial_status dial_attention(const void* q, const void* k_cache, const void* v_cache,
                                    const int32_t* positions, const int32_t* slots, void* out,
                                    void* workspace, size_t workspace_bytes, dial_dtype dt,
                                    int64_t tokens, int n_heads, int n_kv_heads, int head_dim,
                                    int64_t max_seq, int64_t max_len, dial_stream stream);

/* One decode token (text.rs:1485-1531 then 1258-1327 for a single query row):
 * dial_qk_norm_rope_kv_append followed by dial_attention with tokens = 1, as
 * one launch -- the split of the key range holding positions[0] appends the
 * normed, rotated key and the value to the caches, every split computes the
 * query heads of its kv group from the raw qkv row, and the last split of a kv
 * group to finish merges the group's partials.  Same results, bit for bit, as
 * the two-call form.  `workspace` (16-byte aligned) holds
 * dial_decode_attention_workspace_bytes(n_heads, max_len) bytes, zero-filled
 * once by the caller; every call leaves it zeroed again.  Calls sharing a
 * workspace must not overlap on the GPU. */
DIAL_API size_t dial_decode_attention_workspace_bytes(int n_heads, int64_t max_len);
DIAL_API dial_status dial_decode_attention(
    const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_t,
    const void* sin_t, const int32_t* positions, const int32_t* slots, void* k_cache,
    void* v_cache, void* out, void* workspace, size_t workspace_bytes, dial_dtype dt,
    int n_heads, int n_kv_heads, int head_dim, int64_t max_seq, int64_t max_len, float eps,
    int qk_norm, dial_stream stream);

/* SwiGLU of Mlp (text.rs:816-820): out[t, i] = silu(g) * u over the halves of
 * gate_up [T, 2I] (silu result rounded to dt first, as two tensor ops). */
DIAL_API dial_status dial_swiglu(const void* gate_up, void* out, dial_dtype dt, int64_t tokens,
                                 int64_t intermediate, dial_stream stream);

/* Embedding rows: out[t] = table[ids[t]] (table [vocab, dim]).  An id outside
 * [0, vocab) writes zeros and sets the device error flag (DIAL_ERR_INVALID_ARG). */
DIAL_API dial_status dial_embedding(const void* table, const int32_t* ids, void* out,
                                    dial_dtype dt, int64_t tokens, int64_t vocab, int64_t dim,
                                    dial_stream stream);

/* Greedy sampling (qwen3_vl.rs:130-143): out[r] = first index of max(x[r, :]). */
DIAL_API dial_status dial_argmax(const void* x, int32_t* out, dial_dtype dt, int64_t rows,
                                 int64_t n, dial_stream stream);

/* ------------------------------------------------------------------ decoder stage
 * A pipeline stage = a contiguous range of decoder layers (spm::Forwarder /
 * Transformer::forward, text.rs:1636-1688), with the embedding on the first
 * stage and final norm + output head + greedy argmax on the last
 * (qwen3_vl.rs:2420-2451, :130-143).  Weights stay in the quantised formats
 * above; activations are `act_dtype` (f16 as the reference's --dtype f16).
 */
typedef enum {
  DIAL_WFMT_W8A16 = 0,     /* int8 [N,K] + f32 scale [N] (reference layout) */
  DIAL_WFMT_W8A16_F16S = 1, /* int8 [N,K] + f16 scale [N] */
  DIAL_WFMT_Q4_0 = 2,      /* dial_gguf_repack layout: qs + d */
  DIAL_WFMT_Q8_0 = 8
} dial_weight_format;

typedef struct dial_decoder_dims {
  int32_t hidden;         /* 4096 */
  int32_t intermediate;   /* 12288 (Qwen3-8B), 14336 (Llama-3-8B) */
  int32_t n_heads;        /* 32 */
  int32_t n_kv_heads;     /* 8 */
  int32_t head_dim;       /* 128 */
  int32_t vocab;          /* 151936 (Qwen3), 128256 (Llama-3) */
  int32_t qk_norm;        /* 1: per-head q_norm/k_norm (Qwen3); 0: none (Llama) */
  int32_t weight_format;  /* dial_weight_format of the layer linears */
  int32_t head_format;    /* dial_weight_format of the output head */
  int32_t act_dtype;      /* DIAL_F16 or DIAL_BF16 */
  float rms_eps;          /* 1e-6 */
  int64_t max_seq;        /* KV rows per slot */
  int32_t n_slots;        /* KV slots (sequences) */
} dial_decoder_dims;

/* A quantised linear: W8A16 {int8 q, scale}; GGUF {qs, d}. */
typedef struct dial_linear_ref {
  const void* w;
  const void* s;
} dial_linear_ref;

typedef struct dial_layer_weights {
  dial_linear_ref qkv;     /* [(Hq + 2*Hkv)*D, H] -- fused q,k,v (text.rs:1428-1432) */
  dial_linear_ref o;       /* [H, Hq*D] */
  dial_linear_ref gate_up; /* [2*I, H] -- fused gate,up (text.rs:634-637) */
  dial_linear_ref down;    /* [H, I] */
  const void* input_norm;  /* [H] */
  const void* post_norm;   /* [H] */
  const void* q_norm;      /* [D], qk_norm only */
  const void* k_norm;      /* [D] */
  void* k_cache;           /* [n_slots, Hkv, max_seq, D] */
  void* v_cache;
} dial_layer_weights;

/* Workspace for dial_decoder_layers / dial_decoder_head on `tokens` rows whose
 * positions are < max_len.  Zero-fill it once (it holds counters that every
 * call leaves at zero); one workspace sized for the largest call serves all. */
DIAL_API size_t dial_decoder_workspace_bytes(const dial_decoder_dims* dims, int64_t tokens,
                                             int64_t max_len);

/* Runs n_layers consecutive decoder layers on hidden [T, H] in place (the
 * residual stream).  Token t is at positions[t] of KV slot slots[t]; decode
 * passes one token per sequence, prefill a run of one sequence's tokens.
 * cos_t/sin_t come from dial_rope_tables (max_pos >= max_len). */
DIAL_API dial_status dial_decoder_layers(const dial_decoder_dims* dims,
                                         const dial_layer_weights* layers, int n_layers,
                                         void* hidden, const int32_t* positions,
                                         const int32_t* slots, int64_t tokens, int64_t max_len,
                                         const void* cos_t, const void* sin_t, void* workspace,
                                         size_t workspace_bytes, dial_stream stream);

/* Last stage: y = head(rmsnorm(hidden[rows], final_norm)); out_ids[r] = argmax.
 * `rows` selects which hidden rows to sample (row_index[r], NULL = 0..rows-1);
 * logits (optional, [rows, vocab] act_dtype) receives the head output. */
DIAL_API dial_status dial_decoder_head(const dial_decoder_dims* dims, const void* final_norm,
                                       dial_linear_ref head, const void* hidden,
                                       const int32_t* row_index, int64_t rows, int32_t* out_ids,
                                       void* logits, void* workspace, size_t workspace_bytes,
                                       dial_stream stream);

/* Vocabulary-parallel head (a stage's share of the output head): rows
 * [vocab_offset, vocab_offset + shard_rows) of the head, given as their own
 * [shard_rows, hidden] linear; the final norm and the GEMV as
 * dial_decoder_head, then per hidden row the greedy key of the shard's
 * largest logit: out_keys[r] = (order-preserving 32 bits of the rounded logit
 * << 32) | (0xFFFFFFFF - vocabulary index), so the largest key over all
 * shards is the first index of the maximum -- dial_decoder_head's argmax
 * (NaN never wins).  logits (optional, [rows, shard_rows]) receives the
 * shard's logits: the logits hand-back of the reference's output head
 * (worker_gguf.rs:342-386, RemoteOutputKind::Logits qwen3_vl.rs:258-279),
 * gathered by the caller.  The workspace is
 * dial_decoder_workspace_bytes(dims, rows, 1). */
DIAL_API dial_status dial_decoder_head_shard(
    const dial_decoder_dims* dims, const void* final_norm, dial_linear_ref head_shard,
    int64_t vocab_offset, int64_t shard_rows, const void* hidden, const int32_t* row_index,
    int64_t rows, uint64_t* out_keys, void* logits, void* workspace, size_t workspace_bytes,
    dial_stream stream);

/* Greedy token from the shards' keys: keys [n_shards, rows] (shard-major, as
 * gathered), out_ids[r] = the vocabulary index of the largest keys[., r] (0 if
 * every logit was NaN) -- the sampled-token hand-back with greedy sampling
 * (sample_remote_logits at temperature <= 0, qwen3_vl.rs:282-323; the
 * SampledToken kind, qwen3_vl.rs:262-264). */
DIAL_API dial_status dial_head_merge(const uint64_t* keys, int n_shards, int64_t rows,
                                     int32_t* out_ids, dial_stream stream);

/* ------------------------------------------------------------------ stage planner
 * Host-only (no GPU needed).  Restates AutoPlanner::plan_with_algorithm
 * (dial-core/src/spm/planner.rs:378-522, segment_cost :743-836): contiguous
 * layer segments, each on a different device, chosen by an exact DP over
 * (end layer, set of devices used, last device) under per-device memory
 * limits, for one of three objectives.  Devices here are the local GPUs of
 * one node; a worker's rtt/bandwidth/protocol describe the hand-off of a
 * segment's hidden state (NVLink instead of the reference's TCP).  Extension:
 * the model's head_* / embed_* costs (zero = the reference's cost model) are
 * charged to the segment that ends at the last layer / starts at layer 0, which
 * is where this pipeline keeps the output head and the embedding. */
enum { DIAL_PLAN_DIAL = 0, DIAL_PLAN_EDGESHARD_LATENCY = 1, DIAL_PLAN_EDGESHARD_THROUGHPUT = 2 };
enum { DIAL_PLAN_MASTER = 0, DIAL_PLAN_WORKER = 1 };
#define DIAL_PLAN_MAX_DEVICES 12

/* LayerMetric: per_layer[n_layers] when non-NULL, else `uniform` for every layer. */
typedef struct dial_layer_metric {
  const double* per_layer;
  double uniform;
} dial_layer_metric;

typedef struct dial_plan_device {
  int role;    /* DIAL_PLAN_MASTER / DIAL_PLAN_WORKER; exactly one enabled master */
  int enabled;
  double usable_memory_mb, fixed_memory_mb;
  dial_layer_metric layer_memory_mb, prefill_ms, decode_ms;
  int has_prefill_p95, has_decode_p95; /* else the mean profile */
  dial_layer_metric prefill_p95_ms, decode_p95_ms;
  dial_layer_metric prefill_energy_mj, decode_energy_mj;
  double rtt_ms, protocol_ms, bandwidth_mbps;          /* workers only */
  double rtt_p95_ms, protocol_p95_ms, bandwidth_p05_mbps; /* < 0: the mean value */
} dial_plan_device;

typedef struct dial_plan_objective {
  int prompt_tokens, output_tokens, dtype_bytes;
  int kv_context_tokens; /* 0: max_seq_len */
  double ttft_weight, tpot_weight, risk_weight, energy_weight, remote_device_penalty;
  int min_devices, max_devices; /* max_devices <= 0: every enabled device */
} dial_plan_objective;

typedef struct dial_plan_model {
  int num_layers, hidden_size, num_attention_heads, num_key_value_heads, max_seq_len;
  double head_memory_mb, head_prefill_ms, head_decode_ms;    /* segment ending at the last layer */
  double embed_memory_mb, embed_prefill_ms, embed_decode_ms; /* segment starting at layer 0 */
  /* DIAL_PLAN_LINKS_STAR (0, the reference's model, planner.rs:787-805): every
   * worker segment gets its input from the master and returns its output, two
   * hidden states per token over its own link.  DIAL_PLAN_LINKS_CHAIN: the
   * stages of a local GPU pipeline hand off stage to stage -- a segment that
   * does not start at layer 0 receives one hidden state per token over its
   * device's link (rtt + protocol + bytes / bandwidth), the last segment
   * returns a 4-byte token id to the first, and the master holds layer 0 (it
   * takes the prompt and the tokens). */
  int link_topology;
} dial_plan_model;
#define DIAL_PLAN_LINKS_STAR 0
#define DIAL_PLAN_LINKS_CHAIN 1

typedef struct dial_plan_segment {
  int device; /* index into the devices array */
  int start_layer, end_layer; /* inclusive, as PlannedSegment */
  double memory_mb, ttft_ms, tpot_ms, tail_ttft_ms, tail_tpot_ms;
} dial_plan_segment;

typedef struct dial_plan_result {
  int n_segments;
  dial_plan_segment segments[DIAL_PLAN_MAX_DEVICES];
  double ttft_ms, tpot_ms, tail_ttft_ms, tail_tpot_ms, request_energy_mj, score;
  int64_t states_considered, feasible_transitions, rejected_for_memory;
} dial_plan_result;

/* DIAL_ERR_INVALID_ARG with the reference's validation messages (dial_last_error)
 * on a bad profile; DIAL_ERR_SHAPE when no placement fits in memory. */
DIAL_API dial_status dial_plan_stages(const dial_plan_model* model, const dial_plan_objective* objective,
                                      const dial_plan_device* devices, int n_devices, int algorithm,
                                      dial_plan_result* out);

/* ------------------------------------------------------------------ stage hand-off
 * The pipeline's links over NCCL, replacing the reference's serialised TCP
 * hand-off between master and workers: RawTensor::{from_tensor, to_tensor}
 * (dial-core/src/spm/proto/message.rs:147-165) and its framing (:366-408),
 * Client::forward_batch / request (spm/client.rs:389-452, :281-329) and the
 * worker loop (spm/worker.rs:645-765).  One communicator per link (stage s ->
 * s + 1, and the token ring from the last stage to stage 0), two ranks each;
 * transfers are device to device and enqueued on the caller's stream.
 *
 * NCCL is loaded at run time (libnccl.so.2, reusing a copy the process has
 * already loaded); without it these calls return DIAL_ERR_NCCL.  A process
 * that also loads its own NCCL (PyTorch bundles one) should load that first:
 * two libraries with the soname libnccl.so.2 cannot coexist.
 * Communicators are non-blocking: initialisation, a link's first transfer
 * (NCCL connects a link there, which needs the peer's matching call) and
 * teardown are polled against `timeout_s` of host time and return
 * DIAL_ERR_TIMEOUT (the communicator is then aborted) instead of hanging.
 * After a failure the communicator only accepts dial_stage_comm_destroy. */
#define DIAL_STAGE_COMM_ID_BYTES 128
typedef struct dial_stage_comm dial_stage_comm;

/* A new clique id (DIAL_STAGE_COMM_ID_BYTES bytes, host memory), made by one
 * rank of a link and handed to the other out of band. */
DIAL_API dial_status dial_stage_comm_unique_id(uint8_t* id_out);
/* Joins the clique as `rank` of `nranks` on CUDA device `device` (made
 * current); returns once every rank has joined, or DIAL_ERR_TIMEOUT. */
DIAL_API dial_status dial_stage_comm_init(const uint8_t* unique_id, int rank, int nranks, int device,
                                          double timeout_s, dial_stage_comm** out);
/* `bytes` from device memory `buf` to rank `peer`, enqueued on `stream`. */
DIAL_API dial_status dial_stage_comm_send(dial_stage_comm* comm, const void* buf, size_t bytes,
                                          int peer, dial_stream stream);
/* `bytes` from rank `peer` into device memory `buf`, enqueued on `stream`. */
DIAL_API dial_status dial_stage_comm_recv(dial_stage_comm* comm, void* buf, size_t bytes, int peer,
                                          dial_stream stream);
/* Host wait (bounded by the communicator's timeout) until `stream` is idle. */
DIAL_API dial_status dial_stage_comm_wait(dial_stage_comm* comm, dial_stream stream);
/* Finalises (bounded) and frees the communicator; NULL is a no-op. */
DIAL_API dial_status dial_stage_comm_destroy(dial_stage_comm* comm);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DIAL_CUDA_H_ */
