// Decoder glue around the quantised linears (f16/bf16 activations, f32 math).
//
// Reference semantics (lisa301/DIAL-8B-orin):
//   RMSNorm       candle_nn::RmsNorm used at text.rs:1620-1626 (rms_1 / rms_2),
//                 :1466-1467 (q_norm / k_norm), ln_f qwen3_vl.rs:2425-2429:
//                 y = x * rsqrt(mean(x^2) + eps) * w, computed in f32.
//   residual      text.rs:1650-1674: (attn + residual), (mlp + residual) in the
//                 activation dtype -- fused here into the following RMSNorm.
//   RoPE          text.rs:1143-1153 (candle rotary_emb::rope, non-interleaved
//                 halves), tables llama3/cache.rs:24-64: inv_freq_i =
//                 1/theta^(2i/D) in f32, angle = pos * inv_freq, cos/sin stored
//                 in the activation dtype.
//   KV append     llama3/cache.rs:149-217: preallocated [b, kv_h, max_seq, D]
//                 storage, the new token written at its position.
//   attention     text.rs:1258-1327: GQA, softmax(q.K^T / sqrt(D)) V, causal.
//   SwiGLU        text.rs:816-820: silu(gate) * up over the halves of gate_up.
//   argmax        qwen3_vl.rs:130-143 (greedy sampling on the device).
#include <algorithm>
#include <cfloat>
#include <type_traits>

#include "common.cuh"
#include "glue.cuh"

namespace dial {

namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i) {
  return Act<T>::to_f32(p[i]);
}
template <typename T>
__device__ __forceinline__ T rnd(float v) {
  return Act<T>::from_f32(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = threadIdx.x < THREADS / 32 ? red[threadIdx.x] : 0.f;
  if (w == 0) v = warp_sum(v);
  if (threadIdx.x == 0) red[0] = v;
  __syncthreads();
  return red[0];
}

// ------------------------------------------------------------------ RMSNorm (+ residual)
// One CTA per row.  h = x (+ residual, rounded to T); y = h * rsqrt(mean(h^2)+eps) * w.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) rmsnorm_kernel(const T* x,  // x/res may alias h_out
                                                          const T* res,
                                                          T* h_out,
                                                          const T* __restrict__ w,
                                                          T* __restrict__ y, int dim, float eps) {
  pdl_begin();
  extern __shared__ float hbuf[];  // dim floats
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * dim;
  const T* rr = res ? res + row * dim : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += THREADS) {
    float v = ld(xr, i);
    if (rr) v = Act<T>::to_f32(rnd<T>(v + ld(rr, i)));  // residual add in the activation dtype
    hbuf[i] = v;
    ss += v * v;
  }
  ss = block_sum<THREADS>(ss, red);
  const float inv = rsqrtf(ss / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += THREADS) {
    const float v = hbuf[i];
    if (h_out) h_out[row * dim + i] = rnd<T>(v);
    y[row * dim + i] = rnd<T>(v * inv * ld(w, i));
  }
}

// ------------------------------------------------------------------ QK-norm + RoPE + KV append
// One head of 128 values by one warp: lane l owns elements {l, l+32, l+64,
// l+96}, so both RoPE pairs (i, i+64) stay in the lane.  Optional RMSNorm over
// the head (rounded to T), then RoPE at the position whose table rows are
// cr / sr, with every product and the sum in T as candle's rope evaluates them
// over T tensors (a product of two T values is exact in f32, so rounding it to
// T is the T multiplication).  o[i] = the T-rounded result of element lane + 32 i.
template <typename T>
__device__ __forceinline__ void head_norm_rope_warp(const T* __restrict__ src, const T* __restrict__ nw,
                                                    int qk_norm, float eps, const T* __restrict__ cr,
                                                    const T* __restrict__ sr, float (&o)[4]) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = ld(src, lane + 32 * i);
  if (qk_norm) {
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      v[i] = Act<T>::to_f32(rnd<T>(v[i] * inv * ld(nw, lane + 32 * i)));  // normed tensor in T
  }
  auto r = [](float a) { return Act<T>::to_f32(rnd<T>(a)); };
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int e = lane + 32 * i;  // 0..63
    const float c = ld(cr, e), sn = ld(sr, e);
    o[i] = r(r(v[i] * c) - r(v[i + 2] * sn));
    o[i + 2] = r(r(v[i] * sn) + r(v[i + 2] * c));
  }
}

// One warp per (token, head) over Hq + 2*Hkv heads; lane l owns elements
// {l, l+32, l+64, l+96} of the 128-wide head, so both RoPE pairs (i, i+64)
// stay in the lane.  head_dim is fixed to 128 (Qwen3-8B / Llama-3-8B).
template <typename T>
__global__ void qk_rope_kv_kernel(const T* __restrict__ qkv, const T* __restrict__ qn,
                                  const T* __restrict__ kn, const T* __restrict__ cos_t,
                                  const T* __restrict__ sin_t, const int32_t* __restrict__ pos,
                                  const int32_t* __restrict__ slot, T* __restrict__ q_out,
                                  T* __restrict__ kc, T* __restrict__ vc, int64_t tokens, int hq,
                                  int hkv, int64_t max_seq, float eps, int qk_norm) {
  pdl_begin();
  constexpr int D = 128;
  const int heads = hq + 2 * hkv;
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= tokens * heads) return;
  const int64_t t = gw / heads;
  const int h = (int)(gw % heads);
  const T* src = qkv + t * (int64_t)heads * D + (int64_t)h * D;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = ld(src, lane + 32 * i);
  const int p = pos[t];
  const int64_t s = slot[t];
  if (h >= hq + hkv) {  // value head: straight into the cache
    T* dst = vc + ((s * hkv + (h - hq - hkv)) * max_seq + p) * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = rnd<T>(v[i]);
    return;
  }
  const bool is_q = h < hq;
  // rotate_half: out[i] = x[i] c_i - x[i+64] s_i ; out[i+64] = x[i] s_i + x[i+64] c_i
  float o[4];
  head_norm_rope_warp<T>(src, is_q ? qn : kn, qk_norm, eps, cos_t + (int64_t)p * (D / 2),
                         sin_t + (int64_t)p * (D / 2), o);
  T* dst = is_q ? q_out + (t * hq + h) * D : kc + ((s * hkv + (h - hq)) * max_seq + p) * D;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = rnd<T>(o[i]);
}

// ------------------------------------------------------------------ attention
// Query token t attends cache rows 0..pos[t] of slot[t] (decode: one token per
// sequence; prefill: a run of tokens of one sequence, causal through pos).
// CTA = (token, kv head, key split); the n_rep query heads of the group share
// every K/V row.  Scores follow the reference's T tensors (text.rs:1278-1279):
// s = T(T(q.k) * T(1/sqrt(D))) -- the matmul's output in T, then the affine
// `/ sqrt(D)` with its multiplier in T -- and enter the softmax in the log2
// domain (times log2(e) in f32); softmax and accumulation in f32; splits are
// merged by the combine step.
template <typename T>
__global__ void attention_combine_kernel(const float* __restrict__ part, T* __restrict__ out,
                                         int nchunks) {
  pdl_begin();
  constexpr int D = 128;
  const int64_t head = blockIdx.x;
  const int d = threadIdx.x;
  const float* pp = part + head * nchunks * (D + 2);
  float m = -FLT_MAX;
  for (int c = 0; c < nchunks; ++c) m = fmaxf(m, pp[c * (D + 2)]);
  float sum = 0.f, acc = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    const float cm = pp[c * (D + 2)];
    if (cm == -FLT_MAX) continue;
    const float f = exp2f(cm - m);  // partial maxima are in the log2 domain
    sum += pp[c * (D + 2) + 1] * f;
    acc += pp[c * (D + 2) + 2 + d] * f;
  }
  out[head * D + d] = rnd<T>(acc / sum);
}

// ------------------------------------------------------------------ attention on tensor cores
// f16/bf16 caches: the same (token, kv head, key split) CTAs, but each of the 4
// warps takes 16-key tiles (tiles w, w+4, ... of the split) and computes
//   S = Q K^T  (mma.m16n8k16: rows = the n_rep query heads of the group, padded
//               to 16; 8 k-steps over the head dim; two 8-key n-tiles)
//   O += P V   (P from the score fragments, split into hi + lo parts of the
//               operand type so that P keeps 16+ significant bits; 16 n-tiles
//               of 8 dims)
// with the online softmax in f32 on the score fragments (row max / sum over
// the 4 lanes of a quad).  K/V tiles stream through a 2-deep per-warp ring of
// cp.async copies into XOR-swizzled shared memory (16-byte chunk c of key row
// r at chunk (c & 8) | ((c ^ r) & 7)), read back with ldmatrix (.trans for V).
// The warps merge in shared memory; splits leave (max, sum, O) partials for the
// combine step.
constexpr int kTcWarps = 4;
constexpr int kTcTile = 16;                         // keys per tile
constexpr int kTcTileBytes = kTcTile * 128 * 2;     // one K or V tile (4 KB)
constexpr int kTcWarpBytes = 2 * 2 * kTcTileBytes;  // 2 stages x (K, V)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t tc_swz(int r, int c) {
  return (uint32_t)(r * 256 + (((c & 8) | ((c ^ r) & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma_tc(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (sizeof(T) == 2 && std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// (a, b) -> operand pair, and the pair of what rounding left behind
template <typename T>
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const T ha = Act<T>::from_f32(a), hb = Act<T>::from_f32(b);
  const T la = Act<T>::from_f32(a - Act<T>::to_f32(ha)), lb = Act<T>::from_f32(b - Act<T>::to_f32(hb));
  hi = (uint32_t)(*reinterpret_cast<const uint16_t*>(&ha)) |
       ((uint32_t)(*reinterpret_cast<const uint16_t*>(&hb)) << 16);
  lo = (uint32_t)(*reinterpret_cast<const uint16_t*>(&la)) |
       ((uint32_t)(*reinterpret_cast<const uint16_t*>(&lb)) << 16);
}

// (a, b) -> three operand pairs: hi, what hi left behind, and what that left
// (bf16: 8 + 8 + 8 significant bits, the f32 value in the normal range)
template <typename T>
__device__ __forceinline__ void split_pair3(float a, float b, uint32_t& hi, uint32_t& mid,
                                            uint32_t& lo) {
  const T ha = Act<T>::from_f32(a), hb = Act<T>::from_f32(b);
  const float ra = a - Act<T>::to_f32(ha), rb = b - Act<T>::to_f32(hb);
  split_pair<T>(ra, rb, mid, lo);
  hi = (uint32_t)(*reinterpret_cast<const uint16_t*>(&ha)) |
       ((uint32_t)(*reinterpret_cast<const uint16_t*>(&hb)) << 16);
}

// Inputs of the decode form (FUSE): the raw qkv rows, the QK-norm gains, the
// RoPE tables, and the caches to append the new key / value rows to.
template <typename T>
struct QkvIn {
  const T* qkv;
  const T* qn;
  const T* kn;
  const T* cos_t;
  const T* sin_t;
  T* kc;
  T* vc;
  int* ctr;  // [tokens * hkv] split arrival counters, zero between launches
  float eps;
  int qk_norm;
};

// FUSE (decode, one token per sequence): the CTA computes its REP query heads'
// QK-norm + RoPE from the raw qkv row itself (head_norm_rope_warp, the same
// arithmetic as qk_rope_kv_kernel), the split that holds the new position
// appends the token's key (normed, rotated) and value rows to the caches before
// reading its tiles, and the last of the (token, kv head)'s splits to finish
// (an arrival counter, no waiting) merges the splits' partials exactly as
// attention_combine_kernel does -- no qk_rope and no combine launch.
template <typename T, int REP, bool FUSE>
__global__ void __launch_bounds__(kTcWarps * 32)
    attention_tc_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
                        const int32_t* __restrict__ pos, const int32_t* __restrict__ slot,
                        T* __restrict__ out, float* __restrict__ part, int hq, int hkv,
                        int64_t max_seq, int nsplit, float qscale, QkvIn<T> in) {
  pdl_trigger();
  if constexpr (FUSE) {
    // The split's cache rows before the new position were written by kernels
    // that ended long before this one (earlier steps, or the prompt): pull them
    // into L2 while the previous kernel finishes.  Only a hint -- the position
    // read here may still be the previous step's, so it is clamped into the
    // cache and nothing below uses it.
    if (threadIdx.x < 2) {
      int64_t lp = (int64_t)pos[blockIdx.x] + 1;
      lp = lp < 1 ? 1 : (lp > max_seq ? max_seq : lp);
      const int64_t per = (lp + nsplit - 1) / nsplit, k0 = (int64_t)blockIdx.z * per;
      const int64_t k1 = lp < k0 + per ? lp : k0 + per;
      if (k1 > k0) {
        const T* base = (threadIdx.x ? vc : kc) + (((int64_t)slot[blockIdx.x] * hkv + (int64_t)blockIdx.y) * max_seq + k0) * 128;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base),
                     "r"((uint32_t)(k1 - k0) * 256u)
                     : "memory");
      }
    }
  }
  pdl_wait();
  constexpr int D = 128;
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  __shared__ float sm_m[kTcWarps][REP], sm_l[kTcWarps][REP];
  __shared__ float sm_o[kTcWarps][REP][D];
  __shared__ __align__(16) T sm_q[FUSE ? REP : 1][D];
  __shared__ int sm_last;
  const int64_t t = blockIdx.x;
  const int g = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, qd = lane & 3;  // fragment row (query head) and quad index
  const int len = pos[t] + 1;
  const int per = (len + nsplit - 1) / nsplit;
  const int k0 = split * per, k1 = min(len, k0 + per);
  const int64_t s = slot[t];
  const T* kbase = kc + ((s * hkv + g) * max_seq) * D;
  const T* vbase = vc + ((s * hkv + g) * max_seq) * D;
  const uint32_t wbuf = smem_addr(tc_smem) + (uint32_t)(warp * kTcWarpBytes);

  if constexpr (FUSE) {
    const int p = len - 1;
    const T* src = in.qkv + t * (int64_t)(hq + 2 * hkv) * D;
    const T* cr = in.cos_t + (int64_t)p * (D / 2);
    const T* sr = in.sin_t + (int64_t)p * (D / 2);
    for (int h = warp; h < REP; h += kTcWarps) {  // this group's query heads
      float o[4];
      head_norm_rope_warp<T>(src + (int64_t)(g * REP + h) * D, in.qn, in.qk_norm, in.eps, cr, sr, o);
#pragma unroll
      for (int i = 0; i < 4; ++i) sm_q[h][lane + 32 * i] = rnd<T>(o[i]);
    }
    if (p >= k0 && p < k1) {  // the split holding the new position appends its key and value rows
      if (warp == kTcWarps - 1) {
        float o[4];
        head_norm_rope_warp<T>(src + (int64_t)(hq + g) * D, in.kn, in.qk_norm, in.eps, cr, sr, o);
        T* dst = in.kc + ((s * hkv + g) * max_seq + p) * D;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = rnd<T>(o[i]);
      } else if (warp == kTcWarps - 2) {
        const T* vs = src + (int64_t)(hq + hkv + g) * D;
        T* dst = in.vc + ((s * hkv + g) * max_seq + p) * D;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = vs[lane + 32 * i];
      }
      __threadfence();  // the rows are read back below through cp.async (L2)
    }
    __syncthreads();
  }

  // Q fragments: row gr = query head g*REP + gr (zero above REP), k-step ks
  uint32_t qa[8][2];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa[ks][0] = qa[ks][1] = 0u;
    if (gr < REP) {
      const uint32_t* qr = FUSE ? reinterpret_cast<const uint32_t*>(&sm_q[FUSE ? gr : 0][0])
                                : reinterpret_cast<const uint32_t*>(q + (t * hq + g * REP + gr) * D);
      qa[ks][0] = qr[(16 * ks + 2 * qd) >> 1];
      qa[ks][1] = qr[(16 * ks + 8 + 2 * qd) >> 1];
    }
  }

  const int ntile = k1 > k0 ? (k1 - k0 + kTcTile - 1) / kTcTile : 0;
  // issue the copies of tile i (keys k0 + 16 i ..) into stage st of this warp
  auto fetch = [&](int i, int st) {
    const int kb = k0 + i * kTcTile;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int ch = lane + 32 * u, r = ch >> 4, c = ch & 15;
      const int key = min(kb + r, k1 - 1);  // rows past the split repeat its last key (masked)
      const uint32_t off = tc_swz(r, c);
      cp_async16(wbuf + (uint32_t)(st * 2 * kTcTileBytes) + off, kbase + (int64_t)key * D + c * 8);
      cp_async16(wbuf + (uint32_t)(st * 2 * kTcTileBytes + kTcTileBytes) + off,
                 vbase + (int64_t)key * D + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float m = -FLT_MAX, l = 0.f;  // row gr (only gr < REP is a real head)
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;

  int st = 0;
  if (warp < ntile) fetch(warp, 0);
  for (int i = warp; i < ntile; i += kTcWarps) {
    const bool more = i + kTcWarps < ntile;
    if (more) fetch(i + kTcWarps, st ^ 1);
    if (more) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    const uint32_t kt = wbuf + (uint32_t)(st * 2 * kTcTileBytes), vt = kt + kTcTileBytes;
    // ---- S = Q K^T for keys kb .. kb+15
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kt + tc_swz((mi >> 1) * 8 + ri, 2 * ks + (mi & 1)), b0, b1, b2, b3);
      mma_tc<T>(sc[0], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
      mma_tc<T>(sc[1], qa[ks][0], 0u, qa[ks][1], 0u, b2, b3);
    }
    // ---- online softmax on row gr: this lane holds keys 2qd, 2qd+1, 8+2qd, 9+2qd
    const int kb = k0 + i * kTcTile;
    auto score = [&](float a) {  // T(T(a) * T(1/sqrt(D))) * log2(e)
      return Act<T>::to_f32(Act<T>::from_f32(Act<T>::to_f32(Act<T>::from_f32(a)) * qscale)) *
             1.4426950408889634f;
    };
    float p[4] = {score(sc[0][0]), score(sc[0][1]), score(sc[1][0]), score(sc[1][1])};
    const int kk[4] = {2 * qd, 2 * qd + 1, 8 + 2 * qd, 9 + 2 * qd};
    float mx = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (kb + kk[j] >= k1) p[j] = -FLT_MAX;
      mx = fmaxf(mx, p[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float corr = exp2f(m - mn);
    m = mn;
    float ps = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[j] = exp2f(p[j] - mn);
      ps += p[j];
    }
    l = l * corr + ps;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= corr;
      o[nt][1] *= corr;
    }
    // P as operand parts: f16 hi + lo keeps 22 significant bits; bf16 takes a
    // third part (24 bits), as two bf16 parts (16 bits) would round P far more
    // coarsely than the f32 accumulation does
    constexpr bool kThree = !std::is_same<T, __half>::value;
    uint32_t ph0, pl0, ph1, pl1, pm0 = 0u, pm1 = 0u;
    if constexpr (kThree) {
      split_pair3<T>(p[0], p[1], ph0, pm0, pl0);
      split_pair3<T>(p[2], p[3], ph1, pm1, pl1);
    } else {
      split_pair<T>(p[0], p[1], ph0, pl0);
      split_pair<T>(p[2], p[3], ph1, pl1);
    }
    // ---- O += P V over 16 dim n-tiles
#pragma unroll
    for (int nt = 0; nt < 16; nt += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vt + tc_swz((mi & 1) * 8 + ri, nt + (mi >> 1)), b0, b1, b2, b3);
      mma_tc<T>(o[nt], ph0, 0u, ph1, 0u, b0, b1);
      mma_tc<T>(o[nt], pl0, 0u, pl1, 0u, b0, b1);
      if constexpr (kThree) mma_tc<T>(o[nt], pm0, 0u, pm1, 0u, b0, b1);
      mma_tc<T>(o[nt + 1], ph0, 0u, ph1, 0u, b2, b3);
      mma_tc<T>(o[nt + 1], pl0, 0u, pl1, 0u, b2, b3);
      if constexpr (kThree) mma_tc<T>(o[nt + 1], pm0, 0u, pm1, 0u, b2, b3);
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    st ^= 1;
  }
  // row sums over the quad
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- merge the warps (a warp without tiles keeps m = -FLT_MAX, l = 0)
  if (gr < REP) {
    if (qd == 0) {
      sm_m[warp][gr] = m;
      sm_l[warp][gr] = l;
    }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      sm_o[warp][gr][8 * nt + 2 * qd] = o[nt][0];
      sm_o[warp][gr][8 * nt + 2 * qd + 1] = o[nt][1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < REP * D; idx += kTcWarps * 32) {
    const int r = idx / D, d = idx % D;
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, sm_m[w][r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) {
      if (sm_l[w][r] == 0.f) continue;  // warp saw no key
      const float f = exp2f(sm_m[w][r] - M);
      L += sm_l[w][r] * f;
      O += sm_o[w][r][d] * f;
    }
    const int64_t head = t * hq + g * REP + r;
    if (nsplit == 1) {
      out[head * D + d] = Act<T>::from_f32(O / L);
    } else {
      float* pp = part + (head * nsplit + split) * (D + 2);
      if (d == 0) {
        pp[0] = L > 0.f ? M : -FLT_MAX;  // -FLT_MAX for an empty split
        pp[1] = L;
      }
      pp[2 + d] = O;
    }
  }
  if constexpr (FUSE) {
    if (nsplit == 1) return;
    // the last split of this (token, kv head) to arrive merges the partials
    __threadfence();
    __syncthreads();
    int* ctr = in.ctr + t * hkv + g;
    if (threadIdx.x == 0) sm_last = atomicAdd(ctr, 1) == nsplit - 1;
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
    // the arithmetic of attention_combine_kernel in its order: per head, a
    // warp finds the maximum, the split weights f_c = 2^(m_c - m) and the sum;
    // then every output element accumulates its splits' O in split order.
    // Up to 16 splits, warp r owns head r and lane l dims 4l .. 4l+3, and every
    // load (the splits' maxima and sums, and their O) is issued in one round.
    if (nsplit <= 16) {
      for (int r = warp; r < REP; r += kTcWarps) {
        const int64_t head = t * hq + g * REP + r;
        const float* pp = part + head * nsplit * (D + 2);
        const float cm = lane < nsplit ? __ldcg(pp + lane * (D + 2)) : -FLT_MAX;
        const float cl = lane < nsplit ? __ldcg(pp + lane * (D + 2) + 1) : 0.f;
        float2 ov[16][2];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          ov[c][0] = ov[c][1] = make_float2(0.f, 0.f);
          if (c < nsplit) {  // (D + 2) floats per split row: dims 4l.. start 8-byte aligned
            const float2* src = reinterpret_cast<const float2*>(pp + c * (D + 2) + 2 + 4 * lane);
            ov[c][0] = __ldcg(src);
            ov[c][1] = __ldcg(src + 1);
          }
        }
        float m = cm;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const bool ok = lane < nsplit && cm != -FLT_MAX;
        const float f = ok ? exp2f(cm - m) : 0.f;  // partial maxima are in the log2 domain
        const unsigned valid = __ballot_sync(0xffffffffu, ok);
        float sum = 0.f;
        for (int c = 0; c < nsplit; ++c) {
          const float lc = __shfl_sync(0xffffffffu, cl, c), fc = __shfl_sync(0xffffffffu, f, c);
          if ((valid >> c) & 1u) sum += lc * fc;
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float fc = __shfl_sync(0xffffffffu, f, c);
          if (c < nsplit && ((valid >> c) & 1u)) {
            acc[0] += ov[c][0].x * fc;
            acc[1] += ov[c][0].y * fc;
            acc[2] += ov[c][1].x * fc;
            acc[3] += ov[c][1].y * fc;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) out[head * D + 4 * lane + e] = rnd<T>(acc[e] / sum);
      }
    } else {
      __shared__ float sm_f[REP][32];
      __shared__ float sm_sum[REP];
      __shared__ unsigned sm_valid[REP];
      for (int r = warp; r < REP; r += kTcWarps) {
        const float* pp = part + (t * hq + g * REP + r) * nsplit * (D + 2);
        const float cm = lane < nsplit ? __ldcg(pp + lane * (D + 2)) : -FLT_MAX;
        const float cl = lane < nsplit ? __ldcg(pp + lane * (D + 2) + 1) : 0.f;
        float m = cm;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const bool ok = lane < nsplit && cm != -FLT_MAX;
        const float f = ok ? exp2f(cm - m) : 0.f;
        const unsigned valid = __ballot_sync(0xffffffffu, ok);
        float sum = 0.f;
        for (int c = 0; c < nsplit; ++c) {
          const float lc = __shfl_sync(0xffffffffu, cl, c), fc = __shfl_sync(0xffffffffu, f, c);
          if ((valid >> c) & 1u) sum += lc * fc;
        }
        sm_f[r][lane] = f;
        if (lane == 0) sm_sum[r] = sum, sm_valid[r] = valid;
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < REP * D; idx += kTcWarps * 32) {
        const int r = idx / D, d = idx % D;
        const int64_t head = t * hq + g * REP + r;
        const float* pp = part + head * nsplit * (D + 2) + 2 + d;
        float ov[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) ov[c] = c < nsplit ? __ldcg(pp + c * (D + 2)) : 0.f;
        const unsigned valid = sm_valid[r];
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c < nsplit && ((valid >> c) & 1u)) acc += ov[c] * sm_f[r][c];
        out[head * D + d] = rnd<T>(acc / sm_sum[r]);
      }
    }
    if (threadIdx.x == 0) *ctr = 0;  // ready for the next launch
  }
}

// ------------------------------------------------------------------ SwiGLU
// out[t, i] = round(round(silu(g)) * u), g = gate_up[t, i], u = gate_up[t, I + i];
// silu with the fast exp and divide (a few ulp in f32, then rounded to the
// activation dtype)
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t tokens,
                              int64_t inter) {
  pdl_begin();
  const int64_t n = tokens * inter;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / inter, c = i % inter;
    const float g = ld(gu, t * 2 * inter + c);
    const float u = ld(gu, t * 2 * inter + inter + c);
    const float s = Act<T>::to_f32(rnd<T>(__fdividef(g, 1.0f + __expf(-g))));
    out[i] = rnd<T>(s * u);
  }
}

// out = round(a + b), the residual add after the last layer of a stage
// (text.rs:1672-1674); out may be a.
template <typename T>
__global__ void add_kernel(T* out, const T* a, const T* __restrict__ b, int64_t n) {
  pdl_begin();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = rnd<T>(ld(a, i) + ld(b, i));
}

template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ src, const int32_t* __restrict__ idx,
                                   T* __restrict__ dst, int64_t dim) {
  pdl_begin();
  const int64_t r = blockIdx.x;
  const int64_t s = idx[r];
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) dst[r * dim + i] = src[s * dim + i];
}

// ------------------------------------------------------------------ embedding / argmax
template <typename T>
__global__ void embedding_kernel(const T* __restrict__ table, const int32_t* __restrict__ ids,
                                 T* __restrict__ out, int64_t tokens, int64_t vocab, int64_t dim,
                                 int* __restrict__ err) {
  pdl_begin();
  const int64_t t = blockIdx.x;
  const int32_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) atomicCAS(err, 0, (int)DIAL_ERR_INVALID_ARG);
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x)
    out[t * dim + i] = ok ? table[(int64_t)id * dim + i] : rnd<T>(0.f);
}

// First index of the maximum (NaN never wins), one CTA per row.
template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ x,
                                                      int32_t* __restrict__ out, int64_t n) {
  pdl_begin();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * n;
  float best = -FLT_MAX;
  int64_t bidx = n;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = ld(xr, i);
    if (v > best) { best = v; bidx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) { best = ov; bidx = oi; }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { bv[w] = best; bi[w] = (int)bidx; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? bv[threadIdx.x] : -FLT_MAX;
    bidx = threadIdx.x < nw ? bi[threadIdx.x] : n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ov > best || (ov == best && oi < bidx)) { best = ov; bidx = oi; }
    }
    if (threadIdx.x == 0) out[row] = (int32_t)(bidx < n ? bidx : 0);
  }
}

// Per row, the greedy key (argmax_key, indices from `offset`) of the row's
// largest value: argmax_kernel's choice, as a key that merges across shards.
template <typename T>
__global__ void __launch_bounds__(1024) argmax_key_kernel(const T* __restrict__ x,
                                                          unsigned long long* __restrict__ keys,
                                                          int64_t n, int64_t offset) {
  pdl_begin();
  __shared__ unsigned long long bk[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * n;
  unsigned long long best = 0ull;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = argmax_key(ld(xr, i), offset + i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
    best = ok > best ? ok : best;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) bk[w] = best;
  __syncthreads();
  if (w == 0) {
    best = threadIdx.x < (blockDim.x >> 5) ? bk[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
      best = ok > best ? ok : best;
    }
    if (threadIdx.x == 0) keys[row] = best;
  }
}

// keys_out[r] / ids[r] from the n keys keys[r * n .. r * n + n) (or, with
// stride, keys[c * stride + r] for c < n): the largest key, and its index (0
// when every value of the row was NaN, as argmax_kernel).
__global__ void __launch_bounds__(256) key_reduce_kernel(const unsigned long long* __restrict__ keys,
                                                         int64_t n, int64_t elem_stride,
                                                         int64_t row_stride,
                                                         unsigned long long* __restrict__ keys_out,
                                                         int32_t* __restrict__ ids) {
  pdl_begin();
  __shared__ unsigned long long bk[8];
  const int64_t row = blockIdx.x;
  unsigned long long best = 0ull;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = keys[row * row_stride + i * elem_stride];
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
    best = ok > best ? ok : best;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) bk[w] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) best = bk[k] > best ? bk[k] : best;
    if (keys_out) keys_out[row] = best;
    if (ids) ids[row] = (best >> 32) ? (int32_t)(0xFFFFFFFFu - (uint32_t)best) : 0;
  }
}

// cos/sin tables: angle = pos * (1 / theta^(i/ (D/2) ... )) computed in f32 as
// llama3/cache.rs:31-50 (inv_freq from powf in f32, the product in f32).
template <typename T>
__global__ void rope_table_kernel(T* __restrict__ cos_t, T* __restrict__ sin_t, int64_t max_pos,
                                  int half, float theta) {
  const int64_t n = max_pos * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / half;
    const int j = (int)(i % half);
    const float inv = 1.0f / powf(theta, (float)(2 * j) / (float)(2 * half));
    const float a = (float)p * inv;
    cos_t[i] = rnd<T>(cosf(a));
    sin_t[i] = rnd<T>(sinf(a));
  }
}

unsigned grid_cap(int64_t work, int threads, int per_sm = 16) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  return (unsigned)std::max<int64_t>(1, std::min(b, cap));
}

}  // namespace

// ------------------------------------------------------------------ launchers
#define DISPATCH_T(dt, ...)                          \
  do {                                               \
    if ((dt) == DIAL_F16) {                          \
      using T = __half;                              \
      __VA_ARGS__;                                   \
    } else if ((dt) == DIAL_BF16) {                  \
      using T = __nv_bfloat16;                       \
      __VA_ARGS__;                                   \
    } else {                                         \
      using T = float;                               \
      __VA_ARGS__;                                   \
    }                                                \
  } while (0)

dial_status launch_rmsnorm(const void* x, const void* res, void* h_out, const void* w, void* y,
                           dial_dtype dt, int64_t rows, int64_t dim, float eps, cudaStream_t st) {
  const size_t smem = (size_t)dim * sizeof(float);
  if (smem > 96 * 1024) return fail(DIAL_ERR_SHAPE, "rmsnorm dim too large (%lld)", (long long)dim);
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    auto k = rmsnorm_kernel<T, 512>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    s = launch_pdl("rmsnorm_kernel", k, dim3((unsigned)rows), dim3(512), smem, st,
                   static_cast<const T*>(x), static_cast<const T*>(res), static_cast<T*>(h_out),
                   static_cast<const T*>(w), static_cast<T*>(y), (int)dim, eps);
  });
  return s;
}

dial_status launch_qk_rope_kv(const void* qkv, const void* qn, const void* kn, const void* cos_t,
                              const void* sin_t, const int32_t* pos, const int32_t* slot,
                              void* q_out, void* kc, void* vc, dial_dtype dt, int64_t tokens,
                              int hq, int hkv, int64_t max_seq, float eps, int qk_norm,
                              cudaStream_t st) {
  const int64_t warps = tokens * (hq + 2 * hkv);
  const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("qk_rope_kv_kernel", qk_rope_kv_kernel<T>, dim3(grid), dim3(256), 0, st,
                   static_cast<const T*>(qkv), static_cast<const T*>(qn), static_cast<const T*>(kn),
                   static_cast<const T*>(cos_t), static_cast<const T*>(sin_t), pos, slot,
                   static_cast<T*>(q_out), static_cast<T*>(kc), static_cast<T*>(vc), tokens, hq, hkv,
                   max_seq, eps, qk_norm);
  });
  return s;
}

// Key splits per (token, kv head), at least 64 keys each (4 tiles of 16 keys,
// one per warp): the count whose waves of CTAs (three resident per SM: 168
// registers x 128 threads, 72 KB of shared memory) waste least of the last
// wave, with a small charge per split for its partials and the merge (a
// one-token decode is latency bound: more, shorter splits measured faster).
static int attention_splits(int64_t tokens, int hkv, int64_t max_len) {
  const int64_t pairs = tokens * hkv, slots = 3 * (int64_t)sm_count();
  if (pairs >= slots) return 1;  // the unsplit grid already fills the GPU
  const int64_t cap = std::min<int64_t>(32, std::max<int64_t>(1, (max_len + 63) / 64));
  int best = 1;
  double best_t = 1e30;
  for (int n = 1; n <= cap; ++n) {
    const double waves = (double)((pairs * n + slots - 1) / slots);
    const double t = waves / n + 0.005 * n;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = n;
    }
  }
  return best;
}

size_t attention_workspace_bytes(int64_t tokens, int hq, int64_t max_len) {
  // hkv is not known here: size for the largest split count any divisor of hq gives
  int64_t nch = 1;
  for (int hkv = 1; hkv <= hq; ++hkv)
    if (hq % hkv == 0) nch = std::max<int64_t>(nch, attention_splits(tokens, hkv, max_len));
  return nch > 1 ? (size_t)(tokens * hq * nch * (128 + 2)) * sizeof(float) : 0;
}

// One (dtype, n_rep) instance of the tensor-core attention.
template <typename T, int REP>
dial_status launch_attention_rep(dim3 grid, const void* q, const void* kc, const void* vc,
                                 const int32_t* pos, const int32_t* slot, void* out, void* ws,
                                 int hq, int hkv, int64_t max_seq, int nch, float qscale,
                                 cudaStream_t st) {
  if constexpr (sizeof(T) != 2) {
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "attention: f16/bf16 caches only");
  } else {
    constexpr int smem = kTcWarps * kTcWarpBytes;
    const cudaError_t e = ensure_smem<attention_tc_kernel<T, REP, false>>(smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention_tc_kernel)");
    return launch_pdl("attention_tc_kernel", attention_tc_kernel<T, REP, false>, grid,
                      dim3(kTcWarps * 32), smem, st, static_cast<const T*>(q),
                      static_cast<const T*>(kc), static_cast<const T*>(vc), pos, slot,
                      static_cast<T*>(out), static_cast<float*>(ws), hq, hkv, max_seq, nch, qscale,
                      QkvIn<T>{});
  }
}

// The decode form: grid (tokens, hkv, nch).
template <typename T, int REP>
dial_status launch_attention_fused_rep(dim3 grid, const QkvIn<T>& in, const int32_t* pos,
                                       const int32_t* slot, void* out, void* part, int hq, int hkv,
                                       int64_t max_seq, int nch, float qscale, cudaStream_t st) {
  constexpr int smem = kTcWarps * kTcWarpBytes;
  const cudaError_t e = ensure_smem<attention_tc_kernel<T, REP, true>>(smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention_tc_kernel)");
  return launch_pdl("attention_tc_kernel", attention_tc_kernel<T, REP, true>, grid,
                    dim3(kTcWarps * 32), smem, st, static_cast<const T*>(nullptr),
                    static_cast<const T*>(in.kc), static_cast<const T*>(in.vc), pos, slot,
                    static_cast<T*>(out), static_cast<float*>(part), hq, hkv, max_seq, nch, qscale,
                    in);
}

dial_status launch_attention(const void* q, const void* kc, const void* vc, const int32_t* pos,
                             const int32_t* slot, void* out, void* ws, dial_dtype dt,
                             int64_t tokens, int hq, int hkv, int64_t max_seq, int64_t max_len,
                             cudaStream_t st) {
  const int nch = attention_splits(tokens, hkv, max_len);
  // T(1/sqrt(128)): 0x1.6a0p-4 = 0.08837890625 in both f16 and bf16
  const float qscale = 0.08837890625f;
  dim3 grid((unsigned)tokens, (unsigned)hkv, (unsigned)nch);
  const int rep = hq / hkv;
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    auto fn = rep == 1   ? launch_attention_rep<T, 1>
              : rep == 2 ? launch_attention_rep<T, 2>
              : rep == 4 ? launch_attention_rep<T, 4>
              : rep == 8 ? launch_attention_rep<T, 8>
                         : nullptr;
    if (!fn) return fail(DIAL_ERR_SHAPE, "attention supports Hq/Hkv in {1,2,4,8}");
    s = fn(grid, q, kc, vc, pos, slot, out, ws, hq, hkv, max_seq, nch, qscale, st);
  });
  if (s != DIAL_OK || nch == 1) return s;
  DISPATCH_T(dt, {
    s = launch_pdl("attention_combine_kernel", attention_combine_kernel<T>,
                   dim3((unsigned)(tokens * hq)), dim3(128), 0, st, static_cast<const float*>(ws),
                   static_cast<T*>(out), nch);
  });
  return s;
}

size_t attention_decode_workspace_bytes(int hq, int64_t max_len) {
  // partials, then the counters at a 256-byte boundary
  return (attention_workspace_bytes(1, hq, max_len) + 255) / 256 * 256 + (size_t)hq * sizeof(int);
}

dial_status launch_attention_decode(const void* qkv, const void* qn, const void* kn,
                                    const void* cos_t, const void* sin_t, const int32_t* pos,
                                    const int32_t* slot, void* kc, void* vc, void* out, void* ws,
                                    int* ctr, dial_dtype dt, int64_t tokens, int hq, int hkv,
                                    int64_t max_seq, int64_t max_len, float eps, int qk_norm,
                                    cudaStream_t st) {
  if (tokens != 1) return fail(DIAL_ERR_SHAPE, "the fused decode attention takes one token");
  const int nch = attention_splits(tokens, hkv, max_len);  // as launch_attention
  const float qscale = 0.08837890625f;
  dim3 grid((unsigned)tokens, (unsigned)hkv, (unsigned)nch);
  const int rep = hq / hkv;
  dial_status s = DIAL_OK;
  if (dt != DIAL_F16 && dt != DIAL_BF16) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "attention: f16/bf16");
  auto run = [&](auto tag) {
    using T = decltype(tag);
    const QkvIn<T> in{static_cast<const T*>(qkv), static_cast<const T*>(qn), static_cast<const T*>(kn),
                      static_cast<const T*>(cos_t), static_cast<const T*>(sin_t), static_cast<T*>(kc),
                      static_cast<T*>(vc), ctr, eps, qk_norm};
    auto fn = rep == 1   ? launch_attention_fused_rep<T, 1>
              : rep == 2 ? launch_attention_fused_rep<T, 2>
              : rep == 4 ? launch_attention_fused_rep<T, 4>
              : rep == 8 ? launch_attention_fused_rep<T, 8>
                         : nullptr;
    if (!fn) return fail(DIAL_ERR_SHAPE, "attention supports Hq/Hkv in {1,2,4,8}");
    return fn(grid, in, pos, slot, out, ws, hq, hkv, max_seq, nch, qscale, st);
  };
  s = dt == DIAL_F16 ? run(__half{}) : run(__nv_bfloat16{});
  return s;
}

dial_status launch_swiglu(const void* gu, void* out, dial_dtype dt, int64_t tokens, int64_t inter,
                          cudaStream_t st) {
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("swiglu_kernel", swiglu_kernel<T>, dim3(grid_cap(tokens * inter, 256)), dim3(256),
                   0, st, static_cast<const T*>(gu), static_cast<T*>(out), tokens, inter);
  });
  return s;
}

dial_status launch_gather_rows(const void* src, const int32_t* idx, void* dst, dial_dtype dt,
                               int64_t rows, int64_t dim, cudaStream_t st) {
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("gather_rows_kernel", gather_rows_kernel<T>, dim3((unsigned)rows), dim3(256), 0,
                   st, static_cast<const T*>(src), idx, static_cast<T*>(dst), dim);
  });
  return s;
}

dial_status launch_add(void* out, const void* a, const void* b, dial_dtype dt, int64_t n,
                       cudaStream_t st) {
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("add_kernel", add_kernel<T>, dim3(grid_cap(n, 256)), dim3(256), 0, st,
                   static_cast<T*>(out), static_cast<const T*>(a), static_cast<const T*>(b), n);
  });
  return s;
}

dial_status launch_embedding(const void* table, const int32_t* ids, void* out, dial_dtype dt,
                             int64_t tokens, int64_t vocab, int64_t dim, cudaStream_t st) {
  int* err = device_error_ptr();
  if (!err) return fail(DIAL_ERR_CUDA, "device error flag unavailable");
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("embedding_kernel", embedding_kernel<T>, dim3((unsigned)tokens), dim3(256), 0, st,
                   static_cast<const T*>(table), ids, static_cast<T*>(out), tokens, vocab, dim, err);
  });
  return s;
}

dial_status launch_argmax(const void* x, int32_t* out, dial_dtype dt, int64_t rows, int64_t n,
                          cudaStream_t st) {
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("argmax_kernel", argmax_kernel<T>, dim3((unsigned)rows), dim3(1024), 0, st,
                   static_cast<const T*>(x), out, n);
  });
  return s;
}

dial_status launch_argmax_keys(const void* x, unsigned long long* keys, dial_dtype dt, int64_t rows,
                               int64_t n, int64_t offset, cudaStream_t st) {
  dial_status s = DIAL_OK;
  DISPATCH_T(dt, {
    s = launch_pdl("argmax_key_kernel", argmax_key_kernel<T>, dim3((unsigned)rows), dim3(1024), 0, st,
                   static_cast<const T*>(x), keys, n, offset);
  });
  return s;
}

dial_status launch_key_reduce(const unsigned long long* keys, int64_t n, int64_t elem_stride,
                              int64_t row_stride, int64_t rows, unsigned long long* keys_out,
                              int32_t* ids, cudaStream_t st) {
  return launch_pdl("key_reduce_kernel", key_reduce_kernel, dim3((unsigned)rows), dim3(256), 0, st,
                    keys, n, elem_stride, row_stride, keys_out, ids);
}

dial_status launch_rope_tables(void* cos_t, void* sin_t, dial_dtype dt, int64_t max_pos,
                               int head_dim, float theta, cudaStream_t st) {
  DISPATCH_T(dt, {
    rope_table_kernel<T><<<grid_cap(max_pos * head_dim / 2, 256), 256, 0, st>>>(
        static_cast<T*>(cos_t), static_cast<T*>(sin_t), max_pos, head_dim / 2, theta);
  });
  return check_launch("rope_table_kernel");
}

}  // namespace dial
