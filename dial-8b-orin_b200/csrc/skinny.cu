// Decode / small-M linears (M <= 32): stream the packed weights once with
// 128-bit loads, dequantise in registers and let the tensor cores do the dot
// products (mma.sync, f32 or s32 accumulate).
//
// Reference kernels this replaces:
//   dial_w8a16_decode_f16   worker_w8a16.rs:146-184 (one block per output and
//                           per activation row: weights re-read M times)
//   candle QMatMul forward  worker_gguf.rs:584-605 (rows <= 8, MMVQ)
//
// Work unit: a 16-row weight tile x one 128-wide K group.  Two drivers:
//   stream-K (default, needs a small workspace): every warp of a grid sized to
//     the SMs takes an equal contiguous range of units, so all warps finish
//     together whatever N and K are.  A tile split across warps is combined
//     deterministically: each warp stores its partial tile in its own slot,
//     bumps the tile's arrival counter, and the warp that completes the count
//     sums the slots in warp order, writes the output and resets the counter
//     (no float atomics, no waiting on other warps).
//   split (no workspace): the K groups of a tile are split over the warps of
//     one CTA and reduced through shared memory.
//
// W8A16 (f16 or bf16 activations): m16n8k16 MMAs.  Each lane loads 16
// contiguous int8 of weight rows g and g+8 (g = lane/4) per 64-wide K span;
// inside a span, MMA step s consumes bytes 4s..4s+3 of that load.  The same
// permutation of K is applied to the activation fragment (the lane loads the
// matching 16 contiguous activations), so the dot product is unchanged:
// logical k {2t, 2t+1, 2t+8, 2t+9} of step s  <->  physical 16t + 4s + {0,1,2,3}.
// Products of int8 and f16/bf16 are exact in the f32 accumulator, matching
// the reference's `(float)w * __half2float(x)` terms.
//
// GGUF (Q4_0 / Q8_0): activations are first quantised to Q8_0 blocks (as
// candle's CPU QMatMul does, k_quants vec_dot_q4_0_q8_0 / vec_dot_q8_0_q8_0),
// then every 32-wide block is one m16n8k32 s8 MMA (exact integer dot) scaled in
// f32 by d_w * d_x.  Q4_0 nibbles enter the MMA as 0..15 and the -8 offset is
// folded in as -8 * sum(x_q) per block.
#include <algorithm>

#include "common.cuh"
#include "glue.cuh"
#include "layout.cuh"
#include "quant.cuh"
#include "tma.cuh"

namespace dial {

namespace {

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 -> two packed f16x2: (b0, b1) and (b2, b3), exact.
// The byte is biased to u = b + 128 and placed under the f16 exponent of 1024,
// giving 1024 + u exactly; subtracting 1152 leaves b.
__device__ __forceinline__ void i8x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t l = prmt(u, 0x64646464u, 0x4140u);
  const uint32_t h = prmt(u, 0x64646464u, 0x4342u);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  __half2 lf = __hsub2(*reinterpret_cast<const __half2*>(&l), bias);
  __half2 hf = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
  lo = *reinterpret_cast<uint32_t*>(&lf);
  hi = *reinterpret_cast<uint32_t*>(&hf);
}

// Four int8 -> two packed bf16x2, exact.  Each byte b goes into a 16-bit lane
// under the bf16 exponent of 128: v1 = 128 + (b & 127) (bit 7 cleared), and
// v2 = -128 when b >= 0 or -256 when b < 0 (bit 7 of b moved into the exponent
// of -128); v1 + v2 = b, an integer that bf16 holds exactly.
__device__ __forceinline__ void i8x4_to_bf16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t tl = prmt(w, 0x43434343u, 0x4140u), th = prmt(w, 0x43434343u, 0x4342u);
  const uint32_t l1 = tl & 0xFF7FFF7Fu, l2 = (tl & 0x00800080u) | 0xC300C300u;
  const uint32_t h1 = th & 0xFF7FFF7Fu, h2 = (th & 0x00800080u) | 0xC300C300u;
  __nv_bfloat162 l = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&l1),
                             *reinterpret_cast<const __nv_bfloat162*>(&l2));
  __nv_bfloat162 h = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&h1),
                             *reinterpret_cast<const __nv_bfloat162*>(&h2));
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}

constexpr int kWarps = 8;
constexpr int kWarpsPerSM = 16;  // 2 CTAs of 8 warps at <= 128 registers

template <int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[NT][4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
}


// ------------------------------------------------------------------ W8A16 pieces
// acc += W[row0:row0+16, groups g0..g1) . x^T (this lane's fragment)
template <int NT, bool BF16>
__device__ __forceinline__ void w8a16_segment(const int8_t* __restrict__ q,
                                              const uint16_t* __restrict__ x, int M, int N, int K,
                                              int row0, int g0, int g1, float (&acc)[NT][4]) {
  constexpr int U = NT == 1 ? 3 : (NT == 2 ? 2 : 1);
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rlo = min(row0 + g, N - 1), rhi = min(row0 + g + 8, N - 1);
  const int8_t* wlo = q + (size_t)rlo * K;
  const int8_t* whi = q + (size_t)rhi * K;
  const uint4 z = make_uint4(0, 0, 0, 0);
  // U groups per iteration: all their loads are issued before any MMA so that
  // every lane keeps U * 64 bytes of weights in flight.
  for (int gi0 = g0; gi0 < g1; gi0 += U) {
    uint4 al[U][2], ah[U][2];
    uint4 xv[U][NT][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int gi = gi0 + u;
      const int k0 = gi * 128 + 16 * t, k1 = k0 + 64;
      const bool v0 = gi < g1 && k0 < K, v1 = gi < g1 && k1 < K;
      al[u][0] = v0 ? ld_stream16(wlo + k0) : z;
      al[u][1] = v1 ? ld_stream16(wlo + k1) : z;
      ah[u][0] = v0 ? ld_stream16(whi + k0) : z;
      ah[u][1] = v1 ? ld_stream16(whi + k1) : z;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = j * 8 + g;
        const uint16_t* xr = x + (size_t)min(tok, M - 1) * K;
        const bool tv = tok < M;
        xv[u][j][0] = (tv && v0) ? ld_ro16(xr + k0) : z;
        xv[u][j][1] = (tv && v0) ? ld_ro16(xr + k0 + 8) : z;
        xv[u][j][2] = (tv && v1) ? ld_ro16(xr + k1) : z;
        xv[u][j][3] = (tv && v1) ? ld_ro16(xr + k1 + 8) : z;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t wl = word(al[u][h], s), wh = word(ah[u][h], s);
          uint32_t a0, a1, a2, a3;
          if (BF16) {
            i8x4_to_bf16x2(wl, a0, a2);
            i8x4_to_bf16x2(wh, a1, a3);
          } else {
            i8x4_to_f16x2(wl, a0, a2);
            i8x4_to_f16x2(wh, a1, a3);
          }
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4& xs = xv[u][j][2 * h + (s >> 1)];
            const uint32_t b0 = word(xs, 2 * (s & 1)), b1 = word(xs, 2 * (s & 1) + 1);
            if (BF16) mma_bf16(acc[j], a0, a1, a2, a3, b0, b1);
            else mma_f16(acc[j], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
  }
}

// y[tok, row] = round((sum) * scale[row]) for this lane's fragment
template <int NT, bool BF16, typename ST>
__device__ __forceinline__ void w8a16_store(const float (&acc)[NT][4], const ST* __restrict__ scale,
                                            uint16_t* __restrict__ y, int M, int N, int row0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r[2] = {row0 + g, row0 + g + 8};
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    if (r[hr] >= N) continue;
    const float sc = Act<ST>::to_f32(scale[r[hr]]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = j * 8 + 2 * t + c;
        if (tok >= M) continue;
        const float v = acc[j][2 * hr + c] * sc;
        uint16_t bits;
        if (BF16) bits = __bfloat16_as_ushort(__float2bfloat16_rn(v));
        else bits = __half_as_ushort(__float2half_rn(v));
        y[(size_t)tok * N + r[hr]] = bits;
      }
    }
  }
}

// w8a16_store, plus the tile's greedy key per token (the largest argmax_key of
// its 16 rows' rounded outputs, rows numbered from key_off) in
// keys[token * tiles + tile]; y == nullptr stores no outputs.  The whole warp
// calls it.
template <int NT, bool BF16, typename ST>
__device__ __forceinline__ void w8a16_store_keys(const float (&acc)[NT][4], const ST* __restrict__ scale,
                                                 uint16_t* __restrict__ y, int M, int N, int tile,
                                                 unsigned long long* __restrict__ keys, int tiles,
                                                 long long key_off) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = tile * 16;
  const int r[2] = {row0 + g, row0 + g + 8};
  unsigned long long best[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) best[j][0] = best[j][1] = 0ull;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    if (r[hr] >= N) continue;
    const float sc = Act<ST>::to_f32(scale[r[hr]]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = j * 8 + 2 * t + c;
        if (tok >= M) continue;
        const float v = acc[j][2 * hr + c] * sc;
        uint16_t bits;
        float rv;
        if (BF16) {
          const __nv_bfloat16 h = __float2bfloat16_rn(v);
          bits = __bfloat16_as_ushort(h);
          rv = __bfloat162float(h);
        } else {
          const __half h = __float2half_rn(v);
          bits = __half_as_ushort(h);
          rv = __half2float(h);
        }
        if (y) y[(size_t)tok * N + r[hr]] = bits;
        const unsigned long long k = argmax_key(rv, key_off + r[hr]);
        best[j][c] = k > best[j][c] ? k : best[j][c];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      unsigned long long k = best[j][c];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {  // over the 8 row groups g (same t)
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
      }
      const int tok = j * 8 + 2 * t + c;
      if (g == 0 && tok < M) keys[(size_t)tok * tiles + tile] = k;
    }
}

// ------------------------------------------------------------------ GGUF pieces
template <int NT, int TYPE>
__device__ __forceinline__ void gguf_segment(const uint8_t* __restrict__ qs,
                                             const __half* __restrict__ dw,
                                             const int8_t* __restrict__ xq,
                                             const float2* __restrict__ xs, int Mp, int N, int G,
                                             int row0, int g0, int g1, float (&acc)[NT][4]) {
  constexpr int GB = TYPE == DIAL_GGML_Q4_0 ? 64 : 128;
  // groups per iteration, so every lane keeps ~8 loads of 16 bytes in flight
  constexpr int U = TYPE == DIAL_GGML_Q4_0 ? (NT <= 2 ? 4 : 2) : (NT == 1 ? 2 : 1);
  constexpr int NW = TYPE == DIAL_GGML_Q4_0 ? 1 : 2;  // 16-byte loads per row and group
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rlo = min(row0 + g, N - 1), rhi = min(row0 + g + 8, N - 1);
  const uint8_t* qlo = qs + (size_t)rlo * G * GB;
  const uint8_t* qhi = qs + (size_t)rhi * G * GB;
  for (int gi0 = g0; gi0 < g1; gi0 += U) {
    uint4 wl[U][NW], wh[U][NW];
    uint2 dl[U], dh[U];
    uint4 xv[U][NT][2];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int gi = min(gi0 + u, g1 - 1);  // clamped: a repeated group is never used
#pragma unroll
      for (int c = 0; c < NW; ++c) {
        wl[u][c] = ld_stream16(qlo + (size_t)gi * GB + (16 * NW) * t + 16 * c);
        wh[u][c] = ld_stream16(qhi + (size_t)gi * GB + (16 * NW) * t + 16 * c);
      }
      dl[u] = __ldg(reinterpret_cast<const uint2*>(dw + gguf_d_index(rlo, 4 * gi, G)));
      dh[u] = __ldg(reinterpret_cast<const uint2*>(dw + gguf_d_index(rhi, 4 * gi, G)));
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int8_t* xr = xq + (size_t)(j * 8 + g) * G * 128 + (size_t)gi * 128 + 32 * t;
        xv[u][j][0] = ld_ro16(xr);
        xv[u][j][1] = ld_ro16(xr + 16);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int gi = gi0 + u;
      if (gi >= g1) break;
      const float dlv[4] = {__low2float(*reinterpret_cast<const __half2*>(&dl[u].x)),
                            __high2float(*reinterpret_cast<const __half2*>(&dl[u].x)),
                            __low2float(*reinterpret_cast<const __half2*>(&dl[u].y)),
                            __high2float(*reinterpret_cast<const __half2*>(&dl[u].y))};
      const float dhv[4] = {__low2float(*reinterpret_cast<const __half2*>(&dh[u].x)),
                            __high2float(*reinterpret_cast<const __half2*>(&dh[u].x)),
                            __low2float(*reinterpret_cast<const __half2*>(&dh[u].y)),
                            __high2float(*reinterpret_cast<const __half2*>(&dh[u].y))};
#pragma unroll
      for (int jb = 0; jb < 4; ++jb) {
        uint32_t a0, a1, a2, a3;
        if (TYPE == DIAL_GGML_Q4_0) {
          const uint32_t l = word(wl[u][0], jb), h = word(wh[u][0], jb);
          a0 = l & 0x0F0F0F0Fu;
          a2 = (l >> 4) & 0x0F0F0F0Fu;
          a1 = h & 0x0F0F0F0Fu;
          a3 = (h >> 4) & 0x0F0F0F0Fu;
        } else {
          const uint4& l = wl[u][(jb >> 1) % NW];
          const uint4& h = wh[u][(jb >> 1) % NW];
          a0 = word(l, 2 * (jb & 1));
          a2 = word(l, 2 * (jb & 1) + 1);
          a1 = word(h, 2 * (jb & 1));
          a3 = word(h, 2 * (jb & 1) + 1);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4& xw = xv[u][j][jb >> 1];
          int c[4] = {0, 0, 0, 0};
          mma_s8(c, a0, a1, a2, a3, word(xw, 2 * (jb & 1)), word(xw, 2 * (jb & 1) + 1));
          const float4 sc = __ldg(
              reinterpret_cast<const float4*>(xs + (size_t)(gi * 4 + jb) * Mp + j * 8 + 2 * t));
          float v0 = (float)c[0], v1 = (float)c[1], v2 = (float)c[2], v3 = (float)c[3];
          if (TYPE == DIAL_GGML_Q4_0) {
            v0 = fmaf(-8.0f, sc.y, v0);
            v1 = fmaf(-8.0f, sc.w, v1);
            v2 = fmaf(-8.0f, sc.y, v2);
            v3 = fmaf(-8.0f, sc.w, v3);
          }
          acc[j][0] = fmaf(dlv[jb] * sc.x, v0, acc[j][0]);
          acc[j][1] = fmaf(dlv[jb] * sc.z, v1, acc[j][1]);
          acc[j][2] = fmaf(dhv[jb] * sc.x, v2, acc[j][2]);
          acc[j][3] = fmaf(dhv[jb] * sc.z, v3, acc[j][3]);
        }
      }
    }
  }
}

template <int NT, typename YT>
__device__ __forceinline__ void gguf_store(const float (&acc)[NT][4], YT* __restrict__ y, int M,
                                           int N, int row0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r[2] = {row0 + g, row0 + g + 8};
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    if (r[hr] >= N) continue;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = j * 8 + 2 * t + c;
        if (tok >= M) continue;
        y[(size_t)tok * N + r[hr]] = Act<YT>::from_f32(acc[j][2 * hr + c]);
      }
    }
  }
}

// ------------------------------------------------------------------ drivers
// In-CTA split: tile = blockIdx.x * (8/S) + warp/S, K groups split S ways, smem reduce.
struct SplitPlan {
  __device__ __forceinline__ static bool begin(int S, int ng, int& tile, int& g0, int& g1) {
    const int warp = threadIdx.x >> 5;
    const int tiles_per_cta = kWarps / S;
    tile = blockIdx.x * tiles_per_cta + warp / S;
    const int seg = warp % S;
    const int gps = (ng + S - 1) / S;
    g0 = seg * gps;
    g1 = min(ng, g0 + gps);
    return true;
  }
};

template <int NT>
__device__ __forceinline__ bool split_reduce(float (&acc)[NT][4], int S,
                                             float (*red)[NT][4][32]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (S == 1) return true;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp][j][e][lane] = acc[j][e];
  __syncthreads();
  if (warp % S != 0) return false;
  for (int w = 1; w < S; ++w)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] += red[warp + w][j][e][lane];
  return true;
}

// Stream-K bookkeeping: warp w owns units [u_begin(w), u_begin(w+1)),
// u_begin(w) = floor(W * w / NW), W = tiles * ng; NW <= W so no range is empty.
// ------------------------------------------------------------------ TMA-fed stream-K GEMV
// The weight matrix is cut into units of 16 rows x one 128-wide K group (2 KB
// of W8A16 / Q8_0 bytes, 1 KB of Q4_0 plus 128 B of block scales), numbered
// tile-major (unit = tile * ng + group; a tile is 16 output rows).  Warp w owns
// the contiguous range [W*w/NW, W*(w+1)/NW) of the W units (stream-K), so every
// warp streams the same number of bytes whatever the shape.  A tile done by one
// warp alone is stored directly; otherwise each contributing warp leaves its
// partial sum in a slot, and the warp whose arrival completes the tile adds
// the slots in warp order (deterministic) and stores it.
//
// CTA = up to kTmaWarps independent warps, kCtasPerSM CTAs per SM.  Each warp
// owns a ring of kStages unit buffers in shared memory; its lane 0 keeps up to
// kStages unit loads in flight (TMA boxes, no multicast) while the warp
// computes, and writes each stage's (tile, group) next to it.  Weight bytes in
// flight cost no registers: 16 warps x 4 stages x 2 KB = 128 KB per SM.
constexpr int kTmaWarps = 8;
constexpr int kCtasPerSM = 2;
constexpr int kStages = 4;        // power of two
constexpr int kUnitBytes = 2048;  // W8A16 / Q8_0 box: 128 B x 16 rows (Q4_0 uses 64 B x 16)
constexpr int kDBytes = 128;      // GGUF d of one unit: 16 rows x 4 blocks x f16
constexpr int kMinUnits = 4;      // units per warp at least
constexpr int kSlotBytes = (kSkinnyMaxM / 8) * 4 * 32 * 4;  // one partial tile at NT = 4

__host__ __device__ constexpr int ring_bytes(int nwarps) {
  return nwarps * kStages * (kUnitBytes + kDBytes + 8 + 8);
}
constexpr int kTmaSmem = ring_bytes(kTmaWarps) + 1024;  // + alignment slack

struct GemvPlan {
  int tiles;  // 16-row tiles
  int ng;     // 128-wide K groups
  int NW;     // warps
  int64_t W;  // units, tiles * ng
  int mode;   // kStreamK, or kTileCta: CTA c takes tiles c, c + C, ...; its warp j
              // the groups [ng j / 8, ng (j + 1) / 8) of each; partials meet in
              // shared memory (no global fixup)
  int C;      // CTAs (kTileCta)
};
constexpr int kStreamK = 0, kTileCta = 1;

// a / b with a 32-bit division whenever both fit (a 64-bit one is a long routine)
__device__ __forceinline__ int64_t div_u(uint64_t a, uint64_t b) {
  return (a >> 32) == 0 && (b >> 32) == 0 ? (int64_t)((uint32_t)a / (uint32_t)b) : (int64_t)(a / b);
}
__device__ __forceinline__ int64_t ubegin(const GemvPlan& p, int64_t w) {
  return div_u((uint64_t)p.W * w, (uint64_t)p.NW);
}
// warp whose range holds unit u
__device__ __forceinline__ int64_t owner(const GemvPlan& p, int64_t u) {
  return div_u((uint64_t)(u + 1) * p.NW - 1, (uint64_t)p.W);
}

struct Ring {
  uint32_t w;     // unit buffers (1024-aligned, kUnitBytes each)
  uint32_t d;     // GGUF d buffers (kDBytes each)
  uint32_t bar;   // kStages mbarriers
  uint32_t info;  // kStages x {chunk, group} (chunk -1: no more work)
};

// Layout for the launch's warp count: [unit buffers][d][barriers][info][x staging].
__device__ __forceinline__ Ring warp_ring(uint8_t* smem_raw) {
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  Ring r;
  r.w = base + (uint32_t)(warp * kStages * kUnitBytes);
  r.d = base + (uint32_t)(nw * kStages * kUnitBytes + warp * kStages * kDBytes);
  r.bar = base + (uint32_t)(nw * kStages * (kUnitBytes + kDBytes) + warp * kStages * 8);
  r.info = base + (uint32_t)(nw * kStages * (kUnitBytes + kDBytes + 8) + warp * kStages * 8);
  return r;
}

// First byte after the rings (the W8A16 activation staging area).
__device__ __forceinline__ uint32_t ring_end(uint8_t* smem_raw) {
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  return base + (uint32_t)ring_bytes(blockDim.x >> 5);
}

__device__ __forceinline__ uint4 lds16(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds8(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts8(uint32_t a, int x, int y) {
  asm volatile("st.shared.v2.s32 [%0], {%1,%2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// 16-byte chunk c of row r of a 128-byte-row box loaded with SWIZZLE_128B
__device__ __forceinline__ uint32_t sw128(uint32_t base, int r, int c) {
  return base + (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// Error path: waits (1 s in all) for every stage this warp still has in flight.
__device__ __forceinline__ void drain_ring(const Ring& ring, int first, int issued) {
  const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
  for (int i = first; i < issued; ++i)
    if (!tma::mbar_drain(ring.bar + 8u * (uint32_t)(i & (kStages - 1)), (uint32_t)((i / kStages) & 1),
                         deadline))
      return;
}

// Warp-uniform bounded wait for stage i of the ring.
__device__ __forceinline__ bool ring_wait(const Ring& ring, int i, int* err) {
  return __all_sync(0xffffffffu, tma::mbar_wait(ring.bar + 8u * (uint32_t)(i & (kStages - 1)),
                                                (uint32_t)((i / kStages) & 1), err));
}

__device__ __forceinline__ void ring_init(const Ring& ring) {
  if ((threadIdx.x & 31) == 0) {
    for (int s = 0; s < kStages; ++s) tma::mbar_init(ring.bar + 8u * s, 1);
    tma::fence_barrier_init();
    tma::fence_proxy_async();
  }
  __syncwarp();
}

// Orders lane 0's next TMA write into a stage after every lane's shared-memory
// reads of it: each lane first consumes `dep`, a value folded from every word
// it loaded from the stage (so all of its loads have returned), the warp
// synchronises, and a proxy fence orders those generic-proxy reads before the
// async-proxy (TMA) write that follows.  Lane 0's registers alone would not
// do: the warp's lanes need not execute the loads together.  Without the full
// fold and the fence, a refill overwrote a stage that some lane had not
// finished reading (wrong partial sums in about one tile per call at M = 8).
__device__ __forceinline__ uint32_t fold(const uint4& v) { return v.x ^ v.y ^ v.z ^ v.w; }
__device__ __forceinline__ uint32_t fold(const uint2& v) { return v.x ^ v.y; }
__device__ __forceinline__ void stage_reads_done(uint32_t dep) {
  asm volatile("" ::"r"(dep) : "memory");
  __syncwarp();
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Lane 0's side of a warp: which unit goes into the next stage -- the next
// unit of its static range, then the end marker.  kTile: the kernel may run a
// kTileCta plan.
template <bool kTile>
struct Producer {
  GemvPlan pl;
  int64_t su, su1;  // next unit, end
  int st, sg;       // tile and group of su
  int issued;
  bool ended;

  // kTileCta: su, su1 hold this warp's groups [su, su1) of every tile

  __device__ Producer(const GemvPlan& p, int w) : pl(p), issued(0), ended(false) {
    if (kTile && pl.mode == kTileCta) {
      const int j = w % kTmaWarps;
      su = pl.ng * j / kTmaWarps;
      su1 = pl.ng * (j + 1) / kTmaWarps;
      st = w / kTmaWarps;
      sg = (int)su;
      return;
    }
    su = ubegin(pl, w);
    su1 = ubegin(pl, w + 1);
    st = (int)div_u((uint64_t)su, (uint64_t)pl.ng);
    sg = (int)(su - (int64_t)st * pl.ng);
  }
  // One more stage: the next unit, or the end marker (a stage completed with no bytes).
  template <typename Load>
  __device__ __forceinline__ void refill(const Ring& ring, Load& load) {
    if (ended) return;
    const int s = issued & (kStages - 1);
    ++issued;
    const bool done = (kTile && pl.mode == kTileCta) ? st >= pl.tiles : su >= su1;
    if (done) {
      sts8(ring.info + 8u * (uint32_t)s, -1, 0);
      mbar_arrive(ring.bar + 8u * (uint32_t)s);
      ended = true;
      return;
    }
    sts8(ring.info + 8u * (uint32_t)s, st, sg);
    load(s, ring.bar + 8u * (uint32_t)s, st, sg);
    if (kTile && pl.mode == kTileCta) {
      if (++sg == (int)su1) {
        sg = (int)su;
        st += pl.C;
      }
      return;
    }
    if (++sg == pl.ng) {
      sg = 0;
      ++st;
    }
    ++su;
  }
};

// Tile arrival: adds `v` to the tile's count with acquire-release semantics at
// GPU scope (releases this warp's slot stores, which the preceding __syncwarp
// orders before it; acquires the other contributors').
__device__ __forceinline__ int arrive_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Adds n slots (stride NT*128 floats, addresses from slot_of(i), i = 0..n-1) in
// order; the loads of a batch are all issued before its adds.
template <int NT, typename SlotOf>
__device__ __forceinline__ void sum_slots(int n, SlotOf slot_of, float (&sum)[NT][4]) {
  const int lane = threadIdx.x & 31;
  constexpr int B = NT == 1 ? 8 : (NT == 2 ? 4 : 2);
  zero_acc(sum);
  for (int v0 = 0; v0 < n; v0 += B) {
    float part[B][NT][4];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (v0 + b < n) {
        const float* sp = slot_of(v0 + b);
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) part[b][j][e] = __ldcg(sp + (j * 4 + e) * 32 + lane);
      } else {
        zero_acc(part[b]);
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sum[j][e] += part[b][j][e];
  }
}

// Ends warp w's segment of `tile` (`units` units of it).
template <int NT, typename StoreFn>
__device__ __forceinline__ void tile_finish(const GemvPlan& pl, float* __restrict__ slots,
                                            int* __restrict__ cnt, int w, int first_tile, int tile,
                                            int units, float (&acc)[NT][4], StoreFn& store) {
  const int lane = threadIdx.x & 31;
  if (units == pl.ng) {  // the whole tile in this warp
    store(tile, acc);
    return;
  }
  float* mine = slots + ((size_t)w * 2 + (tile == first_tile ? 0 : 1)) * (NT * 128);
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) __stcg(mine + (j * 4 + e) * 32 + lane, acc[j][e]);
  __syncwarp();
  int old = 0;
  if (lane == 0) old = arrive_acq_rel(cnt + tile, units);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old + units != pl.ng) return;  // another warp completes this tile
  __syncwarp();
  const int64_t u0 = (int64_t)tile * pl.ng;
  const int64_t wa = owner(pl, u0), wb = owner(pl, u0 + pl.ng - 1);
  float sum[NT][4];
  sum_slots<NT>((int)(wb - wa + 1), [&](int i) {
    const int64_t v = wa + i;
    return slots + ((size_t)v * 2 + (ubegin(pl, v) >= u0 ? 0 : 1)) * (NT * 128);  // v starts in this tile
  }, sum);
  if (lane == 0) cnt[tile] = 0;  // ready for the next call
  store(tile, sum);
}

// Activation staging for W8A16: with XS the CTA's active warps copy x [M, K]
// (kXsBytes at most) into shared memory once, with plain loads -- a bulk copy
// would queue behind the weight prefetch in the SM's TMA unit -- and every
// lane then reads its fragments from there instead of from L1/L2 on each unit.
//
// Staged activations are f16 whatever the input dtype, and the weights enter
// the f16 MMA exactly converted (i8x4_to_f16x2).  bf16 inputs are scaled per
// token by a power of two that puts max|x| in [2^13, 2^14) and rounded to f16
// (exact for every value within 2^27 of the max); the output is scaled back by
// the same power of two.  f16 inputs are staged unscaled.  (Feeding the MMA
// biased weights 1152 + q and subtracting 1152 sum x with a second MMA saves
// the two subtractions per 4 weights, but the tensor cores accumulate the
// 40x larger biased sums inexactly: 10-15% of f16 outputs came out one ulp
// off, against 0.2% with exact weights.)
constexpr int kXsBytes = 32 * 1024;

// Barrier 1 over the first `threads` threads of the CTA (the warps with work).
__device__ __forceinline__ void active_warps_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}
__device__ __forceinline__ float lds32f(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts32f(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// kTileCta: rounds of partial tiles kept in shared memory (the staging's
// chunk-sum area, 8 KB: 512 B per warp and token group), and their counters:
// cnt[r] arrivals, done[r] the last tile round reduced in slot r.
template <int NT>
__host__ __device__ constexpr int cta_rounds() { return NT == 1 ? 2 : 1; }

__device__ __forceinline__ int atom_add_acq_rel_cta(uint32_t a, int v) {
  int old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], %2;" : "=r"(old) : "r"(a), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int ld_acquire_cta(uint32_t a) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.s32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(uint32_t a, int v) {
  asm volatile("st.release.cta.shared::cta.s32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

// Ends this warp's part of tile `tile`, the CTA's tile round `lt`: the
// partial goes to slot (lt mod R, warp); the CTA's last warp to arrive adds
// the 8 partials in warp order and stores the tile.  A warp R rounds ahead of
// the slot's reduction waits for it (bounded; the flag reports an expiry).
template <int NT, typename StoreFn>
__device__ __forceinline__ void cta_tile_finish(uint32_t part, uint32_t ctr, int lt, int tile,
                                                float (&acc)[NT][4], StoreFn& store, int* err) {
  constexpr int R = cta_rounds<NT>();
  const int lane = threadIdx.x & 31, j = (threadIdx.x >> 5) & (kTmaWarps - 1);
  const int r = lt % R;
  const uint32_t cnt = ctr + 8u * (uint32_t)r, done = cnt + 4u;
  if (lt >= R) {  // slot r must hold no unreduced round
    bool ok = true;
    if (lane == 0) {
      const unsigned long long t0 = tma::global_ns();
      while (ld_acquire_cta(done) != lt - R) {
        if (tma::global_ns() - t0 > tma::kWaitNs) {
          atomicCAS(err, 0, (int)DIAL_ERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
    if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
  }
  const uint32_t slot = part + (uint32_t)((r * kTmaWarps + j) * NT * 512);
#pragma unroll
  for (int jj = 0; jj < NT; ++jj)
#pragma unroll
    for (int e = 0; e < 4; ++e) sts32f(slot + 4u * (uint32_t)((jj * 4 + e) * 32 + lane), acc[jj][e]);
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atom_add_acq_rel_cta(cnt, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != kTmaWarps - 1) return;
  __syncwarp();
  float sum[NT][4];
  zero_acc(sum);
  for (int k = 0; k < kTmaWarps; ++k) {
    const uint32_t sk = part + (uint32_t)((r * kTmaWarps + k) * NT * 512);
#pragma unroll
    for (int jj = 0; jj < NT; ++jj)
#pragma unroll
      for (int e = 0; e < 4; ++e) sum[jj][e] += lds32f(sk + 4u * (uint32_t)((jj * 4 + e) * 32 + lane));
  }
  __syncwarp();
  if (lane == 0) {
    asm volatile("st.shared.s32 [%0], %1;" ::"r"(cnt), "r"(0) : "memory");
    st_release_cta(done, lt);
  }
  store(tile, sum);
}


// Power-of-two exponent e with 2^13 <= max|x| * 2^-e < 2^14 (0 for a zero or
// non-finite max): every bf16 value within 2^27 of the row's max is then an f16
// normal number, so the rounding to f16 is exact for all but negligible values.
__device__ __forceinline__ int tok_exp(float mx) {
  return (mx > 0.0f && isfinite(mx)) ? ilogbf(mx) - 13 : 0;
}

template <bool BF16>
__device__ __forceinline__ float act_f32(uint32_t bits16) {
  return BF16 ? __uint_as_float(bits16 << 16) : __half2float(__ushort_as_half((unsigned short)bits16));
}
template <bool BF16>
__device__ __forceinline__ uint32_t act_rnd(float v) {
  return BF16 ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v))
              : (uint32_t)__half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ uint32_t h16(const uint4& v, int i) {  // 16-bit element i of 8
  return (word(v, i >> 1) >> (16 * (i & 1))) & 0xFFFFu;
}
__device__ __forceinline__ uint4 pack8(const uint32_t (&o)[8]) {
  return make_uint4(o[0] | (o[1] << 16), o[2] | (o[3] << 16), o[4] | (o[5] << 16), o[6] | (o[7] << 16));
}

// Shared-memory scratch of the staging, after x: per-token max |input| [M],
// per-token 1/rms [M], per-token output multipliers [M], the kTileCta round
// counters, per-chunk sums of squares [M*K/8] (<= 2048 floats; after the
// staging, the kTileCta partial tiles).
constexpr int kAuxTm = 0, kAuxInv = 128, kAuxMul = 256, kAuxCnt = 384, kAuxCs = 448;
constexpr int kXsAux = kAuxCs + 2048 * 4;
constexpr int kXsSmem = kTmaSmem + kXsBytes + kXsAux;

// Stages the linear's input for rows [0, M) as f16 into xsm (see the section
// comment), with the per-token multipliers for the kernel.  The input is
// p.mode's function of x: x itself; rmsnorm(x + res) * w (the sum h = x + res,
// rounded to the activation dtype, also written to h_out by CTA 0); or swiglu
// of gate_up = x [M, 2K].  Rounding follows the standalone kernels
// (rmsnorm_kernel, swiglu_kernel): every tensor those produce is rounded to the
// activation dtype here too.  The sums of squares of a row are added in a
// fixed order (per chunk, then per warp lane, then a shuffle tree), so the
// staged values do not depend on timing.  bf16 needs max|input| per token for
// its scale: for the normalised input that is estimated as max|h w| / rms (it
// only picks a power of two).  Run by the CTA's first `active` threads; ends
// with a barrier.
// Staged chunk c (16 bytes, 8 activations) lives at slot xslot(c): within each
// 128-wide K group the 16 chunks are stored transposed (chunk 4t + i at slot
// 4i + t), so that the 4 lanes t of a fragment read load i at 4 consecutive
// 16-byte slots -- 4 different bank groups -- instead of 64 bytes apart (a
// two-way bank conflict).  Used when K % 128 == 0 (groups never straddle rows).
__device__ __forceinline__ uint32_t xslot(uint32_t c) {
  return (c & ~15u) | ((c & 3u) << 2) | ((c >> 2) & 3u);
}

// Chunks per thread whose global loads are issued together: the staging runs
// on the critical path between two linears, while the next linear's weight
// prefetch keeps the memory system busy, so every dependent L2 round trip
// costs about a microsecond.  Each pass loads a batch of its chunks' inputs
// (and the norm gains) before it uses any of them.
constexpr int kStageBatch = 4;

template <bool BF16>
__device__ __forceinline__ void stage_act(const ActPrologue& p, const uint16_t* __restrict__ x, int M,
                                          int K, uint32_t xsm_base, uint32_t aux, int active) {
  const bool perm = (K & 127) == 0;
  auto xa = [&](int c) { return xsm_base + 16u * (perm ? xslot((uint32_t)c) : (uint32_t)c); };
  const uint32_t tm = aux + kAuxTm, tinv = aux + kAuxInv, tmul = aux + kAuxMul, cs = aux + kAuxCs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarp = active >> 5;
  const int per_tok = K / 8, n16 = M * per_tok;
  // bf16 (two passes around the per-token max) measured slower batched on the
  // Qwen3-8B decode (323 against 351 tok/s): it keeps one chunk per round
  constexpr int B = BF16 ? 1 : kStageBatch;
  // per-token output multiplier 2^e (bf16) or 1, once the token's max is final
  auto put_mul = [&]() {
    if (tid < M) sts32f(tmul + 4u * tid, BF16 ? ldexpf(1.0f, tok_exp(lds32f(tm + 4u * tid))) : 1.0f);
  };
  const uint4 z = make_uint4(0, 0, 0, 0);
  unsigned int* tmax = reinterpret_cast<unsigned int*>(__cvta_shared_to_generic(tm));
  if (tid < 8) {  // kTileCta round counters: cnt[r] = 0, done[r] = r - 2 (no round yet)
    asm volatile("st.shared.s32 [%0], %1;" ::"r"(aux + kAuxCnt + 4u * (uint32_t)tid),
                 "r"((tid & 1) ? (tid >> 1) - 2 : 0)
                 : "memory");
  }
  if (BF16) {  // running max |input| per token (non-negative floats compare as ints)
    if (tid < M) sts32f(tm + 4u * tid, 0.0f);
    active_warps_sync(active);
  }
  auto amax = [&](int m, float v) {
    if (BF16) atomicMax(tmax + m, __float_as_uint(v));
  };
  // chunk b of this thread's batch starting at c0 (chunks tid, tid + active, ...)
  auto chunk = [&](int c0, int b) { return c0 + b * active; };
  if (p.mode == kProRms) {
    for (int c0 = tid; c0 < n16; c0 += B * active) {
      uint4 xv[B], rv[B], wv[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        xv[b] = rv[b] = wv[b] = z;
        if (c < n16) {
          const int m = c / per_tok, k8 = (c - m * per_tok) * 8;
          const size_t off = (size_t)m * K + (size_t)k8;
          xv[b] = ld_ro16(x + off);
          if (p.res) rv[b] = ld_ro16(p.res + off);
          wv[b] = ld_ro16(p.w + k8);
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        if (c >= n16) break;
        const int m = c / per_tok, k8 = (c - m * per_tok) * 8;
        const size_t off = (size_t)m * K + (size_t)k8;
        uint32_t o[8];
        float ss = 0.0f, mx = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float h = act_f32<BF16>(h16(xv[b], i));
          if (p.res) h = act_f32<BF16>(act_rnd<BF16>(h + act_f32<BF16>(h16(rv[b], i))));
          o[i] = act_rnd<BF16>(h);
          ss += h * h;
          mx = fmaxf(mx, fabsf(h * act_f32<BF16>(h16(wv[b], i))));
        }
        const uint4 hv = pack8(o);
        if (blockIdx.x == 0 && p.h_out) *reinterpret_cast<uint4*>(p.h_out + off) = hv;
        sts16(xa(c), hv);
        sts32f(cs + 4u * (uint32_t)c, ss);
        amax(m, mx);
      }
    }
    active_warps_sync(active);
    for (int m = warp; m < M; m += nwarp) {
      float s = 0.0f;
      for (int c = lane; c < per_tok; c += 32) s += lds32f(cs + 4u * (uint32_t)(m * per_tok + c));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) {
        const float inv = rsqrtf(s / (float)K + p.eps);
        sts32f(tinv + 4u * m, inv);
        if (BF16) sts32f(tm + 4u * m, lds32f(tm + 4u * m) * inv);
      }
    }
    active_warps_sync(active);
    put_mul();
    for (int c0 = tid; c0 < n16; c0 += B * active) {  // normalise in place, scaled to f16
      uint4 hv[B], wv[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        hv[b] = wv[b] = z;
        if (c < n16) {
          const int m = c / per_tok, k8 = (c - m * per_tok) * 8;
          hv[b] = lds16(xa(c));
          wv[b] = ld_ro16(p.w + k8);
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        if (c >= n16) break;
        const int m = c / per_tok;
        const float inv = lds32f(tinv + 4u * m);
        const int e = BF16 ? tok_exp(lds32f(tm + 4u * m)) : 0;
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float v = act_f32<BF16>(
              act_rnd<BF16>(act_f32<BF16>(h16(hv[b], i)) * inv * act_f32<BF16>(h16(wv[b], i))));
          o[i] = __half_as_ushort(__float2half_rn(BF16 ? ldexpf(v, -e) : v));
        }
        sts16(xa(c), pack8(o));
      }
    }
  } else {
    // x itself or swiglu(gate, up), rounded to the activation dtype.  f16: one
    // pass writes the staged values.  bf16: pass 1 takes the max (and keeps
    // swiglu's values in xsm, computed once), pass 2 writes the scaled f16.
    auto load8 = [&](int c, uint4& gv, uint4& uv) {
      const int m = c / per_tok, k8 = (c - m * per_tok) * 8;
      if (p.mode == kProX) {
        gv = ld_ro16(x + (size_t)m * K + k8);
      } else {
        const uint16_t* gu = x + (size_t)m * 2 * K;
        gv = ld_ro16(gu + k8);
        uv = ld_ro16(gu + K + k8);
      }
    };
    auto input8 = [&](const uint4& gv, const uint4& uv, float (&v)[8]) {
      if (p.mode == kProX) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = act_f32<BF16>(h16(gv, i));
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float gg = act_f32<BF16>(h16(gv, i));
          const float sl = act_f32<BF16>(act_rnd<BF16>(__fdividef(gg, 1.0f + __expf(-gg))));
          v[i] = act_f32<BF16>(act_rnd<BF16>(sl * act_f32<BF16>(h16(uv, i))));
        }
      }
    };
    if (BF16) {
      for (int c0 = tid; c0 < n16; c0 += B * active) {
        uint4 gv[B], uv[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          gv[b] = uv[b] = z;
          if (chunk(c0, b) < n16) load8(chunk(c0, b), gv[b], uv[b]);
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int c = chunk(c0, b);
          if (c >= n16) break;
          float v[8];
          input8(gv[b], uv[b], v);
          float mx = 0.0f;
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            mx = fmaxf(mx, fabsf(v[i]));
            o[i] = act_rnd<BF16>(v[i]);
          }
          if (p.mode != kProX) sts16(xa(c), pack8(o));
          amax(c / per_tok, mx);
        }
      }
      active_warps_sync(active);
    }
    put_mul();
    for (int c0 = tid; c0 < n16; c0 += B * active) {
      uint4 gv[B], uv[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        gv[b] = uv[b] = z;
        if (c < n16) {
          if (BF16 && p.mode != kProX) gv[b] = lds16(xa(c));
          else load8(c, gv[b], uv[b]);
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int c = chunk(c0, b);
        if (c >= n16) break;
        float v[8];
        if (BF16 && p.mode != kProX) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = act_f32<BF16>(h16(gv[b], i));
        } else {
          input8(gv[b], uv[b], v);
        }
        const int e = BF16 ? tok_exp(__uint_as_float(tmax[c / per_tok])) : 0;
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __half_as_ushort(__float2half_rn(BF16 ? ldexpf(v[i], -e) : v[i]));
        sts16(xa(c), pack8(o));
      }
    }
  }
  active_warps_sync(active);
}

// W8A16 unit: 16 rows x 128 K of int8 weights.  Lane (g, t) takes 16-byte
// chunks 2t and 2t+1 of rows g and g+8, i.e. K offsets [32t, 32t+32) of the
// group; word s of chunk 2t+h feeds MMA k-step (h, s) as K positions
// 32t + 16h + 4s + {0,1 | 2,3} <-> logical fragment columns {2t, 2t+1 | 2t+8, 2t+9},
// and the activation fragments follow the same permutation.
template <int NT, bool BF16, typename ST, bool XS>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    w8a16_tma_kernel(const __grid_constant__ CUtensorMap wmap, const ST* __restrict__ scale,
                     const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M, int N, int K,
                     GemvPlan pl, float* __restrict__ slots, int* __restrict__ cnt, int* err,
                     ActPrologue pro) {
  constexpr bool kF16Mma = XS || !BF16;  // staged activations are f16
  extern __shared__ uint8_t smem_raw[];
  const Ring ring = warp_ring(smem_raw);
  const uint32_t xsm = ring_end(smem_raw), tm = xsm + kXsBytes + kAuxMul;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wpc = blockDim.x >> 5;
  const int w = blockIdx.x * wpc + (threadIdx.x >> 5);
  pdl_trigger();
  if (w >= pl.NW) {  // only the last CTA's highest warps: no CTA-wide barrier below
    pdl_wait();
    return;
  }
  if (lane == 0) tma::prefetch_map(&wmap);
  ring_init(ring);
  Producer<XS && NT <= 2> pr(pl, w);
  auto load = [&](int s, uint32_t bar, int tile, int gi) {
    tma::mbar_expect_tx(bar, kUnitBytes);
    tma::load_2d(ring.w + (uint32_t)(s * kUnitBytes), &wmap, bar, gi * 128, tile * 16);
  };
  if (lane == 0)  // the weights are constant: prefetch before the previous kernel ends
    while (pr.issued < kStages && !pr.ended) pr.refill(ring, load);
  pdl_wait();  // x, y and the workspace belong to the stream's earlier kernels
  if (XS) stage_act<BF16>(pro, x, M, K, xsm, xsm + kXsBytes, min(wpc, pl.NW - (int)blockIdx.x * wpc) * 32);
  auto store = [&](int tile, const float (&a)[NT][4]) {
    if (XS) {  // undo the per-token power-of-two scale of the staged activations
      float b[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int t0 = j * 8 + 2 * t;
        const float m0 = t0 < M ? lds32f(tm + 4u * t0) : 1.0f, m1 = t0 + 1 < M ? lds32f(tm + 4u * (t0 + 1)) : 1.0f;
        b[j][0] = a[j][0] * m0, b[j][1] = a[j][1] * m1, b[j][2] = a[j][2] * m0, b[j][3] = a[j][3] * m1;
      }
      w8a16_store<NT, BF16, ST>(b, scale, y, M, N, tile * 16);
    } else {
      w8a16_store<NT, BF16, ST>(a, scale, y, M, N, tile * 16);
    }
  };
  const uint16_t* xr[NT];
  uint32_t xo[NT];  // XS: byte offset of this lane's token row in shared memory
  bool tv[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int tok = j * 8 + g;
    tv[j] = tok < M;
    xr[j] = x + (size_t)(tv[j] ? tok : 0) * K + 32 * t;
    xo[j] = xsm + (uint32_t)(((tv[j] ? tok : 0) * K + 32 * t) * 2);
  }
  float acc[NT][4];
  zero_acc(acc);
  const int first_tile = (int)div_u((uint64_t)ubegin(pl, w), (uint64_t)pl.ng);
  int cur = -1, units = 0, lt = 0;
  const uint4 z = make_uint4(0, 0, 0, 0);
  const uint32_t part = xsm + kXsBytes + kAuxCs, ctr = xsm + kXsBytes + kAuxCnt;
  auto finish = [&](int tile) {  // the end of this warp's part of `tile`
    if (XS && NT <= 2 && pl.mode == kTileCta) cta_tile_finish<NT>(part, ctr, lt++, tile, acc, store, err);
    else tile_finish<NT>(pl, slots, cnt, w, first_tile, tile, units, acc, store);
  };
  for (int i = 0;; ++i) {
    if (!ring_wait(ring, i, err)) {
      if (lane == 0) drain_ring(ring, i, pr.issued);
      return;
    }
    const int s = i & (kStages - 1);
    const uint2 info = lds8(ring.info + 8u * (uint32_t)s);
    const int tile = (int)info.x, gi = (int)info.y;
    if (tile < 0) break;
    if (tile != cur) {
      if (cur >= 0) finish(cur);
      zero_acc(acc);
      cur = tile;
      units = 0;
    }
    ++units;
    const int kb = gi * 128;
    const bool v0 = kb + 32 * t < K, v1 = kb + 32 * t + 16 < K;
    uint4 xv[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      if (XS) {  // staged layout: see xslot (transposed chunks when K % 128 == 0)
        const uint32_t a = xo[j] + (uint32_t)(kb * 2);
        const uint32_t ci = (K & 127) == 0 ? 64u : 16u, c0 = (K & 127) == 0 ? (uint32_t)(16 * t) - (uint32_t)(64 * t) : 0u;
        xv[j][0] = (tv[j] && v0) ? lds16(a + c0) : z;
        xv[j][1] = (tv[j] && v0) ? lds16(a + c0 + ci) : z;
        xv[j][2] = (tv[j] && v1) ? lds16(a + c0 + 2 * ci) : z;
        xv[j][3] = (tv[j] && v1) ? lds16(a + c0 + 3 * ci) : z;
      } else {
        xv[j][0] = (tv[j] && v0) ? ld_ro16(xr[j] + kb) : z;
        xv[j][1] = (tv[j] && v0) ? ld_ro16(xr[j] + kb + 8) : z;
        xv[j][2] = (tv[j] && v1) ? ld_ro16(xr[j] + kb + 16) : z;
        xv[j][3] = (tv[j] && v1) ? ld_ro16(xr[j] + kb + 24) : z;
      }
    }
    const uint32_t buf = ring.w + (uint32_t)(s * kUnitBytes);
    const uint4 al0 = lds16(sw128(buf, g, 2 * t)), al1 = lds16(sw128(buf, g, 2 * t + 1));
    const uint4 ah0 = lds16(sw128(buf, g + 8, 2 * t)), ah1 = lds16(sw128(buf, g + 8, 2 * t + 1));
    stage_reads_done(fold(al0) ^ fold(al1) ^ fold(ah0) ^ fold(ah1) ^ fold(info));
    if (lane == 0) pr.refill(ring, load);  // the stage's bytes are in registers: refill it
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const uint32_t wl = word(h ? al1 : al0, st), wh = word(h ? ah1 : ah0, st);
        uint32_t a0, a1, a2, a3;
        if (XS) {
          i8x4_to_f16x2(wl, a0, a2);
          i8x4_to_f16x2(wh, a1, a3);
        } else if (BF16) {
          i8x4_to_bf16x2(wl, a0, a2);
          i8x4_to_bf16x2(wh, a1, a3);
        } else {
          i8x4_to_f16x2(wl, a0, a2);
          i8x4_to_f16x2(wh, a1, a3);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4& xs = xv[j][2 * h + (st >> 1)];
          const uint32_t b0 = word(xs, 2 * (st & 1)), b1 = word(xs, 2 * (st & 1) + 1);
          if (kF16Mma) mma_f16(acc[j], a0, a1, a2, a3, b0, b1);
          else mma_bf16(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  }
  if (cur >= 0) finish(cur);
}

// ------------------------------------------------------------------ decode GEMV, whole tiles per CTA
// The decode linears (M <= 16 tokens, staged activations, K % 128 == 0, at
// least one 16-row tile per CTA and one 128-wide K group per warp).  CTA c
// takes the tiles c, c + C, ...; its warp j owns the K groups
// [ng j / 8, ng (j + 1) / 8) of every tile and streams them through its own
// 4-stage TMA ring, lane 0 issuing.  The warp's unit sequence (tile-major over
// its groups) is plain arithmetic, so producer and consumer walk it with
// counters and no per-stage bookkeeping.  Per 2 KB unit a lane loads its 64
// weight bytes and converts them to f16 pairs before the warp releases the
// stage (the conversions consume every loaded word), then issues its MMAs into
// 4 independent accumulator chains.  Activation fragments are read for token
// min(g, M - 1), so every MMA column holds a real (possibly repeated) token
// and no load is predicated; the staged rows use the transposed chunk layout
// (xslot), so those reads are free of bank conflicts.  The 8 partial tiles
// meet in shared memory (cta_tile_finish).  (Splitting tiles between CTAs
// balances the last wave but costs a GPU-scope fixup at each CTA's tail,
// which measured slower for every decode shape.)
template <int NT, bool BF16, typename ST>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    w8a16_gemv_kernel(const __grid_constant__ CUtensorMap wmap, const ST* __restrict__ scale,
                      const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M, int N, int K,
                      int tiles, int ng, int* err, ActPrologue pro, unsigned long long* keys,
                      long long key_off) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t ring = base + (uint32_t)(warp * kStages * kUnitBytes);
  const uint32_t bars = base + (uint32_t)(kTmaWarps * kStages * kUnitBytes + warp * kStages * 8);
  const uint32_t xsm = base + (uint32_t)(kTmaWarps * kStages * kUnitBytes + kTmaWarps * kStages * 8);
  const uint32_t aux = xsm + kXsBytes, tm = aux + kAuxMul;
  pdl_trigger();
  const int C = gridDim.x;
  const int g0 = ng * warp / kTmaWarps, g1 = ng * (warp + 1) / kTmaWarps, ngw = g1 - g0;
  const int ntile = (tiles - (int)blockIdx.x + C - 1) / C;
  const int U = ntile * ngw;  // this warp's units
  // producer (lane 0): the next unit to issue and its (tile, group)
  int pu = 0, ptile = blockIdx.x, pg = g0;
  auto issue = [&](int st) {
    const uint32_t bar = bars + 8u * (uint32_t)st;
    tma::mbar_expect_tx(bar, kUnitBytes);
    tma::load_2d(ring + (uint32_t)(st * kUnitBytes), &wmap, bar, pg * 128, ptile * 16);
    ++pu;
    if (++pg == g1) pg = g0, ptile += C;
  };
  if (lane == 0) {
    tma::prefetch_map(&wmap);
    for (int st = 0; st < kStages; ++st) tma::mbar_init(bars + 8u * st, 1);
    tma::fence_barrier_init();
    tma::fence_proxy_async();
    // the weights are constant: start streaming before the previous kernel ends
    for (int st = 0; st < kStages && pu < U; ++st) issue(st);
  }
  __syncwarp();
  pdl_wait();  // x, y and h_out belong to the stream's earlier kernels
  stage_act<BF16>(pro, x, M, K, xsm, aux, kTmaWarps * 32);
  // this lane's activation fragment rows (token min(j * 8 + g, M - 1)); load i of
  // lane t in group gi sits at slot 16 gi + 4 i + t of the token's row (xslot)
  uint32_t xo[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) xo[j] = xsm + (uint32_t)(min(j * 8 + g, M - 1) * K * 2 + 16 * t);
  // this lane's weight chunks in a stage: rows g and g + 8, 16-byte chunks 2t and 2t+1 (SWIZZLE_128B)
  const uint32_t w_lo0 = (uint32_t)(g * 128 + (((2 * t) ^ g) << 4));
  const uint32_t w_lo1 = (uint32_t)(g * 128 + (((2 * t + 1) ^ g) << 4));
  const uint32_t w_hi0 = w_lo0 + 8 * 128, w_hi1 = w_lo1 + 8 * 128;
  auto store = [&](int tile, const float (&a)[NT][4]) {
    float b[NT][4];  // undo the per-token power-of-two scale of the staged activations
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int t0 = j * 8 + 2 * t;
      const float m0 = t0 < M ? lds32f(tm + 4u * t0) : 1.0f, m1 = t0 + 1 < M ? lds32f(tm + 4u * (t0 + 1)) : 1.0f;
      b[j][0] = a[j][0] * m0, b[j][1] = a[j][1] * m1, b[j][2] = a[j][2] * m0, b[j][3] = a[j][3] * m1;
    }
    if (keys) w8a16_store_keys<NT, BF16, ST>(b, scale, y, M, N, tile, keys, tiles, key_off);
    else w8a16_store<NT, BF16, ST>(b, scale, y, M, N, tile * 16);
  };
  const uint32_t part = aux + kAuxCs, ctr = aux + kAuxCnt;
  // kChains independent accumulator chains (MMA m of a unit feeds chain m %
  // kChains): one chain would serialise a tile's MMAs on the tensor pipe's latency
  constexpr int kChains = 4;
  float acc[kChains][NT][4];
#pragma unroll
  for (int q = 0; q < kChains; ++q) zero_acc(acc[q]);
  int ctile = blockIdx.x, cg = g0, lt = 0;
  for (int u0 = 0; u0 < U; u0 += kStages) {
    const uint32_t par = (uint32_t)((u0 / kStages) & 1);
#pragma unroll
    for (int st = 0; st < kStages; ++st) {
      if (u0 + st >= U) break;
      if (!__all_sync(0xffffffffu, tma::mbar_wait(bars + 8u * st, par, err))) {
        if (lane == 0) {  // wait (bounded) for this warp's copies still in flight
          const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
          for (int v = u0 + st; v < pu; ++v)
            if (!tma::mbar_drain(bars + 8u * (uint32_t)(v & (kStages - 1)), (uint32_t)((v / kStages) & 1),
                                 deadline))
              break;
        }
        return;
      }
      const uint32_t sb = ring + (uint32_t)(st * kUnitBytes);
      const uint4 al0 = lds16(sb + w_lo0), al1 = lds16(sb + w_lo1);
      const uint4 ah0 = lds16(sb + w_hi0), ah1 = lds16(sb + w_hi1);
      uint4 xv[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint32_t a = xo[j] + (uint32_t)(cg * 256);
        xv[j][0] = lds16(a);
        xv[j][1] = lds16(a + 64);
        xv[j][2] = lds16(a + 128);
        xv[j][3] = lds16(a + 192);
      }
      // exact f16 weight pairs (this consumes every word loaded from the stage)
      uint32_t fa[2][4][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          i8x4_to_f16x2(word(h ? al1 : al0, k), fa[h][k][0], fa[h][k][2]);
          i8x4_to_f16x2(word(h ? ah1 : ah0, k), fa[h][k][1], fa[h][k][3]);
        }
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (lane == 0 && pu < U) issue(st);  // the stage is free: refill it with unit u + 4
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4& xs = xv[j][2 * h + (k >> 1)];
            mma_f16(acc[(h * 4 + k) % kChains][j], fa[h][k][0], fa[h][k][1], fa[h][k][2], fa[h][k][3],
                    word(xs, 2 * (k & 1)), word(xs, 2 * (k & 1) + 1));
          }
      if (++cg == g1) {  // the end of this warp's part of the tile
#pragma unroll
        for (int q = 1; q < kChains; ++q)
#pragma unroll
          for (int jj = 0; jj < NT; ++jj)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[0][jj][e] += acc[q][jj][e];
        cta_tile_finish<NT>(part, ctr, lt++, ctile, acc[0], store, err);
#pragma unroll
        for (int q = 0; q < kChains; ++q) zero_acc(acc[q]);
        cg = g0;
        ctile += C;
      }
    }
  }
}

template <int NT, int TYPE, typename YT>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    gguf_tma_kernel(const __grid_constant__ CUtensorMap qmap, const __half* __restrict__ dw,
                    const int8_t* __restrict__ xq, const float2* __restrict__ xs,
                    YT* __restrict__ y, int M, int Mp, int N, int G, GemvPlan pl,
                    float* __restrict__ slots, int* __restrict__ cnt, int* err) {
  constexpr int GB = TYPE == DIAL_GGML_Q4_0 ? 64 : 128;
  constexpr uint32_t BOX = GB * 16;
  extern __shared__ uint8_t smem_raw[];
  const Ring ring = warp_ring(smem_raw);
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_trigger();
  if (w >= pl.NW) {
    pdl_wait();
    return;
  }
  if (lane == 0) tma::prefetch_map(&qmap);
  ring_init(ring);
  Producer<false> pr(pl, w);
  auto load = [&](int s, uint32_t bar, int tile, int gi) {
    tma::mbar_expect_tx(bar, BOX + kDBytes);
    tma::load_2d(ring.w + (uint32_t)(s * kUnitBytes), &qmap, bar, gi * GB, tile * 16);
    // d of rows [16 tile, 16 tile + 16) x blocks [4 gi, 4 gi + 4): 128 contiguous bytes
    tma::load_1d(ring.d + (uint32_t)(s * kDBytes), dw + ((int64_t)tile * G + gi) * 64, kDBytes, bar);
  };
  if (lane == 0)  // the weights are constant: prefetch before the previous kernel ends
    while (pr.issued < kStages && !pr.ended) pr.refill(ring, load);
  pdl_wait();  // activations, y and the workspace belong to the stream's earlier kernels
  auto store = [&](int tile, const float (&a)[NT][4]) { gguf_store<NT, YT>(a, y, M, N, tile * 16); };
  float acc[NT][4];
  zero_acc(acc);
  const int first_tile = (int)div_u((uint64_t)ubegin(pl, w), (uint64_t)pl.ng);
  int cur = -1, units = 0;
  for (int i = 0;; ++i) {
    if (!ring_wait(ring, i, err)) {
      if (lane == 0) drain_ring(ring, i, pr.issued);
      return;
    }
    const int s = i & (kStages - 1);
    const uint2 info = lds8(ring.info + 8u * (uint32_t)s);
    const int tile = (int)info.x, gi = (int)info.y;
    if (tile < 0) break;
    if (tile != cur) {
      if (cur >= 0) tile_finish<NT>(pl, slots, cnt, w, first_tile, cur, units, acc, store);
      zero_acc(acc);
      cur = tile;
      units = 0;
    }
    ++units;
    // activations (with more than 2 token tiles the scales are read per block: registers)
    constexpr bool kEarlySc = NT <= 2;
    uint4 xv[NT][2];
    float4 sc[NT][kEarlySc ? 4 : 1];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int8_t* xr = xq + (size_t)(j * 8 + g) * G * 128 + (size_t)gi * 128 + 32 * t;
      xv[j][0] = ld_ro16(xr);
      xv[j][1] = ld_ro16(xr + 16);
      if (kEarlySc)
#pragma unroll
        for (int jb = 0; jb < 4; ++jb)
          sc[j][jb & (kEarlySc ? 3 : 0)] =
              __ldg(reinterpret_cast<const float4*>(xs + (size_t)(gi * 4 + jb) * Mp + j * 8 + 2 * t));
    }
    const uint32_t buf = ring.w + (uint32_t)(s * kUnitBytes);
    uint4 wl[2], wh[2];
    if (TYPE == DIAL_GGML_Q4_0) {  // 64-byte rows, no swizzle
      wl[0] = lds16(buf + (uint32_t)(g * 64 + 16 * t));
      wh[0] = lds16(buf + (uint32_t)((g + 8) * 64 + 16 * t));
      wl[1] = wh[1] = make_uint4(0, 0, 0, 0);
    } else {  // 128-byte rows, SWIZZLE_128B; lane quad t owns chunks 2t, 2t+1
      wl[0] = lds16(sw128(buf, g, 2 * t));
      wl[1] = lds16(sw128(buf, g, 2 * t + 1));
      wh[0] = lds16(sw128(buf, g + 8, 2 * t));
      wh[1] = lds16(sw128(buf, g + 8, 2 * t + 1));
    }
    const uint32_t dbuf = ring.d + (uint32_t)(s * kDBytes);
    const uint2 dl = lds8(dbuf + (uint32_t)(g * 8)), dh = lds8(dbuf + (uint32_t)((g + 8) * 8));
    stage_reads_done(fold(wl[0]) ^ fold(wl[1]) ^ fold(wh[0]) ^ fold(wh[1]) ^ fold(dl) ^ fold(dh) ^
                     fold(info));
    if (lane == 0) pr.refill(ring, load);  // the stage's bytes are in registers: refill it
    const float dlv[4] = {__low2float(*reinterpret_cast<const __half2*>(&dl.x)),
                          __high2float(*reinterpret_cast<const __half2*>(&dl.x)),
                          __low2float(*reinterpret_cast<const __half2*>(&dl.y)),
                          __high2float(*reinterpret_cast<const __half2*>(&dl.y))};
    const float dhv[4] = {__low2float(*reinterpret_cast<const __half2*>(&dh.x)),
                          __high2float(*reinterpret_cast<const __half2*>(&dh.x)),
                          __low2float(*reinterpret_cast<const __half2*>(&dh.y)),
                          __high2float(*reinterpret_cast<const __half2*>(&dh.y))};
#pragma unroll
    for (int jb = 0; jb < 4; ++jb) {
      uint32_t a0, a1, a2, a3;
      if (TYPE == DIAL_GGML_Q4_0) {
        const uint32_t l = word(wl[0], jb), h = word(wh[0], jb);
        a0 = l & 0x0F0F0F0Fu;
        a2 = (l >> 4) & 0x0F0F0F0Fu;
        a1 = h & 0x0F0F0F0Fu;
        a3 = (h >> 4) & 0x0F0F0F0Fu;
      } else {
        a0 = word(wl[jb >> 1], 2 * (jb & 1));
        a2 = word(wl[jb >> 1], 2 * (jb & 1) + 1);
        a1 = word(wh[jb >> 1], 2 * (jb & 1));
        a3 = word(wh[jb >> 1], 2 * (jb & 1) + 1);
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint4& xw = xv[j][jb >> 1];
        int cc[4] = {0, 0, 0, 0};
        mma_s8(cc, a0, a1, a2, a3, word(xw, 2 * (jb & 1)), word(xw, 2 * (jb & 1) + 1));
        const float4 scv =
            kEarlySc ? sc[j][jb & (kEarlySc ? 3 : 0)]
                     : __ldg(reinterpret_cast<const float4*>(xs + (size_t)(gi * 4 + jb) * Mp + j * 8 + 2 * t));
        float v0 = (float)cc[0], v1 = (float)cc[1], v2 = (float)cc[2], v3 = (float)cc[3];
        if (TYPE == DIAL_GGML_Q4_0) {
          v0 = fmaf(-8.0f, scv.y, v0);
          v1 = fmaf(-8.0f, scv.w, v1);
          v2 = fmaf(-8.0f, scv.y, v2);
          v3 = fmaf(-8.0f, scv.w, v3);
        }
        acc[j][0] = fmaf(dlv[jb] * scv.x, v0, acc[j][0]);
        acc[j][1] = fmaf(dlv[jb] * scv.z, v1, acc[j][1]);
        acc[j][2] = fmaf(dhv[jb] * scv.x, v2, acc[j][2]);
        acc[j][3] = fmaf(dhv[jb] * scv.z, v3, acc[j][3]);
      }
    }
  }
  if (cur >= 0) tile_finish<NT>(pl, slots, cnt, w, first_tile, cur, units, acc, store);
}

// ------------------------------------------------------------------ GGUF decode GEMV, whole tiles per CTA
// The W8A16 decode GEMV's structure (w8a16_gemv_kernel) for Q4_0 / Q8_0: CTA c
// takes 16-row tiles c, c + C, ...; warp j streams the groups [G j / 8,
// G (j + 1) / 8) of each tile, GPS groups per ring stage (2 for Q4_0, so a
// stage carries 2 KB of packed weights like Q8_0's 1; the 2D TMA box brings
// the bytes and a bulk copy on the same barrier the tile's GPS x 128 bytes of
// block scales), and the 8 partial tiles meet in shared memory.  FUSED (one
// activation row): each warp first quantises its own K range of the row to
// Q8_0 blocks in shared memory, with the arithmetic of
// q8_0_act_quantize_kernel (GGML quantize_row_q8_0_ref: d = max|x|/127, q =
// round(x * (1/d)), the f16-rounded d used in the dot), so a linear is one
// launch and the quantised row never goes to global memory; every lane then
// reads token 0's values (the MMA's 8 columns repeat it).  Otherwise the
// activations come from q8_0_act_quantize_kernel's global buffers.  Per
// 32-block: one m16n8k32 s8 MMA (exact integer dot), Q4_0's -8 folded in as
// -8 * sum(q_x), scaled in f32 by d_w * d_x.
constexpr int kGvDMax = 2 * kDBytes;                     // block scales of one stage (at most 2 groups)
constexpr int kGvDRing = kTmaWarps * kStages * kGvDMax;  // d stages of all warps
constexpr int kGgufFusedMaxK = 32768;  // the fused row staging: K bytes + K/32 * 8 bytes of smem
constexpr int kGgufGemvSmemMax = 1024 + kTmaWarps * kStages * kUnitBytes + kGvDRing + kTmaWarps * kStages * 8 +
                                 kXsAux + kGgufFusedMaxK + kGgufFusedMaxK / 32 * 8;

template <int NT, int TYPE, typename XT, typename YT, bool FUSED>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    gguf_gemv_kernel(const __grid_constant__ CUtensorMap qmap, const __half* __restrict__ dw,
                     const XT* __restrict__ x, const int8_t* __restrict__ xq_g,
                     const float2* __restrict__ xs_g, YT* __restrict__ y, int M, int Mp, int N, int K,
                     int G, int tiles, int* err) {
  constexpr int GB = TYPE == DIAL_GGML_Q4_0 ? 64 : 128;  // bytes of a group row
  // groups per stage: 2 for the fused Q4_0 row (a 2 KB stage, like Q8_0's 1
  // group); with global activations the per-stage loads are longer and more,
  // shorter tiles let the warps queue on the shared-memory reduction rounds
  constexpr int GPS = TYPE == DIAL_GGML_Q4_0 && FUSED ? 2 : 1;
  constexpr bool kSw = GB * GPS == 128;  // 128-byte box rows, SWIZZLE_128B
  constexpr uint32_t BOX = GB * GPS * 16;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t ring = base + (uint32_t)(warp * kStages * kUnitBytes);
  const uint32_t dring = base + (uint32_t)(kTmaWarps * kStages * kUnitBytes + warp * kStages * kGvDMax);
  const uint32_t bars = base + (uint32_t)(kTmaWarps * kStages * kUnitBytes + kGvDRing + warp * kStages * 8);
  const uint32_t aux = base + (uint32_t)(kTmaWarps * kStages * kUnitBytes + kGvDRing + kTmaWarps * kStages * 8);
  const uint32_t xqs = aux + kXsAux;                 // FUSED: [G * 128] int8, Q8_0 group order
  const uint32_t xss = xqs + (uint32_t)(G * 128);    // FUSED: [G * 4] {d, sum q}
  pdl_trigger();
  const int C = gridDim.x;
  const int g0 = G * warp / kTmaWarps, g1 = G * (warp + 1) / kTmaWarps;
  const int nsw = (g1 - g0) / GPS;  // stages per tile (the launcher makes G / 8 a multiple of GPS)
  const int ntile = (tiles - (int)blockIdx.x + C - 1) / C;
  const int U = ntile * nsw;
  int pu = 0, ptile = blockIdx.x, pg = g0;
  auto issue = [&](int st) {
    const uint32_t bar = bars + 8u * (uint32_t)st;
    tma::mbar_expect_tx(bar, BOX + GPS * kDBytes);
    tma::load_2d(ring + (uint32_t)(st * kUnitBytes), &qmap, bar, pg * GB, ptile * 16);
    // d of rows [16 tile, 16 tile + 16) x groups [pg, pg + GPS): GPS x 128 contiguous bytes
    tma::load_1d(dring + (uint32_t)(st * kGvDMax), dw + ((int64_t)ptile * G + pg) * 64, GPS * kDBytes, bar);
    ++pu;
    if ((pg += GPS) == g1) pg = g0, ptile += C;
  };
  if (lane == 0) {
    tma::prefetch_map(&qmap);
    for (int st = 0; st < kStages; ++st) tma::mbar_init(bars + 8u * st, 1);
    tma::fence_barrier_init();
    tma::fence_proxy_async();
    for (int st = 0; st < kStages && pu < U; ++st) issue(st);  // constant weights: before the wait
  }
  if (threadIdx.x < 8)  // cta_tile_finish round counters: cnt[r] = 0, done[r] = r - 2
    asm volatile("st.shared.s32 [%0], %1;" ::"r"(aux + kAuxCnt + 4u * threadIdx.x),
                 "r"((threadIdx.x & 1) ? (int)(threadIdx.x >> 1) - 2 : 0)
                 : "memory");
  active_warps_sync(kTmaWarps * 32);
  pdl_wait();  // activations, y and the quantised buffers belong to earlier kernels
  if (FUSED) {  // this warp's Q8_0 blocks of the row (padding blocks of the last group: zero)
    const int nb = K / kQK;
    uint8_t* xq8 = reinterpret_cast<uint8_t*>(__cvta_shared_to_generic(xqs));
    float2* ds = reinterpret_cast<float2*>(__cvta_shared_to_generic(xss));
    // a lane per block: 16-byte loads of the block's 32 activations, and the
    // quantised bytes stored as 8 words (4 consecutive elements of a block are
    // 4 consecutive bytes of the group order, q8_0_offset)
    for (int b = g0 * kBlocksPerGroup + lane; b < g1 * kBlocksPerGroup; b += 32) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(xq8 + (b >> 2) * 128);
      const int j = b & 3;
      if (b >= nb) {
#pragma unroll
        for (int w = 0; w < kQK / 4; ++w) dst[q8_0_offset(j, 4 * w) >> 2] = 0u;
        ds[b] = make_float2(0.0f, 0.0f);
        continue;
      }
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)b * kQK);
      float v[kQK];
      if constexpr (sizeof(XT) == 4) {
#pragma unroll
        for (int i = 0; i < kQK / 4; ++i) {
          const uint4 u = src[i];
          v[4 * i] = __uint_as_float(u.x), v[4 * i + 1] = __uint_as_float(u.y);
          v[4 * i + 2] = __uint_as_float(u.z), v[4 * i + 3] = __uint_as_float(u.w);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kQK / 8; ++i) {
          const uint4 u = src[i];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const unsigned short bits = (unsigned short)(word(u, k >> 1) >> (16 * (k & 1)));
            XT h;
            memcpy(&h, &bits, sizeof(bits));
            v[8 * i + k] = Act<XT>::to_f32(h);
          }
        }
      }
      float amax = 0.0f;
#pragma unroll
      for (int p = 0; p < kQK; ++p) amax = fmaxf(amax, fabsf(v[p]));
      const float dd = __fdiv_rn(amax, 127.0f);
      const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
      int sum = 0;
#pragma unroll
      for (int w = 0; w < kQK / 4; ++w) {
        uint32_t packed = 0u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int qv = (int)roundf(__fmul_rn(v[4 * w + k], id));
          sum += qv;
          packed |= (uint32_t)(uint8_t)(int8_t)qv << (8 * k);
        }
        dst[q8_0_offset(j, 4 * w) >> 2] = packed;
      }
      ds[b] = make_float2(__half2float(__float2half_rn(dd)), (float)sum);
    }
    __syncwarp();
  }
  auto store = [&](int tile, const float (&a)[NT][4]) { gguf_store<NT, YT>(a, y, M, N, tile * 16); };
  const uint32_t part = aux + kAuxCs, ctr = aux + kAuxCnt;
  // this lane's weight bytes of group h of a stage (Q4_0: 128-byte rows of 2
  // groups, 64 bytes each, SWIZZLE_128B, chunk 4h + t; Q8_0: 128-byte rows,
  // SWIZZLE_128B, chunks 2t and 2t+1)
  uint32_t w_lo[2], w_hi[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = TYPE == DIAL_GGML_Q4_0 ? 4 * h + t : 2 * t + h;
    w_lo[h] = kSw ? (uint32_t)(g * 128 + ((c ^ g) << 4)) : (uint32_t)(g * 64 + 16 * c);
    w_hi[h] = kSw ? (uint32_t)((g + 8) * 128 + ((c ^ g) << 4)) : (uint32_t)((g + 8) * 64 + 16 * c);
  }
  float acc[NT][4];
  zero_acc(acc);
  int ctile = blockIdx.x, cg = g0, lt = 0;
  for (int u0 = 0; u0 < U; u0 += kStages) {
    const uint32_t par = (uint32_t)((u0 / kStages) & 1);
#pragma unroll
    for (int st = 0; st < kStages; ++st) {
      if (u0 + st >= U) break;
      if (!__all_sync(0xffffffffu, tma::mbar_wait(bars + 8u * st, par, err))) {
        if (lane == 0) {
          const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
          for (int v = u0 + st; v < pu; ++v)
            if (!tma::mbar_drain(bars + 8u * (uint32_t)(v & (kStages - 1)), (uint32_t)((v / kStages) & 1),
                                 deadline))
              break;
        }
        return;
      }
      const uint32_t sb = ring + (uint32_t)(st * kUnitBytes), db = dring + (uint32_t)(st * kGvDMax);
      uint4 wl[2], wh[2];
      uint2 dl[GPS], dh[GPS];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (TYPE == DIAL_GGML_Q4_0 && GPS == 1 && h == 1) {
          wl[1] = wh[1] = make_uint4(0, 0, 0, 0);
        } else {
          wl[h] = lds16(sb + w_lo[h]);
          wh[h] = lds16(sb + w_hi[h]);
        }
      }
#pragma unroll
      for (int q = 0; q < GPS; ++q) {
        dl[q] = lds8(db + (uint32_t)(q * kDBytes + g * 8));
        dh[q] = lds8(db + (uint32_t)(q * kDBytes + (g + 8) * 8));
      }
      // A fragments of the stage's GPS x 4 blocks (this consumes every word loaded from it)
      uint32_t fa[GPS][4][4];
#pragma unroll
      for (int q = 0; q < GPS; ++q)
#pragma unroll
        for (int jb = 0; jb < 4; ++jb) {
          if (TYPE == DIAL_GGML_Q4_0) {
            const uint32_t l = word(wl[q], jb), h = word(wh[q], jb);
            fa[q][jb][0] = l & 0x0F0F0F0Fu;
            fa[q][jb][2] = (l >> 4) & 0x0F0F0F0Fu;
            fa[q][jb][1] = h & 0x0F0F0F0Fu;
            fa[q][jb][3] = (h >> 4) & 0x0F0F0F0Fu;
          } else {
            fa[q][jb][0] = word(wl[jb >> 1], 2 * (jb & 1));
            fa[q][jb][2] = word(wl[jb >> 1], 2 * (jb & 1) + 1);
            fa[q][jb][1] = word(wh[jb >> 1], 2 * (jb & 1));
            fa[q][jb][3] = word(wh[jb >> 1], 2 * (jb & 1) + 1);
          }
        }
      float dlv[GPS][4], dhv[GPS][4];
#pragma unroll
      for (int q = 0; q < GPS; ++q) {
        dlv[q][0] = __low2float(*reinterpret_cast<const __half2*>(&dl[q].x));
        dlv[q][1] = __high2float(*reinterpret_cast<const __half2*>(&dl[q].x));
        dlv[q][2] = __low2float(*reinterpret_cast<const __half2*>(&dl[q].y));
        dlv[q][3] = __high2float(*reinterpret_cast<const __half2*>(&dl[q].y));
        dhv[q][0] = __low2float(*reinterpret_cast<const __half2*>(&dh[q].x));
        dhv[q][1] = __high2float(*reinterpret_cast<const __half2*>(&dh[q].x));
        dhv[q][2] = __low2float(*reinterpret_cast<const __half2*>(&dh[q].y));
        dhv[q][3] = __high2float(*reinterpret_cast<const __half2*>(&dh[q].y));
      }
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (lane == 0 && pu < U) issue(st);  // the stage is free: refill it
#pragma unroll
      for (int q = 0; q < GPS; ++q) {
        const int gq = cg + q;
        // activations of group gq and their block scales
        uint4 xv[NT][2];
        float4 sc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          if (FUSED) {
            const uint32_t a = xqs + (uint32_t)(gq * 128 + 32 * t);
            xv[j][0] = lds16(a);
            xv[j][1] = lds16(a + 16);
#pragma unroll
            for (int jb = 0; jb < 4; ++jb) {
              const uint2 v2 = lds8(xss + 8u * (uint32_t)(gq * 4 + jb));
              sc[j][jb] = make_float4(__uint_as_float(v2.x), __uint_as_float(v2.y), __uint_as_float(v2.x),
                                      __uint_as_float(v2.y));
            }
          } else {
            const int8_t* xr = xq_g + (size_t)(j * 8 + g) * G * 128 + (size_t)gq * 128 + 32 * t;
            xv[j][0] = ld_ro16(xr);
            xv[j][1] = ld_ro16(xr + 16);
#pragma unroll
            for (int jb = 0; jb < 4; ++jb)
              sc[j][jb] =
                  __ldg(reinterpret_cast<const float4*>(xs_g + (size_t)(gq * 4 + jb) * Mp + j * 8 + 2 * t));
          }
        }
#pragma unroll
        for (int jb = 0; jb < 4; ++jb)
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4& xw = xv[j][jb >> 1];
            int cc[4] = {0, 0, 0, 0};
            mma_s8(cc, fa[q][jb][0], fa[q][jb][1], fa[q][jb][2], fa[q][jb][3], word(xw, 2 * (jb & 1)),
                   word(xw, 2 * (jb & 1) + 1));
            const float4 scv = sc[j][jb];
            float v0 = (float)cc[0], v1 = (float)cc[1], v2 = (float)cc[2], v3 = (float)cc[3];
            if (TYPE == DIAL_GGML_Q4_0) {
              v0 = fmaf(-8.0f, scv.y, v0);
              v1 = fmaf(-8.0f, scv.w, v1);
              v2 = fmaf(-8.0f, scv.y, v2);
              v3 = fmaf(-8.0f, scv.w, v3);
            }
            acc[j][0] = fmaf(dlv[q][jb] * scv.x, v0, acc[j][0]);
            acc[j][1] = fmaf(dlv[q][jb] * scv.z, v1, acc[j][1]);
            acc[j][2] = fmaf(dhv[q][jb] * scv.x, v2, acc[j][2]);
            acc[j][3] = fmaf(dhv[q][jb] * scv.z, v3, acc[j][3]);
          }
      }
      if ((cg += GPS) == g1) {
        cta_tile_finish<NT>(part, ctr, lt++, ctile, acc, store, err);
        zero_acc(acc);
        cg = g0;
        ctile += C;
      }
    }
  }
}

// ------------------------------------------------------------------ kernels
template <int NT, bool BF16, typename ST>
__global__ void __launch_bounds__(256, 2)
    w8a16_skinny_kernel(const int8_t* __restrict__ q, const ST* __restrict__ scale,
                        const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M, int N,
                        int K, int S) {
  pdl_begin();
  __shared__ float red[kWarps][NT][4][32];
  const int ng = (K + 127) / 128;
  int tile, g0, g1;
  SplitPlan::begin(S, ng, tile, g0, g1);
  float acc[NT][4];
  zero_acc(acc);
  if (tile * 16 < N) w8a16_segment<NT, BF16>(q, x, M, N, K, tile * 16, g0, g1, acc);
  if (!split_reduce<NT>(acc, S, red)) return;
  if (tile * 16 < N) w8a16_store<NT, BF16, ST>(acc, scale, y, M, N, tile * 16);
}

// Activation Q8_0 quantiser (GGML quantize_row_q8_0_ref arithmetic), writing
// the interleaved Q8_0 order and per-block (d_x, sum of q_x) pairs:
//   xq : int8  [Mp, G*128]
//   xs : float2[G*4, Mp]   {f32(f16 d_x), (float)sum_j q_x[j]}
// Tokens >= M and padding blocks are written as zeros.
template <typename XT>
__global__ void q8_0_act_quantize_kernel(const XT* __restrict__ x, int M, int Mp, int K, int G,
                                         int8_t* __restrict__ xq, float2* __restrict__ xs) {
  pdl_begin();
  const int nbp = G * kBlocksPerGroup, nb = K / kQK;
  const int total = Mp * nbp;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int m = i / nbp, b = i % nbp;
    const int gi = b / kBlocksPerGroup, j = b % kBlocksPerGroup;
    int8_t* dst = xq + (size_t)m * G * 128 + (size_t)gi * 128;
    if (m >= M || b >= nb) {
      for (int p = 0; p < kQK; ++p) dst[q8_0_offset(j, p)] = 0;
      xs[(size_t)b * Mp + m] = make_float2(0.0f, 0.0f);
      continue;
    }
    const XT* src = x + (size_t)m * K + (size_t)b * kQK;
    float v[kQK];
    float amax = 0.0f;
#pragma unroll
    for (int p = 0; p < kQK; ++p) {
      v[p] = Act<XT>::to_f32(src[p]);
      amax = fmaxf(amax, fabsf(v[p]));
    }
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    int sum = 0;
#pragma unroll
    for (int p = 0; p < kQK; ++p) {
      const int qv = (int)roundf(__fmul_rn(v[p], id));
      sum += qv;
      dst[q8_0_offset(j, p)] = (int8_t)qv;
    }
    xs[(size_t)b * Mp + m] = make_float2(__half2float(__float2half_rn(dd)), (float)sum);
  }
}

template <int NT, int TYPE, typename YT>
__global__ void __launch_bounds__(256, 2)
    gguf_skinny_kernel(const uint8_t* __restrict__ qs, const __half* __restrict__ dw,
                       const int8_t* __restrict__ xq, const float2* __restrict__ xs,
                       YT* __restrict__ y, int M, int Mp, int N, int G, int S) {
  pdl_begin();
  __shared__ float red[kWarps][NT][4][32];
  int tile, g0, g1;
  SplitPlan::begin(S, G, tile, g0, g1);
  float acc[NT][4];
  zero_acc(acc);
  if (tile * 16 < N) gguf_segment<NT, TYPE>(qs, dw, xq, xs, Mp, N, G, tile * 16, g0, g1, acc);
  if (!split_reduce<NT>(acc, S, red)) return;
  if (tile * 16 < N) gguf_store<NT, YT>(acc, y, M, N, tile * 16);
}

// K-split of the in-CTA driver: the fewest warps per tile that put >= ~16 warps on every SM.
int pick_split(int64_t tiles, int64_t groups) {
  const int64_t target = (int64_t)sm_count() * kWarpsPerSM;
  int S = 1;
  while (S < kWarps && tiles * S < target && groups >= 2 * S) S *= 2;
  return S;
}

// Stream-K grid: at most kCtasPerSM x kTmaWarps warps per SM, at least kMinUnits units per warp.
// tile_ok: the kernel can reduce tiles in shared memory (staged activations,
// at most 2 token groups).  With at least one tile per SM and one K group per
// warp the CTAs take whole tiles (no global fixup); otherwise stream-K.
// ------------------------------------------------------------------ Q4_K decode GEMV on tensor cores
// The Q4_K linear at M <= 8 tokens with f16/bf16 activations
// (dial_gguf_k_linear; the reference's QMatMul on Q4_K tensors,
// worker_gguf.rs:574-611).  Units of 16 rows x one super-block (16 rows x 144
// bytes: {f16 d, f16 dmin, 12 scale bytes, 128 nibble bytes}) stream through a
// per-warp 4-stage TMA ring (no swizzle; the 144-byte rows are 16-byte
// aligned), whole 16-row tiles per CTA, warp j taking super-blocks
// [nb j / 8, nb (j + 1) / 8) of every tile, as w8a16_gemv_kernel does.
//
// A super-block's weights are w = d sc_j q - dmin m_j for sub-block j (32
// weights; q a 4-bit code), so its dot product with x is
//     sum_j [ d sc_j (sum q x) - dmin m_j (sum x) ].
// Per 32-byte chunk c of the nibbles (sub-block 2c in the low nibbles, 2c + 1
// in the high ones) and k-step s, lane (g, t) takes bytes 8t + 4s .. 8t + 4s + 3
// of rows g and g + 8: the 16 k positions of a step are bytes {0-3, 8-11,
// 16-19, 24-27} (+ 4 s) of the chunk, and the activation fragment follows the
// same order (4 consecutive activations per lane).  The codes enter the MMA
// as f16 (bf16) values bias + q, exact (bias 1024 = 0x6400 in f16, 128 =
// 0x4300 in bf16, q in the mantissa), and an MMA with an all-ones A gives
// sum x of the step for every token column; per sub-block
//     acc += d sc_j * C - (bias d sc_j + dmin m_j) * S,
// C and S the sub-block's two steps of those MMAs.  f32 accumulation; the
// rows' 8 partial sums meet in shared memory (cta_tile_finish) and are
// rounded once to the activation dtype.
constexpr int kKq4Row = 144;                 // bytes of a Q4_K super-block
constexpr int kKq4Unit = 16 * kKq4Row;       // one TMA box: 16 rows x 144 bytes
constexpr int kKq4Smem = 1024 + kTmaWarps * kStages * kKq4Unit + kTmaWarps * kStages * 8 + kXsAux;

template <bool BF16>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    kq4_gemv_kernel(const __grid_constant__ CUtensorMap wmap, const uint16_t* __restrict__ x,
                    uint16_t* __restrict__ y, int M, int N, int K, int tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t ring = base + (uint32_t)(warp * kStages * kKq4Unit);
  const uint32_t bars = base + (uint32_t)(kTmaWarps * kStages * kKq4Unit + warp * kStages * 8);
  const uint32_t aux = base + (uint32_t)(kTmaWarps * kStages * kKq4Unit + kTmaWarps * kStages * 8);
  pdl_trigger();
  const int C = gridDim.x, nb = K / 256;
  const int s0 = nb * warp / kTmaWarps, s1 = nb * (warp + 1) / kTmaWarps;
  const int ntile = (tiles - (int)blockIdx.x + C - 1) / C;
  const int U = ntile * (s1 - s0);
  int pu = 0, ptile = blockIdx.x, psb = s0;
  auto issue = [&](int st) {
    const uint32_t bar = bars + 8u * (uint32_t)st;
    tma::mbar_expect_tx(bar, kKq4Unit);
    tma::load_2d(ring + (uint32_t)(st * kKq4Unit), &wmap, bar, psb * kKq4Row, ptile * 16);
    ++pu;
    if (++psb == s1) psb = s0, ptile += C;
  };
  if (lane == 0) {
    tma::prefetch_map(&wmap);
    for (int st = 0; st < kStages; ++st) tma::mbar_init(bars + 8u * st, 1);
    tma::fence_barrier_init();
    tma::fence_proxy_async();
    for (int st = 0; st < kStages && pu < U; ++st) issue(st);  // constant weights: before the wait
  }
  if (threadIdx.x < 8)  // cta_tile_finish round counters: cnt[r] = 0, done[r] = r - 2
    asm volatile("st.shared.s32 [%0], %1;" ::"r"(aux + kAuxCnt + 4u * threadIdx.x),
                 "r"((threadIdx.x & 1) ? (int)(threadIdx.x >> 1) - 2 : 0)
                 : "memory");
  active_warps_sync(kTmaWarps * 32);
  pdl_wait();  // x and y belong to the stream's earlier kernels
  constexpr uint32_t kMagic = BF16 ? 0x43004300u : 0x64006400u;  // bias + 0 in both halves
  constexpr float kBias = BF16 ? 128.0f : 1024.0f;
  constexpr uint32_t kOnes = BF16 ? 0x3F803F80u : 0x3C003C00u;
  const uint16_t* xr = x + (size_t)min(g, M - 1) * K + 8 * t;  // this lane's token row
  auto store = [&](int tile, const float (&a)[1][4]) {
    const int r0 = tile * 16 + g;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = r0 + 8 * hr;
      if (r >= N) continue;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = 2 * t + c;
        if (tok >= M) continue;
        const float v = a[0][2 * hr + c];
        y[(size_t)tok * N + r] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                      : __half_as_ushort(__float2half_rn(v));
      }
    }
  };
  const uint32_t part = aux + kAuxCs, ctr = aux + kAuxCnt;
  float acc[1][4];
  zero_acc(acc);
  int ctile = blockIdx.x, csb = s0, lt = 0;
  for (int u = 0; u < U; ++u) {
    const int st = u & (kStages - 1);
    if (!__all_sync(0xffffffffu, tma::mbar_wait(bars + 8u * (uint32_t)st, (uint32_t)((u / kStages) & 1), err))) {
      if (lane == 0) {  // wait (bounded) for this warp's copies still in flight
        const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
        for (int v = u; v < pu; ++v)
          if (!tma::mbar_drain(bars + 8u * (uint32_t)(v & (kStages - 1)), (uint32_t)((v / kStages) & 1),
                               deadline))
            break;
      }
      return;
    }
    const uint32_t ub = ring + (uint32_t)(st * kKq4Unit);
    const uint32_t rl = ub + (uint32_t)(g * kKq4Row), rh = ub + (uint32_t)((g + 8) * kKq4Row);
    const uint4 hl = lds16(rl), hh = lds16(rh);  // {d, dmin}, scales[0..11]
    uint2 ql[4], qh[4];                          // chunk c: bytes 8t .. 8t + 7
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      ql[c] = lds8(rl + (uint32_t)(16 + 32 * c + 8 * t));
      qh[c] = lds8(rh + (uint32_t)(16 + 32 * c + 8 * t));
    }
    stage_reads_done(fold(hl) ^ fold(hh) ^ fold(ql[0]) ^ fold(ql[1]) ^ fold(ql[2]) ^ fold(ql[3]) ^
                     fold(qh[0]) ^ fold(qh[1]) ^ fold(qh[2]) ^ fold(qh[3]));
    if (lane == 0 && pu < U) issue(st);  // the stage is free: refill it
    const uint16_t* xs = xr + (size_t)csb * 256;
    const float dl = __half2float(__ushort_as_half((unsigned short)(hl.x & 0xFFFFu)));
    const float ml = __half2float(__ushort_as_half((unsigned short)(hl.x >> 16)));
    const float dh = __half2float(__ushort_as_half((unsigned short)(hh.x & 0xFFFFu)));
    const float mh = __half2float(__ushort_as_half((unsigned short)(hh.x >> 16)));
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      // scales and mins of sub-blocks 2c (byte 0) and 2c + 1 (byte 1), GGML's
      // get_scale_min_k4 on two bytes at once
      const int sh = 16 * (c & 1);
      uint32_t s2[2], m2[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint4& hd = r ? hh : hl;
        const uint32_t a = (hd.y >> sh) & 0xFFFFu, b = (hd.z >> sh) & 0xFFFFu, e = (hd.w >> sh) & 0xFFFFu;
        s2[r] = c >= 2 ? ((e & 0x0F0Fu) | ((a >> 2) & 0x3030u)) : (a & 0x3F3Fu);
        m2[r] = c >= 2 ? (((e >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u)) : (b & 0x3F3Fu);
      }
      const uint4 xlo = ld_ro16(xs + 64 * c), xhi = ld_ro16(xs + 64 * c + 32);
      float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
      float sl[4] = {0.f, 0.f, 0.f, 0.f}, shh[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const uint32_t wl = s ? ql[c].y : ql[c].x, wh = s ? qh[c].y : qh[c].x;
        const uint32_t l01 = prmt(wl, 0u, 0x4140u), l23 = prmt(wl, 0u, 0x4342u);
        const uint32_t h01 = prmt(wh, 0u, 0x4140u), h23 = prmt(wh, 0u, 0x4342u);
        const uint32_t b0l = s ? xlo.z : xlo.x, b1l = s ? xlo.w : xlo.y;
        const uint32_t b0h = s ? xhi.z : xhi.x, b1h = s ? xhi.w : xhi.y;
        // low nibbles: sub-block 2c
        const uint32_t a0 = (l01 & 0x000F000Fu) | kMagic, a2 = (l23 & 0x000F000Fu) | kMagic;
        const uint32_t a1 = (h01 & 0x000F000Fu) | kMagic, a3 = (h23 & 0x000F000Fu) | kMagic;
        // high nibbles: sub-block 2c + 1
        const uint32_t e0 = ((l01 >> 4) & 0x000F000Fu) | kMagic, e2 = ((l23 >> 4) & 0x000F000Fu) | kMagic;
        const uint32_t e1 = ((h01 >> 4) & 0x000F000Fu) | kMagic, e3 = ((h23 >> 4) & 0x000F000Fu) | kMagic;
        if (BF16) {
          mma_bf16(cl, a0, a1, a2, a3, b0l, b1l);
          mma_bf16(ch, e0, e1, e2, e3, b0h, b1h);
          mma_bf16(sl, kOnes, kOnes, kOnes, kOnes, b0l, b1l);
          mma_bf16(shh, kOnes, kOnes, kOnes, kOnes, b0h, b1h);
        } else {
          mma_f16(cl, a0, a1, a2, a3, b0l, b1l);
          mma_f16(ch, e0, e1, e2, e3, b0h, b1h);
          mma_f16(sl, kOnes, kOnes, kOnes, kOnes, b0l, b1l);
          mma_f16(shh, kOnes, kOnes, kOnes, kOnes, b0h, b1h);
        }
      }
      // rows g (acc 0, 1) and g + 8 (acc 2, 3)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float d = r ? dh : dl, dm = r ? mh : ml;
        const float aL = d * (float)(s2[r] & 0xFFu), bL = fmaf(kBias, aL, dm * (float)(m2[r] & 0xFFu));
        const float aH = d * (float)(s2[r] >> 8), bH = fmaf(kBias, aH, dm * (float)(m2[r] >> 8));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float v = acc[0][2 * r + q];
          v = fmaf(aL, cl[2 * r + q], v);
          v = fmaf(-bL, sl[2 * r + q], v);
          v = fmaf(aH, ch[2 * r + q], v);
          v = fmaf(-bH, shh[2 * r + q], v);
          acc[0][2 * r + q] = v;
        }
      }
    }
    if (++csb == s1) {  // the end of this warp's part of the tile
      cta_tile_finish<1>(part, ctr, lt++, ctile, acc, store, err);
      zero_acc(acc);
      csb = s0;
      ctile += C;
    }
  }
}

// ------------------------------------------------------------------ Q6_K decode GEMV on tensor cores
// The Q6_K linear, same plan as kq4_gemv_kernel.  A Q6_K super-block (210
// bytes: ql[128] low nibbles, qh[64] high 2-bit pairs, int8 scales[16], f16 d)
// starts 2 bytes past a 16-byte boundary for odd positions, so each unit is a
// 224-byte TMA box from the boundary below it (the box x coordinate stays
// 16-byte aligned; the block sits at offset o = 210 sb mod 16 inside, past the
// end of a row the box reads the fill value), 3 stages per warp.  Element
// 128 n + 32 p + l (half n, quarter p, l < 32) has code
//     q = ((ql[64 n + 32 (p & 1) + l] >> 4 (p >> 1)) & 15) | ((qh[32 n + l] >> 2 p) & 3) << 4
// and weight d sc[8 n + 2 p + l / 16] (q - 32): each 16-element k-step is one
// scale sub-block.  Lane t takes bytes 4t .. 4t + 3 of the step's 16 ql / qh
// bytes (read as two aligned words and a funnel shift when o mod 4 = 2); the
// codes enter the MMA as bias + q (exact), an all-ones MMA gives the step's
// sum x, and acc += d sc (C - (bias + 32) S).
constexpr int kKq6Block = 210;
constexpr int kKq6Box = 224;                 // 16-byte multiple >= 210 + 14
constexpr int kKq6Unit = 16 * kKq6Box;
constexpr int kKq6Stages = 3;
constexpr int kKq6Smem = 1024 + kTmaWarps * kKq6Stages * kKq6Unit + kTmaWarps * kKq6Stages * 8 + kXsAux;

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a) {
  if ((a & 3u) == 0) return lds32(a);
  const uint32_t lo = lds32(a - 2), hi = lds32(a + 2);
  return __funnelshift_r(lo, hi, 16);
}

template <bool BF16>
__global__ void __launch_bounds__(kTmaWarps * 32, kCtasPerSM)
    kq6_gemv_kernel(const __grid_constant__ CUtensorMap wmap, const uint16_t* __restrict__ x,
                    uint16_t* __restrict__ y, int M, int N, int K, int tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (tma::smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t ring = base + (uint32_t)(warp * kKq6Stages * kKq6Unit);
  const uint32_t bars = base + (uint32_t)(kTmaWarps * kKq6Stages * kKq6Unit + warp * kKq6Stages * 8);
  const uint32_t aux = base + (uint32_t)(kTmaWarps * kKq6Stages * kKq6Unit + kTmaWarps * kKq6Stages * 8);
  pdl_trigger();
  const int C = gridDim.x, nb = K / 256;
  const int s0 = nb * warp / kTmaWarps, s1 = nb * (warp + 1) / kTmaWarps;
  const int ntile = (tiles - (int)blockIdx.x + C - 1) / C;
  const int U = ntile * (s1 - s0);
  int pu = 0, ptile = blockIdx.x, psb = s0;
  auto issue = [&](int st) {
    const uint32_t bar = bars + 8u * (uint32_t)st;
    tma::mbar_expect_tx(bar, kKq6Unit);
    tma::load_2d(ring + (uint32_t)(st * kKq6Unit), &wmap, bar, (psb * kKq6Block) & ~15, ptile * 16);
    ++pu;
    if (++psb == s1) psb = s0, ptile += C;
  };
  if (lane == 0) {
    tma::prefetch_map(&wmap);
    for (int st = 0; st < kKq6Stages; ++st) tma::mbar_init(bars + 8u * st, 1);
    tma::fence_barrier_init();
    tma::fence_proxy_async();
    for (int st = 0; st < kKq6Stages && pu < U; ++st) issue(st);  // constant weights: before the wait
  }
  if (threadIdx.x < 8)  // cta_tile_finish round counters: cnt[r] = 0, done[r] = r - 2
    asm volatile("st.shared.s32 [%0], %1;" ::"r"(aux + kAuxCnt + 4u * threadIdx.x),
                 "r"((threadIdx.x & 1) ? (int)(threadIdx.x >> 1) - 2 : 0)
                 : "memory");
  active_warps_sync(kTmaWarps * 32);
  pdl_wait();  // x and y belong to the stream's earlier kernels
  constexpr uint32_t kMagic = BF16 ? 0x43004300u : 0x64006400u;
  constexpr float kBias = BF16 ? 160.0f : 1056.0f;  // bias + 32
  constexpr uint32_t kOnes = BF16 ? 0x3F803F80u : 0x3C003C00u;
  const uint16_t* xr = x + (size_t)min(g, M - 1) * K + 4 * t;
  auto store = [&](int tile, const float (&a)[1][4]) {
    const int r0 = tile * 16 + g;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = r0 + 8 * hr;
      if (r >= N) continue;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = 2 * t + c;
        if (tok >= M) continue;
        const float v = a[0][2 * hr + c];
        y[(size_t)tok * N + r] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                      : __half_as_ushort(__float2half_rn(v));
      }
    }
  };
  const uint32_t part = aux + kAuxCs, ctr = aux + kAuxCnt;
  float acc[1][4];
  zero_acc(acc);
  int ctile = blockIdx.x, csb = s0, lt = 0;
  for (int u = 0; u < U; ++u) {
    const int st = u % kKq6Stages;
    const uint32_t par = (uint32_t)((u / kKq6Stages) & 1);
    if (!__all_sync(0xffffffffu, tma::mbar_wait(bars + 8u * (uint32_t)st, par, err))) {
      if (lane == 0) {  // wait (bounded) for this warp's copies still in flight
        const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
        for (int v = u; v < pu; ++v)
          if (!tma::mbar_drain(bars + 8u * (uint32_t)(v % kKq6Stages), (uint32_t)((v / kKq6Stages) & 1),
                               deadline))
            break;
      }
      return;
    }
    const uint32_t o = (uint32_t)((csb * kKq6Block) & 15);
    const uint32_t ub = ring + (uint32_t)(st * kKq6Unit) + o;
    uint32_t qa[2][4], qb[2][4], qhw[2][4], scw[2][4], dw[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t rb = ub + (uint32_t)((g + 8 * r) * kKq6Box);
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // i = 2 n + lh
        const int n = i >> 1, lh = i & 1;
        qa[r][i] = lds32_a2(rb + (uint32_t)(64 * n + 16 * lh + 4 * t));
        qb[r][i] = lds32_a2(rb + (uint32_t)(64 * n + 32 + 16 * lh + 4 * t));
        qhw[r][i] = lds32_a2(rb + (uint32_t)(128 + 32 * n + 16 * lh + 4 * t));
        scw[r][i] = lds32_a2(rb + (uint32_t)(192 + 4 * i));
      }
      dw[r] = lds32_a2(rb + 208u);  // d in the low half
    }
    uint32_t dep = dw[0] ^ dw[1];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int i = 0; i < 4; ++i) dep ^= qa[r][i] ^ qb[r][i] ^ qhw[r][i] ^ scw[r][i];
    stage_reads_done(dep);
    if (lane == 0 && pu < U) issue(st);  // the stage is free: refill it
    const float d[2] = {__half2float(__ushort_as_half((unsigned short)(dw[0] & 0xFFFFu))),
                        __half2float(__ushort_as_half((unsigned short)(dw[1] & 0xFFFFu)))};
    const uint16_t* xs = xr + (size_t)csb * 256;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = i >> 1, lh = i & 1;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        // this step's x: elements 128 n + 32 p + 16 lh + 4t .. + 3
        const uint2 xv = *reinterpret_cast<const uint2*>(xs + 128 * n + 32 * p + 16 * lh);
        uint32_t a[2][2];  // [row][pair: bytes 0-1 | bytes 2-3]
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint32_t ql = (p & 1) ? qb[r][i] : qa[r][i];
          const uint32_t qh = qhw[r][i];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t l2 = prmt(ql, 0u, h ? 0x4342u : 0x4140u);  // bytes -> 16-bit lanes
            const uint32_t h2 = prmt(qh, 0u, h ? 0x4342u : 0x4140u);
            const uint32_t nib = (l2 >> (4 * (p >> 1))) & 0x000F000Fu;
            const uint32_t hi = ((h2 >> (2 * p)) & 0x00030003u) << 4;
            a[r][h] = nib | hi | kMagic;
          }
        }
        float cq[4] = {0.f, 0.f, 0.f, 0.f}, sx[4] = {0.f, 0.f, 0.f, 0.f};
        if (BF16) {
          mma_bf16(cq, a[0][0], a[1][0], a[0][1], a[1][1], xv.x, xv.y);
          mma_bf16(sx, kOnes, kOnes, kOnes, kOnes, xv.x, xv.y);
        } else {
          mma_f16(cq, a[0][0], a[1][0], a[0][1], a[1][1], xv.x, xv.y);
          mma_f16(sx, kOnes, kOnes, kOnes, kOnes, xv.x, xv.y);
        }
        const int sub = 8 * n + 2 * p + lh;  // scale index, byte sub % 4 of word sub / 4
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int sc = (int)(int8_t)((scw[r][sub >> 2] >> (8 * (sub & 3))) & 0xFFu);
          const float ds = d[r] * (float)sc;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            float v = fmaf(ds, cq[2 * r + q], acc[0][2 * r + q]);
            acc[0][2 * r + q] = fmaf(-kBias * ds, sx[2 * r + q], v);
          }
        }
      }
    }
    if (++csb == s1) {  // the end of this warp's part of the tile
      cta_tile_finish<1>(part, ctr, lt++, ctile, acc, store, err);
      zero_acc(acc);
      csb = s0;
      ctile += C;
    }
  }
}

GemvPlan plan_gemv(int64_t tiles, int64_t ng, bool tile_ok) {
  const int64_t ctas = (int64_t)sm_count() * kCtasPerSM, resident = ctas * kTmaWarps;
  GemvPlan p;
  p.tiles = (int)tiles;
  p.ng = (int)ng;
  p.W = tiles * ng;
  if (tile_ok && tiles >= sm_count() && ng >= kTmaWarps) {
    p.mode = kTileCta;
    p.C = (int)std::min<int64_t>(tiles, ctas);
    p.NW = p.C * kTmaWarps;
    return p;
  }
  p.mode = kStreamK;
  p.C = 0;
  p.NW = (int)std::min<int64_t>(resident, std::max<int64_t>(1, p.W / kMinUnits));
  return p;
}

int64_t slot_bytes() { return 2ll * sm_count() * kCtasPerSM * kTmaWarps * kSlotBytes; }

// Warps per CTA: enough CTAs to reach every CTA slot before CTAs grow past one warp.
int tma_warps_per_cta(int NW) {
  const int slots = sm_count() * kCtasPerSM;
  const int wpc = (NW + slots - 1) / slots;
  return wpc < 1 ? 1 : (wpc > kTmaWarps ? kTmaWarps : wpc);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

// ------------------------------------------------------------------ workspaces
// GEMV workspace, independent of M and K so that one serves every linear of a
// model: [partial-tile slots: 2 per resident warp][tile counters, zero between calls].
size_t gemv_workspace_bytes(int64_t N) {
  const size_t cnt = (size_t)((N + 15) / 16) * sizeof(int);
  return (size_t)slot_bytes() + (size_t)round_up((int64_t)cnt, 256);
}

size_t gguf_skinny_workspace_bytes(int64_t M, int64_t K) {
  const int64_t G = gguf_groups(K);
  const int64_t Mp = round_up(M, 8);
  const size_t xq = (size_t)round_up(Mp * G * 128, 256);
  const size_t xs = (size_t)(G * 4 * Mp) * sizeof(float2);
  return xq + (size_t)round_up((int64_t)xs, 256);
}

// ------------------------------------------------------------------ launchers
// sk_ws (may be NULL): GEMV workspace of gemv_workspace_bytes(N) bytes whose
// counter part is zero (every call leaves it zero).  Given sk_ws, the TMA-fed
// dynamic-chunk kernel runs; NULL (or an unaligned weight) selects the in-CTA split.
bool w8a16_prologue_ok(int64_t M, int64_t K) { return K >= 128 && K % 16 == 0 && M * K * 2 <= kXsBytes; }

dial_status launch_w8a16_skinny(const void* x, dial_dtype xdt, const int8_t* q, const void* scale,
                                dial_dtype sdt, void* y, int64_t M, int64_t K, int64_t N,
                                cudaStream_t st, void* sk_ws, const ActPrologue* pro_in,
                                unsigned long long* keys, int64_t key_off, bool* keyed) {
  if (keyed) *keyed = false;
  const ActPrologue pro = pro_in ? *pro_in : ActPrologue{kProX, nullptr, nullptr, nullptr, 0.0f};
  if (pro.mode != kProX && !(sk_ws && aligned16(q) && aligned16(x) && w8a16_prologue_ok(M, K)))
    return fail(DIAL_ERR_SHAPE, "the fused prologue needs the staged decode path");
  const int64_t tiles = (N + 15) / 16;
  const int64_t ng = (K + 127) / 128;
  const int nt = (int)((M + 7) / 8);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  uint16_t* yp = static_cast<uint16_t*>(y);
  const bool bf = xdt == DIAL_BF16;
  dial_status s = DIAL_OK;
  if (sk_ws && K >= 128 && aligned16(q)) {
    CUtensorMap map;
    s = tma::make_byte_map(&map, q, N, K, 128, 16, 128);
    if (s != DIAL_OK) return s;
    const bool xs = M * K * 2 <= kXsBytes && aligned16(x);
    const GemvPlan pl = plan_gemv(tiles, ng, xs && nt <= 2);
    int* err0 = device_error_ptr();
    if (!err0) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
    // the decode GEMV: whole tiles per CTA (K a multiple of 128: its activation
    // fragments are read unpredicated from the staged rows)
    if (pl.mode == kTileCta && K % 128 == 0) {
      // as many CTAs as give every CTA the same number of tiles (at most the
      // resident CTAs): a last wave of a few CTAs would stream alone at a
      // fraction of the bandwidth
      const int64_t slots = (int64_t)sm_count() * kCtasPerSM, per = (tiles + slots - 1) / slots;
      const int C = (int)((tiles + per - 1) / per);
      const size_t smem = (size_t)kTmaSmem + kXsBytes + kXsAux;
      cudaError_t ae = cudaSuccess;
#define GV(NT_, BF, ST)                                                                            \
  ae = ensure_smem<w8a16_gemv_kernel<NT_, BF, ST>>((int)smem);                                     \
  if (ae == cudaSuccess)                                                                           \
    s = launch_pdl("w8a16_gemv_kernel", w8a16_gemv_kernel<NT_, BF, ST>, dim3((unsigned)C),         \
                   dim3(kTmaWarps * 32), smem, st, map, static_cast<const ST*>(scale), xp, yp,     \
                   (int)M, (int)N, (int)K, (int)tiles, (int)ng, err0, pro, keys, (long long)key_off)
#define GV_NT(BF, ST)     \
  if (nt == 1) {          \
    GV(1, BF, ST);        \
  } else {                \
    GV(2, BF, ST);        \
  }
      if (sdt == DIAL_F32) {
        if (bf) { GV_NT(true, float) } else { GV_NT(false, float) }
      } else {
        if (bf) { GV_NT(true, __half) } else { GV_NT(false, __half) }
      }
#undef GV_NT
#undef GV
      if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(w8a16_gemv_kernel)");
      if (keyed && keys && s == DIAL_OK) *keyed = true;
      return s;
    }
    if (!yp) return fail(DIAL_ERR_INVALID_ARG, "null output");
    float* slots = static_cast<float*>(sk_ws);
    int* cnt = reinterpret_cast<int*>(static_cast<uint8_t*>(sk_ws) + slot_bytes());
    int* err = device_error_ptr();
    if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
    const int wpc = pl.mode == kTileCta ? kTmaWarps : tma_warps_per_cta(pl.NW);
    const dim3 grid((unsigned)((pl.NW + wpc - 1) / wpc)), block((unsigned)(wpc * 32));
    const size_t smem = (size_t)ring_bytes(wpc) + 1024 + (xs ? kXsBytes + kXsAux : 0);
    cudaError_t ae = cudaSuccess;
#define SKX(NT_, BF, ST, XS)                                                                   \
  ae = ensure_smem<w8a16_tma_kernel<NT_, BF, ST, XS>>(XS ? kXsSmem : kTmaSmem);                \
  if (ae == cudaSuccess)                                                                       \
    s = launch_pdl("w8a16_tma_kernel", w8a16_tma_kernel<NT_, BF, ST, XS>, grid, block, smem, st, \
                   map, static_cast<const ST*>(scale), xp, yp, (int)M, (int)N, (int)K, pl,     \
                   slots, cnt, err, pro)
#define SK(NT_, BF, ST)       \
  if (xs) {                   \
    SKX(NT_, BF, ST, true);   \
  } else {                    \
    SKX(NT_, BF, ST, false);  \
  }
#define SK_NT(BF, ST)             \
  switch (nt) {                   \
    case 1: SK(1, BF, ST); break; \
    case 2: SK(2, BF, ST); break; \
    case 3: SK(3, BF, ST); break; \
    default: SK(4, BF, ST); break; \
  }
    if (sdt == DIAL_F32) {
      if (bf) { SK_NT(true, float) } else { SK_NT(false, float) }
    } else {
      if (bf) { SK_NT(true, __half) } else { SK_NT(false, __half) }
    }
#undef SK_NT
#undef SK
#undef SKX
    if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(w8a16_tma_kernel)");
    return s;
  }
  const int S = pick_split(tiles, ng);
  const int tiles_per_cta = kWarps / S;
  const dim3 grid((unsigned)((tiles + tiles_per_cta - 1) / tiles_per_cta));
#define W8(NT_, BF, ST)                                                                         \
  s = launch_pdl("w8a16_skinny_kernel", w8a16_skinny_kernel<NT_, BF, ST>, grid, dim3(256), 0, st, \
                 q, static_cast<const ST*>(scale), xp, yp, (int)M, (int)N, (int)K, S)
#define W8_NT(BF, ST)            \
  switch (nt) {                  \
    case 1: W8(1, BF, ST); break; \
    case 2: W8(2, BF, ST); break; \
    case 3: W8(3, BF, ST); break; \
    default: W8(4, BF, ST); break; \
  }
  if (sdt == DIAL_F32) {
    if (bf) { W8_NT(true, float) } else { W8_NT(false, float) }
  } else {
    if (bf) { W8_NT(true, __half) } else { W8_NT(false, __half) }
  }
#undef W8_NT
#undef W8
  return s;
}

dial_status launch_gguf_skinny(const void* x, dial_dtype xdt, const void* qs, const uint16_t* d,
                               int type, void* y, int64_t M, int64_t K, int64_t N, void* ws,
                               cudaStream_t st, void* sk_ws) {
  const int64_t G = gguf_groups(K);
  const int64_t Mp = round_up(M, 8);
  int8_t* xq = static_cast<int8_t*>(ws);
  float2* xs = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + round_up(Mp * G * 128, 256));
  dial_status s = DIAL_OK;
  const int64_t tiles = (N + 15) / 16;
  const int nt = (int)(Mp / 8);
  const uint8_t* qp = static_cast<const uint8_t*>(qs);
  const __half* dp = reinterpret_cast<const __half*>(d);
  // whole tiles per CTA from 32 tiles on (fewer CTAs than SMs still beat the
  // stream-K path's global fixups); the fused Q4_0 row takes 2 groups per
  // stage, so its groups per warp must be even
  const bool tile_mode = sk_ws && aligned16(qs) && aligned16(d) && nt <= 2 && G >= kTmaWarps &&
                         G % kTmaWarps == 0 && tiles >= 32;
  const bool fused = tile_mode && M == 1 && K <= kGgufFusedMaxK && aligned16(x) &&
                     (type != DIAL_GGML_Q4_0 || G % (2 * kTmaWarps) == 0);
  const int gps = type == DIAL_GGML_Q4_0 && fused ? 2 : 1;
  if (tile_mode) {  // the decode GEMV: whole tiles per CTA (+ the row's Q8_0 staging when fused)
    const int GB = type == DIAL_GGML_Q4_0 ? 64 : 128;
    CUtensorMap map;
    s = tma::make_byte_map(&map, qs, N, G * GB, GB * gps, 16, GB * gps == 128 ? 128 : 0);
    if (s != DIAL_OK) return s;
    int* err = device_error_ptr();
    if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
    if (!fused) {  // the rows' Q8_0 blocks into the workspace first
      const int64_t total = Mp * G * 4;
      const dim3 qgrid((unsigned)std::min<int64_t>((total + 127) / 128, (int64_t)sm_count() * 8));
      if (xdt == DIAL_F32)
        s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<float>, qgrid, dim3(128), 0,
                       st, static_cast<const float*>(x), (int)M, (int)Mp, (int)K, (int)G, xq, xs);
      else if (xdt == DIAL_F16)
        s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<__half>, qgrid, dim3(128),
                       0, st, static_cast<const __half*>(x), (int)M, (int)Mp, (int)K, (int)G, xq, xs);
      else
        s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<__nv_bfloat16>, qgrid,
                       dim3(128), 0, st, static_cast<const __nv_bfloat16*>(x), (int)M, (int)Mp, (int)K,
                       (int)G, xq, xs);
      if (s != DIAL_OK) return s;
    }
    const int C = (int)std::min<int64_t>(tiles, (int64_t)sm_count() * kCtasPerSM);
    const size_t smem = 1024 + (size_t)kTmaWarps * kStages * kUnitBytes + kGvDRing + kTmaWarps * kStages * 8 +
                        kXsAux + (fused ? (size_t)G * 128 + (size_t)G * 4 * 8 : 0);
    cudaError_t ae = cudaSuccess;
#define GV(NT_, TY, XT, FU)                                                                       \
  ae = ensure_smem<gguf_gemv_kernel<NT_, TY, XT, XT, FU>>(kGgufGemvSmemMax);                       \
  if (ae == cudaSuccess)                                                                          \
    s = launch_pdl("gguf_gemv_kernel", gguf_gemv_kernel<NT_, TY, XT, XT, FU>, dim3((unsigned)C),   \
                   dim3(kTmaWarps * 32), smem, st, map, dp, static_cast<const XT*>(x), xq, xs,    \
                   static_cast<XT*>(y), (int)M, (int)Mp, (int)N, (int)K, (int)G, (int)tiles, err)
#define GV_F(TY, XT)                \
  if (fused) {                      \
    GV(1, TY, XT, true);            \
  } else if (nt == 1) {             \
    GV(1, TY, XT, false);           \
  } else {                          \
    GV(2, TY, XT, false);           \
  }
#define GV_X(TY)                                      \
  if (xdt == DIAL_F32) { GV_F(TY, float) }            \
  else if (xdt == DIAL_F16) { GV_F(TY, __half) }      \
  else { GV_F(TY, __nv_bfloat16) }
    if (type == DIAL_GGML_Q4_0) { GV_X(DIAL_GGML_Q4_0) } else { GV_X(DIAL_GGML_Q8_0) }
#undef GV_X
#undef GV_F
#undef GV
    if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(gguf_gemv_kernel)");
    return s;
  }
  {
    const int64_t total = Mp * G * 4;
    const dim3 qgrid((unsigned)std::min<int64_t>((total + 127) / 128, (int64_t)sm_count() * 8));
    if (xdt == DIAL_F32)
      s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<float>, qgrid, dim3(128), 0,
                     st, static_cast<const float*>(x), (int)M, (int)Mp, (int)K, (int)G, xq, xs);
    else if (xdt == DIAL_F16)
      s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<__half>, qgrid, dim3(128),
                     0, st, static_cast<const __half*>(x), (int)M, (int)Mp, (int)K, (int)G, xq, xs);
    else
      s = launch_pdl("q8_0_act_quantize_kernel", q8_0_act_quantize_kernel<__nv_bfloat16>, qgrid,
                     dim3(128), 0, st, static_cast<const __nv_bfloat16*>(x), (int)M, (int)Mp, (int)K,
                     (int)G, xq, xs);
    if (s != DIAL_OK) return s;
  }
  if (sk_ws && aligned16(qs) && aligned16(d)) {
    const int GB = type == DIAL_GGML_Q4_0 ? 64 : 128;
    CUtensorMap map;
    s = tma::make_byte_map(&map, qs, N, G * GB, GB, 16, type != DIAL_GGML_Q4_0 ? 128 : 0);
    if (s != DIAL_OK) return s;
    const GemvPlan pl = plan_gemv(tiles, G, false);
    float* slots = static_cast<float*>(sk_ws);
    int* cnt = reinterpret_cast<int*>(static_cast<uint8_t*>(sk_ws) + slot_bytes());
    int* err = device_error_ptr();
    if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
    const int wpc = tma_warps_per_cta(pl.NW);
    const dim3 grid((unsigned)((pl.NW + wpc - 1) / wpc)), block((unsigned)(wpc * 32));
    const size_t smem = (size_t)ring_bytes(wpc) + 1024;
    cudaError_t ae = cudaSuccess;
#define GK(NT_, TY, YT)                                                                          \
  ae = ensure_smem<gguf_tma_kernel<NT_, TY, YT>>(kTmaSmem);                                      \
  if (ae == cudaSuccess)                                                                         \
    s = launch_pdl("gguf_tma_kernel", gguf_tma_kernel<NT_, TY, YT>, grid, block, smem, st, map,  \
                   dp, xq, xs, static_cast<YT*>(y), (int)M, (int)Mp, (int)N, (int)G, pl, slots, \
                   cnt, err)
#define GK_NT(TY, YT)             \
  switch (nt) {                   \
    case 1: GK(1, TY, YT); break; \
    case 2: GK(2, TY, YT); break; \
    case 3: GK(3, TY, YT); break; \
    default: GK(4, TY, YT); break; \
  }
#define GK_Y(TY)                                  \
  if (xdt == DIAL_F32) { GK_NT(TY, float) }       \
  else if (xdt == DIAL_F16) { GK_NT(TY, __half) } \
  else { GK_NT(TY, __nv_bfloat16) }
    if (type == DIAL_GGML_Q4_0) { GK_Y(DIAL_GGML_Q4_0) } else { GK_Y(DIAL_GGML_Q8_0) }
#undef GK_Y
#undef GK_NT
#undef GK
    if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(gguf_tma_kernel)");
    return s;
  }
  const int S = pick_split(tiles, G);
  const int tiles_per_cta = kWarps / S;
  const dim3 grid((unsigned)((tiles + tiles_per_cta - 1) / tiles_per_cta));
#define GG(NT_, TY, YT)                                                                          \
  s = launch_pdl("gguf_skinny_kernel", gguf_skinny_kernel<NT_, TY, YT>, grid, dim3(256), 0, st, qp, \
                 dp, xq, xs, static_cast<YT*>(y), (int)M, (int)Mp, (int)N, (int)G, S)
#define GG_NT(TY, YT)             \
  switch (nt) {                   \
    case 1: GG(1, TY, YT); break; \
    case 2: GG(2, TY, YT); break; \
    case 3: GG(3, TY, YT); break; \
    default: GG(4, TY, YT); break; \
  }
#define GG_Y(TY)                                       \
  if (xdt == DIAL_F32) { GG_NT(TY, float) }            \
  else if (xdt == DIAL_F16) { GG_NT(TY, __half) }      \
  else { GG_NT(TY, __nv_bfloat16) }
  if (type == DIAL_GGML_Q4_0) { GG_Y(DIAL_GGML_Q4_0) } else { GG_Y(DIAL_GGML_Q8_0) }
#undef GG_Y
#undef GG_NT
#undef GG
  return s;
}

// ------------------------------------------------------------------ Q4_K decode GEMV launcher
bool kq4_gemv_ok(int64_t M, int64_t K, int64_t N, dial_dtype xdt, const void* x, const void* blocks) {
  return M >= 1 && M <= 8 && (xdt == DIAL_F16 || xdt == DIAL_BF16) && K % 256 == 0 &&
         K / 256 >= kTmaWarps && N >= 1 && N < (1ll << 31) && K < (1ll << 31) && aligned16(x) &&
         aligned16(blocks);
}

bool kq6_gemv_ok(int64_t M, int64_t K, int64_t N, dial_dtype xdt, const void* x, const void* blocks) {
  return M >= 1 && M <= 8 && (xdt == DIAL_F16 || xdt == DIAL_BF16) && K % 2048 == 0 && N >= 1 &&
         N < (1ll << 31) && K < (1ll << 31) && aligned16(x) && aligned16(blocks);
}

dial_status launch_kq6_gemv(const void* x, dial_dtype xdt, const void* blocks, void* y, int64_t M,
                            int64_t K, int64_t N, cudaStream_t st) {
  if (!kq6_gemv_ok(M, K, N, xdt, x, blocks)) return fail(DIAL_ERR_SHAPE, "Q6_K GEMV: unsupported shape");
  CUtensorMap map;  // rows of K / 256 blocks of 210 bytes: a 16-byte multiple for K % 2048 == 0
  dial_status s = tma::make_byte_map(&map, blocks, N, (K / 256) * kKq6Block, kKq6Box, 16, 0);
  if (s != DIAL_OK) return s;
  int* err = device_error_ptr();
  if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
  const int64_t tiles = (N + 15) / 16;
  const int C = (int)std::min<int64_t>(tiles, (int64_t)sm_count() * kCtasPerSM);
  cudaError_t ae;
  if (xdt == DIAL_BF16) {
    ae = ensure_smem<kq6_gemv_kernel<true>>(kKq6Smem);
    if (ae == cudaSuccess)
      s = launch_pdl("kq6_gemv_kernel", kq6_gemv_kernel<true>, dim3((unsigned)C), dim3(kTmaWarps * 32),
                     kKq6Smem, st, map, static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), (int)M,
                     (int)N, (int)K, (int)tiles, err);
  } else {
    ae = ensure_smem<kq6_gemv_kernel<false>>(kKq6Smem);
    if (ae == cudaSuccess)
      s = launch_pdl("kq6_gemv_kernel", kq6_gemv_kernel<false>, dim3((unsigned)C), dim3(kTmaWarps * 32),
                     kKq6Smem, st, map, static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), (int)M,
                     (int)N, (int)K, (int)tiles, err);
  }
  if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(kq6_gemv_kernel)");
  return s;
}

dial_status launch_kq4_gemv(const void* x, dial_dtype xdt, const void* blocks, void* y, int64_t M,
                            int64_t K, int64_t N, cudaStream_t st) {
  if (!kq4_gemv_ok(M, K, N, xdt, x, blocks)) return fail(DIAL_ERR_SHAPE, "Q4_K GEMV: unsupported shape");
  CUtensorMap map;
  dial_status s = tma::make_byte_map(&map, blocks, N, (K / 256) * kKq4Row, kKq4Row, 16, 0);
  if (s != DIAL_OK) return s;
  int* err = device_error_ptr();
  if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
  const int64_t tiles = (N + 15) / 16;
  const int C = (int)std::min<int64_t>(tiles, (int64_t)sm_count() * kCtasPerSM);
  cudaError_t ae;
  if (xdt == DIAL_BF16) {
    ae = ensure_smem<kq4_gemv_kernel<true>>(kKq4Smem);
    if (ae == cudaSuccess)
      s = launch_pdl("kq4_gemv_kernel", kq4_gemv_kernel<true>, dim3((unsigned)C), dim3(kTmaWarps * 32),
                     kKq4Smem, st, map, static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), (int)M,
                     (int)N, (int)K, (int)tiles, err);
  } else {
    ae = ensure_smem<kq4_gemv_kernel<false>>(kKq4Smem);
    if (ae == cudaSuccess)
      s = launch_pdl("kq4_gemv_kernel", kq4_gemv_kernel<false>, dim3((unsigned)C), dim3(kTmaWarps * 32),
                     kKq4Smem, st, map, static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), (int)M,
                     (int)N, (int)K, (int)tiles, err);
  }
  if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(kq4_gemv_kernel)");
  return s;
}

}  // namespace dial
