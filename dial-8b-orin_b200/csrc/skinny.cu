// Decode / small-M linears (M <= 32): stream the packed weights once with
// 128-bit loads, dequantise in registers and let the tensor cores do the dot
// products (mma.sync, f32 or s32 accumulate).  One warp owns a 16-row tile and
// a slice of K; the K-slices of a tile are reduced through shared memory.
//
// Reference kernels this replaces:
//   dial_w8a16_decode_f16   worker_w8a16.rs:146-184 (one block per output and
//                           per activation row: weights re-read M times)
//   candle QMatMul forward  worker_gguf.rs:584-605 (rows <= 8, MMVQ)
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
#include "common.cuh"
#include "layout.cuh"
#include "quant.cuh"

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

// Four int8 -> two packed bf16x2, exact: 2^23 + u as f32 bits, minus 2^23 + 128,
// then packed (integers up to 127 are exact in bf16).
__device__ __forceinline__ void i8x4_to_bf16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float m = 8388736.0f;  // 2^23 + 128
  const float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7440u)) - m;
  const float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7441u)) - m;
  const float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7442u)) - m;
  const float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7443u)) - m;
  __nv_bfloat162 l = __floats2bfloat162_rn(f0, f1);
  __nv_bfloat162 h = __floats2bfloat162_rn(f2, f3);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}

constexpr int kWarps = 8;

// ------------------------------------------------------------------ W8A16
template <int NT, bool BF16, typename ST>
__global__ void __launch_bounds__(256, 2)
    w8a16_skinny_kernel(const int8_t* __restrict__ q, const ST* __restrict__ scale,
                        const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M, int N,
                        int K, int S) {
  constexpr int U = NT == 1 ? 3 : (NT == 2 ? 2 : 1);
  __shared__ float red[kWarps][NT][4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tiles_per_cta = kWarps / S;
  const int tile = blockIdx.x * tiles_per_cta + warp / S;
  const int seg = warp % S;
  const int row0 = tile * 16;
  const int ng = (K + 127) / 128;
  const int gps = (ng + S - 1) / S;
  const int gbeg = seg * gps;
  const int gend = min(ng, gbeg + gps);

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

  const int rlo = min(row0 + g, N - 1), rhi = min(row0 + g + 8, N - 1);
  const int8_t* wlo = q + (size_t)rlo * K;
  const int8_t* whi = q + (size_t)rhi * K;
  const uint4 z = make_uint4(0, 0, 0, 0);

  if (tile * 16 < N) {
    // U groups per iteration: all their loads are issued before any MMA so
    // that every lane keeps U * 64 bytes of weights in flight.
    for (int gi0 = gbeg; gi0 < gend; gi0 += U) {
      uint4 al[U][2], ah[U][2];
      uint4 xv[U][NT][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int gi = gi0 + u;
        const int k0 = gi * 128 + 16 * t, k1 = k0 + 64;
        const bool v0 = gi < gend && k0 < K, v1 = gi < gend && k1 < K;
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

  if (S > 1) {
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][j][e][lane] = acc[j][e];
    __syncthreads();
    if (seg != 0) return;
    for (int w = 1; w < S; ++w)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] += red[warp + w][j][e][lane];
  }
  if (row0 >= N) return;
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

// ------------------------------------------------------------------ GGUF
// Activation Q8_0 quantiser (GGML quantize_row_q8_0_ref arithmetic), writing
// the interleaved Q8_0 order and per-block (d_x, sum of q_x) pairs:
//   xq : int8  [Mp, G*128]
//   xs : float2[G*4, Mp]   {f32(f16 d_x), (float)sum_j q_x[j]}
// Tokens >= M and padding blocks are written as zeros.
template <typename XT>
__global__ void q8_0_act_quantize_kernel(const XT* __restrict__ x, int M, int Mp, int K, int G,
                                         int8_t* __restrict__ xq, float2* __restrict__ xs) {
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
  constexpr int GB = TYPE == DIAL_GGML_Q4_0 ? 64 : 128;
  // groups per iteration, so every lane keeps ~8 loads of 16 bytes in flight
  constexpr int U = TYPE == DIAL_GGML_Q4_0 ? (NT <= 2 ? 4 : 2) : (NT == 1 ? 2 : 1);
  __shared__ float red[kWarps][NT][4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tiles_per_cta = kWarps / S;
  const int tile = blockIdx.x * tiles_per_cta + warp / S;
  const int seg = warp % S;
  const int row0 = tile * 16;
  const int gps = (G + S - 1) / S;
  const int gbeg = seg * gps;
  const int gend = min(G, gbeg + gps);

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

  const int rlo = min(row0 + g, N - 1), rhi = min(row0 + g + 8, N - 1);
  const uint8_t* qlo = qs + (size_t)rlo * G * GB;
  const uint8_t* qhi = qs + (size_t)rhi * G * GB;
  const __half* dlo = dw + (size_t)rlo * G * 4;
  const __half* dhi = dw + (size_t)rhi * G * 4;

  if (row0 < N) {
    for (int gi0 = gbeg; gi0 < gend; gi0 += U) {
      constexpr int NW = TYPE == DIAL_GGML_Q4_0 ? 1 : 2;  // 16-byte loads per row and group
      uint4 wl[U][NW], wh[U][NW];
      uint2 dl[U], dh[U];
      uint4 xv[U][NT][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int gi = min(gi0 + u, gend - 1);  // clamped: a repeated group is never used
#pragma unroll
        for (int c = 0; c < NW; ++c) {
          wl[u][c] = ld_stream16(qlo + (size_t)gi * GB + (16 * NW) * t + 16 * c);
          wh[u][c] = ld_stream16(qhi + (size_t)gi * GB + (16 * NW) * t + 16 * c);
        }
        dl[u] = __ldg(reinterpret_cast<const uint2*>(dlo + (size_t)gi * 4));
        dh[u] = __ldg(reinterpret_cast<const uint2*>(dhi + (size_t)gi * 4));
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
        if (gi >= gend) break;
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

  if (S > 1) {
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][j][e][lane] = acc[j][e];
    __syncthreads();
    if (seg != 0) return;
    for (int w = 1; w < S; ++w)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] += red[warp + w][j][e][lane];
  }
  if (row0 >= N) return;
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

// K-split: the fewest warps per tile that put >= ~16 warps on every SM.
int pick_split(int64_t tiles, int64_t groups) {
  const int64_t target = (int64_t)sm_count() * 16;
  int S = 1;
  while (S < kWarps && tiles * S < target && groups >= 2 * S) S *= 2;
  return S;
}

}  // namespace

// ------------------------------------------------------------------ launchers
dial_status launch_w8a16_skinny(const void* x, dial_dtype xdt, const int8_t* q, const void* scale,
                                dial_dtype sdt, void* y, int64_t M, int64_t K, int64_t N,
                                cudaStream_t st) {
  const int64_t tiles = (N + 15) / 16;
  const int S = pick_split(tiles, (K + 127) / 128);
  const int tiles_per_cta = kWarps / S;
  const unsigned grid = (unsigned)((tiles + tiles_per_cta - 1) / tiles_per_cta);
  const int nt = (int)((M + 7) / 8);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  uint16_t* yp = static_cast<uint16_t*>(y);
#define W8(NT_, BF, ST)                                                                     \
  w8a16_skinny_kernel<NT_, BF, ST><<<grid, 256, 0, st>>>(q, static_cast<const ST*>(scale), \
                                                          xp, yp, (int)M, (int)N, (int)K, S)
#define W8_NT(BF, ST)            \
  switch (nt) {                  \
    case 1: W8(1, BF, ST); break; \
    case 2: W8(2, BF, ST); break; \
    case 3: W8(3, BF, ST); break; \
    default: W8(4, BF, ST); break; \
  }
  const bool bf = xdt == DIAL_BF16;
  if (sdt == DIAL_F32) {
    if (bf) { W8_NT(true, float) } else { W8_NT(false, float) }
  } else {
    if (bf) { W8_NT(true, __half) } else { W8_NT(false, __half) }
  }
#undef W8_NT
#undef W8
  return check_launch("w8a16_skinny_kernel");
}

static int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

size_t gguf_skinny_workspace_bytes(int64_t M, int64_t K) {
  const int64_t G = gguf_groups(K);
  const int64_t Mp = round_up(M, 8);
  const size_t xq = (size_t)round_up(Mp * G * 128, 256);
  const size_t xs = (size_t)(G * 4 * Mp) * sizeof(float2);
  return xq + xs;
}

dial_status launch_gguf_skinny(const void* x, dial_dtype xdt, const void* qs, const uint16_t* d,
                               int type, void* y, int64_t M, int64_t K, int64_t N, void* ws,
                               cudaStream_t st) {
  const int64_t G = gguf_groups(K);
  const int64_t Mp = round_up(M, 8);
  int8_t* xq = static_cast<int8_t*>(ws);
  float2* xs = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + round_up(Mp * G * 128, 256));
  {
    const int64_t total = Mp * G * 4;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 127) / 128, (int64_t)sm_count() * 8);
    if (xdt == DIAL_F32)
      q8_0_act_quantize_kernel<float><<<grid, 128, 0, st>>>(static_cast<const float*>(x), (int)M,
                                                            (int)Mp, (int)K, (int)G, xq, xs);
    else if (xdt == DIAL_F16)
      q8_0_act_quantize_kernel<__half><<<grid, 128, 0, st>>>(static_cast<const __half*>(x), (int)M,
                                                             (int)Mp, (int)K, (int)G, xq, xs);
    else
      q8_0_act_quantize_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(
          static_cast<const __nv_bfloat16*>(x), (int)M, (int)Mp, (int)K, (int)G, xq, xs);
    dial_status s = check_launch("q8_0_act_quantize_kernel");
    if (s != DIAL_OK) return s;
  }
  const int64_t tiles = (N + 15) / 16;
  const int S = pick_split(tiles, G);
  const int tiles_per_cta = kWarps / S;
  const unsigned grid = (unsigned)((tiles + tiles_per_cta - 1) / tiles_per_cta);
  const int nt = (int)(Mp / 8);
  const uint8_t* qp = static_cast<const uint8_t*>(qs);
  const __half* dp = reinterpret_cast<const __half*>(d);
#define GG(NT_, TY, YT)                                                                       \
  gguf_skinny_kernel<NT_, TY, YT><<<grid, 256, 0, st>>>(qp, dp, xq, xs, static_cast<YT*>(y), \
                                                         (int)M, (int)Mp, (int)N, (int)G, S)
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
  return check_launch("gguf_skinny_kernel");
}

}  // namespace dial
