// GGUF K-quant weights (Q4_K, Q6_K) in their native GGML super-block layout:
// bit-exact dequantisation and a decode linear that dequantises on the fly.
//
// The reference loads these formats through candle's QMatMul
// (worker_gguf.rs:462-522 load_worker_gguf_linear, forward at :574-611; the
// deployed files are Q4_K_M, docs/worker_gguf.md:1-6; its GGUF tests all use
// Q4_K, worker_gguf.rs:641-785).  The block arithmetic lives in candle-core
// 0.11.0 (not vendored); it follows the public GGML definitions:
//
//   Q4_K, 144 bytes per 256 weights: {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}
//     weight e = 64c + 32s + j (chunk c < 4, half s < 2, j < 32) is nibble s of
//     qs[32c + j]; sub-block b = e / 32 has a 6-bit scale sc_b and min m_b packed
//     in scales[] (b < 4: sc = scales[b] & 63, m = scales[b+4] & 63; b >= 4:
//     sc = (scales[b+4] & 15) | (scales[b-4] >> 6) << 4,
//     m = (scales[b+4] >> 4) | (scales[b] >> 6) << 4);
//     value = (d*sc_b) * q - (dmin*m_b), each product and the difference
//     rounded to f32 on its own.
//   Q6_K, 210 bytes per 256 weights: {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d}
//     weight e = 128h + 32g + l (h < 2, g < 4, l < 32): low 4 bits are nibble
//     g >> 1 of ql[64h + l + 32(g & 1)], high 2 bits are bits 2g..2g+1 of
//     qh[32h + l]; q = that 6-bit value - 32; value = (d*scales[e/16]) * q.
//
// The kernels use the explicitly rounded intrinsics (__fmul_rn, __fsub_rn), so
// no multiply-add is contracted and the values equal the GGML reference
// dequantisers bit for bit.  A Q4_K row is 144*K/256 bytes (16-byte aligned for
// an aligned base); a Q6_K block starts on an even byte only, so its bytes are
// read as 16-bit words.
#include "common.cuh"
#include "gemm_sm100.cuh"
#include "quant.cuh"

namespace dial {

namespace {

constexpr int kQKK = 256;  // weights per super-block

__host__ __device__ constexpr int kq_block_bytes(int type) {
  return type == DIAL_GGML_Q4_K ? 144 : type == DIAL_GGML_Q6_K ? 210 : 0;
}

// Lane `lane` of a warp owns 8 weights of one super-block:
//   Q4_K: elements 64c + j0 + i (low nibbles) and 64c + 32 + j0 + i (high
//         nibbles), i < 4, with c = lane / 8 and j0 = 4 (lane % 8): one 4-byte
//         word of qs per lane, the warp reads all 128 bytes at once;
//   Q6_K: elements 128h + 32g + l0 + i, g < 4, i < 2, with h = lane / 16 and
//         l0 = 2 (lane % 16).
// w[k] is the weight at kq_elem<TYPE>(lane, k).
template <int TYPE>
__device__ __forceinline__ int kq_elem(int lane, int k) {
  if (TYPE == DIAL_GGML_Q4_K) {
    const int c = lane >> 3, j0 = (lane & 7) * 4;
    return 64 * c + (k < 4 ? 0 : 32) + j0 + (k & 3);
  } else {
    const int h = lane >> 4, l0 = (lane & 15) * 2;
    return 128 * h + 32 * (k >> 1) + l0 + (k & 1);
  }
}

// The bytes lane `lane` needs from one super-block, loaded first (so that a
// warp can have several blocks' loads in flight) and unpacked afterwards.
//   Q4_K: the 16-byte header {d, dmin, scales[12]} (one broadcast vector load)
//         and one 4-byte word of qs;
//   Q6_K: 16-bit words of ql (two), qh, the four scales (each in its own
//         16-bit word: byte 8h + 2g + (l0 >> 4) for g < 4) and d.
template <int TYPE>
struct KqRaw;
template <>
struct KqRaw<DIAL_GGML_Q4_K> {
  uint4 hdr;
  uint32_t q;
};
template <>
struct KqRaw<DIAL_GGML_Q6_K> {
  uint32_t lo, hi, qh, sc[4], d;
};

__device__ __forceinline__ uint32_t u16_at(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

template <int TYPE>
__device__ __forceinline__ void kq_load(const uint8_t* blk, int lane, KqRaw<TYPE>& r) {
  if constexpr (TYPE == DIAL_GGML_Q4_K) {
    r.hdr = *reinterpret_cast<const uint4*>(blk);
    r.q = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * (lane >> 3) + (lane & 7) * 4);
  } else {
    const int h = lane >> 4, l0 = (lane & 15) * 2;
    r.lo = u16_at(blk + 64 * h + l0);       // ql[64h + l0 ..]
    r.hi = u16_at(blk + 64 * h + 32 + l0);  // ql[64h + 32 + l0 ..]
    r.qh = u16_at(blk + 128 + 32 * h + l0);
#pragma unroll
    for (int g = 0; g < 4; ++g) r.sc[g] = u16_at(blk + 192 + 8 * h + 2 * g);  // bytes 8h+2g, 8h+2g+1
    r.d = u16_at(blk + 208);
  }
}

// Exact float of a small unsigned integer v < 2^23 without an I2F (a slow
// pipe): 2^23 + v has v as its mantissa, and the subtraction is exact.
__device__ __forceinline__ float small_u2f(uint32_t v, float bias = 8388608.0f) {
  return __uint_as_float(0x4B000000u | v) - bias;
}

template <int TYPE>
__device__ __forceinline__ void kq_unpack(const KqRaw<TYPE>& r, int lane, float (&w)[8]) {
  if constexpr (TYPE == DIAL_GGML_Q4_K) {
    const float d = __half2float(__ushort_as_half((unsigned short)(r.hdr.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(r.hdr.x >> 16)));
    // sub-blocks j = 2c, 2c + 1 (c = lane / 8); scales[] is header bytes 4..15,
    // i.e. words y (bytes 4-7), z (8-11), w (12-15).  With jj = j mod 4 (here
    // 2 (c mod 2) and the next byte), GGML get_scale_min_k4 reads
    //   j < 4:  sc = y[jj] & 63,                   m = z[jj] & 63
    //   j >= 4: sc = (w[jj] & 15) | (y[jj] >> 6) << 4, m = (w[jj] >> 4) | (z[jj] >> 6) << 4
    // done here on both sub-blocks at once (two bytes of each word).
    const int c = lane >> 3, sh = 16 * (c & 1);
    const uint32_t a = (r.hdr.y >> sh) & 0xFFFFu, b = (r.hdr.z >> sh) & 0xFFFFu, e = (r.hdr.w >> sh) & 0xFFFFu;
    const bool hi = c >= 2;
    const uint32_t s2 = hi ? ((e & 0x0F0Fu) | ((a >> 2) & 0x3030u)) : (a & 0x3F3Fu);
    const uint32_t m2 = hi ? (((e >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u)) : (b & 0x3F3Fu);
    const float d0 = __fmul_rn(d, small_u2f(s2 & 0xFFu)), mm0 = __fmul_rn(dmin, small_u2f(m2 & 0xFFu));
    const float d1 = __fmul_rn(d, small_u2f(s2 >> 8)), mm1 = __fmul_rn(dmin, small_u2f(m2 >> 8));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = __fsub_rn(__fmul_rn(d0, small_u2f((r.q >> (8 * i)) & 15u)), mm0);
      w[4 + i] = __fsub_rn(__fmul_rn(d1, small_u2f((r.q >> (8 * i + 4)) & 15u)), mm1);
    }
  } else {
    const float d = __half2float(__ushort_as_half((unsigned short)r.d));
    const int sh = ((lane & 15) * 2) >> 4 ? 8 : 0;  // l0 >> 4 picks the high byte
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      // int8 scale: (u ^ 0x80) - 128
      const float dg = __fmul_rn(d, small_u2f(((r.sc[g] >> sh) & 0xFFu) ^ 0x80u, 8388736.0f));
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t ql = ((g & 1) ? r.hi : r.lo) >> (8 * i);
        const uint32_t low = (g >> 1) ? ((ql >> 4) & 15u) : (ql & 15u);
        const uint32_t high = (r.qh >> (8 * i + 2 * g)) & 3u;
        w[2 * g + i] = __fmul_rn(dg, small_u2f(low | (high << 4), 8388640.0f));  // q - 32
      }
    }
  }
}

template <int TYPE>
__device__ __forceinline__ void kq_dequant8(const uint8_t* blk, int lane, float (&w)[8]) {
  KqRaw<TYPE> r;
  kq_load<TYPE>(blk, lane, r);
  kq_unpack<TYPE>(r, lane, w);
}

// w[n, k] in wdt.  One warp per (row, super-block).
template <int TYPE, typename T>
__global__ void __launch_bounds__(256) kq_dequantize_kernel(const uint8_t* __restrict__ blocks,
                                                            int64_t N, int64_t nb, T* __restrict__ w) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 8;
  constexpr int BB = kq_block_bytes(TYPE);
  for (int64_t u = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); u < N * nb; u += warps) {
    float v[8];
    kq_dequant8<TYPE>(blocks + u * BB, lane, v);
    T* out = w + u * kQKK;  // row n, block b: (n * nb + b) * 256 = u * 256
#pragma unroll
    for (int k = 0; k < 8; ++k) out[kq_elem<TYPE>(lane, k)] = Act<T>::from_f32(v[k]);
  }
}

// Activations at elements e, e+1 (Q6_K) or e..e+3 (Q4_K) of one row, as f32.
template <typename T>
__device__ __forceinline__ void ld_act2(const T* p, float& a, float& b) {
  if constexpr (sizeof(T) == 4) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    a = v.x;
    b = v.y;
  } else {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    T lo, hi;
    const unsigned short l16 = (unsigned short)(u & 0xFFFFu), h16 = (unsigned short)(u >> 16);
    memcpy(&lo, &l16, 2);
    memcpy(&hi, &h16, 2);
    a = Act<T>::to_f32(lo);
    b = Act<T>::to_f32(hi);
  }
}

// y[m, n] = sum_k x[m, k] * deq(W)[n, k] in f32, rounded once to the activation
// dtype.  KS warps share an output row (8 / KS rows per CTA pass): warp part p
// takes super-blocks p, p + KS, p + 2 KS, ..., loading the bytes of four of
// them before unpacking any, so that each warp keeps four blocks' loads in
// flight.  Every lane dequantises its 8 weights of a block once and multiplies
// them into all MT activation rows (rows m >= M are skipped).  A warp's 32
// partial sums are added by a butterfly of shuffles and the KS parts of a row
// in part order through shared memory, so the summation order is fixed for a
// given K and KS.
template <int TYPE, typename T, int MT, int KS>
__global__ void __launch_bounds__(256) kq_linear_kernel(const T* __restrict__ x,
                                                        const uint8_t* __restrict__ blocks,
                                                        T* __restrict__ y, int M, int64_t K, int64_t N) {
  constexpr int RPC = 8 / KS;  // rows per CTA pass
  constexpr int BB = kq_block_bytes(TYPE);
  constexpr int U = 4;         // blocks in flight per warp
  __shared__ float part[KS > 1 ? 8 : 1][MT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = warp / KS, p = warp % KS;
  const int64_t nb = K / kQKK;
  for (int64_t n0 = (int64_t)blockIdx.x * RPC; n0 < N; n0 += (int64_t)gridDim.x * RPC) {
    const int64_t n = n0 + r;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    if (n < N) {
      const uint8_t* row = blocks + n * nb * BB;
      for (int64_t b0 = p; b0 < nb; b0 += (int64_t)U * KS) {
        KqRaw<TYPE> raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t b = b0 + (int64_t)u * KS;
          if (b < nb) kq_load<TYPE>(row + b * BB, lane, raw[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t b = b0 + (int64_t)u * KS;
          if (b < nb) {
            float w[8];
            kq_unpack<TYPE>(raw[u], lane, w);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              if (m < M) {
                const T* xr = x + (int64_t)m * K + b * kQKK;
                float a[8];
#pragma unroll
                for (int k = 0; k < 8; k += 2) ld_act2(xr + kq_elem<TYPE>(lane, k), a[k], a[k + 1]);
#pragma unroll
                for (int k = 0; k < 8; ++k) acc[m] = fmaf(w[k], a[k], acc[m]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    if constexpr (KS == 1) {
      if (lane == 0 && n < N)
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (m < M) y[(int64_t)m * N + n] = Act<T>::from_f32(acc[m]);
    } else {
      if (lane == 0)
#pragma unroll
        for (int m = 0; m < MT; ++m) part[warp][m] = acc[m];
      __syncthreads();
      if (p == 0 && lane == 0 && n < N) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            float v = part[warp][m];
#pragma unroll
            for (int q = 1; q < KS; ++q) v += part[warp + q][m];
            y[(int64_t)m * N + n] = Act<T>::from_f32(v);
          }
        }
      }
      __syncthreads();  // part[] is rewritten by the next pass
    }
  }
}

template <int TYPE, typename T>
dial_status launch_kq_dequant_t(const void* blocks, int64_t N, int64_t K, void* w, cudaStream_t st) {
  const int64_t units = N * (K / kQKK);
  const int64_t want = (units + 7) / 8, cap = (int64_t)sm_count() * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  kq_dequantize_kernel<TYPE, T><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(blocks), N, K / kQKK,
                                                      static_cast<T*>(w));
  return check_launch("kq_dequantize_kernel");
}

template <int TYPE>
dial_status launch_kq_dequant(const void* blocks, int64_t N, int64_t K, void* w, dial_dtype wdt,
                              cudaStream_t st) {
  if (wdt == DIAL_F32) return launch_kq_dequant_t<TYPE, float>(blocks, N, K, w, st);
  if (wdt == DIAL_F16) return launch_kq_dequant_t<TYPE, __half>(blocks, N, K, w, st);
  return launch_kq_dequant_t<TYPE, __nv_bfloat16>(blocks, N, K, w, st);
}

constexpr int kKqRows = 8;  // activation rows per pass

// Warps per output row: the fewest (1, 2, 4 or 8) that give the GPU about
// 32 warps per SM (four resident 256-thread CTAs at 64 registers a thread),
// keeping at least four super-blocks per warp where the row has them.
int kq_warps_per_row(int64_t N, int64_t nb) {
  const int64_t want = (int64_t)sm_count() * 32;
  int ks = 1;
  while (ks < 8 && N * ks < want && nb >= 4 * ks) ks *= 2;
  return ks;
}

template <int TYPE, typename T, int MT, int KS>
void launch_kq_linear_ks(const T* x, const uint8_t* w, T* y, int mc, int64_t K, int64_t N, cudaStream_t st) {
  constexpr int RPC = 8 / KS;
  // resident CTAs per SM (the same on every B200); worker threads may race to
  // set it, all with the same value
  static std::atomic<int> occ_cache{0};
  int occ = occ_cache.load(std::memory_order_relaxed);
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kq_linear_kernel<TYPE, T, MT, KS>, 256, 0) !=
            cudaSuccess || occ < 1) {
      (void)cudaGetLastError();
      occ = 1;
    }
    occ_cache.store(occ, std::memory_order_relaxed);
  }
  const int64_t want = (N + RPC - 1) / RPC, cap = (int64_t)sm_count() * occ;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  kq_linear_kernel<TYPE, T, MT, KS><<<grid, 256, 0, st>>>(x, w, y, mc, K, N);
}

template <int TYPE, typename T, int MT>
void launch_kq_linear_mt(const T* x, const uint8_t* w, T* y, int mc, int64_t K, int64_t N, int ks,
                         cudaStream_t st) {
  if (ks == 1) launch_kq_linear_ks<TYPE, T, MT, 1>(x, w, y, mc, K, N, st);
  else if (ks == 2) launch_kq_linear_ks<TYPE, T, MT, 2>(x, w, y, mc, K, N, st);
  else if (ks == 4) launch_kq_linear_ks<TYPE, T, MT, 4>(x, w, y, mc, K, N, st);
  else launch_kq_linear_ks<TYPE, T, MT, 8>(x, w, y, mc, K, N, st);
}

template <int TYPE, typename T>
dial_status launch_kq_linear_t(const void* x, const void* blocks, void* y, int64_t M, int64_t K,
                               int64_t N, cudaStream_t st) {
  const uint8_t* wb = static_cast<const uint8_t*>(blocks);
  const int ks = kq_warps_per_row(N, K / kQKK);
  for (int64_t m0 = 0; m0 < M; m0 += kKqRows) {
    const int mc = (int)(M - m0 < kKqRows ? M - m0 : kKqRows);
    const T* xp = static_cast<const T*>(x) + m0 * K;
    T* yp = static_cast<T*>(y) + m0 * N;
    if (mc == 1) launch_kq_linear_mt<TYPE, T, 1>(xp, wb, yp, mc, K, N, ks, st);
    else if (mc == 2) launch_kq_linear_mt<TYPE, T, 2>(xp, wb, yp, mc, K, N, ks, st);
    else if (mc <= 4) launch_kq_linear_mt<TYPE, T, 4>(xp, wb, yp, mc, K, N, ks, st);
    else launch_kq_linear_mt<TYPE, T, 8>(xp, wb, yp, mc, K, N, ks, st);
    const dial_status s = check_launch("kq_linear_kernel");
    if (s != DIAL_OK) return s;
  }
  return DIAL_OK;
}

template <int TYPE>
dial_status launch_kq_linear(const void* x, dial_dtype xdt, const void* blocks, void* y, int64_t M,
                             int64_t K, int64_t N, cudaStream_t st) {
  if (xdt == DIAL_F32) return launch_kq_linear_t<TYPE, float>(x, blocks, y, M, K, N, st);
  if (xdt == DIAL_F16) return launch_kq_linear_t<TYPE, __half>(x, blocks, y, M, K, N, st);
  return launch_kq_linear_t<TYPE, __nv_bfloat16>(x, blocks, y, M, K, N, st);
}

dial_status check_kq(const void* blocks, dial_ggml_type type, int64_t N, int64_t K) {
  if (!blocks) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (type != DIAL_GGML_Q4_K && type != DIAL_GGML_Q6_K)
    return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "ggml type %d is not Q4_K (12) or Q6_K (14)", (int)type);
  if (N <= 0 || K <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (N > (1ll << 31) - 1) return fail(DIAL_ERR_SHAPE, "N exceeds 2^31-1");
  if (K % kQKK) return fail(DIAL_ERR_SHAPE, "K-quants need K %% 256 == 0 (K=%lld)", (long long)K);
  // Q4_K words are read 4 bytes at a time; Q6_K blocks 2 bytes at a time
  if (reinterpret_cast<uintptr_t>(blocks) & (type == DIAL_GGML_Q4_K ? 15u : 1u))
    return fail(DIAL_ERR_MISALIGNED, "Q4_K blocks must be 16-byte aligned, Q6_K blocks 2-byte aligned");
  return DIAL_OK;
}

bool is_act_dtype(dial_dtype t) { return t == DIAL_F32 || t == DIAL_F16 || t == DIAL_BF16; }

}  // namespace

}  // namespace dial

using namespace dial;

extern "C" size_t dial_gguf_k_row_bytes(dial_ggml_type type, int64_t K) {
  const int bb = kq_block_bytes((int)type);
  if (!bb || K <= 0 || K % kQKK) return 0;
  return (size_t)(K / kQKK) * (size_t)bb;
}

extern "C" dial_status dial_gguf_k_dequantize(const void* blocks, dial_ggml_type type, int64_t N,
                                              int64_t K, void* w, dial_dtype wdt, dial_stream stream) {
  clear_error();
  dial_status s = check_kq(blocks, type, N, K);
  if (s != DIAL_OK) return s;
  if (!w) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (!is_act_dtype(wdt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "bad output dtype");
  if (type == DIAL_GGML_Q4_K) return launch_kq_dequant<DIAL_GGML_Q4_K>(blocks, N, K, w, wdt, as_stream(stream));
  return launch_kq_dequant<DIAL_GGML_Q6_K>(blocks, N, K, w, wdt, as_stream(stream));
}

extern "C" dial_status dial_gguf_k_linear(const void* x, dial_dtype xdt, const void* blocks,
                                          dial_ggml_type type, void* y, int64_t M, int64_t K, int64_t N,
                                          dial_stream stream) {
  clear_error();
  dial_status s = check_kq(blocks, type, N, K);
  if (s != DIAL_OK) return s;
  if (!x || !y) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (M <= 0) return fail(DIAL_ERR_INVALID_ARG, "sizes must be positive");
  if (!is_act_dtype(xdt)) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "activation dtype must be f32/f16/bf16");
  if (!aligned16(x)) return fail(DIAL_ERR_MISALIGNED, "x must be 16-byte aligned");
  if (type == DIAL_GGML_Q4_K && kq4_gemv_ok(M, K, N, xdt, x, blocks))
    return launch_kq4_gemv(x, xdt, blocks, y, M, K, N, as_stream(stream));
  // prefill-sized: the tcgen05 GEMM dequantises each super-block once per
  // token tile (the values of the reference's f16 prefill copy)
  if (M > 8 && (xdt == DIAL_F16 || xdt == DIAL_BF16) && aligned16(blocks) && N < (1ll << 31) &&
      K < (1ll << 31) && M < (1ll << 31) && (type == DIAL_GGML_Q4_K || K % 2048 == 0))
    return launch_kquant_gemm_sm100(x, xdt, blocks, (int)type, y, M, K, N, as_stream(stream));
  if (type == DIAL_GGML_Q4_K)
    return launch_kq_linear<DIAL_GGML_Q4_K>(x, xdt, blocks, y, M, K, N, as_stream(stream));
  if (kq6_gemv_ok(M, K, N, xdt, x, blocks))
    return launch_kq6_gemv(x, xdt, blocks, y, M, K, N, as_stream(stream));
  return launch_kq_linear<DIAL_GGML_Q6_K>(x, xdt, blocks, y, M, K, N, as_stream(stream));
}
