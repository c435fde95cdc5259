// Prefill dequant-GEMM on the sm_100a tensor cores: TMA + tcgen05.mma + TMEM.
//
//   y[m, n] = sum_k x[m, k] * deq(W)[n, k]        (M > 32 activation rows)
//
// Replaces the reference's prefill paths: dial_w8a16_prefill_f16
// (worker_w8a16.rs:186-224, a 16x16 scalar tile on CUDA cores) and, for GGUF,
// candle's F32 QMatMul fallback / the resident-f16-copy cuBLAS prefill
// (worker_gguf.rs:399-460, :607-610).  No resident f16 copy: the packed
// weights are dequantised tile by tile into shared memory.
//
// CTA tile: 128 activation rows (UMMA M) x 256 weight rows (UMMA N), K in
// steps of 64 (one 128-byte swizzle atom of f16/bf16), 4-stage ring.
//   warp 0     : TMA producer of the activation tile (SWIZZLE_128B, no multicast)
//   warp 1     : TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9 : dequantisers (one weight row each per 128-wide K group,
//                writing the canonical K-major SWIZZLE_128B layout), then the
//                epilogue (tcgen05.ld -> scale -> global)
// Operands: f16 (f16 or f32 activations) or bf16 (bf16 activations), f32
// accumulation in TMEM.  W8A16 int8 values are exact in f16/bf16 and the row
// scale is applied in the epilogue, as in the reference (sum first, then
// * scale[n]); GGUF values d*q are rounded once to the operand type.
//
// Every mbarrier wait is bounded (1 s on the global timer, or earlier if
// another thread already flagged an error); on expiry the kernel records
// DIAL_ERR_TIMEOUT in a device flag, drains, frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "glue.cuh"
#include "layout.cuh"
#include "tma.cuh"

namespace dial {

__device__ int g_device_error = 0;

namespace {

constexpr int BM = 128;  // activation rows per CTA (UMMA M)
constexpr int BN = 256;  // weight rows per CTA (UMMA N)
constexpr int BK = 64;   // K per stage
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int DQ_WARPS = 8;
constexpr int DQ_THREADS = DQ_WARPS * 32;  // == BN: one weight row per thread
constexpr int THREADS = 64 + DQ_THREADS;
constexpr int TMEM_COLS = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr unsigned long long kTimeoutNs = 1000000000ull;

enum Fmt { kW8F32 = 0, kW8F16 = 1, kQ4 = 2, kQ8 = 3 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false when the deadline passed or another thread flagged an error.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*(volatile int*)&g_device_error != 0) return false;
      if (global_ns() - t0 > kTimeoutNs) {
        atomicCAS(&g_device_error, 0, (int)DIAL_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version for sm_100
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: D f32, A/B f16 (0) or bf16 (1), both K-major.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- dequant helpers
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// int8x4 -> (f16x2 of bytes 0,1 ; f16x2 of bytes 2,3), exact
__device__ __forceinline__ void i8x4_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const __half2 bias = bits_h2(0x64806480u);  // 1152
  lo = h2_bits(__hsub2(bits_h2(prmt(u, 0x64646464u, 0x4140u)), bias));
  hi = h2_bits(__hsub2(bits_h2(prmt(u, 0x64646464u, 0x4342u)), bias));
}

// int8x4 -> 4 exact f32
__device__ __forceinline__ void i8x4_f32(uint32_t w, float (&f)[4]) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __uint_as_float(prmt(u, 0x4B000000u, 0x7440u)) - 8388736.0f;
  f[1] = __uint_as_float(prmt(u, 0x4B000000u, 0x7441u)) - 8388736.0f;
  f[2] = __uint_as_float(prmt(u, 0x4B000000u, 0x7442u)) - 8388736.0f;
  f[3] = __uint_as_float(prmt(u, 0x4B000000u, 0x7443u)) - 8388736.0f;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 8 int8 values (two words) -> one 16-byte chunk of 8 operands, times `d`
// (unscaled for W8A16, whose scale is applied in the epilogue).
template <bool BF16, bool SCALED>
__device__ __forceinline__ uint4 chunk_from_i8(uint32_t w0, uint32_t w1, float d, __half2 dh) {
  uint4 out;
  if (!BF16) {
    uint32_t a, b, c, e;
    i8x4_f16(w0, a, b);
    i8x4_f16(w1, c, e);
    if (SCALED) {
      a = h2_bits(__hmul2(bits_h2(a), dh));
      b = h2_bits(__hmul2(bits_h2(b), dh));
      c = h2_bits(__hmul2(bits_h2(c), dh));
      e = h2_bits(__hmul2(bits_h2(e), dh));
    }
    out = make_uint4(a, b, c, e);
  } else {
    float f0[4], f1[4];
    i8x4_f32(w0, f0);
    i8x4_f32(w1, f1);
    if (SCALED) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f0[i] *= d;
        f1[i] *= d;
      }
    }
    out = make_uint4(pack_bf16(f0[0], f0[1]), pack_bf16(f0[2], f0[3]), pack_bf16(f1[0], f1[1]),
                     pack_bf16(f1[2], f1[3]));
  }
  return out;
}

// 4 nibbles (low or high half of each byte of `w`) -> 4 operands d*(q-8) as 2 words.
template <bool BF16>
__device__ __forceinline__ void nib4(uint32_t w, bool high, float d, __half2 dh, uint32_t& o0,
                                     uint32_t& o1) {
  const uint32_t s = high ? (w >> 4) : w;
  if (!BF16) {
    // bytes 0,1 -> halves of o0 ; bytes 2,3 -> halves of o1, as 1024 + q, then -1032, * d
    const uint32_t p01 = prmt(s, 0u, 0x4140u), p23 = prmt(s, 0u, 0x4342u);
    const __half2 off = bits_h2(0x64086408u);  // 1032
    o0 = h2_bits(__hmul2(__hsub2(bits_h2((p01 & 0x000F000Fu) | 0x64006400u), off), dh));
    o1 = h2_bits(__hmul2(__hsub2(bits_h2((p23 & 0x000F000Fu) | 0x64006400u), off), dh));
  } else {
    const float q0 = (float)((int)(s & 0xF) - 8), q1 = (float)((int)((s >> 8) & 0xF) - 8);
    const float q2 = (float)((int)((s >> 16) & 0xF) - 8), q3 = (float)((int)((s >> 24) & 0xF) - 8);
    o0 = pack_bf16(q0 * d, q1 * d);
    o1 = pack_bf16(q2 * d, q3 * d);
  }
}

__device__ __forceinline__ void st_shared16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a K-major SWIZZLE_128B tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

struct Params {
  const uint8_t* w;   // int8 [N, K] (W8A16) or interleaved qs [N, G*GB] (GGUF)
  const void* scale;  // W8A16 row scale [N] (f32 or f16)
  const __half* gd;   // GGUF d [N, 4G]
  void* y;            // [M, N]
  int M, N, K, G, nk; // nk = number of 64-wide K stages
};

template <int FMT, bool BF16, typename YT>
__device__ __forceinline__ void epilogue_store(const Params& p, int row, int nb, float (&v)[16]) {
  if (FMT == kW8F32) {
    const float* sc = static_cast<const float*>(p.scale) + nb;
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] *= (nb + i < p.N) ? __ldg(sc + i) : 0.f;
  } else if (FMT == kW8F16) {
    const __half* sc = static_cast<const __half*>(p.scale) + nb;
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] *= (nb + i < p.N) ? __half2float(sc[i]) : 0.f;
  }
  YT* out = static_cast<YT*>(p.y) + (size_t)row * p.N + nb;
  if (nb + 16 <= p.N && (p.N % 8) == 0) {
    if (sizeof(YT) == 4) {
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        YT a = Act<YT>::from_f32(v[2 * i]), b = Act<YT>::from_f32(v[2 * i + 1]);
        pk[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&a)) |
                ((uint32_t)(*reinterpret_cast<uint16_t*>(&b)) << 16);
      }
      *reinterpret_cast<uint4*>(out) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<uint4*>(out + 8) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
  } else {
    for (int i = 0; i < 16 && nb + i < p.N; ++i) out[i] = Act<YT>::from_f32(v[i]);
  }
}

template <int FMT, bool BF16, typename YT>
__global__ void __launch_bounds__(THREADS, 1)
    dequant_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full_x[STAGES], full_w[STAGES], empty[STAGES], acc_full, then the TMEM slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t bar_base = smem_u32(bars);
  const uint32_t acc_full = bar_base + 8u * (3 * STAGES);
#define FULL_X(s) (bar_base + 8u * (uint32_t)(s))
#define FULL_W(s) (bar_base + 8u * (uint32_t)(STAGES + (s)))
#define EMPTY(s) (bar_base + 8u * (uint32_t)(2 * STAGES + (s)))
#define A_ADDR(s) (smem_base + (uint32_t)((s) * STAGE_BYTES))
#define B_ADDR(s) (smem_base + (uint32_t)((s) * STAGE_BYTES + A_BYTES))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(FULL_X(s), 1);
      mbar_init(FULL_W(s), DQ_THREADS);
      mbar_init(EMPTY(s), 1);
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (activations)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
      for (int kt = 0; kt < p.nk; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!mbar_wait(EMPTY(s), ph ^ 1u)) break;
        mbar_expect_tx(FULL_X(s), A_BYTES);
        tma_load_2d(A_ADDR(s), &tmap_x, FULL_X(s), kt * BK, m0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BF16, BM, BN);
      for (int kt = 0; kt < p.nk; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!mbar_wait(FULL_X(s), ph) || !mbar_wait(FULL_W(s), ph)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t ad = sw128_desc(A_ADDR(s)), bd = sw128_desc(B_ADDR(s));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16(tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kt | k) != 0);
        umma_commit(EMPTY(s));
      }
      umma_commit(acc_full);  // arrives once every issued MMA has completed
    }
  } else {
    // ------------------------------------------------ dequantisers
    const int r = threadIdx.x - 64;  // weight row within the tile
    const int n = min(n0 + r, p.N - 1);
    const bool row_ok = n0 + r < p.N;
    bool ok = true;
    for (int kt = 0; kt < p.nk && ok; kt += 2) {
      // one 128-wide K group = stages kt and kt+1
      const int gi = kt >> 1;
      uint4 raw[8];
      float dv[4] = {1.f, 1.f, 1.f, 1.f};
      if (FMT == kW8F32 || FMT == kW8F16) {
        const uint8_t* src = p.w + (size_t)n * p.K + (size_t)gi * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          raw[c] = (row_ok && gi * 128 + 16 * c < p.K)
                       ? __ldg(reinterpret_cast<const uint4*>(src) + c)
                       : make_uint4(0, 0, 0, 0);
      } else {
        constexpr int GB = FMT == kQ4 ? 64 : 128;
        const uint8_t* src = p.w + (size_t)n * p.G * GB + (size_t)gi * GB;
#pragma unroll
        for (int c = 0; c < GB / 16; ++c) raw[c] = __ldg(reinterpret_cast<const uint4*>(src) + c);
        const uint2 dd =
            __ldg(reinterpret_cast<const uint2*>(p.gd + gguf_d_index(n, 4 * gi, p.G)));
        dv[0] = __low2float(bits_h2(dd.x));
        dv[1] = __high2float(bits_h2(dd.x));
        dv[2] = __low2float(bits_h2(dd.y));
        dv[3] = __high2float(bits_h2(dd.y));
        if (!row_ok) dv[0] = dv[1] = dv[2] = dv[3] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int st = kt + h;
        if (st >= p.nk) break;
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!mbar_wait(EMPTY(s), ph ^ 1u)) {
          ok = false;
          break;
        }
        const uint32_t tile = B_ADDR(s);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          // chunk c of this stage = group-local K [64h + 8c, 64h + 8c + 8)
          const int cg = 8 * h + c;  // 0..15 within the group
          uint4 v;
          if (FMT == kW8F32 || FMT == kW8F16) {
            const uint4& q = raw[cg >> 1];
            v = (cg & 1) ? chunk_from_i8<BF16, false>(q.z, q.w, 1.f, __half2())
                         : chunk_from_i8<BF16, false>(q.x, q.y, 1.f, __half2());
          } else {
            const int j = cg >> 2, qq = cg & 3;  // block j, quarter qq of its 32 values
            const float d = dv[j];
            const __half2 dh = __float2half2_rn(d);  // exact: d is an f16 value
            if (FMT == kQ4) {
              // lane-chunks t = 2*(qq&1) and +1 hold the bytes; low nibbles for qq < 2
              const uint32_t w0 = word(raw[2 * (qq & 1)], j), w1 = word(raw[2 * (qq & 1) + 1], j);
              uint32_t o0, o1, o2, o3;
              nib4<BF16>(w0, qq >= 2, d, dh, o0, o1);
              nib4<BF16>(w1, qq >= 2, d, dh, o2, o3);
              v = make_uint4(o0, o1, o2, o3);
            } else {
              // Q8_0: lane-chunk t occupies raw[2t], raw[2t+1]; block j's low-half word
              // is word 2j of the 32-byte chunk, its high-half word is 2j+1
              const int t0 = 2 * (qq & 1), wsel = 2 * j + (qq >> 1);
              const uint32_t w0 = word(raw[2 * t0 + (wsel >> 2)], wsel & 3);
              const uint32_t w1 = word(raw[2 * (t0 + 1) + (wsel >> 2)], wsel & 3);
              v = chunk_from_i8<BF16, true>(w0, w1, d, dh);
            }
          }
          st_shared16(tile + sw128_off(r, c), v);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(FULL_W(s));
      }
    }

    // ------------------------------------------------ epilogue
    const int ew = warp - 2;                // 0..7
    const int quarter = warp & 3;           // TMEM lanes this warp may read
    const int col0 = (ew >> 2) * (BN / 2);  // two warps per lane quarter split the columns
    const bool acc_ok = ok && mbar_wait(acc_full, 0);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (__all_sync(0xffffffffu, acc_ok)) {
      const int row = m0 + quarter * 32 + lane;  // activation row (token)
      for (int c = 0; c < BN / 2; c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c), v);
        const int nb = n0 + col0 + c;
        if (row < p.M && nb < p.N) epilogue_store<FMT, BF16, YT>(p, row, nb, v);
      }
    }
  }
#undef FULL_X
#undef FULL_W
#undef EMPTY
#undef A_ADDR
#undef B_ADDR

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

template <typename XT>
__global__ void to_f16_kernel(const XT* __restrict__ x, __half* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(Act<XT>::to_f32(x[i]));
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

dial_status make_x_map(CUtensorMap* map, const void* x, bool bf16, int64_t M, int64_t K) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, BM};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DIAL_OK;
}

template <int FMT, bool BF16, typename YT>
dial_status launch_one(const CUtensorMap& map, const Params& p, cudaStream_t st) {
  auto kern = dequant_gemm_kernel<FMT, BF16, YT>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(dequant_gemm)");
  dim3 grid((unsigned)((p.M + BM - 1) / BM), (unsigned)((p.N + BN - 1) / BN));
  kern<<<grid, THREADS, SMEM_BYTES, st>>>(map, p);
  return check_launch("dequant_gemm_kernel");
}

}  // namespace

namespace tma {
dial_status make_byte_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                          int box_bytes, int box_rows, bool swizzle128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (!aligned16(base) || row_bytes % 16 != 0 || (swizzle128 && box_bytes != 128))
    return fail(DIAL_ERR_MISALIGNED, "tensor map: base and row pitch must be 16-byte aligned");
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DIAL_OK;
}
}  // namespace tma

bool gemm_sm100_supported(int64_t M, int64_t K, int64_t N) {
  (void)N;
  return M > 32 && K % 64 == 0 && K >= 64;
}

size_t gemm_sm100_gguf_workspace_bytes(int64_t M, int64_t K) {
  return M > 32 ? (size_t)((M * K * 2 + 255) / 256 * 256) : 0;
}

dial_status launch_w8a16_gemm_sm100(const void* x, dial_dtype xdt, const int8_t* q,
                                    const void* scale, dial_dtype sdt, void* y, int64_t M,
                                    int64_t K, int64_t N, cudaStream_t st) {
  CUtensorMap map;
  const bool bf = xdt == DIAL_BF16;
  dial_status s = make_x_map(&map, x, bf, M, K);
  if (s != DIAL_OK) return s;
  Params p{reinterpret_cast<const uint8_t*>(q), scale, nullptr, y, (int)M, (int)N, (int)K, 0,
           (int)(K / BK)};
  if (sdt == DIAL_F32)
    return bf ? launch_one<kW8F32, true, __nv_bfloat16>(map, p, st)
              : launch_one<kW8F32, false, __half>(map, p, st);
  return bf ? launch_one<kW8F16, true, __nv_bfloat16>(map, p, st)
            : launch_one<kW8F16, false, __half>(map, p, st);
}

dial_status launch_gguf_gemm_sm100(const void* x, dial_dtype xdt, const void* qs,
                                   const uint16_t* d, int type, void* y, int64_t M, int64_t K,
                                   int64_t N, void* ws, cudaStream_t st) {
  const void* xin = x;
  const bool bf = xdt == DIAL_BF16;
  if (xdt == DIAL_F32) {  // the tensor cores take f16 operands: convert once
    __half* xh = static_cast<__half*>(ws);
    const int64_t n = M * K;
    const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 16);
    to_f16_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), xh, n);
    dial_status s = check_launch("to_f16_kernel");
    if (s != DIAL_OK) return s;
    xin = xh;
  }
  CUtensorMap map;
  dial_status s = make_x_map(&map, xin, bf, M, K);
  if (s != DIAL_OK) return s;
  const int64_t G = gguf_groups(K);
  Params p{static_cast<const uint8_t*>(qs), nullptr, reinterpret_cast<const __half*>(d), y, (int)M,
           (int)N, (int)K, (int)G, (int)(K / BK)};
  if (type == DIAL_GGML_Q4_0) {
    if (xdt == DIAL_F32) return launch_one<kQ4, false, float>(map, p, st);
    if (xdt == DIAL_F16) return launch_one<kQ4, false, __half>(map, p, st);
    return launch_one<kQ4, true, __nv_bfloat16>(map, p, st);
  }
  if (xdt == DIAL_F32) return launch_one<kQ8, false, float>(map, p, st);
  if (xdt == DIAL_F16) return launch_one<kQ8, false, __half>(map, p, st);
  return launch_one<kQ8, true, __nv_bfloat16>(map, p, st);
}

int* device_error_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

dial_status read_device_error(bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(g_device_error)");
  if (v != 0 && clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  return v == 0 ? DIAL_OK : fail((dial_status)v, "a kernel's bounded wait expired");
}

}  // namespace dial

extern "C" dial_status dial_device_error(int clear) {
  dial::clear_error();
  return dial::read_device_error(clear != 0);
}
