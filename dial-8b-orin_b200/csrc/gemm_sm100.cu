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
// CTA tile: 256 weight rows x 128 activation rows (tokens), K in 64-deep
// stages.  The dequantised weights are the MMA's A operand and live in TMEM:
// two tcgen05.mma (M = 128 weight rows each, N = 128 tokens, K = 16) per
// 16-deep K step read A from TMEM and the token tile from shared memory.
//   warp 0     : TMA producer of the token tile (SWIZZLE_128B, 8-stage ring, no multicast)
//   warp 1     : TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..17: dequantisers: warp w owns TMEM lane quarter w % 4 (one weight
//                row per thread) of weight half ((w - 2) / 4) & 1 and K half
//                (w - 2) / 8 of every stage; each thread reads its row's packed
//                group from the weight ring, dequantises its 32 K values per
//                stage to f16/bf16 pairs and writes them with tcgen05.st into
//                the A ring (4 stages), one stage behind so the store's latency
//                hides under the next stage's arithmetic; then the epilogue
//                (tcgen05.ld -> scale -> global, y[token, n])
//   warp 18    : TMA producer of the packed weight groups (and GGUF scales)
// Small grids are split along K over a thread-block cluster of S CTAs
// (1 x 1 x S): each CTA leaves its f32 partial tile in shared memory and CTA z
// adds the S partials of its token slice in rank order through distributed
// shared memory, so the result does not depend on timing.
// TMEM: accumulators in columns [0, 256) (weight half h at 128 h), A stages in
// [256, 512), 64 columns each (32 per weight half: K 64 as f16x2 words).
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

constexpr int BK = 64;    // K per stage (one 128-byte swizzle atom of f16/bf16)
constexpr int A_HALF_COLS = BK / 2;  // TMEM columns of one 128-row weight half per stage
constexpr int kMaxSplit = 8;
constexpr unsigned long long kTimeoutNs = 1000000000ull;

enum Fmt { kW8F32 = 0, kW8F16 = 1, kQ4 = 2, kQ8 = 3, kQ4K = 4, kQ6K = 5 };

// One CTA's tile and resources.  BT: activation rows (tokens) per CTA (UMMA N):
// 256 from 256 rows on (each dequantised weight stage then feeds twice the
// MMAs; one CTA per SM with all 512 TMEM columns), 128 below, or 32 for at
// most 32 rows (batched decode), where wider tiles would spend most MMA cycles
// on padding.  NH: 128-row weight halves per CTA (UMMA M = 128
// each).  NH = 2: 16 dequantising warps (lane quarter x weight half x K half of
// a stage), all 512 TMEM columns, one CTA per SM.  NH = 1: 8 dequantising warps,
// 256 TMEM columns and at most 113 KB of shared memory, so that two CTAs share
// an SM and one's prologue and epilogue overlap the other's main loop.
// Shared memory: [token ring | packed weight ring | GGUF d ring], every stage
// 1024-byte aligned (the swizzle atoms); the split-K partial tile reuses it
// after the main loop.
template <int FMT, int BT, int NH>
struct Cfg {
  static constexpr int BW = 128 * NH;           // weight rows per CTA
  static constexpr int DQ_WARPS = 8 * NH;
  static constexpr int THREADS = 64 + DQ_WARPS * 32 + 32;  // + the weight producer warp
  // two CTAs per SM for the narrow CTA up to 128 tokens; a 256-token tile
  // needs all 512 TMEM columns (one CTA per SM)
  static constexpr int CTAS_PER_SM = NH == 1 && BT <= 128 ? 2 : 1;
  static constexpr int TMEM_COLS = NH == 1 && BT <= 128 ? 256 : 512;
  static constexpr int ACC_COLS = NH * BT;      // NH f32 accumulators of BT columns
  static constexpr int A_COLS = NH * A_HALF_COLS;  // TMEM columns of a dequantised stage
  static constexpr int A_STAGES = 4;
  static_assert(ACC_COLS + A_STAGES * A_COLS <= TMEM_COLS, "TMEM budget");
  static constexpr int B_STAGES = NH == 1 ? 3 : 4;  // token tiles in shared memory
  static constexpr int W_STAGES = FMT == kQ6K ? 2 : (NH == 1 ? 3 : 4);  // packed weight groups
  static constexpr int B_BYTES = BT * BK * 2;   // token tile per stage
  // split-K: at most BT / 4 CTAs (each owns whole float4 column groups); the
  // owner's receive buffer is [S senders][BW rows][BT / S + 4] f32 (the +4 pad
  // keeps the 8 rows of a quarter warp's float4 accesses in distinct banks)
  static constexpr int MAX_SPLIT = BT / 4 < kMaxSplit ? BT / 4 : kMaxSplit;
  static constexpr int RED_BYTES = BW * 4 * (BT + 4 * MAX_SPLIT);
  static constexpr bool GGUF = FMT == kQ4 || FMT == kQ8;
  // packed bytes of a row per weight group: 128 K (2 stages), or for Q4_K one
  // 256-K super-block of 144 bytes (4 stages)
  // (Q6_K: a 224-byte box from the 16-byte boundary at or below the 210-byte
  // super-block, which starts o = 210 g mod 16 bytes into it)
  static constexpr int GB = FMT == kQ4 ? 64 : (FMT == kQ4K ? 144 : (FMT == kQ6K ? 224 : 128));
  static constexpr int SPG = FMT == kQ4K || FMT == kQ6K ? 4 : 2;  // K stages per weight group
  static constexpr int W_BYTES = BW * GB;
  static constexpr int D_BYTES = GGUF ? (BW / 16) * 128 : 0;  // 16-row tiles x 4 blocks x 16 rows
  static constexpr int W_OFF = B_STAGES * B_BYTES;
  static constexpr int D_OFF = W_OFF + W_STAGES * W_BYTES;
  static constexpr int RING = D_OFF + W_STAGES * D_BYTES;
  static constexpr int DATA = RING > RED_BYTES ? RING : RED_BYTES;
  static constexpr int BYTES = DATA + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(BYTES <= (CTAS_PER_SM == 2 ? 113 : 227) * 1024, "shared memory budget");
};

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

// D[tmem_d] (+)= A[tmem_a] * B[bdesc]^T: A (M = 128 rows, K = 16) in TMEM, one
// row per lane, K packed two 16-bit values per 32-bit column (even K low).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
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

// int8x4 -> (bf16x2 of bytes 0,1 ; bf16x2 of bytes 2,3), exact: under the
// exponent of 128, v1 = 128 + (b & 127) and v2 = -128 - 128 * (b < 0), and
// v1 + v2 = b is an integer that bf16 holds exactly.
__device__ __forceinline__ void i8x4_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
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

// 4 int8 values times the block scale d, rounded once to the operand type.
template <bool BF16>
__device__ __forceinline__ void i8x4_scaled(uint32_t w, float d, __half2 dh, uint32_t& lo,
                                            uint32_t& hi) {
  if (!BF16) {
    i8x4_f16(w, lo, hi);  // exact
    lo = h2_bits(__hmul2(bits_h2(lo), dh));
    hi = h2_bits(__hmul2(bits_h2(hi), dh));
  } else {
    float f[4];
    i8x4_f32(w, f);
    lo = pack_bf16(f[0] * d, f[1] * d);
    hi = pack_bf16(f[2] * d, f[3] * d);
  }
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

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

struct Params {
  const uint8_t* w;   // int8 [N, K] (W8A16) or interleaved qs [N, G*GB] (GGUF)
  const void* scale;  // W8A16 row scale [N] (f32 or f16)
  const __half* gd;   // GGUF d [N, 4G]
  void* y;            // [M, N]
  int M, N, K, G, nk; // nk = number of 64-wide K stages
};

__device__ __forceinline__ uint4 ld_shared16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 ld_shared8(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// Row r (0..255) of a packed weight group staged by TMA: 16-byte chunk c sits
// at chunk c ^ (r & 7) of the row (SWIZZLE_128B, 128-byte rows) or
// c ^ ((r >> 1) & 3) (SWIZZLE_64B, 64-byte Q4_0 rows), so the 8 rows a quarter
// warp reads at once fall in distinct banks.  d: the 16-row tile r / 16 of
// group g holds [16 rows][4 blocks] f16, row r's 4 scales at (r & 15) * 8.
template <int FMT>
__device__ __forceinline__ void read_group(uint32_t wbase, uint32_t dbase, int r, uint4 (&raw)[8],
                                           float (&dv)[4], uint4& hdr) {
  if (FMT == kQ6K) return;  // read per stage by dequant_q6k
  if (FMT == kQ4K) {  // 144-byte rows, no swizzle: the 16-byte header, then the 128 nibble bytes
    hdr = ld_shared16(wbase + r * 144);
#pragma unroll
    for (int c = 0; c < 8; ++c) raw[c] = ld_shared16(wbase + r * 144 + 16 + 16 * c);
    return;
  }
  if (FMT == kQ4) {
#pragma unroll
    for (int c = 0; c < 4; ++c) raw[c] = ld_shared16(wbase + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) raw[c] = ld_shared16(wbase + r * 128 + ((c ^ (r & 7)) << 4));
  }
  if (FMT == kQ4 || FMT == kQ8) {
    const uint2 dd = ld_shared8(dbase + (r >> 4) * 128 + (r & 15) * 8);
    dv[0] = __low2float(bits_h2(dd.x));
    dv[1] = __high2float(bits_h2(dd.x));
    dv[2] = __low2float(bits_h2(dd.y));
    dv[3] = __high2float(bits_h2(dd.y));
  }
}

// K 64H + 32KH .. +31 of a group (K half KH of the group's stage H) as 16
// operand pairs: word j holds K 2j (low) and 2j+1 (high) of that range.
template <int FMT, bool BF16, int H, int KH>
__device__ __forceinline__ void dequant_part(const uint4 (&raw)[8], const float (&dv)[4],
                                             uint32_t (&wv)[16]) {
  if (FMT == kW8F32 || FMT == kW8F16) {
    // bytes 64H + 32KH + 16c + 4q .. +3 are word q of chunk 4H + 2KH + c
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = word(raw[4 * H + 2 * KH + c], q);
        if (BF16) i8x4_bf16(w, wv[8 * c + 2 * q], wv[8 * c + 2 * q + 1]);
        else i8x4_f16(w, wv[8 * c + 2 * q], wv[8 * c + 2 * q + 1]);
      }
  } else if (FMT == kQ4) {
    // block b = 2H + KH: qs bytes 4c..4c+3 are word b of chunk c; element e < 16
    // is the low nibble of byte e, element e + 16 its high nibble
    constexpr int b = 2 * H + KH;
    const float d = dv[b];
    const __half2 dh = __float2half2_rn(d);  // exact: d is an f16 value
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w = word(raw[c], b);
      nib4<BF16>(w, false, d, dh, wv[2 * c], wv[2 * c + 1]);
      nib4<BF16>(w, true, d, dh, wv[8 + 2 * c], wv[8 + 2 * c + 1]);
    }
  } else {
    // Q8_0 block b = 2H + KH: lane-chunk t (raw[2t], raw[2t+1]) word 2b + hi
    // holds elements 16 hi + 4t .. +3
    constexpr int b = 2 * H + KH;
    const float d = dv[b];
    const __half2 dh = __float2half2_rn(d);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int hi = u >> 2, t = u & 3, wi = 2 * b + hi;
      const uint32_t w = word(raw[2 * t + (wi >> 2)], wi & 3);
      i8x4_scaled<BF16>(w, d, dh, wv[2 * u], wv[2 * u + 1]);
    }
  }
}

template <int FMT, bool BF16>
__device__ __forceinline__ void dequant_part(int h, int kh, const uint4 (&raw)[8],
                                             const float (&dv)[4], uint32_t (&wv)[16]) {
  if (h == 0) {
    if (kh == 0) dequant_part<FMT, BF16, 0, 0>(raw, dv, wv);
    else dequant_part<FMT, BF16, 0, 1>(raw, dv, wv);
  } else {
    if (kh == 0) dequant_part<FMT, BF16, 1, 0>(raw, dv, wv);
    else dequant_part<FMT, BF16, 1, 1>(raw, dv, wv);
  }
}

// Q4_K stage h of a super-block, K half kh: sub-block j = 2h + kh, the low
// (kh = 0) or high nibbles of qs bytes 32h .. 32h + 31, as 16 operand pairs
// (word w: elements 2w, 2w + 1).  Values as GGML's dequantiser computes them
// (d sc q - dmin m in f32, no contraction), rounded once to the operand type:
// the reference's f16 prefill copy (worker_gguf.rs:399-460) holds the same.
template <bool BF16>
__device__ __forceinline__ void dequant_q4k(int h, int kh, const uint4& hdr, const uint4 (&raw)[8],
                                            uint32_t (&wv)[16]) {
  const int j = 2 * h + kh;
  auto sbyte = [&](int i) {  // scales[i], i < 12: bytes 4 .. 15 of the header
    const uint32_t w = i < 4 ? hdr.y : (i < 8 ? hdr.z : hdr.w);
    return (w >> (8 * (i & 3))) & 0xFFu;
  };
  uint32_t sc, m;
  if (j < 4) {
    sc = sbyte(j) & 63u;
    m = sbyte(j + 4) & 63u;
  } else {
    sc = (sbyte(j + 4) & 15u) | ((sbyte(j - 4) >> 6) << 4);
    m = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
  }
  const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
  const float d0 = __fmul_rn(d, (float)sc), mm0 = __fmul_rn(dmin, (float)m);
  const int sh = 4 * kh;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const uint32_t src = word(raw[2 * h + (w >> 3)], (w & 7) >> 1) >> (16 * (w & 1));
    const float q0 = (float)((src >> sh) & 15u), q1 = (float)((src >> (8 + sh)) & 15u);
    const float v0 = __fsub_rn(__fmul_rn(d0, q0), mm0), v1 = __fsub_rn(__fmul_rn(d0, q1), mm0);
    wv[w] = BF16 ? pack_bf16(v0, v1) : h2_bits(__floats2half2_rn(v0, v1));
  }
}

__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t ld_shared_u32_a2(uint32_t addr) {
  if ((addr & 3u) == 0) return ld_shared_u32(addr);
  return __funnelshift_r(ld_shared_u32(addr - 2), ld_shared_u32(addr + 2), 16);
}

// Q6_K stage h of a super-block (at shared address `blk`, 2-byte aligned), K
// half kh: elements 64h + 32kh + l, l < 32, are half n = h / 2, quarter
// p = 2 (h % 2) + kh of GGML's layout: code ((ql[64n + 32(p & 1) + l] >> 4(p >> 1))
// & 15) | ((qh[32n + l] >> 2p) & 3) << 4, weight d sc[8n + 2p + l / 16] (code - 32),
// computed as GGML does in f32 and rounded once to the operand type.
template <bool BF16>
__device__ __forceinline__ void dequant_q6k(int h, int kh, uint32_t blk, uint32_t (&wv)[16]) {
  const int n = h >> 1, p = 2 * (h & 1) + kh;
  const uint32_t qla = blk + (uint32_t)(64 * n + 32 * (p & 1)), qha = blk + (uint32_t)(128 + 32 * n);
  const uint32_t scw = ld_shared_u32_a2(blk + (uint32_t)(192 + 8 * n + 2 * p));  // scales 8n+2p, +1
  const float d = __half2float(__ushort_as_half((unsigned short)(ld_shared_u32_a2(blk + 208u) & 0xFFFFu)));
  const float d0 = __fmul_rn(d, (float)(int)(int8_t)(scw & 0xFFu));
  const float d1 = __fmul_rn(d, (float)(int)(int8_t)((scw >> 8) & 0xFFu));
  const int ns = 4 * (p >> 1), hs = 2 * p;
#pragma unroll
  for (int q = 0; q < 8; ++q) {  // bytes 4q .. 4q + 3 of the 32 -> words 2q, 2q + 1
    const uint32_t l = ld_shared_u32_a2(qla + 4u * q), hh = ld_shared_u32_a2(qha + 4u * q);
    float v[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int code = (int)(((l >> (8 * b + ns)) & 15u) | (((hh >> (8 * b + hs)) & 3u) << 4));
      v[b] = __fmul_rn(q < 4 ? d0 : d1, (float)(code - 32));
    }
    wv[2 * q] = BF16 ? pack_bf16(v[0], v[1]) : h2_bits(__floats2half2_rn(v[0], v[1]));
    wv[2 * q + 1] = BF16 ? pack_bf16(v[2], v[3]) : h2_bits(__floats2half2_rn(v[2], v[3]));
  }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

template <int FMT>
__device__ __forceinline__ float row_scale(const Params& p, int n) {
  if (n >= p.N) return 0.f;
  if (FMT == kW8F32) return __ldg(static_cast<const float*>(p.scale) + n);
  if (FMT == kW8F16) return __half2float(static_cast<const __half*>(p.scale)[n]);
  return 1.f;
}

// y[t, n] for 4 consecutive tokens t0 .. t0+3 of weight row n (n < N checked by the caller).
template <typename YT>
__device__ __forceinline__ void store4(const Params& p, int t0, int n, float sc, float4 v) {
  YT* y = static_cast<YT*>(p.y);
  const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (t0 + i < p.M) y[(size_t)(t0 + i) * p.N + n] = Act<YT>::from_f32(a[i] * sc);
}

template <int FMT, bool BF16, typename YT, int BT, int NH>
__global__ void __launch_bounds__(Cfg<FMT, BT, NH>::THREADS, Cfg<FMT, BT, NH>::CTAS_PER_SM)
    dequant_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_d, const Params p) {
  using L = Cfg<FMT, BT, NH>;
  constexpr int B_BYTES = L::B_BYTES, ACC_COLS = L::ACC_COLS, A_COLS = L::A_COLS;
  constexpr int B_STAGES = L::B_STAGES, A_STAGES = L::A_STAGES, W_STAGES = L::W_STAGES;
  constexpr int BW = L::BW, DQ_WARPS = L::DQ_WARPS, TMEM_COLS = L::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::DATA);
  // bars: full/empty of the token ring, of the TMEM A ring, of the weight ring, acc_full
  constexpr int NBARS = 2 * B_STAGES + 2 * A_STAGES + 2 * W_STAGES + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t bar_base = smem_u32(bars);
#define FULL_B(s) (bar_base + 8u * (uint32_t)(s))
#define EMPTY_B(s) (bar_base + 8u * (uint32_t)(B_STAGES + (s)))
#define FULL_A(s) (bar_base + 8u * (uint32_t)(2 * B_STAGES + (s)))
#define EMPTY_A(s) (bar_base + 8u * (uint32_t)(2 * B_STAGES + A_STAGES + (s)))
#define FULL_W(s) (bar_base + 8u * (uint32_t)(2 * B_STAGES + 2 * A_STAGES + (s)))
#define EMPTY_W(s) (bar_base + 8u * (uint32_t)(2 * B_STAGES + 2 * A_STAGES + W_STAGES + (s)))
  const uint32_t acc_full = bar_base + 8u * (uint32_t)(NBARS - 1);

  // Programmatic dependent launch: the next kernel may be scheduled now; only
  // the activation producer waits for the previous kernel (weights and scales
  // are constant, so their loads and dequantisation start at once).
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BW;  // weight rows
  const int t0 = blockIdx.y * BT;  // tokens
  const int S = (int)gridDim.z;
  const int split = S > 1 ? (int)cluster_rank() : 0;
  // this CTA's K range, in whole weight groups (SPG stages each)
  const int ngr = (p.nk + L::SPG - 1) / L::SPG;
  const int g0 = (int)((int64_t)ngr * split / S), g1 = (int)((int64_t)ngr * (split + 1) / S);
  const int kt0 = L::SPG * g0, kt1 = min(L::SPG * g1, p.nk);
  const int nst = kt1 - kt0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < B_STAGES; ++s) {
      mbar_init(FULL_B(s), 1);
      mbar_init(EMPTY_B(s), 1);
    }
    for (int s = 0; s < A_STAGES; ++s) {
      mbar_init(FULL_A(s), DQ_WARPS);  // every dequantising warp writes every stage
      mbar_init(EMPTY_A(s), 1);
    }
    for (int s = 0; s < W_STAGES; ++s) {
      mbar_init(FULL_W(s), 1);
      mbar_init(EMPTY_W(s), DQ_WARPS);  // every dequantising warp reads every group
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
    // ------------------------------------------------ TMA producer (tokens)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
      pdl_wait();
      for (int i = 0; i < nst; ++i) {
        const int s = i % B_STAGES;
        const uint32_t ph = (uint32_t)(i / B_STAGES) & 1u;
        if (!mbar_wait(EMPTY_B(s), ph ^ 1u)) break;
        mbar_expect_tx(FULL_B(s), B_BYTES);
        tma_load_2d(smem_base + (uint32_t)(s * B_BYTES), &tmap_x, FULL_B(s), (kt0 + i) * BK, t0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BF16, 128, BT);
      for (int i = 0; i < nst; ++i) {
        const int sb = i % B_STAGES, sa = i % A_STAGES;
        const uint32_t pb = (uint32_t)(i / B_STAGES) & 1u, pa = (uint32_t)(i / A_STAGES) & 1u;
        if (!mbar_wait(FULL_A(sa), pa) || !mbar_wait(FULL_B(sb), pb)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bd = sw128_desc(smem_base + (uint32_t)(sb * B_BYTES));
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_ts(tmem + (uint32_t)(h * BT),
                    tmem + (uint32_t)(ACC_COLS + sa * A_COLS + h * A_HALF_COLS + 8 * k),
                    bd + (uint64_t)(2 * k), idesc, (i | k) != 0);
        umma_commit(EMPTY_A(sa));
        umma_commit(EMPTY_B(sb));
      }
      umma_commit(acc_full);  // arrives once every issued MMA has completed
    }
  } else if (warp == 2 + DQ_WARPS) {
    // ------------------------------------------------ TMA producer (packed weights)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
      constexpr uint32_t tx = L::W_BYTES + L::D_BYTES;
      for (int g = g0; g < g1; ++g) {
        const int i = g - g0, s = i % W_STAGES;
        if (!mbar_wait(EMPTY_W(s), ((uint32_t)(i / W_STAGES) & 1u) ^ 1u)) break;
        mbar_expect_tx(FULL_W(s), tx);
        tma_load_2d(smem_base + (uint32_t)(L::W_OFF + s * L::W_BYTES), &tmap_w, FULL_W(s),
                    FMT == kQ6K ? (g * 210) & ~15 : g * L::GB, n0);
        if (L::GGUF)
          tma_load_2d(smem_base + (uint32_t)(L::D_OFF + s * L::D_BYTES), &tmap_d, FULL_W(s),
                      g * 128, n0 / 16);
      }
    }
  }

  // ------------------------------------------------ dequantisers, then the epilogue
  const bool dq = warp >= 2 && warp < 2 + DQ_WARPS;
  const int quarter = warp & 3;             // TMEM lanes this warp may access
  const int half = NH == 2 ? ((warp - 2) >> 2) & 1 : 0;  // weight half
  const int kh = (warp - 2) >> (NH == 2 ? 3 : 2);  // K half of each stage (token half of the epilogue)
  const int row = half * 128 + quarter * 32 + lane;  // weight row within the tile
  const int n = n0 + row;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  bool ok = true;
  if (dq) {
    const uint32_t a_col = (uint32_t)(ACC_COLS + half * A_HALF_COLS + kh * (A_HALF_COLS / 2));
    int pend = -1;  // A slot written whose FULL_A arrival is still due
    auto publish = [&]() {
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(FULL_A(pend));
      pend = -1;
    };
    for (int g = g0; g < g1 && ok; ++g) {
      const int gi = g - g0, ws = gi % W_STAGES;
      // warp-uniform outcomes: tcgen05.st below needs every lane
      const bool have = mbar_wait(FULL_W(ws), (uint32_t)(gi / W_STAGES) & 1u);
      if (!__all_sync(0xffffffffu, have)) {
        ok = false;
        break;
      }
      uint4 raw[8], hdr;
      float dv[4];
      read_group<FMT>(smem_base + (uint32_t)(L::W_OFF + ws * L::W_BYTES),
                      smem_base + (uint32_t)(L::D_OFF + ws * L::D_BYTES), row, raw, dv, hdr);
#pragma unroll
      for (int h = 0; h < L::SPG; ++h) {
        const int kt = L::SPG * g + h;
        if (kt >= kt1) break;
        const int i = kt - kt0, sa = i % A_STAGES;
        uint32_t wv[16];
        if constexpr (FMT == kQ4K) dequant_q4k<BF16>(h, kh, hdr, raw, wv);
        else if constexpr (FMT == kQ6K)
          dequant_q6k<BF16>(h, kh,
                            smem_base + (uint32_t)(L::W_OFF + ws * L::W_BYTES + row * 224 + ((g * 210) & 15)),
                            wv);
        else dequant_part<FMT, BF16>(h, kh, raw, dv, wv);
        if (pend >= 0) publish();
        const bool free = mbar_wait(EMPTY_A(sa), ((uint32_t)(i / A_STAGES) & 1u) ^ 1u);
        if (!__all_sync(0xffffffffu, free)) {
          ok = false;
          break;
        }
        tmem_st16(tmem + lane_base + a_col + (uint32_t)(sa * A_COLS), wv);
        pend = sa;
      }
      // The slot is released only after the tcgen05.st above consumed values
      // computed from it: the shared-memory loads have then returned, so the
      // producer's next TMA write cannot overtake them.
      __syncwarp();
      if (lane == 0) mbar_arrive(EMPTY_W(ws));
    }
    if (ok && pend >= 0) publish();
    ok = __all_sync(0xffffffffu, ok && mbar_wait(acc_full, 0));
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }

  // epilogue: warp (quarter, half, kh) owns token columns [64 kh, 64 kh + 64) of its rows
  const uint32_t acc = tmem + lane_base + (uint32_t)(half * BT);
  if (S == 1) {
    if (dq && ok) {
      const float sc = row_scale<FMT>(p, n);
      for (int c = kh * (BT / 2); c < (kh + 1) * (BT / 2); c += 16) {
        float v[16];
        tmem_ld16(acc + (uint32_t)c, v);
        if (n < p.N && t0 + c < p.M) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            store4<YT>(p, t0 + c + i, n, sc, make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        }
      }
    }
  } else {
    // split-K: CTA z of the cluster owns token columns [z W, z W + W).  Every
    // CTA pushes each slice of its partial tile into the owner's receive
    // buffer (remote stores, no round trip), and after one cluster barrier the
    // owner adds the S partials in rank order from its own shared memory.
    const int W = BT / S, RS = W + 4;
    float* red = reinterpret_cast<float*>(smem);
    __syncwarp();
    cluster_sync_all();  // every CTA is past its main loop: the receive buffers (rings) are free
    if (dq && ok) {
      for (int c = kh * (BT / 2); c < (kh + 1) * (BT / 2); c += 16) {
        float v[16];
        tmem_ld16(acc + (uint32_t)c, v);
#pragma unroll
        for (int i = 0; i < 16; i += 4) {  // W is a multiple of 4: a float4 has one owner
          const int z = (c + i) / W, cc = c + i - z * W;
          const uint32_t dst = cluster_map(
              smem_base + (uint32_t)(((split * BW + row) * RS + cc) * 4), (uint32_t)z);
          st_cluster_v4(dst, v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // every push has landed; no shared memory is touched remotely after this
    if (dq && ok && n < p.N) {
      const float sc = row_scale<FMT>(p, n);
      const int tb = t0 + split * W;
      // the slice's float4 groups, halved between the two K-half warps of the row
      const int hw = ((W / 4 + 1) / 2) * 4, ca = kh ? hw : 0, cb = kh ? W : hw;
      for (int cc = ca; cc < cb && tb + cc < p.M; cc += 4) {
        float4 a = *reinterpret_cast<const float4*>(red + (row * RS + cc));
        for (int r = 1; r < S; ++r) {
          const float4 v = *reinterpret_cast<const float4*>(red + ((r * BW + row) * RS + cc));
          a.x += v.x;
          a.y += v.y;
          a.z += v.z;
          a.w += v.w;
        }
        store4<YT>(p, tb + cc, n, sc, a);
      }
    }
  }
#undef FULL_B
#undef EMPTY_B
#undef FULL_A
#undef EMPTY_A
#undef FULL_W
#undef EMPTY_W

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

// f32 activations -> f16 operands, 8 values per thread (n is a multiple of 64).
__global__ void to_f16_kernel(const float* __restrict__ x, __half* __restrict__ out, int64_t n8) {
  pdl_begin();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
    const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
    reinterpret_cast<uint4*>(out)[i] = make_uint4(h2_bits(h0), h2_bits(h1), h2_bits(h2), h2_bits(h3));
  }
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

dial_status make_x_map(CUtensorMap* map, const void* x, bool bf16, int64_t M, int64_t K, int rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DIAL_OK;
}

// K splits for a grid of `tiles` CTAs over `ngr` K groups: the fewest waves of
// clusters times the K groups each CTA runs, plus a fixed cost per wave
// (pipeline fill and epilogue, about 4 groups) and one group for the
// cross-CTA reduction.  Cluster capacity comes from the occupancy API.
template <auto KERN>
int choose_split(int64_t tiles, int ngr, int smem_bytes, int max_split, int threads) {
  // active CTAs per device and split (0: not queried); worker threads may race
  // to fill an entry, all with the same value
  static std::atomic<int> cap[64][kMaxSplit + 1];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  int best = 1;
  double best_cost = 1e30;
  for (int S = 1; S <= max_split && S <= ngr; S *= 2) {
    if (S > 1 && ngr / S < 2) break;
    int c = cap[dev][S].load(std::memory_order_relaxed);
    if (c == 0) {
      int clusters = 0;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, (unsigned)S);
      cfg.blockDim = dim3((unsigned)threads);
      cfg.dynamicSmemBytes = smem_bytes;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 1;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = (unsigned)S;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, KERN, &cfg) != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = S == 1 ? sm_count() : 0;
      }
      c = clusters > 0 ? clusters * S : -1;
      cap[dev][S].store(c, std::memory_order_relaxed);
    }
    if (c < 0) continue;
    const double waves = (double)((tiles * S + c - 1) / c);
    const double cost = waves * ((ngr + S - 1) / S + 4 + (S > 1 ? 1 : 0));
    if (cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

// Tensor maps of the packed weights: rows of 128-K groups (GB bytes each) and,
// for GGUF, the tile-major d array as [N / 16 tiles, G * 128 bytes].
template <int FMT, int BW>
dial_status make_w_maps(const Params& p, CUtensorMap* wmap, CUtensorMap* dmap) {
  if (FMT == kQ4K || FMT == kQ6K) {  // the file's rows of super-blocks (144 / 210 bytes each)
    const int bb = FMT == kQ4K ? 144 : 210;
    dial_status s = tma::make_byte_map(wmap, p.w, p.N, (int64_t)(p.K / 256) * bb, FMT == kQ4K ? 144 : 224,
                                       BW, 0);
    *dmap = *wmap;  // unused
    return s;
  }
  constexpr bool gguf = FMT == kQ4 || FMT == kQ8;
  constexpr int GB = FMT == kQ4 ? 64 : 128;
  if (!gguf) {
    dial_status s = tma::make_byte_map(wmap, p.w, p.N, p.K, 128, BW, 128);
    *dmap = *wmap;  // unused
    return s;
  }
  dial_status s = tma::make_byte_map(wmap, p.w, p.N, (int64_t)p.G * GB, GB, BW, GB);
  if (s != DIAL_OK) return s;
  return tma::make_byte_map(dmap, p.gd, (p.N + 15) / 16, (int64_t)p.G * 128, 128, BW / 16, 0);
}

template <int FMT, bool BF16, typename YT, int BT, int NH>
dial_status launch_bt(const void* x, const Params& p, cudaStream_t st) {
  using L = Cfg<FMT, BT, NH>;
  constexpr auto kern = dequant_gemm_kernel<FMT, BF16, YT, BT, NH>;
  constexpr int smem = L::BYTES, BW = L::BW;
  CUtensorMap map;
  dial_status xs = make_x_map(&map, x, BF16, p.M, p.K, BT);
  if (xs != DIAL_OK) return xs;
  CUtensorMap wmap, dmap;
  dial_status ds = make_w_maps<FMT, BW>(p, &wmap, &dmap);
  if (ds != DIAL_OK) return ds;
  cudaError_t e = ensure_smem<kern>(smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dequant_gemm)");
  const int64_t wt = (p.N + BW - 1) / BW, tt = (p.M + BT - 1) / BT;
  const int S = choose_split<kern>(wt * tt, (p.nk + L::SPG - 1) / L::SPG, smem, L::MAX_SPLIT, L::THREADS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)wt, (unsigned)tt, (unsigned)S);
  cfg.blockDim = dim3(L::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)S;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, map, wmap, dmap, p);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(dequant_gemm_kernel)");
  return check_launch("dequant_gemm_kernel");
}

// 32-row token tiles for batched decode (M <= 32), 128-row ones above; the
// narrow CTA (128 weight rows, two per SM) or the wide one (256, one per SM).
constexpr bool kNarrowDecode = true, kNarrowPrefill = true;
template <int FMT, bool BF16, typename YT>
dial_status launch_one(const void* x, const Params& p, cudaStream_t st) {
  if (p.M <= 32) return launch_bt<FMT, BF16, YT, 32, kNarrowDecode ? 1 : 2>(x, p, st);
  if (p.M >= 256) return launch_bt<FMT, BF16, YT, 256, 1>(x, p, st);
  return launch_bt<FMT, BF16, YT, 128, kNarrowPrefill ? 1 : 2>(x, p, st);
}

}  // namespace

namespace tma {
dial_status make_byte_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                          int box_bytes, int box_rows, int swizzle_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (!aligned16(base) || row_bytes % 16 != 0 || (swizzle_bytes && box_bytes != swizzle_bytes))
    return fail(DIAL_ERR_MISALIGNED, "tensor map: base and row pitch must be 16-byte aligned");
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DIAL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DIAL_OK;
}
}  // namespace tma

bool gemm_sm100_supported(int64_t M, int64_t K, int64_t N) {
  (void)N;
  return M >= kGemmMinRows && K % 64 == 0 && K >= 64;
}

size_t gemm_sm100_gguf_workspace_bytes(int64_t M, int64_t K) {
  return M >= kGemmMinRows ? (size_t)((M * K * 2 + 255) / 256 * 256) : 0;
}

dial_status launch_w8a16_gemm_sm100(const void* x, dial_dtype xdt, const int8_t* q,
                                    const void* scale, dial_dtype sdt, void* y, int64_t M,
                                    int64_t K, int64_t N, cudaStream_t st) {
  const bool bf = xdt == DIAL_BF16;
  Params p{reinterpret_cast<const uint8_t*>(q), scale, nullptr, y, (int)M, (int)N, (int)K, 0,
           (int)(K / BK)};
  if (sdt == DIAL_F32)
    return bf ? launch_one<kW8F32, true, __nv_bfloat16>(x, p, st)
              : launch_one<kW8F32, false, __half>(x, p, st);
  return bf ? launch_one<kW8F16, true, __nv_bfloat16>(x, p, st)
            : launch_one<kW8F16, false, __half>(x, p, st);
}

dial_status launch_gguf_gemm_sm100(const void* x, dial_dtype xdt, const void* qs,
                                   const uint16_t* d, int type, void* y, int64_t M, int64_t K,
                                   int64_t N, void* ws, cudaStream_t st) {
  const void* xin = x;
  if (xdt == DIAL_F32) {  // the tensor cores take f16 operands: convert once
    __half* xh = static_cast<__half*>(ws);
    const int64_t n8 = M * K / 8;
    const unsigned grid = (unsigned)std::min<int64_t>((n8 + 255) / 256, (int64_t)sm_count() * 8);
    dial_status s = launch_pdl("to_f16_kernel", to_f16_kernel, dim3(grid), dim3(256), 0, st,
                               static_cast<const float*>(x), xh, n8);
    if (s != DIAL_OK) return s;
    xin = xh;
  }
  const int64_t G = gguf_groups(K);
  Params p{static_cast<const uint8_t*>(qs), nullptr, reinterpret_cast<const __half*>(d), y, (int)M,
           (int)N, (int)K, (int)G, (int)(K / BK)};
  if (type == DIAL_GGML_Q4_0) {
    if (xdt == DIAL_F32) return launch_one<kQ4, false, float>(xin, p, st);
    if (xdt == DIAL_F16) return launch_one<kQ4, false, __half>(xin, p, st);
    return launch_one<kQ4, true, __nv_bfloat16>(xin, p, st);
  }
  if (xdt == DIAL_F32) return launch_one<kQ8, false, float>(xin, p, st);
  if (xdt == DIAL_F16) return launch_one<kQ8, false, __half>(xin, p, st);
  return launch_one<kQ8, true, __nv_bfloat16>(xin, p, st);
}

dial_status launch_kquant_gemm_sm100(const void* x, dial_dtype xdt, const void* blocks, int type,
                                     void* y, int64_t M, int64_t K, int64_t N, cudaStream_t st) {
  if (xdt != DIAL_F16 && xdt != DIAL_BF16) return fail(DIAL_ERR_UNSUPPORTED_DTYPE, "K-quant GEMM: f16/bf16 x");
  Params p{static_cast<const uint8_t*>(blocks), nullptr, nullptr, y, (int)M, (int)N, (int)K, 0,
           (int)(K / BK)};
  if (type == DIAL_GGML_Q4_K) {
    if (xdt == DIAL_F16) return launch_one<kQ4K, false, __half>(x, p, st);
    return launch_one<kQ4K, true, __nv_bfloat16>(x, p, st);
  }
  if (K % 2048) return fail(DIAL_ERR_SHAPE, "Q6_K GEMM: K %% 2048 != 0");
  if (xdt == DIAL_F16) return launch_one<kQ6K, false, __half>(x, p, st);
  return launch_one<kQ6K, true, __nv_bfloat16>(x, p, st);
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
