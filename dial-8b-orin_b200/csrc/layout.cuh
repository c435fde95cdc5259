// Device layout of GGUF Q4_0 / Q8_0 weights used by every kernel here.
//
// A GGUF file (and candle's upload, worker_gguf.rs:500-505) keeps blocks of
// 32 weights with the f16 scale inside the block: Q4_0 {f16 d; u8 qs[16]}
// (element j in the low nibble of qs[j], element j+16 in the high nibble),
// Q8_0 {f16 d; i8 qs[32]}.  dial_gguf_repack splits a row of blocks into
//
//   qs : u8  [N, G*GB]       G = ceil(K/128) groups of 4 blocks (padding zero),
//                            GB = 64 (Q4_0) or 128 (Q8_0) bytes per group
//   d  : f16 [ceil(N/16), G, 16, 4]  the scales of a 16-row tile and one group
//                            are 128 contiguous bytes (one bulk copy); padding 0
//
// and interleaves the bytes of the 4 blocks of a group so that the 16 (Q4_0)
// or 32 (Q8_0) contiguous bytes a lane loads with 128-bit loads are exactly
// that lane's slice of the int8 tensor-core A fragment (m16n8k32: lane quad
// index t holds block elements 4t..4t+3 and 4t+16..4t+19):
//
//   Q4_0 byte 16*t + 4*j + i            = block j of the group, qs[4t + i]
//   Q8_0 byte 32*t + 8*j + i   (i < 4)  = block j, qs[4t + i]
//        byte 32*t + 8*j + i   (i >= 4) = block j, qs[4t + 16 + i - 4]
//
// Values and block scales are unchanged (dequantised weights stay bit-exact);
// only the byte order inside a row changes.  Activations quantised to Q8_0 for
// the integer path use the Q8_0 order.
#pragma once

#include <cstdint>

namespace dial {

constexpr int kQK = 32;           // weights per GGML block
constexpr int kBlocksPerGroup = 4;
constexpr int kGroupK = kQK * kBlocksPerGroup;  // 128 weights per group

__host__ __device__ constexpr int group_bytes(int ggml_type) { return ggml_type == 2 ? 64 : 128; }
__host__ __device__ constexpr int native_block_bytes(int ggml_type) { return ggml_type == 2 ? 18 : 34; }

__host__ __device__ inline int64_t gguf_groups(int64_t K) { return (K / kQK + 3) / 4; }

// Element index of the scale of block b (0 .. 4G-1) of row n in the d array.
__host__ __device__ inline int64_t gguf_d_index(int64_t n, int64_t b, int64_t G) {
  return (((n >> 4) * G + (b >> 2)) * 16 + (n & 15)) * 4 + (b & 3);
}
// Size of the d array in f16 elements.
__host__ __device__ inline int64_t gguf_d_elems(int64_t N, int64_t K) {
  return ((N + 15) / 16) * 16 * gguf_groups(K) * 4;
}

// Byte offset inside a group of qs byte `p` of block `j` (p indexes the
// native qs array: 0..15 for Q4_0, 0..31 for Q8_0).
__host__ __device__ inline int q4_0_offset(int j, int p) { return 16 * (p >> 2) + 4 * j + (p & 3); }
__host__ __device__ inline int q8_0_offset(int j, int p) {
  int hi = p >> 4;    // element in the upper half of the block
  int e = p & 15;
  return 32 * (e >> 2) + 8 * j + 4 * hi + (e & 3);
}

}  // namespace dial
