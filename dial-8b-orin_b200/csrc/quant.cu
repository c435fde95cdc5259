// Weight quantisers, dequantisers and the GGUF repack (load-time work).
//
// Bit-exactness: every rounding step of the reference quantisers is spelled
// out with _rn intrinsics so nvcc cannot contract a multiply and an add into
// one FMA (which rounds once instead of twice).
//   W8A16: worker_w8a16.rs:334-341   scale = max|w|/127 (1 if 0), inv = 1/scale,
//                                     q = clamp(round(w*inv), -127, 127)  (round
//                                     = half away from zero, CUDA roundf)
//   Q4_0 : GGML quantize_row_q4_0_ref  max = signed value of largest |w| (first
//          wins), d = max/-8, id = 1/d (0 if d == 0), q = min(15, (int)(w*id + 8.5))
//   Q8_0 : GGML quantize_row_q8_0_ref  d = max|w|/127, id = 1/d (0 if d == 0),
//          q = roundf(w*id)
#include "common.cuh"
#include "layout.cuh"
#include "quant.cuh"

namespace dial {

// ------------------------------------------------------------------ W8A16
template <typename WT>
__global__ void __launch_bounds__(256) w8a16_quantize_kernel(const WT* __restrict__ w, int64_t K,
                                                             int8_t* __restrict__ q,
                                                             float* __restrict__ s32,
                                                             __half* __restrict__ s16) {
  const int64_t row = blockIdx.x;
  const WT* wr = w + row * K;
  float m = 0.0f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(Act<WT>::to_f32(wr[k])));
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  const float max_abs = red[0];
  const float scale = max_abs > 0.0f ? __fdiv_rn(max_abs, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  int8_t* qr = q + row * K;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    float r = roundf(__fmul_rn(Act<WT>::to_f32(wr[k]), inv));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    qr[k] = (int8_t)(int)r;
  }
  if (threadIdx.x == 0) {
    if (s32) s32[row] = scale;
    if (s16) s16[row] = __float2half_rn(scale);
  }
}

template <typename ST, typename OT>
__global__ void w8a16_dequantize_kernel(const int8_t* __restrict__ q, const ST* __restrict__ scale,
                                        int64_t N, int64_t K, OT* __restrict__ out) {
  const int64_t total = N * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float s = Act<ST>::to_f32(scale[i / K]);
    out[i] = Act<OT>::from_f32(__fmul_rn((float)q[i], s));
  }
}

// ------------------------------------------------------------------ GGUF
// One thread per (row, block): native block -> split/interleaved layout.
__global__ void gguf_repack_kernel(const uint8_t* __restrict__ blocks, int type, int64_t N,
                                   int64_t nb, int64_t G, uint8_t* __restrict__ qs,
                                   __half* __restrict__ d) {
  const int64_t nbp = G * kBlocksPerGroup;  // padded blocks per row
  const int64_t total = N * nbp;
  const int gb = group_bytes(type), bb = native_block_bytes(type), nq = bb - 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / nbp, b = i % nbp;
    const int64_t g = b / kBlocksPerGroup;
    const int j = (int)(b % kBlocksPerGroup);
    uint8_t* dst = qs + n * G * gb + g * gb;
    if (b < nb) {
      const uint8_t* src = blocks + (n * nb + b) * bb;
      d[gguf_d_index(n, b, G)] = __ushort_as_half((unsigned short)(src[0] | (src[1] << 8)));
      for (int p = 0; p < nq; ++p)
        dst[type == DIAL_GGML_Q4_0 ? q4_0_offset(j, p) : q8_0_offset(j, p)] = src[2 + p];
    } else {
      d[gguf_d_index(n, b, G)] = __ushort_as_half(0);
      for (int p = 0; p < nq; ++p) dst[type == DIAL_GGML_Q4_0 ? q4_0_offset(j, p) : q8_0_offset(j, p)] = 0;
    }
  }
}

__global__ void gguf_unpack_kernel(const uint8_t* __restrict__ qs, const __half* __restrict__ d,
                                   int type, int64_t N, int64_t nb, int64_t G,
                                   uint8_t* __restrict__ blocks) {
  const int64_t total = N * nb;
  const int gb = group_bytes(type), bb = native_block_bytes(type), nq = bb - 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / nb, b = i % nb;
    const int64_t g = b / kBlocksPerGroup;
    const int j = (int)(b % kBlocksPerGroup);
    const uint8_t* src = qs + n * G * gb + g * gb;
    uint8_t* dst = blocks + i * bb;
    const unsigned short h = __half_as_ushort(d[gguf_d_index(n, b, G)]);
    dst[0] = (uint8_t)(h & 0xff);
    dst[1] = (uint8_t)(h >> 8);
    for (int p = 0; p < nq; ++p)
      dst[2 + p] = src[type == DIAL_GGML_Q4_0 ? q4_0_offset(j, p) : q8_0_offset(j, p)];
  }
}

// One thread per (row, block) of the f32 weight.
__global__ void gguf_quantize_kernel(const float* __restrict__ w, int type, int64_t N, int64_t K,
                                     int64_t G, uint8_t* __restrict__ qs, __half* __restrict__ d) {
  const int64_t nb = K / kQK, nbp = G * kBlocksPerGroup;
  const int64_t total = N * nbp;
  const int gb = group_bytes(type);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / nbp, b = i % nbp;
    const int64_t g = b / kBlocksPerGroup;
    const int j = (int)(b % kBlocksPerGroup);
    uint8_t* dst = qs + n * G * gb + g * gb;
    if (b >= nb) {
      d[gguf_d_index(n, b, G)] = __ushort_as_half(0);
      const int nq = type == DIAL_GGML_Q4_0 ? 16 : 32;
      for (int p = 0; p < nq; ++p) dst[type == DIAL_GGML_Q4_0 ? q4_0_offset(j, p) : q8_0_offset(j, p)] = 0;
      continue;
    }
    const float* x = w + n * K + b * kQK;
    if (type == DIAL_GGML_Q4_0) {
      float amax = 0.0f, maxv = 0.0f;
      for (int e = 0; e < kQK; ++e) {
        const float v = x[e];
        if (amax < fabsf(v)) { amax = fabsf(v); maxv = v; }
      }
      const float dd = __fdiv_rn(maxv, -8.0f);
      const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
      d[gguf_d_index(n, b, G)] = __float2half_rn(dd);
      for (int p = 0; p < 16; ++p) {
        const float x0 = __fadd_rn(__fmul_rn(x[p], id), 8.5f);
        const float x1 = __fadd_rn(__fmul_rn(x[16 + p], id), 8.5f);
        int i0 = (int)x0, i1 = (int)x1;  // truncation, as the C reference
        i0 = i0 > 15 ? 15 : (i0 < 0 ? 0 : i0);
        i1 = i1 > 15 ? 15 : (i1 < 0 ? 0 : i1);
        dst[q4_0_offset(j, p)] = (uint8_t)(i0 | (i1 << 4));
      }
    } else {
      float amax = 0.0f;
      for (int e = 0; e < kQK; ++e) amax = fmaxf(amax, fabsf(x[e]));
      const float dd = __fdiv_rn(amax, 127.0f);
      const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
      d[gguf_d_index(n, b, G)] = __float2half_rn(dd);
      for (int p = 0; p < 32; ++p) dst[q8_0_offset(j, p)] = (uint8_t)(int8_t)(int)roundf(__fmul_rn(x[p], id));
    }
  }
}

template <typename OT>
__global__ void gguf_dequantize_kernel(const uint8_t* __restrict__ qs, const __half* __restrict__ d,
                                       int type, int64_t N, int64_t K, int64_t G,
                                       OT* __restrict__ out) {
  const int64_t total = N * K;
  const int gb = group_bytes(type);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / K, k = i % K;
    const int64_t b = k / kQK;
    const int e = (int)(k % kQK);
    const int64_t g = b / kBlocksPerGroup;
    const int j = (int)(b % kBlocksPerGroup);
    const uint8_t* src = qs + n * G * gb + g * gb;
    int qv;
    if (type == DIAL_GGML_Q4_0) {
      const uint8_t byte = src[q4_0_offset(j, e & 15)];
      qv = (e < 16 ? (byte & 0xf) : (byte >> 4)) - 8;
    } else {
      qv = (int8_t)src[q8_0_offset(j, e)];
    }
    out[i] = Act<OT>::from_f32(__fmul_rn(__half2float(d[gguf_d_index(n, b, G)]), (float)qv));
  }
}

// ------------------------------------------------------------------ launchers
static unsigned grid_for(int64_t total, int threads) {
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

dial_status launch_w8a16_quantize(const void* w, dial_dtype wdt, int64_t N, int64_t K, int8_t* q,
                                  void* scale, dial_dtype sdt, cudaStream_t st) {
  float* s32 = sdt == DIAL_F32 ? static_cast<float*>(scale) : nullptr;
  __half* s16 = sdt == DIAL_F16 ? static_cast<__half*>(scale) : nullptr;
  if (wdt == DIAL_F32)
    w8a16_quantize_kernel<float><<<(unsigned)N, 256, 0, st>>>(static_cast<const float*>(w), K, q, s32, s16);
  else
    w8a16_quantize_kernel<__half><<<(unsigned)N, 256, 0, st>>>(static_cast<const __half*>(w), K, q, s32, s16);
  return check_launch("w8a16_quantize_kernel");
}

dial_status launch_w8a16_dequantize(const int8_t* q, const void* scale, dial_dtype sdt, int64_t N,
                                    int64_t K, void* w, dial_dtype wdt, cudaStream_t st) {
  const unsigned grid = grid_for(N * K, 256);
#define DQ(ST, OT) \
  w8a16_dequantize_kernel<ST, OT><<<grid, 256, 0, st>>>(q, static_cast<const ST*>(scale), N, K, static_cast<OT*>(w))
  if (sdt == DIAL_F32) {
    if (wdt == DIAL_F32) DQ(float, float);
    else if (wdt == DIAL_F16) DQ(float, __half);
    else DQ(float, __nv_bfloat16);
  } else {
    if (wdt == DIAL_F32) DQ(__half, float);
    else if (wdt == DIAL_F16) DQ(__half, __half);
    else DQ(__half, __nv_bfloat16);
  }
#undef DQ
  return check_launch("w8a16_dequantize_kernel");
}

dial_status launch_gguf_repack(const void* blocks, int type, int64_t N, int64_t K, void* qs,
                               uint16_t* d, cudaStream_t st) {
  const int64_t G = gguf_groups(K);
  gguf_repack_kernel<<<grid_for(N * G * 4, 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(blocks), type, N, K / kQK, G, static_cast<uint8_t*>(qs),
      reinterpret_cast<__half*>(d));
  return check_launch("gguf_repack_kernel");
}

dial_status launch_gguf_unpack(const void* qs, const uint16_t* d, int type, int64_t N, int64_t K,
                               void* blocks, cudaStream_t st) {
  const int64_t G = gguf_groups(K);
  gguf_unpack_kernel<<<grid_for(N * (K / kQK), 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(qs), reinterpret_cast<const __half*>(d), type, N, K / kQK, G,
      static_cast<uint8_t*>(blocks));
  return check_launch("gguf_unpack_kernel");
}

dial_status launch_gguf_quantize(const float* w, int type, int64_t N, int64_t K, void* qs,
                                 uint16_t* d, cudaStream_t st) {
  const int64_t G = gguf_groups(K);
  gguf_quantize_kernel<<<grid_for(N * G * 4, 128), 128, 0, st>>>(
      w, type, N, K, G, static_cast<uint8_t*>(qs), reinterpret_cast<__half*>(d));
  return check_launch("gguf_quantize_kernel");
}

dial_status launch_gguf_dequantize(const void* qs, const uint16_t* d, int type, int64_t N,
                                   int64_t K, void* w, dial_dtype wdt, cudaStream_t st) {
  const int64_t G = gguf_groups(K);
  const unsigned grid = grid_for(N * K, 256);
  const uint8_t* q = static_cast<const uint8_t*>(qs);
  const __half* dd = reinterpret_cast<const __half*>(d);
  if (wdt == DIAL_F32)
    gguf_dequantize_kernel<float><<<grid, 256, 0, st>>>(q, dd, type, N, K, G, static_cast<float*>(w));
  else if (wdt == DIAL_F16)
    gguf_dequantize_kernel<__half><<<grid, 256, 0, st>>>(q, dd, type, N, K, G, static_cast<__half*>(w));
  else
    gguf_dequantize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(q, dd, type, N, K, G,
                                                                 static_cast<__nv_bfloat16*>(w));
  return check_launch("gguf_dequantize_kernel");
}

}  // namespace dial
