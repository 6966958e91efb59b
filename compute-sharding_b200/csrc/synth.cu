// synth.cu — deterministic synthetic weights and activations generated on the device.
//
// The benchmark workloads are seeded synthetic models with the shapes and value distributions
// of the graded configurations (GGUF Q4_K/Q6_K blocks with fp16 d/dmin ~ |N(0, 0.02)|, uniform
// 6-bit sub-scales/mins and 4-bit quants, fp16 tied embedding ~ N(0, 0.02)).  Generating them
// on the device avoids staging gigabytes through the host; the bytes are identical to the host
// generator used by the tests because both use only integer hashing, exact integer-to-float
// conversion and single IEEE round-to-nearest multiplies:
//   mix64(key, c)   = SplitMix64 finaliser of key + (c + 1) * 0x9E3779B97F4A7C15
//   normal(key, c)  = (sum of the four 16-bit fields of mix64(key, c) - 131070) * 2^-16 * 1.7320508
//   Q4_K block b:   d, dmin = fp16(|normal(key, 24b + {0,1})| * sigma); bytes 4..143 are the
//                   little-endian bytes of mix64(key, 24b + 2 + i/8)
//   Q6_K block b:   bytes 0..207 from mix64(key, 32b + i/8); d = fp16(|normal(key, 32b+26)| * sigma/64)
//   F32/F16/BF16:   element i = mean + normal(key, i) * sigma
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

uint64_t mix64_host(uint64_t key, uint64_t ctr) { return mix64(key, ctr); }

uint64_t tensor_key(uint64_t seed, const char *name) {
  uint64_t h = 0xCBF29CE484222325ull;  // FNV-1a 64 of the tensor name
  for (const unsigned char *p = reinterpret_cast<const unsigned char *>(name); *p; ++p) {
    h ^= *p;
    h *= 0x100000001B3ull;
  }
  return mix64(seed, h);
}

__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t ctr) {
  const uint64_t u = mix64(key, ctr);
  const int s = int(u & 0xFFFF) + int((u >> 16) & 0xFFFF) + int((u >> 32) & 0xFFFF) + int((u >> 48) & 0xFFFF);
  const float v = __fmul_rn(float(s - 131070), 1.0f / 65536.0f);
  return __fmul_rn(v, 1.7320508f);
}

__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

__global__ void synth_q4k_kernel(uint64_t key, int64_t n_blocks, float sigma, uint8_t *__restrict__ out) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  uint8_t *p = out + b * BLOCK_Q4_K;
  const uint64_t base = uint64_t(b) * 24;
  const uint16_t d = f2h_bits(__fmul_rn(fabsf(synth_normal(key, base + 0)), sigma));
  const uint16_t dm = f2h_bits(__fmul_rn(fabsf(synth_normal(key, base + 1)), sigma));
  uint32_t *p32 = reinterpret_cast<uint32_t *>(p);  // 144 B blocks are 16 B aligned
  p32[0] = uint32_t(d) | (uint32_t(dm) << 16);
  // bytes 4..143: u64 word k supplies bytes 4 + 8k .. 11 + 8k (the 18th word only its low half)
  for (int k = 0; k < 17; ++k) {
    const uint64_t r = mix64(key, base + 2 + k);
    p32[1 + 2 * k] = uint32_t(r);
    p32[2 + 2 * k] = uint32_t(r >> 32);
  }
  p32[35] = uint32_t(mix64(key, base + 2 + 17));
}

__global__ void synth_q6k_kernel(uint64_t key, int64_t n_blocks, float sigma, uint8_t *__restrict__ out) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  uint8_t *p = out + b * BLOCK_Q6_K;  // 210 B blocks: 2 B aligned
  const uint64_t base = uint64_t(b) * 32;
  uint16_t *p16 = reinterpret_cast<uint16_t *>(p);
  for (int k = 0; k < 26; ++k) {
    const uint64_t r = mix64(key, base + k);
#pragma unroll
    for (int q = 0; q < 4; ++q) p16[4 * k + q] = uint16_t(r >> (16 * q));
  }
  p16[104] = f2h_bits(__fmul_rn(fabsf(synth_normal(key, base + 26)), __fmul_rn(sigma, 0.015625f)));
}

__global__ void synth_dense_kernel(int type, uint64_t key, int64_t n, float sigma, float mean, void *__restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = __fadd_rn(mean, __fmul_rn(synth_normal(key, uint64_t(i)), sigma));
  if (type == T_F16)
    reinterpret_cast<uint16_t *>(out)[i] = f2h_bits(v);
  else if (type == T_F32)
    reinterpret_cast<float *>(out)[i] = v;
  else {
    const uint32_t bits = __float_as_uint(v);
    reinterpret_cast<uint16_t *>(out)[i] = uint16_t((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
  }
}

cudaError_t synth_tensor(int type, uint64_t key, int64_t rows, int64_t K, float sigma, float mean, void *out,
                         cudaStream_t st) {
  if (rows <= 0 || K <= 0) return cudaSuccess;
  if (type == T_Q4_K || type == T_Q6_K) {
    if (K % QK_K) return cudaErrorInvalidValue;
    const int64_t nb = rows * (K / QK_K);
    const unsigned grid = unsigned((nb + 255) / 256);
    if (type == T_Q4_K)
      synth_q4k_kernel<<<grid, 256, 0, st>>>(key, nb, sigma, static_cast<uint8_t *>(out));
    else
      synth_q6k_kernel<<<grid, 256, 0, st>>>(key, nb, sigma, static_cast<uint8_t *>(out));
    return cudaGetLastError();
  }
  if (type != T_F16 && type != T_F32 && type != T_BF16) return cudaErrorInvalidValue;
  const int64_t n = rows * K;
  synth_dense_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(type, key, n, sigma, mean, out);
  return cudaGetLastError();
}

}  // namespace sfc
