// logits.cu — tied-embedding / output logits with softcap and argmax.
//
// Replaces matmul_raw_top_k (crates/stage-forward-lab/src/real_math.rs:2119-2488) as used by
// sample_hidden_state_with_trace (real_forward.rs:904-986): scores = W h over every vocab row,
// 30*tanh(s/30) softcap, argmax with ties to the lowest index (strict '>' in index order).
//
// The 262144 x 2560 fp16 table (1.34 GB) is streamed once per pass: warps own rows, every lane
// reads 16 B per 256-column chunk (coalesced 5 KB per row), the normalised hidden state sits in
// registers (1 token) or shared memory (2..4 tokens).  Each CTA writes its best (score, index);
// a one-CTA pass reduces those.  Scores can also be written out for sampling and verify.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

constexpr int LOGIT_THREADS = 256;
constexpr int LOGIT_MAX_T = 4;

struct Best {
  float s;
  int64_t i;
};

__device__ __forceinline__ bool better(float s, int64_t i, float bs, int64_t bi) {
  return s > bs || (s == bs && i < bi);
}

__device__ __forceinline__ float softcap_score(float s, float cap) { return cap > 0.f ? cap * tanhf(s / cap) : s; }

__device__ __forceinline__ float wload(int type, const void *w, int64_t idx) {
  if (type == T_F16) return __half2float(reinterpret_cast<const __half *>(w)[idx]);
  if (type == T_F32) return reinterpret_cast<const float *>(w)[idx];
  return __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(w)[idx]) << 16);
}

// Vector path: F16 rows, dim % 256 == 0, dim <= 8192.
template <int T>
__global__ void __launch_bounds__(LOGIT_THREADS) logits_f16_kernel(const __half *__restrict__ w, int64_t vocab, int dim,
                                                                  const float *__restrict__ h, float cap,
                                                                  float *__restrict__ all_scores,
                                                                  float *__restrict__ part) {
  extern __shared__ float hs[];  // [T][dim]
  __shared__ float s_best[LOGIT_THREADS / 32][T];
  __shared__ int64_t s_idx[LOGIT_THREADS / 32][T];
  pdl_wait();
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < T * dim; i += blockDim.x) hs[i] = h[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = int64_t(blockIdx.x) * (LOGIT_THREADS / 32) + warp;
  const int64_t nw = int64_t(gridDim.x) * (LOGIT_THREADS / 32);
  const int nchunk = dim / 256;
  float bs[T];
  int64_t bi[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    bs[t] = -INFINITY;
    bi[t] = INT64_MAX;
  }
  for (int64_t r = gw; r < vocab; r += nw) {
    const uint4 *row = reinterpret_cast<const uint4 *>(w + r * dim);
    float acc[T];
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] = 0.f;
    // eight 256-element chunks of the row per pass, their loads issued together (streamed once:
    // evict-first); the sum runs over the chunks in order as before
    for (int c0 = 0; c0 < nchunk; c0 += 8) {
      uint4 u[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < nchunk) u[j] = __ldcs(row + (c0 + j) * 32 + lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (c0 + j >= nchunk) break;
        const int c = c0 + j;
        const __half2 *hp = reinterpret_cast<const __half2 *>(&u[j]);
        float wf[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(hp[k]);
          wf[2 * k] = f.x;
          wf[2 * k + 1] = f.y;
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float4 x0 = *reinterpret_cast<const float4 *>(&hs[t * dim + c * 256 + lane * 8]);
          const float4 x1 = *reinterpret_cast<const float4 *>(&hs[t * dim + c * 256 + lane * 8 + 4]);
          acc[t] += wf[0] * x0.x + wf[1] * x0.y + wf[2] * x0.z + wf[3] * x0.w + wf[4] * x1.x + wf[5] * x1.y +
                    wf[6] * x1.z + wf[7] * x1.w;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float s = softcap_score(warp_sum(acc[t]), cap);
      if (all_scores && lane == 0) all_scores[int64_t(t) * vocab + r] = s;
      if (s > bs[t]) {  // rows visit in increasing order: strict '>' keeps the lowest index
        bs[t] = s;
        bi[t] = r;
      }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int t = 0; t < T; ++t) {
      s_best[warp][t] = bs[t];
      s_idx[warp][t] = bi[t];
    }
  __syncthreads();
  if (threadIdx.x < T) {
    const int t = threadIdx.x;
    float b = -INFINITY;
    int64_t ib = INT64_MAX;
    for (int k = 0; k < LOGIT_THREADS / 32; ++k)
      if (better(s_best[k][t], s_idx[k][t], b, ib)) {
        b = s_best[k][t];
        ib = s_idx[k][t];
      }
    float *pp = part + (int64_t(blockIdx.x) * T + t) * 4;
    pp[0] = b;
    reinterpret_cast<int64_t *>(pp + 2)[0] = ib;
  }
}

// Generic path (any type/dim): one warp per row, scalar strided loads.
__global__ void __launch_bounds__(LOGIT_THREADS) logits_generic_kernel(int type, const void *__restrict__ w,
                                                                      int64_t vocab, int dim, const float *__restrict__ h,
                                                                      int T, float cap, float *__restrict__ all_scores,
                                                                      float *__restrict__ part) {
  __shared__ float s_best[LOGIT_THREADS / 32][LOGIT_MAX_T];
  __shared__ int64_t s_idx[LOGIT_THREADS / 32][LOGIT_MAX_T];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = int64_t(blockIdx.x) * (LOGIT_THREADS / 32) + warp;
  const int64_t nw = int64_t(gridDim.x) * (LOGIT_THREADS / 32);
  float bs[LOGIT_MAX_T];
  int64_t bi[LOGIT_MAX_T];
  for (int t = 0; t < LOGIT_MAX_T; ++t) {
    bs[t] = -INFINITY;
    bi[t] = INT64_MAX;
  }
  for (int64_t r = gw; r < vocab; r += nw) {
    for (int t = 0; t < T; ++t) {
      float a = 0.f;
      for (int k = lane; k < dim; k += 32) a += wload(type, w, r * dim + k) * h[int64_t(t) * dim + k];
      const float s = softcap_score(warp_sum(a), cap);
      if (all_scores && lane == 0) all_scores[int64_t(t) * vocab + r] = s;
      if (s > bs[t]) {
        bs[t] = s;
        bi[t] = r;
      }
    }
  }
  if (lane == 0)
    for (int t = 0; t < T; ++t) {
      s_best[warp][t] = bs[t];
      s_idx[warp][t] = bi[t];
    }
  __syncthreads();
  if (threadIdx.x < T) {
    const int t = threadIdx.x;
    float b = -INFINITY;
    int64_t ib = INT64_MAX;
    for (int k = 0; k < LOGIT_THREADS / 32; ++k)
      if (better(s_best[k][t], s_idx[k][t], b, ib)) {
        b = s_best[k][t];
        ib = s_idx[k][t];
      }
    float *pp = part + (int64_t(blockIdx.x) * T + t) * 4;
    pp[0] = b;
    reinterpret_cast<int64_t *>(pp + 2)[0] = ib;
  }
}

// part layout: per (cta, token) 4 floats = {score, pad, idx (int64)}.
__global__ void logits_reduce_kernel(const float *__restrict__ part, int n_cta, int T, int64_t *argmax_idx,
                                     float *argmax_score) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  float b = -INFINITY;
  int64_t ib = INT64_MAX;
  for (int c = lane; c < n_cta; c += 32) {
    const float *pp = part + (int64_t(c) * T + t) * 4;
    const float s = pp[0];
    const int64_t i = reinterpret_cast<const int64_t *>(pp + 2)[0];
    if (better(s, i, b, ib)) {
      b = s;
      ib = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, b, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, ib, o);
    if (better(os, oi, b, ib)) {
      b = os;
      ib = oi;
    }
  }
  if (lane == 0) {
    argmax_idx[t] = ib == INT64_MAX ? 0 : ib;
    argmax_score[t] = b;
  }
}

// Softcap and argmax of precomputed raw scores [n][vocab] (the tensor-core path of the logits for
// many rows): one CTA per row; thread j scans indices j, j + 1024, ... (four at a time when the row
// is 16-byte aligned) so each warp load is one contiguous piece of the row; every thread meets its
// indices in increasing order with strict '>', and the merge keeps the lowest index on ties, so the
// result is the lowest index of the maximum; capped scores are written back.
constexpr int ARGMAX_THREADS = 1024;

__global__ void __launch_bounds__(ARGMAX_THREADS) scores_argmax_kernel(float *__restrict__ scores, int64_t vocab,
                                                                      float cap, int64_t *__restrict__ idx_out,
                                                                      float *__restrict__ score_out) {
  __shared__ float s_b[ARGMAX_THREADS / 32];
  __shared__ int64_t s_i[ARGMAX_THREADS / 32];
  pdl_wait();
  pdl_launch_dependents();
  float *row = scores + int64_t(blockIdx.x) * vocab;
  float b = -INFINITY;
  int64_t bi = INT64_MAX;
  if (vocab % 4 == 0) {
    float4 *row4 = reinterpret_cast<float4 *>(row);
    for (int64_t j = threadIdx.x; j < vocab / 4; j += ARGMAX_THREADS) {
      float4 v = row4[j];
      v.x = softcap_score(v.x, cap);
      v.y = softcap_score(v.y, cap);
      v.z = softcap_score(v.z, cap);
      v.w = softcap_score(v.w, cap);
      row4[j] = v;
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (e[k] > b) {
          b = e[k];
          bi = 4 * j + k;
        }
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += ARGMAX_THREADS) {
      const float v = softcap_score(row[i], cap);
      row[i] = v;
      if (v > b) {
        b = v;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, b, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ob, oi, b, bi)) {
      b = ob;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    s_b[threadIdx.x >> 5] = b;
    s_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < ARGMAX_THREADS / 32; ++w)
      if (better(s_b[w], s_i[w], b, bi)) {
        b = s_b[w];
        bi = s_i[w];
      }
    idx_out[blockIdx.x] = bi == INT64_MAX ? 0 : bi;
    score_out[blockIdx.x] = b;
  }
}

cudaError_t scores_argmax(float *scores, int64_t n, int64_t vocab, float cap, int64_t *idx, float *score,
                          cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  return launch_pdl(scores_argmax_kernel, dim3(unsigned(n)), dim3(ARGMAX_THREADS), 0, st, scores, vocab, cap, idx,
                    score);
}

// CTAs of a pass over the table with T rows: four per SM for one row (63 registers a thread, so
// 32 warps per SM keep their loads in flight), two per SM for more rows (more registers a thread).
static int logits_ctas(int T) { return (T == 1 ? 4 : 2) * num_sms(); }

size_t logits_scratch_bytes(int64_t n_tok) {
  const int T = int(n_tok < LOGIT_MAX_T ? n_tok : LOGIT_MAX_T);  // the first (widest) pass; a later
  return size_t(logits_ctas(T)) * T * 4 * sizeof(float);         // one-row pass needs no more
}

cudaError_t logits_argmax(int type, const void *w, int64_t vocab, int dim, const float *h, int64_t n_tok, float cap,
                          float *all_scores, int64_t *argmax_idx, float *argmax_score, void *scratch,
                          size_t scratch_bytes, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (vocab <= 0 || dim <= 0) return cudaErrorInvalidValue;
  if (scratch_bytes < logits_scratch_bytes(n_tok)) return cudaErrorInvalidValue;
  float *part = static_cast<float *>(scratch);
  for (int64_t t0 = 0; t0 < n_tok; t0 += LOGIT_MAX_T) {
    const int T = int(n_tok - t0 < LOGIT_MAX_T ? n_tok - t0 : LOGIT_MAX_T);
    const int ctas = logits_ctas(T);
    const float *hx = h + t0 * dim;
    float *as = all_scores ? all_scores + t0 * vocab : nullptr;
    cudaError_t e;
    if (type == T_F16 && dim % 256 == 0 && dim <= 8192) {
      const size_t smem = size_t(T) * dim * sizeof(float);
      const __half *wh = static_cast<const __half *>(w);
      switch (T) {
        case 1:
          cudaFuncSetAttribute(logits_f16_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
          e = launch_pdl(logits_f16_kernel<1>, dim3(ctas), dim3(LOGIT_THREADS), smem, st, wh, vocab, dim, hx, cap, as,
                         part);
          break;
        case 2:
          cudaFuncSetAttribute(logits_f16_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
          e = launch_pdl(logits_f16_kernel<2>, dim3(ctas), dim3(LOGIT_THREADS), smem, st, wh, vocab, dim, hx, cap, as,
                         part);
          break;
        case 3:
          cudaFuncSetAttribute(logits_f16_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
          e = launch_pdl(logits_f16_kernel<3>, dim3(ctas), dim3(LOGIT_THREADS), smem, st, wh, vocab, dim, hx, cap, as,
                         part);
          break;
        default:
          cudaFuncSetAttribute(logits_f16_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
          e = launch_pdl(logits_f16_kernel<4>, dim3(ctas), dim3(LOGIT_THREADS), smem, st, wh, vocab, dim, hx, cap, as,
                         part);
          break;
      }
    } else if (type == T_F16 || type == T_F32 || type == T_BF16) {
      e = launch_pdl(logits_generic_kernel, dim3(ctas), dim3(LOGIT_THREADS), 0, st, type, w, vocab, dim, hx, T, cap,
                     as, part);
    } else {
      return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    e = launch_pdl(logits_reduce_kernel, dim3(1), dim3(32 * LOGIT_MAX_T), 0, st, (const float *)part, ctas, T,
                   argmax_idx + t0, argmax_score + t0);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace sfc
