// ops.cu — norms, embedding, q/k/v post-processing with KV append, and GQA attention.
//
// Reference semantics (crates/stage-forward-lab/src/):
//   rms_norm_inplace            real_math.rs:30-47     x * (1/sqrt(mean(x^2)+eps)) * w
//   per_head_rms_norm(_no_scale) real_math.rs:2746-2776 x *= scale * w   (v: no weight)
//   rope_angles / apply          real_math.rs:2576-2639 NeoX half split, theta = pos*inv_freq*freq
//   gqa_attention_seq_with_window_and_limit real_math.rs:2697-2744 (no 1/sqrt(d) scale)
//   embed_tokens                 real_forward.rs:848-871  f16 row * sqrt(hidden)
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh[i];
  return r;
}

// ---------------------------------------------------------------- rms norm
// The lane's 8 values of 256-element block b of a row of `dim` floats (zero past the row's end).
__device__ __forceinline__ void row_block8(const float *__restrict__ row, int dim, int b, float (&v)[8]) {
  const int c = b * 256 + int(threadIdx.x & 31) * 8;
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = c + e < dim ? row[c + e] : 0.f;
}

// out = (x * scale) * w per row, the sum of squares in the residual-stream norm order (row_sumsq).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                      int dim, float eps, float *__restrict__ out) {
  __shared__ float red[64];
  pdl_wait();
  pdl_launch_dependents();
  const float *xr = x + int64_t(blockIdx.x) * dim;
  float *o = out + int64_t(blockIdx.x) * dim;
  const float ss = row_sumsq<8>((dim + 255) / 256, red, [&](int b, float (&v)[8]) { row_block8(xr, dim, b, v); });
  const float scale = 1.0f / sqrtf(ss / float(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += 256) o[i] = (xr[i] * scale) * w[i];
}

cudaError_t rms_norm(const float *x, const float *w, int64_t n_tok, int dim, float eps, float *out, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  return launch_pdl(rms_norm_kernel, dim3(unsigned(n_tok)), dim3(256), 0, st, x, w, dim, eps, out);
}

// r = resid + (w_post ? rms_norm(a) * w_post : a); r *= layer_scale; resid = r;
// if want_xn: xn = w_next ? rms_norm(r) * w_next : r.  Both norms sum in the residual-stream norm
// order and r is formed as resid_add forms it, so a stage that ends here hands the next stage the
// bits that the fused prologue of the following layer computes inside a single stage.
__global__ void __launch_bounds__(256) add_norm_kernel(float *__restrict__ resid, const float *__restrict__ a,
                                                      const float *__restrict__ w_post,
                                                      const float *__restrict__ layer_scale, int want_xn,
                                                      const float *__restrict__ w_next, float *__restrict__ xn,
                                                      int dim, float eps) {
  extern __shared__ float buf[];
  __shared__ float red[64];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t base = int64_t(blockIdx.x) * dim;
  const int nb = (dim + 255) / 256;
  float sc = 1.0f;
  if (w_post) {
    const float ss = row_sumsq<8>(nb, red, [&](int b, float (&v)[8]) { row_block8(a + base, dim, b, v); });
    sc = 1.0f / sqrtf(ss / float(dim) + eps);
  }
  const float ls = layer_scale ? layer_scale[0] : 1.0f;
  for (int i = threadIdx.x; i < dim; i += 256) {
    const float r = resid_add(a[base + i], sc, w_post, w_post ? w_post[i] : 0.f, resid[base + i], layer_scale, ls);
    resid[base + i] = r;
    buf[i] = r;
  }
  if (!want_xn) return;
  __syncthreads();
  if (!w_next) {
    for (int i = threadIdx.x; i < dim; i += 256) xn[base + i] = buf[i];
    return;
  }
  const float ss2 = row_sumsq<8>(nb, red, [&](int b, float (&v)[8]) { row_block8(buf, dim, b, v); });
  const float sc2 = 1.0f / sqrtf(ss2 / float(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += 256) xn[base + i] = (buf[i] * sc2) * w_next[i];
}

cudaError_t add_norm(float *resid, const float *a, const float *w_post, const float *layer_scale, int want_xn,
                     const float *w_next, float *xn, int64_t n_tok, int dim, float eps, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  return launch_pdl(add_norm_kernel, dim3(unsigned(n_tok)), dim3(256), size_t(dim) * 4, st, resid, a, w_post,
                    layer_scale, want_xn, w_next, xn, dim, eps);
}

// Decode-graph bookkeeping: record the sampled token, advance the step counter and every
// sequence's cache position by its token count.
__global__ void decode_advance_kernel(const int64_t *__restrict__ tok, int64_t *__restrict__ out_tokens,
                                      int32_t *__restrict__ step, SeqInfo *__restrict__ seqs, int n_seq,
                                      int64_t max_steps) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int s = *step;
    if (s < max_steps) out_tokens[s] = tok[0];
    *step = s + 1;
  }
  for (int i = threadIdx.x; i < n_seq; i += blockDim.x) seqs[i].pos0 += seqs[i].n_tok;
}

cudaError_t decode_advance(const int64_t *tok, int64_t *out_tokens, int32_t *step, SeqInfo *seqs, int n_seq,
                           int64_t max_steps, cudaStream_t st) {
  return launch_pdl(decode_advance_kernel, dim3(1), dim3(128), 0, st, tok, out_tokens, step, seqs, n_seq, max_steps);
}

// ---------------------------------------------------------------- embedding
__global__ void __launch_bounds__(256) embed_kernel(int type, const void *__restrict__ table, int64_t vocab, int dim,
                                                   const void *__restrict__ ids, int ids64, float *__restrict__ out,
                                                   unsigned *err) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t id = ids64 ? reinterpret_cast<const int64_t *>(ids)[blockIdx.x]
                           : int64_t(reinterpret_cast<const uint32_t *>(ids)[blockIdx.x]);
  float *o = out + int64_t(blockIdx.x) * dim;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && err) atomicExch(err, DEV_BAD_ARG);
    for (int i = threadIdx.x; i < dim; i += 256) o[i] = 0.f;
    return;
  }
  const float scale = sqrtf(float(dim));
  for (int i = threadIdx.x; i < dim; i += 256) {
    float v;
    if (type == T_F16)
      v = __half2float(reinterpret_cast<const __half *>(table)[int64_t(id) * dim + i]);
    else if (type == T_F32)
      v = reinterpret_cast<const float *>(table)[int64_t(id) * dim + i];
    else
      v = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(table)[int64_t(id) * dim + i]) << 16);
    o[i] = __fmul_rn(v, scale);
  }
}

cudaError_t embed(int type, const void *table, int64_t vocab, int dim, const void *ids, int ids64, int64_t n_tok,
                  float *out, unsigned *err, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (type != T_F16 && type != T_F32 && type != T_BF16) return cudaErrorInvalidValue;
  return launch_pdl(embed_kernel, dim3(unsigned(n_tok)), dim3(256), 0, st, type, table, vocab, dim, ids, ids64, out,
                    err);
}

// ---------------------------------------------------------------- q/k/v post + KV append
// grid (n_tok, n_heads + 2*n_kv); one CTA normalises (and rotates) one head of one token.
__global__ void __launch_bounds__(256) qkv_post_kernel(float *__restrict__ q, const float *__restrict__ k,
                                                      const float *__restrict__ v, int q_ld, int kv_ld, KVLayer kv,
                                                      const SeqInfo *__restrict__ seqs,
                                                      const int32_t *__restrict__ tok_seq,
                                                      const int32_t *__restrict__ rope_pos, AttnParams p) {
  __shared__ float hv[1024];
  __shared__ float sh[8];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, slot = blockIdx.y;
  const int hd = p.head_dim;
  int kind, head;  // 0 q, 1 k, 2 v
  if (slot < p.n_heads) {
    kind = 0;
    head = slot;
  } else if (slot < p.n_heads + p.n_kv) {
    kind = 1;
    head = slot - p.n_heads;
  } else {
    kind = 2;
    head = slot - p.n_heads - p.n_kv;
  }
  const float *src = kind == 0 ? q + int64_t(t) * q_ld : (kind == 1 ? k : v) + int64_t(t) * kv_ld;
  src += head * hd;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hd; i += 256) {
    const float x = src[i];
    hv[i] = x;
    ss += x * x;
  }
  ss = block_sum<256>(ss, sh);
  const float scale = 1.0f / sqrtf(ss / float(hd) + p.eps);
  const float *nw = kind == 0 ? p.q_norm : (kind == 1 ? p.k_norm : nullptr);
  if (kind == 2 || nw) {
    for (int i = threadIdx.x; i < hd; i += 256) hv[i] = hv[i] * (nw ? scale * nw[i] : scale);
  }
  __syncthreads();
  const SeqInfo sq = seqs[tok_seq[t]];
  const int pos = sq.pos0 + (t - sq.tok0);          // cache position of this row
  const int rpos = rope_pos ? rope_pos[t] : pos;     // rotary position (tree nodes: prefix + depth)
  if (kind != 2 && p.rope_freqs) {
    const int hde = hd & ~1;
    const int rd = min(p.rotary_dim, hde) & ~1;
    const int n_ang = rd / 2, half = hde / 2;
    const float denom = p.proportional ? float(hde) : float(rd);
    for (int i = threadIdx.x; i < n_ang; i += 256) {
      const float inv_freq = 1.0f / powf(p.rope_theta, 2.0f * float(i) / denom);
      const float fs = i < p.n_freqs ? p.rope_freqs[i] : 1.0f;
      const float th = float(rpos) * inv_freq * fs;
      float sn, cs;
      sincosf(th, &sn, &cs);
      const float x0 = hv[i], x1 = hv[half + i];
      hv[i] = x0 * cs - x1 * sn;
      hv[half + i] = x0 * sn + x1 * cs;
    }
    __syncthreads();
  }
  if (kind == 0) {
    float *dst = q + int64_t(t) * q_ld + head * hd;
    for (int i = threadIdx.x; i < hd; i += 256) dst[i] = hv[i];
  } else {
    const int64_t off = int64_t(sq.slot) * kv.slot_stride + (kind == 2 ? kv.slot_stride / 2 : 0) +
                        (int64_t(head) * p.max_ctx + pos) * hd;
    if (pos >= p.max_ctx) return;  // host rejects overflow; never write past the slot
    if (p.kv_f32) {
      float *dst = reinterpret_cast<float *>(kv.base) + off;
      for (int i = threadIdx.x; i < hd; i += 256) dst[i] = hv[i];
    } else {
      __half *dst = reinterpret_cast<__half *>(kv.base) + off;
      for (int i = threadIdx.x; i < hd; i += 256) dst[i] = __float2half_rn(hv[i]);
    }
  }
}

cudaError_t qkv_post(float *q, const float *k, const float *v, int q_ld, int kv_ld, KVLayer kv, const SeqInfo *seqs,
                     const int32_t *tok_seq, const int32_t *rope_pos, int64_t n_tok, const AttnParams &p,
                     cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (p.head_dim > 1024) return cudaErrorInvalidValue;
  // a layer reading another layer's cache (kv_shared) normalises and rotates only its q heads
  const unsigned heads = unsigned(p.n_heads + (p.kv_shared ? 0 : 2 * p.n_kv));
  return launch_pdl(qkv_post_kernel, dim3(unsigned(n_tok), heads), dim3(256), 0, st, q, k, v, q_ld, kv_ld, kv, seqs,
                    tok_seq, rope_pos, p);
}

// ---------------------------------------------------------------- attention
// grid (n_tok, n_kv, n_split), 8 warps.  Each warp walks a strided subset of the CTA's key
// range with an online softmax for the G = n_heads/n_kv query heads that share the kv head;
// warps then merge in shared memory.  With n_split > 1 the CTA writes (m, l, acc) partials
// and attn_combine_kernel merges them.
constexpr int ATT_WARPS = 8;
constexpr int ATT_MAXG = 8;

template <int EPL, bool KV32>
__global__ void __launch_bounds__(ATT_WARPS * 32) attention_kernel(
    const float *__restrict__ q, float *__restrict__ out, KVLayer kv, const SeqInfo *__restrict__ seqs,
    const int32_t *__restrict__ tok_seq, const int32_t *__restrict__ tok_limit, const uint64_t *__restrict__ tok_mask,
    AttnParams p, int n_split, float *__restrict__ part) {
  __shared__ float s_m[ATT_WARPS][ATT_MAXG], s_l[ATT_WARPS][ATT_MAXG];
  __shared__ float s_acc[ATT_MAXG][32 * EPL];
  __shared__ float s_tmp[ATT_WARPS][32 * EPL];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = p.head_dim, G = p.n_heads / p.n_kv;
  const SeqInfo sq = seqs[tok_seq[t]];
  const int pos = sq.pos0 + (t - sq.tok0);
  const int limit = tok_limit ? tok_limit[t] : pos + 1;
  const uint64_t mask = tok_mask ? tok_mask[t] : ~0ull;
  const void *kbase = reinterpret_cast<const char *>(kv.base) +
                      (int64_t(sq.slot) * kv.slot_stride) * (KV32 ? 4 : 2);
  const void *vbase = reinterpret_cast<const char *>(kbase) + (kv.slot_stride / 2) * (KV32 ? 4 : 2);
  const int w0 = p.window > 0 ? max(0, limit - p.window) : 0;
  const int span = max(0, limit - w0);
  const int chunk = (span + n_split - 1) / n_split;
  const int k_begin = w0 + split * chunk, k_end = min(limit, k_begin + chunk);

  float qv[ATT_MAXG][EPL];
#pragma unroll
  for (int g = 0; g < ATT_MAXG; ++g)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane * EPL + e;
      qv[g][e] = (g < G && d < hd) ? q[int64_t(t) * p.n_heads * hd + (kvh * G + g) * hd + d] : 0.f;
    }
  float m[ATT_MAXG], l[ATT_MAXG], acc[ATT_MAXG][EPL];
#pragma unroll
  for (int g = 0; g < ATT_MAXG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
  }
  const int64_t head_off = int64_t(kvh) * p.max_ctx * hd;
  for (int key = k_begin + warp; key < k_end; key += ATT_WARPS) {
    if (key >= sq.pos0 && key - sq.pos0 < 64 && !((mask >> (key - sq.pos0)) & 1ull)) continue;
    float kf[EPL], vf[EPL];
    const int64_t off = head_off + int64_t(key) * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const bool in = lane * EPL + e < hd;
      if (KV32) {
        kf[e] = in ? reinterpret_cast<const float *>(kbase)[off + e] : 0.f;
        vf[e] = in ? reinterpret_cast<const float *>(vbase)[off + e] : 0.f;
      } else {
        kf[e] = in ? __half2float(reinterpret_cast<const __half *>(kbase)[off + e]) : 0.f;
        vf[e] = in ? __half2float(reinterpret_cast<const __half *>(vbase)[off + e]) : 0.f;
      }
    }
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
      if (g >= G) break;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) s += qv[g][e] * kf[e];
      s = warp_sum(s);
      const float mn = fmaxf(m[g], s);
      const float alpha = expf(m[g] - mn);  // exp(-inf) = 0 on the first key
      const float pr = expf(s - mn);
      l[g] = l[g] * alpha + pr;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] = acc[g][e] * alpha + pr * vf[e];
      m[g] = mn;
    }
  }
  // merge warps in a fixed order (deterministic)
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
  __syncthreads();
  float mw[ATT_MAXG], lt[ATT_MAXG];
#pragma unroll
  for (int g = 0; g < ATT_MAXG; ++g) {
    float M = -INFINITY;
    for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, s_m[w][g]);
    mw[g] = M;
    float L = 0.f;
    for (int w = 0; w < ATT_WARPS; ++w) L += M == -INFINITY ? 0.f : s_l[w][g] * expf(s_m[w][g] - M);
    lt[g] = L;
  }
#pragma unroll
  for (int g = 0; g < ATT_MAXG; ++g) {
    if (g >= G) break;
    const float scw = mw[g] == -INFINITY ? 0.f : expf(m[g] - mw[g]);
#pragma unroll
    for (int e = 0; e < EPL; ++e) s_tmp[warp][lane * EPL + e] = acc[g][e] * scw;
    __syncthreads();
    for (int d = threadIdx.x; d < 32 * EPL; d += blockDim.x) {
      float a = 0.f;
      for (int w = 0; w < ATT_WARPS; ++w) a += s_tmp[w][d];
      s_acc[g][d] = a;
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
    const int g = idx / hd, d = idx % hd;
    const int h = kvh * G + g;
    if (n_split == 1) {
      out[int64_t(t) * p.n_heads * hd + h * hd + d] = lt[g] > 0.f ? s_acc[g][d] / lt[g] : 0.f;
    } else {
      float *pp = part + ((int64_t(t) * p.n_heads + h) * n_split + split) * (hd + 2);
      pp[2 + d] = s_acc[g][d];
      if (d == 0) {
        pp[0] = mw[g];
        pp[1] = lt[g];
      }
    }
  }
}

__global__ void attn_combine_kernel(const float *__restrict__ part, float *__restrict__ out, int n_heads, int hd,
                                    int n_split) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, h = blockIdx.y;
  const float *pp = part + (int64_t(t) * n_heads + h) * n_split * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, pp[s * (hd + 2)]);
  float L = 0.f;
  for (int s = 0; s < n_split; ++s) {
    const float ms = pp[s * (hd + 2)];
    if (ms != -INFINITY) L += pp[s * (hd + 2) + 1] * expf(ms - M);
  }
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < n_split; ++s) {
      const float ms = pp[s * (hd + 2)];
      if (ms != -INFINITY) a += pp[s * (hd + 2) + 2 + d] * expf(ms - M);
    }
    out[int64_t(t) * n_heads * hd + h * hd + d] = L > 0.f ? a / L : 0.f;
  }
}

cudaError_t attn_combine(const float *part, float *out, int64_t n_tok, int n_heads, int hd, int n_split,
                         cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  return launch_pdl(attn_combine_kernel, dim3(unsigned(n_tok), unsigned(n_heads)), dim3(256), 0, st, part, out, n_heads,
                    hd, n_split);
}

static int attn_splits(int64_t n_tok, const AttnParams &p, int64_t max_keys) {
  const int64_t ctas = n_tok * p.n_kv;
  int64_t want = (2 * num_sms() + ctas - 1) / ctas;
  int64_t cap = (max_keys + 31) / 32;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  if (want > 128) want = 128;
  return int(want);
}

size_t attention_scratch_bytes(int64_t n_tok, const AttnParams &p, int64_t max_keys) {
  const int ns = attn_splits(n_tok, p, max_keys);
  if (ns == 1) return 0;
  return size_t(n_tok) * p.n_heads * ns * (p.head_dim + 2) * sizeof(float);
}

template <int EPL>
static cudaError_t launch_attn(bool kv32, dim3 grid, cudaStream_t st, const float *q, float *out, KVLayer kv,
                               const SeqInfo *seqs, const int32_t *tok_seq, const int32_t *tok_limit,
                               const uint64_t *tok_mask, const AttnParams &p, int ns, float *part) {
  if (kv32)
    return launch_pdl(attention_kernel<EPL, true>, grid, dim3(ATT_WARPS * 32), 0, st, q, out, kv, seqs, tok_seq,
                      tok_limit, tok_mask, p, ns, part);
  return launch_pdl(attention_kernel<EPL, false>, grid, dim3(ATT_WARPS * 32), 0, st, q, out, kv, seqs, tok_seq,
                    tok_limit, tok_mask, p, ns, part);
}

cudaError_t attention(const float *q, float *out, KVLayer kv, const SeqInfo *seqs, const int32_t *tok_seq,
                      const int32_t *tok_limit, const uint64_t *tok_mask, int64_t n_tok, int64_t max_keys,
                      const AttnParams &p, void *scratch, size_t scratch_bytes, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (p.n_kv <= 0 || p.n_heads % p.n_kv || p.n_heads / p.n_kv > ATT_MAXG || p.head_dim > 256)
    return cudaErrorInvalidValue;
  const int ns = attn_splits(n_tok, p, max_keys);
  if (ns > 1 && scratch_bytes < attention_scratch_bytes(n_tok, p, max_keys)) return cudaErrorInvalidValue;
  float *part = static_cast<float *>(scratch);
  dim3 grid(unsigned(n_tok), unsigned(p.n_kv), unsigned(ns));
  const bool kv32 = p.kv_f32 != 0;
  cudaError_t e;
  if (p.head_dim <= 32)
    e = launch_attn<1>(kv32, grid, st, q, out, kv, seqs, tok_seq, tok_limit, tok_mask, p, ns, part);
  else if (p.head_dim <= 64)
    e = launch_attn<2>(kv32, grid, st, q, out, kv, seqs, tok_seq, tok_limit, tok_mask, p, ns, part);
  else if (p.head_dim <= 128)
    e = launch_attn<4>(kv32, grid, st, q, out, kv, seqs, tok_seq, tok_limit, tok_mask, p, ns, part);
  else
    e = launch_attn<8>(kv32, grid, st, q, out, kv, seqs, tok_seq, tok_limit, tok_mask, p, ns, part);
  if (e != cudaSuccess || ns == 1) return e;
  return launch_pdl(attn_combine_kernel, dim3(unsigned(n_tok), unsigned(p.n_heads)), dim3(256), 0, st, part, out,
                    p.n_heads, p.head_dim, ns);
}

// ---------------------------------------------------------------- per-layer embeddings (PLE)
// compute_ple_inputs (real_forward.rs:1157-1299) for the rows of one batch and every model layer.
// In: ple [T][L*P] = per_layer_model_proj x (scaled token embedding).  Per (row t, layer l) chunk of
// P values: v = ple * proj_scale; v = (v * 1/sqrt(mean(v^2) + eps)) * norm   (rms_norm_chunked_inplace,
// eps 1e-6); v = (v + tok_row * embed_scale) * combine_scale, tok_row = the token's row of
// per_layer_token_embd (F16 / BF16 / F32), proj_scale = hidden^-1/2, embed_scale = sqrt(P),
// combine_scale = 2^-1/2.  grid (T, L).
__global__ void __launch_bounds__(256) ple_combine_kernel(float *__restrict__ ple, const void *__restrict__ tok,
                                                         int tok_type, const void *__restrict__ ids, int ids64, int LP,
                                                         int P, const float *__restrict__ norm, float proj_scale,
                                                         float embed_scale, float combine_scale, float eps) {
  __shared__ float sh[8];
  pdl_wait();
  pdl_launch_dependents();
  float *v = ple + int64_t(blockIdx.x) * LP + int64_t(blockIdx.y) * P;
  const int64_t id = ids64 ? static_cast<const int64_t *>(ids)[blockIdx.x]
                           : int64_t(static_cast<const uint32_t *>(ids)[blockIdx.x]);
  const int64_t row = id * LP + int64_t(blockIdx.y) * P;
  float ss = 0.f;
  for (int i = threadIdx.x; i < P; i += 256) {
    const float x = v[i] * proj_scale;
    ss += x * x;
  }
  ss = block_sum<256>(ss, sh);
  const float scale = 1.0f / sqrtf(ss / float(P) + eps);
  for (int i = threadIdx.x; i < P; i += 256) {
    float r;
    if (tok_type == T_F16)
      r = __half2float(static_cast<const __half *>(tok)[row + i]);
    else if (tok_type == T_BF16)
      r = __uint_as_float(uint32_t(static_cast<const uint16_t *>(tok)[row + i]) << 16);
    else
      r = static_cast<const float *>(tok)[row + i];
    const float x = ((v[i] * proj_scale) * scale) * norm[i];
    v[i] = (x + r * embed_scale) * combine_scale;
  }
}

cudaError_t ple_combine(float *ple, int tok_type, const void *tok, const void *ids, int ids64, int64_t n_tok,
                        int layers, int P, const float *norm, float proj_scale, float embed_scale, float combine_scale,
                        cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (tok_type != T_F16 && tok_type != T_BF16 && tok_type != T_F32) return cudaErrorInvalidValue;
  return launch_pdl(ple_combine_kernel, dim3(unsigned(n_tok), unsigned(layers)), dim3(256), 0, st, ple, tok, tok_type,
                    ids, ids64, layers * P, P, norm, proj_scale, embed_scale, combine_scale, 1e-6f);
}

// gated[t][j] = gelu_tanh(g[t][j]) * ple[t][l*P + j]  (real_forward.rs:1753-1778, real_math.rs:79-85)
__global__ void ple_gelu_kernel(float *__restrict__ g, const float *__restrict__ ple, int64_t n, int P, int LP,
                                int l) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / P;
    const int j = int(i - t * P);
    const float v = g[i], u = ple[t * LP + int64_t(l) * P + j];
    const float k = 0.7978845608028654f;
    const float inner = k * (v + 0.044715f * v * v * v);
    g[i] = 0.5f * v * (1.0f + tanhf(inner)) * u;
  }
}

cudaError_t ple_gelu(float *g, const float *ple, int64_t n_tok, int P, int layers, int layer, cudaStream_t st) {
  const int64_t n = n_tok * P;
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
  return launch_pdl(ple_gelu_kernel, dim3(unsigned(blocks)), dim3(256), 0, st, g, ple, n, P, layers * P, layer);
}

// ---------------------------------------------------------------- bounded-wait self-test
// One thread waits, through the same bounded mbarrier wait the streaming kernels use, on a barrier
// that either completes (complete = 1: the thread arrives first) or that nothing ever arrives on
// (complete = 0).  No copy is in flight at any time, so giving up leaves nothing behind: the wait
// runs out after `limit` polls, records DEV_WAIT_TIMEOUT in *err and the kernel returns.
__global__ void wait_selftest_kernel(unsigned limit, int complete, unsigned *err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  if (complete) asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
  mbar_wait_bounded(&bar, 0, err, limit);
}

cudaError_t wait_selftest(unsigned limit, int complete, cudaStream_t st) {
  unsigned *err = device_error_ptr();
  if (!err) return cudaErrorInvalidValue;
  wait_selftest_kernel<<<1, 32, 0, st>>>(limit, complete, err);
  return cudaGetLastError();
}

}  // namespace sfc
