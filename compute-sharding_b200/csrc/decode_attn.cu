// decode_attn.cu — decode-step attention: q/k/v head norms, RoPE, KV append and GQA attention
// over the cache in one kernel, for batches where every sequence contributes one new token.
//
// Replaces, for the decode step, the reference's per-head q/k norms and RoPE
// (crates/stage-forward-lab/src/real_forward.rs:1590-1640), the KV append (:1650-1672) and the
// causal GQA attention over the session cache (real_math.rs:2697-2744).  Multi-token batches
// (prefill, verify) keep the separate qkv_post + attention kernels in ops.cu.
//
// Design (B200):
//  * grid (sequence, kv head, key split).  Each CTA streams its split's cached K and V rows —
//    contiguous runs in the head-major cache — into a shared-memory ring with bulk async copies
//    (the TMA engine).  Those rows do not depend on the previous kernel, so the first tiles are
//    requested before the programmatic-dependent-launch wait and overlap the q/k/v projection.
//  * After the wait every CTA normalises and rotates its own G query heads (cheap, 2 x 256
//    values); the CTA whose split holds the new position also normalises/rotates the new k and
//    v, appends them to the cache and uses its own copy of them as the last key.
//  * Warp w takes keys 4w..4w+3 of every 32-key tile: lane l holds dims 8l..8l+7, scores are
//    warp sums, and one online-softmax update per 4 keys.  Warps merge in a fixed order.
//  * Splits write (max, sum, acc) partials; the last CTA of a (sequence, kv head) to finish
//    (atomic counter) merges them in split order — deterministic, and no combine launch.  The merge
//    stages every split's (max, sum) in shared memory at once and folds the partial vectors with
//    the split loop unrolled, so its L2 reads overlap instead of queueing one latency per split.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

constexpr int DA_WARPS = 8;
constexpr int DA_THREADS = DA_WARPS * 32;
constexpr int DA_MAXG = 4;  // query heads per kv head handled here (registers hold q and acc per head)
constexpr int DA_MAX_HD = 256;
constexpr int DA_MIN_CHUNK = 64;  // keys per split at least
constexpr int DA_MAX_SPLIT = 32;  // key splits per (sequence, kv head) at most
constexpr int DA_STAGES = 3;
constexpr int DA_TILE_BYTES = 32 * DA_MAX_HD * 2;  // K or V of one tile: 32 fp16 keys (16 f32 keys)

template <int N>
struct KeyCount {
  static constexpr int value = N;
};

// a[g] for a runtime g < G without dynamic register indexing
template <int G>
__device__ __forceinline__ float lt_of(const float (&a)[G], int g) {
  float r = a[0];
#pragma unroll
  for (int i = 1; i < G; ++i)
    if (g == i) r = a[i];
  return r;
}

__device__ __forceinline__ void load_row8(const uint8_t *p, bool kv32, float (&v)[8]) {
  if (kv32) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 16);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __half2float(__ushort_as_half(uint16_t(w[i] & 0xFFFFu)));
      v[2 * i + 1] = __half2float(__ushort_as_half(uint16_t(w[i] >> 16)));
    }
  }
}

template <int G, bool KV32>
__global__ void __launch_bounds__(DA_THREADS) decode_attention_kernel(
    const float *__restrict__ qr, const float *__restrict__ kr, const float *__restrict__ vr, int q_ld, int kv_ld,
    float *__restrict__ out, KVLayer kv, const SeqInfo *__restrict__ seqs, AttnParams p, int n_split, int min_chunk,
    float *__restrict__ part, unsigned *__restrict__ counters, unsigned *err) {
  constexpr int ESZ = KV32 ? 4 : 2;
  constexpr int TK = DA_TILE_BYTES / (DA_MAX_HD * ESZ);  // keys per tile
  constexpr int KPW = TK / DA_WARPS;                      // keys per warp per tile
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bars[DA_STAGES];
  __shared__ float s_vec[DA_MAXG + 2][DA_MAX_HD];  // q heads, then the new k and v
  __shared__ float s_red[DA_MAXG + 2][DA_WARPS];
  __shared__ float s_m[DA_WARPS][DA_MAXG], s_l[DA_WARPS][DA_MAXG];
  __shared__ unsigned s_last;
  __shared__ float s_f[DA_MAXG][DA_MAX_SPLIT];  // merge weights exp(m_s - M) / L per head and split

  const int t = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = p.head_dim;
  const SeqInfo sq = seqs[t];
  const int pos = sq.pos0;  // position of the new token
  const int limit = pos + 1;
  const int w0 = p.window > 0 ? max(0, limit - p.window) : 0;
  const int span = limit - w0;
  int chunk = (span + n_split - 1) / n_split;
  if (chunk < min_chunk) chunk = min_chunk;  // min_chunk >= DA_MIN_CHUNK
  const int n_eff = (span + chunk - 1) / chunk;
  if (split >= n_eff) return;  // this sequence needs fewer splits (uniform over the CTA)
  const int k_begin = w0 + split * chunk, k_end = min(limit, k_begin + chunk);
  // keys already in the cache: all of them when another layer's cache is read (kv_shared: that
  // layer appended this step's key earlier in the forward)
  const int k_old_end = p.kv_shared ? k_end : min(k_end, pos);
  const bool owner = k_end == limit && !p.kv_shared;  // this split computes and appends the new key
  const int n_old = max(0, k_old_end - k_begin);
  const int n_tiles = (n_old + TK - 1) / TK;

  const size_t row_bytes = size_t(hd) * ESZ;
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(kv.base) + size_t(sq.slot) * kv.slot_stride * ESZ;
  const uint8_t *vbase = kbase + size_t(kv.slot_stride / 2) * ESZ;
  const size_t head_off = size_t(kvh) * p.max_ctx * row_bytes;
  uint8_t *tiles = smem;  // [DA_STAGES][K tile | V tile]

  auto issue = [&](int i) {
    const int st = i % DA_STAGES;
    const int k0 = k_begin + i * TK;
    const int nk = min(TK, k_old_end - k0);
    const uint32_t bytes = uint32_t(nk * row_bytes);
    mbar_arrive_expect_tx(&bars[st], 2 * bytes);
    bulk_g2s(tiles + st * 2 * DA_TILE_BYTES, kbase + head_off + size_t(k0) * row_bytes, bytes, &bars[st]);
    bulk_g2s(tiles + st * 2 * DA_TILE_BYTES + DA_TILE_BYTES, vbase + head_off + size_t(k0) * row_bytes, bytes,
             &bars[st]);
  };
  if (tid == 0) {
    for (int i = 0; i < DA_STAGES; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    // cached rows never depend on the previous kernel: request them before the dependency wait
    for (int i = 0; i < n_tiles && i < DA_STAGES; ++i) issue(i);
  }
  pdl_wait();
  pdl_launch_dependents();

  // ---- q heads (and, for the owner, the new k and v): per-head RMS norm, RoPE (as qkv_post_kernel)
  const int nvec = G + (owner ? 2 : 0);
  float ss[DA_MAXG + 2];
#pragma unroll
  for (int r = 0; r < DA_MAXG + 2; ++r) {
    ss[r] = 0.f;
    if (r < nvec && tid < hd) {
      const float *src = r < G ? qr + int64_t(t) * q_ld + (kvh * G + r) * hd
                               : (r == G ? kr : vr) + int64_t(t) * kv_ld + kvh * hd;
      const float x = src[tid];
      s_vec[r][tid] = x;
      ss[r] = x * x;
    }
  }
#pragma unroll
  for (int r = 0; r < DA_MAXG + 2; ++r) {
    if (r < nvec) {
      const float w = warp_sum(ss[r]);
      if (lane == 0) s_red[r][warp] = w;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < DA_MAXG + 2; ++r) {
    if (r < nvec && tid < hd) {
      float sum = 0.f;
      for (int w = 0; w < DA_WARPS; ++w) sum += s_red[r][w];
      const float scale = 1.0f / sqrtf(sum / float(hd) + p.eps);
      const float *nw = r < G ? p.q_norm : (r == G ? p.k_norm : nullptr);
      if (r == G + 1 || nw) s_vec[r][tid] = s_vec[r][tid] * (nw ? scale * nw[tid] : scale);
    }
  }
  __syncthreads();
  if (p.rope_freqs) {
    const int hde = hd & ~1;
    const int rd = min(p.rotary_dim, hde) & ~1;
    const int n_ang = rd / 2, half = hde / 2;
    const float denom = p.proportional ? float(hde) : float(rd);
    const int nrot = G + (owner ? 1 : 0);  // q heads and k
    for (int idx = tid; idx < nrot * n_ang; idx += DA_THREADS) {
      const int r = idx / n_ang, i = idx % n_ang;
      const float inv_freq = 1.0f / powf(p.rope_theta, 2.0f * float(i) / denom);
      const float fs = i < p.n_freqs ? p.rope_freqs[i] : 1.0f;
      const float th = float(pos) * inv_freq * fs;
      float sn, cs;
      sincosf(th, &sn, &cs);
      const float x0 = s_vec[r][i], x1 = s_vec[r][half + i];
      s_vec[r][i] = x0 * cs - x1 * sn;
      s_vec[r][half + i] = x0 * sn + x1 * cs;
    }
    __syncthreads();
  }
  if (owner && pos < p.max_ctx && tid < hd) {  // append the new key and value
    const size_t off = head_off + size_t(pos) * row_bytes + size_t(tid) * ESZ;
    if (KV32) {
      *reinterpret_cast<float *>(const_cast<uint8_t *>(kbase) + off) = s_vec[G][tid];
      *reinterpret_cast<float *>(const_cast<uint8_t *>(vbase) + off) = s_vec[G + 1][tid];
    } else {
      // the new key is attended as cached: rounded to fp16 like every other key
      const __half hk = __float2half_rn(s_vec[G][tid]), hv = __float2half_rn(s_vec[G + 1][tid]);
      *reinterpret_cast<__half *>(const_cast<uint8_t *>(kbase) + off) = hk;
      *reinterpret_cast<__half *>(const_cast<uint8_t *>(vbase) + off) = hv;
      s_vec[G][tid] = __half2float(hk);
      s_vec[G + 1][tid] = __half2float(hv);
    }
  }
  __syncthreads();

  // ---- keys: lane l holds dims 8l..8l+7
  const bool lane_on = lane * 8 < hd;
  float qv[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[g][e] = lane_on ? s_vec[g][lane * 8 + e] : 0.f;
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }
  // one online-softmax update with KN keys (rows kf/vf; key k counts when bit k of `valid` is set)
  auto update = [&](auto kn_tag, const float (*kf)[8], const float (*vf)[8], unsigned valid) {
    constexpr int KN = decltype(kn_tag)::value;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s[KN];
      float mx = m[g];
#pragma unroll
      for (int k = 0; k < KN; ++k) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d += qv[g][e] * kf[k][e];
        d = warp_sum(d);
        s[k] = (valid >> k) & 1u ? d : -INFINITY;
        mx = fmaxf(mx, s[k]);
      }
      if (mx == -INFINITY) continue;  // no valid key yet
      const float alpha = expf(m[g] - mx);  // exp(-inf) = 0 on the first keys
      float psum = 0.f;
      float pk[KN];
#pragma unroll
      for (int k = 0; k < KN; ++k) {
        pk[k] = (valid >> k) & 1u ? expf(s[k] - mx) : 0.f;
        psum += pk[k];
      }
      l[g] = l[g] * alpha + psum;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float a = acc[g][e] * alpha;
#pragma unroll
        for (int k = 0; k < KN; ++k) a += pk[k] * vf[k][e];
        acc[g][e] = a;
      }
      m[g] = mx;
    }
  };

  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % DA_STAGES;
    mbar_wait_bounded(&bars[st], (i / DA_STAGES) & 1, err);
    const int k0 = k_begin + i * TK;
    const int nk = min(TK, k_old_end - k0);
    const uint8_t *kt = tiles + st * 2 * DA_TILE_BYTES, *vt = kt + DA_TILE_BYTES;
    float kf[KPW][8], vf[KPW][8];
    unsigned valid = 0;
#pragma unroll
    for (int k = 0; k < KPW; ++k) {
      const int kk = warp * KPW + k;
      if (kk < nk) valid |= 1u << k;
      if (kk < nk && lane_on) {
        load_row8(kt + kk * row_bytes + lane * 8 * ESZ, KV32, kf[k]);
        load_row8(vt + kk * row_bytes + lane * 8 * ESZ, KV32, vf[k]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) kf[k][e] = vf[k][e] = 0.f;
      }
    }
    update(KeyCount<KPW>{}, kf, vf, valid);
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && i + DA_STAGES < n_tiles) issue(i + DA_STAGES);
  }
  if (owner && warp == 0) {  // the new key, from this CTA's own copy
    float kf[1][8], vf[1][8];
    const unsigned valid = 1u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      kf[0][e] = lane_on ? s_vec[G][lane * 8 + e] : 0.f;
      vf[0][e] = lane_on ? s_vec[G + 1][lane * 8 + e] : 0.f;
    }
    update(KeyCount<1>{}, kf, vf, valid);
  }

  // ---- merge the warps in a fixed order (tiles are free: every issued copy has been waited on)
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
  __syncthreads();
  float *s_tmp = reinterpret_cast<float *>(tiles);  // [DA_WARPS][DA_MAX_HD]
  float *s_acc = s_tmp + DA_WARPS * DA_MAX_HD;      // [DA_MAXG][DA_MAX_HD]
  float M[G], L[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mm = -INFINITY;
    for (int w = 0; w < DA_WARPS; ++w) mm = fmaxf(mm, s_m[w][g]);
    float ll = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) ll += s_m[w][g] == -INFINITY ? 0.f : s_l[w][g] * expf(s_m[w][g] - mm);
    M[g] = mm;
    L[g] = ll;
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float scw = m[g] == -INFINITY ? 0.f : expf(m[g] - M[g]);
    if (lane_on)
#pragma unroll
      for (int e = 0; e < 8; ++e) s_tmp[warp * DA_MAX_HD + lane * 8 + e] = acc[g][e] * scw;
    __syncthreads();
    if (tid < hd) {
      float a = 0.f;
      for (int w = 0; w < DA_WARPS; ++w) a += s_tmp[w * DA_MAX_HD + tid];
      s_acc[g * DA_MAX_HD + tid] = a;
    }
    __syncthreads();
  }
  if (n_eff == 1) {
    for (int idx = tid; idx < G * hd; idx += DA_THREADS) {
      const int g = idx / hd, d = idx % hd;
      out[int64_t(t) * p.n_heads * hd + (kvh * G + g) * hd + d] = s_acc[g * DA_MAX_HD + d] / lt_of(L, g);
    }
    return;
  }
  for (int idx = tid; idx < G * hd; idx += DA_THREADS) {
    const int g = idx / hd, d = idx % hd;
    float *pp = part + ((int64_t(t) * p.n_heads + kvh * G + g) * n_split + split) * (hd + 2);
    pp[2 + d] = s_acc[g * DA_MAX_HD + d];
    if (d == 0) {
      pp[0] = lt_of(M, g);
      pp[1] = lt_of(L, g);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&counters[t * p.n_kv + kvh], 1u);
    s_last = prev == unsigned(n_eff - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last split of this (sequence, kv head): merge all partials in split order
  const float *pbase = part + (int64_t(t) * p.n_heads + kvh * G) * n_split * (hd + 2);
  if (tid < G * n_eff) {  // (max, sum) of every split, loaded in parallel
    const int g = tid / n_eff, sp = tid % n_eff;
    s_f[g][sp] = __ldcg(pbase + (g * n_split + sp) * (hd + 2));
    s_vec[g][sp] = __ldcg(pbase + (g * n_split + sp) * (hd + 2) + 1);
  }
  __syncthreads();
  if (tid < G) {
    float mm = -INFINITY;
    for (int sp = 0; sp < n_eff; ++sp) mm = fmaxf(mm, s_f[tid][sp]);
    float ll = 0.f;
    for (int sp = 0; sp < n_eff; ++sp) {
      const float ms = s_f[tid][sp];
      const float f = ms == -INFINITY ? 0.f : expf(ms - mm);
      s_f[tid][sp] = f;
      ll += s_vec[tid][sp] * f;
    }
    const float inv = ll > 0.f ? 1.0f / ll : 0.f;
    for (int sp = 0; sp < n_eff; ++sp) s_f[tid][sp] *= inv;
  }
  __syncthreads();
  for (int idx = tid; idx < G * hd; idx += DA_THREADS) {
    const int g = idx / hd, d = idx % hd;
    const float *pp = pbase + g * n_split * (hd + 2) + 2 + d;
    float a = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < n_eff; ++sp) a += s_f[g][sp] * __ldcg(pp + sp * (hd + 2));
    out[int64_t(t) * p.n_heads * hd + (kvh * G + g) * hd + d] = a;
  }
  if (tid == 0) counters[t * p.n_kv + kvh] = 0u;  // ready for the next launch
}

int decode_attention_splits(int64_t n_seq, const AttnParams &p, int64_t max_keys) {
  const int64_t ctas = n_seq * p.n_kv;
  int64_t want = (4 * num_sms() + ctas - 1) / ctas;
  const int64_t by_len = (max_keys + 511) / 512;
  if (want < by_len) want = by_len;
  const int64_t cap = (max_keys + DA_MIN_CHUNK - 1) / DA_MIN_CHUNK;
  if (want > cap) want = cap;
  if (want > DA_MAX_SPLIT) want = DA_MAX_SPLIT;
  if (want < 1) want = 1;
  return int(want);
}

// Keys per split at least, for a batch of sum_keys keys in total: every CTA pays a fixed cost
// (head norms, RoPE, the warp merge, the partials and the last-CTA merge) that a split of a few
// tiles does not amortise, so large batches spread their keys over about DA_CTAS_PER_SM CTAs per
// SM instead of giving every sequence the split count of the longest one.  A sequence then takes
// max(ceil(span / n_split), min_chunk) keys per split; n_split bounds the grid and the partials.
constexpr int DA_CTAS_PER_SM = 4;  // measured at 64 sequences: 2 and 8 were slower
static void decode_attention_plan(int64_t n_seq, const AttnParams &p, int64_t max_keys, int64_t sum_keys, int *ns,
                                  int *min_chunk) {
  *ns = decode_attention_splits(n_seq, p, max_keys);
  *min_chunk = DA_MIN_CHUNK;
  if (sum_keys <= 0) return;
  const int64_t target = int64_t(DA_CTAS_PER_SM) * num_sms();
  const int64_t c = (sum_keys * p.n_kv + target - 1) / target;
  if (c <= DA_MIN_CHUNK) return;
  *min_chunk = int(c < (int64_t(1) << 30) ? c : (int64_t(1) << 30));
  const int64_t need = (max_keys + *min_chunk - 1) / *min_chunk;
  if (need < *ns) *ns = int(need < 1 ? 1 : need);
}

size_t decode_attention_scratch_bytes(int64_t n_seq, const AttnParams &p, int64_t max_keys) {
  const int ns = decode_attention_splits(n_seq, p, max_keys);
  return size_t(n_seq) * p.n_heads * ns * (p.head_dim + 2) * sizeof(float);
}

bool decode_attention_supported(const AttnParams &p) {
  if (p.n_kv <= 0 || p.n_heads % p.n_kv) return false;
  const int G = p.n_heads / p.n_kv;
  return (G == 1 || G == 2 || G == 4) && p.head_dim <= DA_MAX_HD && p.head_dim % 8 == 0;
}

cudaError_t decode_attention(const float *q, const float *k, const float *v, int q_ld, int kv_ld, float *out,
                             KVLayer kv, const SeqInfo *seqs, int64_t n_seq, int64_t max_keys, int64_t sum_keys,
                             const AttnParams &p, void *scratch, size_t scratch_bytes, unsigned *counters,
                             cudaStream_t st) {
  if (n_seq <= 0) return cudaSuccess;
  if (!decode_attention_supported(p) || !counters) return cudaErrorInvalidValue;
  int ns = 1, min_chunk = DA_MIN_CHUNK;
  decode_attention_plan(n_seq, p, max_keys, sum_keys, &ns, &min_chunk);
  if (scratch_bytes < decode_attention_scratch_bytes(n_seq, p, max_keys)) return cudaErrorInvalidValue;
  const size_t smem = size_t(DA_STAGES) * 2 * DA_TILE_BYTES;
  const dim3 grid(unsigned(n_seq), unsigned(p.n_kv), unsigned(ns));
  const int G = p.n_heads / p.n_kv;
  void (*kern)(const float *, const float *, const float *, int, int, float *, KVLayer, const SeqInfo *, AttnParams,
               int, int, float *, unsigned *, unsigned *) = nullptr;
  switch (G) {
    case 1: kern = p.kv_f32 ? decode_attention_kernel<1, true> : decode_attention_kernel<1, false>; break;
    case 2: kern = p.kv_f32 ? decode_attention_kernel<2, true> : decode_attention_kernel<2, false>; break;
    case 4: kern = p.kv_f32 ? decode_attention_kernel<4, true> : decode_attention_kernel<4, false>; break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, grid, dim3(DA_THREADS), smem, st, q, k, v, q_ld, kv_ld, out, kv, seqs, p, ns, min_chunk,
                    static_cast<float *>(scratch), counters, device_error_ptr());
}

}  // namespace sfc
