// decode_layer.cu — one decoder layer of a one-token decode step as a single persistent kernel.
//
// Replaces, for batch-1 decode, the per-op launches of one forward_layer_seq step
// (crates/stage-forward-lab/src/real_forward.rs:1483-1793): attn_norm -> q/k/v projections ->
// q/k norms, RoPE, KV append, GQA attention (real_math.rs:2697-2744) -> o projection ->
// post-attention norm + residual -> ffn norm -> gate/up + GeGLU -> down.
//
// Design (B200): one CTA per SM, launched cooperatively so that all CTAs are resident and can meet
// at grid barriers between the phases.
//  * The producer warp streams the weights of all four projections (q/k/v, o, gate/up, down) into
//    the shared-memory stage ring back to back: weights never depend on activations, so while
//    the consumers wait at a barrier or run the attention phase the next projection's weights are
//    already landing.  Each projection is split over the CTAs exactly as the GEMV kernel splits
//    it (gemv_core.cuh), with the same exact-integer tensor-pipe units.
//  * Phases: q/k/v (residual + RMSNorm in the activation prologue) | attention: one (kv head, key
//    split) item per CTA, cached rows read with plain 16-byte loads after an L2 prefetch issued at
//    the start of the layer | split merge (only when a head has more than one split) | o | gate/up
//    (residual + norms in the prologue) | down.  A grid barrier separates the phases.
//  * Grid barrier: one monotonically increasing arrival counter in global memory.  A launch reads
//    its base value before its first arrival (no barrier can complete earlier); barrier i is passed
//    once the counter reaches base + i * ctas (bounded poll).
#include <cuda_fp16.h>
#include <math.h>
#include <stdio.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "gemv_core.cuh"

namespace sfc {

constexpr int DL_CW = 15;                  // consumer warps (plus one producer warp)
constexpr int DL_THREADS = (DL_CW + 1) * 32;
constexpr int DL_PHASES = 4;               // q/k/v, o, gate/up, down
constexpr int DL_MIN_CHUNK = 64;           // keys per attention split at least
constexpr int DL_MAX_SPLIT = 32;
constexpr int DL_MAXG = 4;
constexpr int DL_MAX_HD = 256;
constexpr int DL_KEYS = 4;                 // keys per warp per batch of loads
constexpr unsigned DL_BAR_SPIN = 1u << 20; // polls (with a short sleep each) before a barrier gives up

struct DecodeLayerArgs {
  QGemvArgs ph[DL_PHASES];  // per projection: segments, partition, prologue (smem offsets shared)
  int nstage, stage_bytes;  // shared stage ring
  // attention
  const float *q, *k, *v;
  int q_ld, kv_ld;
  float *att;
  KVLayer kv;
  const SeqInfo *seqs;
  AttnParams ap;
  int n_split;
  float *apart;    // split partials [n_heads][n_split][head_dim + 2]
  unsigned *bar;   // grid barrier: [0] arrival counter (wraps)
  unsigned *err;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// All consumer threads of every CTA: returns once every CTA has arrived `target - base` times in
// total (thread 0 polls; unsigned differences survive the counter's wrap).
__device__ __forceinline__ void grid_sync(unsigned *bar, unsigned base, unsigned target, unsigned *err, int tid) {
  consumer_bar<DL_CW>();
  if (tid == 0) {
    __threadfence();  // this CTA's global writes before the arrival
    atomicAdd(bar, 1u);
    unsigned spins = 0;
    while (ld_acquire_gpu(bar) - base < target) {
      if (++spins > DL_BAR_SPIN) {
        if (err) atomicExch(err, DEV_WAIT_TIMEOUT);
        break;
      }
      if (spins > 256) __nanosleep(32);
    }
    __threadfence();
  }
  consumer_bar<DL_CW>();
}

// ---------------------------------------------------------------- attention phase
// The key range of split `split` of the sequence's span (as decode_attention_kernel).
struct AttnSplit {
  int pos, k_begin, k_end, k_old_end, n_eff;
  bool owner;
  __device__ __forceinline__ AttnSplit(const SeqInfo &sq, const AttnParams &p, int n_split, int split) {
    pos = sq.pos0;
    const int limit = pos + 1;
    const int w0 = p.window > 0 ? max(0, limit - p.window) : 0;
    const int span = limit - w0;
    int chunk = (span + n_split - 1) / n_split;
    if (chunk < DL_MIN_CHUNK) chunk = DL_MIN_CHUNK;
    n_eff = (span + chunk - 1) / chunk;
    k_begin = w0 + split * chunk;
    k_end = min(limit, k_begin + chunk);
    k_old_end = min(k_end, pos);
    owner = k_end == limit;
  }
};

// 8 cached elements of a key or value row as raw words (fp16: one 16-byte word, f32: two)
template <bool KV32>
struct KvRaw {
  uint4 w[KV32 ? 2 : 1];
};
template <bool KV32>
__device__ __forceinline__ void load_kv_raw(const uint8_t *p, KvRaw<KV32> &r) {
  r.w[0] = __ldcg(reinterpret_cast<const uint4 *>(p));
  if (KV32) r.w[KV32 ? 1 : 0] = __ldcg(reinterpret_cast<const uint4 *>(p) + 1);
}
template <bool KV32>
__device__ __forceinline__ void kv_floats(const KvRaw<KV32> &r, float (&v)[8]) {
  if (KV32) {
    const uint32_t w[8] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[KV32 ? 1 : 0].x, r.w[KV32 ? 1 : 0].y,
                           r.w[KV32 ? 1 : 0].z, r.w[KV32 ? 1 : 0].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(w[i]);
  } else {
    const uint32_t w[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __half2float(__ushort_as_half(uint16_t(w[i] & 0xFFFFu)));
      v[2 * i + 1] = __half2float(__ushort_as_half(uint16_t(w[i] >> 16)));
    }
  }
}

// One (kv head, split) item: q/k/v head norms, RoPE, KV append (owner), online softmax over the
// split's keys, then the exact output (single split) or the split's (max, sum, acc) partials.
// scr: shared scratch of (G + 2) * 256 + 2 * CW * G + CW * G * 256 floats.
template <int G, bool KV32>
__device__ __forceinline__ void attn_item(const DecodeLayerArgs &d, int kvh, const AttnSplit &sp, int split,
                                          float *scr, int tid, int warp, int lane) {
  constexpr int ESZ = KV32 ? 4 : 2;
  const AttnParams &p = d.ap;
  const int hd = p.head_dim;
  const SeqInfo sq = d.seqs[0];
  float *s_vec = scr;                                 // [G + 2][256]
  float *s_m = s_vec + (DL_MAXG + 2) * DL_MAX_HD;     // [CW][G]
  float *s_l = s_m + DL_CW * DL_MAXG;                 // [CW][G]
  float *s_tmp = s_l + DL_CW * DL_MAXG;               // [CW][G][256]
  __shared__ float s_red[DL_MAXG + 2][DL_CW];
  const size_t row_bytes = size_t(hd) * ESZ;
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(d.kv.base) + size_t(sq.slot) * d.kv.slot_stride * ESZ;
  const uint8_t *vbase = kbase + size_t(d.kv.slot_stride / 2) * ESZ;
  const size_t head_off = size_t(kvh) * p.max_ctx * row_bytes;

  // ---- q heads (and, for the owner, the new k and v): per-head RMS norm, RoPE (as qkv_post_kernel)
  const int nvec = G + (sp.owner ? 2 : 0);
  float ss[DL_MAXG + 2];
#pragma unroll
  for (int r = 0; r < DL_MAXG + 2; ++r) {
    ss[r] = 0.f;
    if (r < nvec && tid < hd) {
      const float *src = r < G ? d.q + (kvh * G + r) * hd : (r == G ? d.k : d.v) + kvh * hd;
      const float x = __ldcg(src + tid);  // written by other CTAs in this launch
      s_vec[r * DL_MAX_HD + tid] = x;
      ss[r] = x * x;
    }
  }
#pragma unroll
  for (int r = 0; r < DL_MAXG + 2; ++r) {
    if (r < nvec) {
      const float w = warp_sum(ss[r]);
      if (lane == 0) s_red[r][warp] = w;
    }
  }
  consumer_bar<DL_CW>();
#pragma unroll
  for (int r = 0; r < DL_MAXG + 2; ++r) {
    if (r < nvec && tid < hd) {
      float sum = 0.f;
      for (int w = 0; w < DL_CW; ++w) sum += s_red[r][w];
      const float scale = 1.0f / sqrtf(sum / float(hd) + p.eps);
      const float *nw = r < G ? p.q_norm : (r == G ? p.k_norm : nullptr);
      if (r == G + 1 || nw) s_vec[r * DL_MAX_HD + tid] = s_vec[r * DL_MAX_HD + tid] * (nw ? scale * nw[tid] : scale);
    }
  }
  consumer_bar<DL_CW>();
  if (p.rope_freqs) {
    const int hde = hd & ~1;
    const int rd = min(p.rotary_dim, hde) & ~1;
    const int n_ang = rd / 2, half = hde / 2;
    const float denom = p.proportional ? float(hde) : float(rd);
    const int nrot = G + (sp.owner ? 1 : 0);  // q heads and k
    for (int idx = tid; idx < nrot * n_ang; idx += DL_CW * 32) {
      const int r = idx / n_ang, i = idx % n_ang;
      const float inv_freq = 1.0f / powf(p.rope_theta, 2.0f * float(i) / denom);
      const float fs = i < p.n_freqs ? p.rope_freqs[i] : 1.0f;
      const float th = float(sp.pos) * inv_freq * fs;
      float sn, cs;
      sincosf(th, &sn, &cs);
      const float x0 = s_vec[r * DL_MAX_HD + i], x1 = s_vec[r * DL_MAX_HD + half + i];
      s_vec[r * DL_MAX_HD + i] = x0 * cs - x1 * sn;
      s_vec[r * DL_MAX_HD + half + i] = x0 * sn + x1 * cs;
    }
    consumer_bar<DL_CW>();
  }
  if (sp.owner && sp.pos < p.max_ctx && tid < hd) {  // append the new key and value
    const size_t off = head_off + size_t(sp.pos) * row_bytes + size_t(tid) * ESZ;
    if (KV32) {
      *reinterpret_cast<float *>(const_cast<uint8_t *>(kbase) + off) = s_vec[G * DL_MAX_HD + tid];
      *reinterpret_cast<float *>(const_cast<uint8_t *>(vbase) + off) = s_vec[(G + 1) * DL_MAX_HD + tid];
    } else {
      // the new key is attended as cached: rounded to fp16 like every other key
      const __half hk = __float2half_rn(s_vec[G * DL_MAX_HD + tid]), hv = __float2half_rn(s_vec[(G + 1) * DL_MAX_HD + tid]);
      *reinterpret_cast<__half *>(const_cast<uint8_t *>(kbase) + off) = hk;
      *reinterpret_cast<__half *>(const_cast<uint8_t *>(vbase) + off) = hv;
      s_vec[G * DL_MAX_HD + tid] = __half2float(hk);
      s_vec[(G + 1) * DL_MAX_HD + tid] = __half2float(hv);
    }
  }
  consumer_bar<DL_CW>();

  // ---- keys: warp w takes keys k_begin + w, + CW, ...; lane l holds dims 8l..8l+7
  const bool lane_on = lane * 8 < hd;
  float qv[G][8], m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      qv[g][e] = lane_on ? s_vec[g * DL_MAX_HD + lane * 8 + e] : 0.f;
      acc[g][e] = 0.f;
    }
  }
  auto update = [&](const float (&kf)[8], const float (&vf)[8]) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s += qv[g][e] * kf[e];
      s = warp_sum(s);  // no 1/sqrt(d) scale (real_math.rs:2697-2744)
      const float mx = fmaxf(m[g], s);
      const float alpha = expf(m[g] - mx), pk = expf(s - mx);
      l[g] = l[g] * alpha + pk;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] = acc[g][e] * alpha + pk * vf[e];
      m[g] = mx;
    }
  };
  for (int k0 = sp.k_begin + warp; k0 < sp.k_old_end; k0 += DL_CW * DL_KEYS) {
    KvRaw<KV32> kr[DL_KEYS], vr[DL_KEYS];
#pragma unroll
    for (int j = 0; j < DL_KEYS; ++j) {  // issue every load of the batch first
      const int kk = k0 + j * DL_CW;
      if (kk < sp.k_old_end && lane_on) {
        load_kv_raw<KV32>(kbase + head_off + size_t(kk) * row_bytes + lane * 8 * ESZ, kr[j]);
        load_kv_raw<KV32>(vbase + head_off + size_t(kk) * row_bytes + lane * 8 * ESZ, vr[j]);
      } else {
        kr[j] = vr[j] = KvRaw<KV32>{};
      }
    }
#pragma unroll
    for (int j = 0; j < DL_KEYS; ++j)
      if (k0 + j * DL_CW < sp.k_old_end) {
        float kf[8], vf[8];
        kv_floats<KV32>(kr[j], kf);
        kv_floats<KV32>(vr[j], vf);
        update(kf, vf);
      }
  }
  if (sp.owner && warp == 0) {  // the new key, from this CTA's own copy
    float kf[8], vf[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      kf[e] = lane_on ? s_vec[G * DL_MAX_HD + lane * 8 + e] : 0.f;
      vf[e] = lane_on ? s_vec[(G + 1) * DL_MAX_HD + lane * 8 + e] : 0.f;
    }
    update(kf, vf);
  }

  // ---- merge the warps in a fixed order (all heads at once)
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[warp * DL_MAXG + g] = m[g];
      s_l[warp * DL_MAXG + g] = l[g];
    }
  consumer_bar<DL_CW>();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mm = -INFINITY;
    for (int w = 0; w < DL_CW; ++w) mm = fmaxf(mm, s_m[w * DL_MAXG + g]);
    const float scw = m[g] == -INFINITY ? 0.f : expf(m[g] - mm);
    if (lane_on)
#pragma unroll
      for (int e = 0; e < 8; ++e) s_tmp[(warp * G + g) * DL_MAX_HD + lane * 8 + e] = acc[g][e] * scw;
  }
  consumer_bar<DL_CW>();
  for (int idx = tid; idx < G * hd; idx += DL_CW * 32) {
    const int g = idx / hd, dd = idx % hd;
    float mm = -INFINITY;
    for (int w = 0; w < DL_CW; ++w) mm = fmaxf(mm, s_m[w * DL_MAXG + g]);
    float ll = 0.f;
    for (int w = 0; w < DL_CW; ++w) {
      const float mw = s_m[w * DL_MAXG + g];
      ll += mw == -INFINITY ? 0.f : s_l[w * DL_MAXG + g] * expf(mw - mm);
    }
    float a = 0.f;
    for (int w = 0; w < DL_CW; ++w) a += s_tmp[(w * G + g) * DL_MAX_HD + dd];
    const int head = kvh * G + g;
    if (sp.n_eff == 1) {
      d.att[head * hd + dd] = ll > 0.f ? a / ll : 0.f;
    } else {
      float *pp = d.apart + (size_t(head) * d.n_split + split) * (hd + 2);
      pp[2 + dd] = a;
      if (dd == 0) {
        pp[0] = mm;
        pp[1] = ll;
      }
    }
  }
}

// Split merge for one query head (n_eff > 1): as the last-CTA merge of decode_attention_kernel.
__device__ __forceinline__ void attn_merge_head(const DecodeLayerArgs &d, int head, int n_eff, float *scr, int tid) {
  const int hd = d.ap.head_dim;
  const float *pb = d.apart + size_t(head) * d.n_split * (hd + 2);
  float *s_f = scr, *s_ls = scr + DL_MAX_SPLIT;
  if (tid < n_eff) {
    s_f[tid] = __ldcg(pb + tid * (hd + 2));
    s_ls[tid] = __ldcg(pb + tid * (hd + 2) + 1);
  }
  consumer_bar<DL_CW>();
  if (tid == 0) {
    float mm = -INFINITY;
    for (int s = 0; s < n_eff; ++s) mm = fmaxf(mm, s_f[s]);
    float ll = 0.f;
    for (int s = 0; s < n_eff; ++s) {
      const float f = s_f[s] == -INFINITY ? 0.f : expf(s_f[s] - mm);
      s_f[s] = f;
      ll += s_ls[s] * f;
    }
    const float inv = ll > 0.f ? 1.0f / ll : 0.f;
    for (int s = 0; s < n_eff; ++s) s_f[s] *= inv;
  }
  consumer_bar<DL_CW>();
  for (int dd = tid; dd < hd; dd += DL_CW * 32) {
    float a = 0.f;
#pragma unroll 8
    for (int s = 0; s < n_eff; ++s) a += s_f[s] * __ldcg(pb + s * (hd + 2) + 2 + dd);
    d.att[head * hd + dd] = a;
  }
  consumer_bar<DL_CW>();
}

// ---------------------------------------------------------------- kernel
template <int NMAT>
__device__ __forceinline__ void gemv_phase(const QGemvArgs &a, int ptype, const GemvStage *tab, RingPos rp,
                                           const uint8_t *ring, uint64_t *full, uint64_t *empty, int *s_sdone,
                                           const XSmem &X, float *red, int *s_tdone, float (*pro_red)[16], int cta,
                                           int tid, int warp, int lane) {
  CtaTiles ct;
  {
    const int u0 = cta * a.uq + (cta < a.ur ? cta : a.ur);
    ct.init(u0, u0 + a.uq + (cta < a.ur ? 1 : 0), a.nb);
  }
  if (tid == 0) s_tdone[0] = s_tdone[1] = 0;  // ordered before use by build_x's closing barrier
  build_x<1, DL_CW>(a.pro, a.nb, cta, X, pro_red, warp, lane);
  if (ptype == T_Q4_K)
    run_units<NMAT, 1, T_Q4_K, DL_CW>(a, ct, tab, rp, ring, full, empty, s_sdone, X, red, s_tdone, cta, warp, lane);
  else if (ptype == T_Q6_K)
    run_units<NMAT, 1, T_Q6_K, DL_CW>(a, ct, tab, rp, ring, full, empty, s_sdone, X, red, s_tdone, cta, warp, lane);
  else
    run_units<NMAT, 1, 0, DL_CW>(a, ct, tab, rp, ring, full, empty, s_sdone, X, red, s_tdone, cta, warp, lane);
  consumer_bar<DL_CW>();
  finish_owned<NMAT, 1, DL_CW>(a, ct, red, tid);
}

__device__ __forceinline__ int phase_type(const QGemvArgs &a) {
  int t = a.seg[0].type;
  for (int i = 1; i < a.nseg; ++i)
    if (a.seg[i].type != t) t = 0;
  return t;
}

template <int G, bool KV32>
__global__ void __launch_bounds__(DL_THREADS, 1) decode_layer_kernel(const __grid_constant__ DecodeLayerArgs d) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float pro_red[GEMV_MAX_T][16];
  __shared__ int s_tdone[2];
  __shared__ int s_sdone[GEMV_MAX_STAGES];
  __shared__ int s_nst[DL_PHASES];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = int(blockIdx.x), nctas = int(gridDim.x);
  const QGemvArgs &a0 = d.ph[0];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem), *empty = full + GEMV_MAX_STAGES;
  float *red = reinterpret_cast<float *>(smem + a0.red_off);
  uint8_t *xreg = smem + a0.x_off;  // activation image of the current projection / attention scratch
  uint8_t *ring = smem + a0.ring_off;

  if (tid == 0) {
    for (int i = 0; i < d.nstage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      s_sdone[i] = 0;
    }
    fence_mbar_init();
  }
  if (lane == 0 && warp < DL_PHASES) {  // the four stage tables, one warp each
    const QGemvArgs &a = d.ph[warp];
    CtaTiles ct;
    const int u0 = cta * a.uq + (cta < a.ur ? cta : a.ur);
    ct.init(u0, u0 + a.uq + (cta < a.ur ? 1 : 0), a.nb);
    s_nst[warp] = build_stage_table(a, ct, reinterpret_cast<GemvStage *>(smem + a.tab_off));
  }
  __syncthreads();

  if (warp == DL_CW) {  // producer: the four projections' weights, back to back
    RingPos rp = {0, 0};
    int issued = 0;
    produce_stages<1>(d.ph[0], reinterpret_cast<const GemvStage *>(smem + d.ph[0].tab_off), s_nst[0], ring, full,
                      empty, rp, issued, lane);
    produce_stages<1>(d.ph[1], reinterpret_cast<const GemvStage *>(smem + d.ph[1].tab_off), s_nst[1], ring, full,
                      empty, rp, issued, lane);
    produce_stages<2>(d.ph[2], reinterpret_cast<const GemvStage *>(smem + d.ph[2].tab_off), s_nst[2], ring, full,
                      empty, rp, issued, lane);
    produce_stages<1>(d.ph[3], reinterpret_cast<const GemvStage *>(smem + d.ph[3].tab_off), s_nst[3], ring, full,
                      empty, rp, issued, lane);
    return;
  }

  pdl_wait();
  pdl_launch_dependents();
  unsigned base = 0, target = 0;  // barrier counter at launch, arrivals needed for the next barrier
  if (tid == 0) base = ld_acquire_gpu(d.bar);  // no barrier of this launch completes before all arrive
  auto sync = [&]() {
    target += unsigned(nctas);
    grid_sync(d.bar, base, target, d.err, tid);
  };

  // this CTA's attention item: warm its cached rows in L2 while the q/k/v projection runs
  const SeqInfo sq = d.seqs[0];
  const int n_items_max = d.ap.n_kv * d.n_split;
  int split = -1, kvh = 0;
  AttnSplit sp(sq, d.ap, d.n_split, 0);
  if (cta < n_items_max) {
    const int n_items = d.ap.n_kv * sp.n_eff;
    if (cta < n_items) {
      kvh = cta / sp.n_eff;
      split = cta % sp.n_eff;
      sp = AttnSplit(sq, d.ap, d.n_split, split);
      if (tid == 0 && sp.k_old_end > sp.k_begin) {
        const int esz = d.ap.kv_f32 ? 4 : 2;
        const size_t row_bytes = size_t(d.ap.head_dim) * esz;
        const uint8_t *kb = reinterpret_cast<const uint8_t *>(d.kv.base) + size_t(sq.slot) * d.kv.slot_stride * esz +
                            size_t(kvh) * d.ap.max_ctx * row_bytes + size_t(sp.k_begin) * row_bytes;
        const uint8_t *vb = kb + size_t(d.kv.slot_stride / 2) * esz;
        const uint32_t bytes = uint32_t(size_t(sp.k_old_end - sp.k_begin) * row_bytes) & ~15u;
        if (bytes) {
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kb), "r"(bytes) : "memory");
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vb), "r"(bytes) : "memory");
        }
      }
    }
  }

  RingPos rp = {0, 0};
  auto after = [&](int p) {
    for (int i = 0; i < s_nst[p]; ++i) rp.advance(d.nstage);
  };
  // ---- q/k/v
  const XSmem X0 = x_view(xreg, d.ph[0].nb, 1);
  gemv_phase<1>(d.ph[0], phase_type(d.ph[0]), reinterpret_cast<const GemvStage *>(smem + d.ph[0].tab_off), rp, ring,
                full, empty, s_sdone, X0, red, s_tdone, pro_red, cta, tid, warp, lane);
  after(0);
  sync();
  // ---- attention
  float *scr = reinterpret_cast<float *>(xreg);
  if (split >= 0) attn_item<G, KV32>(d, kvh, sp, split, scr, tid, warp, lane);
  sync();
  if (sp.n_eff > 1) {  // the same on every CTA
    for (int head = cta; head < d.ap.n_heads; head += nctas) attn_merge_head(d, head, sp.n_eff, scr, tid);
    sync();
  }
  // ---- o
  const XSmem X1 = x_view(xreg, d.ph[1].nb, 1);
  gemv_phase<1>(d.ph[1], phase_type(d.ph[1]), reinterpret_cast<const GemvStage *>(smem + d.ph[1].tab_off), rp, ring,
                full, empty, s_sdone, X1, red, s_tdone, pro_red, cta, tid, warp, lane);
  after(1);
  sync();
  // ---- gate/up + GeGLU
  const XSmem X2 = x_view(xreg, d.ph[2].nb, 1);
  gemv_phase<2>(d.ph[2], phase_type(d.ph[2]), reinterpret_cast<const GemvStage *>(smem + d.ph[2].tab_off), rp, ring,
                full, empty, s_sdone, X2, red, s_tdone, pro_red, cta, tid, warp, lane);
  after(2);
  sync();
  // ---- down (its outputs are read by the next launch after this grid completes)
  const XSmem X3 = x_view(xreg, d.ph[3].nb, 1);
  gemv_phase<1>(d.ph[3], phase_type(d.ph[3]), reinterpret_cast<const GemvStage *>(smem + d.ph[3].tab_off), rp, ring,
                full, empty, s_sdone, X3, red, s_tdone, pro_red, cta, tid, warp, lane);
}

// ---------------------------------------------------------------- host side
constexpr int DL_STAGE_TARGET = 24 * 1024;
constexpr int DL_SMEM = 227 * 1024 - 1024;
constexpr int DL_RED_TARGET = 32 * 1024;

// Partition of one projection over `ctas` CTAs (as launch_qgemv_t); false if it does not fit.
static bool plan_phase(QGemvArgs &a, int nmat, int ctas, int &stage_bytes, int64_t &red_bytes, int64_t &tab_bytes) {
  const int nb = a.nb;
  int64_t tiles = 0;
  int nbs_min = nb;
  for (int i = 0; i < a.nseg; ++i) {
    GemvSegK &S = a.seg[i];
    if (S.rows <= 0 || (S.type != T_Q4_K && S.type != T_Q6_K)) return false;
    S.tile0 = int(tiles);
    tiles += (S.rows + GEMV_TILE - 1) / GEMV_TILE;
    int nbs = DL_STAGE_TARGET / (nmat * S.rec);
    if (nbs < 1) nbs = 1;
    if (nbs > nb) nbs = nb;
    S.nbs = nbs;
    if (nbs < nbs_min) nbs_min = nbs;
    if (nmat * nbs * S.rec > stage_bytes) stage_bytes = nmat * nbs * S.rec;
  }
  if (tiles < ctas || tiles * nb >= (int64_t(1) << 30)) return false;
  a.units = int(tiles * nb);
  const int64_t tile_red = int64_t(GEMV_TILE) * nmat * nb * 4;
  int64_t lt_cap = DL_RED_TARGET / tile_red;
  if (lt_cap < 3) lt_cap = 3;
  if ((tiles + lt_cap - 3) / (lt_cap - 2) > ctas) return false;
  a.uq = int(a.units / ctas);
  a.ur = int(a.units % ctas);
  const int64_t max_units = (a.units + ctas - 1) / ctas;
  const int64_t lt_max = (max_units + nb - 1) / nb + 1;
  a.max_stages = int(max_units / nbs_min + lt_max + 1);
  red_bytes = lt_max * tile_red > red_bytes ? lt_max * tile_red : red_bytes;
  tab_bytes = (a.max_stages * int64_t(sizeof(GemvStage)) + 127) / 128 * 128;
  return true;
}

struct DecodeLayerPlanIn {
  const GemvSeg *qkv;  // 3 segments
  GemvSeg o, gate_up, down;
  GemvPrologue pro_qkv, pro_o, pro_gu, pro_down;
  int64_t hidden, q_dim, ffn;
};

static bool fill_phase(QGemvArgs &a, const GemvSeg *segs, int nseg, int64_t K, const GemvPrologue &pro) {
  if (K % QK_K || K / QK_K > 64) return false;
  a.nseg = nseg;
  a.nb = int(K / QK_K);
  a.pro = pro;
  for (int i = 0; i < nseg; ++i) {
    const GemvSeg &sg = segs[i];
    if (!sg.w[0] || sg.rows <= 0 || sg.rows >= (int64_t(1) << 30)) return false;
    GemvSegK &S = a.seg[i];
    S.w[0] = sg.w[0];
    S.w[1] = sg.w[1];
    S.y = sg.y;
    S.rows = int(sg.rows);
    S.type = sg.type;
    S.rec = kquant_rec_bytes(sg.type);
    S.ldy = sg.ldy;
  }
  return true;
}

static bool plan_layer(const DecodeLayerPlanIn &in, const AttnParams &ap, DecodeLayerArgs &d, size_t &smem) {
  const int ctas = num_sms();
  if (!fill_phase(d.ph[0], in.qkv, 3, in.hidden, in.pro_qkv) || !fill_phase(d.ph[1], &in.o, 1, in.q_dim, in.pro_o) ||
      !fill_phase(d.ph[2], &in.gate_up, 1, in.hidden, in.pro_gu) || !fill_phase(d.ph[3], &in.down, 1, in.ffn, in.pro_down))
    return false;
  if (!in.gate_up.w[1]) return false;
  int stage_bytes = 0;
  int64_t red = 0, tabs[DL_PHASES] = {};
  const int nmat[DL_PHASES] = {1, 1, 2, 1};
  for (int p = 0; p < DL_PHASES; ++p)
    if (!plan_phase(d.ph[p], nmat[p], ctas, stage_bytes, red, tabs[p])) return false;
  int64_t xb = 0;
  for (int p = 0; p < DL_PHASES; ++p) xb = std::max<int64_t>(xb, gemv_x_bytes(d.ph[p].nb, 1));
  const int G = ap.n_kv > 0 ? ap.n_heads / ap.n_kv : 1;
  const int64_t attn_scr = int64_t((DL_MAXG + 2) * DL_MAX_HD + 2 * DL_CW * DL_MAXG + DL_CW * G * DL_MAX_HD) * 4;
  xb = std::max(xb, attn_scr);
  int64_t off = 256;  // barriers: full[12], empty[12]
  const int red_off = int(off);
  off += (red + 127) / 128 * 128;
  int tab_off[DL_PHASES];
  for (int p = 0; p < DL_PHASES; ++p) {
    tab_off[p] = int(off);
    off += tabs[p];
  }
  const int x_off = int(off);
  off += (xb + 127) / 128 * 128;
  const int ring_off = int(off);
  int nst = int((DL_SMEM - off) / stage_bytes);
  if (nst > GEMV_MAX_STAGES) nst = GEMV_MAX_STAGES;
  if (nst < 2) return false;
  d.nstage = nst;
  d.stage_bytes = stage_bytes;
  for (int p = 0; p < DL_PHASES; ++p) {
    QGemvArgs &a = d.ph[p];
    a.nstage = nst;
    a.stage_bytes = stage_bytes;
    a.red_off = red_off;
    a.x_off = x_off;
    a.ring_off = ring_off;
    a.tab_off = tab_off[p];
  }
  smem = size_t(ring_off) + size_t(nst) * stage_bytes;
  return true;
}

bool decode_layer_supported(const AttnParams &ap) {
  if (ap.n_kv <= 0 || ap.n_heads % ap.n_kv) return false;
  const int G = ap.n_heads / ap.n_kv;
  return (G == 1 || G == 2 || G == 4) && ap.head_dim <= DL_MAX_HD && ap.head_dim % 8 == 0;
}

int decode_layer_splits(const AttnParams &ap, int64_t max_keys) {
  int64_t want = (num_sms() + ap.n_kv - 1) / ap.n_kv;  // one item per CTA
  const int64_t cap = (max_keys + DL_MIN_CHUNK - 1) / DL_MIN_CHUNK;
  if (want > cap) want = cap;
  if (want > DL_MAX_SPLIT) want = DL_MAX_SPLIT;
  if (want * ap.n_kv > num_sms()) want = num_sms() / ap.n_kv;
  return int(want < 1 ? 1 : want);
}

size_t decode_layer_scratch_bytes(const AttnParams &ap, int64_t max_keys) {
  return size_t(ap.n_heads) * decode_layer_splits(ap, max_keys) * (ap.head_dim + 2) * sizeof(float);
}

cudaError_t decode_layer(const DecodeLayerIn &in, cudaStream_t st) {
  const AttnParams &ap = in.ap;
  if (ap.kv_shared) return cudaErrorNotSupported;  // the attention item appends the layer's own k/v
  if (!decode_layer_supported(ap) || !in.bar || !in.split || !in.split->cnt || !in.split->part) return cudaErrorInvalidValue;
  DecodeLayerArgs d = {};
  DecodeLayerPlanIn pi = {};
  pi.qkv = in.qkv;
  pi.o = in.o;
  pi.gate_up = in.gate_up;
  pi.down = in.down;
  pi.pro_qkv = in.pro_qkv;
  pi.pro_o = in.pro_o;
  pi.pro_gu = in.pro_gu;
  pi.pro_down = in.pro_down;
  pi.hidden = in.hidden;
  pi.q_dim = in.q_dim;
  pi.ffn = in.ffn;
  size_t smem = 0;
  // shapes the layer kernel does not cover (every projection needs a 16-row tile per SM): the
  // caller runs the per-op launches instead
  if (!plan_layer(pi, ap, d, smem) || num_sms() > in.split->max_ctas) return cudaErrorNotSupported;
  const int n_split = decode_layer_splits(ap, in.max_keys);
  if (in.attn_scratch_bytes < size_t(ap.n_heads) * n_split * (ap.head_dim + 2) * sizeof(float))
    return cudaErrorInvalidValue;
  unsigned *err = device_error_ptr();
  for (int p = 0; p < DL_PHASES; ++p) {
    d.ph[p].err = err;
    d.ph[p].cnt = in.split->cnt;
    d.ph[p].part = in.split->part;
  }
  d.q = in.q;
  d.k = in.k;
  d.v = in.v;
  d.att = in.att;
  d.kv = in.kv;
  d.seqs = in.seqs;
  d.ap = ap;
  d.n_split = n_split;
  d.apart = static_cast<float *>(in.attn_scratch);
  d.bar = in.bar;
  d.err = err;
  const int G = ap.n_heads / ap.n_kv;
  void (*kern)(const DecodeLayerArgs) = nullptr;
  switch (G) {
    case 1: kern = ap.kv_f32 ? decode_layer_kernel<1, true> : decode_layer_kernel<1, false>; break;
    case 2: kern = ap.kv_f32 ? decode_layer_kernel<2, true> : decode_layer_kernel<2, false>; break;
    default: kern = ap.kv_f32 ? decode_layer_kernel<4, true> : decode_layer_kernel<4, false>; break;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  ++g_kernel_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(num_sms()));
  cfg.blockDim = dim3(DL_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phases meet at grid barriers
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, d);
}

}  // namespace sfc
