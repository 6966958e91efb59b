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
#include "tcgen05.cuh"

namespace sfc {

constexpr int DA_WARPS = 8;
constexpr int DA_THREADS = DA_WARPS * 32;
constexpr int DA_MAXG = 4;  // query heads per kv head handled here (registers hold q and acc per head)
constexpr int DA_MAX_HD = 256;
constexpr int DA_MIN_CHUNK = 64;  // keys per split at least
constexpr int DA_MAX_SPLIT = 32;  // key splits per (sequence, kv head) at most
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

// ---- warp-level tensor-core helpers (fp16 cache path)
// Eight 8x8 fp16 matrices' rows: lane L gives the shared-memory address of row L%8 of matrix L/8.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D (16x8 f32) += A (16x16 fp16, row) * B (16x8 fp16, col).  Fragments (lane = 4g + t): a0/a1 = rows
// g / g+8, k 2t..2t+1; a2/a3 = the same rows, k 2t+8..; b0/b1 = column g, k 2t.. / 2t+8..; d0,d1 =
// row g, columns 2t, 2t+1; d2,d3 = row g+8.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Byte offset of (key, dim) (dim a multiple of 8) in a 32-key tile laid out by the cache's tensor
// map: [64-dim chunk][key][64 dims], 16-byte pieces of a 128-byte row XOR-swizzled by key % 8.
__device__ __forceinline__ uint32_t kv_tile_off(int key, int dim) {
  return uint32_t((dim >> 6) * (32 * 128) + key * 128 + ((((dim & 63) >> 3) ^ (key & 7)) << 4));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int G, bool KV32, bool TC>
__global__ void __launch_bounds__(DA_THREADS) decode_attention_kernel(
    const float *__restrict__ qr, const float *__restrict__ kr, const float *__restrict__ vr, int q_ld, int kv_ld,
    float *__restrict__ out, KVLayer kv, const SeqInfo *__restrict__ seqs, AttnParams p, int n_split, int min_chunk,
    float *__restrict__ part, unsigned *__restrict__ counters, unsigned *err, const __grid_constant__ CUtensorMap kv_map,
    int64_t kv_row0, int64_t slot_rows) {
  constexpr int ESZ = KV32 ? 4 : 2;
  constexpr int TK = DA_TILE_BYTES / (DA_MAX_HD * ESZ);  // keys per tile
  constexpr int KPW = TK / DA_WARPS;                      // keys per warp per tile
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NST = TC ? 2 : 3;  // K/V ring stages
  __shared__ uint64_t bars[NST];
  __shared__ __align__(16) float s_vec[DA_MAXG + 2][DA_MAX_HD];  // q heads, then the new k and v
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
  // [NST][K tile | V tile]; the tensor-copy layout (TC) needs 1024-byte alignment
  uint8_t *tiles = TC ? smem + ((1024 - (smem_u32(smem) & 1023)) & 1023) : smem;
  // TC: first cache rows of this (slot, kv head)'s keys and values in the arena's tensor map
  const int64_t krow0 = kv_row0 + int64_t(sq.slot) * slot_rows + int64_t(kvh) * p.max_ctx;
  const int64_t vrow0 = krow0 + int64_t(p.n_kv) * p.max_ctx;

  auto issue = [&](int i) {
    const int st = i % NST;
    const int k0 = k_begin + i * TK;
    if (TC) {  // whole 32-key boxes (rows past the sequence are finite: the arena starts zeroed)
      mbar_arrive_expect_tx(&bars[st], uint32_t(2 * TK * row_bytes));
      tma_load_3d(tiles + st * 2 * DA_TILE_BYTES, &kv_map, 0, int(krow0 + k0), 0, &bars[st]);
      tma_load_3d(tiles + st * 2 * DA_TILE_BYTES + DA_TILE_BYTES, &kv_map, 0, int(vrow0 + k0), 0, &bars[st]);
      return;
    }
    const int nk = min(TK, k_old_end - k0);
    const uint32_t bytes = uint32_t(nk * row_bytes);
    mbar_arrive_expect_tx(&bars[st], 2 * bytes);
    bulk_g2s(tiles + st * 2 * DA_TILE_BYTES, kbase + head_off + size_t(k0) * row_bytes, bytes, &bars[st]);
    bulk_g2s(tiles + st * 2 * DA_TILE_BYTES + DA_TILE_BYTES, vbase + head_off + size_t(k0) * row_bytes, bytes,
             &bars[st]);
  };
  if (tid == 0) {
    for (int i = 0; i < NST; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    // cached rows never depend on the previous kernel: request them before the dependency wait
    for (int i = 0; i < n_tiles && i < NST; ++i) issue(i);
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

  float *s_acc = reinterpret_cast<float *>(tiles) + DA_WARPS * DA_MAX_HD;  // [DA_MAXG][DA_MAX_HD] after the keys
  float M[G], L[G];
  if constexpr (TC) {
    // ---- fp16 cache on the tensor pipe (mma.sync m16n8k16, fp32 accumulate), per 32-key tile:
    //  S^T = K Qc^T   every warp for its own 32 dims (two 16-dim k-steps): A = the key tile
    //                 (ldmatrix), B = the q columns in registers: column 2h = hi, 2h+1 = lo of
    //                 q_h * 2^u_h (fp16 keys exact, q to ~22 bits), so lane (g, t) holds head t's
    //                 partial scores at keys g, g+8, 16+g, 24+g; the partials go to shared memory
    //  softmax        warp 0: adds the warps' partials in warp order, running maximum and sum by
    //                 shuffles, p as fp16 hi + lo into P^T (shared)
    //  O^T += V^T P^T every warp for its 32 dims: A = values transposed by ldmatrix, B = P^T;
    //                 O stays in fragments (column 2h + 2h+1 = head h), rescaled when the maximum moves
    // The partial scores reuse the q rows of s_vec and its rows past the new value (four rows of
    // 256 floats whatever G): every warp holds its q fragments and the new key's score is known
    // before the first tile.
    const bool lane_on = lane * 8 < hd;
    __shared__ uint32_t s_pt[8][TK / 2];  // P^T as fp16 pairs [column][key pair]
    __shared__ float s_alpha[DA_MAXG], s_pnew[DA_MAXG], s_hm[DA_MAXG], s_hl[DA_MAXG];
    const int g8 = lane >> 2, t4 = lane & 3;
    for (int i = tid; i < 8 * (TK / 2); i += DA_THREADS) (&s_pt[0][0])[i] = 0u;
    const int d0w = 32 * warp;  // this warp's dims for S and O
    const bool pv = d0w < hd;   // hd is a multiple of 64
    const int nqk = hd / 32;    // warps holding partial scores
    auto part_slot = [&](int w) {  // warp w's 32 x float4 partials
      const int j = w >> 1;
      return reinterpret_cast<float4 *>(&s_vec[j < G ? j : j + 2][(w & 1) * 128]);
    };
    uint32_t qb[2][2];
    float rs = 1.f, m_run = -INFINITY, l_run = 0.f;  // warp 0: of head t4
    float snew[G];
    {
      float up[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float mx = 0.f;
        if (lane_on)
#pragma unroll
          for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(s_vec[h][lane * 8 + e]));
        mx = warp_max(mx);
        int E = int((__float_as_uint(mx) >> 23) & 0xFF) - 126;  // mx < 2^E
        if (E < -100) E = -100;
        up[h] = __uint_as_float(uint32_t(127 + 15 - E) << 23);  // |q * up| < 2^15
        if (t4 == h) rs = __uint_as_float(uint32_t(127 - 15 + E) << 23);
      }
      const int hh = g8 >> 1, part_lo = g8 & 1;  // this lane's B column: head hh, hi or lo
      const float uph = hh < G ? lt_of(up, hh < G ? hh : 0) : 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int ks = 2 * warp + j;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (hh < G && 16 * ks < hd) {
          const float *qv = s_vec[hh] + 16 * ks + 2 * t4;
          x[0] = qv[0] * uph;
          x[1] = qv[1] * uph;
          x[2] = qv[8] * uph;
          x[3] = qv[9] * uph;
          if (part_lo)
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] -= __half2float(__float2half_rn(x[e]));
        }
        qb[j][0] = pack_h2(x[0], x[1]);
        qb[j][1] = pack_h2(x[2], x[3]);
      }
      // the new key's score per head (owner), from the fp16-rounded key, before the q rows are reused
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float d = 0.f;
        if (owner && warp == 0 && lane_on)
#pragma unroll
          for (int e = 0; e < 8; ++e) d += s_vec[h][lane * 8 + e] * s_vec[G][lane * 8 + e];
        snew[h] = warp_sum(d);
      }
    }
    float o[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    __syncthreads();  // P^T zeroed; every warp is done reading the q rows
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i % NST;
      mbar_wait_bounded(&bars[st], (i / NST) & 1, err);
      const uint32_t kt = smem_u32(tiles + st * 2 * DA_TILE_BYTES), vt = kt + DA_TILE_BYTES;
      const int nk = min(TK, k_old_end - (k_begin + i * TK));
      if (pv) {
        float sc[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[mt][e] = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int ks = 2 * warp + j;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int key = 16 * mt + (lane & 7) + ((lane >> 3) & 1) * 8;
            uint32_t a[4];
            ldsm_x4(kt + kv_tile_off(key, 16 * ks + (lane >> 4) * 8), a);
            mma_f16_16816(sc[mt], a, qb[j][0], qb[j][1]);
          }
        }
        part_slot(warp)[lane] =
            make_float4(sc[0][0] + sc[0][1], sc[0][2] + sc[0][3], sc[1][0] + sc[1][1], sc[1][2] + sc[1][3]);
      }
      __syncthreads();  // this tile's partial scores
      if (warp == 0) {
        float4 acc = part_slot(0)[lane];
        for (int w = 1; w < nqk; ++w) {
          const float4 v = part_slot(w)[lane];
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        float s4[4] = {acc.x * rs, acc.y * rs, acc.z * rs, acc.w * rs};
        const int key4[4] = {g8, g8 + 8, 16 + g8, 24 + g8};
        float mt_ = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (key4[j] >= nk) s4[j] = -INFINITY;
          mt_ = fmaxf(mt_, s4[j]);
        }
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) mt_ = fmaxf(mt_, __shfl_xor_sync(0xFFFFFFFFu, mt_, sh));
        const float m_new = fmaxf(m_run, mt_);
        const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
        float p4[4], psum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          p4[j] = s4[j] == -INFINITY ? 0.f : expf(s4[j] - m_new);
          psum += p4[j];
        }
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) psum += __shfl_xor_sync(0xFFFFFFFFu, psum, sh);
        l_run = l_run * alpha + psum;
        m_run = m_new;
        if (t4 < G) {
          __half *ph = reinterpret_cast<__half *>(&s_pt[2 * t4][0]), *pl = reinterpret_cast<__half *>(&s_pt[2 * t4 + 1][0]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __half h = __float2half_rn(p4[j]);
            ph[key4[j]] = h;
            pl[key4[j]] = __float2half_rn(p4[j] - __half2float(h));
          }
          if (g8 == 0) s_alpha[t4] = alpha;
        }
      }
      __syncthreads();  // P^T and the rescale factors of this tile
      if (pv) {
        const float a_t = t4 < G ? s_alpha[t4] : 1.f;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[mt][e] *= a_t;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
          const uint32_t b0 = s_pt[g8][8 * kk + t4], b1 = s_pt[g8][8 * kk + 4 + t4];
          const int key = 16 * kk + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            uint32_t a[4];
            ldsm_x4_t(vt + kv_tile_off(key, d0w + 16 * mt + ((lane >> 3) & 1) * 8), a);
            mma_f16_16816(o[mt], a, b0, b1);
          }
        }
      }
      __syncthreads();  // every warp is done with this stage, P^T and the rescale factors
      if (tid == 0 && i + NST < n_tiles) issue(i + NST);
    }
    if (owner) {  // the new key and value, from this CTA's own (fp16-rounded) copy
      if (warp == 0 && t4 < G) {
        const float sn = lt_of(snew, t4 < G ? t4 : 0);
        const float m_new = fmaxf(m_run, sn);
        const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
        const float pn = expf(sn - m_new);
        l_run = l_run * alpha + pn;
        m_run = m_new;
        if (g8 == 0) {
          s_alpha[t4] = alpha;
          s_pnew[t4] = pn;
        }
      }
      __syncthreads();
      if (pv && t4 < G) {
        const float a_t = s_alpha[t4], pn = s_pnew[t4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int d = d0w + 16 * mt + g8;
          o[mt][0] = o[mt][0] * a_t + pn * s_vec[G + 1][d];
          o[mt][1] *= a_t;
          o[mt][2] = o[mt][2] * a_t + pn * s_vec[G + 1][d + 8];
          o[mt][3] *= a_t;
        }
      }
    }
    if (warp == 0 && g8 == 0 && t4 < G) {
      s_hm[t4] = m_run;
      s_hl[t4] = l_run;
    }
    if (pv && t4 < G)  // every issued copy has been waited on: the tile area is free
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int d = d0w + 16 * mt + g8;
        s_acc[t4 * DA_MAX_HD + d] = o[mt][0] + o[mt][1];
        s_acc[t4 * DA_MAX_HD + d + 8] = o[mt][2] + o[mt][3];
      }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      M[g] = s_hm[g];
      L[g] = s_hl[g];
    }
  } else {
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
      const int st = i % NST;
      mbar_wait_bounded(&bars[st], (i / NST) & 1, err);
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
      if (tid == 0 && i + NST < n_tiles) issue(i + NST);
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
// Measured at 64 sequences (contexts 512-3584, tensor-pipe kernel, three resident CTAs per SM):
// 11.36 ms per step at 2, 12.06 at 3, 11.79 at 4, 11.88 at 6, 11.64 at 8.
constexpr int DA_CTAS_PER_SM = 2;
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
                             cudaStream_t st, void *kv_arena, int64_t arena_rows) {
  if (n_seq <= 0) return cudaSuccess;
  if (!decode_attention_supported(p) || !counters) return cudaErrorInvalidValue;
  int ns = 1, min_chunk = DA_MIN_CHUNK;
  decode_attention_plan(n_seq, p, max_keys, sum_keys, &ns, &min_chunk);
  if (scratch_bytes < decode_attention_scratch_bytes(n_seq, p, max_keys)) return cudaErrorInvalidValue;
  // fp16 cache with whole 64-dim chunks: keys and values by tensor copies, products on the tensor pipe
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  const bool tc = !p.kv_f32 && p.head_dim % 64 == 0 && kv_tensor_map(kv_arena, arena_rows, p.head_dim, &map);
  const int64_t row0 = tc ? (static_cast<char *>(kv.base) - static_cast<char *>(kv_arena)) / 2 / p.head_dim : 0;
  const int64_t slot_rows = 2 * int64_t(p.n_kv) * p.max_ctx;
  const size_t smem = size_t(tc ? 2 : 3) * 2 * DA_TILE_BYTES + (tc ? 1024 : 0);
  const dim3 grid(unsigned(n_seq), unsigned(p.n_kv), unsigned(ns));
  const int G = p.n_heads / p.n_kv;
  void (*kern)(const float *, const float *, const float *, int, int, float *, KVLayer, const SeqInfo *, AttnParams,
               int, int, float *, unsigned *, unsigned *, const CUtensorMap, int64_t, int64_t) = nullptr;
  switch (G) {
    case 1:
      kern = tc ? decode_attention_kernel<1, false, true>
                : p.kv_f32 ? decode_attention_kernel<1, true, false> : decode_attention_kernel<1, false, false>;
      break;
    case 2:
      kern = tc ? decode_attention_kernel<2, false, true>
                : p.kv_f32 ? decode_attention_kernel<2, true, false> : decode_attention_kernel<2, false, false>;
      break;
    case 4:
      kern = tc ? decode_attention_kernel<4, false, true>
                : p.kv_f32 ? decode_attention_kernel<4, true, false> : decode_attention_kernel<4, false, false>;
      break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, grid, dim3(DA_THREADS), smem, st, q, k, v, q_ld, kv_ld, out, kv, seqs, p, ns, min_chunk,
                    static_cast<float *>(scratch), counters, device_error_ptr(), map, row0, slot_rows);
}

}  // namespace sfc
