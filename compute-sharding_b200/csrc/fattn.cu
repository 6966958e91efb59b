// fattn.cu — multi-token attention (prefill, chunked prompts, draft-tree verification) on the
// 5th-generation tensor cores, for an fp16 KV cache.
//
// Same arithmetic as the CUDA-core attention_kernel in ops.cu (real_forward.rs:1664-1689: causal
// softmax(q . k) v per query head, GQA, optional sliding window, draft-tree ancestor masks),
// reorganised as a flash-attention pass over 32-key tiles:
//   S = Q K^T   tcgen05.mma, A = Q from shared memory (K-major, 128-byte swizzle), B = the key tile
//               straight from the cache (K-major); Q is split exactly enough into two fp16 halves,
//               q*2^u = hi + lo (~22 significant bits), and both products go into the same fp32
//               accumulator, while the fp16 keys are exact operands.
//   softmax     four warps, thread = query row = TMEM lane: masks, running maximum, p = exp(s - m),
//               row sums in fp32; p split into fp16 hi + lo and written to tensor memory.
//   O += P V    tcgen05.mma with A = P from tensor memory and B = the value tile from shared
//               memory read MN-major (the cache stores values key-major, i.e. [key][dim]).
// O stays in tensor memory.  The running maximum used as the exponent reference is only moved (and
// O rescaled) when a tile's maximum exceeds it by more than 8 (p stays below e^8 in fp16 and fp32),
// so most tiles skip the read-modify-write of O; l and O always share the same reference, which
// keeps the result exact up to rounding.
//
// CTA = 128 query rows: TT = 128/G consecutive tokens of one sequence x the G query heads of one kv
// head (row r = g*TT + i), over a split of the tile's key range.  192 threads:
//   warps 0-3: softmax and the final epilogue (TMEM lanes 32w..32w+31)
//   warp 4   : lane 0 copies key tiles, lane 1 value tiles (one 3-D tensor copy each, 16 KB)
//   warp 5   : one thread issues the MMAs: S(j) into one of two S buffers, then O(j-1)
// With several splits each CTA writes (m, l, unnormalised O) and attn_combine_kernel (ops.cu)
// merges them.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace sfc {

constexpr int FA_M = 128;          // query rows per CTA (UMMA M)
constexpr int FA_NK = 32;          // keys per tile
constexpr int FA_THREADS = 192;
constexpr int FA_MAX_HD = 256;
constexpr int FA_KV_STAGES = 2;
constexpr int FA_TILE_BYTES = FA_NK * FA_MAX_HD * 2;  // K or V tile: 32 keys x 256 fp16 = 16 KB
constexpr int FA_Q_BYTES = FA_M * FA_MAX_HD * 2;      // one Q half: 128 rows x 256 fp16 = 64 KB
// TMEM columns: S buffers, P buffers (hi 16 + lo 16 columns of fp16 pairs each), O
constexpr int FA_COL_S = 0;        // 2 x 32
constexpr int FA_COL_P = 64;       // 2 x 32
constexpr int FA_COL_O = 128;      // head_dim columns
constexpr int FA_TMEM_COLS = 512;
constexpr float FA_RESCALE_THRESHOLD = 8.0f;

struct FaTile {
  int32_t seq;   // index into the batch's SeqInfo array
  int32_t t0;    // first token of the tile within the sequence
};

struct FaArgs {
  CUtensorMap kv_map;      // the layer's cache as fp16 [key-row][64-dim chunk][64] (3-D, see make_kv_map)
  const float *q;          // [n_tok][n_heads * hd]
  float *out;              // [n_tok][n_heads * hd]
  const SeqInfo *seqs;
  const FaTile *tiles;
  const int32_t *tok_limit;  // nullable: per-row key limit (tree verification)
  const uint64_t *tok_mask;  // nullable: per-row ancestor bits over the keys [pos0, pos0 + 64)
  float *part;             // [n_tok][n_heads][n_split][hd + 2] when n_split > 1
  unsigned *err;
  int64_t slot_rows;       // cache rows (keys) per slot: 2 * n_kv * max_ctx
  int64_t layer_row0;      // first cache row of this layer's slab
  int n_heads, n_kv, hd, max_ctx, window, n_split;
};

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Shared-memory matrix descriptor, MN-major, 128-byte swizzle: each 128-byte row holds 64
// consecutive MN elements of one K index, 8 K rows form a 1024-byte atom; `lbo` = bytes between
// 64-element MN chunks, `sbo` = bytes between 8-row K groups.
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(FA_THREADS, 1) flash_attention_kernel(const __grid_constant__ FaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *sQ = smem;                                   // [hi | lo][hd/64 chunks][128 rows x 128 B]
  uint8_t *sKV = sQ + 2 * FA_Q_BYTES;                   // [stage][K | V][hd/64 chunks][32 keys x 128 B]
  __shared__ uint64_t kfull[FA_KV_STAGES], vfull[FA_KV_STAGES], kvempty[FA_KV_STAGES];
  __shared__ uint64_t sfull[2], sfree[2], pfull[2], odone[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int s_klo, s_khi;
  __shared__ float s_rowscale[FA_M];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = a.hd, nch = hd / 64;
  const int G = a.n_heads / a.n_kv, TT = FA_M / G;
  const FaTile tile = a.tiles[blockIdx.x];
  const SeqInfo sq = a.seqs[tile.seq];
  const int kvh = blockIdx.y, split = blockIdx.z;

  if (tid == 0) {
    for (int i = 0; i < FA_KV_STAGES; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&vfull[i], 1);
      mbar_init(&kvempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], 4);
      mbar_init(&pfull[i], 4);
      mbar_init(&odone[i], 1);
    }
    s_klo = INT_MAX;
    s_khi = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(FA_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_wait();  // q rows and this batch's keys come from the previous kernels
  pdl_launch_dependents();
  __syncthreads();

  // ---- Q tile into shared memory: row r = g*TT + i, q * 2^u split into fp16 hi + lo (K-major,
  // 128-byte swizzle, one 16 KB tile per 64-dim chunk); lane l holds dims 8l..8l+7
  constexpr int QB = 4;  // rows per warp per pass: their loads are issued together
  for (int r0 = warp * QB; r0 < FA_M; r0 += (FA_THREADS / 32) * QB) {
    float v[QB][8];
#pragma unroll
    for (int b = 0; b < QB; ++b) {
      const int r = r0 + b, g = r / TT, i = r % TT;
      const bool on = r < FA_M && tile.t0 + i < sq.n_tok && lane * 8 < hd;
      if (on) {
        const int64_t t = int64_t(sq.tok0) + tile.t0 + i;
        const float *src = a.q + t * int64_t(a.n_heads) * hd + int64_t(kvh * G + g) * hd + lane * 8;
        const float4 f0 = *reinterpret_cast<const float4 *>(src), f1 = *reinterpret_cast<const float4 *>(src + 4);
        v[b][0] = f0.x; v[b][1] = f0.y; v[b][2] = f0.z; v[b][3] = f0.w;
        v[b][4] = f1.x; v[b][5] = f1.y; v[b][6] = f1.z; v[b][7] = f1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[b][e] = 0.f;
      }
    }
#pragma unroll
    for (int b = 0; b < QB; ++b) {
      const int r = r0 + b;
      if (r >= FA_M) break;
      float mx = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[b][e]));
      mx = warp_max(mx);
      int E = int((__float_as_uint(mx) >> 23) & 0xFF) - 126;  // mx < 2^E
      if (E < -100) E = -100;
      const float up = __uint_as_float(uint32_t(127 + 15 - E) << 23);  // |q * up| < 2^15
      if (lane == 0) s_rowscale[r] = __uint_as_float(uint32_t(127 - 15 + E) << 23);
      if (lane * 8 < hd) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const float x0 = v[b][2 * e2] * up, x1 = v[b][2 * e2 + 1] * up;
          const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
          hw[e2] = pack_half2(__half2float(h0), __half2float(h1));
          lw[e2] = pack_half2(x0 - __half2float(h0), x1 - __half2float(h1));
        }
        const uint32_t off = uint32_t((lane >> 3) * (FA_M * 128)) + sw128_off(r, lane & 7);
        *reinterpret_cast<uint4 *>(sQ + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(sQ + FA_Q_BYTES + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
  }

  // ---- per-row key window (softmax threads: row r = tid): keys [w0, limit), tree bits over
  // [pos0, pos0 + 64); the CTA's key range is the union over its valid rows
  int r_limit = 0, r_w0 = 0;
  uint64_t r_mask = ~0ull;
  bool r_valid = false;
  if (tid < FA_M) {
    const int i = tid % TT;
    r_valid = tile.t0 + i < sq.n_tok;
    if (r_valid) {
      const int64_t t = int64_t(sq.tok0) + tile.t0 + i;
      const int pos = sq.pos0 + tile.t0 + i;
      r_limit = a.tok_limit ? a.tok_limit[t] : pos + 1;
      r_w0 = a.window > 0 ? max(0, r_limit - a.window) : 0;
      if (a.tok_mask) r_mask = a.tok_mask[t];
      atomicMin(&s_klo, r_w0);
      atomicMax(&s_khi, r_limit);
    }
  }
  fence_proxy_async_smem();  // Q (generic stores) -> visible to the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int klo = s_klo == INT_MAX ? 0 : s_klo, khi = max(s_khi, klo);
  const int n_all = (khi - klo + FA_NK - 1) / FA_NK;
  const int per = (n_all + a.n_split - 1) / a.n_split;
  const int kt0 = min(n_all, split * per), kt1 = min(n_all, kt0 + per);
  const int nt = kt1 - kt0;  // key tiles of this CTA: keys klo + 32*(kt0 + j) + [0, 32)

  if (warp == 4) {
    // ---- producer: lane 0 the key tiles, lane 1 the value tiles (bulk copies of one thread complete
    // one after another, so the two streams come from two threads)
    if (lane < 2) {
      const int64_t row0 = a.layer_row0 + int64_t(sq.slot) * a.slot_rows + int64_t(lane) * a.n_kv * a.max_ctx +
                           int64_t(kvh) * a.max_ctx;
      uint64_t *full = lane ? vfull : kfull;
      for (int j = 0; j < nt; ++j) {
        const int s = j % FA_KV_STAGES;
        if (j >= FA_KV_STAGES) mbar_spin(&kvempty[s], ((j / FA_KV_STAGES) & 1) ^ 1, a.err);  // O(j-2) done
        const int key0 = klo + FA_NK * (kt0 + j);
        mbar_arrive_expect_tx(&full[s], uint32_t(FA_NK * hd * 2));
        tma_load_3d(sKV + s * 2 * FA_TILE_BYTES + lane * FA_TILE_BYTES, &a.kv_map, 0, int(row0 + key0), 0, &full[s]);
      }
    }
  } else if (warp == 5) {
    // ---- MMA issuer: S(0), then S(j) ahead of O(j-1) so that the next scores are computed while the
    // softmax of the current tile runs
    if (lane == 0) {
      const uint32_t idesc_s = (1u << 4) | (uint32_t(FA_NK >> 3) << 17) | (uint32_t(FA_M >> 4) << 24);
      const uint32_t idesc_o = (1u << 4) | (1u << 16) | (uint32_t(hd >> 3) << 17) | (uint32_t(FA_M >> 4) << 24);
      const uint32_t qh = smem_u32(sQ), ql = smem_u32(sQ + FA_Q_BYTES);
      auto issue_s = [&](int j) {
        const int s = j % FA_KV_STAGES, sb = j & 1;
        mbar_spin(&kfull[s], (j / FA_KV_STAGES) & 1, a.err);
        if (j >= 2) mbar_spin(&sfree[sb], ((j >> 1) & 1) ^ 1, a.err);  // softmax done with S(j-2)
        tc_fence_after();
        const uint32_t kb = smem_u32(sKV + s * 2 * FA_TILE_BYTES);
        const uint32_t d = tmem + uint32_t(FA_COL_S + 32 * sb);
        for (int c = 0; c < nch; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t bdesc = sw128_desc(kb + uint32_t(c * FA_NK * 128 + k * 32));
            tc_mma_f16(d, sw128_desc(qh + uint32_t(c * FA_M * 128 + k * 32)), bdesc, idesc_s, (c | k) != 0);
            tc_mma_f16(d, sw128_desc(ql + uint32_t(c * FA_M * 128 + k * 32)), bdesc, idesc_s, 1u);
          }
        tc_commit(&sfull[sb]);
      };
      auto issue_o = [&](int j) {
        const int s = j % FA_KV_STAGES, pb = j & 1;
        mbar_spin(&pfull[pb], (j >> 1) & 1, a.err);
        mbar_spin(&vfull[s], (j / FA_KV_STAGES) & 1, a.err);
        tc_fence_after();
        const uint32_t vb = smem_u32(sKV + s * 2 * FA_TILE_BYTES + FA_TILE_BYTES);
        const uint32_t ph = tmem + uint32_t(FA_COL_P + 32 * pb), pl = ph + 16;
#pragma unroll
        for (int kk = 0; kk < FA_NK / 16; ++kk) {
          // values [key][dim]: dims are the MN index (64 per 128-byte row, chunks 4 KB apart), keys K
          const uint64_t bdesc = sw128_desc_mn(vb + uint32_t(kk * 16 * 128), FA_NK * 128, 1024);
          tc_mma_f16_ts(tmem + FA_COL_O, ph + uint32_t(8 * kk), bdesc, idesc_o, (j | kk) != 0);
          tc_mma_f16_ts(tmem + FA_COL_O, pl + uint32_t(8 * kk), bdesc, idesc_o, 1u);
        }
        tc_commit(&kvempty[s]);
        tc_commit(&odone[pb]);
      };
      if (nt > 0) issue_s(0);
      for (int j = 1; j <= nt; ++j) {
        if (j < nt) issue_s(j);
        issue_o(j - 1);
      }
    }
  } else {
    // ---- softmax (warps 0-3, thread = row r = TMEM lane r)
    const int r = tid;
    const uint32_t lane_base = tmem + (uint32_t(32 * warp) << 16);
    const float rs = s_rowscale[r];
    const int pos0 = sq.pos0;
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < nt; ++j) {
      const int sb = j & 1;
      warp_wait(&sfull[sb], (j >> 1) & 1, a.err);
      tc_fence_after();
      uint32_t sraw[32];
      tmem_ld32(lane_base + uint32_t(FA_COL_S + 32 * sb), sraw);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[sb]);
      const int key0 = klo + FA_NK * (kt0 + j);
      float sv[32];
      float mt = -INFINITY;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int key = key0 + k;
        bool ok = r_valid && key >= r_w0 && key < r_limit;
        if (ok && key >= pos0 && key - pos0 < 64) ok = (r_mask >> (key - pos0)) & 1ull;
        sv[k] = ok ? __uint_as_float(sraw[k]) * rs : -INFINITY;
        mt = fmaxf(mt, sv[k]);
      }
      // move the exponent reference only when this tile's maximum exceeds it by the threshold; rows
      // that had no valid key yet (O and l still zero) move it without touching O
      const bool move = mt > m_ref + FA_RESCALE_THRESHOLD || (m_ref == -INFINITY && mt != -INFINITY);
      const bool need_o = move && m_ref != -INFINITY;
      if (__any_sync(0xFFFFFFFFu, need_o)) {
        // O(j-1) must be complete before its rows are rescaled
        warp_wait(&odone[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err);
        tc_fence_after();
        const float alpha = need_o ? expf(m_ref - mt) : 1.0f;
        for (int c = 0; c < hd; c += 32) {
          uint32_t o[32];
          tmem_ld32(lane_base + uint32_t(FA_COL_O + c), o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(lane_base + uint32_t(FA_COL_O + c), o);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (move) m_ref = mt;
      // p = exp(s - m_ref) (0 for masked keys and while no key is valid), split into fp16 hi + lo
      uint32_t phw[16], plw[16];
      float psum = 0.f;
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        const float p0 = sv[k] == -INFINITY ? 0.f : expf(sv[k] - m_ref);
        const float p1 = sv[k + 1] == -INFINITY ? 0.f : expf(sv[k + 1] - m_ref);
        psum += p0 + p1;
        const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
        phw[k >> 1] = pack_half2(__half2float(h0), __half2float(h1));
        plw[k >> 1] = pack_half2(p0 - __half2float(h0), p1 - __half2float(h1));
      }
      l += psum;
      const int pb = j & 1;
      if (j >= 2) warp_wait(&odone[pb], ((j >> 1) & 1) ^ 1, a.err);  // O(j-2) done reading P[pb]
      tc_fence_after();
      tmem_st16(lane_base + uint32_t(FA_COL_P + 32 * pb), phw);
      tmem_st16(lane_base + uint32_t(FA_COL_P + 32 * pb + 16), plw);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[pb]);
    }
    // ---- epilogue: O / l (one split) or the split's (m, l, O) partial
    const int g = r / TT, i = r % TT;
    const int64_t t = int64_t(sq.tok0) + tile.t0 + i;
    const int h = kvh * G + g;
    if (nt > 0) {
      warp_wait(&odone[(nt - 1) & 1], ((nt - 1) >> 1) & 1, a.err);
      tc_fence_after();
    }
    float *dst = nullptr;
    float scale = 1.f;
    if (a.n_split == 1) {
      dst = a.out + t * int64_t(a.n_heads) * hd + int64_t(h) * hd;
      scale = l > 0.f ? 1.0f / l : 0.f;
    } else {
      float *pp = a.part + ((t * a.n_heads + h) * a.n_split + split) * int64_t(hd + 2);
      if (r_valid) {
        pp[0] = m_ref;
        pp[1] = l;
      }
      dst = pp + 2;
    }
    for (int c = 0; c < hd; c += 32) {
      uint32_t o[32];
      if (nt > 0) {
        tmem_ld32(lane_base + uint32_t(FA_COL_O + c), o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0u;
      }
      if (r_valid) {
        if (a.n_split == 1) {  // output rows are 16-byte aligned (head_dim % 64 == 0)
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4 *>(dst + c + e) =
                make_float4(__uint_as_float(o[e]) * scale, __uint_as_float(o[e + 1]) * scale,
                            __uint_as_float(o[e + 2]) * scale, __uint_as_float(o[e + 3]) * scale);
        } else {  // partial rows of hd + 2 floats: 8-byte aligned
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            *reinterpret_cast<float2 *>(dst + c + e) = make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1]));
        }
      }
    }
  }
  __syncwarp();  // single-lane roles: lanes wait for their lane 0 before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FA_TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- host side
// The whole KV arena as a 3-D fp16 tensor [64-dim chunk][cache row][64 dims] (dims innermost; a
// cache row is one key or value of one (layer slab, slot, K|V, kv head, position)), box = 64 dims x
// 32 rows x all chunks, 128-byte swizzle: one copy lands a tile as [chunk][key][64 dims], the
// layout the MMA descriptors describe.  Rows past the arena read as zeros.
static bool make_kv_map(CUtensorMap *m, void *arena, int64_t rows, int hd) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {64, cuuint64_t(rows), cuuint64_t(hd / 64)};
  const cuuint64_t strides[2] = {cuuint64_t(hd) * 2, 128};
  const cuuint32_t box[3] = {64, cuuint32_t(FA_NK), cuuint32_t(hd / 64)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, arena, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool kv_map_cached(void *arena, int64_t rows, int hd, CUtensorMap *out) {
  struct Entry {
    void *arena;
    int64_t rows;
    int hd;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[16];
  static int n = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].arena == arena && cache[i].rows == rows && cache[i].hd == hd) {
      *out = cache[i].map;
      return true;
    }
  Entry e{arena, rows, hd, {}};
  if (!make_kv_map(&e.map, arena, rows, hd)) return false;
  cache[n < 16 ? n++ : 15] = e;
  *out = e.map;
  return true;
}

bool flash_attention_supported(const AttnParams &p) {
  if (p.kv_f32 || p.n_kv <= 0 || p.n_heads % p.n_kv) return false;
  const int G = p.n_heads / p.n_kv;
  return FA_M % G == 0 && p.head_dim % 64 == 0 && p.head_dim <= FA_MAX_HD && p.max_ctx > 0 && encode_fn() != nullptr;
}

int flash_attention_tile_tokens(const AttnParams &p) { return FA_M / (p.n_heads / p.n_kv); }

bool kv_tensor_map(void *kv_arena, int64_t arena_rows, int head_dim, CUtensorMap *out) {
  return kv_arena && arena_rows > 0 && arena_rows < (int64_t(1) << 30) && head_dim % 64 == 0 &&
         head_dim <= FA_MAX_HD && kv_map_cached(kv_arena, arena_rows, head_dim, out);
}

bool flash_attention_prepare(void *kv_arena, int64_t arena_rows, int head_dim) {
  CUtensorMap m;
  return kv_arena && arena_rows > 0 && arena_rows < (int64_t(1) << 30) && head_dim % 64 == 0 &&
         head_dim <= FA_MAX_HD && kv_map_cached(kv_arena, arena_rows, head_dim, &m);
}

constexpr int FA_SPLIT_CAP = 8;

size_t flash_attention_scratch_bytes(int64_t n_tok, const AttnParams &p) {
  return size_t(n_tok) * p.n_heads * FA_SPLIT_CAP * (p.head_dim + 2) * sizeof(float);
}

cudaError_t flash_attention(const float *q, float *out, void *kv_arena, int64_t arena_rows, int64_t layer_row0,
                            const SeqInfo *seqs, const FaTileRef *tiles, int n_tiles, const int32_t *tok_limit,
                            const uint64_t *tok_mask, int64_t n_tok, int64_t max_keys, const AttnParams &p,
                            void *scratch, size_t scratch_bytes, cudaStream_t st) {
  if (n_tok <= 0 || n_tiles <= 0) return cudaSuccess;
  if (!flash_attention_supported(p) || arena_rows >= (int64_t(1) << 30)) return cudaErrorInvalidValue;
  static_assert(sizeof(FaTileRef) == sizeof(FaTile), "tile records");
  FaArgs a;
  memset(&a, 0, sizeof(a));
  if (!kv_map_cached(kv_arena, arena_rows, p.head_dim, &a.kv_map)) return cudaErrorInvalidValue;
  a.q = q;
  a.out = out;
  a.seqs = seqs;
  a.tiles = reinterpret_cast<const FaTile *>(tiles);
  a.tok_limit = tok_limit;
  a.tok_mask = tok_mask;
  a.err = device_error_ptr();
  a.slot_rows = 2 * int64_t(p.n_kv) * p.max_ctx;
  a.layer_row0 = layer_row0;
  a.n_heads = p.n_heads;
  a.n_kv = p.n_kv;
  a.hd = p.head_dim;
  a.max_ctx = int(p.max_ctx);
  a.window = p.window;
  // key splits: enough CTAs for every SM, each split at least two key tiles
  const int64_t ctas = int64_t(n_tiles) * p.n_kv;
  int64_t ns = (num_sms() + ctas - 1) / ctas;
  const int64_t cap = (max_keys + 2 * FA_NK - 1) / (2 * FA_NK);
  if (ns > cap) ns = cap;
  if (ns > FA_SPLIT_CAP) ns = FA_SPLIT_CAP;
  if (ns < 1) ns = 1;
  a.n_split = int(ns);
  if (ns > 1) {
    if (scratch_bytes < size_t(n_tok) * p.n_heads * ns * (p.head_dim + 2) * sizeof(float)) return cudaErrorInvalidValue;
    a.part = static_cast<float *>(scratch);
  }
  const size_t smem = 1024 + 2 * size_t(FA_Q_BYTES) + size_t(FA_KV_STAGES) * 2 * FA_TILE_BYTES;
  cudaError_t e = cudaFuncSetAttribute(flash_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  e = launch_pdl(flash_attention_kernel, dim3(unsigned(n_tiles), unsigned(p.n_kv), unsigned(ns)), dim3(FA_THREADS), smem,
                 st, a);
  if (e != cudaSuccess || ns == 1) return e;
  return attn_combine(a.part, out, n_tok, p.n_heads, p.head_dim, int(ns), st);
}

}  // namespace sfc
