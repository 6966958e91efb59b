// qgemm.cu — K-quant GEMM on the 5th-generation tensor cores (tcgen05 MMA with TMEM
// accumulators) for prefill, batched decode and speculative verify (8 or more tokens), and the
// same GEMM over fp16 weights (the tied-embedding logits).
//
// Replaces the multi-token path of the reference's row dots (crates/stage-forward-lab/src/
// quants.rs:1801-1909 for Q4_K, :2594-2688 for Q6_K) as driven by real_math.rs:398-1124
// (matmul_quantized_many_refs_range and its token-major variant), the gate/up pair of
// real_math.rs:1584-1800 and the RMSNorm / residual steps around them (real_forward.rs:1690-1749).
//
// Arithmetic.  For weight row r and one 256-element block:
//   Q4_K: w_i = d*sc_j*q_i - dmin*m_j      (j = 32-element sub-block, q 4-bit, sc/m 6-bit)
//   Q6_K: w_i = d*sc_j*(q_i - 32)          (j = 16-element sub-block, q 6-bit, sc int8)
// Operand A (weights) holds the integers a_i = sc_j*q_i (Q4_K: <= 945, exact in fp16) or, for
// Q6_K, two tiles 16*sh*(q_i-32) and sl*(q_i-32) with sc_j = 16*sh + sl (each exact in fp16),
// both multiplied into the same accumulator.  Activations of each (token, block) are scaled by a
// power of two s and split x/s = hi + lo into two fp16 values (~22 significant bits together); hi
// and lo rows of every token are the 2*TN columns of operand B.  Per block the MMA chain
// accumulates sum_i a_i*hi_i and sum_i a_i*lo_i in fp32 TMEM columns and the epilogue adds
//   y += (d*s) * (D_hi + D_lo) - dmin * sum_j m_j * S_j       (S_j = fp32 sum of x over sub-block j)
// so products are exact and rounding happens in fp32 sums, as in the reference.  fp16 weights are
// operand A as they are (d = 1, no mins).
//
// Two kernels share the operand-B image (gemm_bprep_kernel), the TMEM accumulators and the
// epilogue arithmetic: qgemm_kq_kernel dequantises K-quant blocks straight into tensor memory;
// qgemm_f16_kernel streams fp16 weight tiles into shared memory with 2-D tensor copies.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <math.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace sfc {

constexpr int QG_M = 128;        // weight rows per tile (UMMA M)
constexpr int QG_KC = 64;        // K elements per chunk: one 128-byte swizzle row of fp16
constexpr int QG_CPB = QK_K / QG_KC;  // chunks per 256-element block
constexpr int QG_AST = 4;        // fp16 kernel: A ring tiles (two slots of two chunks)
constexpr int QG_RST = 2;        // K-quant kernel: raw-block ring slots
constexpr int QG_THREADS = 352;  // fp16 kernel
constexpr int QG_A_BYTES = QG_M * 128;  // one A tile: 128 rows x 64 fp16
constexpr int QG_A_SLOT = 2 * QG_A_BYTES;  // one A ring slot: two chunks
constexpr int QG_RAW_BYTES = (QG_M / KQ_TILE) * REC_Q6_K;  // one block of 128 rows: 8 tiled records
constexpr int QG_MAX_NB = 64;    // K <= 16384
constexpr int QG_META = 9;       // per (token, block): s and 8 sub-block sums
constexpr int QG_MAX_SEG = 3;

// B ring slots for a token-tile width: chunks of 2*TN rows x 128 B, up to 64 KB and 16 chunks
__host__ __device__ constexpr int qg_b_slots(int tn) {
  return (65536 / (tn * 256)) > 16 ? 16 : (65536 / (tn * 256)) < 4 ? 4 : (65536 / (tn * 256));
}

struct QGemmSeg {
  CUtensorMap map[4];  // K-quants: [0] tiled records; fp16: [0] rows
  float *y;
  int64_t ldy;
  int rows;
  int type;
  int tile0;  // first global row tile of this segment
};

struct QGemmArgs {
  QGemmSeg seg[QG_MAX_SEG];
  int nseg;
  int nb;        // 256-element blocks along K
  int n_tok;     // valid tokens
  int n_ttiles;  // token tiles
  const uint8_t *bimg;   // [ttile][K/64 chunks][N rows x 128 B] swizzled fp16 (hi rows, then lo rows)
  const float *bmeta;    // [ttile][nb][9][TN]
  float *part;           // split-K partials [split][n_tok][tiles*128] (null: one split, write y)
  int64_t part_ld;       // tiles * 128
  unsigned *err;
};

// fp16x2 (1024 + q0, 1024 + q1) -> (q0 * s, q1 * s): (1024 + q) * s - 1024 * s is exact and
// representable (q <= 15, s <= 63), so the single rounding of the fused multiply-add is exact.
__device__ __forceinline__ uint32_t half2_times(uint32_t v, __half2 s2, __half2 negbias2) {
  __half2 h = *reinterpret_cast<const __half2 *>(&v);
  h = __hfma2(h, s2, negbias2);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// ---------------------------------------------------------------- fp16-weight GEMM
// CTA = 128 weight rows x TN tokens, 352 threads, warp-specialised around mbarrier rings:
//   warp 8   : producer of the A tiles (2-D tensor copies of 128 rows x 64 fp16, 128-byte swizzle),
//              each step's once its activation chunks have landed
//   warp 10  : producer of the activation chunks (operand B, pre-swizzled by gemm_bprep_kernel) and
//              per-block activation metadata
//   warp 9   : one thread issues tcgen05.mma (M=128, N=2*TN, K=16), 8 per ring step, into one of two
//              TMEM accumulators (double-buffered across 256-element blocks)
//   warps 0-7: the epilogue, one block behind: tcgen05.ld a finished block's accumulator (TMEM lane
//              = row), add s * (D_hi + D_lo) into per-thread fp32 sums, store y at the end
template <int TN>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemm_f16_kernel(const __grid_constant__ QGemmArgs a) {
  constexpr int N = 2 * TN;             // B rows: hi then lo per token
  constexpr int B_BYTES = N * 128;      // one B chunk
  constexpr int TMEM_COLS = 2 * N < 32 ? 32 : 2 * N;
  constexpr int BM_BYTES = QG_META * TN * 4;
  constexpr int BST = qg_b_slots(TN);   // B ring slots: up to 64 KB, at most 16 chunks (4 blocks)
  constexpr int BLOG = BST == 16 ? 4 : BST == 8 ? 3 : 2;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned carve-up (swizzled operand tiles need it)
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *sA = smem;                                  // [2][QG_A_SLOT]
  uint8_t *sB = sA + QG_AST * QG_A_BYTES;              // [BST][B_BYTES]
  float *sBm = reinterpret_cast<float *>(sB + BST * B_BYTES);  // [4][9][TN]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sBm + 4 * QG_META * TN);
  uint64_t *a_full = bars, *a_empty = bars + 2, *b_full = bars + 4, *b_empty = bars + 20;
  uint64_t *acc_full = bars + 36, *acc_empty = bars + 38, *bm_full = bars + 40, *bm_empty = bars + 44;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 48);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int sg = 0;  // global row tile -> segment
  while (sg + 1 < a.nseg && int(blockIdx.x) >= a.seg[sg + 1].tile0) ++sg;
  const QGemmSeg &S = a.seg[sg];
  const int row0 = (int(blockIdx.x) - S.tile0) * QG_M;
  const int tt = blockIdx.y;
  const int nb = a.nb, nchunk = nb * QG_CPB;
  // split-K: this CTA's blocks are kbeg .. kbeg+nbl-1; loops below run over the local index kb
  // (ring slots and phases) and add kbeg where they address data
  const int kbeg = int(int64_t(nb) * blockIdx.z / gridDim.z);
  const int nbl = int(int64_t(nb) * (blockIdx.z + 1) / gridDim.z) - kbeg;
  constexpr int spb = 2;  // MMA steps (two 64-element chunks each) per 256-element block

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bm_full[i], 1);
      mbar_init(&bm_empty[i], 8);
    }
    for (int i = 0; i < BST; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0) {  // TMEM for two accumulators of N fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 8) {
    if (lane == 0)
      for (int kb = 0; kb < nbl; ++kb)
        for (int st = 0; st < spb; ++st) {
          const int gs = kb * spb + st, slot = gs & 1;
          mbar_spin(&a_empty[slot], ((gs >> 1) & 1) ^ 1, a.err);
          for (int h2 = 0; h2 < 2; ++h2) {
            const int gcc = kb * QG_CPB + 2 * st + h2;
            mbar_spin(&b_full[gcc & (BST - 1)], (gcc >> BLOG) & 1, a.err);
          }
          mbar_arrive_expect_tx(&a_full[slot], uint32_t(2 * QG_A_BYTES));
          for (int h2 = 0; h2 < 2; ++h2)
            tma_load_2d(sA + slot * QG_A_SLOT + h2 * QG_A_BYTES, &S.map[0], (kbeg + kb) * QK_K + (2 * st + h2) * QG_KC,
                        row0, &a_full[slot]);
        }
  } else if (warp == 10) {
    // its own warp: spinning lanes of one warp would take turns
    if (lane == 0)
      for (int kb = 0; kb < nbl; ++kb) {
        for (int c = 0; c < QG_CPB; ++c) {
          const int cc = kb * QG_CPB + c, s = cc & (BST - 1);
          mbar_spin(&b_empty[s], ((cc >> BLOG) & 1) ^ 1, a.err);
          mbar_arrive_expect_tx(&b_full[s], B_BYTES);
          bulk_g2s(sB + s * B_BYTES, a.bimg + (int64_t(tt) * nchunk + kbeg * QG_CPB + cc) * B_BYTES, B_BYTES,
                   &b_full[s]);
        }
        const int m = kb & 3;
        mbar_spin(&bm_empty[m], ((kb >> 2) & 1) ^ 1, a.err);  // epilogue done with block kb-4
        mbar_arrive_expect_tx(&bm_full[m], BM_BYTES);
        bulk_g2s(sBm + m * QG_META * TN, a.bmeta + (int64_t(tt) * nb + kbeg + kb) * QG_META * TN, BM_BYTES,
                 &bm_full[m]);
      }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(QG_M >> 4) << 24);
      for (int kb = 0; kb < nbl; ++kb) {
        const int b = kb & 1;
        mbar_spin(&acc_empty[b], ((kb >> 1) & 1) ^ 1, a.err);
        tc_fence_after();
        for (int st = 0; st < spb; ++st) {
          const int gs = kb * spb + st, slot = gs & 1;
          mbar_spin(&a_full[slot], (gs >> 1) & 1, a.err);  // A landed (after the step's B chunks)
          tc_fence_after();
          const uint32_t abase = smem_u32(sA + slot * QG_A_SLOT);
          for (int h2 = 0; h2 < 2; ++h2) {
            const int sb = (kb * QG_CPB + 2 * st + h2) & (BST - 1);
            const uint32_t bbase = smem_u32(sB + sb * B_BYTES);
#pragma unroll
            for (int k = 0; k < QG_KC / 16; ++k)
              tc_mma_f16(tmem + uint32_t(b * N), sw128_desc(abase + h2 * QG_A_BYTES + k * 32),
                         sw128_desc(bbase + k * 32), idesc, (st | h2 | k) != 0);
            tc_commit(&b_empty[sb]);
          }
          tc_commit(&a_empty[slot]);
        }
        tc_commit(&acc_full[b]);
      }
    }
  } else if (warp < 8) {
    // ---------------- warps 0-7: epilogue (thread = row r = TMEM lane r, tokens of half `part`)
    const int r = tid & (QG_M - 1), part = tid >> 7;
    constexpr int TH = TN / 2;
    const int tb = part * TH;
    float yacc[TH];
#pragma unroll
    for (int t = 0; t < TH; ++t) yacc[t] = 0.f;
    const uint32_t lane_base = tmem + (uint32_t(32 * (warp & 3)) << 16);
    for (int kb = 0; kb < nbl; ++kb) {
      const int b = kb & 1, ph = (kb >> 1) & 1;
      mbar_wait_bounded(&bm_full[kb & 3], (kb >> 2) & 1, a.err);
      warp_wait(&acc_full[b], ph, a.err);
      tc_fence_after();
      const float *bm = sBm + (kb & 3) * QG_META * TN;
      constexpr int G = TH < 16 ? TH : 16;
#pragma unroll
      for (int t0 = 0; t0 < TH; t0 += G) {
        uint32_t hi[G], lo[G];
        tmem_ld<G>(lane_base + uint32_t(b * N + tb + t0), hi);
        tmem_ld<G>(lane_base + uint32_t(b * N + TN + tb + t0), lo);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < G; ++i)
          yacc[t0 + i] += bm[tb + t0 + i] * (__uint_as_float(hi[i]) + __uint_as_float(lo[i]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[b]);
        mbar_arrive(&bm_empty[kb & 3]);
      }
    }
    const int row = row0 + r;
    const int tok0 = tt * TN + tb;
    if (a.part) {  // split-K partial of global row blockIdx.x*128 + r
      float *pp = a.part + (int64_t(blockIdx.z) * a.n_tok) * a.part_ld + int64_t(blockIdx.x) * QG_M + r;
#pragma unroll
      for (int t = 0; t < TH; ++t)
        if (tok0 + t < a.n_tok) pp[int64_t(tok0 + t) * a.part_ld] = yacc[t];
    } else if (row < S.rows) {
#pragma unroll
      for (int t = 0; t < TH; ++t)
        if (tok0 + t < a.n_tok) S.y[int64_t(tok0 + t) * S.ldy + row] = yacc[t];
    }
  }
  __syncwarp();  // producer / MMA warps: lanes 1-31 wait for lane 0 before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- K-quant GEMM, operand A in TMEM
// The K-quant variant keeps the dequantised weights out of shared memory: the dequantising warps
// write their fp16 A values straight into tensor memory (tcgen05.st; lane = weight row, 32-bit
// column = two consecutive K elements) and the MMA reads A from there (tcgen05.mma with an [a-tmem]
// operand).  That leaves shared memory to the activation ring, which then holds two 256-element
// blocks, so the next block's activations are in flight while the current one multiplies, and the
// per-block epilogue runs on warps of its own.
//   warps 0-7  : dequantise raw blocks into the TMEM A ring (thread = row r, half `part` of a chunk)
//   warp 8     : producer of the raw weight blocks (4-D tensor copies)
//   warp 9     : one thread issues tcgen05.mma (M=128, N=2*TN, K=16) into two TMEM accumulators
//   warp 10    : lane 0 copies each block's activation chunks (one bulk copy per block), lane 1 the
//                per-block activation metadata
// Bulk copies issued by one thread complete one after another (about 600 cycles each on B200
// whatever their size up to 64 KB), so every stream is one copy per block, each on its own thread.
//   warps 11-18: epilogue (thread = row r = TMEM lane r, tokens of half `part`), one block behind
// TMEM (512 columns): accumulators at [0, 2N), A ring of QK_AST steps x 64 columns from QK_ACOL0.
constexpr int QK_THREADS = 19 * 32;
constexpr int QK_AST = 4;      // A ring steps (Q4_K: two 64-element chunks; Q6_K: one chunk's two tiles)
constexpr int QK_ACOL0 = 256;  // first TMEM column of the A ring
constexpr int QK_TMEM_COLS = 512;

constexpr int QK_BST = 2;      // B ring: two 256-element blocks (QG_CPB chunks of 2*TN rows x 128 B each)

__host__ __device__ constexpr size_t qgemm_kq_smem(int tn) {
  return 1024 + size_t(QK_BST) * QG_CPB * 2 * tn * 128 + size_t(QG_RST) * QG_RAW_BYTES + 4 * QG_META * tn * 4 +
         2 * QG_M * 10 * 4 + 64 * 8;
}

template <int TN>
__global__ void __launch_bounds__(QK_THREADS, 1) qgemm_kq_kernel(const __grid_constant__ QGemmArgs a) {
  constexpr int N = 2 * TN;             // B rows: hi then lo per token
  constexpr int B_BYTES = N * 128;      // one B chunk
  constexpr int BB_BYTES = QG_CPB * B_BYTES;  // one block's chunks (contiguous in the image)
  constexpr int BM_BYTES = QG_META * TN * 4;
  static_assert(2 * N <= QK_ACOL0, "accumulators below the A ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *sB = smem;                                  // [QK_BST][BB_BYTES]
  uint8_t *sRaw = sB + QK_BST * BB_BYTES;              // [QG_RST][QG_RAW_BYTES]
  float *sBm = reinterpret_cast<float *>(sRaw + QG_RST * QG_RAW_BYTES);  // [4][9][TN]
  float *sRm = sBm + 4 * QG_META * TN;                 // [2][128][10]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sRm + 2 * QG_M * 10);
  uint64_t *a_full = bars, *a_empty = bars + 4, *b_full = bars + 8, *b_empty = bars + 24;
  uint64_t *raw_full = bars + 40, *raw_empty = bars + 42, *acc_full = bars + 44, *acc_empty = bars + 46;
  uint64_t *bm_full = bars + 48, *bm_empty = bars + 52, *rm_full = bars + 56;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 59);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int sg = 0;
  while (sg + 1 < a.nseg && int(blockIdx.x) >= a.seg[sg + 1].tile0) ++sg;
  const QGemmSeg &S = a.seg[sg];
  const int row0 = (int(blockIdx.x) - S.tile0) * QG_M;
  const int tt = blockIdx.y;
  const int nb = a.nb, nchunk = nb * QG_CPB;
  const int kbeg = int(int64_t(nb) * blockIdx.z / gridDim.z);
  const int nbl = int(int64_t(nb) * (blockIdx.z + 1) / gridDim.z) - kbeg;
  const bool q6 = S.type == T_Q6_K;
  const int raw_bytes = (QG_M / KQ_TILE) * kquant_rec_bytes(S.type);
  const int spb = q6 ? 4 : 2;   // MMA steps per 256-element block
  const int cps = q6 ? 1 : 2;   // 64-element chunks per step

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
      mbar_init(&bm_full[i], 1);
      mbar_init(&bm_empty[i], 8);
    }
    for (int i = 0; i < QK_BST; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 8);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
      mbar_init(&rm_full[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(QK_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue_raw = [&](int kb) {
    const int rs = kb & 1;
    mbar_arrive_expect_tx(&raw_full[rs], uint32_t(raw_bytes));
    tma_load_rec(sRaw + rs * QG_RAW_BYTES, &S.map[0], kbeg + kb, row0 / KQ_TILE, &raw_full[rs]);
  };
  // weights never depend on the previous kernel: start them before the dependency wait
  if (warp == 8 && lane == 0)
    for (int kb = 0; kb < nbl && kb < QG_RST; ++kb) issue_raw(kb);
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 8) {
    if (lane == 0)
      for (int kb = QG_RST; kb < nbl; ++kb) {
        mbar_spin(&raw_empty[kb & 1], ((kb >> 1) & 1) ^ 1, a.err);
        issue_raw(kb);
      }
  } else if (warp == 10) {
    if (lane == 0)
      for (int kb = 0; kb < nbl; ++kb) {
        const int s = kb & (QK_BST - 1);
        mbar_spin(&b_empty[s], ((kb / QK_BST) & 1) ^ 1, a.err);  // MMA done with block kb-2
        mbar_arrive_expect_tx(&b_full[s], BB_BYTES);
        bulk_g2s(sB + s * BB_BYTES, a.bimg + (int64_t(tt) * nchunk + (kbeg + kb) * QG_CPB) * B_BYTES, BB_BYTES,
                 &b_full[s]);
      }
    else if (lane == 1)
      for (int kb = 0; kb < nbl; ++kb) {
        const int m = kb & 3;
        mbar_spin(&bm_empty[m], ((kb >> 2) & 1) ^ 1, a.err);  // epilogue done with block kb-4
        mbar_arrive_expect_tx(&bm_full[m], BM_BYTES);
        bulk_g2s(sBm + m * QG_META * TN, a.bmeta + (int64_t(tt) * nb + kbeg + kb) * QG_META * TN, BM_BYTES,
                 &bm_full[m]);
      }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(QG_M >> 4) << 24);
      for (int kb = 0; kb < nbl; ++kb) {
        const int b = kb & 1, sbb = kb & (QK_BST - 1);
        mbar_spin(&acc_empty[b], ((kb >> 1) & 1) ^ 1, a.err);
        mbar_spin(&b_full[sbb], (kb / QK_BST) & 1, a.err);
        tc_fence_after();
        for (int st = 0; st < spb; ++st) {
          const int gs = kb * spb + st, slot = gs & (QK_AST - 1);
          mbar_spin(&a_full[slot], (gs / QK_AST) & 1, a.err);
          tc_fence_after();
          const uint32_t abase = tmem + uint32_t(QK_ACOL0 + 64 * slot);
          for (int h2 = 0; h2 < cps; ++h2) {
            const int c = q6 ? st : 2 * st + h2;  // chunk of the block
            const uint32_t bbase = smem_u32(sB + sbb * BB_BYTES + c * B_BYTES);
#pragma unroll
            for (int k = 0; k < QG_KC / 16; ++k) {
              tc_mma_f16_ts(tmem + uint32_t(b * N), abase + uint32_t(32 * h2 + 8 * k), sw128_desc(bbase + k * 32),
                            idesc, (st | h2 | k) != 0);
              if (q6)  // second Q6_K tile: sl*(q-32) (the first holds 16*sh*(q-32))
                tc_mma_f16_ts(tmem + uint32_t(b * N), abase + uint32_t(32 + 8 * k), sw128_desc(bbase + k * 32),
                              idesc, 1u);
            }
          }
          tc_commit(&a_empty[slot]);
        }
        tc_commit(&b_empty[sbb]);
        tc_commit(&acc_full[b]);
      }
    }
  } else if (warp < 8) {
    // ---------------- dequantise: thread = row r (TMEM lane r), half `part` of every chunk
    const int r = tid & (QG_M - 1), part = warp >> 2;
    const int rr = r & (KQ_TILE - 1);
    const uint32_t lane_addr = uint32_t(32 * (warp & 3)) << 16;
    for (int kb = 0; kb < nbl; ++kb) {
      const int rs = kb & 1, ph = (kb >> 1) & 1;
      mbar_wait_bounded(&raw_full[rs], ph, a.err);
      const uint8_t *raw = sRaw + rs * QG_RAW_BYTES;
      const uint8_t *rec = raw + (r / KQ_TILE) * (q6 ? REC_Q6_K : REC_Q4_K);
      uint32_t scw[4];
      if (!q6) {
        const uint4 hd = *reinterpret_cast<const uint4 *>(rec + 16 * rr);
        // get_scale_min_k4 (quants.rs:252-261) for sub-blocks 0..7
        scw[0] = hd.y & 0x3F3F3F3Fu;
        scw[1] = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
        scw[2] = scw[3] = 0u;
        if (part == 0) {
          // per-row block metadata for the epilogue (its buffer is free once block kb-2 is done)
          warp_wait(&acc_empty[rs], ph ^ 1, a.err);
          float *rm = sRm + (rs * QG_M + r) * 10;
          const uint32_t mn_lo = hd.z & 0x3F3F3F3Fu;
          const uint32_t mn_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
          rm[0] = h2f_bits(uint16_t(hd.x & 0xFFFF));
          rm[1] = h2f_bits(uint16_t(hd.x >> 16));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            rm[2 + j] = float((mn_lo >> (8 * j)) & 0xFF);
            rm[6 + j] = float((mn_hi >> (8 * j)) & 0xFF);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&rm_full[rs]);
        }
      } else {
        const uint4 sv = *reinterpret_cast<const uint4 *>(rec + 3072 + 16 * rr);
        scw[0] = sv.x;
        scw[1] = sv.y;
        scw[2] = sv.z;
        scw[3] = sv.w;
        if (part == 0) {
          warp_wait(&acc_empty[rs], ph ^ 1, a.err);
          sRm[(rs * QG_M + r) * 10] = h2f_bits(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * rr));
          __syncwarp();
          if (lane == 0) mbar_arrive(&rm_full[rs]);
        }
      }
      for (int st = 0; st < spb; ++st) {
        const int gs = kb * spb + st, slot = gs & (QK_AST - 1);
        warp_wait(&a_empty[slot], ((gs / QK_AST) & 1) ^ 1, a.err);
        tc_fence_after();
        const uint32_t acol = tmem + lane_addr + uint32_t(QK_ACOL0 + 64 * slot);
        for (int h2 = 0; h2 < cps; ++h2) {
          const int c = q6 ? st : 2 * st + h2;
          if (!q6) {
            // chunk c = elements 64c..64c+63: low nibbles of qs[32c..32c+31] (sub-block 2c) are
            // elements 0-31, high nibbles (sub-block 2c+1) elements 32-63.  This thread: bytes
            // 16*part..16*part+15, i.e. elements 16*part + [0,16) of each half; register j of a
            // half holds elements 2j, 2j+1 of those 16, TMEM column 16*h + 8*part + j of the chunk.
            const uint4 w = *reinterpret_cast<const uint4 *>(rec + 256 + 128 * rr + 16 * ((2 * c + part) ^ (rr & 7)));
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int sub = 2 * c + h;
              const uint32_t scv = ((sub < 4 ? scw[0] : scw[1]) >> (8 * (sub & 3))) & 0xFF;
              const __half2 s2 = __half2half2(__uint2half_rn(scv));
              const __half2 neg = __hneg2(__half2half2(__uint2half_rn(1024u * scv)));
              uint32_t o[8];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t nib = h ? (wv[q] >> 4) & 0x0F0F0F0Fu : wv[q] & 0x0F0F0F0Fu;
                // bytes [q0, 0x64, q1, 0x64] = fp16x2 (1024 + q0, 1024 + q1)
                o[2 * q] = half2_times(__byte_perm(nib, 0x64646464u, 0x4140), s2, neg);
                o[2 * q + 1] = half2_times(__byte_perm(nib, 0x64646464u, 0x4342), s2, neg);
              }
              tmem_st8(acol + uint32_t(32 * h2 + 16 * h + 8 * part), o);
            }
          } else {
            // chunk c: half n = c/2 of the block; h = 0: q1 (c even: ql low, qh bits 0-1) or q3
            // (c odd: ql high, qh bits 4-5); h = 1: q2 / q4 (ql + 32, qh bits 2-3 / 6-7).  This
            // thread: l = 16*part..16*part+15 of both.  sc*(q-32) = 16*sh*(q-32) + sl*(q-32) with
            // sc = 16*sh + sl, sl in [0, 15]: both products are exact in fp16 and go to the two A
            // tiles (TMEM columns 0-31 and 32-63 of the step).
            const int n = c >> 1, odd = c & 1;
            const uint4 qhv =
                *reinterpret_cast<const uint4 *>(rec + 2048 + 64 * rr + 16 * ((2 * n + part) ^ ((rr >> 1) & 3)));
            const uint32_t hwv[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
            const __half2 c1056 = __half2half2(__ushort_as_half(0x6420u));  // 1056.0
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 qlv =
                  *reinterpret_cast<const uint4 *>(rec + 128 * rr + 16 * ((4 * n + 2 * h + part) ^ (rr & 7)));
              const uint32_t lwv[4] = {qlv.x, qlv.y, qlv.z, qlv.w};
              const int shift_l = odd ? 4 : 0;
              const int shift_h = 2 * (2 * odd + h);
              const int si = 8 * n + 2 * (2 * odd + h) + part;
              const int wsel = si >> 2;
              const uint32_t sword = wsel == 0 ? scw[0] : wsel == 1 ? scw[1] : wsel == 2 ? scw[2] : scw[3];
              const int sc = int(int8_t((sword >> (8 * (si & 3))) & 0xFF));
              const __half2 shi = __half2half2(__int2half_rn(16 * (sc >> 4)));
              const __half2 slo = __half2half2(__int2half_rn(sc & 15));
              uint32_t oh[8], ol[8];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t qw = ((lwv[q] >> shift_l) & 0x0F0F0F0Fu) | (((hwv[q] >> shift_h) & 0x03030303u) << 4);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const uint32_t pk = __byte_perm(qw, 0x64646464u, e ? 0x4342 : 0x4140);
                  const __half2 u = __hsub2(*reinterpret_cast<const __half2 *>(&pk), c1056);  // q - 32, exact
                  const __half2 ph2 = __hmul2(u, shi), pl2 = __hmul2(u, slo);
                  oh[2 * q + e] = *reinterpret_cast<const uint32_t *>(&ph2);
                  ol[2 * q + e] = *reinterpret_cast<const uint32_t *>(&pl2);
                }
              }
              tmem_st8(acol + uint32_t(16 * h + 8 * part), oh);
              tmem_st8(acol + uint32_t(32 + 16 * h + 8 * part), ol);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[slot]);  // one arrival per warp
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[rs]);
    }
  } else {
    // ---------------- warps 11-18: epilogue (thread = row r = TMEM lane r, tokens of half `part`)
    const int e = warp - 11;
    const int r = 32 * (warp & 3) + lane, part = e >> 2;
    constexpr int TH = TN / 2;
    const int tb = part * TH;
    float yacc[TH];
#pragma unroll
    for (int t = 0; t < TH; ++t) yacc[t] = 0.f;
    const uint32_t lane_base = tmem + (uint32_t(32 * (warp & 3)) << 16);
    for (int kb = 0; kb < nbl; ++kb) {
      const int b = kb & 1, ph = (kb >> 1) & 1;
      mbar_wait_bounded(&bm_full[kb & 3], (kb >> 2) & 1, a.err);
      warp_wait(&rm_full[b], ph, a.err);
      warp_wait(&acc_full[b], ph, a.err);
      tc_fence_after();
      const float *rm = sRm + (b * QG_M + r) * 10;
      const float *bm = sBm + (kb & 3) * QG_META * TN;
      const float d = rm[0];
      const float dmin = q6 ? 0.f : rm[1];
      float mj[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mj[j] = q6 ? 0.f : rm[2 + j];
      constexpr int G = TH < 16 ? TH : 16;
#pragma unroll
      for (int t0 = 0; t0 < TH; t0 += G) {
        uint32_t hi[G], lo[G];
        tmem_ld<G>(lane_base + uint32_t(b * N + tb + t0), hi);
        tmem_ld<G>(lane_base + uint32_t(b * N + TN + tb + t0), lo);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < G; i += 4) {
          const int t = tb + t0 + i;  // four tokens: their scales and sub-block sums as 16-byte loads
          const float4 s4 = *reinterpret_cast<const float4 *>(bm + t);
          float4 mn = make_float4(0.f, 0.f, 0.f, 0.f);
          if (!q6) {  // Q4_K mins: sum over the sub-blocks of m_j * (sum of x over sub-block j)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 qv = *reinterpret_cast<const float4 *>(bm + (1 + j) * TN + t);
              mn.x += mj[j] * qv.x;
              mn.y += mj[j] * qv.y;
              mn.z += mj[j] * qv.z;
              mn.w += mj[j] * qv.w;
            }
          }
          const float sv[4] = {s4.x, s4.y, s4.z, s4.w}, mv[4] = {mn.x, mn.y, mn.z, mn.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float v = __uint_as_float(hi[i + u]) + __uint_as_float(lo[i + u]);
            yacc[t0 + i + u] += (d * sv[u]) * v - dmin * mv[u];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[b]);
        mbar_arrive(&bm_empty[kb & 3]);
      }
    }
    const int row = row0 + r;
    const int tok0 = tt * TN + tb;
    if (a.part) {  // split-K partial of global row blockIdx.x*128 + r
      float *pp = a.part + (int64_t(blockIdx.z) * a.n_tok) * a.part_ld + int64_t(blockIdx.x) * QG_M + r;
#pragma unroll
      for (int t = 0; t < TH; ++t)
        if (tok0 + t < a.n_tok) pp[int64_t(tok0 + t) * a.part_ld] = yacc[t];
    } else if (row < S.rows) {
#pragma unroll
      for (int t = 0; t < TH; ++t)
        if (tok0 + t < a.n_tok) S.y[int64_t(tok0 + t) * S.ldy + row] = yacc[t];
    }
  }
  __syncwarp();  // single-lane roles: lanes 1-31 wait for lane 0 before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QK_TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- operand B preparation
// One CTA per token (rows of the padded token range; padding tokens write zeros).  Warp w takes
// 256-element blocks w, w+8, ...; lane l holds elements 8l..8l+7 of the block.  The optional
// prologue steps mirror the GEMV prologue (residual add + RMSNorm of the next op) and the GeGLU
// of the gate/up pair (real_math.rs:79-85).
constexpr int BP_WARPS = 8;

__device__ __forceinline__ void ld8(const float *p, float (&v)[8]) {
  const float4 f0 = *reinterpret_cast<const float4 *>(p), f1 = *reinterpret_cast<const float4 *>(p + 4);
  v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
  v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
}

__device__ __forceinline__ float gelu_tanh_mul_b(float v, float u) {
  const float k = 0.7978845608028654f;
  const float inner = k * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner)) * u;
}

__global__ void __launch_bounds__(BP_WARPS * 32) gemm_bprep_kernel(GemmPrologue P, int64_t K, int n_tok, int TN,
                                                                  uint8_t *__restrict__ img,
                                                                  float *__restrict__ meta) {
  __shared__ float red[64];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = int(K / QK_K), nchunk = nb * QG_CPB, N = 2 * TN;
  const int tt = t / TN, tl = t % TN;
  const bool valid = t < n_tok;
  const int64_t roff = int64_t(t) * K;
  float s1 = 1.f, s2 = 1.f;
  auto value8 = [&](int b, int step, float (&v)[8]) {
    const int col = b * QK_K + lane * 8;
    if (P.gate) {  // GeGLU of the gate/up outputs
      float g[8], u[8];
      ld8(P.gate + roff + col, g);
      ld8(P.up + roff + col, u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = gelu_tanh_mul_b(g[e], u[e]);
      return;
    }
    ld8((P.mode == 0 ? P.x : P.a) + roff + col, v);
    if (P.mode == 0 || step == 0) return;
    if (P.mode == 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = v[e] * s1;
    } else {
      float wp[8], rs[8];
      if (P.w_post) ld8(P.w_post + col, wp);
      ld8(P.resid_in + roff + col, rs);
      const float sc = P.scale ? P.scale[0] : 1.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = resid_add(v[e], s1, P.w_post, wp[e], rs[e], P.scale, sc);
    }
    if (step == 1 || !P.w_next) return;
    float wn[8];
    ld8(P.w_next + col, wn);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (v[e] * s2) * wn[e];
  };
  // the token's sum of v^2 after `step` steps, in the residual-stream norm order (row_sumsq)
  auto cta_sumsq = [&](int step, bool store_resid) {
    return row_sumsq<BP_WARPS>(nb, red, [&](int b, float (&v)[8]) {
      value8(b, step, v);
      if (store_resid) {
        float *o = P.resid_out + roff + b * QK_K + lane * 8;
        *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4 *>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
      }
    });
  };
  if (valid && !P.gate && P.mode != 0) {
    if (P.mode == 1 || P.w_post) s1 = 1.0f / sqrtf(cta_sumsq(0, false) / float(K) + P.eps);
    if (P.mode == 2 && (P.w_next || P.resid_out)) {
      const float ss = cta_sumsq(1, P.resid_out != nullptr);
      s2 = 1.0f / sqrtf(ss / float(K) + P.eps);
    }
  }
  for (int b = warp; b < nb; b += BP_WARPS) {
    float v[8];
    if (valid) {
      value8(b, 2, v);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    float m = 0.f, ssum = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      m = fmaxf(m, fabsf(v[e]));
      ssum += v[e];
    }
    m = warp_max(m);
    int E = int((__float_as_uint(m) >> 23) & 0xFF) - 126;  // m < 2^E
    if (E < -100) E = -100;
    const float up = __uint_as_float(uint32_t(127 + 15 - E) << 23);  // 2^(15-E): |x * up| < 2^15
    const float s = __uint_as_float(uint32_t(127 - 15 + E) << 23);   // 2^(E-15)
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      __half h[2], l[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float xs = v[2 * e2 + u] * up;
        h[u] = __float2half_rn(xs);
        l[u] = __float2half_rn(xs - __half2float(h[u]));
      }
      const __half2 h2 = __halves2half2(h[0], h[1]), l2 = __halves2half2(l[0], l[1]);
      hw[e2] = *reinterpret_cast<const uint32_t *>(&h2);
      lw[e2] = *reinterpret_cast<const uint32_t *>(&l2);
    }
    const int cc = b * QG_CPB + (lane >> 3), j = lane & 7;
    uint8_t *chunk = img + (int64_t(tt) * nchunk + cc) * (N * 128);
    *reinterpret_cast<uint4 *>(chunk + sw128_off(tl, j)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(chunk + sw128_off(TN + tl, j)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    // fp32 sums over the 32-element sub-blocks (4 lanes each), fixed order
    ssum += __shfl_xor_sync(0xFFFFFFFFu, ssum, 1);
    ssum += __shfl_xor_sync(0xFFFFFFFFu, ssum, 2);
    float *mt = meta + (int64_t(tt) * nb + b) * QG_META * TN;
    if (lane == 0) mt[tl] = valid ? s : 0.f;
    if ((lane & 3) == 0) mt[(1 + (lane >> 2)) * TN + tl] = ssum;
  }
}

// act = gelu_tanh(gate) * up, elementwise (real_math.rs:79-85)
__global__ void geglu_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ out,
                             int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = gelu_tanh_mul_b(g[i], u[i]);
}

cudaError_t geglu(const float *gate, const float *up, float *out, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 8 * num_sms()) blocks = 8 * num_sms();
  return launch_pdl(geglu_kernel, dim3(unsigned(blocks)), dim3(256), 0, st, gate, up, out, n);
}

// ---------------------------------------------------------------- host side
// Tiled K-quant records as a 4D uint8 view [tile][block][rec/row_x][row_x] (row_x = 256 B for Q4_K,
// 240 B for Q6_K), box = one block's records of 8 tiles (128 weight rows); tiles past the end read
// as zeros.
static bool make_map_rec(CUtensorMap *m, const void *base, int type, int64_t rows, int nb) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int rec = kquant_rec_bytes(type);
  const int row_x = type == T_Q4_K ? 256 : 240;
  const cuuint64_t ntiles = cuuint64_t((rows + KQ_TILE - 1) / KQ_TILE);
  const cuuint64_t dims[4] = {cuuint64_t(row_x), cuuint64_t(rec / row_x), cuuint64_t(nb), ntiles};
  const cuuint64_t strides[3] = {cuuint64_t(row_x), cuuint64_t(rec), cuuint64_t(rec) * nb};
  const cuuint32_t box[4] = {cuuint32_t(row_x), cuuint32_t(rec / row_x), 1, cuuint32_t(QG_M / KQ_TILE)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp16 rows [rows][K]: box 64 elements (128 B) x 128 rows, 128-byte swizzle, i.e. one A tile in
// exactly the shared-memory layout the MMA descriptors describe
static bool make_map_f16(CUtensorMap *m, const void *base, int64_t K, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(K * 2)};
  const cuuint32_t box[2] = {cuuint32_t(QG_KC), cuuint32_t(QG_M)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct MapKey {
  const void *p;
  int type;
  int64_t rows, K;
  bool operator==(const MapKey &o) const { return p == o.p && type == o.type && rows == o.rows && K == o.K; }
};
struct MapKeyHash {
  size_t operator()(const MapKey &k) const {
    return std::hash<const void *>()(k.p) ^ (size_t(k.rows) * 131 + size_t(k.K) * 7 + size_t(k.type));
  }
};
struct MapSet {
  CUtensorMap map[4];
};

static bool weight_maps(int type, const void *w, int64_t rows, int64_t K, CUtensorMap (&out)[4]) {
  static std::mutex mu;
  static std::unordered_map<MapKey, MapSet, MapKeyHash> cache;
  const MapKey key{w, type, rows, K};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it == cache.end()) {
    MapSet s;
    memset(&s, 0, sizeof(s));
    const int nb = int(K / QK_K);
    const bool ok = type == T_F16 ? make_map_f16(&s.map[0], w, K, rows) : make_map_rec(&s.map[0], w, type, rows, nb);
    if (!ok) return false;
    it = cache.emplace(key, s).first;
  }
  memcpy(out, it->second.map, sizeof(out));
  return true;
}

static size_t qgemm_f16_smem(int TN) {
  return 1024 + size_t(QG_AST) * QG_A_BYTES + size_t(qg_b_slots(TN)) * 2 * TN * 128 + 4 * QG_META * TN * 4 + 50 * 8;
}

// Token-tile width: the largest of 64/32/16/8 that still gives every SM a CTA, else 8.
// Token-tile width: every tile costs a CTA about the same time (its block pipeline does not speed
// up with fewer tokens), so use the widest tile the tokens fill: fewest CTAs and waves.
static int pick_tn(int64_t n_tok) { return n_tok <= 8 ? 8 : n_tok <= 16 ? 16 : n_tok <= 32 ? 32 : 64; }

// K splits: shapes with few row and token tiles (o, down: 20 row tiles) split K so the grid still
// covers the SMs; each split keeps at least two 256-element blocks.
static int pick_splits(int64_t ctas, int nb) {
  if (ctas * 2 >= num_sms()) return 1;
  int64_t s = num_sms() / ctas;
  if (s > nb / 2) s = nb / 2;
  return s < 1 ? 1 : int(s);
}

// Largest split-K partial buffer: splits x row tiles x token tiles <= SMs, tokens per tile <= 64.
static size_t qgemm_part_bytes_max() { return size_t(num_sms()) * 64 * QG_M * 4 + 256; }

size_t qgemm_scratch_bytes(int64_t n_tok, int64_t K) {
  const int64_t tpad = (n_tok + 63) / 64 * 64;  // the widest token tile pads the most
  const int64_t nb = K / QK_K;
  return size_t(tpad) * size_t(K) * 4 + 256 + size_t(tpad) * nb * QG_META * 4 + 256 + qgemm_part_bytes_max() + 1024;
}

struct QGemmOutMap {
  float *y[QG_MAX_SEG];
  int64_t ldy[QG_MAX_SEG];
  int rows[QG_MAX_SEG];
  int row0[QG_MAX_SEG];  // first global row (tile0 * 128) of each segment
  int nseg;
};

// y[t][row] = sum over splits of the partials, in split order (deterministic)
__global__ void splitk_reduce_kernel(const float *__restrict__ part, int nsplit, int n_tok, int64_t part_ld,
                                     QGemmOutMap m) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = int64_t(n_tok) * part_ld;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / part_ld);
    const int gr = int(i % part_ld);
    int sg = 0;
    while (sg + 1 < m.nseg && gr >= m.row0[sg + 1]) ++sg;
    const int lr = gr - m.row0[sg];
    if (lr >= m.rows[sg]) continue;
    float v = 0.f;
    for (int z = 0; z < nsplit; ++z) v += part[(int64_t(z) * n_tok + t) * part_ld + gr];
    m.y[sg][int64_t(t) * m.ldy[sg] + lr] = v;
  }
}

bool qgemm_supported(int type, int64_t K) {
  return (type == T_Q4_K || type == T_Q6_K || type == T_F16) && K % QK_K == 0 && K / QK_K <= QG_MAX_NB &&
         encode_fn() != nullptr;
}

template <int TN>
static cudaError_t launch_qgemm_kq_t(QGemmArgs &a, int row_tiles, int nsplit, cudaStream_t st) {
  constexpr size_t smem = qgemm_kq_smem(TN);
  cudaError_t e = cudaFuncSetAttribute(qgemm_kq_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(qgemm_kq_kernel<TN>, dim3(unsigned(row_tiles), unsigned(a.n_ttiles), unsigned(nsplit)),
                    dim3(QK_THREADS), smem, st, a);
}

template <int TN>
static cudaError_t launch_qgemm_f16_t(QGemmArgs &a, int row_tiles, int nsplit, cudaStream_t st) {
  const size_t smem = qgemm_f16_smem(TN);
  cudaError_t e = cudaFuncSetAttribute(qgemm_f16_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(qgemm_f16_kernel<TN>, dim3(unsigned(row_tiles), unsigned(a.n_ttiles), unsigned(nsplit)),
                    dim3(QG_THREADS), smem, st, a);
}

cudaError_t qgemm(const QGemmOut *outs, int nseg, int64_t K, const GemmPrologue &pro, int64_t n_tok, void *scratch,
                  size_t scratch_bytes, cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (nseg < 1 || nseg > QG_MAX_SEG || K % QK_K || K / QK_K > QG_MAX_NB) return cudaErrorInvalidValue;
  if (scratch_bytes < qgemm_scratch_bytes(n_tok, K)) return cudaErrorInvalidValue;
  QGemmArgs a;
  memset(&a, 0, sizeof(a));
  a.nseg = nseg;
  a.nb = int(K / QK_K);
  a.n_tok = int(n_tok);
  a.err = device_error_ptr();
  int tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    const QGemmOut &o = outs[i];
    if ((o.type != T_Q4_K && o.type != T_Q6_K && o.type != T_F16) || !o.w || !o.y || o.rows <= 0)
      return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(o.w) % 16 || (o.type == T_F16) != (outs[0].type == T_F16))
      return cudaErrorInvalidValue;
    QGemmSeg &s = a.seg[i];
    if (!weight_maps(o.type, o.w, o.rows, K, s.map)) return cudaErrorInvalidValue;
    s.y = o.y;
    s.ldy = o.ldy;
    s.rows = int(o.rows);
    s.type = o.type;
    s.tile0 = tiles;
    tiles += int((o.rows + QG_M - 1) / QG_M);
  }
  const int TN = pick_tn(n_tok);
  a.n_ttiles = int((n_tok + TN - 1) / TN);
  const int nsplit = pick_splits(int64_t(tiles) * a.n_ttiles, a.nb);
  const int64_t tpad = int64_t(a.n_ttiles) * TN;
  uint8_t *img = static_cast<uint8_t *>(scratch);
  const size_t img_bytes = size_t(tpad) * size_t(K) * 4;
  float *meta = reinterpret_cast<float *>(img + (img_bytes + 255) / 256 * 256);
  const size_t meta_bytes = size_t(tpad) * a.nb * QG_META * 4;
  a.bimg = img;
  a.bmeta = meta;
  if (nsplit > 1) {
    a.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(meta) + (meta_bytes + 255) / 256 * 256);
    a.part_ld = int64_t(tiles) * QG_M;
    if (size_t(nsplit) * n_tok * a.part_ld * 4 > qgemm_part_bytes_max()) return cudaErrorInvalidValue;
  }
  cudaError_t e = launch_pdl(gemm_bprep_kernel, dim3(unsigned(tpad)), dim3(BP_WARPS * 32), 0, st, pro, K, int(n_tok),
                             TN, img, meta);
  if (e != cudaSuccess) return e;
  // K-quant segments: operand A in tensor memory; fp16 segments: A by tensor copies (not mixed)
  const bool kquant = outs[0].type != T_F16;
  switch (TN) {
    case 64: e = kquant ? launch_qgemm_kq_t<64>(a, tiles, nsplit, st) : launch_qgemm_f16_t<64>(a, tiles, nsplit, st); break;
    case 32: e = kquant ? launch_qgemm_kq_t<32>(a, tiles, nsplit, st) : launch_qgemm_f16_t<32>(a, tiles, nsplit, st); break;
    case 16: e = kquant ? launch_qgemm_kq_t<16>(a, tiles, nsplit, st) : launch_qgemm_f16_t<16>(a, tiles, nsplit, st); break;
    default: e = kquant ? launch_qgemm_kq_t<8>(a, tiles, nsplit, st) : launch_qgemm_f16_t<8>(a, tiles, nsplit, st); break;
  }
  if (e != cudaSuccess || nsplit == 1) return e;
  QGemmOutMap m = {};
  m.nseg = nseg;
  for (int i = 0; i < nseg; ++i) {
    m.y[i] = a.seg[i].y;
    m.ldy[i] = a.seg[i].ldy;
    m.rows[i] = a.seg[i].rows;
    m.row0[i] = a.seg[i].tile0 * QG_M;
  }
  const int64_t total = n_tok * a.part_ld;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
  return launch_pdl(splitk_reduce_kernel, dim3(unsigned(blocks)), dim3(256), 0, st, (const float *)a.part, nsplit,
                    int(n_tok), a.part_ld, m);
}

}  // namespace sfc
