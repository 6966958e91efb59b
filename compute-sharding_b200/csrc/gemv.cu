// gemv.cu — dequant-fused K-quant GEMV for decode (1 or 2 tokens per pass).
//
// Replaces the reference's row-dot hot loop (crates/stage-forward-lab/src/quants.rs:1801-1909
// for Q4_K, :2594-2688 for Q6_K) driven by real_math.rs:398-733 (matmul_quantized_many_refs_range)
// and the gate/up pair path real_math.rs:1584-1800 + GeGLU real_forward.rs:1716-1730.
//
// Design (B200):
//  * Work unit = (16-row tile, 256-element block).  The units of all output rows (tile-major,
//    block fastest) are split evenly over the CTAs, so every SM streams the same number of weight
//    bytes whatever the row count.  A tile cut between two CTAs is finished by whichever of the
//    two arrives second: both write their partial row sums to a small global buffer and the
//    second sums them in a fixed order (deterministic).
//  * Weights are in the tiled device layout (common.cuh): a stage = one tile's run of blocks is one
//    contiguous range, so one producer warp streams it HBM -> shared memory with a single bulk
//    async copy (cp.async.bulk, the TMA engine) per matrix into an mbarrier ring.  Weights never
//    depend on the previous kernel, so the copies are issued before the dependency wait.
//  * 15 consumer warps run the quant x activation products as exact integer MMAs on the tensor
//    pipe (mma.sync m16n8k32, u8 x s8 -> s32): A = 16 rows x 32 quants of one sub-block, B = the
//    activation split exactly into three signed 8-bit digit planes per 256-block,
//    x = 2^e (a*65536 + b*256 + c) with |x| < 2^(e+22), one plane per MMA column.  Sub-block
//    scales multiply the exact int32 results; rounding happens only in the final fp32 combine
//    (more accurate than the reference's fp32 running sum, and not the lossy 8-bit activation
//    quantization of the reference's GPU path, quantize_q8_1).
//  * Q6_K: one MMA covers a 32-quant chunk with its two 16-element scale groups in separate
//    columns (group-0 digit planes in columns 0-2, group-1 in 3-5), and the accumulator input
//    carries -32 x (digit sums), so the MMA returns the exact sum of (q - 32) x digits.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "gemv_core.cuh"

namespace sfc {

__device__ unsigned g_device_error = 0;
long long g_kernel_launches = 0;
// Boundary buffers for callers that pass none.  The counters start at zero and every launch
// leaves them at zero (the second arrival resets its slot).
__device__ unsigned g_gemv_cnt[GEMV_DEFAULT_SPLIT_CTAS];
__device__ float g_gemv_part[GEMV_DEFAULT_SPLIT_CTAS * GEMV_SPLIT_SLOT];

// Segments let one launch cover several matrices with the same K (q, k and v of a layer).
// TYPE: the weight type of every segment (T_Q4_K / T_Q6_K), or 0 for a mix (checked per unit).
template <int NMAT, int T, int TYPE, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) qgemv_kernel(const QGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float pro_red[GEMV_MAX_T][16];
  __shared__ int s_tdone[2];                 // finished units of the shared tiles
  __shared__ int s_sdone[GEMV_MAX_STAGES];  // finished units of the stage in each ring slot
  __shared__ int s_nstages;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = int(blockIdx.x);
  CtaTiles ct;
  {
    const int u0 = cta * a.uq + (cta < a.ur ? cta : a.ur);
    ct.init(u0, u0 + a.uq + (cta < a.ur ? 1 : 0), a.nb);
  }
  uint64_t *full = reinterpret_cast<uint64_t *>(smem), *empty = full + GEMV_MAX_STAGES;
  float *red = reinterpret_cast<float *>(smem + a.red_off);  // [local tile][16][NMAT][T][nb]
  const XSmem X = x_view(smem + a.x_off, a.nb, T);
  uint8_t *ring = smem + a.ring_off;
  GemvStage *tab = reinterpret_cast<GemvStage *>(smem + a.tab_off);  // the CTA's stages in order

  if (tid == 0) {
    for (int i = 0; i < a.nstage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // arrived by the warp that finishes the stage's last unit
      s_sdone[i] = 0;
    }
    fence_mbar_init();
    s_tdone[0] = s_tdone[1] = 0;
  }
  __syncthreads();

  if (warp == CW) {  // producer: weights never depend on the previous kernel, so no dependency wait
    produce_walk<NMAT>(a, ct, ring, full, empty, lane);
    return;
  }
  if (tid == 0) s_nstages = build_stage_table(a, ct, tab);  // the consumers' copy of the same walk
  consumer_bar<CW>();
  pdl_wait();
  pdl_launch_dependents();
  build_x<T, CW>(a.pro, a.nb, cta, X, pro_red, warp, lane);
  run_units<NMAT, T, TYPE, CW>(a, ct, tab, RingPos{0, 0}, ring, full, empty, s_sdone, X, red, s_tdone, cta, warp,
                               lane);
  if (ct.count == ct.np) return;
  consumer_bar<CW>();
  finish_owned<NMAT, T, CW>(a, ct, red, tid);
}

// ---------------------------------------------------------------- float-weight GEMV
// F32 / F16 / BF16 rows: one warp per row, x read through L1.  Used for small F32 test
// packs and non-quantized projections (real_math.rs:106-141, quants.rs:1317-1330).
template <int TYPE, int NMAT>
__global__ void fgemv_kernel(const void *w0, const void *w1, const float *__restrict__ x, float *__restrict__ y,
                             int64_t rows, int64_t K, int T, int64_t ldy) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    for (int t = 0; t < T; ++t) {
      float acc[2] = {0.f, 0.f};
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const void *w = m == 0 ? w0 : w1;
        float a = 0.f;
        for (int64_t k = lane; k < K; k += 32) {
          float wv;
          if (TYPE == T_F32)
            wv = reinterpret_cast<const float *>(w)[r * K + k];
          else if (TYPE == T_F16)
            wv = __half2float(reinterpret_cast<const __half *>(w)[r * K + k]);
          else
            wv = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(w)[r * K + k]) << 16);
          a += wv * x[int64_t(t) * K + k];
        }
        acc[m] = warp_sum(a);
      }
      if (lane == 0) y[int64_t(t) * ldy + r] = NMAT == 2 ? gelu_tanh_mul(acc[0], acc[1]) : acc[0];
    }
  }
}

// ---------------------------------------------------------------- dequantization (bit-exact)
// quants.rs:181-208 (Q4_K) and :210-249 (Q6_K), GGUF layout in, f32 out.  Explicit
// __fmul_rn/__fsub_rn forbid FMA contraction so each value is rounded exactly as the
// reference computes it.
__global__ void dequant_kernel(int type, const uint8_t *__restrict__ w, int64_t n_blocks, float *__restrict__ out) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one thread per 32 elements
  const int64_t b = gid >> 3;
  const int part = int(gid & 7);
  if (b >= n_blocks) return;
  float *o = out + b * QK_K;
  if (type == T_Q4_K) {
    const uint8_t *bp = w + b * BLOCK_Q4_K;
    const float d = h2f_bits(uint16_t(bp[0] | (bp[1] << 8)));
    const float dmin = h2f_bits(uint16_t(bp[2] | (bp[3] << 8)));
    const uint8_t *q = bp + 4;
    const int jgrp = part >> 1, hi = part & 1, is = 2 * jgrp + hi;
    int sc, m;
    if (is < 4) {
      sc = q[is] & 63;
      m = q[is + 4] & 63;
    } else {
      sc = (q[is + 4] & 0x0F) | ((q[is - 4] >> 6) << 4);
      m = (q[is + 4] >> 4) | ((q[is] >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, float(sc)), m1 = __fmul_rn(dmin, float(m));
    const uint8_t *qs = bp + 16 + jgrp * 32;
    for (int l = 0; l < 32; ++l) {
      const int qv = hi ? (qs[l] >> 4) : (qs[l] & 0x0F);
      o[jgrp * 64 + hi * 32 + l] = __fsub_rn(__fmul_rn(d1, float(qv)), m1);
    }
  } else if (type == T_Q6_K) {
    const uint8_t *bp = w + b * BLOCK_Q6_K;
    const float d = h2f_bits(uint16_t(bp[208] | (bp[209] << 8)));
    const int half = part >> 2, grp = part & 3;  // 128-element half, 32-element group
    const uint8_t *ql = bp + half * 64, *qh = bp + 128 + half * 32;
    const int8_t *sc = reinterpret_cast<const int8_t *>(bp + 192 + half * 8);
    for (int l = 0; l < 32; ++l) {
      const uint8_t hb = qh[l];
      int q;
      switch (grp) {
        case 0: q = (ql[l] & 0x0F) | (((hb >> 0) & 3) << 4); break;
        case 1: q = (ql[32 + l] & 0x0F) | (((hb >> 2) & 3) << 4); break;
        case 2: q = (ql[l] >> 4) | (((hb >> 4) & 3) << 4); break;
        default: q = (ql[32 + l] >> 4) | (((hb >> 6) & 3) << 4); break;
      }
      o[half * 128 + grp * 32 + l] = __fmul_rn(__fmul_rn(d, float(sc[l / 16 + 2 * grp])), float(q - 32));
    }
  }
}

// GGUF Q4_K / Q6_K rows -> tiled device records (common.cuh).  One thread per (tile, block, row of
// the tile); rows past the end of the tensor are zero.
__global__ void repack_kquant_kernel(int type, const uint8_t *__restrict__ src, int64_t rows, int nb,
                                     uint8_t *__restrict__ dst) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t ntiles = (rows + KQ_TILE - 1) / KQ_TILE;
  if (gid >= ntiles * nb * KQ_TILE) return;
  const int r = int(gid % KQ_TILE);
  const int64_t rec = gid / KQ_TILE;  // tile * nb + block
  const int b = int(rec % nb);
  const int64_t row = (rec / nb) * KQ_TILE + r;
  const bool valid = row < rows;
  if (type == T_Q4_K) {
    const uint8_t *s = src + (row * nb + b) * BLOCK_Q4_K;
    uint8_t *o = dst + rec * REC_Q4_K;
    for (int i = 0; i < 16; ++i) o[16 * r + i] = valid ? s[i] : 0;
    for (int j = 0; j < 8; ++j)
      for (int i = 0; i < 16; ++i) o[256 + 128 * r + 16 * (j ^ (r & 7)) + i] = valid ? s[16 + 16 * j + i] : 0;
  } else {
    const uint8_t *s = src + (row * nb + b) * BLOCK_Q6_K;
    uint8_t *o = dst + rec * REC_Q6_K;
    for (int j = 0; j < 8; ++j)
      for (int i = 0; i < 16; ++i) o[128 * r + 16 * (j ^ (r & 7)) + i] = valid ? s[16 * j + i] : 0;
    for (int j = 0; j < 4; ++j)
      for (int i = 0; i < 16; ++i) o[2048 + 64 * r + 16 * (j ^ ((r >> 1) & 3)) + i] = valid ? s[128 + 16 * j + i] : 0;
    for (int i = 0; i < 16; ++i) o[3072 + 16 * r + i] = valid ? s[192 + i] : 0;
    o[3328 + 2 * r] = valid ? s[208] : 0;
    o[3329 + 2 * r] = valid ? s[209] : 0;
  }
}

// ---------------------------------------------------------------- host side
int device_row_bytes(int type, int64_t K) {
  if (K <= 0) return -1;
  switch (type) {
    case T_F32: return int(K * 4);
    case T_F16:
    case T_BF16: return int(K * 2);
    case T_Q4_K: return K % QK_K ? -1 : int(K / QK_K * BLOCK_Q4_K);
    case T_Q6_K: return K % QK_K ? -1 : int(K / QK_K * BLOCK_Q6_K);
  }
  return -1;
}

int gguf_row_bytes(int type, int64_t K) { return device_row_bytes(type, K); }

int64_t device_tensor_bytes(int type, int64_t rows, int64_t K) {
  if (rows < 0) return -1;
  if (type == T_Q4_K || type == T_Q6_K) {
    if (K <= 0 || K % QK_K) return -1;
    return (rows + KQ_TILE - 1) / KQ_TILE * (K / QK_K) * kquant_rec_bytes(type);
  }
  const int rb = device_row_bytes(type, K);
  return rb < 0 ? -1 : int64_t(rb) * rows;
}

// Address of this module's device error word on the current device (cached per device).
unsigned *device_error_ptr() {
  static unsigned *cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    unsigned *p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_device_error) == cudaSuccess) cache[dev] = p;
  }
  return cache[dev];
}


constexpr int GEMV_STAGE_TARGET = 24 * 1024;
constexpr int GEMV_SMEM_WIDE = 227 * 1024 - 1024;  // dynamic shared memory (static use is < 1 KB)
constexpr int GEMV_RED_TARGET = 32 * 1024;

size_t gemv_split_bytes(int max_ctas) {
  return size_t(max_ctas) * sizeof(unsigned) + size_t(max_ctas) * GEMV_SPLIT_SLOT * sizeof(float) + 256;
}

GemvSplit gemv_split_view(void *base, int max_ctas) {
  GemvSplit s;
  s.cnt = static_cast<unsigned *>(base);
  const size_t off = (size_t(max_ctas) * sizeof(unsigned) + 255) / 256 * 256;
  s.part = reinterpret_cast<float *>(static_cast<char *>(base) + off);
  s.max_ctas = max_ctas;
  return s;
}

static GemvSplit default_split() {
  static GemvSplit cache[64] = {};
  GemvSplit none = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return none;
  if (!cache[dev].cnt) {
    void *c = nullptr, *p = nullptr;
    if (cudaGetSymbolAddress(&c, g_gemv_cnt) != cudaSuccess || cudaGetSymbolAddress(&p, g_gemv_part) != cudaSuccess)
      return none;
    cache[dev].cnt = static_cast<unsigned *>(c);
    cache[dev].part = static_cast<float *>(p);
    cache[dev].max_ctas = GEMV_DEFAULT_SPLIT_CTAS;
  }
  return cache[dev];
}

template <int NMAT, int T, int TYPE, int CW>
static cudaError_t launch_qgemv_t(QGemvArgs a, const GemvSplit &sp, cudaStream_t st) {
  auto kern = qgemv_kernel<NMAT, T, TYPE, CW>;
  const int budget = GEMV_SMEM_WIDE;
  const int nb = a.nb;
  int64_t tiles = 0;
  int stage_bytes = 0, nbs_min = nb;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].rows <= 0) return cudaErrorInvalidValue;
  for (int i = 0; i < a.nseg; ++i) {
    GemvSegK &S = a.seg[i];
    S.tile0 = int(tiles);
    tiles += (S.rows + GEMV_TILE - 1) / GEMV_TILE;
    int nbs = GEMV_STAGE_TARGET / (NMAT * S.rec);
    if (nbs < 1) nbs = 1;
    if (nbs > nb) nbs = nb;
    S.nbs = nbs;
    if (nbs < nbs_min) nbs_min = nbs;
    if (NMAT * nbs * S.rec > stage_bytes) stage_bytes = NMAT * nbs * S.rec;
  }
  if (tiles * nb >= (int64_t(1) << 30)) return cudaErrorInvalidValue;
  a.units = int(tiles * nb);
  a.stage_bytes = stage_bytes;
  // Grid: every CTA holds at least one tile's worth of units (a tile is then shared by at most
  // two CTAs) and touches at most lt_cap tiles (the partial-sum buffer).
  const int64_t tile_red = int64_t(GEMV_TILE) * NMAT * T * nb * 4;
  int64_t lt_cap = GEMV_RED_TARGET / tile_red;
  if (lt_cap < 3) lt_cap = 3;
  int64_t G = tiles < num_sms() ? tiles : num_sms();
  const int64_t g_min = (tiles + lt_cap - 3) / (lt_cap - 2);
  if (G < g_min) G = g_min;
  if (G > sp.max_ctas || !sp.cnt || !sp.part) return cudaErrorInvalidValue;
  a.uq = int(a.units / G);
  a.ur = int(a.units % G);
  const int64_t max_units = (a.units + G - 1) / G;
  const int64_t lt_max = (max_units + nb - 1) / nb + 1;
  a.max_stages = int(max_units / nbs_min + lt_max + 1);
  const int red_bytes = int((lt_max * tile_red + 127) / 128 * 128);
  a.red_off = 256;  // barriers: full[12], empty[12]
  a.tab_off = a.red_off + red_bytes;
  a.x_off = a.tab_off + (a.max_stages * int(sizeof(GemvStage)) + 127) / 128 * 128;
  a.ring_off = a.x_off + (gemv_x_bytes(nb, T) + 127) / 128 * 128;
  int nst = (budget - a.ring_off) / stage_bytes;
  if (nst > GEMV_MAX_STAGES) nst = GEMV_MAX_STAGES;
  if (nst < 2) return cudaErrorInvalidValue;
  a.nstage = nst;
  a.cnt = sp.cnt;
  a.part = sp.part;
  const size_t smem = size_t(a.ring_off) + size_t(nst) * stage_bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(unsigned(G)), dim3((CW + 1) * 32), smem, st, a);
}

template <int NMAT, int T, int TYPE>
static cudaError_t launch_qgemv_cw(const QGemvArgs &a, const GemvSplit &sp, cudaStream_t st) {
  return launch_qgemv_t<NMAT, T, TYPE, GEMV_CW_WIDE>(a, sp, st);
}

template <int NMAT>
static cudaError_t launch_qgemv_n(const QGemvArgs &a, int T, const GemvSplit &sp, cudaStream_t st) {
  int type = a.seg[0].type;
  for (int i = 1; i < a.nseg; ++i)
    if (a.seg[i].type != type) type = 0;
  if (T == 1) {
    if (type == T_Q4_K) return launch_qgemv_cw<NMAT, 1, T_Q4_K>(a, sp, st);
    if (type == T_Q6_K) return launch_qgemv_cw<NMAT, 1, T_Q6_K>(a, sp, st);
    return launch_qgemv_cw<NMAT, 1, 0>(a, sp, st);
  }
  if (type == T_Q4_K) return launch_qgemv_cw<NMAT, 2, T_Q4_K>(a, sp, st);
  if (type == T_Q6_K) return launch_qgemv_cw<NMAT, 2, T_Q6_K>(a, sp, st);
  return launch_qgemv_cw<NMAT, 2, 0>(a, sp, st);
}

cudaError_t gemv_fused(const GemvSeg *segs, int nseg, int nmat, int64_t K, GemvPrologue pro, int64_t n_tok,
                       cudaStream_t st, const GemvSplit *split) {
  if (n_tok <= 0) return cudaSuccess;
  if (nseg < 1 || nseg > GEMV_MAX_SEG || (nmat != 1 && nmat != 2)) return cudaErrorInvalidValue;
  if (K % QK_K || K / QK_K > 64) return cudaErrorInvalidValue;
  const GemvSplit sp = split ? *split : default_split();
  QGemvArgs a = {};
  a.nseg = nseg;
  a.nb = int(K / QK_K);
  a.err = device_error_ptr();
  a.pro = pro;
  for (int i = 0; i < nseg; ++i) {
    const GemvSeg &sg = segs[i];
    if (sg.type != T_Q4_K && sg.type != T_Q6_K) return cudaErrorInvalidValue;
    if (!sg.w[0] || (nmat == 2 && !sg.w[1]) || sg.rows <= 0 || sg.rows >= (int64_t(1) << 30))
      return cudaErrorInvalidValue;
    GemvSegK &S = a.seg[i];
    S.w[0] = sg.w[0];
    S.w[1] = sg.w[1];
    S.y = sg.y;
    S.rows = int(sg.rows);
    S.type = sg.type;
    S.rec = kquant_rec_bytes(sg.type);
    S.ldy = sg.ldy;
  }
  for (int64_t t0 = 0; t0 < n_tok; t0 += GEMV_MAX_T) {
    const int T = int(n_tok - t0 < GEMV_MAX_T ? n_tok - t0 : GEMV_MAX_T);
    QGemvArgs c = a;
    if (c.pro.x) c.pro.x += t0 * K;
    if (c.pro.a) c.pro.a += t0 * K;
    if (c.pro.resid_in) c.pro.resid_in += t0 * K;
    if (c.pro.resid_out) c.pro.resid_out += t0 * K;
    for (int i = 0; i < nseg; ++i) c.seg[i].y += t0 * c.seg[i].ldy;
    const cudaError_t e = nmat == 2 ? launch_qgemv_n<2>(c, T, sp, st) : launch_qgemv_n<1>(c, T, sp, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t gemv(int type, const void *w0, const void *w1, int64_t rows, int64_t K, const float *x, int64_t n_tok,
                 float *y, int64_t ldy, cudaStream_t st) {
  if (rows <= 0 || n_tok <= 0) return cudaSuccess;
  const int nmat = w1 ? 2 : 1;
  if (type == T_Q4_K || type == T_Q6_K) {
    GemvSeg sg = {};
    sg.w[0] = static_cast<const uint8_t *>(w0);
    sg.w[1] = static_cast<const uint8_t *>(w1);
    sg.y = y;
    sg.rows = rows;
    sg.type = type;
    sg.ldy = int(ldy);
    GemvPrologue pro = {};
    pro.mode = 0;
    pro.x = x;
    return gemv_fused(&sg, 1, nmat, K, pro, n_tok, st);
  }
  const int threads = 256;
  int64_t blocks = (rows * 32 + threads - 1) / threads;
  if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
  const dim3 grid = dim3((unsigned)blocks), block = dim3(threads);
  switch (type) {
    case T_F32:
      return nmat == 2 ? launch_pdl(fgemv_kernel<T_F32, 2>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy)
                       : launch_pdl(fgemv_kernel<T_F32, 1>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy);
    case T_F16:
      return nmat == 2 ? launch_pdl(fgemv_kernel<T_F16, 2>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy)
                       : launch_pdl(fgemv_kernel<T_F16, 1>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy);
    case T_BF16:
      return nmat == 2 ? launch_pdl(fgemv_kernel<T_BF16, 2>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy)
                       : launch_pdl(fgemv_kernel<T_BF16, 1>, grid, block, 0, st, w0, w1, x, y, rows, K, int(n_tok), ldy);
  }
  return cudaErrorInvalidValue;
}

cudaError_t dequantize(int type, const void *w, int64_t n_rows, int64_t K, float *out, cudaStream_t st) {
  if (type != T_Q4_K && type != T_Q6_K) return cudaErrorInvalidValue;
  if (K % QK_K) return cudaErrorInvalidValue;
  const int64_t nblk = n_rows * (K / QK_K);
  if (nblk == 0) return cudaSuccess;
  const int64_t threads = nblk * 8;
  dequant_kernel<<<unsigned((threads + 255) / 256), 256, 0, st>>>(type, static_cast<const uint8_t *>(w), nblk, out);
  return cudaGetLastError();
}

cudaError_t prepare_weights(int type, const void *gguf, int64_t rows, int64_t K, void *dst, cudaStream_t st) {
  if (type == T_Q4_K || type == T_Q6_K) {
    if (K <= 0 || K % QK_K) return cudaErrorInvalidValue;
    const int nb = int(K / QK_K);
    const int64_t threads = (rows + KQ_TILE - 1) / KQ_TILE * nb * KQ_TILE;
    if (threads == 0) return cudaSuccess;
    repack_kquant_kernel<<<unsigned((threads + 255) / 256), 256, 0, st>>>(type, static_cast<const uint8_t *>(gguf),
                                                                           rows, nb, static_cast<uint8_t *>(dst));
    return cudaGetLastError();
  }
  const int rb = device_row_bytes(type, K);
  if (rb < 0) return cudaErrorInvalidValue;
  return cudaMemcpyAsync(dst, gguf, size_t(rows) * rb, cudaMemcpyDeviceToDevice, st);
}

}  // namespace sfc
