// gemv.cu — dequant-fused K-quant GEMV for decode (1..4 tokens per pass).
//
// Replaces the reference's row-dot hot loop (crates/stage-forward-lab/src/quants.rs:1801-1909
// for Q4_K, :2594-2688 for Q6_K) driven by real_math.rs:398-733 (matmul_quantized_many_refs_range)
// and the gate/up pair path real_math.rs:1584-1800 + GeGLU real_forward.rs:1716-1730.
//
// Design (B200):
//  * Each CTA owns a contiguous slab of weight rows and streams it HBM -> shared memory with
//    bulk async copies (the TMA engine, cp.async.bulk) into an mbarrier ring; all stages are
//    requested up front so the whole slab is in flight at once.
//  * Thread t owns one 32-element column slice (block b, 64-group j, half h) of every row and
//    keeps its activations in registers for the whole kernel, so shared memory only carries
//    weights.  Slices of one 256-block sit in 8 consecutive lanes (segment reduction by shuffle).
//  * Activations are split exactly into three signed 8-bit digit planes per 256-block
//    (x = 2^e (a*65536 + b*256 + c), |x| < 2^(e+22)), so nibble x digit products and their sums
//    are exact int32 dp4a work; rounding happens only in the final fp32 combine.  This keeps
//    the integer pipe, not the ALU pipe, as the compute path and stays within 2^-22 of x.
//  * Q6_K weights use a per-row struct-of-arrays device layout (ql | qh | scales | d, row padded
//    to 16 B) prepared once at load so every field is 16-byte aligned for vector smem loads.
#include <cuda_runtime.h>
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

constexpr int GEMV_THREADS = 320;  // 40 Q4_K blocks x 8 slices; 80-slice rows -> 4 row groups
constexpr int GEMV_MAX_T = 4;

__device__ unsigned g_device_error = 0;
long long g_kernel_launches = 0;

// ---------------------------------------------------------------- activations
// Per-thread view of the activation slice for one token: digit planes for the two
// 16-element halves (A = elements j*64+16h+[0,16), B = A+32), block scale 2^e and
// half sums of the quantized values.
struct XSlice {
  uint32_t p[3][2][4];  // [plane a,b,c][half][word] 4 signed digits per word
  float scale;
  float sum[2];
};

__device__ __forceinline__ void load_xslice(const float *__restrict__ x, int blk, int j, int h, int lane,
                                            XSlice &xs) {
  const float *base = x + blk * QK_K + j * 64 + h * 16;
  float v[2][16];
#pragma unroll
  for (int half = 0; half < 2; ++half)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float4 f = *reinterpret_cast<const float4 *>(base + half * 32 + 4 * k);
      v[half][4 * k + 0] = f.x;
      v[half][4 * k + 1] = f.y;
      v[half][4 * k + 2] = f.z;
      v[half][4 * k + 3] = f.w;
    }
  float m = 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half)
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[half][i]));
  // max over the 8 slices of this 256-block (8 consecutive lanes)
  const unsigned seg = 0xFFu << (lane & 24);
  m = fmaxf(m, __shfl_xor_sync(seg, m, 1));
  m = fmaxf(m, __shfl_xor_sync(seg, m, 2));
  m = fmaxf(m, __shfl_xor_sync(seg, m, 4));
  int E = 0;
  if (m > 0.f) frexpf(m, &E);  // m < 2^E
  if (E < -100) E = -100;
  const int up = 22 - E;  // x * 2^up has magnitude < 2^22
  xs.scale = ldexpf(1.0f, -up);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    int isum = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t pa = 0, pb = 0, pc = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int X = __float2int_rn(ldexpf(v[half][4 * w + k], up));
        isum += X;
        int c = (X << 24) >> 24;
        int X1 = (X - c) >> 8;
        int b = (X1 << 24) >> 24;
        int a = (X1 - b) >> 8;
        pa |= uint32_t(a & 0xFF) << (8 * k);
        pb |= uint32_t(b & 0xFF) << (8 * k);
        pc |= uint32_t(c & 0xFF) << (8 * k);
      }
      xs.p[0][half][w] = pa;
      xs.p[1][half][w] = pb;
      xs.p[2][half][w] = pc;
    }
    xs.sum[half] = float(isum) * xs.scale;
  }
}

// sum over the 4 words of one half: exact int32 dot of 16 unsigned weights with 16 digits
__device__ __forceinline__ int dot16(const uint32_t (&wq)[4], const uint32_t (&xp)[4]) {
  int s = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w) s = dp4a_us(wq[w], xp[w], s);
  return s;
}

__device__ __forceinline__ float combine_planes(int ia, int ib, int ic) {
  return (float(ia) * 65536.0f + float(ib) * 256.0f) + float(ic);
}

// ---------------------------------------------------------------- per-row slice dots
// Q4_K (GGUF layout): returns sum over this thread's 32 elements of w*x for each token.
template <int T>
__device__ __forceinline__ void q4k_slice(const uint8_t *__restrict__ row, int blk, int j, int h,
                                          const XSlice (&xs)[T], float (&acc)[T]) {
  const uint8_t *bp = row + blk * BLOCK_Q4_K;
  const uint4 hd = lds128(bp);
  const uint4 qv = lds128(bp + 16 + j * 32 + h * 16);
  const float d = h2f_bits(uint16_t(hd.x & 0xFFFF));
  const float dmin = h2f_bits(uint16_t(hd.x >> 16));
  // get_scale_min_k4 for sub-blocks 2j (A) and 2j+1 (B), quants.rs:252-261
  int scA, mA, scB, mB;
  {
    const uint32_t s0 = hd.y, s1 = hd.z, s2 = hd.w;
    const int k = (2 * j) & 3;
    const uint32_t b0a = (s0 >> (8 * k)) & 0xFF, b1a = (s1 >> (8 * k)) & 0xFF, b2a = (s2 >> (8 * k)) & 0xFF;
    const uint32_t b0b = (s0 >> (8 * k + 8)) & 0xFF, b1b = (s1 >> (8 * k + 8)) & 0xFF,
                   b2b = (s2 >> (8 * k + 8)) & 0xFF;
    if (j < 2) {
      scA = b0a & 63;
      mA = b1a & 63;
      scB = b0b & 63;
      mB = b1b & 63;
    } else {
      scA = (b2a & 15) | ((b0a >> 6) << 4);
      mA = (b2a >> 4) | ((b1a >> 6) << 4);
      scB = (b2b & 15) | ((b0b >> 6) << 4);
      mB = (b2b >> 4) | ((b1b >> 6) << 4);
    }
  }
  uint32_t lo[4], hi[4];
  lo[0] = qv.x & 0x0F0F0F0Fu;
  lo[1] = qv.y & 0x0F0F0F0Fu;
  lo[2] = qv.z & 0x0F0F0F0Fu;
  lo[3] = qv.w & 0x0F0F0F0Fu;
  hi[0] = (qv.x >> 4) & 0x0F0F0F0Fu;
  hi[1] = (qv.y >> 4) & 0x0F0F0F0Fu;
  hi[2] = (qv.z >> 4) & 0x0F0F0F0Fu;
  hi[3] = (qv.w >> 4) & 0x0F0F0F0Fu;
  const float fmA = float(mA), fmB = float(mB);
#pragma unroll
  for (int t = 0; t < T; ++t) {
    int I[3];
#pragma unroll
    for (int p = 0; p < 3; ++p) I[p] = scA * dot16(lo, xs[t].p[p][0]) + scB * dot16(hi, xs[t].p[p][1]);
    const float f = combine_planes(I[0], I[1], I[2]);
    acc[t] += d * (xs[t].scale * f) - dmin * (fmA * xs[t].sum[0] + fmB * xs[t].sum[1]);
  }
}

// Q6_K (device SoA layout per row: ql[nb][128] | qh[nb][64] | sc[nb][16] | d[nb] f16).
template <int T>
__device__ __forceinline__ void q6k_slice(const uint8_t *__restrict__ row, int nb, int blk, int j, int h,
                                          const XSlice (&xs)[T], float (&acc)[T]) {
  const int n = j >> 1, jj = j & 1;
  const uint8_t *ql = row + blk * 128 + n * 64 + h * 16;
  const uint8_t *qh = row + nb * 128 + blk * 64 + n * 32 + h * 16;
  const int8_t *sc = reinterpret_cast<const int8_t *>(row + nb * 192 + blk * 16 + n * 8 + h + 4 * jj);
  const uint16_t dbits = *reinterpret_cast<const uint16_t *>(row + nb * 208 + blk * 2);
  const uint4 qa = lds128(ql), qb = lds128(ql + 32), qhv = lds128(qh);
  const int scA = sc[0], scB = sc[2];
  const float d = h2f_bits(dbits);
  const int sh = 4 * jj;
  const uint32_t qa4[4] = {qa.x, qa.y, qa.z, qa.w}, qb4[4] = {qb.x, qb.y, qb.z, qb.w};
  const uint32_t qh4[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
  uint32_t uA[4], uB[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uA[w] = ((qa4[w] >> sh) & 0x0F0F0F0Fu) | (((qh4[w] >> sh) & 0x03030303u) << 4);
    uB[w] = ((qb4[w] >> sh) & 0x0F0F0F0Fu) | (((qh4[w] >> (sh + 2)) & 0x03030303u) << 4);
  }
#pragma unroll
  for (int t = 0; t < T; ++t) {
    int I[3];
#pragma unroll
    for (int p = 0; p < 3; ++p) I[p] = scA * dot16(uA, xs[t].p[p][0]) + scB * dot16(uB, xs[t].p[p][1]);
    const float f = combine_planes(I[0], I[1], I[2]);
    // sum (u - 32) * sc * x = sc * (sum u x - 32 sum x)
    acc[t] += d * (xs[t].scale * f - 32.0f * (float(scA) * xs[t].sum[0] + float(scB) * xs[t].sum[1]));
  }
}

__device__ __forceinline__ float gelu_tanh_mul(float v, float u) {
  // real_math.rs:79-85
  const float k = 0.7978845608028654f;
  const float inner = k * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner)) * u;
}

// ---------------------------------------------------------------- kernel
struct QGemvArgs {
  const uint8_t *w[2];  // NMAT matrices, device layout
  const float *x;       // [T][K]
  float *y;             // [T][rows] (NMAT==1) or GeGLU act [T][rows] (NMAT==2)
  int64_t rows;
  int nb;               // K / 256
  int row_bytes;        // device-layout bytes per row (multiple of 16)
  int groups;           // row groups per CTA
  int rows_per_stage;
  int nstage;
  int ldy;              // row stride of y in floats (>= rows)
  unsigned *err;
};

template <int TYPE, int NMAT, int T>
__global__ void __launch_bounds__(GEMV_THREADS, 1) qgemv_kernel(const QGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int S = a.nb * 8;
  const int g = tid / S, s = tid % S;
  const int blk = s >> 3, j = (s >> 1) & 3, h = s & 1;
  const int lane = tid & 31;
  const bool active = g < a.groups;

  // CTA row range
  const int64_t r_begin = a.rows * blockIdx.x / gridDim.x;
  const int64_t r_end = a.rows * (blockIdx.x + 1) / gridDim.x;
  const int n_rows = int(r_end - r_begin);
  const int n_iter = (n_rows + a.rows_per_stage - 1) / a.rows_per_stage;
  const int stage_bytes = a.rows_per_stage * a.row_bytes * NMAT;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  float *red = reinterpret_cast<float *>(smem + 128);  // [2][rows_per_stage][NMAT][T][nb]
  const int red_stride = a.rows_per_stage * NMAT * T * a.nb;
  uint8_t *stages = smem + 128 + ((2 * red_stride * 4 + 127) / 128) * 128;

  auto issue = [&](int it) {
    const int slot = it % a.nstage;
    const int64_t r0 = r_begin + int64_t(it) * a.rows_per_stage;
    const int nr = int(r_end - r0 < a.rows_per_stage ? r_end - r0 : a.rows_per_stage);
    const uint32_t bytes = uint32_t(nr) * a.row_bytes;
    mbar_arrive_expect_tx(&bars[slot], bytes * NMAT);
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
      bulk_g2s(stages + slot * stage_bytes + m * a.rows_per_stage * a.row_bytes, a.w[m] + r0 * a.row_bytes,
               bytes, &bars[slot]);
  };

  if (tid == 0) {
    for (int i = 0; i < a.nstage; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    // Weights do not depend on the previous kernel: start streaming them before the
    // dependency wait so their fetch overlaps the producer's tail.
    for (int it = 0; it < min(a.nstage, n_iter); ++it) issue(it);
  }
  pdl_wait();
  pdl_launch_dependents();

  XSlice xs[T];
  if (active) {
#pragma unroll
    for (int t = 0; t < T; ++t) load_xslice(a.x + int64_t(t) * a.nb * QK_K, blk, j, h, lane, xs[t]);
  }
  __syncthreads();  // barrier inits visible to all threads

  const unsigned seg = 0xFFu << (lane & 24);
  for (int it = 0; it < n_iter; ++it) {
    const int slot = it % a.nstage;
    const int64_t r0 = r_begin + int64_t(it) * a.rows_per_stage;
    const int nr = int(r_end - r0 < a.rows_per_stage ? r_end - r0 : a.rows_per_stage);
    mbar_wait_bounded(&bars[slot], (it / a.nstage) & 1, a.err);
    const uint8_t *st = stages + slot * stage_bytes;
    float *rd = red + (it & 1) * red_stride;
    if (active) {
      for (int lr = g; lr < nr; lr += a.groups) {
        float acc[NMAT][T];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
#pragma unroll
          for (int t = 0; t < T; ++t) acc[m][t] = 0.f;
          const uint8_t *row = st + (m * a.rows_per_stage + lr) * a.row_bytes;
          if (TYPE == T_Q4_K)
            q4k_slice<T>(row, blk, j, h, xs, acc[m]);
          else
            q6k_slice<T>(row, a.nb, blk, j, h, xs, acc[m]);
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
          for (int t = 0; t < T; ++t) {
            float v = acc[m][t];
            v += __shfl_xor_sync(seg, v, 1);
            v += __shfl_xor_sync(seg, v, 2);
            v += __shfl_xor_sync(seg, v, 4);
            if ((s & 7) == 0) rd[((lr * NMAT + m) * T + t) * a.nb + blk] = v;
          }
      }
    }
    __syncthreads();  // stage slot fully consumed; partials complete
    if (tid == 0 && it + a.nstage < n_iter) issue(it + a.nstage);
    for (int idx = tid; idx < nr * T; idx += blockDim.x) {
      const int lr = idx / T, t = idx % T;
      float v[NMAT];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const float *p = rd + ((lr * NMAT + m) * T + t) * a.nb;
        float sum = 0.f;
        for (int b = 0; b < a.nb; ++b) sum += p[b];
        v[m] = sum;
      }
      float out = v[0];
      if (NMAT == 2) out = gelu_tanh_mul(v[0], v[NMAT - 1]);
      a.y[int64_t(t) * a.ldy + r0 + lr] = out;
    }
  }
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

// GGUF Q6_K rows -> device SoA rows (see file header).
__global__ void repack_q6k_kernel(const uint8_t *__restrict__ src, int64_t rows, int nb, int dst_row_bytes,
                                  uint8_t *__restrict__ dst) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= rows * nb) return;
  const int64_t r = b / nb;
  const int k = int(b % nb);
  const uint8_t *s = src + b * BLOCK_Q6_K;
  uint8_t *row = dst + r * dst_row_bytes;
  for (int i = 0; i < 128; ++i) row[k * 128 + i] = s[i];
  for (int i = 0; i < 64; ++i) row[nb * 128 + k * 64 + i] = s[128 + i];
  for (int i = 0; i < 16; ++i) row[nb * 192 + k * 16 + i] = s[192 + i];
  row[nb * 208 + 2 * k] = s[208];
  row[nb * 208 + 2 * k + 1] = s[209];
  if (k == 0)
    for (int i = nb * 210; i < dst_row_bytes; ++i) row[i] = 0;
}

// ---------------------------------------------------------------- host side
int device_row_bytes(int type, int64_t K) {
  if (K <= 0) return -1;
  switch (type) {
    case T_F32: return int(K * 4);
    case T_F16:
    case T_BF16: return int(K * 2);
    case T_Q4_K: return K % QK_K ? -1 : int(K / QK_K * BLOCK_Q4_K);
    case T_Q6_K: return K % QK_K ? -1 : int((K / QK_K * BLOCK_Q6_K + 15) / 16 * 16);
  }
  return -1;
}

int gguf_row_bytes(int type, int64_t K) {
  if (type == T_Q6_K) return K % QK_K ? -1 : int(K / QK_K * BLOCK_Q6_K);
  return device_row_bytes(type, K);
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

constexpr int GEMV_SMEM_BUDGET = 200 * 1024;
constexpr int GEMV_STAGE_TARGET = 24 * 1024;

template <int TYPE, int NMAT, int T>
static cudaError_t launch_qgemv_t(QGemvArgs a, cudaStream_t st) {
  auto kern = qgemv_kernel<TYPE, NMAT, T>;
  const int S = a.nb * 8;
  a.groups = GEMV_THREADS / S;
  const int per_row = a.row_bytes * NMAT;
  int rps = (GEMV_STAGE_TARGET / per_row) / a.groups * a.groups;
  if (rps < a.groups) rps = a.groups;
  a.rows_per_stage = rps;
  const int stage_bytes = rps * per_row;
  const int red_bytes = ((2 * rps * NMAT * T * a.nb * 4 + 127) / 128) * 128;
  int nst = (GEMV_SMEM_BUDGET - 128 - red_bytes) / stage_bytes;
  if (nst > 8) nst = 8;
  if (nst < 1) return cudaErrorInvalidValue;
  a.nstage = nst;
  const size_t smem = 128 + red_bytes + size_t(nst) * stage_bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  int64_t ctas = (a.rows + a.groups - 1) / a.groups;
  if (ctas > num_sms()) ctas = num_sms();
  return launch_pdl(kern, dim3(unsigned(ctas)), dim3(a.groups * S), smem, st, a);
}

template <int TYPE, int NMAT>
static cudaError_t launch_qgemv_n(QGemvArgs a, int T, cudaStream_t st) {
  switch (T) {
    case 1: return launch_qgemv_t<TYPE, NMAT, 1>(a, st);
    case 2: return launch_qgemv_t<TYPE, NMAT, 2>(a, st);
    case 3: return launch_qgemv_t<TYPE, NMAT, 3>(a, st);
    default: return launch_qgemv_t<TYPE, NMAT, 4>(a, st);
  }
}

cudaError_t gemv(int type, const void *w0, const void *w1, int64_t rows, int64_t K, const float *x, int64_t n_tok,
                 float *y, int64_t ldy, cudaStream_t st) {
  if (rows <= 0 || n_tok <= 0) return cudaSuccess;
  const int nmat = w1 ? 2 : 1;
  if (type == T_Q4_K || type == T_Q6_K) {
    if (K % QK_K || K / QK_K * 8 > GEMV_THREADS) return cudaErrorInvalidValue;
    QGemvArgs a = {};
    a.w[0] = static_cast<const uint8_t *>(w0);
    a.w[1] = static_cast<const uint8_t *>(w1 ? w1 : w0);
    a.rows = rows;
    a.nb = int(K / QK_K);
    a.row_bytes = device_row_bytes(type, K);
    a.ldy = int(ldy);
    a.err = device_error_ptr();
    for (int64_t t0 = 0; t0 < n_tok; t0 += GEMV_MAX_T) {
      const int T = int(n_tok - t0 < GEMV_MAX_T ? n_tok - t0 : GEMV_MAX_T);
      a.x = x + t0 * K;
      a.y = y + t0 * ldy;
      cudaError_t e;
      if (type == T_Q4_K)
        e = nmat == 2 ? launch_qgemv_n<T_Q4_K, 2>(a, T, st) : launch_qgemv_n<T_Q4_K, 1>(a, T, st);
      else
        e = nmat == 2 ? launch_qgemv_n<T_Q6_K, 2>(a, T, st) : launch_qgemv_n<T_Q6_K, 1>(a, T, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
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
  if (type == T_Q6_K) {
    if (K % QK_K) return cudaErrorInvalidValue;
    const int nb = int(K / QK_K);
    const int64_t nblk = rows * nb;
    if (nblk == 0) return cudaSuccess;
    repack_q6k_kernel<<<unsigned((nblk + 127) / 128), 128, 0, st>>>(
        static_cast<const uint8_t *>(gguf), rows, nb, device_row_bytes(type, K), static_cast<uint8_t *>(dst));
    return cudaGetLastError();
  }
  const int rb = device_row_bytes(type, K);
  if (rb < 0) return cudaErrorInvalidValue;
  return cudaMemcpyAsync(dst, gguf, size_t(rows) * rb, cudaMemcpyDeviceToDevice, st);
}

}  // namespace sfc
