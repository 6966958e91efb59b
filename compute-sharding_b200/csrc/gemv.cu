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

// Threads per CTA: 1-token launches use 512 threads (16 warps, <= 128 registers each), 2-token
// launches 320 (up to 204 registers for the per-token activation planes).
template <int T>
struct GemvCfg {
  static constexpr int THREADS = T == 1 ? 512 : 320;
};
constexpr int GEMV_MAX_THREADS = 512;
constexpr int GEMV_MAX_T = 2;
constexpr int SLICES_PER_BLOCK = 4;

__device__ unsigned g_device_error = 0;
long long g_kernel_launches = 0;

// ---------------------------------------------------------------- activations
// Per-thread view of the activation slice for one token: digit planes for the two 32-element
// halves (A = elements j*64+[0,32), B = A+32) of block `blk`, the block scale 2^e, and sums of
// the quantized values per 32 (Q4_K mins) and per 16 elements (Q6_K offset of 32).
struct XSlice {
  uint32_t p[3][2][8];  // [plane a,b,c][half][word] 4 signed digits per word
  float scale;
  float sum32[2];
  float sum16[4];
};

// Shared-memory record of one 64-element slice: the XSlice fields in order, padded to 60 words
// so that consecutive records start 28 banks apart (conflict-free 16-byte loads).
constexpr int XREC_WORDS = 60;

__device__ __forceinline__ void load8(const float *p, int64_t off, float (&v)[8]) {
  const float4 f0 = *reinterpret_cast<const float4 *>(p + off);
  const float4 f1 = *reinterpret_cast<const float4 *>(p + off + 4);
  v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
  v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
}

__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4 *>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Exact digit planes of one 256-element block held by a warp (lane l: elements 8l..8l+7); the
// lane writes its part of the record of slice l/8 (half (l/4)&1, plane words 2(l&3), +1).
__device__ __forceinline__ void quantize8(const float (&v)[8], int lane, uint32_t *rec) {
  float m = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
  m = warp_max(m);
  // m < 2^E with E = biased exponent - 126 (zero and subnormal maxima clamp to E = -100)
  int E = int((__float_as_uint(m) >> 23) & 0xFF) - 126;
  if (E < -100) E = -100;
  const int up = 22 - E;  // x * 2^up has magnitude < 2^22; up in [-106, 122]
  const float pw = __uint_as_float(uint32_t(127 + up) << 23);     // 2^up, a normal float
  const float scale = __uint_as_float(uint32_t(127 - up) << 23);  // 2^-up
  // X = rint(x * 2^up): x * 2^up is exact and |X| <= 2^22, so adding 1.5 * 2^23 in one fused
  // multiply-add rounds to the nearest integer, which then sits in the low mantissa bits:
  // bits(fma(x, 2^up, 1.5*2^23)) = 0x4B400000 + X.  Balanced base-256 digits without carries:
  // Y = X + 0x808080 lies in [0, 2^24) and its bytes y2, y1, y0 give
  // X = (y2-128)*65536 + (y1-128)*256 + (y0-128); the int8 digit y-128 is the byte y XOR 0x80,
  // so each plane word is a byte gather (prmt) plus an xor.
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr uint32_t kBias = 0x4B400000u - 0x808080u;
  uint32_t Y[8], ys = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    Y[e] = __float_as_uint(fmaf(v[e], pw, kRound)) - kBias;
    ys += Y[e];
  }
  uint32_t wc[2], wb[2], wa[2];
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const uint32_t lo01 = __byte_perm(Y[4 * w], Y[4 * w + 1], 0x5140);  // [Y0.b0, Y1.b0, Y0.b1, Y1.b1]
    const uint32_t lo23 = __byte_perm(Y[4 * w + 2], Y[4 * w + 3], 0x5140);
    const uint32_t hi01 = __byte_perm(Y[4 * w], Y[4 * w + 1], 0x7362);  // [Y0.b2, Y1.b2, Y0.b3, Y1.b3]
    const uint32_t hi23 = __byte_perm(Y[4 * w + 2], Y[4 * w + 3], 0x7362);
    wc[w] = __byte_perm(lo01, lo23, 0x5410) ^ 0x80808080u;  // c: bytes 0
    wb[w] = __byte_perm(lo01, lo23, 0x7632) ^ 0x80808080u;  // b: bytes 1
    wa[w] = __byte_perm(hi01, hi23, 0x5410) ^ 0x80808080u;  // a: bytes 2
  }
  const int h = (lane >> 2) & 1, q = lane & 3;
  uint32_t *pw0 = rec + h * 8 + 2 * q;
  *reinterpret_cast<uint2 *>(pw0) = make_uint2(wa[0], wa[1]);
  *reinterpret_cast<uint2 *>(pw0 + 16) = make_uint2(wb[0], wb[1]);
  *reinterpret_cast<uint2 *>(pw0 + 32) = make_uint2(wc[0], wc[1]);
  // sum of X over 16 (32) elements = sum of Y - 16 (32) * 0x808080, exact in 32-bit arithmetic
  const uint32_t y16 = ys + __shfl_xor_sync(0xFFFFFFFFu, ys, 1);
  const uint32_t y32 = y16 + __shfl_xor_sync(0xFFFFFFFFu, y16, 2);
  if ((q & 1) == 0) rec[51 + 2 * h + (q >> 1)] = __float_as_uint(float(int(y16 - 16u * 0x808080u)) * scale);
  if (q == 0) rec[49 + h] = __float_as_uint(float(int(y32 - 32u * 0x808080u)) * scale);
  if ((lane & 7) == 0) rec[48] = __float_as_uint(scale);
}

__device__ __forceinline__ void load_slice(const uint32_t *rec, XSlice &xs) {
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const uint4 w = *reinterpret_cast<const uint4 *>(rec + 4 * i);
    uint32_t *dst = &xs.p[0][0][0] + 4 * i;
    dst[0] = w.x; dst[1] = w.y; dst[2] = w.z; dst[3] = w.w;
  }
  const uint4 u0 = *reinterpret_cast<const uint4 *>(rec + 48), u1 = *reinterpret_cast<const uint4 *>(rec + 52);
  xs.scale = __uint_as_float(u0.x);
  xs.sum32[0] = __uint_as_float(u0.y);
  xs.sum32[1] = __uint_as_float(u0.z);
  xs.sum16[0] = __uint_as_float(u0.w);
  xs.sum16[1] = __uint_as_float(u1.x);
  xs.sum16[2] = __uint_as_float(u1.y);
  xs.sum16[3] = __uint_as_float(u1.z);
}

__device__ __forceinline__ int dot16(const uint32_t *wq, const uint32_t *xp) {
  int s = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w) s = dp4a_us(wq[w], xp[w], s);
  return s;
}

__device__ __forceinline__ float combine_planes(int ia, int ib, int ic) {
  return (float(ia) * 65536.0f + float(ib) * 256.0f) + float(ic);
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t b) {  // (a & mask) | b
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(b));
  return r;
}

// ---------------------------------------------------------------- per-row slice dots
// Q4_K (GGUF layout): adds this thread's 64-element dot to acc[t] for every token.
template <int T>
__device__ __forceinline__ void q4k_slice(const uint8_t *__restrict__ row, int blk, int j,
                                          const XSlice (&xs)[T], float (&acc)[T]) {
  const uint8_t *bp = row + blk * BLOCK_Q4_K;
  const uint4 hd = lds128(bp);
  const uint4 q0 = lds128(bp + 16 + j * 32), q1 = lds128(bp + 32 + j * 32);
  const float d = h2f_bits(uint16_t(hd.x & 0xFFFF));
  const float dmin = h2f_bits(uint16_t(hd.x >> 16));
  // get_scale_min_k4 for sub-blocks 2j (A) and 2j+1 (B), quants.rs:252-261; the two bytes of
  // each of the three scale words sit side by side, so extract them as a 16-bit pair.
  int scA, mA, scB, mB;
  {
    const uint32_t sel = (j & 1) ? 0x4342u : 0x4140u;  // bytes (2j&3, 2j&3+1) -> 16-bit lanes
    const uint32_t x0 = __byte_perm(hd.y, 0u, sel), x1 = __byte_perm(hd.z, 0u, sel), x2 = __byte_perm(hd.w, 0u, sel);
    uint32_t sc, mn;
    if (j < 2) {
      sc = x0 & 0x003F003Fu;
      mn = x1 & 0x003F003Fu;
    } else {
      sc = (x2 & 0x000F000Fu) | ((x0 >> 2) & 0x00300030u);
      mn = ((x2 >> 4) & 0x000F000Fu) | ((x1 >> 2) & 0x00300030u);
    }
    scA = int(sc & 0xFFFF);
    scB = int(sc >> 16);
    mA = int(mn & 0xFFFF);
    mB = int(mn >> 16);
  }
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    lo[k] = w[k] & 0x0F0F0F0Fu;
    hi[k] = (w[k] >> 4) & 0x0F0F0F0Fu;
  }
  const float fmA = float(mA), fmB = float(mB);
#pragma unroll
  for (int t = 0; t < T; ++t) {
    int I[3];
#pragma unroll
    for (int p = 0; p < 3; ++p)
      I[p] = scA * (dot16(lo, xs[t].p[p][0]) + dot16(lo + 4, xs[t].p[p][0] + 4)) +
             scB * (dot16(hi, xs[t].p[p][1]) + dot16(hi + 4, xs[t].p[p][1] + 4));
    const float f = combine_planes(I[0], I[1], I[2]);
    acc[t] += d * (xs[t].scale * f) - dmin * (fmA * xs[t].sum32[0] + fmB * xs[t].sum32[1]);
  }
}

// Q6_K (device SoA layout per row: ql[nb][128] | qh[nb][64] | sc[nb][16] | d[nb] f16).
// Slice j covers elements j*64..j*64+63 = 128-half n = j/2, quarter groups g = 2(j&1), 2(j&1)+1.
template <int T>
__device__ __forceinline__ void q6k_slice(const uint8_t *__restrict__ row, int nb, int blk, int j,
                                          const XSlice (&xs)[T], float (&acc)[T]) {
  const int n = j >> 1, jj = j & 1;
  const uint8_t *ql = row + blk * 128 + n * 64;
  const uint8_t *qh = row + nb * 128 + blk * 64 + n * 32;
  const uint32_t scw = *reinterpret_cast<const uint32_t *>(row + nb * 192 + blk * 16 + n * 8 + 4 * jj);
  const uint16_t dbits = *reinterpret_cast<const uint16_t *>(row + nb * 208 + blk * 2);
  const uint4 a0 = lds128(ql), a1 = lds128(ql + 16), b0 = lds128(ql + 32), b1 = lds128(ql + 48);
  const uint4 h0 = lds128(qh), h1 = lds128(qh + 16);
  const int sA0 = int(int8_t(scw & 0xFF)), sA1 = int(int8_t((scw >> 8) & 0xFF));
  const int sB0 = int(int8_t((scw >> 16) & 0xFF)), sB1 = int(int8_t(scw >> 24));
  const float d = h2f_bits(dbits);
  const int sh = 4 * jj;
  const uint32_t qa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const uint32_t qb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  const uint32_t qhw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  uint32_t uA[8], uB[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    // 2 high bits of group g sit at bits 2g..2g+1 of each qh byte; move them to bits 4..5
    const uint32_t hA = ((qhw[k] >> sh) << 4) & 0x30303030u;
    const uint32_t hB = ((qhw[k] >> (sh + 2)) << 4) & 0x30303030u;
    uA[k] = lop_and_or(qa[k] >> sh, 0x0F0F0F0Fu, hA);
    uB[k] = lop_and_or(qb[k] >> sh, 0x0F0F0F0Fu, hB);
  }
#pragma unroll
  for (int t = 0; t < T; ++t) {
    int I[3];
#pragma unroll
    for (int p = 0; p < 3; ++p)
      I[p] = sA0 * dot16(uA, xs[t].p[p][0]) + sA1 * dot16(uA + 4, xs[t].p[p][0] + 4) +
             sB0 * dot16(uB, xs[t].p[p][1]) + sB1 * dot16(uB + 4, xs[t].p[p][1] + 4);
    const float f = combine_planes(I[0], I[1], I[2]);
    // sum (u - 32) * sc * x = sc * (sum u x - 32 sum x), per 16-element scale group
    const float corr = float(sA0) * xs[t].sum16[0] + float(sA1) * xs[t].sum16[1] + float(sB0) * xs[t].sum16[2] +
                       float(sB1) * xs[t].sum16[3];
    acc[t] += d * (xs[t].scale * f - 32.0f * corr);
  }
}

__device__ __forceinline__ float gelu_tanh_mul(float v, float u) {
  // real_math.rs:79-85
  const float k = 0.7978845608028654f;
  const float inner = k * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner)) * u;
}

// ---------------------------------------------------------------- kernel
constexpr int MAX_SEG = 3;

struct QGemvArgs {
  GemvSeg seg[MAX_SEG];
  int nseg;
  int64_t total_rows;
  int nb;
  int groups;
  int nstage;
  int stage_bytes;
  int rps_max;
  int rcap;       // rows whose block partials the CTA can hold before it must finalize
  int red_bytes;  // bytes of the partials buffer (also holds the activation slice records)
  GemvPrologue pro;
  unsigned *err;
};

// Segments let one launch cover several matrices with the same K (q, k and v of a layer):
// the CTAs split the concatenated row space evenly and each stage stays inside one segment.
template <int NMAT, int T>
__global__ void __launch_bounds__(GemvCfg<T>::THREADS, 1) qgemv_kernel(const QGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float pro_red[GEMV_MAX_T][GEMV_MAX_THREADS / 32];
  const int tid = threadIdx.x;
  const int S = a.nb * SLICES_PER_BLOCK;
  const int g = tid / S, s = tid % S;
  const int blk = s >> 2, j = s & 3;
  const int lane = tid & 31;
  const int K = a.nb * QK_K;

  const int64_t r_begin = a.total_rows * blockIdx.x / gridDim.x;
  const int64_t r_end = a.total_rows * (blockIdx.x + 1) / gridDim.x;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  float *red = reinterpret_cast<float *>(smem + 128);  // [rcap][NMAT][T][nb] block partials
  uint8_t *stages = smem + 128 + a.red_bytes;

  // stage at global row `pos`: segment, first local row, row count
  auto stage_at = [&](int64_t pos, int &sg, int64_t &local0, int &nr) {
    int64_t base = 0;
    sg = 0;
    while (sg + 1 < a.nseg && pos >= base + a.seg[sg].rows) base += a.seg[sg++].rows;
    local0 = pos - base;
    int64_t n = a.seg[sg].rps;
    if (r_end - pos < n) n = r_end - pos;
    if (a.seg[sg].rows - local0 < n) n = a.seg[sg].rows - local0;
    nr = int(n);
  };
  // Producer cursor: every thread tracks it (it is deterministic) so that refills are a uniform
  // decision; only thread 0 issues the copies.
  int64_t ppos = r_begin;
  int pit = 0;
  auto issue_next = [&]() {
    int sg, nr;
    int64_t l0;
    stage_at(ppos, sg, l0, nr);
    if (tid == 0) {
      const GemvSeg &G = a.seg[sg];
      const int slot = pit % a.nstage;
      const uint32_t bytes = uint32_t(nr) * G.row_bytes;
      mbar_arrive_expect_tx(&bars[slot], bytes * NMAT);
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
        bulk_g2s(stages + slot * a.stage_bytes + m * G.rps * G.row_bytes, G.w[m] + l0 * G.row_bytes, bytes,
                 &bars[slot]);
    }
    ppos += nr;
    ++pit;
  };
  // Writes the outputs of CTA-relative rows [c0, c1) from their block partials.
  auto finalize = [&](int c0, int c1) {
    for (int idx = tid; idx < (c1 - c0) * T; idx += blockDim.x) {
      const int pr = idx / T, t = idx % T;
      int sg, nr;
      int64_t l0;
      stage_at(r_begin + c0 + pr, sg, l0, nr);
      float v[NMAT];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const float *p = red + ((pr * NMAT + m) * T + t) * a.nb;
        float sum = 0.f;
        for (int b = 0; b < a.nb; ++b) sum += p[b];
        v[m] = sum;
      }
      a.seg[sg].y[int64_t(t) * a.seg[sg].ldy + l0] = NMAT == 2 ? gelu_tanh_mul(v[0], v[NMAT - 1]) : v[0];
    }
  };

  if (tid == 0) {
    for (int i = 0; i < a.nstage; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  // Weights never depend on the previous kernel: stream them before the dependency wait so their
  // fetch overlaps the producer's tail (programmatic dependent launch).  Every thread advances
  // the cursor; thread 0 (which initialised the barriers just above) issues the copies.
  while (pit < a.nstage && ppos < r_end) issue_next();
  pdl_wait();
  pdl_launch_dependents();

  // ---- activations, computed once per CTA.  Unit u = (token t, 256-block b) belongs to warp
  // u % nwarps and lane l holds its elements 8l..8l+7, so every global access is a coalesced
  // 1 KB piece of a row.  The optional fused residual add + RMSNorm passes run first; the last
  // pass writes each 64-element slice's digit planes and sums into a shared-memory record
  // (aliasing the row-partials buffer), from which every thread loads its own slice.
  XSlice xs[T];
  {
    const GemvPrologue &P = a.pro;
    uint32_t *xrec = reinterpret_cast<uint32_t *>(red);
    const int nwarps = int(blockDim.x) >> 5, warp = tid >> 5;
    const int units = T * a.nb;
    float s1[T], s2[T];
#pragma unroll
    for (int t = 0; t < T; ++t) s1[t] = s2[t] = 1.0f;
    // the 8 values of unit (t, b) after `step` prologue steps: 0 = input, 1 = after the first
    // norm (+ residual), 2 = after the norm of the next op
    auto value8 = [&](int t, int b, int step, float (&v)[8]) {
      const int64_t off = int64_t(t) * K + b * QK_K + lane * 8;
      const int col = b * QK_K + lane * 8;
      load8(P.mode == 0 ? P.x : P.a, off, v);
      if (P.mode == 0 || step == 0) return;
      const float s1t = (T == 1 || t == 0) ? s1[0] : s1[T - 1];
      if (P.mode == 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * s1t;  // (x * scale) * w, real_math.rs:43
      } else {
        float wp[8], rs[8];
        if (P.w_post) load8(P.w_post, col, wp);
        load8(P.resid_in, off, rs);
        const float sc = P.scale ? P.scale[0] : 1.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float r = (P.w_post ? (v[e] * s1t) * wp[e] : v[e]) + rs[e];
          if (P.scale) r = r * sc;
          v[e] = r;
        }
      }
      if (step == 1 || !P.w_next) return;
      const float s2t = (T == 1 || t == 0) ? s2[0] : s2[T - 1];
      float wn[8];
      load8(P.w_next, col, wn);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (v[e] * s2t) * wn[e];
    };
    // per-token sums over the CTA of sum(v^2) after `step` steps, in a fixed order
    auto cta_sumsq = [&](int step, bool store_resid, float (&out)[T]) {
      float part[T];
#pragma unroll
      for (int t = 0; t < T; ++t) part[t] = 0.f;
      for (int u = warp; u < units; u += nwarps) {
        const int t = u / a.nb, b = u % a.nb;
        float v[8];
        value8(t, b, step, v);
        float q = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) q += v[e] * v[e];
        if (T == 1 || t == 0) part[0] += q; else part[T - 1] += q;
        if (store_resid) store8(P.resid_out + int64_t(t) * K + b * QK_K + lane * 8, v);
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float w = warp_sum(part[t]);
        if (lane == 0) pro_red[t][warp] = w;
      }
      __syncthreads();
#pragma unroll
      for (int t = 0; t < T; ++t) {
        float sum = 0.f;
        for (int w = 0; w < nwarps; ++w) sum += pro_red[t][w];
        out[t] = sum;
      }
      __syncthreads();
    };
    if (P.mode != 0) {
      float tot[T];
      if (P.mode == 1 || P.w_post) {
        cta_sumsq(0, false, tot);
#pragma unroll
        for (int t = 0; t < T; ++t) s1[t] = 1.0f / sqrtf(tot[t] / float(K) + P.eps);
      }
      if (P.mode == 2 && (P.w_next || (P.resid_out && blockIdx.x == 0))) {
        cta_sumsq(1, P.resid_out && blockIdx.x == 0, tot);
#pragma unroll
        for (int t = 0; t < T; ++t) s2[t] = 1.0f / sqrtf(tot[t] / float(K) + P.eps);
      }
    }
    for (int u = warp; u < units; u += nwarps) {
      const int t = u / a.nb, b = u % a.nb;
      float v[8];
      value8(t, b, 2, v);
      quantize8(v, lane, xrec + ((t * a.nb + b) * SLICES_PER_BLOCK + (lane >> 3)) * XREC_WORDS);
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < T; ++t) load_slice(xrec + ((t * a.nb + blk) * SLICES_PER_BLOCK + j) * XREC_WORDS, xs[t]);
  }
  __syncthreads();  // slices loaded (the records alias the partials) and barrier inits visible

  const unsigned seg = 0xFu << (lane & 28);
  int64_t pos = r_begin;
  int pend0 = 0;  // CTA-relative row held in red[0]
  for (int it = 0; pos < r_end; ++it) {
    int sg, nr;
    int64_t l0;
    stage_at(pos, sg, l0, nr);
    const int crow = int(pos - r_begin);
    if (crow + nr - pend0 > a.rcap) {  // partial buffer full: emit the pending rows first
      __syncthreads();
      finalize(pend0, crow);
      __syncthreads();
      pend0 = crow;
    }
    const GemvSeg &G = a.seg[sg];
    const int slot = it % a.nstage;
    mbar_wait_bounded(&bars[slot], (it / a.nstage) & 1, a.err);
    const uint8_t *st = stages + slot * a.stage_bytes;
    const bool q4 = G.type == T_Q4_K;
    for (int lr = g; lr < nr; lr += a.groups) {
      float acc[NMAT][T];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
#pragma unroll
        for (int t = 0; t < T; ++t) acc[m][t] = 0.f;
        const uint8_t *row = st + (m * G.rps + lr) * G.row_bytes;
        if (q4)
          q4k_slice<T>(row, blk, j, xs, acc[m]);
        else
          q6k_slice<T>(row, a.nb, blk, j, xs, acc[m]);
      }
      float *rd = red + (crow - pend0 + lr) * NMAT * T * a.nb;
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int t = 0; t < T; ++t) {
          float v = acc[m][t];
          v += __shfl_xor_sync(seg, v, 1);
          v += __shfl_xor_sync(seg, v, 2);
          if ((s & 3) == 0) rd[(m * T + t) * a.nb + blk] = v;
        }
    }
    if (ppos < r_end) {  // this slot is needed again: wait until every thread is done with it
      __syncthreads();
      issue_next();
    }
    pos += nr;
  }
  __syncthreads();
  finalize(pend0, int(r_end - r_begin));
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

constexpr int GEMV_STAGE_TARGET = 24 * 1024;

template <int NMAT, int T>
static cudaError_t launch_qgemv_t(QGemvArgs a, cudaStream_t st) {
  auto kern = qgemv_kernel<NMAT, T>;
  constexpr int THREADS = GemvCfg<T>::THREADS;
  const int S = a.nb * SLICES_PER_BLOCK;
  a.groups = THREADS / S;
  if (a.groups < 1) return cudaErrorInvalidValue;
  a.stage_bytes = 0;
  a.rps_max = 0;
  for (int i = 0; i < a.nseg; ++i) {
    GemvSeg &sg = a.seg[i];
    // rows per stage: a multiple of the row-group count so every group has the same rows
    int rps = (GEMV_STAGE_TARGET / (sg.row_bytes * NMAT) + a.groups / 2) / a.groups * a.groups;
    if (rps < a.groups) rps = a.groups;
    sg.rps = rps;
    if (rps * sg.row_bytes * NMAT > a.stage_bytes) a.stage_bytes = rps * sg.row_bytes * NMAT;
    if (rps > a.rps_max) a.rps_max = rps;
  }
  int64_t ctas = (a.total_rows + a.groups - 1) / a.groups;
  if (ctas > num_sms()) ctas = num_sms();
  // hold every row of the CTA's slab when that fits (one finalize at the end), else rps_max rows
  const int per_row = NMAT * T * a.nb * 4;
  const int rows_per_cta = int((a.total_rows + ctas - 1) / ctas);
  a.rcap = rows_per_cta * per_row <= 32 * 1024 ? rows_per_cta : a.rps_max;
  if (a.rcap < a.rps_max) a.rcap = a.rps_max;
  const int budget = 200 * 1024;  // one CTA per SM (the register file is full)
  int red_bytes = a.rcap * per_row;
  const int rec_bytes = T * a.nb * SLICES_PER_BLOCK * XREC_WORDS * 4;
  if (rec_bytes > red_bytes) red_bytes = rec_bytes;
  red_bytes = (red_bytes + 127) / 128 * 128;
  a.red_bytes = red_bytes;
  int nst = (budget - 128 - red_bytes) / a.stage_bytes;
  if (nst > 8) nst = 8;
  if (nst < 1) return cudaErrorInvalidValue;
  a.nstage = nst;
  const size_t smem = 128 + red_bytes + size_t(nst) * a.stage_bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(unsigned(ctas)), dim3(a.groups * S), smem, st, a);
}

template <int NMAT>
static cudaError_t launch_qgemv_n(const QGemvArgs &a, int T, cudaStream_t st) {
  switch (T) {
    case 1: return launch_qgemv_t<NMAT, 1>(a, st);
    default: return launch_qgemv_t<NMAT, 2>(a, st);
  }
}

cudaError_t gemv_fused(const GemvSeg *segs, int nseg, int nmat, int64_t K, GemvPrologue pro, int64_t n_tok,
                       cudaStream_t st) {
  if (n_tok <= 0) return cudaSuccess;
  if (nseg < 1 || nseg > MAX_SEG || (nmat != 1 && nmat != 2)) return cudaErrorInvalidValue;
  if (K % QK_K || K / QK_K * SLICES_PER_BLOCK > 320) return cudaErrorInvalidValue;
  QGemvArgs a = {};
  a.nseg = nseg;
  a.nb = int(K / QK_K);
  a.err = device_error_ptr();
  a.pro = pro;
  for (int i = 0; i < nseg; ++i) {
    GemvSeg sg = segs[i];
    if (sg.type != T_Q4_K && sg.type != T_Q6_K) return cudaErrorInvalidValue;
    if (!sg.w[0] || (nmat == 2 && !sg.w[1]) || sg.rows <= 0) return cudaErrorInvalidValue;
    sg.row_bytes = device_row_bytes(sg.type, K);
    a.seg[i] = sg;
    a.total_rows += sg.rows;
  }
  for (int64_t t0 = 0; t0 < n_tok; t0 += GEMV_MAX_T) {
    const int T = int(n_tok - t0 < GEMV_MAX_T ? n_tok - t0 : GEMV_MAX_T);
    QGemvArgs c = a;
    if (c.pro.x) c.pro.x += t0 * K;
    if (c.pro.a) c.pro.a += t0 * K;
    if (c.pro.resid_in) c.pro.resid_in += t0 * K;
    if (c.pro.resid_out) c.pro.resid_out += t0 * K;
    for (int i = 0; i < nseg; ++i) c.seg[i].y += t0 * c.seg[i].ldy;
    const cudaError_t e = nmat == 2 ? launch_qgemv_n<2>(c, T, st) : launch_qgemv_n<1>(c, T, st);
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
