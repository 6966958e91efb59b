// gemv_core.cuh — device core of the K-quant GEMV (see gemv.cu): activation image, tensor-pipe
// MMA units, the CTA work partition and stage walk, and the cross-CTA finish of shared tiles.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace sfc {

constexpr int GEMV_TILE = 16;       // weight rows per MMA tile
// Consumer warps per CTA (plus one producer warp): 15, 512 threads and one CTA per SM.
constexpr int GEMV_CW_WIDE = 15;
constexpr int GEMV_MAX_T = 2;
constexpr int GEMV_MAX_STAGES = 12;
constexpr int GEMV_MAX_SEG = 3;
// floats of one CTA-boundary slot: two sides x 16 rows x (2 matrices x 2 tokens)
constexpr int GEMV_SPLIT_SLOT = 2 * GEMV_TILE * 2 * GEMV_MAX_T;
constexpr int GEMV_DEFAULT_SPLIT_CTAS = 1024;


// ---------------------------------------------------------------- small helpers
// Activations are read through L2 only (.cg): in the fused layer kernel the same buffers are
// rewritten by other CTAs between phases of one launch, so no SM may hold them in L1.
__device__ __forceinline__ void load8(const float *p, int64_t off, float (&v)[8]) {
  const float4 f0 = __ldcg(reinterpret_cast<const float4 *>(p + off));
  const float4 f1 = __ldcg(reinterpret_cast<const float4 *>(p + off + 4));
  v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
  v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
}

__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4 *>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t b) {  // (a & mask) | b
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(b));
  return r;
}

// Byte permute against zero: selector 0x4440 | b zero-extends byte b; sext_sel(b) sign-extends it.
__device__ __forceinline__ int prmt0(uint32_t a, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(a), "r"(sel));
  return int(r);
}
__host__ __device__ constexpr uint32_t sext_sel(uint32_t b) {
  return b | ((8u | b) << 4) | ((8u | b) << 8) | ((8u | b) << 12);
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int r;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// D = A (16 x 32 u8, row) * B (32 x 8 s8, col) + C, exact int32.  Fragment layout (lane = 4g + t):
// a0/a2 = row g, k 4t..4t+3 / 16+4t..; a1/a3 = row g+8; b0/b1 = column g, k 4t.. / 16+4t..;
// d0,d1 = row g, columns 2t, 2t+1; d2,d3 = row g+8.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, int c0, int c1, int c2, int c3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Barrier of the consumer warps only (the producer warp never joins).
template <int CW>
__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}

__device__ __forceinline__ float gelu_tanh_mul(float v, float u) {
  // real_math.rs:79-85
  const float k = 0.7978845608028654f;
  const float inner = k * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner)) * u;
}

// ---------------------------------------------------------------- activation fragments
// Shared-memory image of the activations of all T tokens, built once per CTA:
//  frag  [nb][4 chunk pairs][3T columns][4 t][4 words]  digit words in MMA B-fragment order:
//        word k of (block b, pair cp, column P = 3*token + plane, t) holds the digits of elements
//        32c + 4t + [0,4) (k even) or 32c + 16 + 4t + [0,4) (k odd), c = 2cp + k/2
//  scale [nb][T]         2^-e of the block
//  sum32 [nb][T][8]      sum of x over each 32-element sub-block (Q4_K mins)
//  q6c   [nb][T][4 t][8 chunks][2]  Q6_K accumulator inputs of the two columns 2t, 2t+1 a lane
//        holds: -32 x (digit sum of plane n%3 over 16-element group 2c + n/3), 0 for n >= 6
struct XSmem {
  uint32_t *frag;
  float *scale;
  float *sum32;
  int *q6c;
};

__host__ __device__ inline int gemv_x_bytes(int nb, int T) {
  const int scale_b = (nb * T * 4 + 15) / 16 * 16;
  return nb * 768 * T + scale_b + nb * T * 32 + nb * T * 256;
}

__device__ __forceinline__ XSmem x_view(uint8_t *base, int nb, int T) {
  XSmem x;
  x.frag = reinterpret_cast<uint32_t *>(base);
  uint8_t *p = base + nb * 768 * T;
  x.scale = reinterpret_cast<float *>(p);
  p += (nb * T * 4 + 15) / 16 * 16;
  x.sum32 = reinterpret_cast<float *>(p);
  p += nb * T * 32;
  x.q6c = reinterpret_cast<int *>(p);
  return x;
}

// Exact digit planes of one 256-element block held by a warp (lane l: elements 8l..8l+7).
template <int T>
__device__ __forceinline__ void emit_block(const float (&v)[8], int lane, int b, int tok, const XSmem &X) {
  constexpr int NP = 3 * T;
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
  uint32_t planes[3][2];  // [a, b, c][elements 8l..8l+3, 8l+4..8l+7]
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const uint32_t lo01 = __byte_perm(Y[4 * w], Y[4 * w + 1], 0x5140);  // [Y0.b0, Y1.b0, Y0.b1, Y1.b1]
    const uint32_t lo23 = __byte_perm(Y[4 * w + 2], Y[4 * w + 3], 0x5140);
    const uint32_t hi01 = __byte_perm(Y[4 * w], Y[4 * w + 1], 0x7362);  // [Y0.b2, Y1.b2, Y0.b3, Y1.b3]
    const uint32_t hi23 = __byte_perm(Y[4 * w + 2], Y[4 * w + 3], 0x7362);
    planes[2][w] = __byte_perm(lo01, lo23, 0x5410) ^ 0x80808080u;  // c: bytes 0
    planes[1][w] = __byte_perm(lo01, lo23, 0x7632) ^ 0x80808080u;  // b: bytes 1
    planes[0][w] = __byte_perm(hi01, hi23, 0x5410) ^ 0x80808080u;  // a: bytes 2
  }
  // lane l = 4c + q holds elements 32c + 8q + [0, 8): words t = 2(q&1), 2(q&1)+1 of half q>>1
  const int c = lane >> 2, q = lane & 3, t0 = 2 * (q & 1), k = (c & 1) * 2 + (q >> 1);
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    uint32_t *dst = X.frag + (((b * 4 + (c >> 1)) * NP + tok * 3 + p) * 4 + t0) * 4 + k;
    dst[0] = planes[p][0];
    dst[4] = planes[p][1];
  }
  // sum of X over 32 elements = sum of Y - 32 * 0x808080, exact in 32-bit arithmetic
  const uint32_t y16 = ys + __shfl_xor_sync(0xFFFFFFFFu, ys, 1);
  const uint32_t y32 = y16 + __shfl_xor_sync(0xFFFFFFFFu, y16, 2);
  if (q == 0) X.sum32[(b * T + tok) * 8 + c] = float(int(y32 - 32u * 0x808080u)) * scale;
  if (lane == 0) X.scale[b * T + tok] = scale;
  // Q6_K accumulator inputs: lanes 4c + {0,1} hold group 2c, lanes 4c + {2,3} group 2c + 1
  int *q6 = X.q6c + (b * T + tok) * 64;
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    int s = dp4a_ss(planes[p][1], 0x01010101u, dp4a_ss(planes[p][0], 0x01010101u, 0));
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    const int n = (q >> 1) * 3 + p;  // column (group parity, plane)
    if ((q & 1) == 0) q6[(n >> 1) * 16 + c * 2 + (n & 1)] = -32 * s;
  }
  if (q == 0) {
    q6[3 * 16 + c * 2] = 0;
    q6[3 * 16 + c * 2 + 1] = 0;
  }
}

// ---------------------------------------------------------------- MMA units
// Per-lane output columns n = 2t, 2t+1: plane weight (65536, 256, 1; 0 when unused) and token.
__device__ __forceinline__ float plane_weight(int n, int ncols) {
  if (n >= ncols) return 0.f;
  const int p = n % 3;
  return p == 0 ? 65536.0f : (p == 1 ? 256.0f : 1.0f);
}

// Q4_K (tiled records; matrix m's records of the stage at `stage + m * mstride`): this lane's share
// of rows g and g+8 for block b (record lb of the stage), v[m][row][token], summed over the four t
// lanes by the caller.  Chunk c = sub-block c; even sub-blocks are the low nibbles of bytes
// 32(c/2) + [0,32), odd ones the high nibbles (quants.rs:181-208).  High nibbles stay in place
// (16 q) and the low-nibble sums are scaled by 16 to match, so d/16 is applied at the end.
template <int NMAT, int T>
__device__ __forceinline__ void unit_q4k(const uint8_t *__restrict__ stage, int mstride, int lb, int b,
                                         const XSmem &X, int g, int t, float (&v)[NMAT][2][T]) {
  constexpr int NP = 3 * T;
  const uint32_t keep = g < NP ? 0xFFFFFFFFu : 0u;
  const int P = g < NP ? g : 0;
  uint32_t bf[8][2];
#pragma unroll
  for (int cp = 0; cp < 4; ++cp) {
    const uint4 w = *reinterpret_cast<const uint4 *>(X.frag + (((b * 4 + cp) * NP + P) * 4 + t) * 4);
    bf[2 * cp][0] = w.x & keep;
    bf[2 * cp][1] = w.y & keep;
    bf[2 * cp + 1][0] = w.z & keep;
    bf[2 * cp + 1][1] = w.w & keep;
  }
  const int n0 = 2 * t, n1 = 2 * t + 1, tk0 = n0 / 3 < T ? n0 / 3 : T - 1, tk1 = n1 / 3 < T ? n1 / 3 : T - 1;
  const float W0 = plane_weight(n0, NP) * X.scale[b * T + tk0];
  const float W1 = plane_weight(n1, NP) * X.scale[b * T + tk1];
  float S[T][2];
#pragma unroll
  for (int k = 0; k < T; ++k) {
    const float2 s = *reinterpret_cast<const float2 *>(X.sum32 + (b * T + k) * 8 + 2 * t);
    S[k][0] = s.x;
    S[k][1] = s.y;
  }
  const uint32_t msel0 = 0x4440u | uint32_t(2 * (t & 1)), msel1 = msel0 + 1;
#pragma unroll
  for (int m = 0; m < NMAT; ++m) {
    const uint8_t *rec = stage + m * mstride + lb * REC_Q4_K;
    const uint4 hg = lds128(rec + 16 * g), hh = lds128(rec + 16 * (g + 8));
    const uint8_t *qg = rec + 256 + 128 * g, *qh8 = qg + 8 * 128;  // rows g, g+8: same chunk swizzle
    // get_scale_min_k4 (quants.rs:252-261), four 6-bit values per word: sub-blocks 0-3, 4-7
    const uint32_t scg03 = hg.y & 0x3F3F3F3Fu, sch03 = hh.y & 0x3F3F3F3Fu;
    const uint32_t scg47 = lop_and_or(hg.w, 0x0F0F0F0Fu, (hg.y >> 2) & 0x30303030u);
    const uint32_t sch47 = lop_and_or(hh.w, 0x0F0F0F0Fu, (hh.y >> 2) & 0x30303030u);
    // mins of sub-blocks 2t, 2t+1 (this lane's share of the min term)
    const uint32_t mg = t < 2 ? (hg.z & 0x3F3F3F3Fu) : lop_and_or(hg.w >> 4, 0x0F0F0F0Fu, (hg.z >> 2) & 0x30303030u);
    const uint32_t mh = t < 2 ? (hh.z & 0x3F3F3F3Fu) : lop_and_or(hh.w >> 4, 0x0F0F0F0Fu, (hh.z >> 2) & 0x30303030u);
    int ae[4] = {0, 0, 0, 0}, ao[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // bytes 32j + 4t (chunk 2j) and 32j + 16 + 4t (chunk 2j + 1) of the row's quants
      const int o0 = (((2 * j) ^ (g & 7)) << 4) + 4 * t, o1 = (((2 * j + 1) ^ (g & 7)) << 4) + 4 * t;
      const uint32_t w0g = lds32(qg + o0), w1g = lds32(qg + o1), w0h = lds32(qh8 + o0), w1h = lds32(qh8 + o1);
      const uint32_t swg = j < 2 ? scg03 : scg47, swh = j < 2 ? sch03 : sch47;
      const uint32_t se = 0x4440u | uint32_t((2 * j) & 3), so = se + 1;
      int d[4];
      mma_u8s8(d, w0g & 0x0F0F0F0Fu, w0h & 0x0F0F0F0Fu, w1g & 0x0F0F0F0Fu, w1h & 0x0F0F0F0Fu, bf[2 * j][0],
               bf[2 * j][1], 0, 0, 0, 0);
      const int sge = prmt0(swg, se), she = prmt0(swh, se);
      ae[0] += sge * d[0];
      ae[1] += sge * d[1];
      ae[2] += she * d[2];
      ae[3] += she * d[3];
      mma_u8s8(d, w0g & 0xF0F0F0F0u, w0h & 0xF0F0F0F0u, w1g & 0xF0F0F0F0u, w1h & 0xF0F0F0F0u, bf[2 * j + 1][0],
               bf[2 * j + 1][1], 0, 0, 0, 0);
      const int sgo = prmt0(swg, so), sho = prmt0(swh, so);
      ao[0] += sgo * d[0];
      ao[1] += sgo * d[1];
      ao[2] += sho * d[2];
      ao[3] += sho * d[3];
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 &h = i ? hh : hg;
      const uint32_t mw = i ? mh : mg;
      const float d16 = h2f_bits(uint16_t(h.x & 0xFFFF)) * 0.0625f;
      const float dmin = h2f_bits(uint16_t(h.x >> 16));
      const float m0 = float(prmt0(mw, msel0)), m1 = float(prmt0(mw, msel1));
      const float F0 = float(ae[2 * i] * 16 + ao[2 * i]) * W0;
      const float F1 = float(ae[2 * i + 1] * 16 + ao[2 * i + 1]) * W1;
#pragma unroll
      for (int k = 0; k < T; ++k) {
        const float f = (tk0 == k ? F0 : 0.f) + (tk1 == k ? F1 : 0.f);
        v[m][i][k] = d16 * f - dmin * (m0 * S[k][0] + m1 * S[k][1]);
      }
    }
  }
}

// Q6_K (tiled records, as unit_q4k).  Chunk c = 4n + q covers elements 128n + 32q + l, l in [0,32):
// q6 = ((ql[64n + 32(q&1) + l] >> 4(q>>1)) & 15) | (((qh[32n + l] >> 2q) & 3) << 4), scale group
// 2c + l/16 (quants.rs:210-249).  The B columns are masked per group (columns 0-2: elements
// l < 16, columns 3-5: l >= 16) so that each output column sees one scale group.
template <int NMAT, int T>
__device__ __forceinline__ void unit_q6k(const uint8_t *__restrict__ stage, int mstride, int lb, int b,
                                         const XSmem &X, int g, int t, float (&v)[NMAT][2][T]) {
  constexpr int NP = 3 * T;
  const uint32_t keep0 = g < 3 ? 0xFFFFFFFFu : 0u, keep1 = (g >= 3 && g < 6) ? 0xFFFFFFFFu : 0u;
  const int gp = g < 6 ? g % 3 : 0;
  // output columns of this lane: n = 2t + k -> scale group parity p_k (columns >= 6 are zero)
  const int n0 = 2 * t, n1 = 2 * t + 1;
  const uint32_t p0 = n0 >= 3 ? 1u : 0u, p1 = n1 >= 3 ? 1u : 0u;
  const uint32_t se0 = sext_sel(p0), se1 = sext_sel(p1), so0 = sext_sel(2u + p0), so1 = sext_sel(2u + p1);
  float W0[T], W1[T];
#pragma unroll
  for (int k = 0; k < T; ++k) {
    const float xs = X.scale[b * T + k];
    W0[k] = plane_weight(n0, 6) * xs;
    W1[k] = plane_weight(n1, 6) * xs;
  }
  const int *q6c = X.q6c + (b * T) * 64 + t * 16;
#pragma unroll
  for (int m = 0; m < NMAT; ++m) {
    const uint8_t *rec = stage + m * mstride + lb * REC_Q6_K;
    const uint4 scg = lds128(rec + 3072 + 16 * g), sch = lds128(rec + 3072 + 16 * (g + 8));
    const float dg = h2f_bits(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * g));
    const float dh = h2f_bits(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * (g + 8)));
    const int sw_l = g & 7, sw_h = (g >> 1) & 3;  // chunk swizzles of ql / qh (rows g and g+8 alike)
    int acc[T][4];
#pragma unroll
    for (int k = 0; k < T; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      // ql bytes 64n + 32qq + 16k + 4t (chunk 4n + 2qq + k), qh bytes 32n + 16k + 4t (chunk 2n + k)
      const uint8_t *lg = rec + 128 * g + 4 * t, *lh = lg + 8 * 128;
      const uint8_t *hg_ = rec + 2048 + 64 * g + 4 * t, *hh_ = hg_ + 8 * 64;
      uint32_t Lg[2][2], Lh[2][2], Hg[2], Hh[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int ol = ((4 * n + 2 * qq + k) ^ sw_l) << 4;
          Lg[qq][k] = lds32(lg + ol);
          Lh[qq][k] = lds32(lh + ol);
        }
        const int oh = ((2 * n + k) ^ sw_h) << 4;
        Hg[k] = lds32(hg_ + oh);
        Hh[k] = lds32(hh_ + oh);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = 4 * n + q;
        uint32_t ug[2], uh[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint32_t lwg = Lg[q & 1][k], lwh = Lh[q & 1][k];
          if (q == 0) {
            ug[k] = lop_and_or(lwg, 0x0F0F0F0Fu, (Hg[k] << 4) & 0x30303030u);
            uh[k] = lop_and_or(lwh, 0x0F0F0F0Fu, (Hh[k] << 4) & 0x30303030u);
          } else if (q == 1) {
            ug[k] = lop_and_or(lwg, 0x0F0F0F0Fu, (Hg[k] << 2) & 0x30303030u);
            uh[k] = lop_and_or(lwh, 0x0F0F0F0Fu, (Hh[k] << 2) & 0x30303030u);
          } else if (q == 2) {
            ug[k] = lop_and_or(lwg >> 4, 0x0F0F0F0Fu, Hg[k] & 0x30303030u);
            uh[k] = lop_and_or(lwh >> 4, 0x0F0F0F0Fu, Hh[k] & 0x30303030u);
          } else {
            ug[k] = lop_and_or(lwg >> 4, 0x0F0F0F0Fu, (Hg[k] >> 2) & 0x30303030u);
            uh[k] = lop_and_or(lwh >> 4, 0x0F0F0F0Fu, (Hh[k] >> 2) & 0x30303030u);
          }
        }
        const uint32_t swg = (c >> 1) == 0 ? scg.x : (c >> 1) == 1 ? scg.y : (c >> 1) == 2 ? scg.z : scg.w;
        const uint32_t swh = (c >> 1) == 0 ? sch.x : (c >> 1) == 1 ? sch.y : (c >> 1) == 2 ? sch.z : sch.w;
        const uint32_t s0 = (c & 1) ? so0 : se0, s1 = (c & 1) ? so1 : se1;
        const int sg0 = prmt0(swg, s0), sg1 = prmt0(swg, s1), sh0 = prmt0(swh, s0), sh1 = prmt0(swh, s1);
#pragma unroll
        for (int k = 0; k < T; ++k) {
          const uint4 w =
              *reinterpret_cast<const uint4 *>(X.frag + (((b * 4 + (c >> 1)) * NP + 3 * k + gp) * 4 + t) * 4);
          const uint32_t b0 = ((c & 1) ? w.z : w.x) & keep0, b1 = ((c & 1) ? w.w : w.y) & keep1;
          const int2 co = *reinterpret_cast<const int2 *>(q6c + k * 64 + c * 2);
          int d[4];
          mma_u8s8(d, ug[0], uh[0], ug[1], uh[1], b0, b1, co.x, co.y, co.x, co.y);
          acc[k][0] += sg0 * d[0];
          acc[k][1] += sg1 * d[1];
          acc[k][2] += sh0 * d[2];
          acc[k][3] += sh1 * d[3];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < T; ++k) {
      v[m][0][k] = dg * (float(acc[k][0]) * W0[k] + float(acc[k][1]) * W1[k]);
      v[m][1][k] = dh * (float(acc[k][2]) * W0[k] + float(acc[k][3]) * W1[k]);
    }
  }
}

// ---------------------------------------------------------------- kernel
struct GemvSegK {
  const uint8_t *w[2];
  float *y;
  int rows;
  int tile0;  // first global tile of the segment
  int type;
  int rec;  // record bytes (REC_Q4_K / REC_Q6_K)
  int nbs;  // blocks per stage at most (a matrix's records of a stage: nbs * rec bytes)
  int ldy;
};

struct QGemvArgs {
  GemvSegK seg[GEMV_MAX_SEG];
  int nseg;
  int nb;
  int units;      // tiles * nb
  int uq, ur;     // CTA c owns units [c*uq + min(c, ur), ...), uq + (c < ur) of them
  int nstage;     // ring slots
  int max_stages; // stage-table entries per CTA
  int stage_bytes;
  int red_off, x_off, ring_off, tab_off;  // dynamic shared-memory offsets
  GemvPrologue pro;
  unsigned *err;
  unsigned *cnt;  // per CTA boundary: arrivals of the two CTAs sharing a tile
  float *part;    // per CTA boundary: GEMV_SPLIT_SLOT floats of partial row sums
};

// The tiles a CTA touches, in processing order: the tiles it shares with its neighbours come first
// (its last tile, then its first) so that their partial sums are published early, then the tiles
// it owns alone, ascending.
struct CtaTiles {
  int u0, u1, tf, tl, np, count;
  bool fs, ls;  // first tile shared with CTA cta-1 / last tile shared with CTA cta+1
  __device__ __forceinline__ void init(int u0_, int u1_, int nb) {
    u0 = u0_;
    u1 = u1_;
    tf = u0 / nb;
    tl = (u1 - 1) / nb;
    fs = u0 != tf * nb;
    ls = u1 != (tl + 1) * nb;
    np = (fs ? 1 : 0) + (ls ? 1 : 0);
    count = tl - tf + 1;
  }
  __device__ __forceinline__ int tile(int i) const {
    if (i < np) return (ls && i == 0) ? tl : tf;
    return tf + (fs ? 1 : 0) + (i - np);
  }
};

// Stage = one tile's rows over a block range [b0, b0 + nbs) of the CTA's units.
struct GemvStage {
  int lt;   // processing index of the tile within the CTA
  int tau;  // global tile
  int r0;   // first row of the tile within its segment
  int ks;   // CTA-local index of the stage's first unit
  int sg, b0, nbs, nr;
};

__device__ __forceinline__ int seg_of_tile(const QGemvArgs &a, int tau) {
  int sg = 0;
  while (sg + 1 < a.nseg && tau >= a.seg[sg + 1].tile0) ++sg;
  return sg;
}

// Cursor over the CTA's stages (the producer and every consumer warp walk the same sequence).
struct StageWalk {
  int i, b, hi, tau, sg, ku;
  __device__ __forceinline__ void set_tile(const QGemvArgs &a, const CtaTiles &ct) {
    tau = ct.tile(i);
    const int base = tau * a.nb;
    b = ct.u0 > base ? ct.u0 - base : 0;
    hi = ct.u1 - base < a.nb ? ct.u1 - base : a.nb;
    sg = seg_of_tile(a, tau);
  }
  __device__ __forceinline__ void init(const QGemvArgs &a, const CtaTiles &ct) {
    i = 0;
    ku = 0;
    set_tile(a, ct);
  }
  __device__ __forceinline__ bool more(const CtaTiles &ct) const { return i < ct.count; }
  __device__ __forceinline__ void next(const QGemvArgs &a, const CtaTiles &ct, GemvStage &s) {
    const GemvSegK &S = a.seg[sg];
    s.lt = i;
    s.tau = tau;
    s.b0 = b;
    s.sg = sg;
    s.ks = ku;
    const int n = S.nbs < hi - b ? S.nbs : hi - b;
    s.nbs = n;
    s.r0 = (tau - S.tile0) * GEMV_TILE;
    s.nr = S.rows - s.r0 < GEMV_TILE ? S.rows - s.r0 : GEMV_TILE;
    ku += n;
    b += n;
    if (b == hi && ++i < ct.count) set_tile(a, ct);
  }
};

// Called by a warp after each unit of a shared tile (processing index lt < np).  The warp that
// completes the CTA's part of the tile sums its rows over the CTA's blocks, publishes the partial
// sums for the neighbour, and, if the neighbour's part is already published, writes the outputs:
// lower part (blocks from 0) + upper part, in that order whichever CTA finishes second.
template <int NMAT, int T>
__device__ __forceinline__ void finish_shared(const QGemvArgs &a, const CtaTiles &ct, int lt, int tau, int cta,
                                           const float *red, int *s_done, int lane) {
  const int nb = a.nb;
  __syncwarp();
  int old = 0;
  if (lane == 0) {
    __threadfence_block();
    old = atomicAdd(&s_done[lt], 1);
  }
  old = __shfl_sync(0xFFFFFFFFu, old, 0);
  const int base = tau * nb;
  const int lo = ct.u0 > base ? ct.u0 - base : 0, hi = ct.u1 - base < nb ? ct.u1 - base : nb;
  if (old != hi - lo - 1) return;
  __syncwarp();
  __threadfence_block();
  const bool upper = ct.fs && tau == ct.tf;  // blocks [lo, nb) here, [0, lo) in CTA cta-1
  const int bslot = upper ? cta - 1 : cta;
  float *mine = a.part + bslot * GEMV_SPLIT_SLOT + (upper ? GEMV_SPLIT_SLOT / 2 : 0);
  const float *other = a.part + bslot * GEMV_SPLIT_SLOT + (upper ? 0 : GEMV_SPLIT_SLOT / 2);
  const int row = lane & 15, kk = lane >> 4;
  float vm[NMAT];
  if (kk < T) {
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float *p = red + (((lt * GEMV_TILE + row) * NMAT + m) * T + kk) * nb;
      float sum = 0.f;
      for (int bb = lo; bb < hi; ++bb) sum += p[bb];
      vm[m] = sum;
      mine[(row * NMAT + m) * T + kk] = sum;
    }
  }
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    __threadfence();  // this warp's partials, then the arrival
    last = atomicAdd(&a.cnt[bslot], 1u) == 1u;
    if (last) {
      a.cnt[bslot] = 0;  // both parts are in: reset for the next launch
      __threadfence();
    }
  }
  last = __shfl_sync(0xFFFFFFFFu, last, 0);
  __syncwarp();
  if (!last || kk >= T) return;
  const GemvSegK &S = a.seg[seg_of_tile(a, tau)];
  const int r = (tau - S.tile0) * GEMV_TILE + row;
  if (r >= S.rows) return;
  float w[NMAT];
#pragma unroll
  for (int m = 0; m < NMAT; ++m) {
    const float o = __ldcg(other + (row * NMAT + m) * T + kk);
    w[m] = upper ? o + vm[m] : vm[m] + o;
  }
  S.y[int64_t(kk) * S.ldy + r] = NMAT == 2 ? gelu_tanh_mul(w[0], w[NMAT - 1]) : w[0];
}

// ---------------------------------------------------------------- phase building blocks
// Position in the stage ring: slot and mbarrier phase of the next stage (producer and consumers
// each keep one; they advance through the same stage sequence).
struct RingPos {
  int slot, phase;
  __device__ __forceinline__ void advance(int nstage) {
    if (++slot == nstage) {
      slot = 0;
      phase ^= 1;
    }
  }
};

// Fills the CTA's stage table (thread 0); returns the stage count.
__device__ __forceinline__ int build_stage_table(const QGemvArgs &a, const CtaTiles &ct, GemvStage *tab) {
  StageWalk wk;
  wk.init(a, ct);
  int n = 0;
  while (wk.more(ct) && n < a.max_stages) wk.next(a, ct, tab[n++]);
  if (wk.more(ct) && a.err) atomicExch(a.err, DEV_BAD_ARG);
  return n;
}

// Producer warp of a one-projection launch: walks the CTA's stages itself (the same walk that fills
// the consumers' table) so the first copies leave without waiting for the table.
template <int NMAT>
__device__ __forceinline__ void produce_walk(const QGemvArgs &a, const CtaTiles &ct, uint8_t *ring, uint64_t *full,
                                             uint64_t *empty, int lane) {
  StageWalk wk;
  wk.init(a, ct);
  RingPos rp = {0, 0};
  for (int s = 0; wk.more(ct) && s < a.max_stages; ++s) {
    GemvStage st;
    wk.next(a, ct, st);
    if (s >= a.nstage) {  // wait for the slot's previous stage to be consumed
      if (lane == 0) mbar_wait_bounded(&empty[rp.slot], uint32_t(rp.phase ^ 1), a.err);
      __syncwarp();
    }
    if (lane == 0) {
      const GemvSegK &S = a.seg[st.sg];
      const uint32_t bytes = uint32_t(st.nbs) * uint32_t(S.rec);
      const int64_t first = int64_t(st.tau - S.tile0) * a.nb + st.b0;
      mbar_arrive_expect_tx(&full[rp.slot], bytes * NMAT);
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
        bulk_g2s(ring + size_t(rp.slot) * a.stage_bytes + m * S.nbs * S.rec, S.w[m] + first * S.rec, bytes,
                 &full[rp.slot]);
    }
    __syncwarp();
    rp.advance(a.nstage);
  }
}

// Activations of T tokens into the CTA's image X (consumer warps; ends with a consumer barrier).
// Unit (token t, 256-block b) belongs to warp (t*nb + b) % CW and lane l holds its elements
// 8l..8l+7, so every global access is a coalesced 1 KB piece of a row.  The optional fused
// residual add + RMSNorm passes run first.
template <int T, int CW>
__device__ __forceinline__ void build_x(const GemvPrologue &P, int nb, int cta, const XSmem &X,
                                        float (*pro_red)[16], int warp, int lane) {
  const int K = nb * QK_K;
  const int units = T * nb;
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
      for (int e = 0; e < 8; ++e) v[e] = resid_add(v[e], s1t, P.w_post, wp[e], rs[e], P.scale, sc);
    }
    if (step == 1 || !P.w_next) return;
    const float s2t = (T == 1 || t == 0) ? s2[0] : s2[T - 1];
    float wn[8];
    load8(P.w_next, col, wn);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (v[e] * s2t) * wn[e];
  };
  // per-token sums of v^2 after `step` steps in the residual-stream norm order (block_sumsq per
  // unit, then the block sums in block order); the block sums pass through the start of X, which
  // is written only after the norm passes
  float *bsum = reinterpret_cast<float *>(X.frag);
  auto cta_sumsq = [&](int step, bool store_resid, float (&out)[T]) {
    for (int u = warp; u < units; u += CW) {
      const int t = u / nb, b = u % nb;
      float v[8];
      value8(t, b, step, v);
      const float s = block_sumsq(v);
      if (lane == 0) bsum[u] = s;
      if (store_resid) store8(P.resid_out + int64_t(t) * K + b * QK_K + lane * 8, v);
    }
    consumer_bar<CW>();
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float sum = 0.f;
      for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, bsum[t * nb + b]);
      out[t] = sum;
    }
    consumer_bar<CW>();
  };
  if (P.mode != 0 && units <= CW) {
    // one unit per warp at most: every input is loaded once into registers, then the norm passes
    // run on them (the same arithmetic in the same order as the general path below)
    const bool has = warp < units;
    const int t = has ? warp / nb : 0, b = has ? warp % nb : 0;
    const int64_t off = int64_t(t) * K + b * QK_K + lane * 8;
    const int col = b * QK_K + lane * 8;
    float v[8], wp[8], rs[8], wn[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = wp[e] = rs[e] = wn[e] = 0.f;
    if (has) {
      load8(P.a, off, v);
      if (P.mode == 2) {
        if (P.w_post) load8(P.w_post, col, wp);
        load8(P.resid_in, off, rs);
      }
      if (P.w_next) load8(P.w_next, col, wn);
    }
    // per-token CTA sum in the residual-stream norm order: warp = t * nb + b, so the warps of a
    // token hold its block sums in block order (the other warps add zeros)
    auto reduce = [&](const float (&vq)[8], float (&out)[T]) {
      const float bs = block_sumsq(vq);
#pragma unroll
      for (int tt = 0; tt < T; ++tt) {
        const float w = (T == 1 || tt == t) ? bs : 0.f;
        if (lane == 0) pro_red[tt][warp] = has ? w : 0.f;
      }
      consumer_bar<CW>();
#pragma unroll
      for (int tt = 0; tt < T; ++tt) {
        float sum = 0.f;
        for (int w = 0; w < CW; ++w) sum = __fadd_rn(sum, pro_red[tt][w]);
        out[tt] = sum;
      }
      consumer_bar<CW>();
    };
    float tot[T];
    if (P.mode == 1 || P.w_post) {
      reduce(v, tot);
#pragma unroll
      for (int tt = 0; tt < T; ++tt) s1[tt] = 1.0f / sqrtf(tot[tt] / float(K) + P.eps);
    }
    const float s1t = (T == 1 || t == 0) ? s1[0] : s1[T - 1];
    if (P.mode == 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = v[e] * s1t;
    } else {
      const float sc = P.scale ? P.scale[0] : 1.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = resid_add(v[e], s1t, P.w_post, wp[e], rs[e], P.scale, sc);
      if (P.w_next || (P.resid_out && cta == 0)) {
        if (P.resid_out && cta == 0 && has) store8(P.resid_out + off, v);
        reduce(v, tot);
#pragma unroll
        for (int tt = 0; tt < T; ++tt) s2[tt] = 1.0f / sqrtf(tot[tt] / float(K) + P.eps);
      }
    }
    if (P.w_next) {
      const float s2t = (T == 1 || t == 0) ? s2[0] : s2[T - 1];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (v[e] * s2t) * wn[e];
    }
    if (has) emit_block<T>(v, lane, b, t, X);
    consumer_bar<CW>();
    return;
  }
  if (P.mode != 0) {
    float tot[T];
    if (P.mode == 1 || P.w_post) {
      cta_sumsq(0, false, tot);
#pragma unroll
      for (int t = 0; t < T; ++t) s1[t] = 1.0f / sqrtf(tot[t] / float(K) + P.eps);
    }
    if (P.mode == 2 && (P.w_next || (P.resid_out && cta == 0))) {
      cta_sumsq(1, P.resid_out && cta == 0, tot);
#pragma unroll
      for (int t = 0; t < T; ++t) s2[t] = 1.0f / sqrtf(tot[t] / float(K) + P.eps);
    }
  }
  for (int u = warp; u < units; u += CW) {
    const int t = u / nb, b = u % nb;
    float v[8];
    value8(t, b, 2, v);
    emit_block<T>(v, lane, b, t, X);
  }
  consumer_bar<CW>();
}

// Consumer warps: the CTA's units of one GEMV (CTA-local unit k, in stage order with blocks
// fastest, belongs to warp k % CW).  rp: ring position of the table's first stage (the same in
// every warp); s_sdone: per-slot counters of finished units.
template <int NMAT, int T, int TYPE, int CW>
__device__ __forceinline__ void run_units(const QGemvArgs &a, const CtaTiles &ct, const GemvStage *tab, RingPos rp,
                                          const uint8_t *ring, uint64_t *full, uint64_t *empty, int *s_sdone,
                                          const XSmem &X, float *red, int *s_tdone, int cta, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int total = ct.u1 - ct.u0;
  for (int k = warp, si = 0; k < total; k += CW) {
    while (k >= tab[si].ks + tab[si].nbs) {
      ++si;
      rp.advance(a.nstage);
    }
    const GemvStage st = tab[si];
    mbar_wait_bounded(&full[rp.slot], uint32_t(rp.phase), a.err);
    const GemvSegK &S = a.seg[st.sg];
    const uint8_t *tile = ring + size_t(rp.slot) * a.stage_bytes;
    const int b = st.b0 + (k - st.ks);
    float v[NMAT][2][T];
    if (TYPE == T_Q4_K || (TYPE == 0 && S.type == T_Q4_K))
      unit_q4k<NMAT, T>(tile, S.nbs * S.rec, b - st.b0, b, X, g, t, v);
    else
      unit_q6k<NMAT, T>(tile, S.nbs * S.rec, b - st.b0, b, X, g, t, v);
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int kk = 0; kk < T; ++kk) {
          float x = v[m][i][kk];
          x += __shfl_xor_sync(0xFFFFFFFFu, x, 1);
          x += __shfl_xor_sync(0xFFFFFFFFu, x, 2);
          if (t == 0) red[(((st.lt * GEMV_TILE + g + 8 * i) * NMAT + m) * T + kk) * a.nb + b] = x;
        }
    // release the ring slot once every unit of its stage is done (its reads precede the count)
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&s_sdone[rp.slot], 1) == st.nbs - 1) {
        s_sdone[rp.slot] = 0;
        __threadfence_block();
        mbar_arrive_cta(&empty[rp.slot]);
      }
    }
    if (st.lt < ct.np) finish_shared<NMAT, T>(a, ct, st.lt, st.tau, cta, red, s_tdone, lane);
  }
}

// Consumer threads (after a consumer barrier): outputs of the tiles the CTA owns alone, row sums
// over all blocks in block order.
template <int NMAT, int T, int CW>
__device__ __forceinline__ void finish_owned(const QGemvArgs &a, const CtaTiles &ct, const float *red, int tid) {
  const int nb = a.nb;
  for (int item = tid; item < (ct.count - ct.np) * GEMV_TILE * T; item += CW * 32) {
    const int kk = item % T, row = (item / T) % GEMV_TILE, lt = ct.np + item / (T * GEMV_TILE);
    const int tau = ct.tile(lt);
    const GemvSegK &S = a.seg[seg_of_tile(a, tau)];
    const int r = (tau - S.tile0) * GEMV_TILE + row;
    if (r >= S.rows) continue;
    float vm[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float *p = red + (((lt * GEMV_TILE + row) * NMAT + m) * T + kk) * nb;
      float sum = 0.f;
      for (int bb = 0; bb < nb; ++bb) sum += p[bb];
      vm[m] = sum;
    }
    S.y[int64_t(kk) * S.ldy + r] = NMAT == 2 ? gelu_tanh_mul(vm[0], vm[NMAT - 1]) : vm[0];
  }
}

}  // namespace sfc
