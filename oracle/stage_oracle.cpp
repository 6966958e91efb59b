// stage_oracle.cpp — CPU oracle (test infrastructure only; see stage_oracle.h).
//
// Restates the arithmetic of the reference Rust CPU path. Citations are to
// crates/stage-forward-lab/src/<file>:<line> of Compute-Network/compute-sharding.
// Build: oracle/Makefile (g++ -O2 -ffp-contract=off).

#include "stage_oracle.h"

#include <math.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

namespace {

constexpr int QK_K = 256;              // quants.rs:10
constexpr int K_SCALE_SIZE = 12;       // quants.rs:11
constexpr int BLOCK_Q4_K = 144;        // quants.rs:19
constexpr int BLOCK_Q5_K = 176;        // quants.rs:20
constexpr int BLOCK_Q6_K = 210;        // quants.rs:21

// Run fn(lo, hi) over [0, n) split into contiguous chunks on `threads` threads.
template <class F>
void parallel_rows(int64_t n, int threads, F fn) {
  if (threads <= 1 || n < 64) {
    fn(int64_t(0), n);
    return;
  }
  int64_t nt = std::min<int64_t>(threads, n);
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (int64_t t = 0; t < nt; ++t) {
    int64_t lo = n * t / nt, hi = n * (t + 1) / nt;
    pool.emplace_back([=] { fn(lo, hi); });
  }
  for (auto &th : pool) th.join();
}

inline float h2f(const uint8_t *p) { return or_fp16_to_f32(uint16_t(p[0] | (p[1] << 8))); }

// quants.rs:252-261 get_scale_min_k4
inline void get_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// quants.rs:181-208
void dequant_q4k_block(const uint8_t *b, float *out) {
  float d = h2f(b), dmin = h2f(b + 2);
  const uint8_t *scales = b + 4, *qs = b + 4 + K_SCALE_SIZE;
  int is = 0, qo = 0;
  for (int j = 0; j < QK_K; j += 64) {
    uint8_t sc, m;
    get_scale_min_k4(is, scales, &sc, &m);
    float d1 = d * float(sc), m1 = dmin * float(m);
    get_scale_min_k4(is + 1, scales, &sc, &m);
    float d2 = d * float(sc), m2 = dmin * float(m);
    for (int l = 0; l < 32; ++l) {
      uint8_t q = qs[qo + l];
      out[j + l] = d1 * float(q & 0x0F) - m1;
      out[j + 32 + l] = d2 * float(q >> 4) - m2;
    }
    qo += 32;
    is += 2;
  }
}

// quants.rs:119-159
void dequant_q5k_block(const uint8_t *b, float *out) {
  float d = h2f(b), dmin = h2f(b + 2);
  const uint8_t *scales = b + 4, *qh = b + 4 + K_SCALE_SIZE, *qs = qh + QK_K / 8;
  int is = 0, qo = 0;
  uint8_t u1 = 1, u2 = 2;
  for (int j = 0; j < QK_K; j += 64) {
    uint8_t sc, m;
    get_scale_min_k4(is, scales, &sc, &m);
    float d1 = d * float(sc), m1 = dmin * float(m);
    get_scale_min_k4(is + 1, scales, &sc, &m);
    float d2 = d * float(sc), m2 = dmin * float(m);
    for (int l = 0; l < 32; ++l) {
      uint8_t ql = qs[qo + l], hb = qh[l];
      float h1 = (hb & u1) ? 16.f : 0.f, h2 = (hb & u2) ? 16.f : 0.f;
      out[j + l * 2] = d1 * (float(ql & 0x0F) + h1) - m1;
      out[j + l * 2 + 1] = d2 * (float(ql >> 4) + h2) - m2;
    }
    qo += 32;
    is += 2;
    u1 <<= 2;
    u2 <<= 2;
  }
}

inline int q6_val(const uint8_t *ql, const uint8_t *qh, int half, int l, int g) {
  // quants.rs:229-240 (q1..q4 of one 128-element half)
  uint8_t h = qh[half * 32 + l];
  const uint8_t *lq = ql + half * 64;
  switch (g) {
    case 0: return int((lq[l] & 0x0F) | (((h >> 0) & 3) << 4)) - 32;
    case 1: return int((lq[32 + l] & 0x0F) | (((h >> 2) & 3) << 4)) - 32;
    case 2: return int(((lq[l] >> 4) & 0x0F) | (((h >> 4) & 3) << 4)) - 32;
    default: return int(((lq[32 + l] >> 4) & 0x0F) | (((h >> 6) & 3) << 4)) - 32;
  }
}

// quants.rs:210-249
void dequant_q6k_block(const uint8_t *b, float *out) {
  const uint8_t *ql = b, *qh = b + 128;
  const int8_t *sc = (const int8_t *)(b + 192);
  float d = h2f(b + 208);
  for (int half = 0; half < 2; ++half)
    for (int l = 0; l < 32; ++l) {
      int is = l / 16;
      for (int g = 0; g < 4; ++g)
        out[half * 128 + g * 32 + l] = d * float(sc[half * 8 + is + 2 * g]) * float(q6_val(ql, qh, half, l, g));
    }
}

// Q4_K row dot, per-row order of dot_many_q4_k_four_blocks_with_offset (quants.rs:1850-1904):
// sum += a1 * left + a2 * right, accumulated across all blocks of the row.
float dot_q4k_row(const uint8_t *row, int64_t nb, const float *x) {
  float sum = 0.f;
  for (int64_t bi = 0; bi < nb; ++bi) {
    const uint8_t *b = row + bi * BLOCK_Q4_K;
    const float *xb = x + bi * QK_K;
    float d = h2f(b), dmin = h2f(b + 2);
    const uint8_t *scales = b + 4, *qs = b + 16;
    for (int j = 0, is = 0; j < QK_K; j += 64, is += 2) {
      uint8_t sc, m;
      get_scale_min_k4(is, scales, &sc, &m);
      float d1 = d * float(sc), m1 = dmin * float(m);
      get_scale_min_k4(is + 1, scales, &sc, &m);
      float d2 = d * float(sc), m2 = dmin * float(m);
      for (int l = 0; l < 32; ++l) {
        uint8_t q = qs[j / 2 + l];
        float a1 = d1 * float(q & 0x0F) - m1;
        float a2 = d2 * float(q >> 4) - m2;
        sum += a1 * xb[j + l] + a2 * xb[j + 32 + l];
      }
    }
  }
  return sum;
}

// Q6_K row dot, per-row order of dot_many_q6_k_two_blocks_with_offset (quants.rs:2620-2688).
float dot_q6k_row(const uint8_t *row, int64_t nb, const float *x) {
  float sum = 0.f;
  for (int64_t bi = 0; bi < nb; ++bi) {
    const uint8_t *b = row + bi * BLOCK_Q6_K;
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = h2f(b + 208);
    for (int half = 0; half < 2; ++half) {
      float sf[8];
      for (int k = 0; k < 8; ++k) sf[k] = d * float(sc[half * 8 + k]);
      const float *xb = x + bi * QK_K + half * 128;
      for (int l = 0; l < 32; ++l) {
        int s = l / 16;
        float q1 = float(q6_val(ql, qh, half, l, 0)), q2 = float(q6_val(ql, qh, half, l, 1));
        float q3 = float(q6_val(ql, qh, half, l, 2)), q4 = float(q6_val(ql, qh, half, l, 3));
        sum += sf[s] * q1 * xb[l] + sf[s + 2] * q2 * xb[32 + l] + sf[s + 4] * q3 * xb[64 + l] +
               sf[s + 6] * q4 * xb[96 + l];
      }
    }
  }
  return sum;
}

// quants.rs:1317-1330 (F16) and real_math.rs:136-141 (F32): sequential sum of w*x.
float dot_f16_row(const uint8_t *row, int64_t n, const float *x) {
  float sum = 0.f;
  for (int64_t i = 0; i < n; ++i) sum += h2f(row + 2 * i) * x[i];
  return sum;
}
float dot_f32_row(const uint8_t *row, int64_t n, const float *x) {
  float sum = 0.f;
  for (int64_t i = 0; i < n; ++i) {
    float w;
    memcpy(&w, row + 4 * i, 4);
    sum += w * x[i];
  }
  return sum;
}
float dot_bf16_row(const uint8_t *row, int64_t n, const float *x) {
  float sum = 0.f;
  for (int64_t i = 0; i < n; ++i) {
    uint32_t bits = uint32_t(row[2 * i] | (row[2 * i + 1] << 8)) << 16;
    float w;
    memcpy(&w, &bits, 4);
    sum += w * x[i];
  }
  return sum;
}

float dot_row(int type, const uint8_t *row, int64_t in_dim, const float *x) {
  switch (type) {
    case OR_TYPE_Q4_K: return dot_q4k_row(row, in_dim / QK_K, x);
    case OR_TYPE_Q6_K: return dot_q6k_row(row, in_dim / QK_K, x);
    case OR_TYPE_F16: return dot_f16_row(row, in_dim, x);
    case OR_TYPE_F32: return dot_f32_row(row, in_dim, x);
    case OR_TYPE_BF16: return dot_bf16_row(row, in_dim, x);
    case OR_TYPE_Q5_K: {
      // Q5_K has no dedicated fast path on the hot path; dequantize then sum.
      std::vector<float> w(in_dim);
      for (int64_t b = 0; b < in_dim / QK_K; ++b) dequant_q5k_block(row + b * BLOCK_Q5_K, &w[b * QK_K]);
      float sum = 0.f;
      for (int64_t i = 0; i < in_dim; ++i) sum += w[i] * x[i];
      return sum;
    }
  }
  return 0.f;
}

}  // namespace

extern "C" {

int64_t or_bytes_per_row(int type, int64_t in_dim) {
  if (in_dim <= 0) return 0;
  switch (type) {
    case OR_TYPE_F32: return in_dim * 4;
    case OR_TYPE_F16:
    case OR_TYPE_BF16: return in_dim * 2;
    case OR_TYPE_Q4_K: return in_dim % QK_K ? 0 : in_dim / QK_K * BLOCK_Q4_K;
    case OR_TYPE_Q5_K: return in_dim % QK_K ? 0 : in_dim / QK_K * BLOCK_Q5_K;
    case OR_TYPE_Q6_K: return in_dim % QK_K ? 0 : in_dim / QK_K * BLOCK_Q6_K;
  }
  return 0;
}

float or_fp16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400));
      bits = sign | (uint32_t(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t or_f32_to_fp16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  uint32_t absx = x & 0x7FFFFFFF;
  if (absx >= 0x7F800000) return uint16_t(sign | 0x7C00 | (absx > 0x7F800000 ? 0x200 : 0));
  if (absx >= 0x477FF000) return uint16_t(sign | 0x7C00);  // rounds to inf
  if (absx < 0x33000001) return uint16_t(sign);            // < half of min subnormal -> 0
  int e = int(absx >> 23);
  uint32_t man = (absx & 0x7FFFFF) | 0x800000;
  int shift;  // bits to drop from the 24-bit significand
  uint32_t hexp;
  if (e < 113) {  // subnormal half
    shift = 13 + (113 - e);
    hexp = 0;
  } else {
    shift = 13;
    hexp = uint32_t(e - 112);
  }
  uint32_t q = man >> shift;
  uint32_t rem = man & ((1u << shift) - 1), halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (q & 1))) ++q;
  uint32_t out;
  if (hexp == 0) {
    out = q;  // may carry into the exponent field, which is correct
  } else {
    out = (hexp << 10) + (q - 0x400);  // q includes the hidden bit
    if (q == 0x800) out = ((hexp + 1) << 10);
  }
  return uint16_t(sign | out);
}

int or_dequantize_rows(int type, const uint8_t *raw, int64_t n_rows, int64_t in_dim, float *out) {
  int64_t rb = or_bytes_per_row(type, in_dim);
  if (rb == 0 || n_rows < 0) return -1;
  for (int64_t r = 0; r < n_rows; ++r) {
    const uint8_t *row = raw + r * rb;
    float *o = out + r * in_dim;
    switch (type) {
      case OR_TYPE_Q4_K:
        for (int64_t b = 0; b < in_dim / QK_K; ++b) dequant_q4k_block(row + b * BLOCK_Q4_K, o + b * QK_K);
        break;
      case OR_TYPE_Q5_K:
        for (int64_t b = 0; b < in_dim / QK_K; ++b) dequant_q5k_block(row + b * BLOCK_Q5_K, o + b * QK_K);
        break;
      case OR_TYPE_Q6_K:
        for (int64_t b = 0; b < in_dim / QK_K; ++b) dequant_q6k_block(row + b * BLOCK_Q6_K, o + b * QK_K);
        break;
      case OR_TYPE_F16:
        for (int64_t i = 0; i < in_dim; ++i) o[i] = h2f(row + 2 * i);
        break;
      case OR_TYPE_BF16:
        for (int64_t i = 0; i < in_dim; ++i) {
          uint32_t bits = uint32_t(row[2 * i] | (row[2 * i + 1] << 8)) << 16;
          memcpy(&o[i], &bits, 4);
        }
        break;
      case OR_TYPE_F32:
        memcpy(o, row, size_t(in_dim) * 4);
        break;
      default:
        return -1;
    }
  }
  return 0;
}

}  // extern "C"

namespace {

// Eight tokens side by side: lane t is token t's running sum, so each lane sees exactly the
// operations (and roundings) of dot_row for its token; no lane ever mixes with another.
typedef float v8f __attribute__((vector_size(32)));

// A row's terms in dot_row order.  Q4_K: per (block, 64-element group j, l) the pair
// (a1, a2) = (d1*q_lo - m1, d2*q_hi - m2) applied as sum += a1*x[j+l] + a2*x[j+32+l]
// (quants.rs:1878-1904).  Q6_K: per (block, half, l) the four products sf*q applied as
// sum += ((w1*x1 + w2*x2) + w3*x3) + w4*x4 (quants.rs:2640-2688).  Others: w[i], sum += w*x.
void row_terms(int type, const uint8_t *row, int64_t in_dim, float *w) {
  const int64_t nb = in_dim / QK_K;
  if (type == OR_TYPE_Q4_K) {
    for (int64_t bi = 0; bi < nb; ++bi) {
      const uint8_t *b = row + bi * BLOCK_Q4_K;
      const float d = h2f(b), dmin = h2f(b + 2);
      const uint8_t *scales = b + 4, *qs = b + 16;
      float *o = w + bi * QK_K;
      for (int j = 0, is = 0; j < QK_K; j += 64, is += 2) {
        uint8_t sc, m;
        get_scale_min_k4(is, scales, &sc, &m);
        const float d1 = d * float(sc), m1 = dmin * float(m);
        get_scale_min_k4(is + 1, scales, &sc, &m);
        const float d2 = d * float(sc), m2 = dmin * float(m);
        for (int l = 0; l < 32; ++l) {
          const uint8_t q = qs[j / 2 + l];
          o[j + l] = d1 * float(q & 0x0F) - m1;
          o[j + 32 + l] = d2 * float(q >> 4) - m2;
        }
      }
    }
  } else if (type == OR_TYPE_Q6_K) {
    for (int64_t bi = 0; bi < nb; ++bi) {
      const uint8_t *b = row + bi * BLOCK_Q6_K;
      const uint8_t *ql = b, *qh = b + 128;
      const int8_t *sc = (const int8_t *)(b + 192);
      const float d = h2f(b + 208);
      float *o = w + bi * QK_K;
      for (int half = 0; half < 2; ++half) {
        float sf[8];
        for (int k = 0; k < 8; ++k) sf[k] = d * float(sc[half * 8 + k]);
        for (int l = 0; l < 32; ++l) {
          const int s = l / 16;
          for (int g = 0; g < 4; ++g) o[half * 128 + g * 32 + l] = sf[s + 2 * g] * float(q6_val(ql, qh, half, l, g));
        }
      }
    }
  } else {
    or_dequantize_rows(type, row, 1, in_dim, w);
  }
}

__attribute__((target_clones("avx2", "default")))
void dot_terms8(int type, const float *w, int64_t in_dim, const v8f *X, v8f &out) {
  v8f sum = {0, 0, 0, 0, 0, 0, 0, 0};
  if (type == OR_TYPE_Q4_K) {
    for (int64_t base = 0; base < in_dim; base += 64)
      for (int l = 0; l < 32; ++l) sum = sum + (w[base + l] * X[base + l] + w[base + 32 + l] * X[base + 32 + l]);
  } else if (type == OR_TYPE_Q6_K) {
    for (int64_t base = 0; base < in_dim; base += 128)
      for (int l = 0; l < 32; ++l)
        sum = sum + (((w[base + l] * X[base + l] + w[base + 32 + l] * X[base + 32 + l]) +
                      w[base + 64 + l] * X[base + 64 + l]) +
                     w[base + 96 + l] * X[base + 96 + l]);
  } else {
    for (int64_t i = 0; i < in_dim; ++i) sum = sum + w[i] * X[i];
  }
  out = sum;
}

}  // namespace

extern "C" {

int or_matmul(int type, const uint8_t *raw, int64_t out_dim, int64_t in_dim, const float *x,
              int64_t n_tok, float *y, int threads) {
  int64_t rb = or_bytes_per_row(type, in_dim);
  if (rb == 0 || out_dim < 0 || n_tok < 0) return -1;
  if (n_tok >= 2 && type != OR_TYPE_Q5_K) {
    // Several tokens: a row's terms are formed once and applied to 8 tokens per pass, with each
    // token's sum in the exact order of dot_row (bit-identical to the one-token loop below).
    const int64_t ng = (n_tok + 7) / 8;
    std::vector<v8f> xt(size_t(ng * in_dim));
    for (int64_t g = 0; g < ng; ++g)
      for (int64_t k = 0; k < in_dim; ++k) {
        v8f v = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int t = 0; t < 8 && g * 8 + t < n_tok; ++t) v[t] = x[(g * 8 + t) * in_dim + k];
        xt[size_t(g * in_dim + k)] = v;
      }
    parallel_rows(out_dim, threads, [&](int64_t lo, int64_t hi) {
      std::vector<float> w(static_cast<size_t>(in_dim));
      for (int64_t r = lo; r < hi; ++r) {
        row_terms(type, raw + r * rb, in_dim, w.data());
        for (int64_t g = 0; g < ng; ++g) {
          v8f s;
          dot_terms8(type, w.data(), in_dim, xt.data() + g * in_dim, s);
          for (int t = 0; t < 8 && g * 8 + t < n_tok; ++t) y[(g * 8 + t) * out_dim + r] = s[t];
        }
      }
    });
    return 0;
  }
  parallel_rows(out_dim, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; ++r)
      for (int64_t t = 0; t < n_tok; ++t) y[t * out_dim + r] = dot_row(type, raw + r * rb, in_dim, x + t * in_dim);
  });
  return 0;
}

void or_rms_norm_inplace(float *x, int64_t n, const float *w, int64_t wlen, float eps) {
  if (n == 0) return;
  float mean_sq = 0.f;
  for (int64_t i = 0; i < n; ++i) mean_sq += x[i] * x[i];
  mean_sq = mean_sq / float(n);
  float scale = 1.0f / sqrtf(mean_sq + eps);
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] * scale * w[wlen == n ? i : i % wlen];
}

void or_per_head_rms_norm(float *x, const float *w, int64_t wlen, int n_heads, int head_dim, float eps) {
  for (int h = 0; h < n_heads; ++h) {
    float *s = x + int64_t(h) * head_dim;
    float mean_sq = 0.f;
    for (int i = 0; i < head_dim; ++i) mean_sq += s[i] * s[i];
    mean_sq = mean_sq / float(head_dim);
    float scale = 1.0f / sqrtf(mean_sq + eps);
    if (w) {
      for (int i = 0; i < head_dim; ++i) s[i] *= scale * w[wlen == head_dim ? i : i % wlen];
    } else {
      for (int i = 0; i < head_dim; ++i) s[i] *= scale;
    }
  }
}

void or_gelu_tanh_mul_inplace(float *g, const float *u, int64_t n) {
  const float k = sqrtf(2.0f / 3.14159265358979323846f);
  for (int64_t i = 0; i < n; ++i) {
    float v = g[i];
    float inner = k * (v + 0.044715f * v * v * v);
    g[i] = 0.5f * v * (1.0f + tanhf(inner)) * u[i];
  }
}

void or_rope_apply(float *x, int n_heads, int head_dim, const float *freqs, int64_t n_freqs,
                   uint32_t position, float base_theta, int rotary_dim, int proportional) {
  int hd = head_dim & ~1;
  int rd = std::min(rotary_dim, hd) & ~1;
  if (rd == 0 || hd == 0) return;
  int n_ang = rd / 2;
  float denom = proportional ? float(hd) : float(rd);
  float pos = float(position);
  std::vector<float> cs(n_ang), sn(n_ang);
  for (int i = 0; i < n_ang; ++i) {
    float inv_freq = 1.0f / powf(base_theta, 2.0f * float(i) / denom);
    float fs = i < n_freqs ? freqs[i] : 1.0f;
    float theta = pos * inv_freq * fs;
    cs[i] = cosf(theta);
    sn[i] = sinf(theta);
  }
  int half = hd / 2;
  for (int h = 0; h < n_heads; ++h) {
    float *b = x + int64_t(h) * head_dim;
    for (int i = 0; i < n_ang; ++i) {
      float x0 = b[i], x1 = b[half + i];
      b[i] = x0 * cs[i] - x1 * sn[i];
      b[half + i] = x0 * sn[i] + x1 * cs[i];
    }
  }
}

// Cached key / value rows come either as one [n_pos][n_kv * head_dim] matrix or as one pointer per
// row (the stage driver's per-position rows, read in place); the arithmetic is the same.
extern "C++" {
template <typename KRow, typename VRow>
static void gqa_attention_impl(const float *q, KRow krow, VRow vrow, int64_t n_pos, int64_t limit, int64_t window,
                               int n_heads, int n_kv, int head_dim, float *out) {
  int groups = n_heads / n_kv;
  int64_t seq_len = limit >= 0 ? std::min(limit, n_pos) : n_pos;
  for (int64_t i = 0; i < int64_t(n_heads) * head_dim; ++i) out[i] = 0.f;
  if (seq_len <= 0) return;
  int64_t w0 = window > 0 ? std::max<int64_t>(0, seq_len - window) : 0;
  std::vector<float> scores(seq_len - w0);
  for (int h = 0; h < n_heads; ++h) {
    int kvh = h / groups;
    const float *qh = q + int64_t(h) * head_dim;
    for (int64_t t = w0; t < seq_len; ++t) {
      const float *k = krow(t) + int64_t(kvh) * head_dim;
      float s = 0.f;
      for (int d = 0; d < head_dim; ++d) s += qh[d] * k[d];
      scores[t - w0] = s;
    }
    // softmax, real_math.rs:93-104
    float mx = -INFINITY;
    for (float s : scores) mx = std::max(mx, s);
    float sum = 0.f;
    for (float &s : scores) {
      s = expf(s - mx);
      sum += s;
    }
    int64_t n = int64_t(scores.size());
    if (sum == 0.f) {
      for (float &s : scores) s = 1.0f / float(n);
    } else {
      for (float &s : scores) s = s / sum;
    }
    float *o = out + int64_t(h) * head_dim;
    for (int64_t t = w0; t < seq_len; ++t) {
      const float *v = vrow(t) + int64_t(kvh) * head_dim;
      float wt = scores[t - w0];
      for (int d = 0; d < head_dim; ++d) o[d] += wt * v[d];
    }
  }
}
}  // extern "C++"

void or_gqa_attention(const float *q, const float *kc, const float *vc, int64_t n_pos, int64_t limit,
                      int64_t window, int n_heads, int n_kv, int head_dim, float *out) {
  const int64_t row = int64_t(n_kv) * head_dim;
  gqa_attention_impl(
      q, [&](int64_t t) { return kc + t * row; }, [&](int64_t t) { return vc + t * row; }, n_pos, limit, window,
      n_heads, n_kv, head_dim, out);
}

void or_gqa_attention_rows(const float *q, const float *const *krows, const float *const *vrows, int64_t n_pos,
                           int64_t limit, int64_t window, int n_heads, int n_kv, int head_dim, float *out) {
  gqa_attention_impl(
      q, [&](int64_t t) { return krows[t]; }, [&](int64_t t) { return vrows[t]; }, n_pos, limit, window, n_heads,
      n_kv, head_dim, out);
}

void or_gqa_attention_rows_batch(const float *q, const float *const *krows, const float *const *vrows, int64_t n_pos,
                                 const int64_t *limits, int64_t n_tok, int64_t window, int n_heads, int n_kv,
                                 int head_dim, float *out, int threads) {
  const int64_t w = int64_t(n_heads) * head_dim;
  auto one = [&](int64_t lo, int64_t hi) {
    for (int64_t t = lo; t < hi; ++t)
      or_gqa_attention_rows(q + t * w, krows, vrows, n_pos, limits[t], window, n_heads, n_kv, head_dim, out + t * w);
  };
  if (threads <= 1 || n_tok < 2) {
    one(0, n_tok);
    return;
  }
  // tokens with more visible keys cost more: interleave them over the threads
  const int64_t nt = std::min<int64_t>(threads, n_tok);
  std::vector<std::thread> pool;
  for (int64_t k = 0; k < nt; ++k)
    pool.emplace_back([=, &one] {
      for (int64_t t = k; t < n_tok; t += nt) one(t, t + 1);
    });
  for (auto &th : pool) th.join();
}

int or_logits_top_k(int type, const uint8_t *raw, int64_t vocab, int64_t hidden, const float *h, int k,
                    float cap, int64_t *argmax_idx, float *argmax_score, int64_t *top_idx, float *top_score,
                    float *all_scores, int threads) {
  int64_t rb = or_bytes_per_row(type, hidden);
  if (rb == 0 || vocab <= 0) return -1;
  std::vector<float> sc(vocab);
  parallel_rows(vocab, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; ++r) {
      float s = dot_row(type, raw + r * rb, hidden, h);
      sc[r] = cap > 0.f ? cap * tanhf(s / cap) : s;  // real_math.rs:2442-2448
    }
  });
  // argmax: strict '>' in index order keeps the lowest index on ties (real_math.rs:2450-2456)
  int64_t best = 0;
  float bs = -INFINITY;
  for (int64_t r = 0; r < vocab; ++r)
    if (sc[r] > bs) {
      bs = sc[r];
      best = r;
    }
  *argmax_idx = best;
  *argmax_score = bs;
  // top-k: insertion before the first strictly smaller score (real_math.rs:2472-2488)
  if (k > 0) {
    std::vector<std::pair<int64_t, float>> top;
    for (int64_t r = 0; r < vocab; ++r) {
      float s = sc[r];
      size_t at = top.size();
      for (size_t i = 0; i < top.size(); ++i)
        if (s > top[i].second) {
          at = i;
          break;
        }
      if (at < size_t(k)) {
        top.insert(top.begin() + at, {r, s});
        if (top.size() > size_t(k)) top.pop_back();
      }
    }
    for (size_t i = 0; i < top.size(); ++i) {
      top_idx[i] = top[i].first;
      top_score[i] = top[i].second;
    }
    for (size_t i = top.size(); i < size_t(k); ++i) {
      top_idx[i] = -1;
      top_score[i] = -INFINITY;
    }
  }
  if (all_scores) memcpy(all_scores, sc.data(), size_t(vocab) * 4);
  return 0;
}

// ---- synthetic generators -------------------------------------------------
// Counter-based SplitMix64 finaliser; identical on host and device.
uint64_t or_mix64(uint64_t key, uint64_t ctr) {
  uint64_t z = key + (ctr + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t or_tensor_key(uint64_t seed, const char *name) {
  uint64_t h = 0xCBF29CE484222325ull;  // FNV-1a 64
  for (const unsigned char *p = (const unsigned char *)name; *p; ++p) {
    h ^= *p;
    h *= 0x100000001B3ull;
  }
  return or_mix64(seed, h);
}

// Irwin-Hall(4) approximation of N(0,1): four 16-bit uniforms, summed exactly in
// integers; scaled by 2^-16 (exact) and sqrt(3) (one rounding).
float or_synth_normal(uint64_t key, uint64_t ctr) {
  uint64_t u = or_mix64(key, ctr);
  int32_t s = int32_t(u & 0xFFFF) + int32_t((u >> 16) & 0xFFFF) + int32_t((u >> 32) & 0xFFFF) +
              int32_t((u >> 48) & 0xFFFF);
  float v = float(s - 131070);
  v = v * (1.0f / 65536.0f);
  return v * 1.7320508f;
}

int or_synth_tensor(int type, uint64_t key, int64_t n_rows, int64_t in_dim, float sigma, float mean,
                    uint8_t *out, int threads) {
  int64_t rb = or_bytes_per_row(type, in_dim);
  if (rb == 0) return -1;
  if (type == OR_TYPE_Q4_K || type == OR_TYPE_Q6_K) {
    int64_t nb = n_rows * (in_dim / QK_K);
    parallel_rows(nb, threads, [&](int64_t lo, int64_t hi) {
      for (int64_t b = lo; b < hi; ++b) {
        if (type == OR_TYPE_Q4_K) {
          uint8_t *p = out + b * BLOCK_Q4_K;
          uint64_t base = uint64_t(b) * 24;
          uint16_t d = or_f32_to_fp16(fabsf(or_synth_normal(key, base + 0)) * sigma);
          uint16_t dm = or_f32_to_fp16(fabsf(or_synth_normal(key, base + 1)) * sigma);
          p[0] = uint8_t(d);
          p[1] = uint8_t(d >> 8);
          p[2] = uint8_t(dm);
          p[3] = uint8_t(dm >> 8);
          for (int i = 0; i < 140; ++i) p[4 + i] = uint8_t(or_mix64(key, base + 2 + i / 8) >> (8 * (i % 8)));
        } else {
          uint8_t *p = out + b * BLOCK_Q6_K;
          uint64_t base = uint64_t(b) * 32;
          for (int i = 0; i < 208; ++i) p[i] = uint8_t(or_mix64(key, base + i / 8) >> (8 * (i % 8)));
          uint16_t d = or_f32_to_fp16(fabsf(or_synth_normal(key, base + 26)) * (sigma * 0.015625f));
          p[208] = uint8_t(d);
          p[209] = uint8_t(d >> 8);
        }
      }
    });
    return 0;
  }
  int64_t n = n_rows * in_dim;
  parallel_rows(n, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      float v = mean + or_synth_normal(key, uint64_t(i)) * sigma;
      if (type == OR_TYPE_F16) {
        uint16_t hb = or_f32_to_fp16(v);
        out[2 * i] = uint8_t(hb);
        out[2 * i + 1] = uint8_t(hb >> 8);
      } else if (type == OR_TYPE_F32) {
        memcpy(out + 4 * i, &v, 4);
      } else {  // BF16 by truncation-free RNE
        uint32_t bits;
        memcpy(&bits, &v, 4);
        uint32_t r = bits + 0x7FFF + ((bits >> 16) & 1);
        out[2 * i] = uint8_t(r >> 16);
        out[2 * i + 1] = uint8_t(r >> 24);
      }
    }
  });
  return 0;
}

}  // extern "C"
