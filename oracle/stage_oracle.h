/*
 * stage_oracle.h — CPU oracle for the stage-forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain C++ restatement of the reference's
 * Rust CPU path (crates/stage-forward-lab/src/{quants,real_math,real_forward}.rs)
 * used as the parity checker for the CUDA kernels. Only tests/, the smoke check
 * and the bench's CPU-baseline leg may load it; the product never does.
 *
 * Every function cites the reference file:line whose arithmetic it follows.
 * Compiled with -ffp-contract=off so that `a*b - c` stays two roundings, as in
 * Rust (which never contracts to FMA).
 */
#ifndef STAGE_ORACLE_H
#define STAGE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, crates/stage-forward-lab/src/quants.rs:12-17 */
enum {
  OR_TYPE_F32 = 0,
  OR_TYPE_F16 = 1,
  OR_TYPE_Q4_K = 12,
  OR_TYPE_Q5_K = 13,
  OR_TYPE_Q6_K = 14,
  OR_TYPE_BF16 = 30,
};

/* Bytes of one row of `in_dim` elements (quants.rs bytes_per_row); 0 if invalid. */
int64_t or_bytes_per_row(int type, int64_t in_dim);

/* Exact IEEE half -> float and round-to-nearest-even float -> half. */
float or_fp16_to_f32(uint16_t h);
uint16_t or_f32_to_fp16(float f);

/* Dequantize n_rows rows of in_dim elements. quants.rs:181-249 (Q4_K/Q6_K),
 * :44-98 (F32/F16/BF16), :119-159 (Q5_K). Returns 0 or -1 on bad shape. */
int or_dequantize_rows(int type, const uint8_t *raw, int64_t n_rows, int64_t in_dim, float *out);

/* y[t][r] = sum_k W[r][k] * x[t][k] for r in [0, out_dim), t in [0, n_tok).
 * Summation order per row follows the reference's multi-row fast paths:
 * Q4_K quants.rs:1878-1904, Q6_K quants.rs:2640-2688, F16/F32 quants.rs:1317-1330.
 * Row-parallel over `threads` host threads (rayon equivalent, real_math.rs:455-491);
 * each row's sum is sequential, so results do not depend on the thread count. */
int or_matmul(int type, const uint8_t *raw, int64_t out_dim, int64_t in_dim, const float *x,
              int64_t n_tok, float *y, int threads);

/* real_math.rs:30-47 */
void or_rms_norm_inplace(float *x, int64_t n, const float *w, int64_t wlen, float eps);
/* real_math.rs:2746-2776; w may be NULL (no-scale variant) */
void or_per_head_rms_norm(float *x, const float *w, int64_t wlen, int n_heads, int head_dim,
                          float eps);
/* real_math.rs:79-85 */
void or_gelu_tanh_mul_inplace(float *g, const float *u, int64_t n);
/* real_math.rs:2576-2639: NeoX half-split rotation of n_heads heads in place. */
void or_rope_apply(float *x, int n_heads, int head_dim, const float *freqs, int64_t n_freqs,
                   uint32_t position, float base_theta, int rotary_dim, int proportional);
/* real_math.rs:2697-2744. kc/vc: [n_pos][n_kv*head_dim] f32 rows (position-major).
 * limit<0 means none; window<=0 means none. */
void or_gqa_attention(const float *q, const float *kc, const float *vc, int64_t n_pos,
                      int64_t limit, int64_t window, int n_heads, int n_kv, int head_dim,
                      float *out);
// Same, with the cached rows as one pointer per position (read in place).
void or_gqa_attention_rows(const float *q, const float *const *krows, const float *const *vrows, int64_t n_pos,
                           int64_t limit, int64_t window, int n_heads, int n_kv, int head_dim, float *out);
// n_tok queries [n_tok][n_heads*head_dim] over the same cached rows, query t seeing limits[t]
// positions (each query's arithmetic is or_gqa_attention_rows'; queries run on `threads`).
void or_gqa_attention_rows_batch(const float *q, const float *const *krows, const float *const *vrows, int64_t n_pos,
                                 const int64_t *limits, int64_t n_tok, int64_t window, int n_heads, int n_kv,
                                 int head_dim, float *out, int threads);

/* real_math.rs:2119-2488 (matmul_raw_top_k). logits over rows [0, vocab), softcap if cap>0,
 * argmax with ties to the lowest index, top-k descending (k may be 0).
 * all_scores (nullable) receives every capped score. */
int or_logits_top_k(int type, const uint8_t *raw, int64_t vocab, int64_t hidden, const float *h,
                    int k, float cap, int64_t *argmax_idx, float *argmax_score, int64_t *top_idx,
                    float *top_score, float *all_scores, int threads);

/* Deterministic synthetic generators (the same spec is implemented on the GPU side;
 * tests compare bytes). key = seed-derived tensor key. */
uint64_t or_mix64(uint64_t key, uint64_t ctr);
uint64_t or_tensor_key(uint64_t seed, const char *name);
float or_synth_normal(uint64_t key, uint64_t ctr);
/* Fill an n_rows x in_dim tensor of `type` per the synthetic spec:
 *  Q4_K block b: d, dmin = fp16(|N(key, 24b+{0,1})| * sigma); bytes 4..143 from
 *                mix64(key, 24b+2+i/8) little-endian.
 *  Q6_K block b: bytes 0..207 from mix64(key, 32b+i/8); d = fp16(|N(key, 32b+26)| * sigma/64).
 *  F32/F16/BF16 element i: mean + N(key, i) * sigma (RNE to 16 bits where needed). */
int or_synth_tensor(int type, uint64_t key, int64_t n_rows, int64_t in_dim, float sigma, float mean,
                    uint8_t *out, int threads);

#ifdef __cplusplus
}
#endif
#endif
