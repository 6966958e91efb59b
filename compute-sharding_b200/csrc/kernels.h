// kernels.h — host-side launchers for the sm_100a stage-forward kernels (internal API).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace sfc {

// ---- launch helpers
// SM count of the current device, cached per device ordinal (concurrent first calls on one device
// store the same value).
inline int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
  int n = dev >= 0 ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (n <= 0) {
    if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0) cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Number of kernels launched through launch_pdl by this process (graph captures count the
// kernels they record).
extern long long g_kernel_launches;

// Launch with programmatic stream serialization so the kernel may begin (and start its
// independent weight prefetch) while the previous kernel on the stream drains.
template <class K, class... Args>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  ++g_kernel_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

unsigned *device_error_ptr();

// ---- weights (gemv.cu)
int device_row_bytes(int type, int64_t K);  // bytes per row (K-quants: of the GGUF row; their device
                                            // layout is tiled, see common.cuh)
int64_t device_tensor_bytes(int type, int64_t rows, int64_t K);  // bytes of `rows` rows in the device layout
int gguf_row_bytes(int type, int64_t K);
cudaError_t prepare_weights(int type, const void *gguf, int64_t rows, int64_t K, void *dst, cudaStream_t st);
cudaError_t dequantize(int type, const void *w_gguf, int64_t n_rows, int64_t K, float *out, cudaStream_t st);
// y[t*ldy + r] = sum_k W[r][k] x[t*K + k]; with w1 != null: GeGLU(W0 x, W1 x).
cudaError_t gemv(int type, const void *w0, const void *w1, int64_t rows, int64_t K, const float *x, int64_t n_tok,
                 float *y, int64_t ldy, cudaStream_t st);

// One matrix (or gate/up pair) of a fused K-quant GEMV launch; all segments share K.
struct GemvSeg {
  const uint8_t *w[2];  // device layout; w[1] only for pairs
  float *y;             // output rows [T][ldy]
  int64_t rows;
  int type;             // T_Q4_K or T_Q6_K
  int ldy;
};
// How the launch forms x:  mode 0: x given;  mode 1: x = rms_norm(a) * w_next;
// mode 2: r = resid_in + (w_post ? rms_norm(a) * w_post : a), r *= scale, resid_out = r (CTA 0),
//         x = w_next ? rms_norm(r) * w_next : r.   resid_out must not alias resid_in.
struct GemvPrologue {
  int mode;
  const float *x, *a, *resid_in;
  float *resid_out;
  const float *w_post, *scale, *w_next;
  float eps;
};
// Boundary buffers of the GEMV: a 16-row tile cut between two CTAs is summed by the second CTA
// to arrive.  cnt must start zeroed (each launch leaves it zeroed); launches that run at the same
// time on one device need separate buffers.  max_ctas bounds the grid.
struct GemvSplit {
  unsigned *cnt;
  float *part;
  int max_ctas;
};
size_t gemv_split_bytes(int max_ctas);
GemvSplit gemv_split_view(void *base, int max_ctas);  // base: gemv_split_bytes(max_ctas) bytes
// K-quant GEMV over 1..3 segments (nmat = 2: every segment is a gate/up pair with GeGLU).
// split == nullptr uses the module's own buffers (shared by every caller on the device).
cudaError_t gemv_fused(const GemvSeg *segs, int nseg, int nmat, int64_t K, GemvPrologue pro, int64_t n_tok,
                       cudaStream_t st, const GemvSplit *split = nullptr);

// ---- elementwise / norms / attention (ops.cu)
// out[t] = rms_norm(x[t]) * w   (real_math.rs:30-47)
cudaError_t rms_norm(const float *x, const float *w, int64_t n_tok, int dim, float eps, float *out, cudaStream_t st);
// r = resid + (w_post ? rms_norm(a) * w_post : a); r *= *layer_scale (if given); resid = r;
// if want_xn: xn = w_next ? rms_norm(r) * w_next : r.  (real_forward.rs:1690-1696, 1738-1786)
cudaError_t add_norm(float *resid, const float *a, const float *w_post, const float *layer_scale, int want_xn,
                     const float *w_next, float *xn, int64_t n_tok, int dim, float eps, cudaStream_t st);
// embedding rows of an F16 / F32 / BF16 table scaled by sqrt(dim) (real_forward.rs:848-871);
// ids are uint32 (ids64 = 0) or int64 (ids64 = 1); out-of-range ids set DEV_BAD_ARG.
cudaError_t embed(int type, const void *table, int64_t vocab, int dim, const void *ids, int ids64, int64_t n_tok,
                  float *out, unsigned *err, cudaStream_t st);

struct AttnParams {
  int n_heads, n_kv, head_dim;
  int kv_f32;          // 0: fp16 cache, 1: f32 cache
  int64_t max_ctx;     // positions per head in the cache
  float eps;
  float rope_theta;
  int rotary_dim;
  int proportional;
  const float *rope_freqs;  // may be null: no RoPE (real_forward.rs:1616)
  int n_freqs;
  const float *q_norm, *k_norm;  // may be null
  int window;          // <= 0: none
  int kv_shared;       // 1: the layer attends over another layer's cache, already holding this step's
                       // positions; it has no k/v of its own and appends nothing
};

// One sequence of the current batch.  Its cache for a layer lives in slot `slot` of that
// layer's KV region: K at base + slot*slot_stride, V at K + slot_stride/2, each laid out
// [n_kv][max_ctx][head_dim] (head-major, so a head's keys are one contiguous run).
struct SeqInfo {
  int32_t slot;
  int32_t pos0;   // positions already in the cache before this call
  int32_t n_tok;  // tokens of this sequence in the current batch
  int32_t tok0;   // first row of this sequence in the batch
};
struct KVLayer {
  void *base;
  int64_t slot_stride;  // elements per slot (K and V)
};

// q/k/v post-processing for a batch: per-head norms, RoPE, KV append (real_forward.rs:1583-1662).
// rope_pos (nullable): per-row rotary position when it differs from the cache position (tree
// verification: prefix length + node depth).
cudaError_t qkv_post(float *q, const float *k, const float *v, int q_ld, int kv_ld, KVLayer kv, const SeqInfo *seqs,
                     const int32_t *tok_seq, const int32_t *rope_pos, int64_t n_tok, const AttnParams &p,
                     cudaStream_t st);
// KV of tree nodes kept after verification: for every layer, rows pos0 + path[i] -> pos0 + i of
// `slot` (path strictly increasing, path[i] >= i, so no copy reads a row another one writes).
cudaError_t kv_compact(void *kv_arena, int n_layers, int max_sessions, int64_t slot_stride, int slot, int n_kv,
                       int64_t max_ctx, int head_dim, int elt_bytes, int pos0, const int32_t *path, int m,
                       cudaStream_t st);
// Temperature sampling of n rows of scores [n][vocab]: p ~ exp((s - max) / temperature), one
// counter-based uniform per row (mix64(seed, row) >> 40, times 2^-24); contiguous vocabulary
// segments of ceil(vocab / 1024) per thread, summed in index order, so the walk is reproducible.
// Softcap in place and argmax (lowest index on ties) of raw score rows [n][vocab].
cudaError_t scores_argmax(float *scores, int64_t n, int64_t vocab, float cap, int64_t *idx, float *score,
                          cudaStream_t st);
cudaError_t sample_rows_temperature(const float *scores, int64_t n, int64_t vocab, float temperature, uint64_t seed,
                                    int64_t *out, cudaStream_t st);
// Tensor-core K-quant GEMM (qgemm.cu) for 8+ tokens.  The activation operand is prepared from
// the prologue inputs: mode 0 x; mode 1 RMSNorm(a) * w_next; mode 2 residual add + norms as in
// GemvPrologue; `gate`/`up` non-null: x = gelu_tanh(gate) * up.  Up to 3 output matrices with the
// same K per launch (e.g. q, k, v).
struct GemmPrologue {
  int mode;
  const float *x, *a, *gate, *up, *resid_in;
  float *resid_out;
  const float *w_post, *scale, *w_next;
  float eps;
};
struct QGemmOut {
  int type;
  const void *w;  // device layout (sfc_prepare_weights), 16-byte aligned
  int64_t rows;
  float *y;
  int64_t ldy;
};
bool qgemm_supported(int type, int64_t K);
size_t qgemm_scratch_bytes(int64_t n_tok, int64_t K);
cudaError_t qgemm(const QGemmOut *outs, int nseg, int64_t K, const GemmPrologue &pro, int64_t n_tok, void *scratch,
                  size_t scratch_bytes, cudaStream_t st);
cudaError_t geglu(const float *gate, const float *up, float *out, int64_t n, cudaStream_t st);
// Tokens from which the stage and the kernel-level API use the tensor-core GEMM.
constexpr int64_t QGEMM_MIN_TOKENS = 8;

// Decode step (one new token per sequence, row t = sequence t): q/k/v head norms + RoPE, KV
// append and attention in one launch (decode_attn.cu).  counters: n_seq * n_kv words, zero
// before the first launch; every launch leaves them zero.  sum_keys: the batch's keys summed over
// its sequences (new ones included), or 0; it only sets how many keys a split takes at least.
bool decode_attention_supported(const AttnParams &p);
size_t decode_attention_scratch_bytes(int64_t n_seq, const AttnParams &p, int64_t max_keys);
cudaError_t decode_attention(const float *q, const float *k, const float *v, int q_ld, int kv_ld, float *out,
                             KVLayer kv, const SeqInfo *seqs, int64_t n_seq, int64_t max_keys, int64_t sum_keys,
                             const AttnParams &p, void *scratch, size_t scratch_bytes, unsigned *counters,
                             cudaStream_t st, void *kv_arena = nullptr, int64_t arena_rows = 0);
// causal GQA attention over the cache (real_math.rs:2697-2744); tree masks via parent links.
size_t attention_scratch_bytes(int64_t n_tok, const AttnParams &p, int64_t max_keys);
// tok_limit (nullable): per-token number of visible cache positions (default pos+1);
// tok_mask (nullable): per-token bitmask over the batch's own positions of its sequence
// (bit j = row tok0+j visible), used for tree-masked verification.
cudaError_t attention(const float *q, float *out, KVLayer kv, const SeqInfo *seqs, const int32_t *tok_seq,
                      const int32_t *tok_limit, const uint64_t *tok_mask, int64_t n_tok, int64_t max_keys,
                      const AttnParams &p, void *scratch, size_t scratch_bytes, cudaStream_t st);
// Merge of split-key partials [n_tok][n_heads][n_split][hd + 2] (m, l, unnormalised sums).
cudaError_t attn_combine(const float *part, float *out, int64_t n_tok, int n_heads, int hd, int n_split,
                         cudaStream_t st);

// The same attention on the tensor cores (fattn.cu) for an fp16 cache: the batch's rows in query
// tiles of flash_attention_tile_tokens(p) consecutive tokens of one sequence (FaTileRef: sequence
// index, first token within it), the cache as the arena of `arena_rows` rows of head_dim fp16
// (layer slab, slot, K|V, kv head, position), this layer's slab from row `layer_row0`.
struct FaTileRef {
  int32_t seq, t0;
};
bool flash_attention_supported(const AttnParams &p);
int flash_attention_tile_tokens(const AttnParams &p);
// The cache's tensor map for 32-key tiles ([64-dim chunk][row][64 dims], 128-byte swizzle; built once
// per arena and cached); false when the arena cannot be described.
bool kv_tensor_map(void *kv_arena, int64_t arena_rows, int head_dim, CUtensorMap *out);
// Builds (and caches) the cache's tensor map; false when the arena cannot be described.
bool flash_attention_prepare(void *kv_arena, int64_t arena_rows, int head_dim);
size_t flash_attention_scratch_bytes(int64_t n_tok, const AttnParams &p);
cudaError_t flash_attention(const float *q, float *out, void *kv_arena, int64_t arena_rows, int64_t layer_row0,
                            const SeqInfo *seqs, const FaTileRef *tiles, int n_tiles, const int32_t *tok_limit,
                            const uint64_t *tok_mask, int64_t n_tok, int64_t max_keys, const AttnParams &p,
                            void *scratch, size_t scratch_bytes, cudaStream_t st);

// Per-layer embeddings (ops.cu).  ple_combine: in place on ple [n_tok][layers*P] holding the
// model projection of the scaled token embeddings -> the combined per-layer inputs
// (compute_ple_inputs, real_forward.rs:1157-1299).  ple_gelu: g[t][j] = gelu_tanh(g[t][j]) *
// ple[t][layer*P + j].
// ids: uint32 (ids64 = 0) or int64 token ids, checked against the vocabulary by the embedding.
cudaError_t ple_combine(float *ple, int tok_type, const void *tok, const void *ids, int ids64, int64_t n_tok,
                        int layers, int P, const float *norm, float proj_scale, float embed_scale, float combine_scale,
                        cudaStream_t st);
cudaError_t ple_gelu(float *g, const float *ple, int64_t n_tok, int P, int layers, int layer, cudaStream_t st);

// Bounded-wait self-test (ops.cu): one bounded mbarrier wait of `limit` polls on a barrier that
// completes (complete = 1) or never does (complete = 0, which records DEV_WAIT_TIMEOUT).
cudaError_t wait_selftest(unsigned limit, int complete, cudaStream_t st);

// Decode-graph bookkeeping (see ops.cu).
cudaError_t decode_advance(const int64_t *tok, int64_t *out_tokens, int32_t *step, SeqInfo *seqs, int n_seq,
                           int64_t max_steps, cudaStream_t st);

// ---- logits (logits.cu)
// Tied / output projection + softcap + argmax (lowest index on ties) over rows of `w`.
size_t logits_scratch_bytes(int64_t n_tok);
cudaError_t logits_argmax(int type, const void *w, int64_t vocab, int dim, const float *h, int64_t n_tok, float cap,
                          float *all_scores /*nullable [n_tok][vocab]*/, int64_t *argmax_idx, float *argmax_score,
                          void *scratch, size_t scratch_bytes, cudaStream_t st);

// ---- synthetic generators (synth.cu), same spec as the oracle
cudaError_t synth_tensor(int type, uint64_t key, int64_t rows, int64_t K, float sigma, float mean, void *out,
                         cudaStream_t st);
uint64_t tensor_key(uint64_t seed, const char *name);
uint64_t mix64_host(uint64_t key, uint64_t ctr);

}  // namespace sfc
