/*
 * stagefwd.h — C ABI of the B200 stage-forward backend (libstagefwd.so).
 *
 * Drop-in boundary for the stage workers of Compute-Network/compute-sharding: every
 * entry point names the reference interface it replaces (paths are relative to the
 * reference repository).  Plain pointers and sizes only; no torch types.
 *
 * Conventions
 *  - Return value: 0 on success, a negative SFC_E_* code on failure.  The message of the
 *    last failure on the calling thread is available from sfc_last_error().  Bad input
 *    (shapes, ids, offsets, sizes) is rejected on the host before any kernel runs.
 *  - "dev" pointers are device pointers on the handle's / current device; `stream` is a
 *    cudaStream_t (NULL = legacy default stream).  Host-pointer entry points run on the stage's
 *    own stream and synchronise it before returning; device-pointer work a caller queued on
 *    another stream for the same stage must be complete (or event-ordered) before them.
 *  - Weight layouts are GGUF (ggml_type ids: F32=0, F16=1, Q4_K=12, Q6_K=14, BF16=30);
 *    rows hold `in_dim` elements, tensor dims are GGUF [in_dim, out_dim].
 *  - A stage handle is not re-entrant: one host thread drives it at a time (the reference's
 *    "caller serializes" contract, crates/llama-stage-backend/src/lib.rs:580-588).
 */
#ifndef STAGEFWD_H
#define STAGEFWD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SFC_ABI_VERSION 1

enum {
  SFC_OK = 0,
  SFC_E_INVALID = -1,  /* bad argument, shape or state */
  SFC_E_CUDA = -2,     /* CUDA runtime error */
  SFC_E_IO = -3,       /* pack / index file error */
  SFC_E_NOMEM = -4,    /* device allocation failed or a fixed capacity is exceeded */
  SFC_E_DEVICE = -5,   /* a kernel reported a device-side error (bounded wait expired, bad id) */
  SFC_ABSENT = 1,      /* a query found no such key / tensor / split (not an error) */
};

/* ------------------------------------------------------------------ misc */
int sfc_abi_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char *sfc_last_error(void);
/* Read and clear the device-side error word of the current device (0 = none; 1 = a bounded
 * device wait ran out; 2 = a kernel rejected an argument, e.g. a token id past the vocabulary). */
int sfc_device_error(unsigned *code);
/* Failure-detection self-test: one thread runs the bounded mbarrier wait that every streaming
 * kernel uses, with `spin_limit` polls, on a barrier that completes (complete != 0) or that
 * nothing ever arrives on (complete == 0).  A wait that runs out gives up, records code 1 in the
 * device error word (read and cleared by sfc_device_error) and the kernel returns; the context
 * stays usable.  Synchronises `stream`.  No counterpart in the reference, whose failure detection
 * is host-side (connect timeouts and retries, crates/llama-stage-backend/src/lib.rs:2417-2538). */
int sfc_selftest_bounded_wait(unsigned spin_limit, int complete, void *stream);
/* Number of compute-kernel launches this library has issued in this process (stream launches
 * and launches recorded into CUDA graphs; replays of a graph are not counted).  Load-time
 * kernels (weight repacking, synthetic weight generation) are not counted. */
int64_t sfc_kernel_launches(void);

/* ------------------------------------------------------------------ kernel-level API
 * Device pointers, caller's stream.  Weights for sfc_matmul* must be in the device layout
 * produced by sfc_prepare_weights: identical to GGUF for F32/F16/BF16; Q4_K and Q6_K rows are
 * grouped in tiles of 16 (zero-padded) with one contiguous record per (tile, 256-element block)
 * holding the 16 rows' scales and quants field by field, so a tile's run of blocks is a single
 * bulk copy for the GEMV and a single tensor copy for the GEMM.                          */

/* Bytes of `rows` rows in the device layout. <0 on unsupported type/shape. */
int64_t sfc_weight_device_bytes(int ggml_type, int64_t rows, int64_t in_dim);

/* GGUF rows (device) -> device layout.  Replaces the pack read of
 * StageTensorStore::read (crates/stage-forward-lab/src/lib.rs:3693-3727). */
int sfc_prepare_weights(int ggml_type, const void *gguf_dev, int64_t rows, int64_t in_dim, void *dst_dev,
                        void *stream);

/* Bit-exact dequantization of GGUF Q4_K / Q6_K rows to f32.
 * Replaces quants.rs:181-249 dequantize_q4_k_block / dequantize_q6_k_block. */
int sfc_dequantize_rows(int ggml_type, const void *gguf_dev, int64_t rows, int64_t in_dim, float *out_dev,
                        void *stream);

/* y[t][r] = sum_k W[r][k] x[t][k] (token-major).  Replaces real_math.rs:398-1124
 * matmul_quantized_many_refs_range(_token_major) and the row dots quants.rs:829-3700. */
int sfc_matmul(int ggml_type, const void *w_dev, int64_t out_dim, int64_t in_dim, const float *x_dev, int64_t n_tok,
               float *y_dev, void *stream);

/* act[t][r] = gelu_tanh(G x)[r] * (U x)[r] in one pass over both matrices.  Replaces
 * real_math.rs:1584-1800 (pair matmul) + real_math.rs:79-85 (GeGLU), as called at
 * crates/stage-forward-lab/src/real_forward.rs:1716-1730. */
int sfc_matmul_pair_geglu(int ggml_type, const void *w_gate_dev, const void *w_up_dev, int64_t out_dim,
                          int64_t in_dim, const float *x_dev, int64_t n_tok, float *act_dev, void *stream);

/* out[t] = x[t] * (1/sqrt(mean(x[t]^2) + eps)) * w.  Replaces real_math.rs:30-47. */
int sfc_rms_norm(const float *x_dev, const float *w_dev, int64_t n_tok, int64_t dim, float eps, float *out_dev,
                 void *stream);

/* Logits over `vocab` rows of W (dims [dim, vocab]) for each of n_tok hidden vectors, softcap
 * cap*tanh(s/cap) (cap <= 0: none), argmax with ties to the lowest index; optionally all
 * capped scores [n_tok][vocab].  Replaces real_math.rs:2119-2488 matmul_raw_top_k. */
int sfc_logits_argmax(int ggml_type, const void *w_dev, int64_t vocab, int64_t dim, const float *h_dev,
                      int64_t n_tok, float cap, float *all_scores_dev, int64_t *argmax_dev, float *score_dev,
                      void *stream);

/* Seeded temperature sampling of n rows of scores [n][vocab] (e.g. the softcapped logits written
 * by sfc_logits_argmax): row r draws from softmax(scores / temperature) with the uniform
 * (mix64(seed, r) >> 40) * 2^-24, summing weights over 1024 contiguous vocabulary segments in index
 * order.  No counterpart in the reference (it samples greedily); used by sfc_sample_tree. */
int sfc_sample_temperature(const float *scores_dev, int64_t n, int64_t vocab, float temperature, uint64_t seed,
                           int64_t *tokens_dev, void *stream);

/* Same computation as sfc_logits_argmax, for callers that cannot allocate device memory
 * (serving processes whose device memory is reserved up front and owned by their own allocator,
 * so a cudaMalloc inside the library would fail or fragment it).  No counterpart in the reference.  It allocates nothing: its per-CTA partials live
 * in a fixed 64 KiB array inside the library (enough for GPUs with up to 512 SMs; larger needs
 * return SFC_E_NOMEM).  The first call on each device looks up that array's device address, so
 * make it before any stream capture; the address is kept for the life of the process, so a
 * caller that resets a device (cudaDeviceReset) must not call this entry point on it afterwards.
 * All calls share the array: calls whose kernels overlap on the GPU (e.g. on two streams at once)
 * race; nothing in it needs to start at zero. */
int sfc_logits_argmax_noalloc(int ggml_type, const void *w_dev, int64_t vocab, int64_t dim, const float *h_dev,
                              int64_t n_tok, float cap, float *all_scores_dev, int64_t *argmax_dev,
                              float *score_dev, void *stream);

/* Seeded synthetic tensor in GGUF layout (deterministic; same bytes on every device). */
int sfc_synth_tensor(int ggml_type, uint64_t seed, const char *name, int64_t rows, int64_t in_dim, float sigma,
                     float mean, void *out_dev, void *stream);

/* ------------------------------------------------------------------ stage-level API
 * Implements the StageForwardBackend trait (crates/stage-forward-lab/src/lib.rs:4663-4674)
 * with RealGemmaBackend semantics (crates/stage-forward-lab/src/real_forward.rs:112-2411).  */

typedef struct sfc_stage sfc_stage;

/* StageLayout, crates/stage-forward-lab/src/lib.rs:212-219 */
typedef struct {
  const char *model_id;
  const char *stage_id;
  uint32_t start_layer;
  uint32_t end_layer;
  int is_head;
  int is_tail;
} sfc_layout;

typedef struct {
  float rope_theta;    /* 0 -> 1e6, the reference's hard-coded base (real_forward.rs:2284) */
  float logit_softcap; /* 0 -> 30 (real_forward.rs:2285); <0 -> none */
  float eps;           /* 0 -> 1e-6 (real_math.rs:5) */
  int kv_f32;          /* 0: fp16 KV cache (default); 1: f32 KV cache, the reference's precision */
  int max_ctx;         /* positions per session; 0 -> 4096 */
  int max_sessions;    /* KV slots; 0 -> 64 (real_forward.rs:23 DECODE_SESSION_LIMIT) */
  int max_batch_tokens;/* rows per forward chunk; 0 -> 512 */
} sfc_options;

/* Synthetic Gemma-style stage: same tensor names, types and shapes as a packed stage. */
typedef struct {
  uint64_t seed;
  int hidden, n_heads, n_kv, head_dim, ffn, n_layers_total;
  int64_t vocab;
  int type_q, type_k, type_v, type_o, type_gate, type_up, type_down, type_embd;
  float w_sigma, embd_sigma, norm_sigma;
} sfc_synth_spec;

typedef struct {
  int hidden, n_heads, n_kv, head_dim, ffn, n_layers;
  int64_t vocab;
  int is_head, is_tail;
  int64_t weight_bytes;
  int64_t kv_bytes;
} sfc_stage_info;

/* RealGemmaBackend::new(index_path) + load_layout (real_forward.rs:162, :2258-2363): loads a
 * `<stage>.index.json` + `.pack` (PackedStageIndex, lib.rs:2908-2927; validation
 * lib.rs:3645-3750) onto `device`. */
int sfc_stage_open(const char *index_json_path, const sfc_layout *layout, const sfc_options *opts, int device,
                   sfc_stage **out);
/* Same, with weights generated on the device from `spec` (layers start..end of the layout). */
int sfc_stage_open_synthetic(const sfc_synth_spec *spec, const sfc_layout *layout, const sfc_options *opts,
                             int device, sfc_stage **out);
int sfc_stage_close(sfc_stage *h);
int sfc_stage_get_info(sfc_stage *h, sfc_stage_info *info);

/* Head ingress: begin_token_ids (real_forward.rs:1123, :988-1121).  ids[n] -> hidden [n][H]
 * (host).  n > 1 starts a new session for request_id; n == 1 continues its KV (or starts one). */
int sfc_begin_token_ids(sfc_stage *h, const char *request_id, const uint32_t *ids, int64_t n, float *out_hidden);
/* continue_forward (real_forward.rs:2376-2405, :2054-2254): hidden [n][H] -> [n][H] (host),
 * same session rule as sfc_begin_token_ids. */
int sfc_continue_forward(sfc_stage *h, const char *request_id, const float *in_hidden, int64_t n, float *out_hidden);
/* sample_tail (real_forward.rs:2407-2410, :904-986): output_norm, logits, softcap, argmax of
 * the LAST row of hidden [n][H] (host). */
int sfc_sample_tail(sfc_stage *h, const float *hidden, int64_t n, uint32_t *token, float *score);

/* Batched device path (pipelines): n_seq sessions, seq_tokens[i] rows each, concatenated.
 * Head: ids_dev [sum] token ids; other stages: in_dev [sum][H].  out_dev [sum][H].
 * append = 1 continues every session; append = 0 restarts them (prefill). */
int sfc_forward_dev(sfc_stage *h, const char *const *request_ids, const int32_t *seq_tokens, int n_seq,
                    const uint32_t *ids_dev, const float *in_dev, float *out_dev, int append, void *stream);
/* Tail: greedy sample of rows of hidden_dev [n][H] -> tokens_dev [n] (int64), scores_dev [n]. */
int sfc_sample_dev(sfc_stage *h, const float *hidden_dev, int64_t n, int64_t *tokens_dev, float *scores_dev,
                   void *stream);

/* Greedy speculative verification at the tail (crates/llama-stage-backend/src/lib.rs:2022-2234):
 * hidden [k+1][H] for [last, d1..dk] already forwarded; accept while argmax_i == d_{i+1}; bonus =
 * argmax at the first mismatch (or at k).  Returns accepted count and bonus token. */
int sfc_verify_greedy(sfc_stage *h, const float *hidden, const uint32_t *drafts, int64_t k, int64_t *accepted,
                      uint32_t *bonus);

/* Draft-tree verification, generalising verify_batch_at_tail's chain rule (lib.rs:2143-2185) to a
 * tree.  Nodes 0..n-1 (n <= 64) in breadth-first order: node 0 is the last accepted token (the
 * root, parent -1), parent[i] < i.  sfc_forward_tree runs the nodes after the session's cached
 * positions (cache rows len .. len+n-1) with rotary position len + depth(i) and attention to
 * the cache plus the node's ancestors only; the session length is left unchanged.  Head stages
 * take token ids, other stages the previous stage's rows; out_hidden gets [n][H]. */
int sfc_forward_tree(sfc_stage *h, const char *request_id, const uint32_t *ids, const float *in_hidden,
                     const int32_t *parent, int64_t n, float *out_hidden);
/* Tail: draws a token at every node (temperature <= 0: argmax of the softcapped logits; else a
 * seeded sample of softmax(logits / temperature), one uniform per node from mix64(seed, node))
 * and walks from the root while a child carries the drawn token.  path gets the node indices
 * (starting with 0), n_path their count, next_token the token drawn where the walk stops. */
int sfc_sample_tree(sfc_stage *h, const float *hidden, const int32_t *parent, const uint32_t *node_tokens, int64_t n,
                    float temperature, uint64_t seed, int32_t *path, int64_t *n_path, uint32_t *next_token);
/* Keeps the KV rows of the accepted path (len + path[i] -> len + i on every layer) and advances
 * the session by n_path.  Call on every stage after sfc_sample_tree. */
int sfc_commit_tree(sfc_stage *h, const char *request_id, const int32_t *path, int64_t n_path);

/* Hand-off payloads as the reference's StageTensor::bytes: f32 little-endian rows [T][hidden], bare
 * or framed "stb1" | u32 hidden_len | u32 aux_len | hidden | aux (crates/stage-forward-lab/src/
 * lib.rs:36-118).  sfc_stage_tensor_sections: stage_tensor_byte_sections — offsets and lengths of
 * the two sections; SFC_ABSENT (with the whole buffer as the hidden section) when the bytes are not
 * a well-formed frame.  sfc_encode_stage_tensor_bytes: encode_stage_tensor_bytes — bare hidden
 * bytes without aux, else the frame; out = NULL queries the size. */
int sfc_stage_tensor_sections(const void *bytes, uint64_t n, uint64_t *hidden_offset, uint64_t *hidden_len,
                              uint64_t *aux_offset, uint64_t *aux_len);
int sfc_encode_stage_tensor_bytes(const void *hidden, uint64_t hidden_len, const void *aux, uint64_t aux_len,
                                  void *out, uint64_t cap, uint64_t *out_len);
/* begin_prompt's StageTensor payload for token ids (begin_token_sequence, real_forward.rs:988-1121,
 * aux :1096-1103): the output rows framed with the prompt aux section when there is one ("rsa1":
 * the prefix hashes of a multi-token prompt and, for a model with per-layer embeddings, the
 * per-layer inputs of every model layer, real_forward.rs:1852-1894); bare rows otherwise.
 * *out_len = the payload size (also set when cap is too small). */
int sfc_begin_token_ids_bytes(sfc_stage *h, const char *request_id, const uint32_t *ids, int64_t n, void *out,
                              uint64_t cap, uint64_t *out_len);
/* continue_forward on a StageTensor payload (real_forward.rs:2054-2254): decodes the hidden rows
 * (decode_hidden_states, :1826-1850: the byte length must be a multiple of hidden_dim * 4), runs
 * sfc_continue_forward and writes the output rows framed with the input's aux section unchanged
 * (:2383-2387); *out_len = the output size (also set when cap is too small).  out may be bytes
 * itself but must not otherwise overlap it.  A stage with per-layer embedding (PLE) layers takes
 * their inputs from the aux section (decode_prompt_aux, :1896-1990) and fails without it. */
int sfc_continue_forward_bytes(sfc_stage *h, const char *request_id, const void *bytes, uint64_t n,
                               uint64_t hidden_dim, void *out, uint64_t cap, uint64_t *out_len);
/* sample_tail on a StageTensor payload: the last hidden row (decode_hidden_state, real_forward.rs:1818-1824). */
int sfc_sample_tail_bytes(sfc_stage *h, const void *bytes, uint64_t n, uint64_t hidden_dim, uint32_t *token,
                          float *score);

/* Session management (real_forward.rs:294-317; rollback lib.rs:2236-2269). */
int sfc_clear_decode_session(sfc_stage *h, const char *request_id);
int sfc_rollback_kv(sfc_stage *h, const char *request_id, int64_t keep);
int64_t sfc_session_len(sfc_stage *h, const char *request_id);
/* Fill a session's cache with `n_pos` positions of seeded N(0,1) keys/values (benchmarks:
 * a decode step's cost does not depend on the cached values). */
int sfc_session_fill_synthetic(sfc_stage *h, const char *request_id, int64_t n_pos, uint64_t seed);

/* Single-GPU greedy generation through a whole model (head+tail in one stage):
 * prompt ids[n_prompt] prefill, then n_steps greedy tokens into out_tokens (host).
 * The decode step runs as one captured CUDA graph.  Mirrors the bench loop of
 * crates/stage-forward-lab/src/bin/real_two_stage_generate_bench.rs:215-290. */
int sfc_generate_greedy(sfc_stage *h, const char *request_id, const uint32_t *prompt, int64_t n_prompt,
                        int64_t n_steps, uint32_t *out_tokens);

/* Per-phase device times of the last forward (RealForwardProfile, real_forward.rs:28-47), us. */
typedef struct {
  int64_t seq_len, layers;
  double embed_us, attn_us, ffn_us, logits_us, total_us;
  int64_t kernels; /* kernels launched by the timed region (graph replays included) */
} sfc_profile;
int sfc_last_profile(sfc_stage *h, sfc_profile *out);

/* ------------------------------------------------------------------ GGUF shards, splits, packs
 * The reference's on-disk path: GgufFile (crates/stage-forward-lab/src/gguf.rs:138-365), the shard
 * manifest bundle (plan_for_splits / build_manifest / write_bundle, gguf.rs:366-751), the runtime
 * bundle loader and the stage pack writer (LoadedRuntimeBundle / StageResidencyAdapter,
 * lib.rs:3283-3613).  Files written here have the reference's names, layout and JSON field order. */

typedef struct sfc_gguf sfc_gguf;

/* TensorRole (gguf.rs:49-57), from classify_tensor_role (gguf.rs:753-786) */
enum {
  SFC_ROLE_LAYER = 0,          /* blk.<n>.* */
  SFC_ROLE_PROMPT_INGRESS = 1, /* token_embd.weight */
  SFC_ROLE_POSITIONAL = 2,     /* rope_freqs.weight */
  SFC_ROLE_SHARED_AUX = 3,     /* per_layer_token_embd / per_layer_model_proj / per_layer_proj_norm */
  SFC_ROLE_TAIL_ONLY = 4,      /* output* */
  SFC_ROLE_UNKNOWN_GLOBAL = 5,
};

typedef struct {
  uint32_t version;
  uint64_t tensor_count, metadata_count, file_size_bytes, tensor_data_offset;
  int64_t layer_count;          /* inferred_layer_count (gguf.rs:235-247); -1 if none */
  int64_t hidden_size;          /* <arch>.embedding_length for gemma4 / gemma / llama; -1 if absent */
  int64_t feed_forward_length;  /* <arch>.feed_forward_length; -1 if absent */
  int64_t attention_head_count; /* <arch>.attention.head_count; -1 if absent */
  const char *architecture;     /* general.architecture if a string, else NULL (valid while open) */
} sfc_gguf_info;

typedef struct {
  const char *name;       /* valid while the handle is open */
  uint32_t n_dims;
  const uint64_t *dims;   /* [n_dims], GGUF order (dims[0] = elements per row) */
  uint32_t ggml_type;
  uint64_t offset;        /* relative to the tensor data section */
  uint64_t file_offset;   /* tensor_file_offset (gguf.rs:345-350) */
  uint64_t byte_len;      /* tensor_byte_len (gguf.rs:331-343): distance to the next tensor by offset */
  int32_t role;           /* SFC_ROLE_* */
  int64_t layer;          /* layer index for SFC_ROLE_LAYER, else -1 */
} sfc_gguf_tensor;

/* StageSplit (gguf.rs:42-47) */
typedef struct {
  uint32_t stage_index, start_layer, end_layer;
} sfc_stage_split;

/* GgufFile::parse_file / parse_bytes (gguf.rs:139-210): versions 1 (32-bit counts) and 2/3; the
 * tensor data starts at general.alignment (u32/u64, default 32).  Malformed files return
 * SFC_E_IO with the reason.  open maps the file read-only and keeps it mapped until close. */
int sfc_gguf_open(const char *path, sfc_gguf **out);
int sfc_gguf_parse(const void *bytes, uint64_t n, sfc_gguf **out);
int sfc_gguf_close(sfc_gguf *g);
int sfc_gguf_get_info(const sfc_gguf *g, sfc_gguf_info *info);
int sfc_gguf_get_tensor(const sfc_gguf *g, uint64_t index, sfc_gguf_tensor *out);
/* First tensor with that name; SFC_ABSENT if none. */
int sfc_gguf_find_tensor(const sfc_gguf *g, const char *name, uint64_t *index);
/* Metadata keys in sorted order (the reference keeps a BTreeMap; a repeated key keeps its last value). */
int sfc_gguf_metadata_key(const sfc_gguf *g, uint64_t index, const char **key, uint32_t *value_type);
/* metadata_string (gguf.rs:249-251 with metadata_value_to_string :800-823): any value as text, floats
 * in Rust's shortest round-trip form without exponent, arrays as "[a, b]".  Writes at most cap-1
 * bytes and a NUL; *len = the full length.  SFC_ABSENT if the key is missing. */
int sfc_gguf_metadata_string(const sfc_gguf *g, const char *key, char *buf, uint64_t cap, uint64_t *len);
/* metadata_u32 (gguf.rs:279-287): u32, or u64 / i32 / i64 values that fit; else SFC_ABSENT. */
int sfc_gguf_metadata_u32(const sfc_gguf *g, const char *key, uint32_t *value);
/* An array value: its element type and length; SFC_ABSENT if the key is missing or not an array. */
int sfc_gguf_metadata_array(const sfc_gguf *g, const char *key, uint32_t *elem_type, uint64_t *count);
/* metadata_f32_array (gguf.rs:262-277): f32 / f64 / i32 / u32 elements as f32, any other type 0.
 * *n = the array's length, the first cap written.  SFC_ABSENT if not an array. */
int sfc_gguf_metadata_f32_array(const sfc_gguf *g, const char *key, float *out, uint64_t cap, uint64_t *n);
/* metadata_string_array (gguf.rs:253-260): element `index` as text (metadata_value_to_string);
 * same buffer rule as sfc_gguf_metadata_string. */
int sfc_gguf_metadata_array_string(const sfc_gguf *g, const char *key, uint64_t index, char *buf, uint64_t cap,
                                   uint64_t *len);
/* block_indices (gguf.rs:219-233): sorted distinct n of blk.<n>.*; *n = count, first cap written. */
int sfc_gguf_block_indices(const sfc_gguf *g, uint32_t *out, uint64_t cap, uint64_t *n);
/* suggest_even_stage_split (gguf.rs:307-329): out[stages]; the first (layers % stages) stages take
 * one extra layer.  SFC_ABSENT when stages is 0, exceeds the layer count, or no count is known. */
int sfc_gguf_even_split(const sfc_gguf *g, uint32_t stages, sfc_stage_split *out);
/* plan_for_splits + write_bundle (gguf.rs:366-400, :636-751): model-shard-manifest.json,
 * stage-N.json and its six tensor lists, runtime-stage-N.json, -required.txt, -optional.txt and
 * -slices.json in out_dir (created). */
int sfc_gguf_write_bundle(const sfc_gguf *g, const sfc_stage_split *splits, uint32_t n_splits, const char *out_dir);
/* StageResidencyAdapter::load + pack_required_tensors / pack_all_tensors (lib.rs:3424-3613): checks
 * the bundle against itself and the GGUF, then writes stage-N-required.pack and
 * stage-N-required.index.json (N = stage_index + 1) into out_dir; include_optional adds the
 * stage's optional tensors (the tied embedding on non-head stages).  The index path is copied to
 * index_path (cap bytes, NUL included) when cap > 0. */
int sfc_pack_stage(const char *bundle_dir, const char *gguf_path, uint32_t stage_index, int include_optional,
                   const char *out_dir, char *index_path, uint64_t cap);
/* StageResidencyAdapter::load + materialize_required_tensors (lib.rs:3424-3510; the
 * bin/materialize_stage_required.rs tool): each required tensor of the stage as its own file in
 * out_dir (created), named by sanitize_tensor_filename (lib.rs:3627-3636: characters other than
 * ASCII letters, digits, '-' and '_' become '_'). */
int sfc_materialize_stage(const char *bundle_dir, const char *gguf_path, uint32_t stage_index, const char *out_dir,
                          uint64_t *n_written);
/* A stage straight from a GGUF file (no pack): the layout's layers start..end plus, as the
 * runtime plan would give it, rope_freqs and the shared auxiliaries, token_embd on the head (and on
 * the tail when the file has no output.weight: tied logits) and output* on the tail.  Tensors are
 * read at the size their dimensions imply, straight from the mapped file.  Otherwise as
 * sfc_stage_open. */
int sfc_stage_open_gguf(const char *gguf_path, const sfc_layout *layout, const sfc_options *opts, int device,
                        sfc_stage **out);

#ifdef __cplusplus
}
#endif
#endif
