// stage.cpp — the stage backend behind the C ABI: packed-stage loading, KV sessions, the
// Gemma-style layer loop, tail sampling and CUDA-graph greedy decode.
//
// Semantics follow RealGemmaBackend (crates/stage-forward-lab/src/real_forward.rs):
//   load_layout            :2258-2363  config inference, rope_freqs, token_embd, tail tensors
//   begin_token_sequence   :988-1121   head ingress, sessions
//   forward_layer_seq      :1483-1793  the per-layer math (run by the kernels in *.cu)
//   continue_forward_inner :2054-2254
//   sample_hidden_state_with_trace :904-986
// Packed stage files follow PackedStageIndex / StageTensorStore (crates/stage-forward-lab/src/
// lib.rs:2908-2927, :3645-3806).
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <set>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "capi_common.h"
#include "gguf.h"
#include "json.h"
#include "payload.h"
#include "common.cuh"
#include "kernels.h"

namespace sfc {

// ------------------------------------------------------------------ stage
struct DevTensor {
  std::string name;
  int type = 0;
  std::vector<int64_t> dims;
  int64_t in_dim = 0, rows = 1;
  void *dev = nullptr;  // device layout
};

struct Layer {
  int index = 0;
  DevTensor *attn_norm = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *q_norm = nullptr, *k_norm = nullptr,
            *o = nullptr, *post_attn = nullptr, *ffn_norm = nullptr, *gate = nullptr, *up = nullptr,
            *down = nullptr, *post_ffw = nullptr, *scale = nullptr;
  // per-layer embedding block (PLE, real_forward.rs:1753-1778): gate [hidden -> P], projection
  // [P -> hidden], optional post norm
  DevTensor *inp_gate = nullptr, *ple_proj = nullptr, *post_norm = nullptr;
  bool has_ple() const { return inp_gate && ple_proj; }
  // attention schedule (LayerAttentionConfig, real_forward.rs:1407-1457); zeros: the stage's defaults
  float theta = 0.f;     // RoPE base
  int rotary_dim = 0;    // rotated dims (0: head_dim)
  int proportional = 0;  // inv_freq over head_dim instead of rotary_dim
  int window = 0;        // sliding window in keys
  int kv_source = -1;    // index in sfc_stage::layers of the layer whose cache this one attends over
  int slab = 0;          // KV cache slab (its own, or its source's)
  bool own_kv() const { return kv_source < 0; }
};

struct Session {
  int slot = -1;
  int64_t len = 0;
  // The draft tree of the last sfc_forward_tree (its rows sit after `len`, not yet committed):
  // parents of its nodes, empty when none is pending.  Any other forward call clears it.
  std::vector<int32_t> tree_parent;
};

// Pinned host staging ring for per-call tables (safe reuse via events).
struct PinnedRing {
  static constexpr int N = 8;
  void *buf[N] = {};
  cudaEvent_t ev[N] = {};
  size_t bytes = 0;
  int next = 0;
  int init(size_t b) {
    bytes = b;
    for (int i = 0; i < N; ++i) {
      SFC_CUDA(cudaMallocHost(&buf[i], b));
      SFC_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
    }
    return SFC_OK;
  }
  void *acquire(int *idx) {
    int i = next;
    next = (next + 1) % N;
    cudaEventSynchronize(ev[i]);
    *idx = i;
    return buf[i];
  }
  void release(int i, cudaStream_t st) { cudaEventRecord(ev[i], st); }
  void destroy() {
    for (int i = 0; i < N; ++i) {
      if (ev[i]) cudaEventDestroy(ev[i]);
      if (buf[i]) cudaFreeHost(buf[i]);
    }
  }
};

}  // namespace sfc

using namespace sfc;

struct sfc_stage {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string model_id, stage_id;
  uint32_t start_layer = 0, end_layer = 0;
  bool is_head = false, is_tail = false;
  // options
  float theta = 1e6f, softcap = 30.f, eps = 1e-6f;
  int kv_f32 = 0, max_ctx = 4096, max_sessions = 64, max_batch = 512;
  // config
  int hidden = 0, n_heads = 0, n_kv = 0, head_dim = 0, ffn = 0, q_dim = 0, k_dim = 0;
  int64_t vocab = 0;
  // weights
  std::vector<std::unique_ptr<DevTensor>> tensors;
  std::vector<Layer> layers;
  DevTensor *token_embd = nullptr, *output_norm = nullptr, *logits_w = nullptr, *rope_freqs = nullptr;
  // PLE (real_forward.rs:1157-1299, :2320-2338): per-token table [layers*P][vocab], model projection
  // [hidden -> layers*P], chunk norm [P]; P = ple_dim, ple_layers = layers of the whole model
  DevTensor *ple_tok = nullptr, *ple_model_proj = nullptr, *ple_proj_norm = nullptr;
  int ple_dim = 0, ple_layers = 0;
  bool ple = false;             // some layer of this stage has a PLE block
  float *ple_all = nullptr;     // [max_batch][ple_layers*P]: the current chunk's per-layer inputs
  float *ple_gate = nullptr;    // [max_batch][P]
  const float *ple_in = nullptr;  // host rows [n][ple_layers*P] for the next non-head forward (aux)
  float *ple_out = nullptr;       // host rows [n][ple_layers*P] the next head forward also returns
  void *weight_arena = nullptr;
  int64_t weight_bytes = 0;
  // KV cache: [n_layers][max_sessions][K|V][n_kv][max_ctx][head_dim]
  void *kv_arena = nullptr;
  int64_t kv_slot_stride = 0;  // elements
  int64_t kv_bytes = 0;
  // activations
  float *resid2 = nullptr;  // residual ping-pong partner for the fused GEMV prologues
  bool fused = false;       // every layer matrix is a K-quant the fused GEMV handles
  bool rope_unit = false;   // RoPE without packed frequencies (every scale 1): the Gemma-4 e4b rule
  int kv_slabs = 0;         // KV cache slabs (layers that read another layer's cache hold none)
  float *resid = nullptr, *xn = nullptr, *proj = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
        *act = nullptr, *hn = nullptr, *score_dev = nullptr;
  uint32_t *ids_dev = nullptr;
  int64_t *tok_dev = nullptr, *gen_tokens_dev = nullptr;
  int32_t *tok_seq_dev = nullptr, *step_dev = nullptr;
  SeqInfo *seq_dev = nullptr;
  void *scratch = nullptr;
  unsigned *attn_counters = nullptr;  // decode attention split counters, [max_batch][n_kv], kept zero
  int64_t attn_sum_keys = 0;  // keys of the eager batch being run (0: graph capture, fixed splits)
  void *gemv_split_mem = nullptr;     // GEMV tile-boundary counters (kept zero) and partial sums
  GemvSplit gemv_split = {};
  // tensor-core GEMM path for 8+ rows (K-quant stages): operand-B staging and the up-projection
  bool gemm_ok = false;
  void *gemm_scratch = nullptr;
  size_t gemm_scratch_bytes = 0;
  float *act2 = nullptr;
  // draft-tree verification: per-row rotary positions, visible-key limits and ancestor masks of the
  // current tree batch (set only while a tree forward runs), and the tail's score rows
  int32_t *tree_rope_dev = nullptr, *tree_limit_dev = nullptr, *tree_path_dev = nullptr;
  uint64_t *tree_mask_dev = nullptr;
  bool tree_active = false;
  float *tree_scores = nullptr;
  // tensor-core attention for multi-row batches (fp16 cache): query tiles of the current batch
  bool fa_ok = false;
  int fa_tt = 0;                       // tokens per query tile
  FaTileRef *fa_tiles_dev = nullptr;   // [max_batch + max_sessions]
  int fa_ntiles = 0;
  int64_t kv_rows = 0;                 // head_dim-element rows of the KV arena
  int64_t tree_scores_rows = 0;
  // tensor-core logits for 8+ rows (fp16 tied embedding): raw then capped scores of up to 64 rows
  float *logit_scores = nullptr;
  size_t attn_scratch = 0, logit_scratch = 0;
  int64_t gen_capacity = 0;
  PinnedRing ring;
  // sessions
  std::unordered_map<std::string, Session> sessions;
  std::vector<char> slot_used;
  // graph for greedy decode
  cudaGraphExec_t decode_graph = nullptr;
  long long graph_kernels = 0;  // kernels per captured decode step
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  sfc_profile profile = {};
};

namespace {

const char *type_name(int t) {
  switch (t) {
    case T_F32: return "F32";
    case T_F16: return "F16";
    case T_Q4_K: return "Q4_K";
    case T_Q5_K: return "Q5_K";
    case T_Q6_K: return "Q6_K";
    case T_BF16: return "BF16";
  }
  return "UNKNOWN";
}

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// Which layer slot a tensor name fills (lib.rs:4287-4335 build_operator_view).
DevTensor **layer_field(Layer &L, const std::string &name) {
  struct {
    const char *key;
    DevTensor *Layer::*f;
  } map[] = {{".attn_q.weight", &Layer::q},
             {".attn_k.weight", &Layer::k},
             {".attn_v.weight", &Layer::v},
             {".attn_output.weight", &Layer::o},
             {".attn_norm.weight", &Layer::attn_norm},
             {".attn_q_norm.weight", &Layer::q_norm},
             {".attn_k_norm.weight", &Layer::k_norm},
             {".ffn_up.weight", &Layer::up},
             {".ffn_down.weight", &Layer::down},
             {".ffn_gate.weight", &Layer::gate},
             {".ffn_norm.weight", &Layer::ffn_norm},
             {".post_attention_norm.weight", &Layer::post_attn},
             {".post_ffw_norm.weight", &Layer::post_ffw},
             {".layer_output_scale.weight", &Layer::scale},
             {".inp_gate.weight", &Layer::inp_gate},
             {".proj.weight", &Layer::ple_proj},
             {".post_norm.weight", &Layer::post_norm}};
  for (auto &m : map)
    if (name.find(m.key) != std::string::npos) return &(L.*(m.f));
  return nullptr;
}

// Parse "blk.<n>." prefix; -1 when the name is not a layer tensor (lib.rs:4265-4285).
int layer_of(const std::string &name) {
  if (name.compare(0, 4, "blk.") != 0) return -1;
  size_t dot = name.find('.', 4);
  if (dot == std::string::npos || dot == 4) return -1;
  int v = 0;
  for (size_t i = 4; i < dot; ++i) {
    if (name[i] < '0' || name[i] > '9') return -1;
    v = v * 10 + (name[i] - '0');
  }
  return v;
}

struct HostTensor {
  std::string name;
  int type;
  std::vector<int64_t> dims;
  const uint8_t *data;  // GGUF bytes (null for synthetic)
  int64_t bytes;
  // synthetic generation parameters
  uint64_t key = 0;
  float sigma = 0, mean = 0;
  bool synthetic = false;
  bool ones = false;
};

int64_t gguf_tensor_bytes(int type, const std::vector<int64_t> &dims) {
  if (dims.empty()) return -1;
  int64_t rows = 1;
  for (size_t i = 1; i < dims.size(); ++i) rows *= dims[i];
  const int rb = gguf_row_bytes(type, dims[0]);
  return rb < 0 ? -1 : rb * rows;
}

int64_t device_tensor_bytes(int type, const std::vector<int64_t> &dims) {
  if (dims.empty()) return -1;
  int64_t rows = 1;
  for (size_t i = 1; i < dims.size(); ++i) rows *= dims[i];
  return ::sfc::device_tensor_bytes(type, rows, dims[0]);
}

int apply_options(sfc_stage *h, const sfc_options *o) {
  if (o) {
    if (o->rope_theta > 0) h->theta = o->rope_theta;
    if (o->logit_softcap > 0) h->softcap = o->logit_softcap;
    if (o->logit_softcap < 0) h->softcap = 0.f;
    if (o->eps > 0) h->eps = o->eps;
    h->kv_f32 = o->kv_f32 ? 1 : 0;
    if (o->max_ctx > 0) h->max_ctx = o->max_ctx;
    if (o->max_sessions > 0) h->max_sessions = o->max_sessions;
    if (o->max_batch_tokens > 0) h->max_batch = o->max_batch_tokens;
  }
  SFC_REQUIRE(h->max_ctx <= (1 << 24), "max_ctx too large");
  SFC_REQUIRE(h->max_batch <= (1 << 16), "max_batch_tokens too large");
  return SFC_OK;
}

// Builds device tensors, infers the config, allocates caches and buffers.
int build_stage(sfc_stage *h, std::vector<HostTensor> &hts) {
  // classification + config inference (real_forward.rs:2258-2283)
  std::map<int, Layer> layer_map;
  std::vector<std::pair<HostTensor *, DevTensor *>> uploads;
  int64_t arena = 0;
  for (auto &ht : hts) {
    SFC_REQUIRE(!ht.dims.empty(), "tensor %s has no dimensions", ht.name.c_str());
    const bool supported = ht.type == T_F32 || ht.type == T_F16 || ht.type == T_BF16 || ht.type == T_Q4_K ||
                           ht.type == T_Q6_K;
    SFC_REQUIRE(supported, "tensor %s has unsupported type %s (%d)", ht.name.c_str(), type_name(ht.type), ht.type);
    const int64_t gb = gguf_tensor_bytes(ht.type, ht.dims);
    SFC_REQUIRE(gb >= 0, "tensor %s: dims incompatible with %s", ht.name.c_str(), type_name(ht.type));
    SFC_REQUIRE(ht.synthetic || ht.ones || gb == ht.bytes, "tensor %s: byte_len %lld != %lld implied by dims",
                ht.name.c_str(), (long long)ht.bytes, (long long)gb);
    auto dt = std::make_unique<DevTensor>();
    dt->name = ht.name;
    dt->type = ht.type;
    dt->dims = ht.dims;
    dt->in_dim = ht.dims[0];
    dt->rows = 1;
    for (size_t i = 1; i < ht.dims.size(); ++i) dt->rows *= ht.dims[i];
    arena += align256(device_tensor_bytes(ht.type, ht.dims) + 16);
    DevTensor *raw = dt.get();
    h->tensors.push_back(std::move(dt));
    uploads.emplace_back(&ht, raw);
    const int li = layer_of(ht.name);
    if (li >= 0) {
      Layer &L = layer_map[li];
      L.index = li;
      DevTensor **f = layer_field(L, ht.name);
      if (f) *f = raw;  // unknown layer tensors are ignored, as the reference does
    } else if (ht.name == "token_embd.weight") {
      h->token_embd = raw;
    } else if (ht.name == "rope_freqs.weight") {
      h->rope_freqs = raw;
    } else if (ht.name == "output_norm.weight") {
      h->output_norm = raw;
    } else if (ht.name == "output.weight") {
      h->logits_w = raw;
    } else if (ht.name == "per_layer_token_embd.weight") {
      h->ple_tok = raw;
    } else if (ht.name == "per_layer_model_proj.weight") {
      h->ple_model_proj = raw;
    } else if (ht.name == "per_layer_proj_norm.weight") {
      h->ple_proj_norm = raw;
    }
  }
  for (auto &kv : layer_map) h->layers.push_back(kv.second);
  SFC_REQUIRE(!h->layers.empty() || h->is_tail, "stage has no layer tensors");
  if (!h->logits_w) h->logits_w = h->token_embd;  // tied embedding (real_forward.rs:803-816)

  // norms must be F32 (real_forward.rs:478-488)
  for (auto &L : h->layers)
    for (DevTensor *t : {L.attn_norm, L.q_norm, L.k_norm, L.post_attn, L.ffn_norm, L.post_ffw, L.scale, L.post_norm})
      SFC_REQUIRE(!t || t->type == T_F32, "Expected F32 tensor for %s, got type %d", t->name.c_str(), t->type);
  if (h->rope_freqs) SFC_REQUIRE(h->rope_freqs->type == T_F32, "rope_freqs.weight must be F32");
  if (h->output_norm) SFC_REQUIRE(h->output_norm->type == T_F32, "output_norm.weight must be F32");

  if (!h->layers.empty()) {
    const Layer &L0 = h->layers.front();
    SFC_REQUIRE(L0.q && L0.k && L0.v && L0.o, "layer %d lacks attention projections", L0.index);
    SFC_REQUIRE(L0.gate && L0.up && L0.down, "layer %d lacks FFN projections", L0.index);
    h->hidden = int(L0.q->dims[0]);
    h->q_dim = int(L0.q->rows);
    h->k_dim = int(L0.k->rows);
    h->ffn = int(L0.up->rows);
    int hd = 0;
    const DevTensor *qn = L0.q_norm ? L0.q_norm : L0.k_norm;
    if (qn && qn->dims[0] > 0 && h->q_dim % qn->dims[0] == 0 && h->k_dim % qn->dims[0] == 0) hd = int(qn->dims[0]);
    if (!hd) {  // GemmaLayerConfig::infer_head_dim (real_math.rs:2889-2907)
      for (int c : {256, 128, 64})
        if (h->q_dim % c == 0 && h->k_dim % c == 0) {
          int nh = h->q_dim / c, nk = h->k_dim / c;
          if (nk >= 1 && nh >= nk && nh % nk == 0) {
            hd = c;
            break;
          }
        }
      if (!hd) {
        int a = h->q_dim, b = h->k_dim;
        while (b) {
          int t = a % b;
          a = b;
          b = t;
        }
        hd = a;
      }
    }
    h->head_dim = hd;
    h->n_heads = h->q_dim / hd;
    h->n_kv = std::max(1, h->k_dim / hd);
    SFC_REQUIRE(h->n_heads % h->n_kv == 0 && h->n_heads / h->n_kv <= 8, "unsupported GQA grouping %d/%d",
                h->n_heads, h->n_kv);
    SFC_REQUIRE(hd <= 256, "head_dim %d > 256 unsupported", hd);
    // Gemma-4 e4b attention schedule (layer_attention_config_for_layout, real_forward.rs:1407-1457):
    // layers 5, 11, 17, .. are global (base 1e6, proportional RoPE over head_dim/4 dims), the others
    // slide over 512 keys (base 1e4); from layer 24 on a layer attends over the cache of layer 23
    // (global) or 22 (sliding) instead of its own.  The packed rope_freqs are not used for this
    // model; RoPE still runs, every frequency scale 1 (real_forward.rs:158-160, :2287-2297).
    if (h->model_id.find("gemma-4-e4b") != std::string::npos && h->hidden == 2560 && (hd == 256 || hd == 512)) {
      h->rope_unit = true;
      for (auto &L : h->layers) {
        const bool global = L.index % 6 == 5;
        L.theta = global ? 1000000.0f : 10000.0f;
        L.rotary_dim = global ? hd / 4 : hd;
        L.proportional = global ? 1 : 0;
        L.window = global ? 0 : 512;
        if (L.index < 24) continue;
        const int src = global ? 23 : 22;
        // validate_stage_split_constraints (real_forward.rs:1459-1481)
        if (src < int(h->start_layer) || src > int(h->end_layer)) {
          set_error("real_forward stage %s (layers %u-%u) is unsupported for %s: layer %d requires shared KV from "
                    "layer %d outside this stage; current contract keeps shared-KV caches stage-local",
                    h->stage_id.c_str(), h->start_layer, h->end_layer, h->model_id.c_str(), L.index, src);
          return SFC_E_INVALID;
        }
        for (size_t j = 0; j < h->layers.size(); ++j)
          if (h->layers[j].index == src) L.kv_source = int(j);
        SFC_REQUIRE(L.kv_source >= 0, "layer %d reads the KV of layer %d, whose tensors this stage lacks", L.index,
                    src);
      }
    }
    for (auto &L : h->layers) {
      if (!L.own_kv()) {  // its k/v projections are not used (real_forward.rs:1561-1592): any or none
        L.k = nullptr;
        L.v = nullptr;
        L.k_norm = nullptr;
      }
      SFC_REQUIRE(L.q && (!L.own_kv() || (L.k && L.v)) && L.o && L.gate && L.up && L.down, "layer %d is incomplete",
                  L.index);
      for (DevTensor *t : {L.q_norm, L.k_norm})
        SFC_REQUIRE(!t || t->in_dim == hd, "%s has %lld elements but head_dim is %d", t->name.c_str(),
                    (long long)t->in_dim, hd);
      for (DevTensor *t : {L.attn_norm, L.post_attn, L.ffn_norm, L.post_ffw})
        SFC_REQUIRE(!t || t->in_dim == h->hidden, "%s has %lld elements but hidden is %d", t->name.c_str(),
                    (long long)t->in_dim, h->hidden);
      SFC_REQUIRE(L.q->dims[0] == h->hidden && L.q->rows == h->q_dim && (!L.k || L.k->rows == h->k_dim) &&
                      (!L.v || L.v->rows == h->k_dim) && L.o->dims[0] == h->q_dim && L.o->rows == h->hidden &&
                      L.gate->dims[0] == h->hidden && L.gate->rows == h->ffn && L.up->rows == h->ffn &&
                      L.down->dims[0] == h->ffn && L.down->rows == h->hidden,
                  "layer %d shapes differ from layer %d", L.index, h->layers.front().index);
      SFC_REQUIRE(L.gate->type == L.up->type, "layer %d: gate/up types differ", L.index);
      for (DevTensor *t : {L.q, L.k, L.v, L.o, L.gate, L.up, L.down})
        SFC_REQUIRE(!t || (t->type != T_Q4_K && t->type != T_Q6_K) || t->in_dim <= 10240,
                    "%s: K-quant rows of %lld elements exceed the GEMV limit 10240", t->name.c_str(),
                    (long long)t->in_dim);
    }
  } else {
    SFC_REQUIRE(h->logits_w && h->output_norm, "tail without layers needs logits tensors");
    h->hidden = int(h->output_norm->dims[0]);
  }
  // PLE configuration (real_forward.rs:2320-2338): width from per_layer_proj_norm, layer count from
  // the model projection (or, on a stage without it, from the per-layer inputs it receives)
  for (auto &L : h->layers) {
    if (!L.inp_gate != !L.ple_proj) {
      set_error("layer %d has only one of inp_gate / proj", L.index);
      return SFC_E_INVALID;
    }
    h->ple = h->ple || L.has_ple();
  }
  if (h->ple) {
    SFC_REQUIRE(h->ple_proj_norm && h->ple_proj_norm->type == T_F32, "PLE layers need per_layer_proj_norm.weight (F32)");
    h->ple_dim = int(h->ple_proj_norm->in_dim);
    SFC_REQUIRE(h->ple_dim > 0, "per_layer_proj_norm.weight is empty");
    if (h->ple_model_proj) {
      SFC_REQUIRE(h->ple_model_proj->in_dim == h->hidden && h->ple_model_proj->rows % h->ple_dim == 0,
                  "per_layer_model_proj.weight dims do not match hidden %d / ple_dim %d", h->hidden, h->ple_dim);
      h->ple_layers = int(h->ple_model_proj->rows / h->ple_dim);
    } else {
      h->ple_layers = int(h->end_layer) + 1;
    }
    for (auto &L : h->layers) {
      if (!L.has_ple()) continue;
      SFC_REQUIRE(L.index < h->ple_layers, "layer %d has no per-layer input (%d PLE layers)", L.index,
                  h->ple_layers);
      SFC_REQUIRE(L.inp_gate->in_dim == h->hidden && L.inp_gate->rows == h->ple_dim && L.ple_proj->in_dim == h->ple_dim &&
                      L.ple_proj->rows == h->hidden && (!L.post_norm || L.post_norm->in_dim == h->hidden),
                  "layer %d: PLE tensor shapes do not match hidden %d / ple_dim %d", L.index, h->hidden, h->ple_dim);
    }
    if (h->is_head) {
      SFC_REQUIRE(h->ple_model_proj && h->ple_tok, "a head stage with PLE layers needs per_layer_model_proj.weight "
                                                   "and per_layer_token_embd.weight");
      SFC_REQUIRE(h->ple_tok->in_dim == int64_t(h->ple_layers) * h->ple_dim &&
                      (h->ple_tok->type == T_F16 || h->ple_tok->type == T_BF16 || h->ple_tok->type == T_F32),
                  "per_layer_token_embd.weight must be F16/BF16/F32 with %d x %d values per token", h->ple_layers,
                  h->ple_dim);
    }
  }
  h->fused = !h->layers.empty() && h->hidden % 256 == 0 && h->q_dim % 256 == 0 && h->ffn % 256 == 0 &&
             h->hidden <= 10240 && h->q_dim <= 10240 && h->ffn <= 10240;
  for (auto &L : h->layers)
    for (DevTensor *t : {L.q, L.k, L.v, L.o, L.gate, L.up, L.down})
      if (t && t->type != T_Q4_K && t->type != T_Q6_K) h->fused = false;
  {  // KV slabs: one per layer with its own cache; readers of another layer's cache share its slab
    int slabs = 0;
    for (auto &L : h->layers) L.slab = L.own_kv() ? slabs++ : -1;
    for (auto &L : h->layers)
      if (!L.own_kv()) L.slab = h->layers[size_t(L.kv_source)].slab;
    h->kv_slabs = slabs;
  }
  if (h->output_norm)
    SFC_REQUIRE(h->output_norm->in_dim == h->hidden, "output_norm.weight has %lld elements but hidden is %d",
                (long long)h->output_norm->in_dim, h->hidden);
  if (h->token_embd) {
    SFC_REQUIRE(h->token_embd->dims.size() == 2 && h->token_embd->dims[0] == h->hidden,
                "token_embd.weight dims do not match hidden %d", h->hidden);
  }
  if (h->is_head) SFC_REQUIRE(h->token_embd, "head stage needs token_embd.weight");
  if (h->is_tail) {
    SFC_REQUIRE(h->logits_w, "Tail stage has no logits tensor");
    SFC_REQUIRE(h->logits_w->type == T_F16 || h->logits_w->type == T_F32 || h->logits_w->type == T_BF16,
                "logits tensor type %s unsupported", type_name(h->logits_w->type));
    // dims [hidden, vocab] (real_forward.rs:818-846)
    if (h->logits_w->dims[0] == h->hidden)
      h->vocab = h->logits_w->rows;
    else
      SFC_REQUIRE(false, "Logits tensor %s dimensions do not match hidden_dim %d", h->logits_w->name.c_str(),
                  h->hidden);
  }
  if (h->token_embd && !h->vocab) h->vocab = h->token_embd->rows;

  // ---- device memory
  SFC_CUDA(cudaSetDevice(h->device));
  SFC_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  SFC_CUDA(cudaEventCreate(&h->ev0));
  SFC_CUDA(cudaEventCreate(&h->ev1));
  if (cudaMalloc(&h->weight_arena, size_t(arena)) != cudaSuccess) {
    set_error("cannot allocate %lld bytes of weights", (long long)arena);
    return SFC_E_NOMEM;
  }
  h->weight_bytes = arena;
  int64_t off = 0;
  void *staging = nullptr;
  int64_t staging_bytes = 0;
  for (auto &u : uploads) {
    HostTensor *ht = u.first;
    DevTensor *dt = u.second;
    dt->dev = static_cast<char *>(h->weight_arena) + off;
    const int64_t db = device_tensor_bytes(ht->type, ht->dims);
    off += align256(db + 16);
    if (ht->ones) {
      std::vector<float> ones(size_t(dt->in_dim * dt->rows), 1.0f);
      SFC_CUDA(cudaMemcpy(dt->dev, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice));
      continue;
    }
    const bool needs_repack = ht->type == T_Q4_K || ht->type == T_Q6_K;  // tiled device layout
    if (ht->synthetic) {
      if (!needs_repack) {
        SFC_CUDA(synth_tensor(ht->type, ht->key, dt->rows, dt->in_dim, ht->sigma, ht->mean, dt->dev, h->stream));
        continue;
      }
    }
    const int64_t gb = gguf_tensor_bytes(ht->type, ht->dims);
    void *src = dt->dev;
    if (needs_repack) {
      if (staging_bytes < gb) {
        if (staging) cudaFree(staging);
        SFC_CUDA(cudaMalloc(&staging, size_t(gb)));
        staging_bytes = gb;
      }
      src = staging;
    }
    if (ht->synthetic)
      SFC_CUDA(synth_tensor(ht->type, ht->key, dt->rows, dt->in_dim, ht->sigma, ht->mean, src, h->stream));
    else
      SFC_CUDA(cudaMemcpyAsync(src, ht->data, size_t(gb), cudaMemcpyHostToDevice, h->stream));
    if (needs_repack) {
      SFC_CUDA(prepare_weights(ht->type, src, dt->rows, dt->in_dim, dt->dev, h->stream));
      SFC_CUDA(cudaStreamSynchronize(h->stream));  // staging reused by the next tensor
    }
  }
  SFC_CUDA(cudaStreamSynchronize(h->stream));
  if (staging) cudaFree(staging);

  // KV cache
  const int64_t elt = h->kv_f32 ? 4 : 2;
  h->kv_slot_stride = 2 * int64_t(h->n_kv) * h->max_ctx * h->head_dim;
  h->kv_bytes = int64_t(h->kv_slabs) * h->max_sessions * h->kv_slot_stride * elt;
  if (h->kv_bytes > 0) {
    if (cudaMalloc(&h->kv_arena, size_t(h->kv_bytes)) != cudaSuccess) {
      set_error("cannot allocate %lld bytes of KV cache (max_ctx %d x %d sessions)", (long long)h->kv_bytes,
                h->max_ctx, h->max_sessions);
      return SFC_E_NOMEM;
    }
    // positions past a sequence's end are read (and multiplied by zero weights) by the tensor-core
    // attention's whole key tiles: keep every cache row finite from the start
    SFC_CUDA(cudaMemset(h->kv_arena, 0, size_t(h->kv_bytes)));
  }
  h->kv_rows = h->head_dim > 0 ? h->kv_bytes / elt / h->head_dim : 0;
  h->slot_used.assign(size_t(h->max_sessions), 0);

  // activations
  const int64_t T = h->max_batch;
  auto alloc = [&](void **p, int64_t bytes) -> int {
    if (cudaMalloc(p, size_t(std::max<int64_t>(bytes, 256))) != cudaSuccess) {
      set_error("cannot allocate activation buffer of %lld bytes", (long long)bytes);
      return SFC_E_NOMEM;
    }
    return SFC_OK;
  };
  int rc;
  const int64_t H = h->hidden;
  if ((rc = alloc((void **)&h->resid, T * H * 4)) || (rc = alloc((void **)&h->resid2, T * H * 4)) ||
      (rc = alloc((void **)&h->xn, T * H * 4)) ||
      (rc = alloc((void **)&h->proj, T * H * 4)) || (rc = alloc((void **)&h->q, T * std::max(h->q_dim, 1) * 4)) ||
      (rc = alloc((void **)&h->k, T * std::max(h->k_dim, 1) * 4)) ||
      (rc = alloc((void **)&h->v, T * std::max(h->k_dim, 1) * 4)) ||
      (rc = alloc((void **)&h->att, T * std::max(h->q_dim, 1) * 4)) ||
      (rc = alloc((void **)&h->act, T * std::max(h->ffn, 1) * 4)) || (rc = alloc((void **)&h->hn, T * H * 4)) ||
      (rc = alloc((void **)&h->score_dev, T * 4)) || (rc = alloc((void **)&h->ids_dev, T * 4)) ||
      (rc = alloc((void **)&h->tok_dev, T * 8)) || (rc = alloc((void **)&h->tok_seq_dev, T * 4)) ||
      (rc = alloc((void **)&h->step_dev, 4)) || (rc = alloc((void **)&h->tree_rope_dev, T * 4)) ||
      (rc = alloc((void **)&h->tree_limit_dev, T * 4)) || (rc = alloc((void **)&h->tree_path_dev, T * 4)) ||
      (rc = alloc((void **)&h->tree_mask_dev, T * 8)) ||
      (rc = alloc((void **)&h->seq_dev, int64_t(h->max_sessions) * sizeof(SeqInfo))))
    return rc;
  if (h->ple && ((rc = alloc((void **)&h->ple_all, T * int64_t(h->ple_layers) * h->ple_dim * 4)) ||
                 (rc = alloc((void **)&h->ple_gate, T * int64_t(h->ple_dim) * 4))))
    return rc;
  AttnParams ap = {};
  ap.n_heads = std::max(h->n_heads, 1);
  ap.n_kv = std::max(h->n_kv, 1);
  ap.head_dim = std::max(h->head_dim, 1);
  size_t amax = 0;
  for (int64_t t = 1; t <= T; ++t) {
    amax = std::max(amax, attention_scratch_bytes(t, ap, h->max_ctx));
    amax = std::max(amax, decode_attention_scratch_bytes(t, ap, h->max_ctx));
  }
  ap.kv_f32 = h->kv_f32;
  ap.max_ctx = h->max_ctx;
  h->fa_ok = T >= 2 && flash_attention_supported(ap) && flash_attention_prepare(h->kv_arena, h->kv_rows, h->head_dim);
  if (h->fa_ok) {
    h->fa_tt = flash_attention_tile_tokens(ap);
    amax = std::max(amax, flash_attention_scratch_bytes(T, ap));
    if ((rc = alloc((void **)&h->fa_tiles_dev, (T + h->max_sessions) * int64_t(sizeof(FaTileRef))))) return rc;
  }
  h->attn_scratch = amax;
  h->logit_scratch = logits_scratch_bytes(T);
  if ((rc = alloc(&h->scratch, int64_t(std::max(h->attn_scratch, h->logit_scratch))))) return rc;
  if ((rc = alloc((void **)&h->attn_counters, T * ap.n_kv * 4))) return rc;
  constexpr int kGemvSplitCtas = 1024;
  if ((rc = alloc(&h->gemv_split_mem, int64_t(gemv_split_bytes(kGemvSplitCtas))))) return rc;
  h->gemv_split = gemv_split_view(h->gemv_split_mem, kGemvSplitCtas);
  SFC_CUDA(cudaMemset(h->gemv_split_mem, 0, gemv_split_bytes(kGemvSplitCtas)));
  if (h->fused && T >= QGEMM_MIN_TOKENS) {
    bool ok = true;
    for (const Layer &L : h->layers) {
      for (const DevTensor *w : {L.q, L.k, L.v, L.o, L.gate, L.up, L.down})
        ok = ok && (w ? qgemm_supported(w->type, w->in_dim) && reinterpret_cast<uintptr_t>(w->dev) % 16 == 0
                      : (w == L.k || w == L.v) && !L.own_kv());
      // one GEMM launch covers q/k/v and the gate/up pair: fp16 and K-quant weights do not mix in one
      for (const DevTensor *w : {L.k, L.v})
        ok = ok && (!w || !L.q || (w->type == T_F16) == (L.q->type == T_F16));
      ok = ok && (!L.gate || !L.up || (L.gate->type == T_F16) == (L.up->type == T_F16));
    }
    if (ok) {
      size_t gb = 0;
      for (int64_t K : {int64_t(H), int64_t(h->q_dim), int64_t(h->ffn)}) gb = std::max(gb, qgemm_scratch_bytes(T, K));
      if ((rc = alloc(&h->gemm_scratch, int64_t(gb))) || (rc = alloc((void **)&h->act2, T * std::max(h->ffn, 1) * 4)))
        return rc;
      h->gemm_scratch_bytes = gb;
      h->gemm_ok = true;
      if (h->is_tail && h->logits_w && h->logits_w->type == T_F16 && qgemm_supported(T_F16, H) &&
          reinterpret_cast<uintptr_t>(h->logits_w->dev) % 16 == 0)
        if ((rc = alloc((void **)&h->logit_scores, int64_t(64) * h->vocab * 4))) return rc;
    }
  }
  SFC_CUDA(cudaMemset(h->attn_counters, 0, size_t(T) * ap.n_kv * 4));
  rc = h->ring.init(size_t(T) * 8 + size_t(h->max_sessions) * sizeof(SeqInfo) +
                    size_t(T + h->max_sessions) * sizeof(FaTileRef) + 256);
  if (rc) return rc;
  return SFC_OK;
}

int new_stage(const sfc_layout *layout, const sfc_options *opts, int device, sfc_stage **out,
              std::unique_ptr<sfc_stage> &h) {
  SFC_REQUIRE(layout && out, "null argument");
  h.reset(new sfc_stage());
  h->device = device;
  h->model_id = layout->model_id ? layout->model_id : "";
  h->stage_id = layout->stage_id ? layout->stage_id : "";
  h->start_layer = layout->start_layer;
  h->end_layer = layout->end_layer;
  h->is_head = layout->is_head != 0;
  h->is_tail = layout->is_tail != 0;
  return apply_options(h.get(), opts);
}

void destroy_stage(sfc_stage *h) {
  if (!h) return;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  if (h->decode_graph) cudaGraphExecDestroy(h->decode_graph);
  for (void *p : {(void *)h->resid, (void *)h->resid2, (void *)h->xn, (void *)h->proj, (void *)h->q, (void *)h->k, (void *)h->v,
                  (void *)h->att, (void *)h->act, (void *)h->hn, (void *)h->score_dev, (void *)h->ids_dev,
                  (void *)h->tok_dev, (void *)h->gen_tokens_dev, (void *)h->tok_seq_dev, (void *)h->step_dev,
                  (void *)h->seq_dev, h->scratch, (void *)h->attn_counters, h->gemv_split_mem, h->gemm_scratch, (void *)h->act2, (void *)h->tree_rope_dev,
                  (void *)h->tree_limit_dev, (void *)h->tree_path_dev, (void *)h->tree_mask_dev, (void *)h->tree_scores, (void *)h->logit_scores, (void *)h->fa_tiles_dev,
                  (void *)h->ple_all, (void *)h->ple_gate, h->kv_arena, h->weight_arena})
    if (p) cudaFree(p);
  h->ring.destroy();
  if (h->ev0) cudaEventDestroy(h->ev0);
  if (h->ev1) cudaEventDestroy(h->ev1);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
}

// ---- sessions
int session_for(sfc_stage *h, const std::string &id, bool restart, Session **out) {
  auto it = h->sessions.find(id);
  if (it == h->sessions.end()) {
    int slot = -1;
    for (int i = 0; i < h->max_sessions; ++i)
      if (!h->slot_used[i]) {
        slot = i;
        break;
      }
    if (slot < 0) {
      set_error("all %d decode sessions are in use", h->max_sessions);
      return SFC_E_NOMEM;
    }
    h->slot_used[slot] = 1;
    Session fresh;
    fresh.slot = slot;
    it = h->sessions.emplace(id, fresh).first;
  }
  if (restart) it->second.len = 0;
  it->second.tree_parent.clear();  // a forward writes the rows a pending draft tree occupied
  *out = &it->second;
  return SFC_OK;
}

KVLayer kv_layer(sfc_stage *h, size_t li) {
  KVLayer kv;
  const int64_t elt = h->kv_f32 ? 4 : 2;
  kv.base = static_cast<char *>(h->kv_arena) + int64_t(h->layers[li].slab) * h->max_sessions * h->kv_slot_stride * elt;
  kv.slot_stride = h->kv_slot_stride;
  return kv;
}

AttnParams attn_params(sfc_stage *h, const Layer &L) {
  AttnParams p = {};
  p.n_heads = h->n_heads;
  p.n_kv = h->n_kv;
  p.head_dim = h->head_dim;
  p.kv_f32 = h->kv_f32;
  p.max_ctx = h->max_ctx;
  p.eps = h->eps;
  p.rope_theta = L.theta > 0.f ? L.theta : h->theta;
  p.rotary_dim = L.rotary_dim > 0 ? L.rotary_dim : h->head_dim;
  p.proportional = L.proportional;
  if (h->rope_unit) {  // RoPE on, no frequency table: the kernels read rope_freqs[i] only for i < n_freqs = 0
    p.rope_freqs = static_cast<const float *>(h->resid);
    p.n_freqs = 0;
  } else {
    p.rope_freqs = h->rope_freqs ? static_cast<const float *>(h->rope_freqs->dev) : nullptr;
    p.n_freqs = h->rope_freqs ? int(h->rope_freqs->in_dim) : 0;
  }
  p.q_norm = L.q_norm ? static_cast<const float *>(L.q_norm->dev) : nullptr;
  p.k_norm = L.k_norm ? static_cast<const float *>(L.k_norm->dev) : nullptr;
  p.window = L.window;
  p.kv_shared = L.own_kv() ? 0 : 1;
  return p;
}

#define F32P(t) ((t) ? static_cast<const float *>((t)->dev) : nullptr)

GemvSeg seg_of(const DevTensor *w, const DevTensor *w2, float *y, int64_t ldy) {
  GemvSeg g = {};
  g.w[0] = static_cast<const uint8_t *>(w->dev);
  g.w[1] = w2 ? static_cast<const uint8_t *>(w2->dev) : nullptr;
  g.y = y;
  g.rows = w->rows;
  g.type = w->type;
  g.ldy = int(ldy);
  return g;
}

// Head ingress on the device: embedding rows of `ids` (uint32, or int64 with ids64) into h->resid and,
// for PLE models, every layer's per-layer inputs into h->ple_all (compute_ple_inputs,
// real_forward.rs:1157-1299: the model projection of the scaled embedding, then ple_combine).
cudaError_t head_ingress(sfc_stage *h, const void *ids, int ids64, int64_t T, cudaStream_t st) {
  cudaError_t e = embed(h->token_embd->type, h->token_embd->dev, h->vocab, h->hidden, ids, ids64, T, h->resid,
                        device_error_ptr(), st);
  if (e || !h->ple) return e;
  const int64_t LP = int64_t(h->ple_layers) * h->ple_dim;
  e = gemv(h->ple_model_proj->type, h->ple_model_proj->dev, nullptr, LP, h->hidden, h->resid, T, h->ple_all, LP, st);
  if (e) return e;
  return ple_combine(h->ple_all, h->ple_tok->type, h->ple_tok->dev, ids, ids64, T, h->ple_layers, h->ple_dim,
                     F32P(h->ple_proj_norm), powf(float(h->hidden), -0.5f), sqrtf(float(h->ple_dim)),
                     powf(2.0f, -0.5f), st);
}

// The per-layer embedding block of layer L (real_forward.rs:1753-1778) on the T rows of `states`:
// states += rms_norm(proj(gelu_tanh(inp_gate(states)) * ple_in[layer])) * post_norm, then
// states *= layer_output_scale.  states holds the full residual stream (nothing pending).
cudaError_t ple_block(sfc_stage *h, const Layer &L, float *states, int64_t T, cudaStream_t st) {
  const int P = h->ple_dim;
  cudaError_t e = gemv(L.inp_gate->type, L.inp_gate->dev, nullptr, P, h->hidden, states, T, h->ple_gate, P, st);
  if (!e) e = ple_gelu(h->ple_gate, h->ple_all, T, P, h->ple_layers, L.index, st);
  if (!e) e = gemv(L.ple_proj->type, L.ple_proj->dev, nullptr, h->hidden, P, h->ple_gate, T, h->proj, h->hidden, st);
  if (!e) e = add_norm(states, h->proj, F32P(L.post_norm), F32P(L.scale), 0, nullptr, nullptr, T, h->hidden, h->eps, st);
  return e;
}

// q/k/v post-processing, KV append and attention of one layer.  Decode batches (one new token
// per sequence) use the single fused decode kernel; other batches the two-kernel path.
cudaError_t layer_attention(sfc_stage *h, const AttnParams &ap, const KVLayer &kv, int64_t T, int64_t max_keys,
                            bool decode, cudaStream_t st) {
  if (decode && !h->tree_active && decode_attention_supported(ap))
    return decode_attention(h->q, h->k, h->v, h->q_dim, h->k_dim, h->att, kv, h->seq_dev, T, max_keys,
                            h->attn_sum_keys, ap, h->scratch, h->attn_scratch, h->attn_counters, st, h->kv_arena,
                            h->kv_rows);
  const bool tr = h->tree_active;
  cudaError_t e = qkv_post(h->q, h->k, h->v, h->q_dim, h->k_dim, kv, h->seq_dev, h->tok_seq_dev,
                           tr ? h->tree_rope_dev : nullptr, T, ap, st);
  if (e) return e;
  if (h->fa_ok && h->fa_ntiles > 0 && !decode && flash_attention_supported(ap)) {
    const int64_t elt = h->kv_f32 ? 4 : 2;
    const int64_t row0 = (static_cast<char *>(kv.base) - static_cast<char *>(h->kv_arena)) / elt / h->head_dim;
    return flash_attention(h->q, h->att, h->kv_arena, h->kv_rows, row0, h->seq_dev, h->fa_tiles_dev, h->fa_ntiles,
                           tr ? h->tree_limit_dev : nullptr, tr ? h->tree_mask_dev : nullptr, T, max_keys, ap,
                           h->scratch, h->attn_scratch, st);
  }
  return attention(h->q, h->att, kv, h->seq_dev, h->tok_seq_dev, tr ? h->tree_limit_dev : nullptr,
                   tr ? h->tree_mask_dev : nullptr, T, max_keys, ap, h->scratch, h->attn_scratch, st);
}

// Fused layer loop for K-quant stages: the residual add + RMSNorm that precede the q/k/v and
// gate/up projections run in those GEMVs' prologues (real_forward.rs:1690-1696 and :1738-1749),
// so a layer is 5-6 launches.  Residual rows ping-pong between h->resid and h->resid2.
// Layer loop on the tensor-core GEMM (8+ rows): the same fused prologues run in the operand-B
// preparation of each GEMM; q/k/v share one launch, gate and up another, and the GeGLU of the
// pair is applied while preparing the down projection's input.
cudaError_t run_layers_gemm(sfc_stage *h, int64_t T, int64_t max_keys, bool decode, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const int H = h->hidden;
  float *cur = h->resid, *other = h->resid2;
  void *gs = h->gemm_scratch;
  const size_t gsb = h->gemm_scratch_bytes;
  bool pending = false;  // the previous layer's post-FFN residual add still runs in this layer's prologue
  for (size_t li = 0; li < h->layers.size(); ++li) {
    const Layer &L = h->layers[li];
    GemmPrologue pro = {};
    pro.eps = h->eps;
    pro.w_next = F32P(L.attn_norm);
    if (!pending) {
      pro.mode = L.attn_norm ? 1 : 0;
      pro.x = cur;
      pro.a = cur;
    } else {
      const Layer &P = h->layers[li - 1];
      pro.mode = 2;
      pro.a = h->proj;
      pro.resid_in = cur;
      pro.resid_out = other;
      pro.w_post = F32P(P.post_ffw);
      pro.scale = F32P(P.scale);
      std::swap(cur, other);
    }
    QGemmOut qkv[3] = {{L.q->type, L.q->dev, L.q->rows, h->q, h->q_dim}, {}, {}};
    if (L.own_kv()) {  // a layer reading another layer's cache projects q only
      qkv[1] = {L.k->type, L.k->dev, L.k->rows, h->k, h->k_dim};
      qkv[2] = {L.v->type, L.v->dev, L.v->rows, h->v, h->k_dim};
    }
    if ((e = qgemm(qkv, L.own_kv() ? 3 : 1, H, pro, T, gs, gsb, st))) return e;
    const AttnParams ap = attn_params(h, L);
    const KVLayer kv = kv_layer(h, li);
    if ((e = layer_attention(h, ap, kv, T, max_keys, decode, st))) return e;
    const QGemmOut o = {L.o->type, L.o->dev, L.o->rows, h->proj, H};
    GemmPrologue po = {};
    po.mode = 0;
    po.x = h->att;
    if ((e = qgemm(&o, 1, h->q_dim, po, T, gs, gsb, st))) return e;
    GemmPrologue pf = {};
    pf.mode = 2;
    pf.eps = h->eps;
    pf.a = h->proj;
    pf.resid_in = cur;
    pf.resid_out = other;
    pf.w_post = F32P(L.post_attn);
    pf.w_next = F32P(L.ffn_norm);
    std::swap(cur, other);
    const QGemmOut gu[2] = {{L.gate->type, L.gate->dev, L.gate->rows, h->act, h->ffn},
                            {L.up->type, L.up->dev, L.up->rows, h->act2, h->ffn}};
    if ((e = qgemm(gu, 2, H, pf, T, gs, gsb, st))) return e;
    const QGemmOut d = {L.down->type, L.down->dev, L.down->rows, h->proj, H};
    GemmPrologue pd = {};
    pd.mode = 0;
    pd.gate = h->act;
    pd.up = h->act2;
    if ((e = qgemm(&d, 1, h->ffn, pd, T, gs, gsb, st))) return e;
    pending = true;
    if (L.has_ple()) {  // the residual stream is needed whole: add the FFN output, then the PLE block
      if ((e = add_norm(cur, h->proj, F32P(L.post_ffw), nullptr, 0, nullptr, nullptr, T, H, h->eps, st))) return e;
      if ((e = ple_block(h, L, cur, T, st))) return e;
      pending = false;
    }
  }
  const Layer &Z = h->layers.back();
  if (pending && (e = add_norm(cur, h->proj, F32P(Z.post_ffw), F32P(Z.scale), 0, nullptr, nullptr, T, H, h->eps, st)))
    return e;
  if (cur != h->resid) e = cudaMemcpyAsync(h->resid, cur, size_t(T) * H * 4, cudaMemcpyDeviceToDevice, st);
  return e;
}

cudaError_t run_layers_fused(sfc_stage *h, int64_t T, int64_t max_keys, bool decode, cudaStream_t st) {
  if (h->gemm_ok && T >= QGEMM_MIN_TOKENS) return run_layers_gemm(h, T, max_keys, decode, st);
  cudaError_t e = cudaSuccess;
  const int H = h->hidden;
  float *cur = h->resid, *other = h->resid2;
  bool pending = false;  // the previous layer's post-FFN residual add still runs in this layer's prologue
  for (size_t li = 0; li < h->layers.size(); ++li) {
    const Layer &L = h->layers[li];
    GemvPrologue pro = {};
    pro.eps = h->eps;
    pro.w_next = F32P(L.attn_norm);
    if (!pending) {
      pro.mode = L.attn_norm ? 1 : 0;
      pro.x = cur;
      pro.a = cur;
    } else {
      const Layer &P = h->layers[li - 1];
      pro.mode = 2;
      pro.a = h->proj;
      pro.resid_in = cur;
      pro.resid_out = other;
      pro.w_post = F32P(P.post_ffw);
      pro.scale = F32P(P.scale);
      std::swap(cur, other);
    }
    GemvSeg qkv[3] = {seg_of(L.q, nullptr, h->q, h->q_dim), {}, {}};
    if (L.own_kv()) {  // a layer reading another layer's cache projects q only
      qkv[1] = seg_of(L.k, nullptr, h->k, h->k_dim);
      qkv[2] = seg_of(L.v, nullptr, h->v, h->k_dim);
    }
    const int nqkv = L.own_kv() ? 3 : 1;
    const AttnParams ap = attn_params(h, L);
    const KVLayer kv = kv_layer(h, li);
    if ((e = gemv_fused(qkv, nqkv, 1, H, pro, T, st, &h->gemv_split))) return e;
    if ((e = layer_attention(h, ap, kv, T, max_keys, decode, st))) return e;
    const GemvSeg o = seg_of(L.o, nullptr, h->proj, H);
    GemvPrologue po = {};
    po.mode = 0;
    po.x = h->att;
    if ((e = gemv_fused(&o, 1, 1, h->q_dim, po, T, st, &h->gemv_split))) return e;
    GemvPrologue pf = {};
    pf.mode = 2;
    pf.eps = h->eps;
    pf.a = h->proj;
    pf.resid_in = cur;
    pf.resid_out = other;
    pf.w_post = F32P(L.post_attn);
    pf.w_next = F32P(L.ffn_norm);
    std::swap(cur, other);
    const GemvSeg gu = seg_of(L.gate, L.up, h->act, h->ffn);
    if ((e = gemv_fused(&gu, 1, 2, H, pf, T, st, &h->gemv_split))) return e;
    const GemvSeg d = seg_of(L.down, nullptr, h->proj, H);
    GemvPrologue pd = {};
    pd.mode = 0;
    pd.x = h->act;
    if ((e = gemv_fused(&d, 1, 1, h->ffn, pd, T, st, &h->gemv_split))) return e;
    pending = true;
    if (L.has_ple()) {  // the residual stream is needed whole: add the FFN output, then the PLE block
      if ((e = add_norm(cur, h->proj, F32P(L.post_ffw), nullptr, 0, nullptr, nullptr, T, H, h->eps, st))) return e;
      if ((e = ple_block(h, L, cur, T, st))) return e;
      pending = false;
    }
  }
  const Layer &Z = h->layers.back();
  if (pending && (e = add_norm(cur, h->proj, F32P(Z.post_ffw), F32P(Z.scale), 0, nullptr, nullptr, T, H, h->eps, st)))
    return e;
  if (cur != h->resid) e = cudaMemcpyAsync(h->resid, cur, size_t(T) * H * 4, cudaMemcpyDeviceToDevice, st);
  return e;
}

// All layers over the T rows in h->resid (device tables already uploaded).
cudaError_t run_layers(sfc_stage *h, int64_t T, int64_t max_keys, bool decode, cudaStream_t st) {
  if (h->fused) return run_layers_fused(h, T, max_keys, decode, st);
  cudaError_t e = cudaSuccess;
  const int H = h->hidden;
  for (size_t li = 0; li < h->layers.size(); ++li) {
    const Layer &L = h->layers[li];
    if (li == 0) {
      if (L.attn_norm)
        e = rms_norm(h->resid, F32P(L.attn_norm), T, H, h->eps, h->xn, st);
      else
        e = cudaMemcpyAsync(h->xn, h->resid, size_t(T) * H * 4, cudaMemcpyDeviceToDevice, st);
      if (e) return e;
    }
    if ((e = gemv(L.q->type, L.q->dev, nullptr, h->q_dim, H, h->xn, T, h->q, h->q_dim, st))) return e;
    if (L.own_kv()) {
      if ((e = gemv(L.k->type, L.k->dev, nullptr, h->k_dim, H, h->xn, T, h->k, h->k_dim, st))) return e;
      if ((e = gemv(L.v->type, L.v->dev, nullptr, h->k_dim, H, h->xn, T, h->v, h->k_dim, st))) return e;
    }
    const AttnParams ap = attn_params(h, L);
    const KVLayer kv = kv_layer(h, li);
    if ((e = layer_attention(h, ap, kv, T, max_keys, decode, st))) return e;
    if ((e = gemv(L.o->type, L.o->dev, nullptr, H, h->q_dim, h->att, T, h->proj, H, st))) return e;
    if ((e = add_norm(h->resid, h->proj, F32P(L.post_attn), nullptr, 1, F32P(L.ffn_norm), h->xn, T, H, h->eps, st)))
      return e;
    if ((e = gemv(L.gate->type, L.gate->dev, L.up->dev, h->ffn, H, h->xn, T, h->act, h->ffn, st))) return e;
    if ((e = gemv(L.down->type, L.down->dev, nullptr, H, h->ffn, h->act, T, h->proj, H, st))) return e;
    const bool more = li + 1 < h->layers.size();
    if (L.has_ple()) {
      if ((e = add_norm(h->resid, h->proj, F32P(L.post_ffw), nullptr, 0, nullptr, nullptr, T, H, h->eps, st))) return e;
      if ((e = ple_block(h, L, h->resid, T, st))) return e;
      if (more) {
        const DevTensor *nn = h->layers[li + 1].attn_norm;
        e = nn ? rms_norm(h->resid, F32P(nn), T, H, h->eps, h->xn, st)
               : cudaMemcpyAsync(h->xn, h->resid, size_t(T) * H * 4, cudaMemcpyDeviceToDevice, st);
        if (e) return e;
      }
      continue;
    }
    if ((e = add_norm(h->resid, h->proj, F32P(L.post_ffw), F32P(L.scale), more ? 1 : 0,
                      more ? F32P(h->layers[li + 1].attn_norm) : nullptr, h->xn, T, H, h->eps, st)))
      return e;
  }
  return e;
}

struct SeqReq {
  Session *s;
  int32_t n;
};

// One forward chunk (sum of rows <= max_batch).  ids (uint32, host or device) for the head,
// `in_dev` rows for other stages.  Output stays in h->resid.
int forward_chunk(sfc_stage *h, const std::vector<SeqReq> &seqs, const uint32_t *ids, bool ids_on_device,
                  const float *in_dev, cudaStream_t st, const float *ple_host = nullptr) {
  int64_t T = 0, max_keys = 1, sum_keys = 0;
  for (auto &s : seqs) {
    SFC_REQUIRE(s.n > 0, "empty sequence in batch");
    if (s.s->len + s.n > h->max_ctx) {
      set_error("session needs %lld positions but max_ctx is %d", (long long)(s.s->len + s.n), h->max_ctx);
      return SFC_E_NOMEM;
    }
    T += s.n;
    max_keys = std::max<int64_t>(max_keys, s.s->len + s.n);
    sum_keys += s.s->len + s.n;
  }
  SFC_REQUIRE(T <= h->max_batch, "batch of %lld rows exceeds max_batch_tokens %d", (long long)T, h->max_batch);
  int ri;
  char *pin = static_cast<char *>(h->ring.acquire(&ri));
  SeqInfo *si = reinterpret_cast<SeqInfo *>(pin);
  int32_t *ts = reinterpret_cast<int32_t *>(pin + h->max_sessions * sizeof(SeqInfo));
  int32_t row = 0;
  for (size_t i = 0; i < seqs.size(); ++i) {
    si[i] = SeqInfo{seqs[i].s->slot, int32_t(seqs[i].s->len), seqs[i].n, row};
    for (int j = 0; j < seqs[i].n; ++j) ts[row + j] = int32_t(i);
    row += seqs[i].n;
  }
  SFC_CUDA(cudaMemcpyAsync(h->seq_dev, si, seqs.size() * sizeof(SeqInfo), cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaMemcpyAsync(h->tok_seq_dev, ts, size_t(T) * 4, cudaMemcpyHostToDevice, st));
  h->fa_ntiles = 0;
  if (h->fa_ok && T > 1) {  // query tiles for the tensor-core attention (after ids in the staging buffer)
    FaTileRef *ft = reinterpret_cast<FaTileRef *>(ts + 2 * T);
    for (size_t i = 0; i < seqs.size(); ++i)
      for (int32_t t0 = 0; t0 < seqs[i].n; t0 += h->fa_tt) ft[h->fa_ntiles++] = FaTileRef{int32_t(i), t0};
    SFC_CUDA(cudaMemcpyAsync(h->fa_tiles_dev, ft, size_t(h->fa_ntiles) * sizeof(FaTileRef), cudaMemcpyHostToDevice,
                             st));
  }
  if (h->is_head) {
    const uint32_t *idd = ids;
    if (!ids_on_device) {
      uint32_t *idh = reinterpret_cast<uint32_t *>(ts + T);
      SFC_REQUIRE(int64_t(h->max_sessions * sizeof(SeqInfo) + size_t(T) * 8) <= int64_t(h->ring.bytes),
                  "staging too small");
      for (int64_t i = 0; i < T; ++i) {
        if (ids[i] >= h->vocab) {
          h->ring.release(ri, st);
          set_error("Token ID %u exceeds vocab size %lld", ids[i], (long long)h->vocab);
          return SFC_E_INVALID;
        }
        idh[i] = ids[i];
      }
      SFC_CUDA(cudaMemcpyAsync(h->ids_dev, idh, size_t(T) * 4, cudaMemcpyHostToDevice, st));
      idd = h->ids_dev;
    }
    SFC_CUDA(head_ingress(h, idd, 0, T, st));
  } else {
    SFC_CUDA(cudaMemcpyAsync(h->resid, in_dev, size_t(T) * h->hidden * 4, cudaMemcpyDeviceToDevice, st));
    if (h->ple) {
      if (!ple_host) {
        h->ring.release(ri, st);
        set_error("stage %s has per-layer embedding (PLE) layers: its rows need the per-layer inputs of the "
                  "prompt aux section (continue_forward on StageTensor bytes)", h->stage_id.c_str());
        return SFC_E_INVALID;
      }
      SFC_CUDA(cudaMemcpyAsync(h->ple_all, ple_host, size_t(T) * h->ple_layers * h->ple_dim * 4,
                               cudaMemcpyHostToDevice, st));
    }
  }
  h->ring.release(ri, st);
  h->attn_sum_keys = sum_keys;
  const cudaError_t lerr = run_layers(h, T, max_keys, T == int64_t(seqs.size()), st);
  h->attn_sum_keys = 0;
  SFC_CUDA(lerr);
  for (auto &s : seqs) s.s->len += s.n;
  return SFC_OK;
}

// Single-sequence forward of n rows, chunked by max_batch; rows land in out (device or host).
int forward_single(sfc_stage *h, const char *req, const uint32_t *ids_host, const float *in_host, int64_t n,
                   float *out_host, bool restart) {
  SFC_REQUIRE(req, "null request id");
  SFC_REQUIRE(n > 0, "Empty prompt");
  SFC_CUDA(cudaSetDevice(h->device));
  Session *s = nullptr;
  int rc = session_for(h, req, restart, &s);
  if (rc) return rc;
  SFC_REQUIRE(s->len + n <= h->max_ctx, "session needs %lld positions but max_ctx is %d", (long long)(s->len + n),
              h->max_ctx);
  cudaStream_t st = h->stream;
  SFC_CUDA(cudaEventRecord(h->ev0, st));
  for (int64_t t0 = 0; t0 < n; t0 += h->max_batch) {
    const int32_t c = int32_t(std::min<int64_t>(h->max_batch, n - t0));
    if (!h->is_head) {
      SFC_CUDA(cudaMemcpyAsync(h->hn, in_host + t0 * h->hidden, size_t(c) * h->hidden * 4, cudaMemcpyHostToDevice,
                               st));
    }
    rc = forward_chunk(h, {SeqReq{s, c}}, ids_host ? ids_host + t0 : nullptr, false, h->hn, st,
                       h->ple_in ? h->ple_in + t0 * int64_t(h->ple_layers) * h->ple_dim : nullptr);
    if (rc) return rc;
    if (out_host)
      SFC_CUDA(cudaMemcpyAsync(out_host + t0 * h->hidden, h->resid, size_t(c) * h->hidden * 4,
                               cudaMemcpyDeviceToHost, st));
    if (h->ple_out && h->ple && h->is_head) {  // the chunk's per-layer inputs, for the aux section
      const int64_t LP = int64_t(h->ple_layers) * h->ple_dim;
      SFC_CUDA(cudaMemcpyAsync(h->ple_out + t0 * LP, h->ple_all, size_t(c) * LP * 4, cudaMemcpyDeviceToHost, st));
    }
  }
  SFC_CUDA(cudaEventRecord(h->ev1, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  float ms = 0;
  cudaEventElapsedTime(&ms, h->ev0, h->ev1);
  h->profile.seq_len = n;
  h->profile.layers = int64_t(h->layers.size());
  h->profile.total_us = ms * 1e3;
  unsigned derr = 0;
  unsigned *dp = device_error_ptr();
  if (dp) {
    cudaMemcpy(&derr, dp, 4, cudaMemcpyDeviceToHost);
    if (derr) {
      unsigned z = 0;
      cudaMemcpy(dp, &z, 4, cudaMemcpyHostToDevice);
      set_error("device reported error code %u", derr);
      return SFC_E_DEVICE;
    }
  }
  return SFC_OK;
}

// Tail: output_norm + logits argmax on `n` device rows.
// Logits of rows [t0, t0+c) (c <= 64) on the tensor cores: output_norm runs in the GEMM's operand
// preparation, the fp16 tied embedding is operand A, scores land in h->logit_scores and are then
// capped in place with their argmax.
int tail_logits_gemm(sfc_stage *h, const float *rows_dev, int64_t c, int64_t *tok_dev, float *score_dev,
                     cudaStream_t st) {
  GemmPrologue pro = {};
  pro.mode = h->output_norm ? 1 : 0;
  pro.x = rows_dev;
  pro.a = rows_dev;
  pro.w_next = F32P(h->output_norm);
  pro.eps = h->eps;
  const QGemmOut o = {T_F16, h->logits_w->dev, h->vocab, h->logit_scores, h->vocab};
  SFC_CUDA(qgemm(&o, 1, h->hidden, pro, c, h->gemm_scratch, h->gemm_scratch_bytes, st));
  SFC_CUDA(scores_argmax(h->logit_scores, c, h->vocab, h->softcap, tok_dev, score_dev, st));
  return SFC_OK;
}

bool tail_gemm_eligible(sfc_stage *h, int64_t n) { return h->logit_scores && n >= QGEMM_MIN_TOKENS; }

int sample_rows(sfc_stage *h, const float *rows_dev, int64_t n, int64_t *tok_dev, float *score_dev, cudaStream_t st) {
  SFC_REQUIRE(h->is_tail, "Only the tail stage may sample");
  SFC_REQUIRE(n > 0 && n <= h->max_batch, "sample rows %lld out of range", (long long)n);
  if (tail_gemm_eligible(h, n)) {
    for (int64_t t0 = 0; t0 < n; t0 += 64) {
      const int64_t c = std::min<int64_t>(64, n - t0);
      int rc = tail_logits_gemm(h, rows_dev + t0 * h->hidden, c, tok_dev + t0, score_dev + t0, st);
      if (rc) return rc;
    }
    return SFC_OK;
  }
  if (h->output_norm)
    SFC_CUDA(rms_norm(rows_dev, F32P(h->output_norm), n, h->hidden, h->eps, h->hn, st));
  else
    SFC_CUDA(cudaMemcpyAsync(h->hn, rows_dev, size_t(n) * h->hidden * 4, cudaMemcpyDeviceToDevice, st));
  SFC_CUDA(logits_argmax(h->logits_w->type, h->logits_w->dev, h->vocab, h->hidden, h->hn, n, h->softcap, nullptr,
                         tok_dev, score_dev, h->scratch, std::max(h->attn_scratch, h->logit_scratch), st));
  return SFC_OK;
}

}  // namespace

extern "C" {

int sfc_stage_open(const char *index_json_path, const sfc_layout *layout, const sfc_options *opts, int device,
                   sfc_stage **out) {
  clear_error();
  SFC_REQUIRE(index_json_path && out, "null argument");
  std::unique_ptr<sfc_stage> h;
  int rc = new_stage(layout, opts, device, out, h);
  if (rc) return rc;
  const std::string ip = index_json_path;
  const std::string suffix = ".index.json";
  if (ip.size() < suffix.size() || ip.compare(ip.size() - suffix.size(), suffix.size(), suffix) != 0) {
    set_error("Packed stage index must end with .index.json");
    return SFC_E_INVALID;
  }
  std::string js, pack;
  if (!read_file(ip, js)) {
    set_error("Failed to read %s", ip.c_str());
    return SFC_E_IO;
  }
  JsonParser jp{js.data(), js.data() + js.size()};
  Json idx = jp.value();
  if (!jp.ok || idx.kind != Json::Obj) {
    set_error("%s is not valid JSON", ip.c_str());
    return SFC_E_IO;
  }
  const std::string pack_path = ip.substr(0, ip.size() - suffix.size()) + ".pack";
  if (!read_file(pack_path, pack)) {
    set_error("Packed stage file %s does not exist", pack_path.c_str());
    return SFC_E_IO;
  }
  const Json *tb = idx.get("total_bytes");
  const Json *ts = idx.get("tensors");
  if (!tb || tb->kind != Json::Num || !ts || ts->kind != Json::Arr) {
    set_error("index lacks total_bytes/tensors");
    return SFC_E_IO;
  }
  if (int64_t(pack.size()) != int64_t(tb->num)) {
    set_error("Packed stage size %lld does not match index total_bytes %lld", (long long)pack.size(),
              (long long)tb->num);
    return SFC_E_IO;
  }
  std::vector<HostTensor> hts;
  int64_t expected = 0;
  for (const Json &t : ts->arr) {
    const Json *nm = t.get("name"), *po = t.get("pack_offset"), *bl = t.get("byte_len"), *dm = t.get("dimensions"),
               *gt = t.get("ggml_type");
    if (!nm || !po || !bl || !dm || !gt || nm->kind != Json::Str || dm->kind != Json::Arr) {
      set_error("malformed tensor entry in index");
      return SFC_E_IO;
    }
    const int64_t o = int64_t(po->num), n = int64_t(bl->num);
    if (o != expected) {  // validate_offsets, lib.rs:3729-3750
      set_error("Packed tensor %s has pack_offset %lld but expected %lld", nm->str.c_str(), (long long)o,
                (long long)expected);
      return SFC_E_IO;
    }
    expected += n;
    if (expected > int64_t(pack.size())) {
      set_error("Packed tensor %s extends past the pack", nm->str.c_str());
      return SFC_E_IO;
    }
    HostTensor ht;
    ht.name = nm->str;
    ht.type = int(gt->num);
    for (const Json &d : dm->arr) ht.dims.push_back(int64_t(d.num));
    ht.data = reinterpret_cast<const uint8_t *>(pack.data()) + o;
    ht.bytes = n;
    hts.push_back(ht);
  }
  if (expected != int64_t(pack.size())) {
    set_error("Packed tensor coverage %lld does not match total_bytes %lld", (long long)expected,
              (long long)pack.size());
    return SFC_E_IO;
  }
  rc = build_stage(h.get(), hts);
  if (rc) {
    destroy_stage(h.release());
    return rc;
  }
  *out = h.release();
  return SFC_OK;
}

int sfc_stage_open_gguf(const char *gguf_path, const sfc_layout *layout, const sfc_options *opts, int device,
                        sfc_stage **out) {
  clear_error();
  SFC_REQUIRE(gguf_path && layout && out, "null argument");
  std::unique_ptr<sfc_stage> h;
  int rc = new_stage(layout, opts, device, out, h);
  if (rc) return rc;
  GgufFile f;  // mapped until this call returns (build_stage finishes its uploads first)
  std::string err;
  if (!f.bytes.map_file(gguf_path, err) || !f.parse(err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  // The tensors a runtime plan gives this stage (gguf.rs:560-616): its layers, the positional and
  // shared auxiliary tensors, the embedding on the head (and on a tail without output.weight, whose
  // logits use the tied embedding, real_forward.rs:803-816) and output* on the tail.
  const bool head = layout->is_head != 0, tail = layout->is_tail != 0;
  const bool has_output = f.find("output.weight") >= 0;
  std::vector<HostTensor> hts;
  std::set<std::string> seen;
  for (size_t k = 0; k < f.tensors.size(); ++k) {
    const GgufTensorInfo &t = f.tensors[k];
    bool take = false;
    switch (f.role[k]) {
      case ROLE_LAYER: take = f.layer[k] >= int64_t(layout->start_layer) && f.layer[k] <= int64_t(layout->end_layer); break;
      case ROLE_PROMPT_INGRESS: take = head || (tail && !has_output); break;
      case ROLE_POSITIONAL:
      case ROLE_SHARED_AUX: take = true; break;
      case ROLE_TAIL_ONLY: take = tail; break;
      default: take = false;
    }
    if (!take || !seen.insert(t.name).second) continue;  // a repeated name: the first one, as lookups find
    HostTensor ht;
    ht.name = t.name;
    ht.type = int(t.type);
    double elems = 1.0;
    for (uint64_t d : t.dims) {
      SFC_REQUIRE(d < (uint64_t(1) << 40), "tensor %s: dimension %llu too large", t.name.c_str(),
                  (unsigned long long)d);
      ht.dims.push_back(int64_t(d));
      elems *= double(d);
    }
    SFC_REQUIRE(elems < 281474976710656.0, "tensor %s: %.0f elements is too many", t.name.c_str(), elems);  // 2^48
    const int64_t gb = gguf_tensor_bytes(ht.type, ht.dims);
    const uint64_t off = f.data_offset + t.offset;
    if (gb >= 0) {
      SFC_REQUIRE(uint64_t(gb) <= f.byte_len[k], "tensor %s: %lld bytes implied by its dims but %llu before the next tensor",
                  t.name.c_str(), (long long)gb, (unsigned long long)f.byte_len[k]);
      SFC_REQUIRE(off <= f.file_size && uint64_t(gb) <= f.file_size - off, "tensor %s runs past the end of %s",
                  t.name.c_str(), gguf_path);
    }
    ht.data = f.bytes.data + (off <= f.file_size ? off : 0);
    ht.bytes = gb >= 0 ? gb : int64_t(f.byte_len[k]);  // an unsupported type fails in build_stage
    hts.push_back(ht);
  }
  rc = build_stage(h.get(), hts);
  if (rc) {
    destroy_stage(h.release());
    return rc;
  }
  *out = h.release();
  return SFC_OK;
}

int sfc_stage_open_synthetic(const sfc_synth_spec *spec, const sfc_layout *layout, const sfc_options *opts,
                             int device, sfc_stage **out) {
  clear_error();
  SFC_REQUIRE(spec && out, "null argument");
  std::unique_ptr<sfc_stage> h;
  int rc = new_stage(layout, opts, device, out, h);
  if (rc) return rc;
  SFC_REQUIRE(spec->hidden > 0 && spec->n_heads > 0 && spec->n_kv > 0 && spec->head_dim > 0 && spec->ffn > 0 &&
                  spec->vocab > 0,
              "bad synthetic spec");
  SFC_REQUIRE(h->start_layer <= h->end_layer && int(h->end_layer) < spec->n_layers_total, "bad layer range");
  std::vector<HostTensor> hts;
  const int64_t H = spec->hidden, Q = int64_t(spec->n_heads) * spec->head_dim,
                K = int64_t(spec->n_kv) * spec->head_dim, F = spec->ffn, D = spec->head_dim;
  auto add = [&](const std::string &name, int type, std::vector<int64_t> dims, float sigma, float mean, bool ones) {
    HostTensor ht;
    ht.name = name;
    ht.type = type;
    ht.dims = dims;
    ht.data = nullptr;
    ht.bytes = 0;
    ht.synthetic = !ones;
    ht.ones = ones;
    ht.key = tensor_key(spec->seed, name.c_str());
    ht.sigma = sigma;
    ht.mean = mean;
    hts.push_back(ht);
  };
  if (h->is_head || h->is_tail) add("token_embd.weight", spec->type_embd, {H, spec->vocab}, spec->embd_sigma, 0, false);
  add("rope_freqs.weight", T_F32, {D / 2}, 0, 0, true);
  for (uint32_t i = h->start_layer; i <= h->end_layer; ++i) {
    const std::string p = "blk." + std::to_string(i);
    add(p + ".attn_norm.weight", T_F32, {H}, spec->norm_sigma, 1.0f, false);
    add(p + ".attn_q.weight", spec->type_q, {H, Q}, spec->w_sigma, 0, false);
    add(p + ".attn_k.weight", spec->type_k, {H, K}, spec->w_sigma, 0, false);
    add(p + ".attn_v.weight", spec->type_v, {H, K}, spec->w_sigma, 0, false);
    add(p + ".attn_q_norm.weight", T_F32, {D}, spec->norm_sigma, 1.0f, false);
    add(p + ".attn_k_norm.weight", T_F32, {D}, spec->norm_sigma, 1.0f, false);
    add(p + ".attn_output.weight", spec->type_o, {Q, H}, spec->w_sigma, 0, false);
    add(p + ".post_attention_norm.weight", T_F32, {H}, spec->norm_sigma, 1.0f, false);
    add(p + ".ffn_norm.weight", T_F32, {H}, spec->norm_sigma, 1.0f, false);
    add(p + ".ffn_gate.weight", spec->type_gate, {H, F}, spec->w_sigma, 0, false);
    add(p + ".ffn_up.weight", spec->type_up, {H, F}, spec->w_sigma, 0, false);
    add(p + ".ffn_down.weight", spec->type_down, {F, H}, spec->w_sigma, 0, false);
    add(p + ".post_ffw_norm.weight", T_F32, {H}, spec->norm_sigma, 1.0f, false);
  }
  if (h->is_tail) add("output_norm.weight", T_F32, {H}, spec->norm_sigma, 1.0f, false);
  rc = build_stage(h.get(), hts);
  if (rc) {
    destroy_stage(h.release());
    return rc;
  }
  *out = h.release();
  return SFC_OK;
}

int sfc_stage_close(sfc_stage *h) {
  destroy_stage(h);
  return SFC_OK;
}

int sfc_stage_get_info(sfc_stage *h, sfc_stage_info *info) {
  SFC_REQUIRE(h && info, "null argument");
  info->hidden = h->hidden;
  info->n_heads = h->n_heads;
  info->n_kv = h->n_kv;
  info->head_dim = h->head_dim;
  info->ffn = h->ffn;
  info->n_layers = int(h->layers.size());
  info->vocab = h->vocab;
  info->is_head = h->is_head;
  info->is_tail = h->is_tail;
  info->weight_bytes = h->weight_bytes;
  info->kv_bytes = h->kv_bytes;
  return SFC_OK;
}

int sfc_begin_token_ids(sfc_stage *h, const char *request_id, const uint32_t *ids, int64_t n, float *out_hidden) {
  clear_error();
  SFC_REQUIRE(h && ids, "null argument");
  SFC_REQUIRE(h->is_head, "Only the head stage may accept prompt ingress");
  return forward_single(h, request_id, ids, nullptr, n, out_hidden, n > 1);
}

int sfc_begin_token_ids_bytes(sfc_stage *h, const char *request_id, const uint32_t *ids, int64_t n, void *out,
                              uint64_t cap, uint64_t *out_len) {
  clear_error();
  SFC_REQUIRE(h && ids && out_len, "null argument");
  SFC_REQUIRE(h->is_head, "Only the head stage may accept prompt ingress");
  SFC_REQUIRE(n > 0, "Empty prompt");
  const int64_t LP = h->ple ? int64_t(h->ple_layers) * h->ple_dim : 0;
  const uint64_t hidden_len = uint64_t(n) * h->hidden * 4;
  const uint64_t aux_len = (LP || n > 1) ? 20 + uint64_t(n) * LP * 4 + (n > 1 ? uint64_t(n) * 8 : 0) : 0;
  const uint64_t need = encoded_stage_tensor_bytes(hidden_len, aux_len);
  *out_len = need;
  SFC_REQUIRE(out && cap >= need, "output holds %llu bytes, the payload needs %llu", (unsigned long long)cap,
              (unsigned long long)need);
  std::vector<float> rows(size_t(n) * h->hidden), ple(size_t(n * LP));
  h->ple_out = LP ? ple.data() : nullptr;
  const int rc = forward_single(h, request_id, ids, nullptr, n, rows.data(), n > 1);
  h->ple_out = nullptr;
  if (rc) return rc;
  // begin_token_sequence (real_forward.rs:1096-1103): prefix hashes of a multi-token prompt and the
  // per-layer inputs of every model layer travel in the aux section
  const std::vector<uint8_t> aux = encode_prompt_aux(LP ? ple.data() : nullptr, uint32_t(n), uint32_t(h->ple_layers),
                                                     uint32_t(h->ple_dim),
                                                     n > 1 ? prefix_hashes(ids, n) : std::vector<uint64_t>());
  SFC_REQUIRE(aux.size() == aux_len, "prompt aux size %zu, expected %llu", aux.size(), (unsigned long long)aux_len);
  encode_stage_tensor(reinterpret_cast<const uint8_t *>(rows.data()), hidden_len, aux.data(), aux.size(),
                      static_cast<uint8_t *>(out));
  return SFC_OK;
}

int sfc_continue_forward(sfc_stage *h, const char *request_id, const float *in_hidden, int64_t n, float *out_hidden) {
  clear_error();
  SFC_REQUIRE(h && in_hidden, "null argument");
  SFC_REQUIRE(!h->is_head, "Head stage should use begin_prompt, not continue_forward");
  return forward_single(h, request_id, nullptr, in_hidden, n, out_hidden, n > 1);
}

int sfc_sample_tail(sfc_stage *h, const float *hidden, int64_t n, uint32_t *token, float *score) {
  clear_error();
  SFC_REQUIRE(h && hidden && token, "null argument");
  SFC_REQUIRE(n > 0, "Hidden-state payload is empty");
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  SFC_CUDA(cudaMemcpyAsync(h->proj, hidden + (n - 1) * h->hidden, size_t(h->hidden) * 4, cudaMemcpyHostToDevice, st));
  int rc = sample_rows(h, h->proj, 1, h->tok_dev, h->score_dev, st);
  if (rc) return rc;
  int64_t t = 0;
  float s = 0;
  SFC_CUDA(cudaMemcpyAsync(&t, h->tok_dev, 8, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaMemcpyAsync(&s, h->score_dev, 4, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  *token = uint32_t(t);
  if (score) *score = s;
  return SFC_OK;
}

// The hidden rows of a hand-off payload, checked as decode_hidden_states (real_forward.rs:1826-1850).
static int payload_rows(const sfc_stage *h, const void *bytes, uint64_t n, uint64_t hidden_dim, PayloadSections &s,
                        std::vector<float> &rows) {
  SFC_REQUIRE(bytes || n == 0, "null argument");
  stage_tensor_sections(static_cast<const uint8_t *>(bytes), n, s);
  SFC_REQUIRE(hidden_dim != 0, "Hidden-state hidden_dim must be nonzero");
  SFC_REQUIRE(s.hidden_len % (hidden_dim * 4) == 0,
              "Hidden-state byte length %llu is not a multiple of hidden_dim * 4 = %llu",
              (unsigned long long)s.hidden_len, (unsigned long long)(hidden_dim * 4));
  SFC_REQUIRE(hidden_dim == uint64_t(h->hidden), "payload hidden_dim %llu, stage hidden size %d",
              (unsigned long long)hidden_dim, h->hidden);
  SFC_REQUIRE(s.hidden_len > 0, "Hidden-state payload is empty");
  rows.resize(size_t(s.hidden_len / 4));
  memcpy(rows.data(), s.hidden, size_t(s.hidden_len));  // any alignment in, aligned floats out
  return SFC_OK;
}

int sfc_continue_forward_bytes(sfc_stage *h, const char *request_id, const void *bytes, uint64_t n,
                               uint64_t hidden_dim, void *out, uint64_t cap, uint64_t *out_len) {
  clear_error();
  SFC_REQUIRE(h && request_id && out_len, "null argument");
  SFC_REQUIRE(!h->is_head, "Head stage should use begin_prompt, not continue_forward");
  PayloadSections s;
  std::vector<float> in;
  int rc = payload_rows(h, bytes, n, hidden_dim, s, in);
  if (rc) return rc;
  const uint64_t need = encoded_stage_tensor_bytes(s.hidden_len, s.aux_len);
  *out_len = need;
  SFC_REQUIRE(out && cap >= need, "output holds %llu bytes, the payload needs %llu", (unsigned long long)cap,
              (unsigned long long)need);
  const std::string aux(reinterpret_cast<const char *>(s.aux), s.aux ? size_t(s.aux_len) : 0);  // out may be bytes
  const int64_t rows = int64_t(in.size() / size_t(h->hidden));
  std::vector<float> ple;  // per-layer inputs of the rows, [rows][ple_layers * ple_dim]
  if (h->ple) {
    // decode_prompt_aux (real_forward.rs:1896-1990); the per-layer inputs of every model layer
    SFC_REQUIRE(s.aux, "stage %s has per-layer embedding (PLE) layers but the payload carries no prompt aux",
                h->stage_id.c_str());
    PromptAux pa;
    std::string err;
    SFC_REQUIRE(decode_prompt_aux(reinterpret_cast<const uint8_t *>(aux.data()), aux.size(), pa, err), "%s",
                err.c_str());
    SFC_REQUIRE(pa.ple && int64_t(pa.seq) == rows && int(pa.ple_dim) == h->ple_dim && int(pa.layers) >= h->ple_layers,
                "prompt aux holds %u x %u x %u per-layer inputs; the stage needs %lld rows x %d layers x %d",
                pa.seq, pa.layers, pa.ple_dim, (long long)rows, h->ple_layers, h->ple_dim);
    const int64_t LP = int64_t(h->ple_layers) * h->ple_dim, LPin = int64_t(pa.layers) * pa.ple_dim;
    ple.resize(size_t(rows * LP));
    for (int64_t r = 0; r < rows; ++r)
      memcpy(ple.data() + r * LP, reinterpret_cast<const uint8_t *>(pa.ple) + r * LPin * 4, size_t(LP) * 4);
  }
  std::vector<float> res(in.size());
  h->ple_in = h->ple ? ple.data() : nullptr;
  rc = sfc_continue_forward(h, request_id, in.data(), rows, res.data());
  h->ple_in = nullptr;
  if (rc) return rc;
  encode_stage_tensor(reinterpret_cast<const uint8_t *>(res.data()), s.hidden_len,
                      reinterpret_cast<const uint8_t *>(aux.data()), aux.size(), static_cast<uint8_t *>(out));
  return SFC_OK;
}

int sfc_sample_tail_bytes(sfc_stage *h, const void *bytes, uint64_t n, uint64_t hidden_dim, uint32_t *token,
                          float *score) {
  clear_error();
  SFC_REQUIRE(h && token, "null argument");
  PayloadSections s;
  std::vector<float> rows;
  int rc = payload_rows(h, bytes, n, hidden_dim, s, rows);
  if (rc) return rc;
  return sfc_sample_tail(h, rows.data(), int64_t(rows.size() / size_t(h->hidden)), token, score);  // last row
}

int sfc_forward_dev(sfc_stage *h, const char *const *request_ids, const int32_t *seq_tokens, int n_seq,
                    const uint32_t *ids_dev, const float *in_dev, float *out_dev, int append, void *stream) {
  clear_error();
  SFC_REQUIRE(h && request_ids && seq_tokens && n_seq > 0 && out_dev, "null argument");
  SFC_REQUIRE(n_seq <= h->max_sessions, "batch of %d sequences exceeds max_sessions %d", n_seq, h->max_sessions);
  SFC_REQUIRE(h->is_head ? ids_dev != nullptr : in_dev != nullptr, "missing input");
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL = the legacy default stream, as documented
  std::vector<SeqReq> seqs;
  int64_t T = 0;
  for (int i = 0; i < n_seq; ++i) {
    SFC_REQUIRE(request_ids[i], "null request id");
    Session *s = nullptr;
    int rc = session_for(h, request_ids[i], !append, &s);
    if (rc) return rc;
    for (auto &o : seqs) SFC_REQUIRE(o.s != s, "request %s appears twice in one batch", request_ids[i]);
    seqs.push_back(SeqReq{s, seq_tokens[i]});
    T += seq_tokens[i];
  }
  if (n_seq == 1 && T > h->max_batch) {  // long single sequence: chunk it
    for (int64_t t0 = 0; t0 < T; t0 += h->max_batch) {
      const int32_t c = int32_t(std::min<int64_t>(h->max_batch, T - t0));
      int rc = forward_chunk(h, {SeqReq{seqs[0].s, c}}, ids_dev ? ids_dev + t0 : nullptr, true,
                             in_dev ? in_dev + t0 * h->hidden : nullptr, st);
      if (rc) return rc;
      SFC_CUDA(cudaMemcpyAsync(out_dev + t0 * h->hidden, h->resid, size_t(c) * h->hidden * 4,
                               cudaMemcpyDeviceToDevice, st));
    }
    return SFC_OK;
  }
  int rc = forward_chunk(h, seqs, ids_dev, true, in_dev, st);
  if (rc) return rc;
  SFC_CUDA(cudaMemcpyAsync(out_dev, h->resid, size_t(T) * h->hidden * 4, cudaMemcpyDeviceToDevice, st));
  return SFC_OK;
}

int sfc_sample_dev(sfc_stage *h, const float *hidden_dev, int64_t n, int64_t *tokens_dev, float *scores_dev,
                   void *stream) {
  clear_error();
  SFC_REQUIRE(h && hidden_dev && tokens_dev && scores_dev, "null argument");
  SFC_CUDA(cudaSetDevice(h->device));
  return sample_rows(h, hidden_dev, n, tokens_dev, scores_dev,
                     static_cast<cudaStream_t>(stream));
}

int sfc_verify_greedy(sfc_stage *h, const float *hidden, const uint32_t *drafts, int64_t k, int64_t *accepted,
                      uint32_t *bonus) {
  clear_error();
  SFC_REQUIRE(h && hidden && accepted && bonus && (k == 0 || drafts), "null argument");
  SFC_REQUIRE(k >= 0 && k + 1 <= h->max_batch, "k out of range");
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  SFC_CUDA(cudaMemcpyAsync(h->proj, hidden, size_t(k + 1) * h->hidden * 4, cudaMemcpyHostToDevice, st));
  int rc = sample_rows(h, h->proj, k + 1, h->tok_dev, h->score_dev, st);
  if (rc) return rc;
  std::vector<int64_t> am((size_t)(k + 1));
  SFC_CUDA(cudaMemcpyAsync(am.data(), h->tok_dev, size_t(k + 1) * 8, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  // lib.rs:2143-2164: accept while argmax at position i equals draft i; bonus = first mismatch.
  int64_t acc = 0;
  while (acc < k && uint32_t(am[size_t(acc)]) == drafts[acc]) ++acc;
  *accepted = acc;
  *bonus = uint32_t(am[size_t(acc)]);
  return SFC_OK;
}

int sfc_forward_tree(sfc_stage *h, const char *request_id, const uint32_t *ids, const float *in_hidden,
                     const int32_t *parent, int64_t n, float *out_hidden) {
  clear_error();
  SFC_REQUIRE(h && request_id && parent && out_hidden, "null argument");
  SFC_REQUIRE(h->is_head ? ids != nullptr : in_hidden != nullptr,
              h->is_head ? "head stage needs token ids" : "non-head stage needs hidden rows");
  SFC_REQUIRE(n >= 1 && n <= 64 && n <= h->max_batch, "tree of %lld nodes (1..64 and <= max_batch_tokens)",
              (long long)n);
  SFC_REQUIRE(parent[0] == -1, "node 0 must be the root (parent -1)");
  auto it = h->sessions.find(request_id);
  SFC_REQUIRE(it != h->sessions.end(), "unknown session %s", request_id);
  Session *s = &it->second;
  SFC_REQUIRE(s->len + n <= h->max_ctx, "session needs %lld positions but max_ctx is %d", (long long)(s->len + n),
              h->max_ctx);
  std::vector<int32_t> rope(static_cast<size_t>(n)), limit(static_cast<size_t>(n));
  std::vector<uint64_t> mask(static_cast<size_t>(n));
  std::vector<int32_t> depth(static_cast<size_t>(n), 0);
  for (int64_t i = 0; i < n; ++i) {
    if (i > 0) {
      SFC_REQUIRE(parent[i] >= 0 && parent[i] < i, "parent[%lld] = %d must precede its node", (long long)i,
                  parent[i]);
      depth[size_t(i)] = depth[size_t(parent[i])] + 1;
      mask[size_t(i)] = mask[size_t(parent[i])];
    }
    mask[size_t(i)] |= 1ull << i;  // ancestors and the node itself
    rope[size_t(i)] = int32_t(s->len + depth[size_t(i)]);
    limit[size_t(i)] = int32_t(s->len + i + 1);
  }
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  SFC_CUDA(cudaMemcpyAsync(h->tree_rope_dev, rope.data(), size_t(n) * 4, cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaMemcpyAsync(h->tree_limit_dev, limit.data(), size_t(n) * 4, cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaMemcpyAsync(h->tree_mask_dev, mask.data(), size_t(n) * 8, cudaMemcpyHostToDevice, st));
  if (!h->is_head)
    SFC_CUDA(cudaMemcpyAsync(h->hn, in_hidden, size_t(n) * h->hidden * 4, cudaMemcpyHostToDevice, st));
  const int64_t len0 = s->len;
  h->tree_active = true;
  int rc = forward_chunk(h, {SeqReq{s, int32_t(n)}}, ids, false, h->hn, st);
  h->tree_active = false;
  s->len = len0;  // tentative: sfc_commit_tree keeps the accepted path
  if (rc) return rc;
  s->tree_parent.assign(parent, parent + n);
  SFC_CUDA(cudaMemcpyAsync(out_hidden, h->resid, size_t(n) * h->hidden * 4, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  return SFC_OK;
}

int sfc_sample_tree(sfc_stage *h, const float *hidden, const int32_t *parent, const uint32_t *node_tokens, int64_t n,
                    float temperature, uint64_t seed, int32_t *path, int64_t *n_path, uint32_t *next_token) {
  clear_error();
  SFC_REQUIRE(h && hidden && parent && node_tokens && path && n_path && next_token, "null argument");
  SFC_REQUIRE(h->is_tail, "Only the tail stage may sample");
  SFC_REQUIRE(n >= 1 && n <= 64 && n <= h->max_batch, "tree of %lld nodes (1..64 and <= max_batch_tokens)",
              (long long)n);
  SFC_REQUIRE(parent[0] == -1, "node 0 must be the root (parent -1)");
  for (int64_t i = 1; i < n; ++i)
    SFC_REQUIRE(parent[i] >= 0 && parent[i] < i, "parent[%lld] = %d must precede its node", (long long)i, parent[i]);
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  if (!tail_gemm_eligible(h, n) && h->tree_scores_rows < n) {
    if (h->tree_scores) cudaFree(h->tree_scores);
    h->tree_scores = nullptr;
    h->tree_scores_rows = 0;
    SFC_CUDA(cudaMalloc(&h->tree_scores, size_t(64) * h->vocab * 4));
    h->tree_scores_rows = 64;
  }
  SFC_CUDA(cudaMemcpyAsync(h->proj, hidden, size_t(n) * h->hidden * 4, cudaMemcpyHostToDevice, st));
  const float *capped = h->tree_scores;
  if (tail_gemm_eligible(h, n)) {  // tensor-core logits: capped scores in h->logit_scores
    int rc = tail_logits_gemm(h, h->proj, n, h->tok_dev, h->score_dev, st);
    if (rc) return rc;
    capped = h->logit_scores;
  } else {
    if (h->output_norm)
      SFC_CUDA(rms_norm(h->proj, F32P(h->output_norm), n, h->hidden, h->eps, h->hn, st));
    else
      SFC_CUDA(cudaMemcpyAsync(h->hn, h->proj, size_t(n) * h->hidden * 4, cudaMemcpyDeviceToDevice, st));
    SFC_CUDA(logits_argmax(h->logits_w->type, h->logits_w->dev, h->vocab, h->hidden, h->hn, n, h->softcap,
                           h->tree_scores, h->tok_dev, h->score_dev, h->scratch,
                           std::max(h->attn_scratch, h->logit_scratch), st));
  }
  if (temperature > 0.f) SFC_CUDA(sample_rows_temperature(capped, n, h->vocab, temperature, seed, h->tok_dev, st));
  std::vector<int64_t> drawn(static_cast<size_t>(n));
  SFC_CUDA(cudaMemcpyAsync(drawn.data(), h->tok_dev, size_t(n) * 8, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  // walk from the root: the token drawn at a node is accepted if a child carries it (the first
  // such child in node order); the token drawn where the walk stops is the next token
  int64_t m = 0, cur = 0;
  path[m++] = 0;
  for (;;) {
    int64_t nxt = -1;
    for (int64_t c = cur + 1; c < n; ++c)
      if (parent[c] == cur && node_tokens[c] == uint32_t(drawn[size_t(cur)])) {
        nxt = c;
        break;
      }
    if (nxt < 0) break;
    path[m++] = int32_t(nxt);
    cur = nxt;
  }
  *n_path = m;
  *next_token = uint32_t(drawn[size_t(cur)]);
  return SFC_OK;
}

int sfc_commit_tree(sfc_stage *h, const char *request_id, const int32_t *path, int64_t n_path) {
  clear_error();
  SFC_REQUIRE(h && request_id && path, "null argument");
  auto it = h->sessions.find(request_id);
  SFC_REQUIRE(it != h->sessions.end(), "unknown session %s", request_id);
  Session *s = &it->second;
  const int64_t pending = int64_t(s->tree_parent.size());
  SFC_REQUIRE(pending > 0, "session %s has no draft tree pending (sfc_forward_tree first; a tree is committed once)",
              request_id);
  SFC_REQUIRE(n_path >= 1 && n_path <= pending && path[0] == 0, "path must start at the root and hold 1..%lld nodes",
              (long long)pending);
  for (int64_t i = 1; i < n_path; ++i)
    SFC_REQUIRE(path[i] > 0 && path[i] < pending && s->tree_parent[size_t(path[i])] == path[i - 1],
                "path[%lld] = %d is not a child of node %d in the pending tree", (long long)i, path[i], path[i - 1]);
  SFC_REQUIRE(s->len + path[n_path - 1] < h->max_ctx, "path leaves the cache");
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  if (h->kv_arena && !h->layers.empty()) {
    SFC_CUDA(cudaMemcpyAsync(h->tree_path_dev, path, size_t(n_path) * 4, cudaMemcpyHostToDevice, st));
    SFC_CUDA(kv_compact(h->kv_arena, h->kv_slabs, h->max_sessions, h->kv_slot_stride, s->slot, h->n_kv,
                        h->max_ctx, h->head_dim, h->kv_f32 ? 4 : 2, int(s->len), h->tree_path_dev, int(n_path), st));
    SFC_CUDA(cudaStreamSynchronize(st));
  }
  s->len += n_path;
  s->tree_parent.clear();
  return SFC_OK;
}

int sfc_clear_decode_session(sfc_stage *h, const char *request_id) {
  SFC_REQUIRE(h && request_id, "null argument");
  auto it = h->sessions.find(request_id);
  if (it != h->sessions.end()) {
    h->slot_used[size_t(it->second.slot)] = 0;
    h->sessions.erase(it);
  }
  return SFC_OK;
}

int sfc_rollback_kv(sfc_stage *h, const char *request_id, int64_t keep) {
  SFC_REQUIRE(h && request_id, "null argument");
  auto it = h->sessions.find(request_id);
  SFC_REQUIRE(it != h->sessions.end(), "unknown session %s", request_id);
  SFC_REQUIRE(keep >= 0 && keep <= it->second.len, "keep_count %lld exceeds session length %lld", (long long)keep,
              (long long)it->second.len);
  it->second.len = keep;
  it->second.tree_parent.clear();
  return SFC_OK;
}

int64_t sfc_session_len(sfc_stage *h, const char *request_id) {
  if (!h || !request_id) return SFC_E_INVALID;
  auto it = h->sessions.find(request_id);
  return it == h->sessions.end() ? 0 : it->second.len;
}

int sfc_session_fill_synthetic(sfc_stage *h, const char *request_id, int64_t n_pos, uint64_t seed) {
  clear_error();
  SFC_REQUIRE(h && request_id, "null argument");
  SFC_REQUIRE(n_pos >= 0 && n_pos <= h->max_ctx, "n_pos %lld out of range", (long long)n_pos);
  SFC_CUDA(cudaSetDevice(h->device));
  Session *s = nullptr;
  int rc = session_for(h, request_id, true, &s);
  if (rc) return rc;
  const int64_t elt = h->kv_f32 ? 4 : 2;
  for (size_t li = 0; li < h->layers.size(); ++li) {
    if (!h->layers[li].own_kv()) continue;  // its cache is its source layer's
    KVLayer kv = kv_layer(h, li);
    for (int part = 0; part < 2; ++part)
      for (int kh = 0; kh < h->n_kv; ++kh) {
        char *base = static_cast<char *>(kv.base) +
                     (int64_t(s->slot) * kv.slot_stride + part * (kv.slot_stride / 2) +
                      int64_t(kh) * h->max_ctx * h->head_dim) *
                         elt;
        const std::string nm = "kv." + std::to_string(li) + "." + std::to_string(part) + "." + std::to_string(kh);
        SFC_CUDA(synth_tensor(h->kv_f32 ? T_F32 : T_F16, tensor_key(seed, nm.c_str()), n_pos, h->head_dim, 1.0f,
                              0.0f, base, h->stream));
      }
  }
  SFC_CUDA(cudaStreamSynchronize(h->stream));
  s->len = n_pos;
  return SFC_OK;
}

int sfc_generate_greedy(sfc_stage *h, const char *request_id, const uint32_t *prompt, int64_t n_prompt,
                        int64_t n_steps, uint32_t *out_tokens) {
  clear_error();
  SFC_REQUIRE(h && request_id && prompt && out_tokens, "null argument");
  SFC_REQUIRE(h->is_head && h->is_tail, "greedy generation needs a whole-model stage (head and tail)");
  SFC_REQUIRE(n_prompt > 0 && n_steps > 0, "empty prompt or no steps");
  SFC_REQUIRE(n_prompt + n_steps <= h->max_ctx, "prompt + steps exceed max_ctx %d", h->max_ctx);
  SFC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = h->stream;
  int rc = forward_single(h, request_id, prompt, nullptr, n_prompt, nullptr, true);
  if (rc) return rc;
  Session *s = &h->sessions[request_id];
  // first token from the last prompt row
  const int64_t last = (n_prompt - 1) % h->max_batch;
  rc = sample_rows(h, h->resid + last * h->hidden, 1, h->tok_dev, h->score_dev, st);
  if (rc) return rc;
  if (h->gen_capacity < n_steps) {
    if (h->decode_graph) {  // the graph holds the old token buffer and step bound
      cudaGraphExecDestroy(h->decode_graph);
      h->decode_graph = nullptr;
    }
    if (h->gen_tokens_dev) cudaFree(h->gen_tokens_dev);
    h->gen_tokens_dev = nullptr;
    SFC_CUDA(cudaMalloc(&h->gen_tokens_dev, size_t(n_steps) * 8));
    h->gen_capacity = n_steps;
  }
  SFC_CUDA(cudaMemcpyAsync(h->gen_tokens_dev, h->tok_dev, 8, cudaMemcpyDeviceToDevice, st));
  const int32_t one = 1;
  SeqInfo si{s->slot, int32_t(s->len), 1, 0};
  const int32_t zero = 0;
  SFC_CUDA(cudaMemcpyAsync(h->step_dev, &one, 4, cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaMemcpyAsync(h->seq_dev, &si, sizeof(si), cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaMemcpyAsync(h->tok_seq_dev, &zero, 4, cudaMemcpyHostToDevice, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  if (n_steps > 1) {
    if (!h->decode_graph) {
      cudaGraph_t g = nullptr;
      const long long k0 = g_kernel_launches;
      SFC_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      cudaError_t e = head_ingress(h, h->tok_dev, 1, 1, st);
      if (!e) e = run_layers(h, 1, h->max_ctx, true, st);
      if (!e) {
        if (h->output_norm)
          e = rms_norm(h->resid, F32P(h->output_norm), 1, h->hidden, h->eps, h->hn, st);
        else
          e = cudaMemcpyAsync(h->hn, h->resid, size_t(h->hidden) * 4, cudaMemcpyDeviceToDevice, st);
      }
      if (!e)
        e = logits_argmax(h->logits_w->type, h->logits_w->dev, h->vocab, h->hidden, h->hn, 1, h->softcap, nullptr,
                          h->tok_dev, h->score_dev, h->scratch, std::max(h->attn_scratch, h->logit_scratch), st);
      if (!e) e = decode_advance(h->tok_dev, h->gen_tokens_dev, h->step_dev, h->seq_dev, 1, h->gen_capacity, st);
      cudaError_t e2 = cudaStreamEndCapture(st, &g);
      if (e) return cuda_fail(e, "decode graph capture");
      if (e2) return cuda_fail(e2, "cudaStreamEndCapture");
      h->graph_kernels = g_kernel_launches - k0;
      e = cudaGraphInstantiate(&h->decode_graph, g, 0);
      cudaGraphDestroy(g);
      if (e) return cuda_fail(e, "cudaGraphInstantiate");
    }
    SFC_CUDA(cudaEventRecord(h->ev0, st));
    for (int64_t i = 1; i < n_steps; ++i) SFC_CUDA(cudaGraphLaunch(h->decode_graph, st));
    SFC_CUDA(cudaEventRecord(h->ev1, st));
  }
  std::vector<int64_t> toks((size_t)n_steps);
  SFC_CUDA(cudaMemcpyAsync(toks.data(), h->gen_tokens_dev, size_t(n_steps) * 8, cudaMemcpyDeviceToHost, st));
  SFC_CUDA(cudaStreamSynchronize(st));
  for (int64_t i = 0; i < n_steps; ++i) out_tokens[i] = uint32_t(toks[size_t(i)]);
  s->len += n_steps - 1;
  if (n_steps > 1) {
    float ms = 0;
    cudaEventElapsedTime(&ms, h->ev0, h->ev1);
    h->profile.total_us = ms * 1e3;
    h->profile.seq_len = n_steps - 1;
    h->profile.kernels = h->graph_kernels * (n_steps - 1);
  }
  unsigned derr = 0;
  unsigned *dp = device_error_ptr();
  if (dp && cudaMemcpy(&derr, dp, 4, cudaMemcpyDeviceToHost) == cudaSuccess && derr) {
    unsigned z = 0;
    cudaMemcpy(dp, &z, 4, cudaMemcpyHostToDevice);
    set_error("device reported error code %u", derr);
    return SFC_E_DEVICE;
  }
  return SFC_OK;
}

int sfc_last_profile(sfc_stage *h, sfc_profile *out) {
  SFC_REQUIRE(h && out, "null argument");
  *out = h->profile;
  return SFC_OK;
}

}  // extern "C"
