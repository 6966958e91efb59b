// gguf.h — GGUF shard files on the host: parsing, tensor roles, stage splits, the shard manifest
// bundle and packed stages (crates/stage-forward-lab/src/gguf.rs, lib.rs:3283-3613).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace sfc {

// One metadata value (GGUF types 0..12: u8 i8 u16 i16 u32 i32 f32 bool string array u64 i64 f64).
struct GgufValue {
  uint32_t type = 0;
  uint64_t u = 0;  // unsigned types and bool
  int64_t i = 0;   // signed types
  double f = 0;    // f32 (exactly widened) and f64
  std::string s;
  std::vector<GgufValue> arr;
};

struct GgufTensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;  // relative to the tensor data section
};

// A read-only memory mapping of a file (or an owned copy of caller bytes).
struct GgufBytes {
  const uint8_t *data = nullptr;
  uint64_t size = 0;
  void *map = nullptr;  // mmap base, if mapped
  std::vector<uint8_t> copy;
  GgufBytes() = default;
  GgufBytes(const GgufBytes &) = delete;
  GgufBytes &operator=(const GgufBytes &) = delete;
  ~GgufBytes();
  bool map_file(const std::string &path, std::string &err);
  void own(const void *bytes, uint64_t n);
};

enum GgufRole { ROLE_LAYER = 0, ROLE_PROMPT_INGRESS = 1, ROLE_POSITIONAL = 2, ROLE_SHARED_AUX = 3, ROLE_TAIL_ONLY = 4,
                ROLE_UNKNOWN_GLOBAL = 5 };

struct GgufFile {
  uint32_t version = 0;
  uint64_t tensor_count = 0, file_size = 0, data_offset = 0;
  std::map<std::string, GgufValue> meta;  // sorted by key, a repeated key keeps its last value
  std::vector<GgufTensorInfo> tensors;
  GgufBytes bytes;
  // derived per tensor (same order as `tensors`)
  std::vector<uint64_t> byte_len;  // tensor_byte_len of the tensor's name
  std::vector<int> role;
  std::vector<int64_t> layer;      // layer index of ROLE_LAYER, else -1

  // gguf.rs:144-210.  Returns false with `err` set on malformed input.
  bool parse(std::string &err);
  const GgufValue *get(const std::string &key) const;
  bool architecture(std::string &out) const;                       // gguf.rs:212-217
  std::vector<uint32_t> block_indices() const;                     // :219-233
  int64_t layer_count() const;                                     // :235-247, -1 if none
  bool meta_string(const std::string &key, std::string &out) const;  // :249-251
  bool meta_u32(const std::string &key, uint32_t &out) const;      // :279-287
  int64_t hidden_size() const;                                     // :289-293, -1 if none
  int64_t feed_forward_length() const;                             // :295-299
  int64_t attention_head_count() const;                            // :301-305
  int64_t find(const std::string &name) const;                     // first tensor of that name, -1
  bool tensor_byte_len(const std::string &name, uint64_t &out) const;  // :331-343
};

struct StageSplitC {
  uint32_t stage_index, start_layer, end_layer;
};

bool gguf_even_split(const GgufFile &f, uint32_t stages, std::vector<StageSplitC> &out);  // gguf.rs:307-329
int classify_tensor_role(const std::string &name, int64_t *layer);                      // gguf.rs:753-786
std::string gguf_value_string(const GgufValue &v);                                       // gguf.rs:800-823
bool parse_block_index(const std::string &name, uint32_t &idx);  // "blk.<u32>." prefix rule

// plan_for_splits + build_manifest + write_bundle (gguf.rs:366-751) into out_dir.
bool gguf_write_bundle(const GgufFile &f, const std::vector<StageSplitC> &splits, const std::string &out_dir,
                       std::string &err);
// StageResidencyAdapter::load + materialize_required_tensors (lib.rs:3424-3510): one file per
// required tensor, named by sanitize_tensor_filename.
bool materialize_stage_from_bundle(const std::string &bundle_dir, const std::string &gguf_path, uint32_t stage_index,
                                   const std::string &out_dir, std::vector<std::string> &written, std::string &err);
// StageResidencyAdapter::load + pack_required_tensors / pack_all_tensors (lib.rs:3283-3613).
bool pack_stage_from_bundle(const std::string &bundle_dir, const std::string &gguf_path, uint32_t stage_index,
                            bool include_optional, const std::string &out_dir, std::string &index_path,
                            std::string &err);

}  // namespace sfc
