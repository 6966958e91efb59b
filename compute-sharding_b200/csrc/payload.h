// payload.h — stage hand-off byte layout (bare or "stb1"-framed hidden rows plus an aux section).
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace sfc {

struct PayloadSections {
  const uint8_t *hidden;
  uint64_t hidden_len;
  const uint8_t *aux;  // null when there is none
  uint64_t aux_len;
};

// stage_tensor_byte_sections (lib.rs:75-96): true for a well-formed frame; otherwise the whole
// buffer is the hidden section.
bool stage_tensor_sections(const uint8_t *bytes, uint64_t n, PayloadSections &s);
// encode_stage_tensor_bytes (lib.rs:98-118): bare hidden bytes without aux, else the frame.
uint64_t encoded_stage_tensor_bytes(uint64_t hidden_len, uint64_t aux_len);
void encode_stage_tensor(const uint8_t *hidden, uint64_t hidden_len, const uint8_t *aux, uint64_t aux_len,
                         uint8_t *out);

// Prompt aux section (real_forward.rs:1852-1990): "rsa1" | u32 seq | u32 layers | u32 ple_dim |
// u32 n_hashes | f32 per-layer inputs [seq][layers][ple_dim] | u64 prefix hashes, or the older
// "rpl1" | u32 seq | u32 layers | u32 ple_dim | f32 [seq][layers][ple_dim].
struct PromptAux {
  uint32_t seq = 0, layers = 0, ple_dim = 0;
  const float *ple = nullptr;  // unaligned: read with memcpy
  std::vector<uint64_t> hashes;
};
// decode_prompt_aux; false with `err` set on a malformed section.
bool decode_prompt_aux(const uint8_t *b, uint64_t n, PromptAux &out, std::string &err);
// encode_prompt_aux: empty when there is neither a per-layer input nor a hash.
std::vector<uint8_t> encode_prompt_aux(const float *ple, uint32_t seq, uint32_t layers, uint32_t ple_dim,
                                       const std::vector<uint64_t> &hashes);
// prefix_hashes (real_forward.rs:319-333): 64-bit FNV-1a over each id's little-endian bytes, one
// running hash per prefix.
std::vector<uint64_t> prefix_hashes(const uint32_t *ids, int64_t n);

}  // namespace sfc
