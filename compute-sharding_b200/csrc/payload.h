// payload.h — stage hand-off byte layout (bare or "stb1"-framed hidden rows plus an aux section).
#pragma once

#include <stdint.h>

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

}  // namespace sfc
