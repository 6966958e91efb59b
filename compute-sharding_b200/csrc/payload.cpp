// payload.cpp — the byte layout of a stage hand-off (StageTensor::bytes) at the C ABI.
//
// A hidden-state payload is f32 little-endian rows [T][hidden], either bare or framed as
// "stb1" | u32 hidden_len | u32 aux_len | hidden bytes | aux bytes
// (stage_tensor_byte_sections / encode_stage_tensor_bytes, crates/stage-forward-lab/src/lib.rs:36-118;
// decode_hidden_states, real_forward.rs:1818-1850).  The aux section ("rsa1": per-layer embedding
// inputs and prompt prefix hashes, real_forward.rs:1852-1950) is carried through a stage unchanged.
#include <string.h>

#include <algorithm>

#include "capi_common.h"
#include "payload.h"

namespace sfc {

static uint32_t rd_u32(const uint8_t *p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

bool stage_tensor_sections(const uint8_t *b, uint64_t n, PayloadSections &s) {
  s.hidden = b;
  s.hidden_len = n;
  s.aux = nullptr;
  s.aux_len = 0;
  if (n < 12 || memcmp(b, "stb1", 4) != 0) return false;
  const uint64_t hl = rd_u32(b + 4), al = rd_u32(b + 8);
  if (12 + hl + al != n) return false;  // not a frame: the bytes are bare hidden rows
  s.hidden = b + 12;
  s.hidden_len = hl;
  s.aux = al ? b + 12 + hl : nullptr;
  s.aux_len = al;
  return true;
}

uint64_t encoded_stage_tensor_bytes(uint64_t hidden_len, uint64_t aux_len) {
  return aux_len ? 12 + hidden_len + aux_len : hidden_len;
}

void encode_stage_tensor(const uint8_t *hidden, uint64_t hidden_len, const uint8_t *aux, uint64_t aux_len,
                         uint8_t *out) {
  if (!aux_len) {
    if (hidden_len) memmove(out, hidden, size_t(hidden_len));
    return;
  }
  // lengths saturate at u32::MAX, as the reference's try_from(..).unwrap_or(u32::MAX)
  const uint32_t hl = uint32_t(std::min<uint64_t>(hidden_len, 0xFFFFFFFFull));
  const uint32_t al = uint32_t(std::min<uint64_t>(aux_len, 0xFFFFFFFFull));
  memmove(out + 12, hidden, size_t(hidden_len));  // hidden may already sit in `out`
  memcpy(out + 12 + hidden_len, aux, size_t(aux_len));
  memcpy(out, "stb1", 4);
  memcpy(out + 4, &hl, 4);
  memcpy(out + 8, &al, 4);
}

bool decode_prompt_aux(const uint8_t *b, uint64_t n, PromptAux &out, std::string &err) {
  auto u32 = [&](uint64_t off) {
    uint32_t v;
    memcpy(&v, b + off, 4);
    return v;
  };
  out = PromptAux();
  if (n >= 20 && memcmp(b, "rsa1", 4) == 0) {
    out.seq = u32(4);
    out.layers = u32(8);
    out.ple_dim = u32(12);
    const uint32_t nh = u32(16);
    const uint64_t vals = uint64_t(out.seq) * out.layers * out.ple_dim;
    const uint64_t want = 20 + vals * 4 + uint64_t(nh) * 8;
    if (n != want) {
      err = "Invalid prompt-aux byte length " + std::to_string(n) + " (expected " + std::to_string(want) + ")";
      return false;
    }
    out.ple = vals ? reinterpret_cast<const float *>(b + 20) : nullptr;
    out.hashes.resize(nh);
    if (nh) memcpy(out.hashes.data(), b + 20 + vals * 4, size_t(nh) * 8);
    return true;
  }
  if (n < 16 || memcmp(b, "rpl1", 4) != 0) {
    err = "Invalid prompt-aux payload";
    return false;
  }
  out.seq = u32(4);
  out.layers = u32(8);
  out.ple_dim = u32(12);
  const uint64_t vals = uint64_t(out.seq) * out.layers * out.ple_dim;
  if (n != 16 + vals * 4) {
    err = "Invalid prompt-aux byte length " + std::to_string(n) + " (expected " + std::to_string(16 + vals * 4) + ")";
    return false;
  }
  out.ple = vals ? reinterpret_cast<const float *>(b + 16) : nullptr;
  return true;
}

std::vector<uint8_t> encode_prompt_aux(const float *ple, uint32_t seq, uint32_t layers, uint32_t ple_dim,
                                       const std::vector<uint64_t> &hashes) {
  const uint64_t vals = ple ? uint64_t(seq) * layers * ple_dim : 0;
  if (vals == 0 && hashes.empty()) return {};
  if (!ple) seq = layers = 0;
  std::vector<uint8_t> out(20 + vals * 4 + hashes.size() * 8);
  const uint32_t nh = uint32_t(hashes.size());
  memcpy(out.data(), "rsa1", 4);
  memcpy(out.data() + 4, &seq, 4);
  memcpy(out.data() + 8, &layers, 4);
  memcpy(out.data() + 12, &ple_dim, 4);
  memcpy(out.data() + 16, &nh, 4);
  if (vals) memcpy(out.data() + 20, ple, size_t(vals) * 4);
  if (nh) memcpy(out.data() + 20 + vals * 4, hashes.data(), size_t(nh) * 8);
  return out;
}

std::vector<uint64_t> prefix_hashes(const uint32_t *ids, int64_t n) {
  std::vector<uint64_t> out(size_t(n > 0 ? n : 0));
  uint64_t h = 0xCBF29CE484222325ull;
  for (int64_t i = 0; i < n; ++i) {
    for (int k = 0; k < 4; ++k) h = (h ^ ((ids[i] >> (8 * k)) & 0xFF)) * 0x100000001B3ull;
    out[size_t(i)] = h;
  }
  return out;
}

}  // namespace sfc

using namespace sfc;

extern "C" {

int sfc_stage_tensor_sections(const void *bytes, uint64_t n, uint64_t *hidden_offset, uint64_t *hidden_len,
                              uint64_t *aux_offset, uint64_t *aux_len) {
  clear_error();
  SFC_REQUIRE((bytes || n == 0) && hidden_offset && hidden_len && aux_offset && aux_len, "null argument");
  PayloadSections s;
  const uint8_t *b = static_cast<const uint8_t *>(bytes);
  const bool framed = stage_tensor_sections(b, n, s);
  *hidden_offset = uint64_t(s.hidden - b);
  *hidden_len = s.hidden_len;
  *aux_offset = s.aux ? uint64_t(s.aux - b) : 0;
  *aux_len = s.aux_len;
  return framed ? SFC_OK : SFC_ABSENT;
}

int sfc_encode_stage_tensor_bytes(const void *hidden, uint64_t hidden_len, const void *aux, uint64_t aux_len,
                                  void *out, uint64_t cap, uint64_t *out_len) {
  clear_error();
  SFC_REQUIRE(out_len && (hidden || hidden_len == 0) && (aux || aux_len == 0), "null argument");
  const uint64_t need = encoded_stage_tensor_bytes(hidden_len, aux_len);
  *out_len = need;
  if (!out) return SFC_OK;  // size query
  SFC_REQUIRE(cap >= need, "output holds %llu bytes, the payload needs %llu", (unsigned long long)cap,
              (unsigned long long)need);
  encode_stage_tensor(static_cast<const uint8_t *>(hidden), hidden_len, static_cast<const uint8_t *>(aux), aux_len,
                      static_cast<uint8_t *>(out));
  return SFC_OK;
}

}  // extern "C"
