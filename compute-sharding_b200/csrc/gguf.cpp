// gguf.cpp — GGUF shard files on the host side of the stage backend.
//
// Replaces, for the B200 backend, the reference's GGUF tooling in crates/stage-forward-lab:
//   GgufFile::parse_bytes and its queries       gguf.rs:138-365
//   plan_for_splits / build_manifest / bundle   gguf.rs:366-751 (classify_tensor_role :753-786)
//   LoadedRuntimeBundle::load                   lib.rs:3283-3420
//   StageResidencyAdapter + pack writers        lib.rs:3424-3613
// The files written here (manifest bundle, `stage-N-required.pack` + `.index.json`) have the
// reference's layout and JSON field order, so either side can read the other's.  The parser maps
// the file and keeps the mapping, so `sfc_stage_open_gguf` uploads tensors straight from it.
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <charconv>
#include <memory>
#include <set>

#include "capi_common.h"
#include "gguf.h"
#include "json.h"

namespace sfc {

// ------------------------------------------------------------------ bytes
GgufBytes::~GgufBytes() {
  if (map) munmap(map, size_t(size));
}

bool GgufBytes::map_file(const std::string &path, std::string &err) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    err = "Failed to open " + path + ": " + strerror(errno);
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    err = "Failed to stat " + path + ": " + strerror(errno);
    close(fd);
    return false;
  }
  size = uint64_t(st.st_size);
  if (size == 0) {
    close(fd);
    data = nullptr;
    return true;
  }
  void *p = mmap(nullptr, size_t(size), PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    err = "Failed to map " + path + ": " + strerror(errno);
    size = 0;
    return false;
  }
  map = p;
  data = static_cast<const uint8_t *>(p);
  return true;
}

void GgufBytes::own(const void *bytes, uint64_t n) {
  copy.assign(static_cast<const uint8_t *>(bytes), static_cast<const uint8_t *>(bytes) + n);
  data = copy.data();
  size = n;
}

// ------------------------------------------------------------------ reader
namespace {

// Little-endian cursor over the file bytes; every read is bounds-checked (Cursor::read_exact).
struct Cursor {
  const uint8_t *p;
  uint64_t n, pos = 0;
  bool ok = true;
  std::string err;
  bool take(void *dst, uint64_t k) {
    if (!ok) return false;
    if (k > n - pos) {
      ok = false;
      err = "GGUF truncated: needs " + std::to_string(k) + " bytes at offset " + std::to_string(pos) + " of " +
            std::to_string(n);
      return false;
    }
    if (k) memcpy(dst, p + pos, size_t(k));
    pos += k;
    return true;
  }
  template <typename T>
  T get() {
    T v{};
    take(&v, sizeof(T));  // the host is little-endian, like the format
    return v;
  }
  uint64_t count(uint32_t version) { return version == 1 ? uint64_t(get<uint32_t>()) : get<uint64_t>(); }
};

// Well-formed UTF-8 (String::from_utf8): no overlong forms, no surrogates, at most U+10FFFF.
bool utf8_valid(const std::string &s) {
  const auto *b = reinterpret_cast<const unsigned char *>(s.data());
  const size_t n = s.size();
  size_t i = 0;
  while (i < n) {
    const unsigned c = b[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    int len;
    unsigned lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
    } else if (c >= 0xE0 && c <= 0xEF) {
      len = 3;
      if (c == 0xE0) lo = 0xA0;
      if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      len = 4;
      if (c == 0xF0) lo = 0x90;
      if (c == 0xF4) hi = 0x8F;
    } else {
      return false;
    }
    if (i + size_t(len) > n) return false;
    if (b[i + 1] < lo || b[i + 1] > hi) return false;
    for (int k = 2; k < len; ++k)
      if (b[i + size_t(k)] < 0x80 || b[i + size_t(k)] > 0xBF) return false;
    i += size_t(len);
  }
  return true;
}

bool read_string(Cursor &c, uint32_t version, std::string &out) {
  const uint64_t len = c.count(version);
  if (!c.ok) return false;
  if (len > c.n - c.pos) {
    c.ok = false;
    c.err = "GGUF string of " + std::to_string(len) + " bytes runs past the end of the file";
    return false;
  }
  out.assign(reinterpret_cast<const char *>(c.p + c.pos), size_t(len));
  c.pos += len;
  if (!utf8_valid(out)) {
    c.ok = false;
    c.err = "GGUF string at offset " + std::to_string(c.pos - len) + " is not valid UTF-8";
    return false;
  }
  return true;
}

// read_metadata_value (gguf.rs:825-857)
bool read_value(Cursor &c, uint32_t version, uint32_t type, GgufValue &v, int depth) {
  v.type = type;
  switch (type) {
    case 0: v.u = c.get<uint8_t>(); break;
    case 1: v.i = c.get<int8_t>(); break;
    case 2: v.u = c.get<uint16_t>(); break;
    case 3: v.i = c.get<int16_t>(); break;
    case 4: v.u = c.get<uint32_t>(); break;
    case 5: v.i = c.get<int32_t>(); break;
    case 6: v.f = double(c.get<float>()); break;
    case 7: v.u = c.get<uint8_t>() != 0 ? 1 : 0; break;
    case 8: return read_string(c, version, v.s);
    case 9: {
      if (depth > 64) {
        c.ok = false;
        c.err = "GGUF metadata arrays nested too deeply";
        return false;
      }
      v.u = c.get<uint32_t>();  // element type
      const uint64_t count = c.count(version);
      if (!c.ok) return false;
      // every element takes at least one byte: the file bounds the count
      v.arr.reserve(size_t(std::min<uint64_t>(count, c.n - c.pos)));
      for (uint64_t k = 0; k < count && c.ok; ++k) {
        v.arr.emplace_back();
        if (!read_value(c, version, uint32_t(v.u), v.arr.back(), depth + 1)) return false;
      }
      break;
    }
    case 10: v.u = c.get<uint64_t>(); break;
    case 11: v.i = c.get<int64_t>(); break;
    case 12: v.f = c.get<double>(); break;
    default:
      c.ok = false;
      c.err = "Unsupported GGUF metadata type " + std::to_string(type);
      return false;
  }
  return c.ok;
}

uint64_t align_to(uint64_t v, uint64_t a) {  // gguf.rs:788-798
  if (a == 0) return v;
  const uint64_t r = v % a;
  return r == 0 ? v : v + (a - r);
}

}  // namespace

bool parse_block_index(const std::string &name, uint32_t &idx) {
  // "blk." then the text up to the next '.', parsed as u32 (Rust's parse: optional '+', digits)
  if (name.compare(0, 4, "blk.") != 0) return false;
  const size_t start = 4, dot = name.find('.', start);
  const std::string part = name.substr(start, dot == std::string::npos ? std::string::npos : dot - start);
  size_t i = 0;
  if (i < part.size() && part[i] == '+') ++i;
  if (i == part.size()) return false;
  uint64_t v = 0;
  for (; i < part.size(); ++i) {
    if (part[i] < '0' || part[i] > '9') return false;
    v = v * 10 + uint64_t(part[i] - '0');
    if (v > 0xFFFFFFFFull) return false;
  }
  idx = uint32_t(v);
  return true;
}

int classify_tensor_role(const std::string &name, int64_t *layer) {
  uint32_t idx = 0;
  if (layer) *layer = -1;
  if (parse_block_index(name, idx)) {
    if (layer) *layer = int64_t(idx);
    return ROLE_LAYER;
  }
  if (name == "token_embd.weight") return ROLE_PROMPT_INGRESS;
  if (name == "rope_freqs.weight") return ROLE_POSITIONAL;
  if (name == "per_layer_token_embd.weight" || name == "per_layer_model_proj.weight" ||
      name == "per_layer_proj_norm.weight")
    return ROLE_SHARED_AUX;
  if (name.compare(0, 6, "output") == 0) return ROLE_TAIL_ONLY;
  return ROLE_UNKNOWN_GLOBAL;
}

bool GgufFile::parse(std::string &err) {
  Cursor c{bytes.data, bytes.size};
  char magic[4] = {0, 0, 0, 0};
  if (!c.take(magic, 4) || memcmp(magic, "GGUF", 4) != 0) {
    err = c.ok ? "Not a GGUF file" : c.err;
    return false;
  }
  version = c.get<uint32_t>();
  tensor_count = c.count(version);
  const uint64_t meta_count = c.count(version);
  for (uint64_t k = 0; k < meta_count && c.ok; ++k) {
    std::string key;
    if (!read_string(c, version, key)) break;
    const uint32_t vt = c.get<uint32_t>();
    GgufValue v;
    if (!c.ok || !read_value(c, version, vt, v, 0)) break;
    meta[key] = std::move(v);
  }
  // every tensor record takes at least 24 bytes: the file bounds the count
  if (c.ok) tensors.reserve(size_t(std::min<uint64_t>(tensor_count, (c.n - c.pos) / 24 + 1)));
  for (uint64_t k = 0; k < tensor_count && c.ok; ++k) {
    GgufTensorInfo t;
    if (!read_string(c, version, t.name)) break;
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok) break;
    if (uint64_t(nd) * (version == 1 ? 4 : 8) > c.n - c.pos) {
      c.ok = false;
      c.err = "GGUF tensor " + t.name + " declares " + std::to_string(nd) + " dimensions past the end of the file";
      break;
    }
    t.dims.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) t.dims[d] = c.count(version);
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (c.ok) tensors.push_back(std::move(t));
  }
  if (!c.ok) {
    err = c.err;
    return false;
  }
  uint64_t alignment = 32;
  if (const GgufValue *a = get("general.alignment"))
    if (a->type == 4 || a->type == 10) alignment = a->u;
  data_offset = align_to(c.pos, alignment);
  file_size = bytes.size;

  // tensor_byte_len (gguf.rs:331-343): the distance to the next tensor by offset (stable order);
  // the last one runs to the end of the file.  Repeated names take the first in offset order.
  const size_t nt = tensors.size();
  std::vector<size_t> ord(nt);
  for (size_t k = 0; k < nt; ++k) ord[k] = k;
  std::stable_sort(ord.begin(), ord.end(), [&](size_t a2, size_t b2) { return tensors[a2].offset < tensors[b2].offset; });
  std::map<std::string, uint64_t> len_of;
  const uint64_t data_bytes = file_size > data_offset ? file_size - data_offset : 0;
  for (size_t k = 0; k < nt; ++k) {
    const GgufTensorInfo &t = tensors[ord[k]];
    const uint64_t next = k + 1 < nt ? tensors[ord[k + 1]].offset : data_bytes;
    len_of.emplace(t.name, next > t.offset ? next - t.offset : 0);
  }
  byte_len.resize(nt);
  role.resize(nt);
  layer.resize(nt);
  for (size_t k = 0; k < nt; ++k) {
    byte_len[k] = len_of[tensors[k].name];
    role[k] = classify_tensor_role(tensors[k].name, &layer[k]);
  }
  return true;
}

const GgufValue *GgufFile::get(const std::string &key) const {
  auto it = meta.find(key);
  return it == meta.end() ? nullptr : &it->second;
}

bool GgufFile::architecture(std::string &out) const {
  const GgufValue *v = get("general.architecture");
  if (!v || v->type != 8) return false;
  out = v->s;
  return true;
}

std::vector<uint32_t> GgufFile::block_indices() const {
  std::set<uint32_t> s;
  uint32_t idx = 0;
  for (auto &t : tensors)
    if (parse_block_index(t.name, idx)) s.insert(idx);
  return std::vector<uint32_t>(s.begin(), s.end());
}

bool GgufFile::meta_u32(const std::string &key, uint32_t &out) const {
  const GgufValue *v = get(key);
  if (!v) return false;
  switch (v->type) {
    case 4: out = uint32_t(v->u); return true;
    case 10:
      if (v->u > 0xFFFFFFFFull) return false;
      out = uint32_t(v->u);
      return true;
    case 5:
    case 11:
      if (v->i < 0 || v->i > int64_t(0xFFFFFFFFll)) return false;
      out = uint32_t(v->i);
      return true;
    default: return false;
  }
}

int64_t GgufFile::layer_count() const {
  uint32_t v = 0;
  for (const char *k : {"gemma4.block_count", "gemma.block_count", "llama.block_count"})
    if (meta_u32(k, v)) return int64_t(v);
  const std::vector<uint32_t> b = block_indices();
  return b.empty() ? -1 : int64_t(b.back()) + 1;
}

static int64_t first_u32(const GgufFile &f, const char *suffix) {
  uint32_t v = 0;
  for (const char *arch : {"gemma4.", "gemma.", "llama."})
    if (f.meta_u32(std::string(arch) + suffix, v)) return int64_t(v);
  return -1;
}
int64_t GgufFile::hidden_size() const { return first_u32(*this, "embedding_length"); }
int64_t GgufFile::feed_forward_length() const { return first_u32(*this, "feed_forward_length"); }
int64_t GgufFile::attention_head_count() const { return first_u32(*this, "attention.head_count"); }

bool GgufFile::meta_string(const std::string &key, std::string &out) const {
  const GgufValue *v = get(key);
  if (!v) return false;
  out = gguf_value_string(*v);
  return true;
}

int64_t GgufFile::find(const std::string &name) const {
  for (size_t k = 0; k < tensors.size(); ++k)
    if (tensors[k].name == name) return int64_t(k);
  return -1;
}

bool GgufFile::tensor_byte_len(const std::string &name, uint64_t &out) const {
  const int64_t k = find(name);
  if (k < 0) return false;
  out = byte_len[size_t(k)];
  return true;
}

// Rust's `Display` of a float: the shortest digits that read back to the same value, written
// without an exponent ("1", "0.1", "0.0000001", "NaN", "inf").
template <typename F>
static std::string float_display(F x) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x < 0 ? "-inf" : "inf";
  // shortest round-trip digits d.ddd and exponent, then placed in positional form (zeros pad
  // the digits: 3e38f prints as 3 followed by 38 zeros, not the float's exact integer value)
  char buf[64];
  const auto r = std::to_chars(buf, buf + sizeof(buf), x, std::chars_format::scientific);
  std::string sci(buf, r.ptr), out;
  if (!sci.empty() && sci[0] == '-') {
    out = "-";
    sci.erase(0, 1);
  }
  const size_t epos = sci.find('e');
  const int exp10 = atoi(sci.c_str() + epos + 1);
  std::string digits;
  for (size_t k = 0; k < epos; ++k)
    if (sci[k] != '.') digits += sci[k];
  const int n = int(digits.size());
  if (exp10 >= n - 1) {
    out += digits + std::string(size_t(exp10 - (n - 1)), '0');
  } else if (exp10 >= 0) {
    out += digits.substr(0, size_t(exp10 + 1)) + "." + digits.substr(size_t(exp10 + 1));
  } else {
    out += "0." + std::string(size_t(-exp10 - 1), '0') + digits;
  }
  return out;
}

std::string gguf_value_string(const GgufValue &v) {  // metadata_value_to_string, gguf.rs:800-823
  switch (v.type) {
    case 0:
    case 2:
    case 4:
    case 10: return std::to_string(v.u);
    case 1:
    case 3:
    case 5:
    case 11: return std::to_string(v.i);
    case 6: return float_display(float(v.f));
    case 12: return float_display(v.f);
    case 7: return v.u ? "true" : "false";
    case 8: return v.s;
    case 9: {
      std::string s = "[";
      for (size_t k = 0; k < v.arr.size(); ++k) {
        if (k) s += ", ";
        s += gguf_value_string(v.arr[k]);
      }
      return s + "]";
    }
    default: return std::string();
  }
}

bool gguf_even_split(const GgufFile &f, uint32_t stages, std::vector<StageSplitC> &out) {
  out.clear();
  const int64_t total = f.layer_count();
  if (total < 0 || stages == 0 || int64_t(stages) > total) return false;
  const uint32_t t = uint32_t(total), base = t / stages, rem = t % stages;
  uint32_t start = 0;
  for (uint32_t s = 0; s < stages; ++s) {
    const uint32_t end = start + base + (s < rem ? 1 : 0) - 1;
    out.push_back(StageSplitC{s, start, end});
    start = end + 1;
  }
  return true;
}

// ------------------------------------------------------------------ plan, manifest, bundle
namespace {

struct Planned {  // PlannedTensor (gguf.rs:59-65)
  std::string name;
  int role;
  bool assigned;
  uint32_t stage;
  uint64_t byte_len;
};

struct Group {  // TensorGroup (gguf.rs:73-78)
  std::string name;
  std::vector<std::string> names;
  uint64_t total = 0;
};

struct StageMan {  // StageManifest (gguf.rs:80-91)
  uint32_t stage_index, start_layer, end_layer;
  Group prompt_ingress, positional, replicated_aux, owned, tail_only, unknown_global;
};

struct RuntimePlan {  // StageRuntimePlan (gguf.rs:93-99)
  uint32_t stage_index = 0;
  std::string role;
  Group required, optional;
};

struct Slice {  // TensorSlice (gguf.rs:101-108)
  std::string name;
  uint64_t file_offset = 0, byte_len = 0;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
};

std::vector<Planned> plan_for_splits(const GgufFile &f, const std::vector<StageSplitC> &splits) {  // :366-400
  std::vector<Planned> out;
  for (size_t k = 0; k < f.tensors.size(); ++k) {
    Planned p{f.tensors[k].name, f.role[k], false, 0, 0};
    if (p.role == ROLE_LAYER) {
      for (auto &s : splits)
        if (uint64_t(f.layer[k]) >= s.start_layer && uint64_t(f.layer[k]) <= s.end_layer) {
          p.assigned = true;
          p.stage = s.stage_index;
          break;
        }
    } else if (p.role == ROLE_TAIL_ONLY && !splits.empty()) {
      p.assigned = true;
      p.stage = splits.back().stage_index;
    }
    uint64_t bl = 0;
    p.byte_len = f.tensor_byte_len(p.name, bl) ? bl : 0;
    out.push_back(p);
  }
  return out;
}

Group group_of(const std::vector<Planned> &plan, int role, const char *name) {
  Group g;
  g.name = name;
  for (auto &p : plan)
    if (p.role == role) {
      g.names.push_back(p.name);
      g.total += p.byte_len;
    }
  return g;
}

uint64_t bytes_of_names(const std::vector<Planned> &plan, const std::vector<std::string> &names) {
  uint64_t t = 0;
  for (auto &n : names)
    for (auto &p : plan)
      if (p.name == n) {
        t += p.byte_len;
        break;
      }
  return t;
}

// build_manifest (gguf.rs:452-634)
void build_manifest(const std::vector<Planned> &plan, const std::vector<StageSplitC> &splits,
                    std::vector<StageMan> &stages, std::vector<RuntimePlan> &runtime) {
  const Group pi = group_of(plan, ROLE_PROMPT_INGRESS, "prompt_ingress");
  const Group pos = group_of(plan, ROLE_POSITIONAL, "positional");
  const Group aux = group_of(plan, ROLE_SHARED_AUX, "replicated_aux");
  const Group tail = group_of(plan, ROLE_TAIL_ONLY, "tail_only");
  const Group unk = group_of(plan, ROLE_UNKNOWN_GLOBAL, "unknown_global");
  stages.clear();
  for (auto &s : splits) {
    StageMan m{s.stage_index, s.start_layer, s.end_layer, pi, pos, aux, {}, {}, unk};
    m.owned.name = "stage" + std::to_string(uint64_t(s.stage_index) + 1) + "_owned";
    for (auto &p : plan)
      if (p.role == ROLE_LAYER && p.assigned && p.stage == s.stage_index) {
        m.owned.names.push_back(p.name);
        m.owned.total += p.byte_len;
      }
    m.tail_only.name = "tail_only";
    if (uint64_t(s.stage_index) + 1 == splits.size()) m.tail_only = tail;
    stages.push_back(m);
  }
  runtime.clear();
  for (size_t idx = 0; idx < stages.size(); ++idx) {
    const StageMan &st = stages[idx];
    RuntimePlan r;
    r.stage_index = st.stage_index;
    r.role = idx == 0 ? "head" : idx + 1 == stages.size() ? "tail" : "middle";
    auto &req = r.required.names;
    if (idx == 0) req.insert(req.end(), st.prompt_ingress.names.begin(), st.prompt_ingress.names.end());
    req.insert(req.end(), st.positional.names.begin(), st.positional.names.end());
    req.insert(req.end(), st.replicated_aux.names.begin(), st.replicated_aux.names.end());
    req.insert(req.end(), st.owned.names.begin(), st.owned.names.end());
    if (idx + 1 == stages.size()) req.insert(req.end(), st.tail_only.names.begin(), st.tail_only.names.end());
    if (idx != 0) r.optional.names = st.prompt_ingress.names;
    r.required.name = "required_runtime";
    r.optional.name = "optional_runtime";
    r.required.total = bytes_of_names(plan, r.required.names);
    r.optional.total = bytes_of_names(plan, r.optional.names);
    runtime.push_back(r);
  }
}

void put_group(JsonWriter &w, const char *key, const Group &g) {
  w.key(key);
  w.begin_obj();
  w.key("name");
  w.str(g.name);
  w.key("tensor_names");
  w.str_array(g.names);
  w.key("total_bytes");
  w.num(g.total);
  w.end_obj();
}

void put_stage(JsonWriter &w, const StageMan &m) {
  w.begin_obj();
  w.key("stage_index");
  w.num(m.stage_index);
  w.key("start_layer");
  w.num(m.start_layer);
  w.key("end_layer");
  w.num(m.end_layer);
  put_group(w, "prompt_ingress", m.prompt_ingress);
  put_group(w, "positional", m.positional);
  put_group(w, "replicated_aux", m.replicated_aux);
  put_group(w, "owned", m.owned);
  put_group(w, "tail_only", m.tail_only);
  put_group(w, "unknown_global", m.unknown_global);
  w.end_obj();
}

void put_runtime(JsonWriter &w, const RuntimePlan &r) {
  w.begin_obj();
  w.key("stage_index");
  w.num(r.stage_index);
  w.key("role");
  w.str(r.role);
  put_group(w, "required", r.required);
  put_group(w, "optional", r.optional);
  w.end_obj();
}

void put_slice(JsonWriter &w, const Slice &s) {
  w.begin_obj();
  w.key("name");
  w.str(s.name);
  w.key("file_offset");
  w.num(s.file_offset);
  w.key("byte_len");
  w.num(s.byte_len);
  w.key("dimensions");
  w.num_array(s.dims);
  w.key("ggml_type");
  w.num(s.type);
  w.end_obj();
}

void put_opt(JsonWriter &w, const char *key, int64_t v) {
  w.key(key);
  if (v < 0) w.null();
  else w.num(uint64_t(v));
}

std::string join_lines(const std::vector<std::string> &v) {  // names.join("\n") + "\n"
  std::string s;
  for (size_t k = 0; k < v.size(); ++k) {
    if (k) s += '\n';
    s += v[k];
  }
  return s + "\n";
}

bool mkdirs(const std::string &dir, std::string &err) {  // create_dir_all
  std::string cur;
  size_t i = 0;
  while (i <= dir.size()) {
    const size_t j = dir.find('/', i);
    cur = dir.substr(0, j == std::string::npos ? dir.size() : j);
    if (!cur.empty() && mkdir(cur.c_str(), 0777) != 0 && errno != EEXIST) {
      err = "Failed to create " + cur + ": " + strerror(errno);
      return false;
    }
    if (j == std::string::npos) break;
    i = j + 1;
  }
  struct stat st;
  if (stat(dir.c_str(), &st) != 0 || !S_ISDIR(st.st_mode)) {
    err = dir + " is not a directory";
    return false;
  }
  return true;
}

bool put_file(const std::string &path, const std::string &bytes, std::string &err) {
  if (!write_file(path, bytes)) {
    err = "Failed to write " + path;
    return false;
  }
  return true;
}

std::string path_join(const std::string &dir, const std::string &name) {
  if (dir.empty()) return name;
  return dir.back() == '/' ? dir + name : dir + "/" + name;
}

bool slice_of(const GgufFile &f, const std::string &name, Slice &s) {  // tensor_slice, gguf.rs:352-364
  const int64_t k = f.find(name);
  if (k < 0) return false;
  s.name = name;
  s.file_offset = f.data_offset + f.tensors[size_t(k)].offset;
  s.byte_len = f.byte_len[size_t(k)];
  s.dims = f.tensors[size_t(k)].dims;
  s.type = f.tensors[size_t(k)].type;
  return true;
}

}  // namespace

bool gguf_write_bundle(const GgufFile &f, const std::vector<StageSplitC> &splits, const std::string &out_dir,
                       std::string &err) {
  if (!mkdirs(out_dir, err)) return false;
  const std::vector<Planned> plan = plan_for_splits(f, splits);
  std::vector<StageMan> stages;
  std::vector<RuntimePlan> runtime;
  build_manifest(plan, splits, stages, runtime);

  std::string model_name = "unknown", arch = "unknown";
  if (!f.meta_string("general.name", model_name)) model_name = "unknown";
  if (!f.architecture(arch)) arch = "unknown";
  const int64_t layers = f.layer_count();
  JsonWriter w;
  w.begin_obj();
  w.key("model_name");
  w.str(model_name);
  w.key("architecture");
  w.str(arch);
  put_opt(w, "hidden_size", f.hidden_size());
  put_opt(w, "feed_forward_size", f.feed_forward_length());
  put_opt(w, "attention_heads", f.attention_head_count());
  w.key("total_layers");
  w.num(layers < 0 ? 0 : uint64_t(layers));
  w.key("stages");
  w.begin_arr();
  for (auto &m : stages) put_stage(w, m);
  w.end_arr();
  w.key("runtime_plan");
  w.begin_arr();
  for (auto &r : runtime) put_runtime(w, r);
  w.end_arr();
  w.end_obj();
  if (!put_file(path_join(out_dir, "model-shard-manifest.json"), w.out, err)) return false;

  for (auto &m : stages) {
    const std::string n = std::to_string(uint64_t(m.stage_index) + 1);
    JsonWriter ws;
    put_stage(ws, m);
    if (!put_file(path_join(out_dir, "stage-" + n + ".json"), ws.out, err)) return false;
    const std::pair<const char *, const Group *> lists[] = {
        {"-prompt-ingress.txt", &m.prompt_ingress}, {"-positional.txt", &m.positional},
        {"-replicated-aux.txt", &m.replicated_aux}, {"-owned.txt", &m.owned},
        {"-tail-only.txt", &m.tail_only},           {"-unknown-global.txt", &m.unknown_global}};
    for (auto &l : lists)
      if (!put_file(path_join(out_dir, "stage-" + n + l.first), join_lines(l.second->names), err)) return false;
  }
  for (auto &r : runtime) {
    const std::string n = std::to_string(uint64_t(r.stage_index) + 1);
    JsonWriter wr;
    put_runtime(wr, r);
    if (!put_file(path_join(out_dir, "runtime-stage-" + n + ".json"), wr.out, err)) return false;
    if (!put_file(path_join(out_dir, "runtime-stage-" + n + "-required.txt"), join_lines(r.required.names), err) ||
        !put_file(path_join(out_dir, "runtime-stage-" + n + "-optional.txt"), join_lines(r.optional.names), err))
      return false;
    JsonWriter wl;
    wl.begin_obj();
    wl.key("stage_index");
    wl.num(r.stage_index);
    wl.key("role");
    wl.str(r.role);
    for (int which = 0; which < 2; ++which) {
      wl.key(which ? "optional" : "required");
      wl.begin_arr();
      for (auto &name : (which ? r.optional : r.required).names) {
        Slice s;
        if (!slice_of(f, name, s)) {
          err = std::string("Missing tensor slice for ") + (which ? "optional" : "required") + " tensor " + name;
          return false;
        }
        put_slice(wl, s);
      }
      wl.end_arr();
    }
    wl.end_obj();
    if (!put_file(path_join(out_dir, "runtime-stage-" + n + "-slices.json"), wl.out, err)) return false;
  }
  return true;
}

// ------------------------------------------------------------------ bundle load + stage pack
namespace {

bool load_json(const std::string &path, Json &j, std::string &err) {
  std::string text;
  if (!read_file(path, text)) {
    err = "Failed to read " + path;
    return false;
  }
  if (!json_parse(text, j)) {
    err = path + " is not valid JSON";
    return false;
  }
  return true;
}

bool get_u64(const Json *j, uint64_t &v) {
  if (!j || j->kind != Json::Num || j->num < 0 || j->num != floor(j->num)) return false;
  v = uint64_t(j->num);
  return true;
}

bool get_group(const Json *j, Group &g) {
  if (!j || j->kind != Json::Obj) return false;
  const Json *n = j->get("name"), *t = j->get("tensor_names");
  if (!n || n->kind != Json::Str || !t || t->kind != Json::Arr || !get_u64(j->get("total_bytes"), g.total))
    return false;
  g.name = n->str;
  g.names.clear();
  for (auto &e : t->arr) {
    if (e.kind != Json::Str) return false;
    g.names.push_back(e.str);
  }
  return true;
}

bool get_runtime(const Json &j, RuntimePlan &r) {
  uint64_t si = 0;
  const Json *role = j.get("role");
  if (j.kind != Json::Obj || !get_u64(j.get("stage_index"), si) || !role || role->kind != Json::Str) return false;
  r.stage_index = uint32_t(si);
  r.role = role->str;
  return get_group(j.get("required"), r.required) && get_group(j.get("optional"), r.optional);
}

bool same_group(const Group &a, const Group &b) { return a.name == b.name && a.names == b.names && a.total == b.total; }

bool get_slices(const Json *j, std::vector<Slice> &out) {
  if (!j || j->kind != Json::Arr) return false;
  for (auto &e : j->arr) {
    Slice s;
    const Json *n = e.get("name"), *d = e.get("dimensions");
    uint64_t ty = 0;
    if (e.kind != Json::Obj || !n || n->kind != Json::Str || !get_u64(e.get("file_offset"), s.file_offset) ||
        !get_u64(e.get("byte_len"), s.byte_len) || !d || d->kind != Json::Arr || !get_u64(e.get("ggml_type"), ty))
      return false;
    s.name = n->str;
    s.type = uint32_t(ty);
    for (auto &x : d->arr) {
      uint64_t v = 0;
      if (!get_u64(&x, v)) return false;
      s.dims.push_back(v);
    }
    out.push_back(s);
  }
  return true;
}

std::set<std::string> read_tensor_set(const std::string &path, bool &ok) {  // lib.rs:3617-3625
  std::set<std::string> s;
  std::string text;
  ok = read_file(path, text);
  size_t i = 0;
  while (ok && i <= text.size()) {
    size_t j = text.find('\n', i);
    if (j == std::string::npos) j = text.size();
    std::string line = text.substr(i, j - i);
    const size_t a = line.find_first_not_of(" \t\r\f\v");
    const size_t b = line.find_last_not_of(" \t\r\f\v");
    if (a != std::string::npos) s.insert(line.substr(a, b - a + 1));
    i = j + 1;
  }
  return s;
}

std::set<std::string> name_set(const std::vector<std::string> &v) { return std::set<std::string>(v.begin(), v.end()); }
std::set<std::string> slice_names(const std::vector<Slice> &v) {
  std::set<std::string> s;
  for (auto &x : v) s.insert(x.name);
  return s;
}

struct BundleStage {
  uint32_t stage_index = 0, start_layer = 0, end_layer = 0;
  std::string role;
  std::set<std::string> required, optional;
  std::vector<Slice> req_slices, opt_slices;
};

// LoadedRuntimeBundle::load (lib.rs:3283-3403)
bool load_bundle(const std::string &root, std::string &model_name, std::string &arch, std::vector<BundleStage> &out,
                 std::string &err) {
  Json man;
  if (!load_json(path_join(root, "model-shard-manifest.json"), man, err)) return false;
  const Json *mn = man.get("model_name"), *ar = man.get("architecture"), *rp = man.get("runtime_plan");
  if (!mn || mn->kind != Json::Str || !ar || ar->kind != Json::Str || !rp || rp->kind != Json::Arr) {
    err = "model-shard-manifest.json lacks model_name/architecture/runtime_plan";
    return false;
  }
  model_name = mn->str;
  arch = ar->str;
  for (auto &rj : rp->arr) {
    RuntimePlan r;
    if (!get_runtime(rj, r)) {
      err = "malformed runtime_plan entry in model-shard-manifest.json";
      return false;
    }
    const std::string n = std::to_string(uint64_t(r.stage_index) + 1);
    const std::string stage_path = path_join(root, "stage-" + n + ".json");
    const std::string runtime_path = path_join(root, "runtime-stage-" + n + ".json");
    Json sj, fj;
    if (!load_json(stage_path, sj, err) || !load_json(runtime_path, fj, err)) return false;
    uint64_t si = 0, sl = 0, el = 0;
    if (!get_u64(sj.get("stage_index"), si) || !get_u64(sj.get("start_layer"), sl) ||
        !get_u64(sj.get("end_layer"), el)) {
      err = stage_path + " lacks stage_index/start_layer/end_layer";
      return false;
    }
    if (si != r.stage_index) {
      err = "Stage manifest " + stage_path + " does not match runtime stage index " + n;
      return false;
    }
    RuntimePlan fr;
    if (!get_runtime(fj, fr) || fr.stage_index != r.stage_index || fr.role != r.role ||
        !same_group(fr.required, r.required) || !same_group(fr.optional, r.optional)) {
      err = "Runtime plan file " + runtime_path + " does not match top-level manifest for stage " + n;
      return false;
    }
    const std::string req_path = path_join(root, "runtime-stage-" + n + "-required.txt");
    const std::string opt_path = path_join(root, "runtime-stage-" + n + "-optional.txt");
    const std::string slices_path = path_join(root, "runtime-stage-" + n + "-slices.json");
    bool ok1 = false, ok2 = false;
    BundleStage st;
    st.required = read_tensor_set(req_path, ok1);
    st.optional = read_tensor_set(opt_path, ok2);
    if (!ok1 || !ok2) {
      err = "Failed to read " + (ok1 ? opt_path : req_path);
      return false;
    }
    Json lj;
    if (!load_json(slices_path, lj, err)) return false;
    if (!get_slices(lj.get("required"), st.req_slices) || !get_slices(lj.get("optional"), st.opt_slices)) {
      err = slices_path + " is not a slice manifest";
      return false;
    }
    const std::set<std::string> want_req = name_set(r.required.names), want_opt = name_set(r.optional.names);
    if (st.required != want_req) {
      err = "Required runtime tensor list " + req_path + " does not match manifest for stage " + n;
      return false;
    }
    if (st.optional != want_opt) {
      err = "Optional runtime tensor list " + opt_path + " does not match manifest for stage " + n;
      return false;
    }
    if (slice_names(st.req_slices) != want_req || slice_names(st.opt_slices) != want_opt) {
      err = "Slice manifest " + slices_path + " does not match runtime tensor lists for stage " + n;
      return false;
    }
    st.stage_index = r.stage_index;
    st.start_layer = uint32_t(sl);
    st.end_layer = uint32_t(el);
    st.role = r.role;
    out.push_back(std::move(st));
  }
  return true;
}

void put_index_entry(JsonWriter &w, const Slice &s, uint64_t pack_offset) {  // PackedTensorEntry, lib.rs:2907-2915
  w.begin_obj();
  w.key("name");
  w.str(s.name);
  w.key("pack_offset");
  w.num(pack_offset);
  w.key("byte_len");
  w.num(s.byte_len);
  w.key("source_file_offset");
  w.num(s.file_offset);
  w.key("dimensions");
  w.num_array(s.dims);
  w.key("ggml_type");
  w.num(s.type);
  w.end_obj();
}

}  // namespace

namespace {

// StageResidencyAdapter::load (lib.rs:3424-3453): the bundle, checked against itself and the GGUF
// file, and the stage with that index.
struct Adapter {
  std::string model_name, arch;
  std::vector<BundleStage> stages;
  GgufFile f;
  const BundleStage *st = nullptr;
  bool load(const std::string &bundle_dir, const std::string &gguf_path, uint32_t stage_index, std::string &err) {
    if (!load_bundle(bundle_dir, model_name, arch, stages, err)) return false;
    if (!f.bytes.map_file(gguf_path, err) || !f.parse(err)) return false;
    for (auto &s : stages)  // validate_against_gguf (lib.rs:3405-3422)
      for (const auto *set : {&s.required, &s.optional})
        for (auto &name : *set)
          if (f.find(name) < 0) {
            err = "Stage " + std::to_string(uint64_t(s.stage_index) + 1) + " references tensor " + name +
                  " which is not present in GGUF";
            return false;
          }
    for (auto &s : stages)
      if (s.stage_index == stage_index) {
        st = &s;
        break;
      }
    if (!st) {
      err = "Stage " + std::to_string(uint64_t(stage_index) + 1) + " not found in runtime bundle";
      return false;
    }
    return true;
  }
  // read_slice (lib.rs:3606-3613): the slice's bytes inside the mapped file
  const uint8_t *slice_bytes(const Slice &s, const std::string &gguf_path, std::string &err) const {
    if (s.file_offset > f.bytes.size || s.byte_len > f.bytes.size - s.file_offset) {
      err = "Tensor " + s.name + " slice runs past the end of " + gguf_path;
      return nullptr;
    }
    return f.bytes.data + s.file_offset;
  }
};

// sanitize_tensor_filename (lib.rs:3627-3636): ASCII letters, digits, '-' and '_' stay; every other
// character (a whole UTF-8 sequence) becomes one '_'.
std::string sanitize_tensor_filename(const std::string &name) {
  std::string out;
  for (size_t i = 0; i < name.size();) {
    const unsigned char c = static_cast<unsigned char>(name[i]);
    const bool keep = (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '-' ||
                      c == '_';
    out += keep ? char(c) : '_';
    size_t len = 1;
    if (c >= 0xF0) len = 4;
    else if (c >= 0xE0) len = 3;
    else if (c >= 0xC0) len = 2;
    i += len;
  }
  return out;
}

}  // namespace

bool materialize_stage_from_bundle(const std::string &bundle_dir, const std::string &gguf_path, uint32_t stage_index,
                                   const std::string &out_dir, std::vector<std::string> &written, std::string &err) {
  Adapter a;
  if (!a.load(bundle_dir, gguf_path, stage_index, err) || !mkdirs(out_dir, err)) return false;
  for (const Slice &s : a.st->req_slices) {  // materialize_required_tensors (lib.rs:3500-3510)
    const uint8_t *b = a.slice_bytes(s, gguf_path, err);
    if (!b) return false;
    const std::string path = path_join(out_dir, sanitize_tensor_filename(s.name));
    if (!put_file(path, std::string(reinterpret_cast<const char *>(b), size_t(s.byte_len)), err)) return false;
    written.push_back(path);
  }
  return true;
}

bool pack_stage_from_bundle(const std::string &bundle_dir, const std::string &gguf_path, uint32_t stage_index,
                            bool include_optional, const std::string &out_dir, std::string &index_path,
                            std::string &err) {
  Adapter a;
  if (!a.load(bundle_dir, gguf_path, stage_index, err)) return false;
  const BundleStage *st = a.st;
  const std::string &model_name = a.model_name, &arch = a.arch;
  if (!mkdirs(out_dir, err)) return false;
  const std::string n = std::to_string(uint64_t(stage_index) + 1);
  const std::string pack_path = path_join(out_dir, "stage-" + n + "-required.pack");
  index_path = path_join(out_dir, "stage-" + n + "-required.index.json");
  FILE *pf = fopen(pack_path.c_str(), "wb");
  if (!pf) {
    err = "Failed to create " + pack_path + ": " + strerror(errno);
    return false;
  }
  std::vector<const Slice *> slices;
  for (auto &s : st->req_slices) slices.push_back(&s);
  if (include_optional)
    for (auto &s : st->opt_slices) slices.push_back(&s);
  std::vector<uint64_t> offs;
  uint64_t off = 0;
  for (const Slice *s : slices) {
    const uint8_t *b = a.slice_bytes(*s, gguf_path, err);
    if (!b) {
      fclose(pf);
      return false;
    }
    if (s->byte_len && fwrite(b, 1, size_t(s->byte_len), pf) != size_t(s->byte_len)) {
      fclose(pf);
      err = "Failed to write " + pack_path;
      return false;
    }
    offs.push_back(off);
    off += s->byte_len;
  }
  if (fclose(pf) != 0) {
    err = "Failed to write " + pack_path;
    return false;
  }
  // PackedStageIndex (lib.rs:2917-2926)
  JsonWriter w;
  w.begin_obj();
  w.key("model_name");
  w.str(model_name);
  w.key("architecture");
  w.str(arch);
  w.key("stage_index");
  w.num(stage_index);
  w.key("role");
  w.str(st->role);
  w.key("total_bytes");
  w.num(off);
  w.key("tensor_count");
  w.num(slices.size());
  w.key("tensors");
  w.begin_arr();
  for (size_t k = 0; k < slices.size(); ++k) put_index_entry(w, *slices[k], offs[k]);
  w.end_arr();
  w.end_obj();
  return put_file(index_path, w.out, err);
}

}  // namespace sfc

// ------------------------------------------------------------------ C ABI
struct sfc_gguf {
  sfc::GgufFile f;
  std::vector<const std::string *> keys;  // metadata keys in sorted order
  std::string arch;
  bool has_arch = false;
};

using namespace sfc;

static int gguf_finish(std::unique_ptr<sfc_gguf> &g, sfc_gguf **out) {
  std::string err;
  if (!g->f.parse(err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  for (auto &kv : g->f.meta) g->keys.push_back(&kv.first);
  g->has_arch = g->f.architecture(g->arch);
  *out = g.release();
  return SFC_OK;
}

extern "C" {

int sfc_gguf_open(const char *path, sfc_gguf **out) {
  clear_error();
  SFC_REQUIRE(path && out, "null argument");
  auto g = std::make_unique<sfc_gguf>();
  std::string err;
  if (!g->f.bytes.map_file(path, err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  return gguf_finish(g, out);
}

int sfc_gguf_parse(const void *bytes, uint64_t n, sfc_gguf **out) {
  clear_error();
  SFC_REQUIRE(out && (bytes || n == 0), "null argument");
  auto g = std::make_unique<sfc_gguf>();
  g->f.bytes.own(bytes, n);
  return gguf_finish(g, out);
}

int sfc_gguf_close(sfc_gguf *g) {
  delete g;
  return SFC_OK;
}

int sfc_gguf_get_info(const sfc_gguf *g, sfc_gguf_info *info) {
  clear_error();
  SFC_REQUIRE(g && info, "null argument");
  const GgufFile &f = g->f;
  info->version = f.version;
  info->tensor_count = f.tensor_count;
  info->metadata_count = uint64_t(f.meta.size());
  info->file_size_bytes = f.file_size;
  info->tensor_data_offset = f.data_offset;
  info->layer_count = f.layer_count();
  info->hidden_size = f.hidden_size();
  info->feed_forward_length = f.feed_forward_length();
  info->attention_head_count = f.attention_head_count();
  info->architecture = g->has_arch ? g->arch.c_str() : nullptr;
  return SFC_OK;
}

int sfc_gguf_get_tensor(const sfc_gguf *g, uint64_t i, sfc_gguf_tensor *t) {
  clear_error();
  SFC_REQUIRE(g && t, "null argument");
  const GgufFile &f = g->f;
  SFC_REQUIRE(i < f.tensors.size(), "tensor index %llu out of range (%zu tensors)", (unsigned long long)i,
              f.tensors.size());
  const GgufTensorInfo &ti = f.tensors[size_t(i)];
  t->name = ti.name.c_str();
  t->n_dims = uint32_t(ti.dims.size());
  t->dims = ti.dims.data();
  t->ggml_type = ti.type;
  t->offset = ti.offset;
  t->file_offset = f.data_offset + ti.offset;
  t->byte_len = f.byte_len[size_t(i)];
  t->role = f.role[size_t(i)];
  t->layer = f.layer[size_t(i)];
  return SFC_OK;
}

int sfc_gguf_find_tensor(const sfc_gguf *g, const char *name, uint64_t *index) {
  clear_error();
  SFC_REQUIRE(g && name && index, "null argument");
  const int64_t k = g->f.find(name);
  if (k < 0) return SFC_ABSENT;
  *index = uint64_t(k);
  return SFC_OK;
}

int sfc_gguf_metadata_key(const sfc_gguf *g, uint64_t i, const char **key, uint32_t *value_type) {
  clear_error();
  SFC_REQUIRE(g && key, "null argument");
  SFC_REQUIRE(i < g->keys.size(), "metadata index %llu out of range (%zu keys)", (unsigned long long)i,
              g->keys.size());
  *key = g->keys[size_t(i)]->c_str();
  if (value_type) *value_type = g->f.meta.at(*g->keys[size_t(i)]).type;
  return SFC_OK;
}

int sfc_gguf_metadata_string(const sfc_gguf *g, const char *key, char *buf, uint64_t cap, uint64_t *len) {
  clear_error();
  SFC_REQUIRE(g && key && (buf || cap == 0), "null argument");
  std::string s;
  if (!g->f.meta_string(key, s)) return SFC_ABSENT;
  if (len) *len = uint64_t(s.size());
  if (cap > 0) {
    const size_t k = size_t(std::min<uint64_t>(cap - 1, s.size()));
    memcpy(buf, s.data(), k);
    buf[k] = '\0';
  }
  return SFC_OK;
}

int sfc_gguf_metadata_u32(const sfc_gguf *g, const char *key, uint32_t *value) {
  clear_error();
  SFC_REQUIRE(g && key && value, "null argument");
  return g->f.meta_u32(key, *value) ? SFC_OK : SFC_ABSENT;
}

int sfc_gguf_metadata_array(const sfc_gguf *g, const char *key, uint32_t *elem_type, uint64_t *count) {
  clear_error();
  SFC_REQUIRE(g && key && count, "null argument");
  const GgufValue *v = g->f.get(key);
  if (!v || v->type != 9) return SFC_ABSENT;
  if (elem_type) *elem_type = uint32_t(v->u);
  *count = uint64_t(v->arr.size());
  return SFC_OK;
}

int sfc_gguf_metadata_f32_array(const sfc_gguf *g, const char *key, float *out, uint64_t cap, uint64_t *n) {
  clear_error();
  SFC_REQUIRE(g && key && n && (out || cap == 0), "null argument");
  const GgufValue *v = g->f.get(key);
  if (!v || v->type != 9) return SFC_ABSENT;
  *n = uint64_t(v->arr.size());
  for (size_t k = 0; k < v->arr.size() && k < cap; ++k) {  // metadata_f32_array (gguf.rs:262-277)
    const GgufValue &e = v->arr[k];
    switch (e.type) {
      case 6:
      case 12: out[k] = float(e.f); break;
      case 5: out[k] = float(e.i); break;
      case 4: out[k] = float(e.u); break;
      default: out[k] = 0.0f;
    }
  }
  return SFC_OK;
}

int sfc_gguf_metadata_array_string(const sfc_gguf *g, const char *key, uint64_t index, char *buf, uint64_t cap,
                                   uint64_t *len) {
  clear_error();
  SFC_REQUIRE(g && key && (buf || cap == 0), "null argument");
  const GgufValue *v = g->f.get(key);
  if (!v || v->type != 9) return SFC_ABSENT;
  SFC_REQUIRE(index < v->arr.size(), "array %s has %zu elements, index %llu", key, v->arr.size(),
              (unsigned long long)index);
  const std::string s = gguf_value_string(v->arr[size_t(index)]);  // metadata_string_array (gguf.rs:253-260)
  if (len) *len = uint64_t(s.size());
  if (cap > 0) {
    const size_t k = size_t(std::min<uint64_t>(cap - 1, s.size()));
    memcpy(buf, s.data(), k);
    buf[k] = '\0';
  }
  return SFC_OK;
}

int sfc_gguf_block_indices(const sfc_gguf *g, uint32_t *out, uint64_t cap, uint64_t *n) {
  clear_error();
  SFC_REQUIRE(g && n && (out || cap == 0), "null argument");
  const std::vector<uint32_t> b = g->f.block_indices();
  *n = uint64_t(b.size());
  for (size_t k = 0; k < b.size() && k < cap; ++k) out[k] = b[k];
  return SFC_OK;
}

int sfc_gguf_even_split(const sfc_gguf *g, uint32_t stages, sfc_stage_split *out) {
  clear_error();
  SFC_REQUIRE(g && (out || stages == 0), "null argument");
  std::vector<StageSplitC> s;
  if (!gguf_even_split(g->f, stages, s)) {
    set_error("no even split of %lld layers into %u stages", (long long)g->f.layer_count(), stages);
    return SFC_ABSENT;
  }
  for (size_t k = 0; k < s.size(); ++k) out[k] = sfc_stage_split{s[k].stage_index, s[k].start_layer, s[k].end_layer};
  return SFC_OK;
}

int sfc_gguf_write_bundle(const sfc_gguf *g, const sfc_stage_split *splits, uint32_t n_splits, const char *out_dir) {
  clear_error();
  SFC_REQUIRE(g && out_dir && (splits || n_splits == 0), "null argument");
  std::vector<StageSplitC> s;
  for (uint32_t k = 0; k < n_splits; ++k) s.push_back(StageSplitC{splits[k].stage_index, splits[k].start_layer,
                                                                  splits[k].end_layer});
  std::string err;
  if (!gguf_write_bundle(g->f, s, out_dir, err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  return SFC_OK;
}

int sfc_materialize_stage(const char *bundle_dir, const char *gguf_path, uint32_t stage_index, const char *out_dir,
                          uint64_t *n_written) {
  clear_error();
  SFC_REQUIRE(bundle_dir && gguf_path && out_dir, "null argument");
  std::vector<std::string> written;
  std::string err;
  if (!materialize_stage_from_bundle(bundle_dir, gguf_path, stage_index, out_dir, written, err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  if (n_written) *n_written = uint64_t(written.size());
  return SFC_OK;
}

int sfc_pack_stage(const char *bundle_dir, const char *gguf_path, uint32_t stage_index, int include_optional,
                   const char *out_dir, char *index_path, uint64_t cap) {
  clear_error();
  SFC_REQUIRE(bundle_dir && gguf_path && out_dir && (index_path || cap == 0), "null argument");
  std::string idx, err;
  if (!pack_stage_from_bundle(bundle_dir, gguf_path, stage_index, include_optional != 0, out_dir, idx, err)) {
    set_error("%s", err.c_str());
    return SFC_E_IO;
  }
  if (cap > 0) {
    SFC_REQUIRE(idx.size() < cap, "index path needs %zu bytes, buffer holds %llu", idx.size() + 1,
                (unsigned long long)cap);
    memcpy(index_path, idx.c_str(), idx.size() + 1);
  }
  return SFC_OK;
}

}  // extern "C"
