// gguf.cuh -- GGUF model files into the device model (the reference's
// Model::load, src/model.rs:266-420, and Qwen35::new's metadata geometry,
// src/graph.rs:2966-3100).  Host code only.
//
// The file is read whole and parsed with every extent checked: header
// (magic "GGUF", version 2 or 3, tensor and key counts), typed metadata
// (scalars, strings, arrays), the tensor table (name, up to 4 dimensions in
// ggml order, type, offset) and the data section at general.alignment
// (default 32).  A tensor's bytes follow from its type and dimensions; it
// must lie inside the file, aligned, with a unique name.  The Qwen35
// geometry is read from the reference's `qwen35.*` keys, the vocabulary from
// token_embd.weight, and every tensor is bound by its GGUF name: F32
// tensors as vectors, packed kinds as weights.
#pragma once

#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "model.cuh"

struct prism_b200_gguf {
  struct Value {
    uint32_t type = 0;  // GGUF value type
    uint64_t u = 0;     // unsigned integers and booleans
    int64_t i = 0;      // signed integers
    double f = 0.0;     // floats
    std::string s;
    uint32_t atype = 0;
    std::vector<Value> arr;
  };
  struct Tensor {
    std::string name;
    uint32_t ndims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0, bytes = 0, elements = 0;
  };
  std::vector<uint8_t> file;
  uint32_t version = 0;
  std::map<std::string, Value> kv;
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> index;
  uint64_t data_start = 0;
};

namespace prism {

// Bytes per block and elements per block of a GGUF tensor type this library
// binds: F32, F16, and the packed kinds of the projection executor.
inline bool gguf_type_layout(uint32_t type, uint64_t &block_bytes, uint64_t &block_elems) {
  switch (type) {
    case 0: block_bytes = 4; block_elems = 1; return true;    // F32
    case 1: block_bytes = 2; block_elems = 1; return true;    // F16
    case 10: block_bytes = 84; block_elems = 256; return true;
    case 11: block_bytes = 110; block_elems = 256; return true;
    case 12: block_bytes = 144; block_elems = 256; return true;
    case 13: block_bytes = 176; block_elems = 256; return true;
    case 14: block_bytes = 210; block_elems = 256; return true;
    case 34: block_bytes = 54; block_elems = 256; return true;
    case 35: block_bytes = 66; block_elems = 256; return true;
    case 142: block_bytes = 34; block_elems = 128; return true;
    case 143: block_bytes = 28; block_elems = 128; return true;
    default: return false;
  }
}

struct GgufReader {
  const uint8_t *p;
  size_t n, at = 0;
  bool ok = true;
  bool take(void *dst, size_t k) {
    if (!ok || k > n - at) return ok = false;
    memcpy(dst, p + at, k);
    at += k;
    return true;
  }
  template <typename T> T get() {
    T v{};
    take(&v, sizeof(T));
    return v;
  }
  bool str(std::string &s) {
    const uint64_t len = get<uint64_t>();
    if (!ok || len > n - at || len > (1u << 20)) return ok = false;
    s.assign(reinterpret_cast<const char *>(p + at), (size_t)len);
    at += (size_t)len;
    return true;
  }
  bool value(uint32_t type, prism_b200_gguf::Value &v, int depth) {
    v.type = type;
    switch (type) {
      case 0: v.u = get<uint8_t>(); break;
      case 1: v.i = get<int8_t>(); break;
      case 2: v.u = get<uint16_t>(); break;
      case 3: v.i = get<int16_t>(); break;
      case 4: v.u = get<uint32_t>(); break;
      case 5: v.i = get<int32_t>(); break;
      case 6: v.f = get<float>(); break;
      case 7: {
        const uint8_t b = get<uint8_t>();
        if (b > 1) return ok = false;
        v.u = b;
        break;
      }
      case 8: return str(v.s);
      case 9: {
        if (depth > 0) return ok = false;  // no nested arrays
        v.atype = get<uint32_t>();
        const uint64_t count = get<uint64_t>();
        if (!ok || count > (1u << 24) || count > n - at) return ok = false;
        v.arr.resize((size_t)count);
        for (auto &e : v.arr)
          if (!value(v.atype, e, depth + 1)) return false;
        break;
      }
      case 10: v.u = get<uint64_t>(); break;
      case 11: v.i = get<int64_t>(); break;
      case 12: v.f = get<double>(); break;
      default: return ok = false;
    }
    return ok;
  }
};

// IEEE binary16 bits to binary32 (exact), on the host.
inline float gguf_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, ex = (h >> 10) & 31, man = h & 1023;
  uint32_t bits;
  if (ex == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else if (ex != 0) {
    bits = sign | ((ex + 112) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {  // subnormal: normalise
    int e = -1;
    uint32_t m = man;
    do {
      ++e;
      m <<= 1;
    } while (!(m & 1024));
    bits = sign | ((uint32_t)(112 - e) << 23) | ((m & 1023) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// A metadata value as an unsigned integer (any integer type, non-negative).
inline bool gguf_uint(const prism_b200_gguf::Value &v, uint64_t &out) {
  if (v.type == 0 || v.type == 2 || v.type == 4 || v.type == 10) {
    out = v.u;
    return true;
  }
  if ((v.type == 1 || v.type == 3 || v.type == 5 || v.type == 11) && v.i >= 0) {
    out = (uint64_t)v.i;
    return true;
  }
  return false;
}

inline bool gguf_parse(prism_b200_gguf &g, std::string &why) {
  GgufReader r{g.file.data(), g.file.size()};
  char magic[4];
  if (!r.take(magic, 4) || memcmp(magic, "GGUF", 4)) return why = "not a GGUF file", false;
  g.version = r.get<uint32_t>();
  if (g.version != 2 && g.version != 3) return why = "unsupported GGUF version", false;
  const uint64_t ntensors = r.get<uint64_t>(), nkv = r.get<uint64_t>();
  if (!r.ok || ntensors > (1u << 20) || nkv > (1u << 20)) return why = "bad GGUF counts", false;
  for (uint64_t k = 0; k < nkv; ++k) {
    std::string key;
    prism_b200_gguf::Value v;
    if (!r.str(key) || !r.value(r.get<uint32_t>(), v, 0))
      return why = "malformed metadata", false;
    if (!g.kv.emplace(key, std::move(v)).second)
      return why = "duplicate metadata key " + key, false;
  }
  uint64_t alignment = 32;
  auto al = g.kv.find("general.alignment");
  if (al != g.kv.end() &&
      (!gguf_uint(al->second, alignment) || alignment == 0 || (alignment & (alignment - 1))))
    return why = "bad general.alignment", false;
  g.tensors.resize((size_t)ntensors);
  for (auto &t : g.tensors) {
    if (!r.str(t.name)) return why = "malformed tensor table", false;
    t.ndims = r.get<uint32_t>();
    if (!r.ok || t.ndims == 0 || t.ndims > 4)
      return why = "bad tensor rank for " + t.name, false;
    for (uint32_t d = 0; d < t.ndims; ++d) t.dims[d] = r.get<uint64_t>();
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (!r.ok) return why = "malformed tensor table", false;
    uint64_t bb, be;
    if (!gguf_type_layout(t.type, bb, be))
      return why = "unsupported tensor type " + std::to_string(t.type) + " for " + t.name, false;
    uint64_t elems = 1;
    for (uint32_t d = 0; d < t.ndims; ++d) {
      if (t.dims[d] == 0 || t.dims[d] > (1ull << 32) || elems > (1ull << 40) / t.dims[d])
        return why = "bad dimensions for " + t.name, false;
      elems *= t.dims[d];
    }
    if (t.dims[0] % be) return why = "partial block in " + t.name, false;
    t.elements = elems;
    t.bytes = elems / be * bb;
    if (t.offset % alignment) return why = "misaligned tensor " + t.name, false;
    if (!g.index.emplace(t.name, &t - g.tensors.data()).second)
      return why = "duplicate tensor " + t.name, false;
  }
  g.data_start = (r.at + alignment - 1) / alignment * alignment;
  for (const auto &t : g.tensors)
    if (g.data_start > g.file.size() || t.offset > g.file.size() - g.data_start ||
        t.bytes > g.file.size() - g.data_start - t.offset)
      return why = "tensor " + t.name + " lies outside the file", false;
  return true;
}

inline int gguf_config(const prism_b200_gguf &g, uint32_t context, uint32_t kv_policy,
                       prism_b200_qwen35_config &c, std::string &why) {
  auto u32 = [&](const char *key, uint32_t &out) {
    auto it = g.kv.find(key);
    uint64_t v;
    if (it == g.kv.end() || !gguf_uint(it->second, v) || v > 0xffffffffull) {
      why = std::string("missing or invalid ") + key;
      return false;
    }
    out = (uint32_t)v;
    return true;
  };
  auto f32 = [&](const char *key, float &out) {
    auto it = g.kv.find(key);
    if (it == g.kv.end() || (it->second.type != 6 && it->second.type != 12)) {
      why = std::string("missing or invalid ") + key;
      return false;
    }
    out = (float)it->second.f;
    return true;
  };
  memset(&c, 0, sizeof(c));
  uint32_t value_length, inner;
  if (!u32("qwen35.embedding_length", c.hidden) || !u32("qwen35.block_count", c.layers) ||
      !u32("qwen35.attention.head_count", c.heads) ||
      !u32("qwen35.attention.head_count_kv", c.kv_heads) ||
      !u32("qwen35.attention.key_length", c.head_dim) ||
      !u32("qwen35.attention.value_length", value_length) ||
      !u32("qwen35.rope.dimension_count", c.rope_dim) ||
      !f32("qwen35.rope.freq_base", c.rope_base) ||
      !f32("qwen35.attention.layer_norm_rms_epsilon", c.eps) ||
      !u32("qwen35.feed_forward_length", c.ffn) || !u32("qwen35.ssm.state_size", c.ssm_state) ||
      !u32("qwen35.ssm.group_count", c.ssm_groups) ||
      !u32("qwen35.ssm.time_step_rank", c.ssm_values) ||
      !u32("qwen35.ssm.conv_kernel", c.conv_kernel) || !u32("qwen35.ssm.inner_size", inner))
    return PRISM_B200_E_INVALID;
  if (value_length != c.head_dim || (uint64_t)inner != (uint64_t)c.ssm_state * c.ssm_values) {
    why = "value length or SSM inner size disagrees with the geometry";
    return PRISM_B200_E_INVALID;
  }
  auto sec = g.kv.find("qwen35.rope.dimension_sections");
  if (sec == g.kv.end() || sec->second.type != 9 || sec->second.arr.size() != 4) {
    why = "missing or invalid qwen35.rope.dimension_sections";
    return PRISM_B200_E_INVALID;
  }
  for (int k = 0; k < 4; ++k) {
    uint64_t v;
    if (!gguf_uint(sec->second.arr[k], v) || v > 0xffffffffull) {
      why = "invalid RoPE section";
      return PRISM_B200_E_INVALID;
    }
    c.rope_sections[k] = (uint32_t)v;
  }
  c.full_interval = 4;  // the reference's default
  if (g.kv.count("qwen35.full_attention_interval") &&
      !u32("qwen35.full_attention_interval", c.full_interval))
    return PRISM_B200_E_INVALID;
  if (c.full_interval == 0) {
    why = "full attention interval must be positive";
    return PRISM_B200_E_INVALID;
  }
  auto rec = g.kv.find("qwen35.attention.recurrent_layers");
  if (rec != g.kv.end()) {  // must agree with the interval this model derives
    if (rec->second.type != 9 || rec->second.arr.size() != c.layers) {
      why = "recurrent layer flags must cover all blocks";
      return PRISM_B200_E_INVALID;
    }
    for (uint32_t l = 0; l < c.layers; ++l) {
      const auto &f = rec->second.arr[l];
      if (f.type != 7 || (f.u != 0) != (((l + 1) % c.full_interval) != 0)) {
        why = "recurrent layer flags differ from the full attention interval";
        return PRISM_B200_E_UNSUPPORTED;
      }
    }
  }
  auto emb = g.index.find("token_embd.weight");
  if (emb == g.index.end()) {
    why = "missing token_embd.weight";
    return PRISM_B200_E_INVALID;
  }
  const auto &e = g.tensors[emb->second];
  if (e.ndims != 2 || e.dims[0] != c.hidden) {
    why = "token_embd.weight does not match the embedding length";
    return PRISM_B200_E_INVALID;
  }
  if (g.index.count("output.weight")) {
    why = "an untied output.weight is not served (the head is tied to token_embd.weight)";
    return PRISM_B200_E_UNSUPPORTED;
  }
  c.vocab = (uint32_t)e.dims[1];
  c.weight_kind = e.type;
  c.context = context;
  c.kv_policy = kv_policy;
  return PRISM_B200_OK;
}

}  // namespace prism

extern "C" {

int prism_b200_gguf_open(const char *path, prism_b200_gguf **out, char *err, size_t err_len) {
  auto fail = [&](int code, const std::string &why) {
    if (err && err_len) snprintf(err, err_len, "%s", why.c_str());
    return code;
  };
  if (!path || !out) return fail(PRISM_B200_E_INVALID, "null argument");
  *out = nullptr;
  FILE *f = fopen(path, "rb");
  if (!f) return fail(PRISM_B200_E_INVALID, std::string("cannot open ") + path);
  auto *g = new prism_b200_gguf();
  bool read_ok = fseek(f, 0, SEEK_END) == 0;
  const long size = read_ok ? ftell(f) : -1;
  read_ok = read_ok && size >= 0 && fseek(f, 0, SEEK_SET) == 0;
  if (read_ok) {
    g->file.resize((size_t)size);
    read_ok = size == 0 || fread(g->file.data(), 1, (size_t)size, f) == (size_t)size;
  }
  fclose(f);
  std::string why;
  if (!read_ok) why = "read error";
  if (!read_ok || !prism::gguf_parse(*g, why)) {
    delete g;
    return fail(PRISM_B200_E_INVALID, why);
  }
  *out = g;
  return PRISM_B200_OK;
}

void prism_b200_gguf_close(prism_b200_gguf *g) { delete g; }

int64_t prism_b200_gguf_tensor_count(const prism_b200_gguf *g) {
  return g ? (int64_t)g->tensors.size() : -1;
}

int prism_b200_gguf_tensor(const prism_b200_gguf *g, size_t index, const char **name,
                           uint32_t *type, uint64_t dims[4], uint32_t *ndims, const void **data,
                           uint64_t *bytes) {
  if (!g || index >= g->tensors.size()) return PRISM_B200_E_INVALID;
  const auto &t = g->tensors[index];
  if (name) *name = t.name.c_str();
  if (type) *type = t.type;
  if (dims)
    for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
  if (ndims) *ndims = t.ndims;
  if (data) *data = g->file.data() + g->data_start + t.offset;
  if (bytes) *bytes = t.bytes;
  return PRISM_B200_OK;
}

int prism_b200_gguf_qwen35_config(const prism_b200_gguf *g, uint32_t context, uint32_t kv_policy,
                                  prism_b200_qwen35_config *cfg, char *err, size_t err_len) {
  if (!g || !cfg) return PRISM_B200_E_INVALID;
  std::string why;
  const int st = prism::gguf_config(*g, context, kv_policy, *cfg, why);
  if (st && err && err_len) snprintf(err, err_len, "%s", why.c_str());
  return st;
}

int prism_b200_model_load_gguf(prism_b200_executor *ex, const prism_b200_gguf *g,
                               uint32_t context, uint32_t kv_policy, prism_b200_model **out) {
  if (!g || !out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  int st = check_open(ex);
  if (st) return st;
  prism_b200_qwen35_config c;
  std::string why;
  if ((st = prism::gguf_config(*g, context, kv_policy, c, why)))
    return ex->fail(st, "GGUF: %s", why.c_str());
  prism_b200_model *m = nullptr;
  if ((st = prism_b200_model_create(ex, &c, &m))) return st;
  for (const auto &t : g->tensors) {
    const uint8_t *data = g->file.data() + g->data_start + t.offset;
    if (t.type == 0 || t.type == 1) {
      // vectors: F32 copied out (the data is aligned only to
      // general.alignment), F16 widened
      std::vector<float> v((size_t)t.elements);
      if (t.type == 0) {
        memcpy(v.data(), data, (size_t)t.bytes);
      } else {
        for (size_t k = 0; k < v.size(); ++k)
          v[k] = prism::gguf_half_to_float((uint16_t)(data[2 * k] | (data[2 * k + 1] << 8)));
      }
      st = prism_b200_model_set_vector(m, t.name.c_str(), v.data(), v.size());
    } else {
      prism_b200_tensor pt{t.type, t.dims[0], t.elements / t.dims[0], data};
      st = prism_b200_model_set_tensor(m, t.name.c_str(), &pt);
    }
    if (st) {
      prism_b200_model_destroy(m);
      return st;
    }
  }
  if ((st = prism_b200_model_finalize(m))) {
    prism_b200_model_destroy(m);
    return st;
  }
  *out = m;
  return PRISM_B200_OK;
}

}  // extern "C"
