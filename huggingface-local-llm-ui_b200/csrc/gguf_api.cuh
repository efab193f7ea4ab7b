// gguf_api.cuh -- C ABI of the GGUF parser and loader (b2q_gguf_*,
// b2q_model_load_gguf), included by b2q_api.cu after model_api.cuh.
#pragma once

#include <cerrno>
#include <climits>

#include "gguf.cuh"

struct b2q_gguf : gguf::File {
  std::vector<std::string> keys;  // metadata keys in file order (first occurrence)
};

namespace {

b2q_status gguf_missing(const char* what, const std::string& key) {
  return set_error(B2Q_EINVAL, "missing %s metadata '%s' in GGUF", what, key.c_str());
}

b2q_status gguf_int(const b2q_gguf* g, const std::string& key, int* out) {
  uint64_t v;
  if (!g->get_usize(key, &v)) return gguf_missing("integer", key);
  if (v == 0 || v > (uint64_t)INT_MAX) return set_error(B2Q_EINVAL, "GGUF metadata '%s' = %llu is out of range",
                                                       key.c_str(), (unsigned long long)v);
  *out = (int)v;
  return B2Q_OK;
}

// Rows 0.. of `t` that this rank supplies, and the tensor handed to
// set_tensor_impl: matrices are cut to the rank's shard straight from the
// mapping; 1-D F16/BF16 tensors (norms, biases) are widened to F32 on the
// host, as tensor_f32_1d dequantises them (src/inference.rs:494-500).
b2q_status load_tensor(b2q_model* M, const b2q_gguf* g, const gguf::Tensor& t, const char* as_name) {
  const uint8_t* src = g->data + t.abs_offset;
  if (t.n_dims < 1) return set_error(B2Q_EINVAL, "tensor %s: no dims", t.name.c_str());
  uint64_t n = 1;  // outer rows (the parser has checked that all dims multiply within 64 bits)
  for (int j = 0; j + 1 < t.n_dims; ++j)
    if (__builtin_mul_overflow(n, (uint64_t)t.dims[j], &n))
      return set_error(B2Q_EINVAL, "tensor %s: dims overflow", t.name.c_str());
  if (t.n_dims == 1 || n == 1) {
    const int64_t k = t.dims[t.n_dims - 1];
    if ((t.ggml_type == kF16 || t.ggml_type == kBF16) && (uint64_t)k * 2 > t.byte_len)
      return set_error(B2Q_EINVAL, "tensor %s: %lld elements in %llu bytes", t.name.c_str(), (long long)k,
                       (unsigned long long)t.byte_len);
    if (t.ggml_type == kF32)
      return set_tensor_impl(M, as_name, kF32, t.dims, t.n_dims, 0, 1, src, (size_t)t.byte_len);
    if (t.ggml_type != kF16 && t.ggml_type != kBF16)
      return set_error(B2Q_EUNSUP, "tensor %s: 1-D tensors of GGML type %d are not supported", t.name.c_str(),
                       t.ggml_type);
    std::vector<float> f((size_t)k);
    for (int64_t i = 0; i < k; ++i) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      if (t.ggml_type == kF16) {
        f[(size_t)i] = gguf::f16_to_f32(h);
      } else {
        const uint32_t b = (uint32_t)h << 16;
        memcpy(&f[(size_t)i], &b, 4);
      }
    }
    return set_tensor_impl(M, as_name, kF32, t.dims, t.n_dims, 0, 1, f.data(), f.size() * 4);
  }
  const int64_t rows = t.dims[0];
  if (rows <= 0 || t.byte_len % (uint64_t)rows)
    return set_error(B2Q_EINVAL, "tensor %s: %llu bytes do not split into %lld rows", t.name.c_str(),
                     (unsigned long long)t.byte_len, (long long)rows);
  const uint64_t row_bytes = t.byte_len / (uint64_t)rows;
  int layer = -1;
  const std::string role = role_of(as_name, &layer);
  int64_t sb = 0, se = rows;
  if (role != "token_embd") shard_range(M, role, rows, &sb, &se);
  return set_tensor_impl(M, as_name, t.ggml_type, t.dims, t.n_dims, sb, se, src + sb * row_bytes,
                         (size_t)((se - sb) * row_bytes));
}

}  // namespace

extern "C" {

b2q_status b2q_gguf_open(const char* path, b2q_gguf** out) {
  if (!path || !out) return set_error(B2Q_EINVAL, "b2q_gguf_open: NULL argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return set_error(B2Q_EINVAL, "cannot open GGUF file %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int e = errno;
    close(fd);
    return set_error(B2Q_EINVAL, "cannot stat GGUF file %s: %s", path, strerror(e));
  }
  if (st.st_size < 16) {
    close(fd);
    return set_error(B2Q_EINVAL, "%s: not a GGUF file (no 'GGUF' header)", path);
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  const int e = errno;
  close(fd);
  if (p == MAP_FAILED) return set_error(B2Q_EINVAL, "cannot map GGUF file %s: %s", path, strerror(e));
  b2q_gguf* g = new (std::nothrow) b2q_gguf;
  if (!g) {
    munmap(p, (size_t)st.st_size);
    return set_error(B2Q_ENOMEM, "b2q_gguf_open: out of host memory");
  }
  g->data = static_cast<const uint8_t*>(p);
  g->size = (size_t)st.st_size;
  const std::string err = gguf::parse(g, &g->keys);
  if (!err.empty()) {
    delete g;
    return set_error(B2Q_EINVAL, "%s: %s", path, err.c_str());
  }
  *out = g;
  return B2Q_OK;
}

b2q_status b2q_gguf_close(b2q_gguf* g) {
  delete g;
  return B2Q_OK;
}

int b2q_gguf_version(const b2q_gguf* g) { return g ? (int)g->version : -1; }

int64_t b2q_gguf_n_tensors(const b2q_gguf* g) { return g ? (int64_t)g->tensors.size() : -1; }

int64_t b2q_gguf_n_kv(const b2q_gguf* g) { return g ? (int64_t)g->keys.size() : -1; }

b2q_status b2q_gguf_kv_key(const b2q_gguf* g, int64_t i, const char** key, int* value_type) {
  if (!g || !key) return set_error(B2Q_EINVAL, "b2q_gguf_kv_key: NULL argument");
  if (i < 0 || i >= (int64_t)g->keys.size()) return set_error(B2Q_EINVAL, "b2q_gguf_kv_key: index %lld out of range", (long long)i);
  *key = g->keys[(size_t)i].c_str();
  if (value_type) *value_type = (int)g->get(g->keys[(size_t)i])->type;
  return B2Q_OK;
}

b2q_status b2q_gguf_tensor_info(const b2q_gguf* g, int64_t i, const char** name, int* ggml_type, int* n_dims,
                                int64_t* dims, uint64_t* abs_offset, uint64_t* byte_len) {
  if (!g) return set_error(B2Q_EINVAL, "b2q_gguf_tensor_info: NULL file");
  if (i < 0 || i >= (int64_t)g->tensors.size())
    return set_error(B2Q_EINVAL, "b2q_gguf_tensor_info: index %lld out of range", (long long)i);
  const gguf::Tensor& t = g->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = t.ggml_type;
  if (n_dims) *n_dims = t.n_dims;
  if (dims)
    for (int j = 0; j < gguf::kMaxDims; ++j) dims[j] = j < t.n_dims ? t.dims[j] : 0;
  if (abs_offset) *abs_offset = t.abs_offset;
  if (byte_len) *byte_len = t.byte_len;
  return B2Q_OK;
}

b2q_status b2q_gguf_find_tensor(const b2q_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return set_error(B2Q_EINVAL, "b2q_gguf_find_tensor: NULL argument");
  auto it = g->index.find(name);
  if (it == g->index.end()) return set_error(B2Q_EINVAL, "tensor '%s' not found in GGUF", name);
  *index = (int64_t)it->second;
  return B2Q_OK;
}

const void* b2q_gguf_tensor_data(const b2q_gguf* g, int64_t i) {
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return nullptr;
  return g->data + g->tensors[(size_t)i].abs_offset;
}

b2q_status b2q_gguf_get_usize(const b2q_gguf* g, const char* key, uint64_t* out) {
  if (!g || !key || !out) return set_error(B2Q_EINVAL, "b2q_gguf_get_usize: NULL argument");
  return g->get_usize(key, out) ? B2Q_OK : gguf_missing("integer", key);
}

b2q_status b2q_gguf_get_f32(const b2q_gguf* g, const char* key, float* out) {
  if (!g || !key || !out) return set_error(B2Q_EINVAL, "b2q_gguf_get_f32: NULL argument");
  return g->get_f32(key, out) ? B2Q_OK : gguf_missing("float", key);
}

b2q_status b2q_gguf_get_str(const b2q_gguf* g, const char* key, const char** s, size_t* len) {
  if (!g || !key || !s || !len) return set_error(B2Q_EINVAL, "b2q_gguf_get_str: NULL argument");
  const gguf::Value* v = g->get(key);
  if (!v || v->type != gguf::kString) return gguf_missing("string", key);
  *s = reinterpret_cast<const char*>(g->data + v->off);
  *len = (size_t)v->len;
  return B2Q_OK;
}

b2q_status b2q_gguf_llama_config(const b2q_gguf* g, const char* arch, b2q_model_config* cfg) {
  if (!g || !cfg) return set_error(B2Q_EINVAL, "b2q_gguf_llama_config: NULL argument");
  const std::string a = arch ? arch : "llama";
  const std::string p = g->get(a + ".block_count") ? a : std::string("llama");
  b2q_model_config c = *cfg;
  b2q_status s;
  if ((s = gguf_int(g, p + ".block_count", &c.n_layers)) != B2Q_OK) return s;
  if ((s = gguf_int(g, p + ".embedding_length", &c.n_embd)) != B2Q_OK) return s;
  if ((s = gguf_int(g, p + ".attention.head_count", &c.n_heads)) != B2Q_OK) return s;
  uint64_t v;
  c.n_kv_heads = g->get_usize(p + ".attention.head_count_kv", &v) ? (int)v : c.n_heads;
  c.head_dim = g->get_usize(p + ".attention.key_length", &v) ? (int)v : c.n_embd / c.n_heads;
  if (!g->get_f32(p + ".attention.layer_norm_rms_epsilon", &c.rms_eps)) c.rms_eps = 1e-5f;
  if (!g->get_f32(p + ".rope.freq_base", &c.rope_theta)) c.rope_theta = 10000.0f;
  const gguf::Tensor* tok = g->tensor("token_embd.weight");
  const gguf::Tensor* gate = g->tensor("blk.0.ffn_gate.weight");
  if (!tok || tok->n_dims < 2) return set_error(B2Q_EINVAL, "tensor 'token_embd.weight' not found in GGUF");
  if (!gate || gate->n_dims < 2) return set_error(B2Q_EINVAL, "tensor 'blk.0.ffn_gate.weight' not found in GGUF");
  if (tok->dims[0] > INT_MAX || gate->dims[0] > INT_MAX || c.n_kv_heads <= 0 || c.head_dim <= 0)
    return set_error(B2Q_EINVAL, "GGUF hyperparameters out of range");
  c.n_vocab = (int)tok->dims[0];
  c.n_ff = (int)gate->dims[0];
  *cfg = c;
  return B2Q_OK;
}

b2q_status b2q_model_load_gguf(b2q_model* M, const b2q_gguf* g) {
  if (!M || !g) return set_error(B2Q_EINVAL, "b2q_model_load_gguf: NULL argument");
  auto need = [&](const std::string& name, bool optional) -> b2q_status {
    const gguf::Tensor* t = g->tensor(name);
    if (!t) return optional ? B2Q_OK : set_error(B2Q_EINVAL, "tensor '%s' not found in GGUF", name.c_str());
    return load_tensor(M, g, *t, name.c_str());
  };
  b2q_status s;
  // output before token_embd: a present output.weight makes the tied copy unnecessary
  if ((s = need("output.weight", true)) != B2Q_OK) return s;
  if ((s = need("token_embd.weight", false)) != B2Q_OK) return s;
  if ((s = need("output_norm.weight", false)) != B2Q_OK) return s;
  static const char* const kRequired[] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight",
                                          "attn_v.weight", "attn_output.weight", "ffn_norm.weight",
                                          "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
  static const char* const kOptional[] = {"attn_q.bias", "attn_k.bias", "attn_v.bias"};
  for (int l = 0; l < M->c.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    for (const char* r : kRequired)
      if ((s = need(p + r, false)) != B2Q_OK) return s;
    for (const char* r : kOptional)
      if ((s = need(p + r, true)) != B2Q_OK) return s;
  }
  return B2Q_OK;
}

}  // extern "C"
