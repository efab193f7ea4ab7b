// gguf.cuh -- GGUF container parser and model loader (host code).
//
// Restates GgufModelFile::open (src/inference.rs:343-446) with its
// ByteCursor (:262-340) and the GgufValue accessors (:186-232) on a POSIX
// read-only mapping instead of the reference's Win32 mapping (:15-110):
//   header "GGUF", u32 version 1..3; tensor and key/value counts, string and
//   array lengths and tensor dims are u32 in version 1 and u64 after;
//   metadata values of types 0..12; tensor infos (name, n_dims, dims in GGML
//   order [inner, outer..] reversed to [outer.., inner], GGML type, u64
//   offset relative to the data section); the data section starts at the
//   next multiple of general.alignment (default 32, at least 1);
//   byte_len = elements / block_size * type_size and must end inside the
//   file.  Later duplicates of a key or tensor name replace earlier ones
//   (HashMap::insert).
//
// b2q_model_load_gguf follows StandardNativeEngine::from_gguf
// (src/inference.rs:2513-2587): hyperparameters from "{arch}.*" keys with
// "llama" as the fallback prefix, token_embd / output_norm / output (tied
// to token_embd when absent) and per block attn_norm, attn_q/k/v (+
// optional biases), attn_output, ffn_norm, ffn_gate/up/down.  Each rank
// uploads only the rows of its tensor-parallel shard, straight from the
// mapping.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace gguf {

constexpr int kMaxDims = 8;     // GGML itself uses at most 4
constexpr int kMaxNesting = 16; // arrays of arrays

enum VType : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

struct Value {
  uint32_t type = 0;
  uint64_t bits = 0;        // scalar payload, little-endian, zero-extended
  uint64_t off = 0, len = 0; // string: bytes in the file; array: first element, element count
  uint32_t elem_type = 0;   // array element type
};

struct Tensor {
  std::string name;
  int n_dims = 0;
  int64_t dims[kMaxDims] = {};  // [outer.., inner]
  int ggml_type = 0;
  uint64_t abs_offset = 0, byte_len = 0;
};

// GgmlDType::from_u32 / block_size / type_size (src/inference.rs:136-185)
inline bool type_geometry(uint32_t t, int* block, int* size) {
  switch (t) {
    case 0: *block = 1; *size = 4; return true;     // F32
    case 1: *block = 1; *size = 2; return true;     // F16
    case 2: *block = 32; *size = 18; return true;   // Q4_0
    case 3: *block = 32; *size = 20; return true;   // Q4_1
    case 6: *block = 32; *size = 22; return true;   // Q5_0
    case 7: *block = 32; *size = 24; return true;   // Q5_1
    case 8: *block = 32; *size = 34; return true;   // Q8_0
    case 9: *block = 32; *size = 36; return true;   // Q8_1
    case 10: *block = 256; *size = 84; return true; // Q2_K
    case 11: *block = 256; *size = 110; return true;// Q3_K
    case 12: *block = 256; *size = 144; return true;// Q4_K
    case 13: *block = 256; *size = 176; return true;// Q5_K
    case 14: *block = 256; *size = 210; return true;// Q6_K
    case 15: *block = 256; *size = 292; return true;// Q8_K
    case 30: *block = 1; *size = 2; return true;    // BF16
    default: return false;
  }
}

struct File {
  const uint8_t* data = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t data_offset = 0;
  std::unordered_map<std::string, Value> kv;
  std::vector<Tensor> tensors;                   // file order, duplicates removed
  std::unordered_map<std::string, size_t> index; // name -> tensors[i]

  ~File() {
    if (data) munmap(const_cast<uint8_t*>(data), size);
  }

  const Value* get(const std::string& key) const {
    auto it = kv.find(key);
    return it == kv.end() ? nullptr : &it->second;
  }
  // GgufValue::as_usize (src/inference.rs:203-213)
  bool as_usize(const Value& v, uint64_t* out) const {
    switch (v.type) {
      case kU32: case kU64: case kU16: case kU8: *out = v.bits; return true;
      case kI32: if ((int32_t)(uint32_t)v.bits < 0) return false; *out = (uint64_t)(int32_t)(uint32_t)v.bits; return true;
      case kI64: if ((int64_t)v.bits < 0) return false; *out = v.bits; return true;
      default: return false;
    }
  }
  // GgufValue::as_f32 (src/inference.rs:215-223)
  bool as_f32(const Value& v, float* out) const {
    switch (v.type) {
      case kF32: { uint32_t b = (uint32_t)v.bits; memcpy(out, &b, 4); return true; }
      case kF64: { double d; memcpy(&d, &v.bits, 8); *out = (float)d; return true; }
      case kU32: *out = (float)(uint32_t)v.bits; return true;
      case kI32: *out = (float)(int32_t)(uint32_t)v.bits; return true;
      default: return false;
    }
  }
  bool get_usize(const std::string& key, uint64_t* out) const {
    const Value* v = get(key);
    return v && as_usize(*v, out);
  }
  bool get_f32(const std::string& key, float* out) const {
    const Value* v = get(key);
    return v && as_f32(*v, out);
  }
  const Tensor* tensor(const std::string& name) const {
    auto it = index.find(name);
    return it == index.end() ? nullptr : &tensors[it->second];
  }
};

// Bounds-checked little-endian reader over the mapping (ByteCursor).
struct Cursor {
  const uint8_t* d;
  size_t n, pos;
  uint32_t version;
  std::string err;

  bool fail_eof() {
    if (err.empty()) err = "unexpected end of GGUF file at position " + std::to_string(pos);
    return false;
  }
  bool bytes(size_t k, const uint8_t** p) {
    if (k > n - pos) return fail_eof();
    *p = d + pos;
    pos += k;
    return true;
  }
  bool uint(int k, uint64_t* v) {
    const uint8_t* p;
    if (!bytes((size_t)k, &p)) return false;
    uint64_t x = 0;
    for (int i = k - 1; i >= 0; --i) x = (x << 8) | p[i];
    *v = x;
    return true;
  }
  bool u32(uint32_t* v) {
    uint64_t x;
    if (!uint(4, &x)) return false;
    *v = (uint32_t)x;
    return true;
  }
  bool len(uint64_t* v) { return uint(version == 1 ? 4 : 8, v); }
  bool str(uint64_t* off, uint64_t* l) {
    const uint8_t* p;
    if (!len(l)) return false;
    if (*l > n - pos) return fail_eof();
    *off = pos;
    return bytes((size_t)*l, &p);
  }
  bool value(uint32_t type, Value* v, int depth) {
    v->type = type;
    switch (type) {
      case kU8: case kI8: case kBool: return uint(1, &v->bits);
      case kU16: case kI16: return uint(2, &v->bits);
      case kU32: case kI32: case kF32: return uint(4, &v->bits);
      case kU64: case kI64: case kF64: return uint(8, &v->bits);
      case kString: return str(&v->off, &v->len);
      case kArray: {
        if (depth >= kMaxNesting) {
          err = "GGUF arrays nested too deeply";
          return false;
        }
        if (!u32(&v->elem_type) || !len(&v->len)) return false;
        v->off = pos;
        Value e;
        for (uint64_t i = 0; i < v->len; ++i)
          if (!value(v->elem_type, &e, depth + 1)) return false;
        return true;
      }
      default:
        err = "unknown GGUF metadata value type " + std::to_string(type);
        return false;
    }
  }
};

// Parse an already-mapped file; `f->data`/`f->size` are set.  Metadata keys
// are appended to `keys` in file order (first occurrence).  Returns an empty
// string or the reason for rejecting the file.
inline std::string parse(File* f, std::vector<std::string>* keys) {
  if (f->size < 16 || memcmp(f->data, "GGUF", 4) != 0) return "not a GGUF file (no 'GGUF' header)";
  Cursor c{f->data, f->size, 4, 0, {}};
  uint32_t version;
  c.u32(&version);
  if (version < 1 || version > 3) return "unsupported GGUF version " + std::to_string(version);
  f->version = c.version = version;
  uint64_t n_tensors, n_kv;
  if (!c.len(&n_tensors) || !c.len(&n_kv)) return c.err;
  for (uint64_t i = 0; i < n_kv; ++i) {
    uint64_t ko, kl;
    uint32_t vt;
    Value v;
    if (!c.str(&ko, &kl) || !c.u32(&vt) || !c.value(vt, &v, 0)) return c.err;
    std::string key(reinterpret_cast<const char*>(f->data + ko), (size_t)kl);
    if (f->kv.find(key) == f->kv.end()) keys->push_back(key);
    f->kv[key] = v;
  }
  struct Raw { Tensor t; uint64_t rel; };
  std::vector<Raw> raw;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    Raw r;
    uint64_t no, nl;
    uint32_t nd, type;
    if (!c.str(&no, &nl) || !c.u32(&nd)) return c.err;
    r.t.name.assign(reinterpret_cast<const char*>(f->data + no), (size_t)nl);
    if (nd > (uint32_t)kMaxDims) return "tensor '" + r.t.name + "': " + std::to_string(nd) + " dims";
    r.t.n_dims = (int)nd;
    for (uint32_t j = 0; j < nd; ++j) {
      uint64_t dj;
      if (!c.len(&dj)) return c.err;
      if (dj > (uint64_t)INT64_MAX) return "tensor '" + r.t.name + "': dim out of range";
      r.t.dims[nd - 1 - j] = (int64_t)dj;  // [inner, outer..] -> [outer.., inner]
    }
    if (!c.u32(&type)) return c.err;
    int bs, ts;
    if (!type_geometry(type, &bs, &ts)) return "unknown GGML type " + std::to_string(type) + " in GGUF";
    r.t.ggml_type = (int)type;
    if (!c.uint(8, &r.rel)) return c.err;
    raw.push_back(r);
  }
  uint64_t align = 32;
  if (const Value* a = f->get("general.alignment")) {
    uint64_t x;
    if (f->as_usize(*a, &x)) align = x;
  }
  if (align < 1) align = 1;
  const uint64_t pad = (align - c.pos % align) % align;
  f->data_offset = c.pos + pad;
  for (Raw& r : raw) {
    int bs, ts;
    type_geometry((uint32_t)r.t.ggml_type, &bs, &ts);
    // element count in 64 bits, overflow rejected: a product that wrapped
    // would give a small byte length for dims that describe a huge tensor
    uint64_t elems = 1;
    for (int j = 0; j < r.t.n_dims; ++j)
      if (__builtin_mul_overflow(elems, (uint64_t)r.t.dims[j], &elems))
        return "tensor '" + r.t.name + "': element count overflows 64 bits";
    const unsigned __int128 blen = (unsigned __int128)(elems / (unsigned)bs) * (unsigned)ts;
    const unsigned __int128 end = (unsigned __int128)f->data_offset + r.rel + blen;
    if (end > f->size)
      return "tensor '" + r.t.name + "' extends past the end of the GGUF file (" +
             std::to_string((unsigned long long)(end > ~0ull ? ~0ull : (uint64_t)end)) + " > " +
             std::to_string(f->size) + ")";
    r.t.abs_offset = f->data_offset + r.rel;
    r.t.byte_len = (uint64_t)blen;
    auto it = f->index.find(r.t.name);
    if (it != f->index.end()) {
      f->tensors[it->second] = r.t;
    } else {
      f->index[r.t.name] = f->tensors.size();
      f->tensors.push_back(r.t);
    }
  }
  return {};
}

// IEEE binary16 -> binary32, exact for every pattern (f16_to_f32,
// src/inference.rs:868-890).
inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
  if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    int e = 113;  // normalise the subnormal
    while (!(man & 0x400u)) {
      man <<= 1;
      --e;
    }
    bits = sign | ((uint32_t)e << 23) | ((man & 0x3ffu) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

}  // namespace gguf
