// Sanitizer harness for the GGUF parser (csrc/gguf.cuh, host code), built by
// tests/test_gguf_sanitize.py with -fsanitize=address,undefined.
//
// Every case is parsed from a heap copy of exactly its size, so a read past
// the end of the file is an AddressSanitizer error rather than a silent read
// of mapped memory.  For every file the parser accepts, the harness checks
// what the loader relies on and touches every byte the parser points at:
//   * each tensor's [abs_offset, abs_offset + byte_len) lies inside the file;
//   * its element count fits in 64 bits and byte_len = elements / block *
//     type size (the reference's byte_len, inference.rs:403-420);
//   * each string value's bytes lie inside the file.
//
//   gguf_parse_harness one FILE   parse FILE: prints "ok" or "rejected: why"
//   gguf_parse_harness fuzz FILE  FILE (which must parse), every prefix of it,
//                                 and every header byte set to each of six
//                                 values: prints the accepted / rejected counts
// Exit status 0, or 2 when an invariant does not hold.
#include "gguf.cuh"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>

namespace {

volatile uint64_t g_sink;

bool touch(const uint8_t* base, size_t size, uint64_t off, uint64_t len, const char* what) {
  if (off > size || len > size - off) {
    fprintf(stderr, "invariant: %s [%llu, +%llu) outside a %zu-byte file\n", what, (unsigned long long)off,
            (unsigned long long)len, size);
    return false;
  }
  uint64_t s = 0;
  for (uint64_t i = 0; i < len; ++i) s += base[off + i];
  g_sink += s;
  return true;
}

// 0: rejected, 1: accepted, 2: an invariant failed
int check(const uint8_t* bytes, size_t n, std::string* why) {
  uint8_t* copy = static_cast<uint8_t*>(malloc(n ? n : 1));
  if (n) memcpy(copy, bytes, n);
  int rc = 1;
  {
    gguf::File f;
    f.data = copy;
    f.size = n;
    std::vector<std::string> keys;
    const std::string err = gguf::parse(&f, &keys);
    if (!err.empty()) {
      rc = 0;
      if (why) *why = err;
    } else {
      for (const gguf::Tensor& t : f.tensors) {
        int bs = 0, ts = 0;
        uint64_t elems = 1;
        bool over = false;
        for (int j = 0; j < t.n_dims; ++j) over |= __builtin_mul_overflow(elems, (uint64_t)t.dims[j], &elems);
        if (!gguf::type_geometry((uint32_t)t.ggml_type, &bs, &ts) || over ||
            (unsigned __int128)(elems / (unsigned)bs) * (unsigned)ts != t.byte_len) {
          fprintf(stderr, "invariant: tensor '%s' byte_len %llu does not follow from its dims\n", t.name.c_str(),
                  (unsigned long long)t.byte_len);
          rc = 2;
        }
        if (!touch(copy, n, t.abs_offset, t.byte_len, t.name.c_str())) rc = 2;
      }
      for (const std::string& k : keys) {
        const gguf::Value* v = f.get(k);
        uint64_t u;
        float x;
        f.as_usize(*v, &u);
        f.as_f32(*v, &x);
        if (v->type == gguf::kString && !touch(copy, n, v->off, v->len, k.c_str())) rc = 2;
      }
    }
    f.data = nullptr;  // a heap copy, not a mapping: the destructor must not unmap it
  }
  free(copy);
  return rc;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: %s one|fuzz FILE\n", argv[0]);
    return 1;
  }
  std::ifstream in(argv[2], std::ios::binary);
  const std::vector<uint8_t> file((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  std::string why;
  if (std::string(argv[1]) == "one") {
    const int rc = check(file.data(), file.size(), &why);
    if (rc == 2) return 2;
    printf(rc ? "ok\n" : "rejected: %s\n", why.c_str());
    return 0;
  }
  if (check(file.data(), file.size(), &why) != 1) {
    fprintf(stderr, "the seed file does not parse: %s\n", why.c_str());
    return 1;
  }
  long accepted = 0, rejected = 0;
  for (size_t len = 0; len < file.size(); ++len) {
    const int rc = check(file.data(), len, nullptr);
    if (rc == 2) return 2;
    (rc ? accepted : rejected) += 1;
  }
  // header bytes: everything before the data section of the seed file
  gguf::File seed;
  std::vector<uint8_t> copy(file);
  seed.data = copy.data();
  seed.size = copy.size();
  std::vector<std::string> keys;
  gguf::parse(&seed, &keys);
  const size_t head = std::min<size_t>(seed.data_offset, 8192);
  seed.data = nullptr;
  static const uint8_t kVals[] = {0x00, 0xff, 0x7f, 0x80, 0x01, 0x40};
  for (size_t pos = 0; pos < head; ++pos)
    for (uint8_t v : kVals) {
      if (copy[pos] == v) continue;
      const uint8_t keep = copy[pos];
      copy[pos] = v;
      const int rc = check(copy.data(), copy.size(), nullptr);
      copy[pos] = keep;
      if (rc == 2) return 2;
      (rc ? accepted : rejected) += 1;
    }
  printf("accepted %ld rejected %ld\n", accepted, rejected);
  return 0;
}
