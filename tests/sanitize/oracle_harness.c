/* Sanitizer driver for the CPU oracle (oracle/gguf_oracle.c,
 * oracle/llama_oracle.c), built by tests/test_oracle_sanitize.py together with
 * the oracle sources under -fsanitize=address,undefined.
 *
 * Every buffer is a heap allocation of exactly the size the call may touch,
 * so a read or write past it is an AddressSanitizer error:
 *   - every supported block type through oracle_dequantize and both
 *     matvecs (m = 1 and m = 3; x holding NaN, inf and huge values);
 *   - a 2-layer Llama model with q/k/v biases through oracle_forward_ref,
 *     oracle_forward_f64 (prompt, then single-token steps up to the KV
 *     capacity) and oracle_sample.
 * Values are random bytes: only memory safety is checked here.  Prints "ok"
 * and exits 0. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  int n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, n_vocab;
  float rms_eps, rope_theta;
} OracleConfig;

int oracle_block_size(int t);
int oracle_type_size(int t);
int oracle_dequantize(const uint8_t* bytes, int dtype, int64_t out_len, float* out);
int oracle_matmul_batched(const uint8_t* w, int dtype, int64_t n, int64_t k, const float* x, int64_t m, float* out);
int oracle_matmul_f64(const uint8_t* w, int dtype, int64_t n, int64_t k, const float* x, int64_t m, double* out);
void oracle_set_threads(int n);
void* oracle_model_create(const OracleConfig* cfg, int64_t kv_capacity);
void oracle_model_free(void* p);
int oracle_model_set(void* p, int role, int layer, const void* bytes, int dtype, int64_t n, int64_t k);
int oracle_forward_ref(void* p, const uint32_t* tokens, int64_t seq_len, int64_t start_pos, float* logits);
int oracle_forward_f64(void* p, const uint32_t* tokens, int64_t seq_len, int64_t start_pos, int kv_f16,
                       double* logits);
uint32_t oracle_sample(const float* logits, int64_t n, float temperature, float top_p, uint64_t* state,
                       int* drew);

static uint64_t g_rng = 0x9E3779B97F4A7C15ull;
static uint8_t next_byte(void) {
  g_rng ^= g_rng << 13;
  g_rng ^= g_rng >> 7;
  g_rng ^= g_rng << 17;
  return (uint8_t)(g_rng >> 24);
}

static void* xmalloc(size_t n) {
  void* p = malloc(n ? n : 1);
  if (!p) {
    fprintf(stderr, "out of memory\n");
    exit(1);
  }
  return p;
}

static uint8_t* rand_bytes(size_t n) {
  uint8_t* p = (uint8_t*)xmalloc(n);
  for (size_t i = 0; i < n; ++i) p[i] = next_byte();
  return p;
}

static size_t tensor_bytes(int dtype, int64_t n, int64_t k) {
  return (size_t)(n * (k / oracle_block_size(dtype)) * oracle_type_size(dtype));
}

/* random bytes, with every f32 element finite and small when the type is F32 */
static uint8_t* rand_tensor(int dtype, int64_t n, int64_t k) {
  const size_t nb = tensor_bytes(dtype, n, k);
  uint8_t* p = rand_bytes(nb);
  if (dtype == 0)
    for (size_t i = 0; i < nb / 4; ++i) {
      float v = (float)((int)next_byte() - 128) / 128.0f;
      memcpy(p + 4 * i, &v, 4);
    }
  return p;
}

static void matvec_types(void) {
  static const int types[] = {0, 1, 2, 8, 12, 13, 14, 30};
  const int64_t n = 5, k = 512;
  for (size_t i = 0; i < sizeof types / sizeof types[0]; ++i) {
    const int t = types[i];
    if (oracle_block_size(t) == 0) continue;
    uint8_t* w = rand_bytes(tensor_bytes(t, n, k));
    float* deq = (float*)xmalloc(sizeof(float) * (size_t)(n * k));
    oracle_dequantize(w, t, n * k, deq);
    for (int m = 1; m <= 3; m += 2) {
      float* x = (float*)xmalloc(sizeof(float) * (size_t)(m * k));
      for (int64_t j = 0; j < m * k; ++j) x[j] = (float)((int)next_byte() - 128) * 0.01f;
      x[3] = NAN;
      x[k / 2] = INFINITY;
      x[k - 1] = 3.0e38f;
      float* y = (float*)xmalloc(sizeof(float) * (size_t)(m * n));
      double* y64 = (double*)xmalloc(sizeof(double) * (size_t)(m * n));
      oracle_matmul_batched(w, t, n, k, x, m, y);
      oracle_matmul_f64(w, t, n, k, x, m, y64);
      free(x);
      free(y);
      free(y64);
    }
    free(w);
    free(deq);
  }
}

static void llama_model(void) {
  const OracleConfig c = {2, 256, 4, 2, 64, 512, 64, 1e-5f, 500000.0f};
  const int64_t cap = 12;
  void* m = oracle_model_create(&c, cap);
  uint8_t* keep[64];
  int nk = 0;
#define SET(role, layer, dtype, n, k)                                            \
  do {                                                                           \
    keep[nk] = rand_tensor(dtype, n, k);                                         \
    if (oracle_model_set(m, role, layer, keep[nk], dtype, n, k) != 0) {          \
      fprintf(stderr, "oracle_model_set(role %d, layer %d) failed\n", role, layer); \
      exit(1);                                                                   \
    }                                                                            \
    ++nk;                                                                        \
  } while (0)
  SET(0, -1, 12, c.n_vocab, c.n_embd);  /* token_embd, Q4_K */
  SET(1, -1, 14, c.n_vocab, c.n_embd);  /* output, Q6_K */
  SET(2, -1, 0, 1, c.n_embd);           /* output_norm */
  for (int l = 0; l < c.n_layers; ++l) {
    const int64_t qd = (int64_t)c.n_heads * c.head_dim, kvd = (int64_t)c.n_kv_heads * c.head_dim;
    SET(3, l, 0, 1, c.n_embd);
    SET(4, l, 12, qd, c.n_embd);
    SET(5, l, 12, kvd, c.n_embd);
    SET(6, l, 14, kvd, c.n_embd);
    SET(7, l, 12, c.n_embd, qd);
    SET(8, l, 0, 1, c.n_embd);
    SET(9, l, 12, c.n_ff, c.n_embd);
    SET(10, l, 12, c.n_ff, c.n_embd);
    SET(11, l, 14, c.n_embd, c.n_ff);
    SET(12, l, 0, 1, qd);
    SET(13, l, 0, 1, kvd);
    SET(14, l, 0, 1, kvd);
  }
#undef SET
  uint32_t* prompt = (uint32_t*)xmalloc(sizeof(uint32_t) * 5);
  for (int i = 0; i < 5; ++i) prompt[i] = (uint32_t)(next_byte() % c.n_vocab);
  float* logits = (float*)xmalloc(sizeof(float) * (size_t)c.n_vocab);
  double* logits64 = (double*)xmalloc(sizeof(double) * (size_t)c.n_vocab);
  uint64_t state = 42;
  for (int pass = 0; pass < 2; ++pass) {  /* pass 0: reference f32 path; pass 1: fp64 path */
    int rc = pass ? oracle_forward_f64(m, prompt, 5, 0, 1, logits64) : oracle_forward_ref(m, prompt, 5, 0, logits);
    if (rc != 0) {
      fprintf(stderr, "forward over the prompt failed: %d\n", rc);
      exit(1);
    }
    for (int64_t pos = 5; pos < cap; ++pos) {
      uint32_t tok = (uint32_t)(pos % c.n_vocab);
      rc = pass ? oracle_forward_f64(m, &tok, 1, pos, 0, logits64) : oracle_forward_ref(m, &tok, 1, pos, logits);
      if (rc != 0) {
        fprintf(stderr, "forward at position %lld failed: %d\n", (long long)pos, rc);
        exit(1);
      }
      int drew = 0;
      if (!pass) oracle_sample(logits, c.n_vocab, 0.8f, 0.9f, &state, &drew);
    }
  }
  free(prompt);
  free(logits);
  free(logits64);
  for (int i = 0; i < nk; ++i) free(keep[i]);
  oracle_model_free(m);
}

int main(void) {
  oracle_set_threads(2);
  matvec_types();
  llama_model();
  printf("ok\n");
  return 0;
}
