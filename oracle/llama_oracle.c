/*
 * llama_oracle.c -- CPU oracle of StandardNativeEngine::forward.
 *
 * TEST INFRASTRUCTURE ONLY (see gguf_oracle.c for the rules that apply).
 *
 * Two forwards over the same borrowed GGUF tensors:
 *   oracle_forward_ref  the reference's own f32 CPU path, restated from
 *                       src/inference.rs:2695-2860 (quantised-x AVX2 matvecs
 *                       via oracle_matmul_batched, f32 KV cache, f32 RoPE
 *                       tables, f32 softmax).  This is the timed CPU baseline.
 *   oracle_forward_f64  the same block loop in double precision over the
 *                       bit-exact dequantised weights; the KV cache can be
 *                       rounded to f16 on store, as the device cache is.
 *                       This is the tolerance oracle (rel-L2 <= 1e-3).
 * Parity unpinned: the reference cannot run here and ships no golden
 * logits, so neither forward is checked against reference outputs; the f32
 * path follows the cited lines operation by operation, and the fp64 path is
 * the gate.
 * The RoPE cos/sin tables follow the reference's f32 recipe
 * (inference.rs:2538-2549) in both paths: they are part of the model
 * definition, like the weights.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

int oracle_block_size(int t);
int oracle_type_size(int t);
int oracle_dequantize(const uint8_t* bytes, int dtype, int64_t out_len, float* out);
int oracle_matmul_batched(const uint8_t* w, int dtype, int64_t n, int64_t k,
                          const float* x, int64_t m, float* out);
float oracle_vec_dot_f32(const float* a, const float* b, int64_t n);
void oracle_axpy_f32(float* dst, float scale, const float* src, int64_t n);

typedef struct {
  int n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, n_vocab;
  float rms_eps, rope_theta;
} OracleConfig;

typedef struct { const uint8_t* bytes; int dtype; int64_t n, k; } OTensor;

typedef struct {
  OTensor q, k, v, o, gate, up, down;
  const float *attn_norm, *ffn_norm, *q_bias, *k_bias, *v_bias;
  float *kc32, *vc32;   /* reference path cache [t][kv_head][head_dim] */
  double *kc64, *vc64;  /* fp64 path cache, same layout */
  int64_t len32, len64;
} OLayer;

typedef struct {
  OracleConfig c;
  OTensor tok_embd, output;
  const float* output_norm;
  OLayer* layers;
  float *rope_cos, *rope_sin; /* [8192][head_dim/2] */
  int64_t cap;                /* KV capacity in tokens */
} OModel;

#define MAX_SEQ 8192

void* oracle_model_create(const OracleConfig* cfg, int64_t kv_capacity) {
  OModel* m = (OModel*)calloc(1, sizeof(OModel));
  m->c = *cfg;
  m->cap = kv_capacity;
  m->layers = (OLayer*)calloc((size_t)cfg->n_layers, sizeof(OLayer));
  int hd = cfg->head_dim, half = hd / 2;
  m->rope_cos = (float*)malloc(sizeof(float) * MAX_SEQ * half);
  m->rope_sin = (float*)malloc(sizeof(float) * MAX_SEQ * half);
  /* inference.rs:2538-2549: freq = 1/theta^(2j/hd) in f32 powf, angle in f32 */
  for (int pos = 0; pos < MAX_SEQ; pos++) {
    for (int j = 0; j < half; j++) {
      float freq = 1.0f / powf(cfg->rope_theta, (float)(2 * j) / (float)hd);
      float angle = (float)pos * freq;
      m->rope_cos[pos * half + j] = cosf(angle);
      m->rope_sin[pos * half + j] = sinf(angle);
    }
  }
  size_t kvn = (size_t)kv_capacity * cfg->n_kv_heads * hd;
  for (int l = 0; l < cfg->n_layers; l++) {
    m->layers[l].kc32 = (float*)calloc(kvn, sizeof(float));
    m->layers[l].vc32 = (float*)calloc(kvn, sizeof(float));
    m->layers[l].kc64 = (double*)calloc(kvn, sizeof(double));
    m->layers[l].vc64 = (double*)calloc(kvn, sizeof(double));
  }
  return m;
}

void oracle_model_free(void* p) {
  OModel* m = (OModel*)p;
  if (!m) return;
  for (int l = 0; l < m->c.n_layers; l++) {
    free(m->layers[l].kc32); free(m->layers[l].vc32);
    free(m->layers[l].kc64); free(m->layers[l].vc64);
  }
  free(m->layers); free(m->rope_cos); free(m->rope_sin); free(m);
}

void oracle_clear_state(void* p) {
  OModel* m = (OModel*)p;
  for (int l = 0; l < m->c.n_layers; l++) { m->layers[l].len32 = 0; m->layers[l].len64 = 0; }
}

/* Timing set-up for the CPU baseline (not part of the reference): the f32
 * reference-path KV cache of every layer holds `n` positions of seeded
 * synthetic rows, uniform in [-1, 1), as after an n-token prompt, so that
 * decode steps can be timed at that context without the prompt pass. */
int oracle_fill_kv(void* p, int64_t n, uint64_t seed) {
  OModel* m = (OModel*)p;
  if (n < 0 || n > m->cap) return -1;
  const int64_t row = (int64_t)m->c.n_kv_heads * m->c.head_dim;
  for (int l = 0; l < m->c.n_layers; l++) {
    OLayer* L = &m->layers[l];
    uint64_t s = seed ^ ((uint64_t)(l + 1) * 0x9e3779b97f4a7c15ull);
    for (int64_t i = 0; i < n * row; i++) {
      s ^= s << 13; s ^= s >> 7; s ^= s << 17;
      L->kc32[i] = (float)(s >> 40) * (1.0f / 8388608.0f) - 1.0f;
      s ^= s << 13; s ^= s >> 7; s ^= s << 17;
      L->vc32[i] = (float)(s >> 40) * (1.0f / 8388608.0f) - 1.0f;
    }
    L->len32 = n;
  }
  return 0;
}

const float* oracle_rope_table(void* p, int cos_not_sin) {
  OModel* m = (OModel*)p;
  return cos_not_sin ? m->rope_cos : m->rope_sin;
}

/* role ids for oracle_model_set */
enum { R_TOK = 0, R_OUT, R_OUT_NORM, R_ATTN_NORM, R_Q, R_K, R_V, R_O, R_FFN_NORM,
       R_GATE, R_UP, R_DOWN, R_QB, R_KB, R_VB };

int oracle_model_set(void* p, int role, int layer, const void* bytes, int dtype, int64_t n, int64_t k) {
  OModel* m = (OModel*)p;
  OTensor t = {(const uint8_t*)bytes, dtype, n, k};
  if (role == R_TOK) { m->tok_embd = t; return 0; }
  if (role == R_OUT) { m->output = t; return 0; }
  if (role == R_OUT_NORM) { m->output_norm = (const float*)bytes; return 0; }
  if (layer < 0 || layer >= m->c.n_layers) return -1;
  OLayer* L = &m->layers[layer];
  switch (role) {
    case R_ATTN_NORM: L->attn_norm = (const float*)bytes; return 0;
    case R_FFN_NORM: L->ffn_norm = (const float*)bytes; return 0;
    case R_Q: L->q = t; return 0;
    case R_K: L->k = t; return 0;
    case R_V: L->v = t; return 0;
    case R_O: L->o = t; return 0;
    case R_GATE: L->gate = t; return 0;
    case R_UP: L->up = t; return 0;
    case R_DOWN: L->down = t; return 0;
    case R_QB: L->q_bias = (const float*)bytes; return 0;
    case R_KB: L->k_bias = (const float*)bytes; return 0;
    case R_VB: L->v_bias = (const float*)bytes; return 0;
    default: return -1;
  }
}

/* MmapWeight::get_row_f32: inference.rs:575-582 */
static int get_row_f32(const OTensor* t, int64_t row, float* out) {
  int bs = oracle_block_size(t->dtype), ts = oracle_type_size(t->dtype);
  int64_t row_bytes = (t->k / bs) * ts;
  return oracle_dequantize(t->bytes + row * row_bytes, t->dtype, t->k, out);
}

/* rms_norm_rows: inference.rs:1501-1512 */
static void rms_norm_rows_f32(const float* x, const float* w, int64_t rows, int dim, float eps, float* out) {
  for (int64_t r = 0; r < rows; r++) {
    const float* xi = x + r * dim;
    float* yo = out + r * dim;
    float ss = oracle_vec_dot_f32(xi, xi, dim);
    float inv = 1.0f / sqrtf((ss / (float)dim) + eps);
    for (int i = 0; i < dim; i++) yo[i] = xi[i] * inv * w[i];
  }
}

static inline float silu_f32(float x) { return x / (1.0f + expf(-x)); } /* inference.rs:1481 */

/* NeoX half-split RoPE: inference.rs:2755-2777 */
static void rope_f32(float* v, int nheads, int hd, const float* cs, const float* sn) {
  int half = hd / 2;
  for (int h = 0; h < nheads; h++) {
    float* b = v + (int64_t)h * hd;
    for (int j = 0; j < half; j++) {
      float x0 = b[j], x1 = b[half + j];
      b[j] = x0 * cs[j] - x1 * sn[j];
      b[half + j] = x1 * cs[j] + x0 * sn[j];
    }
  }
}

static void add_bias_f32(float* v, const float* b, int64_t rows, int n) {
  if (!b) return;
  for (int64_t r = 0; r < rows; r++) for (int i = 0; i < n; i++) v[r * n + i] += b[i];
}

/* StandardNativeEngine::forward, f32 reference path: inference.rs:2695-2860 */
int oracle_forward_ref(void* p, const uint32_t* tokens, int64_t seq_len, int64_t start_pos, float* logits) {
  OModel* m = (OModel*)p;
  const OracleConfig* c = &m->c;
  int E = c->n_embd, H = c->n_heads, KV = c->n_kv_heads, hd = c->head_dim, half = hd / 2;
  int F = c->n_ff;
  if (seq_len <= 0) return -1;
  float* x = (float*)calloc((size_t)(seq_len * E), sizeof(float));
  for (int64_t t = 0; t < seq_len; t++)
    if (get_row_f32(&m->tok_embd, tokens[t], x + t * E) != 0) { free(x); return -2; }
  float* normed = (float*)malloc(sizeof(float) * seq_len * E);
  float* q = (float*)malloc(sizeof(float) * seq_len * H * hd);
  float* kk = (float*)malloc(sizeof(float) * seq_len * KV * hd);
  float* vv = (float*)malloc(sizeof(float) * seq_len * KV * hd);
  float* attn = (float*)malloc(sizeof(float) * seq_len * H * hd);
  float* proj = (float*)malloc(sizeof(float) * seq_len * E);
  float* gate = (float*)malloc(sizeof(float) * seq_len * F);
  float* up = (float*)malloc(sizeof(float) * seq_len * F);
  int rc = 0;
  for (int l = 0; l < c->n_layers && rc == 0; l++) {
    OLayer* L = &m->layers[l];
    if (L->len32 + seq_len > m->cap) { rc = -3; break; }
    rms_norm_rows_f32(x, L->attn_norm, seq_len, E, c->rms_eps, normed);
    oracle_matmul_batched(L->q.bytes, L->q.dtype, L->q.n, E, normed, seq_len, q);
    oracle_matmul_batched(L->k.bytes, L->k.dtype, L->k.n, E, normed, seq_len, kk);
    oracle_matmul_batched(L->v.bytes, L->v.dtype, L->v.n, E, normed, seq_len, vv);
    add_bias_f32(q, L->q_bias, seq_len, H * hd);
    add_bias_f32(kk, L->k_bias, seq_len, KV * hd);
    add_bias_f32(vv, L->v_bias, seq_len, KV * hd);
    for (int64_t s = 0; s < seq_len; s++) {
      int64_t pos = start_pos + s < 8191 ? start_pos + s : 8191;
      rope_f32(q + s * H * hd, H, hd, m->rope_cos + pos * half, m->rope_sin + pos * half);
      rope_f32(kk + s * KV * hd, KV, hd, m->rope_cos + pos * half, m->rope_sin + pos * half);
    }
    memcpy(L->kc32 + L->len32 * KV * hd, kk, sizeof(float) * seq_len * KV * hd);
    memcpy(L->vc32 + L->len32 * KV * hd, vv, sizeof(float) * seq_len * KV * hd);
    L->len32 += seq_len;
    int64_t total_seq = L->len32;
    int gqa = H / KV;
    float scale = 1.0f / sqrtf((float)hd);
    memset(attn, 0, sizeof(float) * seq_len * H * hd);
    for (int64_t s = 0; s < seq_len; s++) {
      int64_t valid_t = start_pos + s + 1 < total_seq ? start_pos + s + 1 : total_seq;
#pragma omp parallel for schedule(static)
      for (int h = 0; h < H; h++) {
        int kh = h / gqa;
        const float* qh = q + (s * H + h) * hd;
        float* oh = attn + (s * H + h) * hd;
        float* scores = (float*)malloc(sizeof(float) * (size_t)valid_t);
        float maxs = -INFINITY;
        for (int64_t t = 0; t < valid_t; t++) {
          float sc = oracle_vec_dot_f32(qh, L->kc32 + (t * KV + kh) * hd, hd) * scale;
          scores[t] = sc;
          if (sc > maxs) maxs = sc;
        }
        float sum = 0.0f;
        for (int64_t t = 0; t < valid_t; t++) { scores[t] = expf(scores[t] - maxs); sum += scores[t]; }
        float inv_sum = 1.0f / (sum > 1e-12f ? sum : 1e-12f);
        for (int64_t t = 0; t < valid_t; t++) {
          oracle_axpy_f32(oh, scores[t] * inv_sum, L->vc32 + (t * KV + kh) * hd, hd);
        }
        free(scores);
      }
    }
    oracle_matmul_batched(L->o.bytes, L->o.dtype, L->o.n, H * hd, attn, seq_len, proj);
    for (int64_t i = 0; i < seq_len * E; i++) x[i] += proj[i];
    rms_norm_rows_f32(x, L->ffn_norm, seq_len, E, c->rms_eps, normed);
    oracle_matmul_batched(L->gate.bytes, L->gate.dtype, L->gate.n, E, normed, seq_len, gate);
    oracle_matmul_batched(L->up.bytes, L->up.dtype, L->up.n, E, normed, seq_len, up);
    for (int64_t i = 0; i < seq_len * F; i++) gate[i] = silu_f32(gate[i]) * up[i];
    oracle_matmul_batched(L->down.bytes, L->down.dtype, L->down.n, F, gate, seq_len, proj);
    for (int64_t i = 0; i < seq_len * E; i++) x[i] += proj[i];
  }
  if (rc == 0) {
    rms_norm_rows_f32(x + (seq_len - 1) * E, m->output_norm, 1, E, c->rms_eps, normed);
    oracle_matmul_batched(m->output.bytes, m->output.dtype, m->output.n, E, normed, 1, logits);
  }
  free(x); free(normed); free(q); free(kk); free(vv); free(attn); free(proj); free(gate); free(up);
  return rc;
}

/* ------------------------------------------------------------------------ */
/* fp64 forward over the bit-exact dequantised weights                       */
/* ------------------------------------------------------------------------ */
static void matvec_f64(const OTensor* w, const double* x, int64_t m, int64_t k, double* out) {
  int bs = oracle_block_size(w->dtype), ts = oracle_type_size(w->dtype);
  int64_t row_bytes = (k / bs) * ts;
  int64_t n = w->n;
#pragma omp parallel
  {
    float* wf = (float*)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(dynamic, 16)
    for (int64_t r = 0; r < n; r++) {
      oracle_dequantize(w->bytes + r * row_bytes, w->dtype, k, wf);
      for (int64_t t = 0; t < m; t++) {
        const double* xt = x + t * k;
        double acc = 0.0;
        for (int64_t c2 = 0; c2 < k; c2++) acc += (double)wf[c2] * xt[c2];
        out[t * n + r] = acc;
      }
    }
    free(wf);
  }
}

static void rms_norm_f64(const double* x, const float* w, int64_t rows, int dim, float eps, double* out) {
  for (int64_t r = 0; r < rows; r++) {
    const double* xi = x + r * dim;
    double ss = 0.0;
    for (int i = 0; i < dim; i++) ss += xi[i] * xi[i];
    double inv = 1.0 / sqrt(ss / (double)dim + (double)eps);
    for (int i = 0; i < dim; i++) out[r * dim + i] = xi[i] * inv * (double)w[i];
  }
}

static void rope_f64(double* v, int nheads, int hd, const float* cs, const float* sn) {
  int half = hd / 2;
  for (int h = 0; h < nheads; h++) {
    double* b = v + (int64_t)h * hd;
    for (int j = 0; j < half; j++) {
      double x0 = b[j], x1 = b[half + j];
      b[j] = x0 * (double)cs[j] - x1 * (double)sn[j];
      b[half + j] = x1 * (double)cs[j] + x0 * (double)sn[j];
    }
  }
}

/* f32 -> f16 -> f32 rounding (round to nearest even), via F16C */
__attribute__((target("f16c"))) static inline double round_f16(double v) {
  __m128 f = _mm_set_ss((float)v);
  __m128i h = _mm_cvtps_ph(f, _MM_FROUND_TO_NEAREST_INT);
  return (double)_mm_cvtss_f32(_mm_cvtph_ps(h));
}

int oracle_forward_f64(void* p, const uint32_t* tokens, int64_t seq_len, int64_t start_pos,
                       int kv_f16, double* logits) {
  OModel* m = (OModel*)p;
  const OracleConfig* c = &m->c;
  int E = c->n_embd, H = c->n_heads, KV = c->n_kv_heads, hd = c->head_dim, half = hd / 2;
  int F = c->n_ff;
  if (seq_len <= 0) return -1;
  double* x = (double*)calloc((size_t)(seq_len * E), sizeof(double));
  float* row = (float*)malloc(sizeof(float) * E);
  for (int64_t t = 0; t < seq_len; t++) {
    if (get_row_f32(&m->tok_embd, tokens[t], row) != 0) { free(x); free(row); return -2; }
    for (int i = 0; i < E; i++) x[t * E + i] = row[i];
  }
  free(row);
  double* normed = (double*)malloc(sizeof(double) * seq_len * E);
  double* q = (double*)malloc(sizeof(double) * seq_len * H * hd);
  double* kk = (double*)malloc(sizeof(double) * seq_len * KV * hd);
  double* vv = (double*)malloc(sizeof(double) * seq_len * KV * hd);
  double* attn = (double*)malloc(sizeof(double) * seq_len * H * hd);
  double* proj = (double*)malloc(sizeof(double) * seq_len * E);
  double* gate = (double*)malloc(sizeof(double) * seq_len * F);
  double* up = (double*)malloc(sizeof(double) * seq_len * F);
  int rc = 0;
  for (int l = 0; l < c->n_layers && rc == 0; l++) {
    OLayer* L = &m->layers[l];
    if (L->len64 + seq_len > m->cap) { rc = -3; break; }
    rms_norm_f64(x, L->attn_norm, seq_len, E, c->rms_eps, normed);
    matvec_f64(&L->q, normed, seq_len, E, q);
    matvec_f64(&L->k, normed, seq_len, E, kk);
    matvec_f64(&L->v, normed, seq_len, E, vv);
    for (int64_t s = 0; s < seq_len; s++) {
      if (L->q_bias) for (int i = 0; i < H * hd; i++) q[s * H * hd + i] += L->q_bias[i];
      if (L->k_bias) for (int i = 0; i < KV * hd; i++) kk[s * KV * hd + i] += L->k_bias[i];
      if (L->v_bias) for (int i = 0; i < KV * hd; i++) vv[s * KV * hd + i] += L->v_bias[i];
      int64_t pos = start_pos + s < 8191 ? start_pos + s : 8191;
      rope_f64(q + s * H * hd, H, hd, m->rope_cos + pos * half, m->rope_sin + pos * half);
      rope_f64(kk + s * KV * hd, KV, hd, m->rope_cos + pos * half, m->rope_sin + pos * half);
    }
    for (int64_t i = 0; i < seq_len * KV * hd; i++) {
      L->kc64[L->len64 * KV * hd + i] = kv_f16 ? round_f16(kk[i]) : kk[i];
      L->vc64[L->len64 * KV * hd + i] = kv_f16 ? round_f16(vv[i]) : vv[i];
    }
    L->len64 += seq_len;
    int64_t total_seq = L->len64;
    int gqa = H / KV;
    double scale = 1.0 / sqrt((double)hd);
    memset(attn, 0, sizeof(double) * seq_len * H * hd);
    for (int64_t s = 0; s < seq_len; s++) {
      int64_t valid_t = start_pos + s + 1 < total_seq ? start_pos + s + 1 : total_seq;
#pragma omp parallel for schedule(static)
      for (int h = 0; h < H; h++) {
        int kh = h / gqa;
        const double* qh = q + (s * H + h) * hd;
        double* oh = attn + (s * H + h) * hd;
        double* scores = (double*)malloc(sizeof(double) * (size_t)valid_t);
        double maxs = -INFINITY;
        for (int64_t t = 0; t < valid_t; t++) {
          const double* kt = L->kc64 + (t * KV + kh) * hd;
          double acc = 0.0;
          for (int i = 0; i < hd; i++) acc += qh[i] * kt[i];
          scores[t] = acc * scale;
          if (scores[t] > maxs) maxs = scores[t];
        }
        double sum = 0.0;
        for (int64_t t = 0; t < valid_t; t++) { scores[t] = exp(scores[t] - maxs); sum += scores[t]; }
        double inv_sum = 1.0 / (sum > 1e-12 ? sum : 1e-12);
        for (int64_t t = 0; t < valid_t; t++) {
          const double* vt = L->vc64 + (t * KV + kh) * hd;
          double a = scores[t] * inv_sum;
          for (int i = 0; i < hd; i++) oh[i] += a * vt[i];
        }
        free(scores);
      }
    }
    matvec_f64(&L->o, attn, seq_len, H * hd, proj);
    for (int64_t i = 0; i < seq_len * E; i++) x[i] += proj[i];
    rms_norm_f64(x, L->ffn_norm, seq_len, E, c->rms_eps, normed);
    matvec_f64(&L->gate, normed, seq_len, E, gate);
    matvec_f64(&L->up, normed, seq_len, E, up);
    for (int64_t i = 0; i < seq_len * F; i++) gate[i] = gate[i] / (1.0 + exp(-gate[i])) * up[i];
    matvec_f64(&L->down, gate, seq_len, F, proj);
    for (int64_t i = 0; i < seq_len * E; i++) x[i] += proj[i];
  }
  if (rc == 0) {
    rms_norm_f64(x + (seq_len - 1) * E, m->output_norm, 1, E, c->rms_eps, normed);
    matvec_f64(&m->output, normed, 1, E, logits);
  }
  free(x); free(normed); free(q); free(kk); free(vv); free(attn); free(proj); free(gate); free(up);
  return rc;
}

/* ------------------------------------------------------------------------- */
/* SelfMadeSampler (inference.rs:1600-1681), restated: xorshift64 state,      */
/* greedy first-max at temperature <= 1e-5, else candidates within           */
/* 14 * temperature of the max logit, p = exp((v - max) / T) summed in index */
/* order, sorted by p descending (the reference's unstable sort leaves ties  */
/* unordered; here ties go by index), the shortest prefix reaching           */
/* top_p * sum, and r = u * min(cum, sum) walked through the prefix.         */
/* Returns the token; *drew = 1 when the random number was consumed.        */
/* ------------------------------------------------------------------------- */
typedef struct { uint32_t id; float p; } OCand;

static int ocand_cmp(const void* a, const void* b) {
  const OCand* x = (const OCand*)a;
  const OCand* y = (const OCand*)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return x->id < y->id ? -1 : x->id > y->id ? 1 : 0;
}

float oracle_xorshift_f32(uint64_t* state) {
  uint64_t x = *state;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *state = x;
  return (float)(uint32_t)(x >> 40) / (float)(1u << 24);
}

uint32_t oracle_sample(const float* logits, int64_t n, float temperature, float top_p, uint64_t* state,
                       int* drew) {
  *drew = 0;
  if (temperature <= 1e-5f) {
    int64_t best = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < n; i++)
      if (logits[i] > bv) { bv = logits[i]; best = i; }
    return (uint32_t)best;
  }
  const float inv_temp = 1.0f / temperature;
  float max_logit = -INFINITY;
  for (int64_t i = 0; i < n; i++)
    if (logits[i] > max_logit) max_logit = logits[i];
  const float cutoff = max_logit - 14.0f * temperature;
  OCand* c = (OCand*)malloc(sizeof(OCand) * (size_t)(n > 0 ? n : 1));
  int64_t nc = 0;
  float sum_prob = 0.0f;
  for (int64_t i = 0; i < n; i++) {
    if (logits[i] >= cutoff) {
      const float p = expf((logits[i] - max_logit) * inv_temp);
      c[nc].id = (uint32_t)i;
      c[nc].p = p;
      nc++;
      sum_prob += p;
    }
  }
  if (nc == 0 || sum_prob <= 0.0f) {
    free(c);
    return 0;
  }
  qsort(c, (size_t)nc, sizeof(OCand), ocand_cmp);
  const float target = sum_prob * top_p;
  float cum = 0.0f;
  int64_t keep = nc;
  for (int64_t i = 0; i < nc; i++) {
    cum += c[i].p;
    if (cum >= target) { keep = i + 1; break; }
  }
  *drew = 1;
  const float r = oracle_xorshift_f32(state) * (cum < sum_prob ? cum : sum_prob);
  float acc = 0.0f;
  uint32_t tok = c[0].id;
  for (int64_t i = 0; i < keep; i++) {
    acc += c[i].p;
    if (r <= acc) { tok = c[i].id; break; }
  }
  free(c);
  return tok;
}

/* ------------------------------------------------------------------------- */
/* Gated DeltaNet mixer core of Qwen35Mixer::GatedDeltaNet, restated         */
/* (inference.rs:2296-2374 with ssm_head_step_avx2 :1535-1583, silu /        */
/* sigmoid / softplus :1481-1499, l2_norm_inplace :1525-1532): causal        */
/* convolution with state + SiLU, L2 norm of q and k per head, per value     */
/* head the state update and output, RMS norm * ssm_norm * silu(z), token    */
/* by token.  Dot products are plain sequential f32 sums (the reference's    */
/* AVX2 lane order differs by rounding only).                                */
/* ------------------------------------------------------------------------- */
static float o_silu(float x) { return x / (1.0f + expf(-x)); }
static float o_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
static float o_softplus(float x) { return x > 20.0f ? x : x < -20.0f ? expf(x) : logf(1.0f + expf(x)); }

int oracle_gdn_step(int n_k, int n_v, int d_k, int d_v, int K, float eps, int n_tokens, const float* qkv,
                    const float* z, const float* alpha, const float* beta, const float* conv_w,
                    const float* ssm_a, const float* dt_bias, const float* ssm_norm, float* conv_state,
                    float* S, float* y) {
  const int q_dim = n_k * d_k, channels = 2 * q_dim + n_v * d_v, hist = K - 1, vdim = n_v * d_v;
  const float scale = 1.0f / sqrtf((float)d_k);
  float* c = (float*)malloc(sizeof(float) * (size_t)channels);
  if (!c) return 1;
  for (int t = 0; t < n_tokens; t++) {
    const float* x = qkv + (size_t)t * channels;
    for (int ch = 0; ch < channels; ch++) {
      float* st = conv_state + (size_t)ch * hist;
      const float* w = conv_w + (size_t)ch * K;
      float acc = 0.0f;
      for (int k = 0; k < hist; k++) acc += st[k] * w[k];
      acc += x[ch] * w[hist];
      c[ch] = o_silu(acc);
      for (int k = 0; k + 1 < hist; k++) st[k] = st[k + 1];
      if (hist > 0) st[hist - 1] = x[ch];
    }
    for (int h = 0; h < 2 * n_k; h++) {  /* q heads then k heads */
      float* v = c + (size_t)h * d_k;
      float ss = 0.0f;
      for (int i = 0; i < d_k; i++) ss += v[i] * v[i];
      const float inv = 1.0f / sqrtf(ss + eps);
      for (int i = 0; i < d_k; i++) v[i] *= inv;
    }
    for (int vh = 0; vh < n_v; vh++) {
      const int kh = vh % n_k;
      const float* q = c + (size_t)kh * d_k;
      const float* kk = c + (size_t)q_dim + (size_t)kh * d_k;
      const float* vv = c + (size_t)2 * q_dim + (size_t)vh * d_v;
      const float b = o_sigmoid(beta[(size_t)t * n_v + vh]);
      const float g = expf(o_softplus(alpha[(size_t)t * n_v + vh] + dt_bias[vh]) * ssm_a[vh]);
      float* out = y + (size_t)t * vdim + (size_t)vh * d_v;
      for (int i = 0; i < d_v; i++) {
        float* row = S + ((size_t)vh * d_v + i) * d_k;
        float sk = 0.0f;
        for (int j = 0; j < d_k; j++) sk += row[j] * kk[j];
        const float d = (vv[i] - g * sk) * b;
        float o = 0.0f;
        for (int j = 0; j < d_k; j++) {
          row[j] = fmaf(d, kk[j], g * row[j]);
          o += row[j] * q[j];
        }
        out[i] = o * scale;
      }
      float ss = 0.0f;
      for (int i = 0; i < d_v; i++) ss += out[i] * out[i];
      const float inv = 1.0f / sqrtf(ss / (float)d_v + eps);
      const float* zz = z + (size_t)t * vdim + (size_t)vh * d_v;
      for (int i = 0; i < d_v; i++) out[i] = out[i] * inv * ssm_norm[i] * o_silu(zz[i]);
    }
  }
  free(c);
  return 0;
}
