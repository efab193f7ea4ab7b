/*
 * gguf_oracle.c -- CPU oracle for the GGUF dequant-GEMV decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and the CPU-baseline
 * leg of bench.py do, and only as the checker / the timed CPU reference.
 *
 * It is a C restatement of the reference engine's CPU path
 * (roblar658/huggingface-Local-LLM-UI, src/inference.rs), function by
 * function, with each function citing the lines it follows:
 *   - the GGML block formats and their f32 dequantisation (bit-exact spec),
 *   - the activation quantisers (Q8_K / Q8_0) and the AVX2/FMA integer dot
 *     kernels, with the same intrinsic sequence, and the Rayon row-chunked
 *     matvec driver (OpenMP here, chunks of 64 rows),
 *   - RMSNorm / SiLU / NeoX RoPE tables / GQA attention and the Llama
 *     block loop of StandardNativeEngine::forward.
 * It adds an fp64 path (dequantised-exact weights, f64 accumulation, KV
 * cache optionally rounded to f16) that gates the GPU results by rel-L2.
 *
 * Parity pinning: the reference is Rust and Windows-only and cannot be
 * compiled in this environment, and it ships no tests or golden vectors.
 * The dequantisers here are pinned bit-for-bit against gguf-py 0.19.0
 * (llama.cpp's Python decoder of the same block formats, which performs the
 * same f32 operation sequence) by tests/golden/make_golden.py.  Parity
 * unpinned beyond dequantisation: no output of the reference itself checks
 * the quantisers, the dot kernels or the matvec driver restated here; the
 * GPU's matvec, layer and logits numerics are gated against the fp64 path
 * below (rel-L2 <= 1e-3), which is exact by construction.
 *
 * Build: oracle/Makefile (gcc -O3 -mavx2 -mfma -ffp-contract=off -fopenmp).
 * -ffp-contract=off matters: Rust never fuses a*b-c into an FMA, gcc would.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK_K 256
#define QK8_0 32

/* GgmlDType ids, block sizes and type sizes: inference.rs:116-185 */
enum {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7,
  T_Q8_0 = 8, T_Q8_1 = 9, T_Q2K = 10, T_Q3K = 11, T_Q4K = 12, T_Q5K = 13,
  T_Q6K = 14, T_Q8K = 15, T_BF16 = 30
};

int oracle_block_size(int t) {
  switch (t) {
    case T_F32: case T_F16: case T_BF16: return 1;
    case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: case T_Q8_1: return 32;
    case T_Q2K: case T_Q3K: case T_Q4K: case T_Q5K: case T_Q6K: case T_Q8K: return 256;
    default: return 0;
  }
}

int oracle_type_size(int t) {
  switch (t) {
    case T_F32: return 4;
    case T_F16: case T_BF16: return 2;
    case T_Q4_0: return 18; case T_Q4_1: return 20; case T_Q5_0: return 22;
    case T_Q5_1: return 24; case T_Q8_0: return 34; case T_Q8_1: return 36;
    case T_Q2K: return 84; case T_Q3K: return 110; case T_Q4K: return 144;
    case T_Q5K: return 176; case T_Q6K: return 210; case T_Q8K: return 292;
    default: return 0;
  }
}

/* f16_to_f32: inference.rs:868-890.  Bit construction, subnormals
 * renormalised by shifting the mantissa, inf/NaN keep their payload. */
static inline float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x03ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      uint32_t e = 127 - 14;
      while ((man & 0x0400u) == 0) { man <<= 1; e -= 1; }
      man &= 0x03ffu;
      bits = sign | (e << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

float oracle_f16_to_f32(uint16_t h) { return f16_bits_to_f32(h); }

/* bf16_to_f32: inference.rs:892-895 */
static inline float bf16_bits_to_f32(uint16_t b) {
  uint32_t bits = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* decode_q4k_scales: inference.rs:988-1000.  12 packed bytes -> eight
 * 6-bit scales and eight 6-bit mins. */
void oracle_decode_q4k_scales(const uint8_t* s, uint8_t* sc, uint8_t* m) {
  for (int j = 0; j < 4; j++) {
    sc[j] = s[j] & 63;
    m[j] = s[j + 4] & 63;
  }
  for (int j = 4; j < 8; j++) {
    sc[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
    m[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* dequantize_slice: inference.rs:1347-1474.  `out_len` elements.  The f32
 * operation order of every branch is the reference's (no contraction). */
int oracle_dequantize(const uint8_t* bytes, int dtype, int64_t out_len, float* out) {
  switch (dtype) {
    case T_F32:
      for (int64_t i = 0; i < out_len; i++) memcpy(&out[i], bytes + 4 * i, 4);
      return 0;
    case T_F16:
      for (int64_t i = 0; i < out_len; i++) out[i] = f16_bits_to_f32(rd_u16(bytes + 2 * i));
      return 0;
    case T_BF16:
      for (int64_t i = 0; i < out_len; i++) out[i] = bf16_bits_to_f32(rd_u16(bytes + 2 * i));
      return 0;
    case T_Q4K: {
      int64_t nb = out_len / QK_K;
      for (int64_t blk = 0; blk < nb; blk++) {
        const uint8_t* b = bytes + blk * 144;
        float d = f16_bits_to_f32(rd_u16(b));
        float dmin = f16_bits_to_f32(rd_u16(b + 2));
        uint8_t sc[8], m[8];
        oracle_decode_q4k_scales(b + 4, sc, m);
        const uint8_t* qs = b + 16;
        float* dst = out + blk * QK_K;
        for (int chunk = 0; chunk < 4; chunk++) {
          int is = chunk * 2;
          float d1 = d * (float)sc[is];
          float m1 = dmin * (float)m[is];
          float d2 = d * (float)sc[is + 1];
          float m2 = dmin * (float)m[is + 1];
          const uint8_t* q = qs + chunk * 32;
          for (int l = 0; l < 32; l++) {
            dst[chunk * 64 + l] = d1 * (float)(q[l] & 0x0F) - m1;
            dst[chunk * 64 + 32 + l] = d2 * (float)(q[l] >> 4) - m2;
          }
        }
      }
      return 0;
    }
    case T_Q6K: {
      int64_t nb = out_len / QK_K;
      for (int64_t blk = 0; blk < nb; blk++) {
        const uint8_t* b = bytes + blk * 210;
        const uint8_t* ql = b;
        const uint8_t* qh = b + 128;
        const int8_t* sc = (const int8_t*)(b + 192);
        float d = f16_bits_to_f32(rd_u16(b + 208));
        float* dst = out + blk * QK_K;
        for (int half = 0; half < 2; half++) {
          const uint8_t* qlh = ql + half * 64;
          const uint8_t* qhh = qh + half * 32;
          const int8_t* sch = sc + half * 8;
          float* dh = dst + half * 128;
          for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int8_t q1 = (int8_t)((qlh[l] & 0x0F) | (((qhh[l] >> 0) & 3) << 4)) - 32;
            int8_t q2 = (int8_t)((qlh[l + 32] & 0x0F) | (((qhh[l] >> 2) & 3) << 4)) - 32;
            int8_t q3 = (int8_t)((qlh[l] >> 4) | (((qhh[l] >> 4) & 3) << 4)) - 32;
            int8_t q4 = (int8_t)((qlh[l + 32] >> 4) | (((qhh[l] >> 6) & 3) << 4)) - 32;
            /* `d * sc * q` evaluates left to right: (d*sc)*q */
            dh[l] = d * (float)sch[is] * (float)q1;
            dh[l + 32] = d * (float)sch[is + 2] * (float)q2;
            dh[l + 64] = d * (float)sch[is + 4] * (float)q3;
            dh[l + 96] = d * (float)sch[is + 6] * (float)q4;
          }
        }
      }
      return 0;
    }
    case T_Q5K: {
      int64_t nb = out_len / QK_K;
      for (int64_t blk = 0; blk < nb; blk++) {
        const uint8_t* b = bytes + blk * 176;
        float d = f16_bits_to_f32(rd_u16(b));
        float dmin = f16_bits_to_f32(rd_u16(b + 2));
        uint8_t sc[8], m[8];
        oracle_decode_q4k_scales(b + 4, sc, m);
        const uint8_t* qh = b + 16;
        const uint8_t* qs = b + 48;
        float* dst = out + blk * QK_K;
        uint8_t u1 = 1, u2 = 2;
        for (int chunk = 0; chunk < 4; chunk++) {
          int is = chunk * 2;
          float d1 = d * (float)sc[is];
          float m1 = dmin * (float)m[is];
          float d2 = d * (float)sc[is + 1];
          float m2 = dmin * (float)m[is + 1];
          const uint8_t* q = qs + chunk * 32;
          for (int l = 0; l < 32; l++) {
            uint8_t v0 = (uint8_t)((q[l] & 0x0F) | ((qh[l] & u1) ? 16 : 0));
            uint8_t v1 = (uint8_t)((q[l] >> 4) | ((qh[l] & u2) ? 16 : 0));
            dst[chunk * 64 + l] = d1 * (float)v0 - m1;
            dst[chunk * 64 + 32 + l] = d2 * (float)v1 - m2;
          }
          u1 = (uint8_t)(u1 << 2);
          u2 = (uint8_t)(u2 << 2);
        }
      }
      return 0;
    }
    case T_Q8_0: {
      int64_t nb = out_len / QK8_0;
      for (int64_t blk = 0; blk < nb; blk++) {
        const uint8_t* b = bytes + blk * 34;
        float d = f16_bits_to_f32(rd_u16(b));
        for (int i = 0; i < 32; i++) out[blk * 32 + i] = d * (float)(int8_t)b[2 + i];
      }
      return 0;
    }
    case T_Q4_0: {
      int64_t nb = out_len / QK8_0;
      for (int64_t blk = 0; blk < nb; blk++) {
        const uint8_t* b = bytes + blk * 18;
        float d = f16_bits_to_f32(rd_u16(b));
        for (int i = 0; i < 16; i++) {
          out[blk * 32 + i] = d * (float)((int)(b[2 + i] & 0x0F) - 8);
          out[blk * 32 + i + 16] = d * (float)((int)(b[2 + i] >> 4) - 8);
        }
      }
      return 0;
    }
    default:
      return -1; /* the reference bails for other types */
  }
}

/* ------------------------------------------------------------------------ */
/* Activation quantisers: inference.rs:897-985                               */
/* ------------------------------------------------------------------------ */
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } BlockQ8K;
typedef struct { float d; int8_t qs[32]; } BlockQ8_0;

/* Rust's f32::round: half away from zero == C roundf.  The clamp + `as i8`
 * saturating cast are reproduced; a NaN lands on 0 as Rust's cast does. */
static inline int8_t round_clamp_i8(float v) {
  float r = roundf(v);
  if (r != r) return 0;
  if (r < -127.0f) r = -127.0f;
  if (r > 127.0f) r = 127.0f;
  return (int8_t)r;
}

/* quantize_row_q8_k: inference.rs:933-962.  Signed max, iscale=-127/max. */
void oracle_quantize_row_q8_k(const float* x, int64_t k, BlockQ8K* out) {
  int64_t nb = k / QK_K;
  for (int64_t bi = 0; bi < nb; bi++) {
    const float* src = x + bi * QK_K;
    BlockQ8K* blk = &out[bi];
    float max_abs = 0.0f, max_val = 0.0f;
    for (int i = 0; i < QK_K; i++) {
      float a = fabsf(src[i]);
      if (a > max_abs) { max_abs = a; max_val = src[i]; }
    }
    if (max_abs == 0.0f) { memset(blk, 0, sizeof(*blk)); continue; }
    float iscale = -127.0f / max_val;
    blk->d = 1.0f / iscale;
    for (int j = 0; j < 16; j++) {
      int16_t bsum = 0;
      for (int l = 0; l < 16; l++) {
        int8_t q = round_clamp_i8(src[j * 16 + l] * iscale);
        blk->qs[j * 16 + l] = q;
        bsum = (int16_t)(bsum + q);
      }
      blk->bsums[j] = bsum;
    }
  }
}

/* quantize_row_q8_0: inference.rs:964-985.  d = max|x|/127, q=round(x/d). */
void oracle_quantize_row_q8_0(const float* x, int64_t k, BlockQ8_0* out) {
  int64_t nb = k / QK8_0;
  for (int64_t bi = 0; bi < nb; bi++) {
    const float* src = x + bi * QK8_0;
    BlockQ8_0* blk = &out[bi];
    float max_abs = 0.0f;
    for (int i = 0; i < 32; i++) { float a = fabsf(src[i]); if (a > max_abs) max_abs = a; }
    if (max_abs == 0.0f) { memset(blk, 0, sizeof(*blk)); continue; }
    float d = max_abs / 127.0f;
    float id = 1.0f / d;
    blk->d = d;
    for (int i = 0; i < 32; i++) blk->qs[i] = round_clamp_i8(src[i] * id);
  }
}

/* ------------------------------------------------------------------------ */
/* AVX2 helpers and dot kernels: inference.rs:1002-1344                      */
/* ------------------------------------------------------------------------ */
__attribute__((target("avx2,fma"))) static inline int hsum_epi32(__m256i v) {
  __m128i hi128 = _mm256_extracti128_si256(v, 1);
  __m128i lo128 = _mm256_castsi256_si128(v);
  __m128i s128 = _mm_add_epi32(lo128, hi128);
  __m128i hi64 = _mm_unpackhi_epi64(s128, s128);
  __m128i s64 = _mm_add_epi32(s128, hi64);
  __m128i hi32 = _mm_shuffle_epi32(s64, 0x55);
  return _mm_cvtsi128_si32(_mm_add_epi32(s64, hi32));
}

__attribute__((target("avx2,fma"))) static inline int hsum_128_epi32(__m128i v) {
  __m128i hi64 = _mm_unpackhi_epi64(v, v);
  __m128i s64 = _mm_add_epi32(v, hi64);
  __m128i hi32 = _mm_shuffle_epi32(s64, 0x55);
  return _mm_cvtsi128_si32(_mm_add_epi32(s64, hi32));
}

__attribute__((target("avx2,fma"))) static inline float hsum_ps(__m256 v) {
  __m128 hi128 = _mm256_extractf128_ps(v, 1);
  __m128 lo128 = _mm256_castps256_ps128(v);
  __m128 s128 = _mm_add_ps(lo128, hi128);
  __m128 shuf = _mm_movehdup_ps(s128);
  __m128 sums = _mm_add_ps(s128, shuf);
  __m128 shuf2 = _mm_movehl_ps(sums, sums);
  return _mm_cvtss_f32(_mm_add_ss(sums, shuf2));
}

/* vec_dot_q4k_q8k_avx2: inference.rs:1031-1078 */
__attribute__((target("avx2,fma")))
static float vec_dot_q4k_q8k(const uint8_t* w, const BlockQ8K* xb, int64_t nb) {
  const __m256i mask_0f = _mm256_set1_epi8(0x0F);
  const __m256i ones_16 = _mm256_set1_epi16(1);
  float total = 0.0f;
  for (int64_t bi = 0; bi < nb; bi++) {
    const BlockQ8K* x = &xb[bi];
    if (x->d == 0.0f) continue;
    const uint8_t* b = w + bi * 144;
    float d = f16_bits_to_f32(rd_u16(b)) * x->d;
    float dmin = f16_bits_to_f32(rd_u16(b + 2)) * x->d;
    uint8_t sc[8], m[8];
    oracle_decode_q4k_scales(b + 4, sc, m);
    const uint8_t* qs = b + 16;
    int isum = 0, msum = 0;
    for (int chunk = 0; chunk < 4; chunk++) {
      int is = chunk * 2;
      __m256i qb = _mm256_loadu_si256((const __m256i*)(qs + chunk * 32));
      __m256i q_lo = _mm256_and_si256(qb, mask_0f);
      __m256i q_hi = _mm256_and_si256(_mm256_srli_epi16(qb, 4), mask_0f);
      __m256i x_lo = _mm256_loadu_si256((const __m256i*)(x->qs + chunk * 64));
      __m256i x_hi = _mm256_loadu_si256((const __m256i*)(x->qs + chunk * 64 + 32));
      __m256i p_lo = _mm256_maddubs_epi16(q_lo, x_lo);
      __m256i p_hi = _mm256_maddubs_epi16(q_hi, x_hi);
      int s_lo = hsum_epi32(_mm256_madd_epi16(p_lo, ones_16));
      int s_hi = hsum_epi32(_mm256_madd_epi16(p_hi, ones_16));
      isum += s_lo * (int)sc[is] + s_hi * (int)sc[is + 1];
      int b_lo = (int)x->bsums[chunk * 4] + (int)x->bsums[chunk * 4 + 1];
      int b_hi = (int)x->bsums[chunk * 4 + 2] + (int)x->bsums[chunk * 4 + 3];
      msum += b_lo * (int)m[is] + b_hi * (int)m[is + 1];
    }
    total += d * (float)isum - dmin * (float)msum;
  }
  return total;
}

/* vec_dot_q6k_q8k_avx2: inference.rs:1083-1184 */
__attribute__((target("avx2,fma")))
static float vec_dot_q6k_q8k(const uint8_t* w, const BlockQ8K* xb, int64_t nb) {
  const __m256i mask_0f = _mm256_set1_epi8(0x0F);
  const __m256i mask_30 = _mm256_set1_epi8(0x30);
  const __m256i ones_16 = _mm256_set1_epi16(1);
  float total = 0.0f;
  for (int64_t bi = 0; bi < nb; bi++) {
    const BlockQ8K* x = &xb[bi];
    if (x->d == 0.0f) continue;
    const uint8_t* b = w + bi * 210;
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = f16_bits_to_f32(rd_u16(b + 208)) * x->d;
    int isum = 0;
    for (int half = 0; half < 2; half++) {
      __m256i ql0 = _mm256_loadu_si256((const __m256i*)(ql + half * 64));
      __m256i ql1 = _mm256_loadu_si256((const __m256i*)(ql + half * 64 + 32));
      __m256i qh0 = _mm256_loadu_si256((const __m256i*)(qh + half * 32));
      __m256i q1 = _mm256_or_si256(_mm256_and_si256(ql0, mask_0f),
                                   _mm256_and_si256(_mm256_slli_epi16(qh0, 4), mask_30));
      __m256i q2 = _mm256_or_si256(_mm256_and_si256(ql1, mask_0f),
                                   _mm256_and_si256(_mm256_slli_epi16(qh0, 2), mask_30));
      __m256i q3 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql0, 4), mask_0f),
                                   _mm256_and_si256(qh0, mask_30));
      __m256i q4 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql1, 4), mask_0f),
                                   _mm256_and_si256(_mm256_srli_epi16(qh0, 2), mask_30));
      const int8_t* xp = x->qs + half * 128;
      __m256i x1 = _mm256_loadu_si256((const __m256i*)(xp));
      __m256i x2 = _mm256_loadu_si256((const __m256i*)(xp + 32));
      __m256i x3 = _mm256_loadu_si256((const __m256i*)(xp + 64));
      __m256i x4 = _mm256_loadu_si256((const __m256i*)(xp + 96));
      __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(q1, x1), ones_16);
      __m256i p2 = _mm256_madd_epi16(_mm256_maddubs_epi16(q2, x2), ones_16);
      __m256i p3 = _mm256_madd_epi16(_mm256_maddubs_epi16(q3, x3), ones_16);
      __m256i p4 = _mm256_madd_epi16(_mm256_maddubs_epi16(q4, x4), ones_16);
      int g = half * 8;
      const int16_t* bs = x->bsums;
      int d0 = hsum_128_epi32(_mm256_castsi256_si128(p1)) - 32 * (int)bs[g];
      int d1 = hsum_128_epi32(_mm256_extracti128_si256(p1, 1)) - 32 * (int)bs[g + 1];
      int d2 = hsum_128_epi32(_mm256_castsi256_si128(p2)) - 32 * (int)bs[g + 2];
      int d3 = hsum_128_epi32(_mm256_extracti128_si256(p2, 1)) - 32 * (int)bs[g + 3];
      int d4 = hsum_128_epi32(_mm256_castsi256_si128(p3)) - 32 * (int)bs[g + 4];
      int d5 = hsum_128_epi32(_mm256_extracti128_si256(p3, 1)) - 32 * (int)bs[g + 5];
      int d6 = hsum_128_epi32(_mm256_castsi256_si128(p4)) - 32 * (int)bs[g + 6];
      int d7 = hsum_128_epi32(_mm256_extracti128_si256(p4, 1)) - 32 * (int)bs[g + 7];
      isum += d0 * sc[g] + d1 * sc[g + 1] + d2 * sc[g + 2] + d3 * sc[g + 3] +
              d4 * sc[g + 4] + d5 * sc[g + 5] + d6 * sc[g + 6] + d7 * sc[g + 7];
    }
    total += d * (float)isum;
  }
  return total;
}

/* vec_dot_q5k_q8k_avx2 (scalar in the reference): inference.rs:1189-1232 */
static float vec_dot_q5k_q8k(const uint8_t* w, const BlockQ8K* xb, int64_t nb) {
  float total = 0.0f;
  for (int64_t bi = 0; bi < nb; bi++) {
    const BlockQ8K* x = &xb[bi];
    if (x->d == 0.0f) continue;
    const uint8_t* b = w + bi * 176;
    float d = f16_bits_to_f32(rd_u16(b)) * x->d;
    float dmin = f16_bits_to_f32(rd_u16(b + 2)) * x->d;
    uint8_t sc[8], m[8];
    oracle_decode_q4k_scales(b + 4, sc, m);
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    int isum = 0, msum = 0;
    uint8_t u1 = 1, u2 = 2;
    for (int chunk = 0; chunk < 4; chunk++) {
      int is = chunk * 2;
      const uint8_t* q = qs + chunk * 32;
      const int8_t* x0 = x->qs + chunk * 64;
      const int8_t* x1 = x->qs + chunk * 64 + 32;
      int s0 = 0, s1 = 0;
      for (int l = 0; l < 32; l++) {
        int v0 = (q[l] & 0x0F) | ((qh[l] & u1) ? 16 : 0);
        int v1 = (q[l] >> 4) | ((qh[l] & u2) ? 16 : 0);
        s0 += v0 * x0[l];
        s1 += v1 * x1[l];
      }
      isum += s0 * (int)sc[is] + s1 * (int)sc[is + 1];
      int b_lo = (int)x->bsums[chunk * 4] + (int)x->bsums[chunk * 4 + 1];
      int b_hi = (int)x->bsums[chunk * 4 + 2] + (int)x->bsums[chunk * 4 + 3];
      msum += b_lo * (int)m[is] + b_hi * (int)m[is + 1];
      u1 = (uint8_t)(u1 << 2);
      u2 = (uint8_t)(u2 << 2);
    }
    total += d * (float)isum - dmin * (float)msum;
  }
  return total;
}

/* vec_dot_q8_0_q8_0_avx2: inference.rs:1236-1256 (sign trick for maddubs) */
__attribute__((target("avx2,fma")))
static float vec_dot_q8_0_q8_0(const uint8_t* w, const BlockQ8_0* xb, int64_t nb) {
  const __m256i ones_16 = _mm256_set1_epi16(1);
  float total = 0.0f;
  for (int64_t bi = 0; bi < nb; bi++) {
    const BlockQ8_0* x = &xb[bi];
    if (x->d == 0.0f) continue;
    const uint8_t* b = w + bi * 34;
    float d = f16_bits_to_f32(rd_u16(b)) * x->d;
    __m256i wv = _mm256_loadu_si256((const __m256i*)(b + 2));
    __m256i xv = _mm256_loadu_si256((const __m256i*)(x->qs));
    __m256i w_abs = _mm256_abs_epi8(wv);
    __m256i x_signed = _mm256_sign_epi8(xv, wv);
    __m256i p16 = _mm256_maddubs_epi16(w_abs, x_signed);
    int isum = hsum_epi32(_mm256_madd_epi16(p16, ones_16));
    total += d * (float)isum;
  }
  return total;
}

/* vec_dot_q4_0_q8_0_avx2 (scalar in the reference): inference.rs:1260-1278 */
static float vec_dot_q4_0_q8_0(const uint8_t* w, const BlockQ8_0* xb, int64_t nb) {
  float total = 0.0f;
  for (int64_t bi = 0; bi < nb; bi++) {
    const BlockQ8_0* x = &xb[bi];
    if (x->d == 0.0f) continue;
    const uint8_t* b = w + bi * 18;
    float d = f16_bits_to_f32(rd_u16(b)) * x->d;
    int isum = 0;
    for (int i = 0; i < 16; i++) {
      int v0 = (int)(b[2 + i] & 0x0F) - 8;
      int v1 = (int)(b[2 + i] >> 4) - 8;
      isum += v0 * x->qs[i] + v1 * x->qs[i + 16];
    }
    total += d * (float)isum;
  }
  return total;
}

/* vec_dot_f32_avx2: inference.rs:1282-1313 (2 x 8-wide accumulators) */
__attribute__((target("avx2,fma")))
float oracle_vec_dot_f32(const float* a, const float* b, int64_t n) {
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  int64_t i = 0;
  while (i + 16 <= n) {
    acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), acc1);
    i += 16;
  }
  acc0 = _mm256_add_ps(acc0, acc1);
  while (i + 8 <= n) {
    acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
    i += 8;
  }
  float sum = hsum_ps(acc0);
  while (i < n) { sum += a[i] * b[i]; i++; }
  return sum;
}

/* vec_axpy_f32_avx2: inference.rs:1317-1344 */
__attribute__((target("avx2,fma")))
static void vec_axpy_f32(float* dst, float scale, const float* src, int64_t n) {
  __m256 s = _mm256_set1_ps(scale);
  int64_t i = 0;
  while (i + 16 <= n) {
    __m256 d0 = _mm256_loadu_ps(dst + i), s0 = _mm256_loadu_ps(src + i);
    __m256 d1 = _mm256_loadu_ps(dst + i + 8), s1 = _mm256_loadu_ps(src + i + 8);
    _mm256_storeu_ps(dst + i, _mm256_fmadd_ps(s, s0, d0));
    _mm256_storeu_ps(dst + i + 8, _mm256_fmadd_ps(s, s1, d1));
    i += 16;
  }
  while (i + 8 <= n) {
    _mm256_storeu_ps(dst + i, _mm256_fmadd_ps(s, _mm256_loadu_ps(src + i), _mm256_loadu_ps(dst + i)));
    i += 8;
  }
  while (i < n) { dst[i] += scale * src[i]; i++; }
}

void oracle_axpy_f32(float* dst, float scale, const float* src, int64_t n) {
  vec_axpy_f32(dst, scale, src, n);
}

/* ------------------------------------------------------------------------ */
/* MmapWeight::matmul_batched: inference.rs:589-760.                          */
/* Y[m,n] = X[m,k] * W[n,k]^T.  Quantised-x integer path for K-quants and   */
/* Q8_0/Q4_0; per-row dequant + f32 dot otherwise.  m == 1 splits the n     */
/* outputs into chunks of 64 rows over the thread pool; m > 1 chunks 32     */
/* rows, writes [n][m] and transposes.                                       */
/* ------------------------------------------------------------------------ */
static int g_threads = 0; /* 0: OpenMP default */

void oracle_set_threads(int n) { g_threads = n; }
int oracle_get_max_threads(void) { return omp_get_max_threads(); }

static inline int nthreads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

static float dot_row_kq(int dtype, const uint8_t* row, const BlockQ8K* x, int64_t nb) {
  switch (dtype) {
    case T_Q4K: return vec_dot_q4k_q8k(row, x, nb);
    case T_Q6K: return vec_dot_q6k_q8k(row, x, nb);
    default: return vec_dot_q5k_q8k(row, x, nb);
  }
}

static float dot_row_q80(int dtype, const uint8_t* row, const BlockQ8_0* x, int64_t nb) {
  return dtype == T_Q8_0 ? vec_dot_q8_0_q8_0(row, x, nb) : vec_dot_q4_0_q8_0(row, x, nb);
}

int oracle_matmul_batched(const uint8_t* w, int dtype, int64_t n, int64_t k,
                          const float* x, int64_t m, float* out) {
  int bs = oracle_block_size(dtype), ts = oracle_type_size(dtype);
  if (bs == 0 || k % bs != 0) return -1;
  int64_t row_bytes = (k / bs) * ts;
  int nt = nthreads();
  if (dtype == T_Q4K || dtype == T_Q6K || dtype == T_Q5K) {
    int64_t nb = k / QK_K;
    BlockQ8K* xq = (BlockQ8K*)malloc(sizeof(BlockQ8K) * (size_t)(m * nb));
    for (int64_t t = 0; t < m; t++) oracle_quantize_row_q8_k(x + t * k, k, xq + t * nb);
    if (m == 1) {
      int64_t nchunks = (n + 63) / 64;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
      for (int64_t c = 0; c < nchunks; c++) {
        int64_t end = (c + 1) * 64 < n ? (c + 1) * 64 : n;
        for (int64_t col = c * 64; col < end; col++)
          out[col] = dot_row_kq(dtype, w + col * row_bytes, xq, nb);
      }
    } else {
      float* onm = (float*)malloc(sizeof(float) * (size_t)(n * m));
      int64_t nchunks = (n + 31) / 32;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
      for (int64_t c = 0; c < nchunks; c++) {
        int64_t end = (c + 1) * 32 < n ? (c + 1) * 32 : n;
        for (int64_t col = c * 32; col < end; col++)
          for (int64_t t = 0; t < m; t++)
            onm[col * m + t] = dot_row_kq(dtype, w + col * row_bytes, xq + t * nb, nb);
      }
      for (int64_t t = 0; t < m; t++)
        for (int64_t col = 0; col < n; col++) out[t * n + col] = onm[col * m + t];
      free(onm);
    }
    free(xq);
    return 0;
  }
  if (dtype == T_Q8_0 || dtype == T_Q4_0) {
    int64_t nb = k / QK8_0;
    BlockQ8_0* xq = (BlockQ8_0*)malloc(sizeof(BlockQ8_0) * (size_t)(m * nb));
    for (int64_t t = 0; t < m; t++) oracle_quantize_row_q8_0(x + t * k, k, xq + t * nb);
    if (m == 1) {
      int64_t nchunks = (n + 63) / 64;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
      for (int64_t c = 0; c < nchunks; c++) {
        int64_t end = (c + 1) * 64 < n ? (c + 1) * 64 : n;
        for (int64_t col = c * 64; col < end; col++)
          out[col] = dot_row_q80(dtype, w + col * row_bytes, xq, nb);
      }
    } else {
      float* onm = (float*)malloc(sizeof(float) * (size_t)(n * m));
      int64_t nchunks = (n + 31) / 32;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
      for (int64_t c = 0; c < nchunks; c++) {
        int64_t end = (c + 1) * 32 < n ? (c + 1) * 32 : n;
        for (int64_t col = c * 32; col < end; col++)
          for (int64_t t = 0; t < m; t++)
            onm[col * m + t] = dot_row_q80(dtype, w + col * row_bytes, xq + t * nb, nb);
      }
      for (int64_t t = 0; t < m; t++)
        for (int64_t col = 0; col < n; col++) out[t * n + col] = onm[col * m + t];
      free(onm);
    }
    free(xq);
    return 0;
  }
  /* f32/f16/bf16: per-row dequant then vec_dot_f32 (inference.rs:729-756) */
  {
    float* onm = (float*)malloc(sizeof(float) * (size_t)(n * m));
    int64_t nchunks = (n + 31) / 32;
    int rc = 0;
#pragma omp parallel num_threads(nt)
    {
      float* wf = (float*)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(dynamic, 1)
      for (int64_t c = 0; c < nchunks; c++) {
        int64_t end = (c + 1) * 32 < n ? (c + 1) * 32 : n;
        for (int64_t col = c * 32; col < end; col++) {
          if (oracle_dequantize(w + col * row_bytes, dtype, k, wf) != 0) rc = -1;
          for (int64_t t = 0; t < m; t++) onm[col * m + t] = oracle_vec_dot_f32(wf, x + t * k, k);
        }
      }
      free(wf);
    }
    for (int64_t t = 0; t < m; t++)
      for (int64_t col = 0; col < n; col++) out[t * n + col] = onm[col * m + t];
    free(onm);
    return rc;
  }
}

/* fp64 matvec of the bit-exact dequantised weights: the tolerance oracle.
 * y[t][r] = sum_c (double)dequant(W)[r][c] * (double)x[t][c]. */
int oracle_matmul_f64(const uint8_t* w, int dtype, int64_t n, int64_t k,
                      const float* x, int64_t m, double* out) {
  int bs = oracle_block_size(dtype), ts = oracle_type_size(dtype);
  if (bs == 0 || k % bs != 0) return -1;
  int64_t row_bytes = (k / bs) * ts;
  int rc = 0;
#pragma omp parallel num_threads(nthreads())
  {
    float* wf = (float*)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(dynamic, 16)
    for (int64_t r = 0; r < n; r++) {
      if (oracle_dequantize(w + r * row_bytes, dtype, k, wf) != 0) rc = -1;
      for (int64_t t = 0; t < m; t++) {
        const float* xt = x + t * k;
        double acc = 0.0;
        for (int64_t c = 0; c < k; c++) acc += (double)wf[c] * (double)xt[c];
        out[t * n + r] = acc;
      }
    }
    free(wf);
  }
  return rc;
}
