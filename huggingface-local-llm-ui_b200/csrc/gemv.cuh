// gemv.cuh -- dequantise-and-multiply GEMV for repacked GGUF weights.
//
// y[t][r] = sum_c dequant(W)[r][c] * x[t][c] for t in [0, MT).
//
// Design (HBM-bound integer/byte work; no tensor cores):
//  * Weights stream from HBM as 16-byte vector loads, coalesced across the
//    warp: lane l of a warp reads unit u = l + 32*j of each of its R rows, and
//    the repacked layout puts the 16-byte pieces of consecutive units next to
//    each other.  A unit is 64 weights (Q4_K, Q6_K) or 32 (Q8_0).
//  * The activation x arrives pre-quantised to int16 per 32-element block
//    (quant.cuh) and is staged once per CTA into shared memory with a bulk
//    async copy; all R rows of a lane reuse each shared-memory read.
//  * The inner product is integer: dp2a multiplies two int16 activations by
//    two weight bytes and accumulates in int32.  Q4_K nibbles are masked in
//    place (low nibbles as 0..15, high nibbles as 16*q, shifted after the
//    sum), Q6_K codes are rebuilt from ql/qh as unsigned 0..63 with the -32
//    offset applied through the precomputed 16-element sums.  Per 32-block
//    the int32 partial is scaled once in f32 by d * sub-scale * x-scale.
//  * The grid is persistent (CTAs = SMs x occupancy) and walks row tiles of
//    one or more segments (weights sharing the same x); a segment may pair
//    two weights (gate/up) for a fused SwiGLU epilogue.
#pragma once

#include "quant.cuh"

namespace b2q {

enum : int { kEpiStore = 0, kEpiAdd = 1, kEpiSwiglu = 2 };

// Device view of a repacked weight.
struct WeightDev {
  const uint8_t* qs;    // quant stream [n][S][U][16]
  const uint8_t* aux;   // Q4_K hdr u32 [n][U]; Q6_K scale words u32 [n][U]; Q8_0 d u16 [n][U]
  const uint8_t* aux2;  // Q6_K d u16 [n][nb]
  int dtype, n, k, U, nb;
  int64_t row_qs;       // bytes per row of the quant stream
};

struct GemvSeg {
  WeightDev w;       // weight (gate for SwiGLU)
  WeightDev w2;      // up (SwiGLU only)
  float* y;          // output: y[t * ldy + row]
  int ldy;
  int tile0;         // first global tile of this segment
  int rows_out;      // output rows (n)
};

constexpr int kMaxSegs = 4;

struct GemvArgs {
  GemvSeg seg[kMaxSegs];
  int nseg;
  int tiles_total;
  // quantised activations, tokens [t0, t0 + MT)
  const int16_t* xq;
  const float* xscale;
  const float* xfsum;
  const int32_t* xs16;
  int kpad;
  int t0;
};

// Shared-memory view of the staged activations (MT tokens).
struct SX {
  const int16_t* q;
  const float* scale;
  const float* fsum;
  const int32_t* s16;
  int kpad;
};

__host__ __device__ inline size_t gemv_smem_bytes(int kpad, int mt) {
  return (size_t)mt * kpad * 2 + (size_t)mt * (kpad / 32) * 8 + (size_t)mt * (kpad / 16) * 4;
}

// ---------------------------------------------------------------------------
// Q4_K
// ---------------------------------------------------------------------------
struct FmtQ4K {
  struct Reg { uint4 a, b; uint32_t h; };
  __device__ __forceinline__ static void zero(Reg& r) {
    r.a = make_uint4(0, 0, 0, 0); r.b = r.a; r.h = 0;
  }
  __device__ __forceinline__ static void load(Reg& r, const WeightDev& w, int row, int u, uint64_t pol) {
    const uint8_t* base = w.qs + (int64_t)row * w.row_qs;
    r.a = ldg_stream128(base + (int64_t)u * 16, pol);
    r.b = ldg_stream128(base + (int64_t)(w.U + u) * 16, pol);
    r.h = ldg_stream32(w.aux + ((int64_t)row * w.U + u) * 4, pol);
  }

#define B2Q_Q4K_WORD(W, XA, XB, YA, YB)                       \
  {                                                           \
    const uint32_t lo_ = (W)&0x0F0F0F0Fu, hi_ = (W)&0xF0F0F0F0u; \
    ia = dp2a_lo_ss((XA), (int)lo_, ia);                      \
    ia = dp2a_hi_ss((XB), (int)lo_, ia);                      \
    ib = dp2a_lo_su((YA), hi_, ib);                           \
    ib = dp2a_hi_su((YB), hi_, ib);                           \
  }

  template <int R, int MT>
  __device__ __forceinline__ static void compute(const Reg (&r)[R], int u, const SX& sx,
                                                 float (&acc)[R][MT]) {
    const int c = u & 3;
    const int base = (u >> 2) * 256 + c * 64;
    const int xb = base >> 5;
    float d[R], dm[R], ma[R], mb[R];
    int sca[R], scb[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const uint32_t h = r[i].h;
      sca[i] = (int)(h & 63u);
      scb[i] = (int)((h >> 6) & 63u);
      ma[i] = (float)((h >> 12) & 63u);
      mb[i] = (float)((h >> 18) & 63u);
      uint32_t dd = (h >> 24) << (8 * c);
      dd |= __shfl_xor_sync(B2Q_FULL, dd, 1);
      dd |= __shfl_xor_sync(B2Q_FULL, dd, 2);
      d[i] = f16_bits_fast(dd & 0xffffu);
      dm[i] = f16_bits_fast(dd >> 16);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int4* xv = reinterpret_cast<const int4*>(sx.q + (int64_t)t * sx.kpad + base);
      const int4 xl0 = xv[0], xl1 = xv[1], xl2 = xv[2], xl3 = xv[3];  // base + 0..31
      const int4 xh0 = xv[4], xh1 = xv[5], xh2 = xv[6], xh3 = xv[7];  // base + 32..63
      const int nb32 = sx.kpad >> 5;
      const float xsa = sx.scale[t * nb32 + xb], xsb = sx.scale[t * nb32 + xb + 1];
      const float fsa = sx.fsum[t * nb32 + xb], fsb = sx.fsum[t * nb32 + xb + 1];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        int ia = 0, ib = 0;
        B2Q_Q4K_WORD(r[i].a.x, xl0.x, xl0.y, xh0.x, xh0.y)
        B2Q_Q4K_WORD(r[i].a.y, xl0.z, xl0.w, xh0.z, xh0.w)
        B2Q_Q4K_WORD(r[i].a.z, xl1.x, xl1.y, xh1.x, xh1.y)
        B2Q_Q4K_WORD(r[i].a.w, xl1.z, xl1.w, xh1.z, xh1.w)
        B2Q_Q4K_WORD(r[i].b.x, xl2.x, xl2.y, xh2.x, xh2.y)
        B2Q_Q4K_WORD(r[i].b.y, xl2.z, xl2.w, xh2.z, xh2.w)
        B2Q_Q4K_WORD(r[i].b.z, xl3.x, xl3.y, xh3.x, xh3.y)
        B2Q_Q4K_WORD(r[i].b.w, xl3.z, xl3.w, xh3.z, xh3.w)
        const float t1 = xsa * (float)(sca[i] * ia) + xsb * (float)(scb[i] * (ib >> 4));
        const float t2 = ma[i] * fsa + mb[i] * fsb;
        acc[i][t] += d[i] * t1 - dm[i] * t2;
      }
    }
  }
#undef B2Q_Q4K_WORD
};

// ---------------------------------------------------------------------------
// Q6_K
// ---------------------------------------------------------------------------
struct FmtQ6K {
  struct Reg { uint4 a, b, c; uint32_t s; uint32_t d; };
  __device__ __forceinline__ static void zero(Reg& r) {
    r.a = make_uint4(0, 0, 0, 0); r.b = r.a; r.c = r.a; r.s = 0; r.d = 0;
  }
  __device__ __forceinline__ static void load(Reg& r, const WeightDev& w, int row, int u, uint64_t pol) {
    const uint8_t* base = w.qs + (int64_t)row * w.row_qs;
    r.a = ldg_stream128(base + (int64_t)u * 16, pol);
    r.b = ldg_stream128(base + (int64_t)(w.U + u) * 16, pol);
    r.c = ldg_stream128(base + (int64_t)(2 * w.U + u) * 16, pol);
    r.s = ldg_stream32(w.aux + ((int64_t)row * w.U + u) * 4, pol);
    r.d = ldg_stream16(w.aux2 + ((int64_t)row * w.nb + (u >> 2)) * 2, pol);
  }

  template <int R, int MT>
  __device__ __forceinline__ static void compute(const Reg (&r)[R], int u, const SX& sx,
                                                 float (&acc)[R][MT]) {
    const int base0 = (u >> 2) * 256 + ((u >> 1) & 1) * 128 + (u & 1) * 16;
    float d[R];
    int sc[R][4];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      d[i] = f16_bits_fast(r[i].d);
#pragma unroll
      for (int g = 0; g < 4; ++g) sc[i][g] = (int)(int8_t)((r[i].s >> (8 * g)) & 0xffu);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int16_t* xt = sx.q + (int64_t)t * sx.kpad;
      int4 X[4][2];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int4* xv = reinterpret_cast<const int4*>(xt + base0 + 32 * g);
        X[g][0] = xv[0];
        X[g][1] = xv[1];
      }
      const int nb32 = sx.kpad >> 5, nb16 = sx.kpad >> 4;
      float xs[4];
      int s16[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        xs[g] = sx.scale[t * nb32 + ((base0 + 32 * g) >> 5)];
        s16[g] = sx.s16[t * nb16 + ((base0 + 32 * g) >> 4)];
      }
#pragma unroll
      for (int i = 0; i < R; ++i) {
        int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
        const uint32_t qa[4] = {r[i].a.x, r[i].a.y, r[i].a.z, r[i].a.w};
        const uint32_t qb[4] = {r[i].b.x, r[i].b.y, r[i].b.z, r[i].b.w};
        const uint32_t qh[4] = {r[i].c.x, r[i].c.y, r[i].c.z, r[i].c.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t q1 = (qa[j] & 0x0F0F0F0Fu) | ((qh[j] << 4) & 0x30303030u);
          const uint32_t q2 = (qb[j] & 0x0F0F0F0Fu) | ((qh[j] << 2) & 0x30303030u);
          const uint32_t q3 = ((qa[j] >> 4) & 0x0F0F0F0Fu) | (qh[j] & 0x30303030u);
          const uint32_t q4 = ((qb[j] >> 4) & 0x0F0F0F0Fu) | ((qh[j] >> 2) & 0x30303030u);
          const int4& x0 = X[0][j >> 1];
          const int4& x1 = X[1][j >> 1];
          const int4& x2 = X[2][j >> 1];
          const int4& x3 = X[3][j >> 1];
          const bool up = (j & 1) != 0;
          a0 = dp2a_lo_ss(up ? x0.z : x0.x, (int)q1, a0);
          a0 = dp2a_hi_ss(up ? x0.w : x0.y, (int)q1, a0);
          a1 = dp2a_lo_ss(up ? x1.z : x1.x, (int)q2, a1);
          a1 = dp2a_hi_ss(up ? x1.w : x1.y, (int)q2, a1);
          a2 = dp2a_lo_ss(up ? x2.z : x2.x, (int)q3, a2);
          a2 = dp2a_hi_ss(up ? x2.w : x2.y, (int)q3, a2);
          a3 = dp2a_lo_ss(up ? x3.z : x3.x, (int)q4, a3);
          a3 = dp2a_hi_ss(up ? x3.w : x3.y, (int)q4, a3);
        }
        float f = xs[0] * (float)(sc[i][0] * (a0 - 32 * s16[0]));
        f += xs[1] * (float)(sc[i][1] * (a1 - 32 * s16[1]));
        f += xs[2] * (float)(sc[i][2] * (a2 - 32 * s16[2]));
        f += xs[3] * (float)(sc[i][3] * (a3 - 32 * s16[3]));
        acc[i][t] += d[i] * f;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Q8_0
// ---------------------------------------------------------------------------
struct FmtQ80 {
  struct Reg { uint4 a, b; uint32_t d; };
  __device__ __forceinline__ static void zero(Reg& r) {
    r.a = make_uint4(0, 0, 0, 0); r.b = r.a; r.d = 0;
  }
  __device__ __forceinline__ static void load(Reg& r, const WeightDev& w, int row, int u, uint64_t pol) {
    const uint8_t* base = w.qs + (int64_t)row * w.row_qs;
    r.a = ldg_stream128(base + (int64_t)u * 16, pol);
    r.b = ldg_stream128(base + (int64_t)(w.U + u) * 16, pol);
    r.d = ldg_stream16(w.aux + ((int64_t)row * w.U + u) * 2, pol);
  }
  template <int R, int MT>
  __device__ __forceinline__ static void compute(const Reg (&r)[R], int u, const SX& sx,
                                                 float (&acc)[R][MT]) {
    float d[R];
#pragma unroll
    for (int i = 0; i < R; ++i) d[i] = f16_bits_fast(r[i].d);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int4* xv = reinterpret_cast<const int4*>(sx.q + (int64_t)t * sx.kpad + u * 32);
      const int4 x0 = xv[0], x1 = xv[1], x2 = xv[2], x3 = xv[3];
      const float xs = sx.scale[t * (sx.kpad >> 5) + u];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        int s = 0;
        s = dp2a_lo_ss(x0.x, (int)r[i].a.x, s); s = dp2a_hi_ss(x0.y, (int)r[i].a.x, s);
        s = dp2a_lo_ss(x0.z, (int)r[i].a.y, s); s = dp2a_hi_ss(x0.w, (int)r[i].a.y, s);
        s = dp2a_lo_ss(x1.x, (int)r[i].a.z, s); s = dp2a_hi_ss(x1.y, (int)r[i].a.z, s);
        s = dp2a_lo_ss(x1.z, (int)r[i].a.w, s); s = dp2a_hi_ss(x1.w, (int)r[i].a.w, s);
        s = dp2a_lo_ss(x2.x, (int)r[i].b.x, s); s = dp2a_hi_ss(x2.y, (int)r[i].b.x, s);
        s = dp2a_lo_ss(x2.z, (int)r[i].b.y, s); s = dp2a_hi_ss(x2.w, (int)r[i].b.y, s);
        s = dp2a_lo_ss(x3.x, (int)r[i].b.z, s); s = dp2a_hi_ss(x3.y, (int)r[i].b.z, s);
        s = dp2a_lo_ss(x3.z, (int)r[i].b.w, s); s = dp2a_hi_ss(x3.w, (int)r[i].b.w, s);
        acc[i][t] += d[i] * (xs * (float)s);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Tile driver
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <class F, int R, int WK, int MT, int EPI>
__device__ __forceinline__ void gemv_tile(const GemvSeg& sg, int local_tile, int warp, int lane,
                                          const SX& sx, uint64_t pol, float* red) {
  constexpr int RG = 8 / WK;                        // row groups per CTA
  constexpr int RO = (EPI == kEpiSwiglu) ? R / 2 : R;  // output rows per warp
  const int rg = warp / WK, wk = warp % WK;
  const int r0 = (local_tile * RG + rg) * RO;
  const int n = sg.rows_out;

  // row slot -> (weight, row)
  int rows[R];
  bool rv[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int rr = r0 + (i % RO);
    rows[i] = rr;
    rv[i] = rr < n;
  }
  const WeightDev& wa = sg.w;
  const WeightDev& wb = (EPI == kEpiSwiglu) ? sg.w2 : sg.w;
  const int U = wa.U;
  const int step = 32 * WK;
  const int nj = (U + step - 1) / step;

  float acc[R][MT];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[i][t] = 0.0f;

  typename F::Reg cur[R], nxt[R];
  {
    const int u = lane + 32 * wk;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (u < U && rv[i]) F::load(cur[i], (i < RO) ? wa : wb, rows[i], u, pol);
      else F::zero(cur[i]);
    }
  }
  for (int j = 0; j < nj; ++j) {
    const int u = lane + 32 * wk + step * j;
    const int un = u + step;
    if (j + 1 < nj) {
#pragma unroll
      for (int i = 0; i < R; ++i) {
        if (un < U && rv[i]) F::load(nxt[i], (i < RO) ? wa : wb, rows[i], un, pol);
        else F::zero(nxt[i]);
      }
    }
    F::template compute<R, MT>(cur, u < U ? u : 0, sx, acc);
    if (j + 1 < nj) {
#pragma unroll
      for (int i = 0; i < R; ++i) cur[i] = nxt[i];
    }
  }

  // reduce over the warp, then over the WK warps sharing the rows
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[i][t] = warp_sum(acc[i][t]);
  if (WK > 1) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int t = 0; t < MT; ++t) red[(warp * R + i) * MT + t] = acc[i][t];
    }
    __syncthreads();
    if (wk == 0 && lane == 0) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          float v = 0.0f;
          for (int w2 = 0; w2 < WK; ++w2) v += red[((warp + w2) * R + i) * MT + t];
          acc[i][t] = v;
        }
    }
    __syncthreads();
  }
  if (wk == 0 && lane == 0) {
#pragma unroll
    for (int i = 0; i < RO; ++i) {
      if (!rv[i]) continue;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        float* yp = sg.y + (int64_t)t * sg.ldy + rows[i];
        if (EPI == kEpiStore) *yp = acc[i][t];
        else if (EPI == kEpiAdd) *yp += acc[i][t];
        else *yp = silu_f(acc[i][t]) * acc[i + RO][t];
      }
    }
  }
}

template <int R, int WK, int MT, int EPI>
__global__ void __launch_bounds__(256, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ float red[8 * R * MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kp = a.kpad;
  SX sx;
  sx.q = reinterpret_cast<const int16_t*>(smem);
  sx.scale = reinterpret_cast<const float*>(smem + (size_t)MT * kp * 2);
  sx.fsum = sx.scale + MT * (kp / 32);
  sx.s16 = reinterpret_cast<const int32_t*>(sx.fsum + MT * (kp / 32));
  sx.kpad = kp;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the activations come from the previous kernel
  if (threadIdx.x == 0) {
    const uint32_t bq = (uint32_t)(MT * kp * 2), bs = (uint32_t)(MT * (kp / 32) * 4),
                   b16 = (uint32_t)(MT * (kp / 16) * 4);
    mbar_arrive_expect_tx(&bar, bq + 2 * bs + b16);
    bulk_g2s((void*)sx.q, a.xq + (int64_t)a.t0 * kp, bq, &bar);
    bulk_g2s((void*)sx.scale, a.xscale + (int64_t)a.t0 * (kp / 32), bs, &bar);
    bulk_g2s((void*)sx.fsum, a.xfsum + (int64_t)a.t0 * (kp / 32), bs, &bar);
    bulk_g2s((void*)sx.s16, a.xs16 + (int64_t)a.t0 * (kp / 16), b16, &bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0);
  if (__syncthreads_or(!ok)) return;
  pdl_launch_dependents();

  const uint64_t pol = make_evict_first_policy();
  for (int tile = blockIdx.x; tile < a.tiles_total; tile += gridDim.x) {
    int s = 0;
#pragma unroll
    for (int q = 1; q < kMaxSegs; ++q)
      if (q < a.nseg && tile >= a.seg[q].tile0) s = q;
    const GemvSeg& sg = a.seg[s];
    const int lt = tile - sg.tile0;
    switch (sg.w.dtype) {
      case kQ4_K: gemv_tile<FmtQ4K, R, WK, MT, EPI>(sg, lt, warp, lane, sx, pol, red); break;
      case kQ6_K: gemv_tile<FmtQ6K, R, WK, MT, EPI>(sg, lt, warp, lane, sx, pol, red); break;
      default: gemv_tile<FmtQ80, R, WK, MT, EPI>(sg, lt, warp, lane, sx, pol, red); break;
    }
  }
}

}  // namespace b2q
