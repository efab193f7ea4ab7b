// gemv.cuh -- dequantise-and-multiply GEMV for repacked GGUF weights.
//
// y[t][r] = sum_c dequant(W)[r][c] * x[t][c] for t in [0, MT).
//
// Design (HBM-bound integer/byte work; no tensor cores):
//  * Weights are stored tiled (quant.cuh): a tile is 8 rows x one k-chunk
//    of <= 64 units and is one contiguous byte range.
//  * One persistent CTA per SM owns a contiguous range of 8-row groups of
//    one weight (segment).  A producer warp streams the CTA's tiles into a
//    shared-memory ring with 1-D bulk async copies (the TMA engine), one copy
//    per stage.  Weight copies are issued before the kernel waits for its
//    predecessor (programmatic dependent launch): weights never depend on an
//    earlier kernel, so the first stages stream while the previous kernel
//    drains; the kernel lets its own dependent launch at its start, so the
//    next launch's CTAs take each SM as soon as this grid's CTA there exits.
//  * The CTA walks its tiles chunk-major: for each k-chunk c, every 8-row
//    group it owns.  A stage holds NR = 2 tiles when they fit (two groups, or
//    the gate and up tiles of the fused SwiGLU), else one.
//  * Sixteen consumer warps, activation-stationary: warp 2p+h owns row p of
//    every tile and unit half h (unit u = c*KC + 32h + lane) of the chunk, so
//    a lane's 64 activations stay in registers for the whole chunk pass and
//    the steady state reads only weights from shared memory.  Lane -> one
//    unit of 64 (Q4_K, Q6_K) or 32 (Q8_0) weights.  After each stage every
//    row partial is reduced across the warp and added into a per-CTA
//    shared-memory accumulator (one writer per entry, fixed order:
//    deterministic); the epilogue writes y once at the end.  There is no
//    CTA-wide barrier in the steady state.
//  * The activation arrives pre-quantised to int16 per 64-element block
//    (quant.cuh) in a swizzled layout that makes every lane pattern below
//    bank-conflict-free, and is staged once per CTA.
//  * The inner product is integer: dp2a multiplies two int16 activations by
//    two weight bytes with int32 accumulation.  Q4_K nibbles are masked in
//    place (low nibbles as 0..15, high nibbles as 16*q, shifted after the
//    sum); Q6_K codes are rebuilt from ql/qh as unsigned 0..63 and the -32
//    offset is applied with the precomputed 16-element activation sums.  The
//    sub-block scales and mins are applied in int32 too; each unit ends with
//    one or two int->f32 conversions scaled by d (and dmin) and the
//    activation block scale.
#pragma once

#include "quant.cuh"

namespace b2q {

enum : int { kEpiStore = 0, kEpiAdd = 1, kEpiSwiglu = 2 };

constexpr int kGemvConsumerWarps = 16;  // two per row of an 8-row tile
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvMaxStages = 10;
constexpr int kGemvSmemBudget = 225 * 1024;

// Device view of a repacked weight.
struct WeightDev {
  const uint8_t* base;  // tiles, (group, chunk) major
  TileLayout L;
};

struct GemvSeg {
  WeightDev w;       // weight (gate for SwiGLU)
  WeightDev w2;      // up (SwiGLU only)
  float* y;          // output: y[t * ldy + row]
  int ldy;
  int rows_out;      // output rows (n)
  int cta0, ncta;    // CTAs [cta0, cta0 + ncta) own this segment
  int nr;            // 8-row tiles per stage (1 or 2; SwiGLU: gate + up = 2)
};

// Most rows one CTA may own (sizes the shared-memory row accumulators).
__host__ __device__ inline int gemv_rows_cap(int G, int ncta) { return ((G + ncta - 1) / ncta) * 8; }

constexpr int kMaxSegs = 4;

struct GemvArgs {
  GemvSeg seg[kMaxSegs];
  int nseg;
  int ns;              // pipeline stages
  int slot_bytes;      // bytes per stage slot
  int rows_cap;        // max rows per CTA over the segments
  // quantised activations, tokens [t0, t0 + MT)
  const int16_t* xq;
  const float* xscale;
  const int32_t* xs16;
  int kpad;
  int t0;
};

// Shared-memory view of the staged activations (MT tokens).
struct SX {
  const int16_t* q;
  const float* scale;
  const int32_t* s16;
  int kpad;
};

__host__ __device__ inline size_t gemv_x_bytes(int kpad, int mt) {
  return (size_t)mt * kpad * 2 + (size_t)mt * (kpad / 64) * 4 + (size_t)mt * (kpad / 16) * 4;
}

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Per-lane activation swizzle phase.  A consumer lane processes units
// u = c*KC + 32*h + lane with KC a multiple of 8 (16 for Q8_0), so the
// low bits of every activation group it touches depend only on the lane:
// the chunk permutation (xswz_f) is a per-lane constant, precomputed as the
// byte-offset xor mask F = xswz_f(...) << 4.
struct XPhase {
  int f4;       // Q4_K: group u
  int f6a, f6b; // Q6_K: group 4b+2h and 4b+2h+1
  int f8;       // Q8_0: group u >> 1
};

__device__ __forceinline__ XPhase make_xphase(int lane) {
  XPhase p;
  p.f4 = xswz_f(lane & 7) << 4;
  const int g6 = 4 * ((lane >> 2) & 1) + 2 * ((lane >> 1) & 1);
  p.f6a = xswz_f(g6) << 4;
  p.f6b = xswz_f(g6 + 1) << 4;
  p.f8 = xswz_f((lane >> 1) & 7) << 4;
  return p;
}

// 16-byte chunk c of the 64-element group at byte address `gb` (shared
// memory), given the xor mask F of that group.
__device__ __forceinline__ int4 xld(const uint8_t* gb, int c, int F) {
  return *reinterpret_cast<const int4*>(gb + ((c << 4) ^ F));
}

// ---------------------------------------------------------------------------
// Activations of one unit held in registers (x-stationary): the 64 int16
// values of activation block `u` as 8 x 16 bytes, its scale and its
// 16-element sums.
// ---------------------------------------------------------------------------
struct XUnit {
  int4 v[8];
  float xs;      // Q4_K / Q8_0: scale of the unit's block
  float2 xs2;    // Q6_K: scales of its two blocks
  int4 s16;      // Q4_K: .x, .y = sums of each 32-element half; Q6_K: .x..w = 32 * sums of groups 0..3
};

// Q4_K unit u = activation block u: chunks 0..7 of group u.
__device__ __forceinline__ void xload_q4k(XUnit& X, const SX& sx, int t, int u, int F) {
  const uint8_t* gb = reinterpret_cast<const uint8_t*>(sx.q + (int64_t)t * sx.kpad) + u * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) X.v[c] = xld(gb, c, F);
  X.xs = sx.scale[t * (sx.kpad >> 6) + u];
  const int4 q = *reinterpret_cast<const int4*>(sx.s16 + t * (sx.kpad >> 4) + 4 * u);
  X.s16 = make_int4(q.x + q.y, q.z + q.w, 0, 0);
}

// Q6_K unit u = 4b + 2h + s: group g = 16 elements of block grp0 + (g >> 1),
// chunks 2s + 4(g & 1) and the next one.
__device__ __forceinline__ void xload_q6k(XUnit& X, const SX& sx, int t, int u, int Fa, int Fb) {
  const int s = u & 1;
  const int grp0 = (u >> 2) * 4 + ((u >> 1) & 1) * 2;
  const uint8_t* gb0 = reinterpret_cast<const uint8_t*>(sx.q + (int64_t)t * sx.kpad) + grp0 * 128;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint8_t* gb = gb0 + (g >> 1) * 128;
    const int F = (g >> 1) ? Fb : Fa;
    const int c0 = 2 * s + 4 * (g & 1);
    X.v[2 * g] = xld(gb, c0, F);
    X.v[2 * g + 1] = xld(gb, c0 + 1, F);
  }
  X.xs2 = *reinterpret_cast<const float2*>(sx.scale + t * (sx.kpad >> 6) + grp0);
  const int32_t* q16 = sx.s16 + t * (sx.kpad >> 4) + 4 * grp0 + s;
  X.s16 = make_int4(32 * q16[0], 32 * q16[2], 32 * q16[4], 32 * q16[6]);
}

// Q8_0 unit u = 32 elements: chunks (u & 1) * 4 .. +3 of group u >> 1.
__device__ __forceinline__ void xload_q80(XUnit& X, const SX& sx, int t, int u, int F) {
  const uint8_t* gb = reinterpret_cast<const uint8_t*>(sx.q + (int64_t)t * sx.kpad) + (u >> 1) * 128;
  const int c0 = (u & 1) * 4;
#pragma unroll
  for (int c = 0; c < 4; ++c) X.v[c] = xld(gb, c0 + c, F);
  X.xs = sx.scale[t * (sx.kpad >> 6) + (u >> 1)];
}

// Q4_0 unit u = one 32-element block: the Q8_0 chunks, plus the sum of its
// 32 activations (the -8 offset of the codes).
__device__ __forceinline__ void xload_q40(XUnit& X, const SX& sx, int t, int u, int F) {
  xload_q80(X, sx, t, u, F);
  const int32_t* q16 = sx.s16 + t * (sx.kpad >> 4) + 4 * (u >> 1) + 2 * (u & 1);
  X.s16 = make_int4(q16[0] + q16[1], 0, 0, 0);
}

// ---------------------------------------------------------------------------
// Per-row unit kernels.  rc: row-chunk base of the row in shared memory;
// ul: unit index within the chunk.  Return the row's contribution.
// ---------------------------------------------------------------------------
#define B2Q_Q4K_WORD(W, IA, IB, XA, XB, YA, YB)                  \
  {                                                              \
    const uint32_t lo_ = (W)&0x0F0F0F0Fu, hi_ = (W)&0xF0F0F0F0u; \
    IA = dp2a_lo_ss((XA), (int)lo_, IA);                         \
    IA = dp2a_hi_ss((XB), (int)lo_, IA);                         \
    IB = dp2a_lo_su((YA), hi_, IB);                              \
    IB = dp2a_hi_su((YB), hi_, IB);                              \
  }

// Q4_K: qs bytes 32c..32c+31 of block b (u = 4b + c); its two 32-element
// sub-blocks share activation block u.  `csel` = u & 3.
__device__ __forceinline__ float row_q4k(const uint8_t* rc, int KC, int o_aux, int ul, int csel,
                                         const XUnit& X) {
  const uint4 a = lds128(rc + ul * 16);
  const uint4 b = lds128(rc + (KC + ul) * 16);
  const uint4 hb = lds128(rc + o_aux + (ul >> 2) * 16);  // the 4 header words of this block
  const uint32_t h = (csel & 2) ? ((csel & 1) ? hb.w : hb.z) : ((csel & 1) ? hb.y : hb.x);
  // d | dmin << 16 from the top bytes of the 4 words
  const uint32_t dd = __byte_perm(__byte_perm(hb.x, hb.y, 0x0073), __byte_perm(hb.z, hb.w, 0x0073), 0x5410);
  const float d = f16_bits_fast(dd & 0xffffu), dm = f16_bits_fast(dd >> 16);
  int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
  B2Q_Q4K_WORD(a.x, ia0, ib0, X.v[0].x, X.v[0].y, X.v[4].x, X.v[4].y)
  B2Q_Q4K_WORD(a.y, ia1, ib1, X.v[0].z, X.v[0].w, X.v[4].z, X.v[4].w)
  B2Q_Q4K_WORD(a.z, ia0, ib0, X.v[1].x, X.v[1].y, X.v[5].x, X.v[5].y)
  B2Q_Q4K_WORD(a.w, ia1, ib1, X.v[1].z, X.v[1].w, X.v[5].z, X.v[5].w)
  B2Q_Q4K_WORD(b.x, ia0, ib0, X.v[2].x, X.v[2].y, X.v[6].x, X.v[6].y)
  B2Q_Q4K_WORD(b.y, ia1, ib1, X.v[2].z, X.v[2].w, X.v[6].z, X.v[6].w)
  B2Q_Q4K_WORD(b.z, ia0, ib0, X.v[3].x, X.v[3].y, X.v[7].x, X.v[7].y)
  B2Q_Q4K_WORD(b.w, ia1, ib1, X.v[3].z, X.v[3].w, X.v[7].z, X.v[7].w)
  // sum_l (d sc q_l - dmin m) x_l over both sub-blocks, in units of xs
  const int isum = (int)(h & 63u) * (ia0 + ia1) + (int)((h >> 6) & 63u) * ((ib0 + ib1) >> 4);
  const int msum = (int)((h >> 12) & 63u) * X.s16.x + (int)((h >> 18) & 63u) * X.s16.y;
  return X.xs * (d * (float)isum - dm * (float)msum);
}
#undef B2Q_Q4K_WORD

// Q6_K: u = 4b + 2h + s covers l = 16s..16s+15 of half h for all four
// groups g (weights 128h + 32g + l); groups 0,1 lie in activation block
// 4b+2h, groups 2,3 in the next one.
__device__ __forceinline__ float row_q6k(const uint8_t* rc, int KC, int o_aux, int o_aux2, int ul,
                                         const XUnit& X) {
  const uint4 va = lds128(rc + ul * 16);
  const uint4 vb = lds128(rc + (KC + ul) * 16);
  const uint4 vh = lds128(rc + (2 * KC + ul) * 16);
  const uint32_t sw = *reinterpret_cast<const uint32_t*>(rc + o_aux + ul * 4);
  const float d = f16_bits_fast(*reinterpret_cast<const uint16_t*>(rc + o_aux2 + (ul >> 2) * 2));
  const uint32_t qa[4] = {va.x, va.y, va.z, va.w};
  const uint32_t qb[4] = {vb.x, vb.y, vb.z, vb.w};
  const uint32_t qh[4] = {vh.x, vh.y, vh.z, vh.w};
  int s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t q1 = (qa[j] & 0x0F0F0F0Fu) | ((qh[j] << 4) & 0x30303030u);
    const uint32_t q2 = (qb[j] & 0x0F0F0F0Fu) | ((qh[j] << 2) & 0x30303030u);
    const uint32_t q3 = ((qa[j] >> 4) & 0x0F0F0F0Fu) | (qh[j] & 0x30303030u);
    const uint32_t q4 = ((qb[j] >> 4) & 0x0F0F0F0Fu) | ((qh[j] >> 2) & 0x30303030u);
    // word j covers elements 4j..4j+3 of each group: chunk j/2 of the pair
    const int4& x1 = X.v[0 + (j >> 1)];
    const int4& x2 = X.v[2 + (j >> 1)];
    const int4& x3 = X.v[4 + (j >> 1)];
    const int4& x4 = X.v[6 + (j >> 1)];
    const bool up = (j & 1) != 0;
    s0[0] = dp2a_lo_ss(up ? x1.z : x1.x, (int)q1, s0[0]);
    s1[0] = dp2a_hi_ss(up ? x1.w : x1.y, (int)q1, s1[0]);
    s0[1] = dp2a_lo_ss(up ? x2.z : x2.x, (int)q2, s0[1]);
    s1[1] = dp2a_hi_ss(up ? x2.w : x2.y, (int)q2, s1[1]);
    s0[2] = dp2a_lo_ss(up ? x3.z : x3.x, (int)q3, s0[2]);
    s1[2] = dp2a_hi_ss(up ? x3.w : x3.y, (int)q3, s1[2]);
    s0[3] = dp2a_lo_ss(up ? x4.z : x4.x, (int)q4, s0[3]);
    s1[3] = dp2a_hi_ss(up ? x4.w : x4.y, (int)q4, s1[3]);
  }
  const int sc0 = (int)(int8_t)(sw & 0xffu), sc1 = (int)(int8_t)((sw >> 8) & 0xffu);
  const int sc2 = (int)(int8_t)((sw >> 16) & 0xffu), sc3 = (int)(int8_t)(sw >> 24);
  const int i01 = sc0 * (s0[0] + s1[0] - X.s16.x) + sc1 * (s0[1] + s1[1] - X.s16.y);
  const int i23 = sc2 * (s0[2] + s1[2] - X.s16.z) + sc3 * (s0[3] + s1[3] - X.s16.w);
  return d * (X.xs2.x * (float)i01 + X.xs2.y * (float)i23);
}

// Q5_K: as Q4_K with the fifth bit of every code (dequantize_slice,
// inference.rs:1418-1447): word j of a qs half holds elements 4j..4j+3 of
// both sub-blocks; their fifth bits sit at bits 8i + j of the unit's two
// bit words, moved to bit 4 of each byte with one shift and mask.  Codes are
// 0..31 in both halves (no 16x trick), so both partial sums are in code units.
template <int J>
__device__ __forceinline__ uint32_t q5_bits(uint32_t m) {
  return (J <= 4 ? (m << (4 - J)) : (m >> (J - 4))) & 0x10101010u;
}

#define B2Q_Q5K_WORD(J, W, IA, IB, XA, XB, YA, YB)                                  \
  {                                                                                \
    const uint32_t lo_ = ((W)&0x0F0F0F0Fu) | q5_bits<J>(mb.x);                     \
    const uint32_t hi_ = (((W) >> 4) & 0x0F0F0F0Fu) | q5_bits<J>(mb.y);            \
    IA = dp2a_lo_ss((XA), (int)lo_, IA);                                           \
    IA = dp2a_hi_ss((XB), (int)lo_, IA);                                           \
    IB = dp2a_lo_ss((YA), (int)hi_, IB);                                           \
    IB = dp2a_hi_ss((YB), (int)hi_, IB);                                           \
  }

__device__ __forceinline__ float row_q5k(const uint8_t* rc, int KC, int o_aux, int o_aux2, int ul, int csel,
                                         const XUnit& X) {
  const uint4 a = lds128(rc + ul * 16);
  const uint4 b = lds128(rc + (KC + ul) * 16);
  const uint2 mb = *reinterpret_cast<const uint2*>(rc + o_aux + ul * 8);
  const uint4 hb = lds128(rc + o_aux2 + (ul >> 2) * 16);
  const uint32_t h = (csel & 2) ? ((csel & 1) ? hb.w : hb.z) : ((csel & 1) ? hb.y : hb.x);
  const uint32_t dd = __byte_perm(__byte_perm(hb.x, hb.y, 0x0073), __byte_perm(hb.z, hb.w, 0x0073), 0x5410);
  const float d = f16_bits_fast(dd & 0xffffu), dm = f16_bits_fast(dd >> 16);
  int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
  B2Q_Q5K_WORD(0, a.x, ia0, ib0, X.v[0].x, X.v[0].y, X.v[4].x, X.v[4].y)
  B2Q_Q5K_WORD(1, a.y, ia1, ib1, X.v[0].z, X.v[0].w, X.v[4].z, X.v[4].w)
  B2Q_Q5K_WORD(2, a.z, ia0, ib0, X.v[1].x, X.v[1].y, X.v[5].x, X.v[5].y)
  B2Q_Q5K_WORD(3, a.w, ia1, ib1, X.v[1].z, X.v[1].w, X.v[5].z, X.v[5].w)
  B2Q_Q5K_WORD(4, b.x, ia0, ib0, X.v[2].x, X.v[2].y, X.v[6].x, X.v[6].y)
  B2Q_Q5K_WORD(5, b.y, ia1, ib1, X.v[2].z, X.v[2].w, X.v[6].z, X.v[6].w)
  B2Q_Q5K_WORD(6, b.z, ia0, ib0, X.v[3].x, X.v[3].y, X.v[7].x, X.v[7].y)
  B2Q_Q5K_WORD(7, b.w, ia1, ib1, X.v[3].z, X.v[3].w, X.v[7].z, X.v[7].w)
  // codes <= 31, |x| <= 16383, 32 per sub-block, scales <= 63: |isum| < 2^31
  const int isum = (int)(h & 63u) * (ia0 + ia1) + (int)((h >> 6) & 63u) * (ib0 + ib1);
  const int msum = (int)((h >> 12) & 63u) * X.s16.x + (int)((h >> 18) & 63u) * X.s16.y;
  return X.xs * (d * (float)isum - dm * (float)msum);
}
#undef B2Q_Q5K_WORD

// Q4_0: one block of 32 codes 0..15 with offset -8 (dequantize_slice,
// inference.rs:1459-1469): element i in the low nibble of byte i, i + 16 in
// the high nibble.
__device__ __forceinline__ float row_q40(const uint8_t* rc, int o_aux, int ul, const XUnit& X) {
  const uint4 a = lds128(rc + ul * 16);
  const float d = f16_bits_fast(*reinterpret_cast<const uint16_t*>(rc + o_aux + ul * 2));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
  int s0 = 0, s1 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
    const int4& xl = X.v[j >> 1];
    const int4& xh = X.v[2 + (j >> 1)];
    s0 = dp2a_lo_ss((j & 1) ? xl.z : xl.x, (int)lo, s0);
    s1 = dp2a_hi_ss((j & 1) ? xl.w : xl.y, (int)lo, s1);
    s0 = dp2a_lo_ss((j & 1) ? xh.z : xh.x, (int)hi, s0);
    s1 = dp2a_hi_ss((j & 1) ? xh.w : xh.y, (int)hi, s1);
  }
  return d * (X.xs * (float)(s0 + s1 - 8 * X.s16.x));
}

// Q8_0: one block (32 weights).
__device__ __forceinline__ float row_q80(const uint8_t* rc, int KC, int o_aux, int ul, const XUnit& X) {
  const uint4 a = lds128(rc + ul * 16);
  const uint4 b = lds128(rc + (KC + ul) * 16);
  const float d = f16_bits_fast(*reinterpret_cast<const uint16_t*>(rc + o_aux + ul * 2));
  int s0 = 0, s1 = 0;
  s0 = dp2a_lo_ss(X.v[0].x, (int)a.x, s0); s1 = dp2a_hi_ss(X.v[0].y, (int)a.x, s1);
  s0 = dp2a_lo_ss(X.v[0].z, (int)a.y, s0); s1 = dp2a_hi_ss(X.v[0].w, (int)a.y, s1);
  s0 = dp2a_lo_ss(X.v[1].x, (int)a.z, s0); s1 = dp2a_hi_ss(X.v[1].y, (int)a.z, s1);
  s0 = dp2a_lo_ss(X.v[1].z, (int)a.w, s0); s1 = dp2a_hi_ss(X.v[1].w, (int)a.w, s1);
  s0 = dp2a_lo_ss(X.v[2].x, (int)b.x, s0); s1 = dp2a_hi_ss(X.v[2].y, (int)b.x, s1);
  s0 = dp2a_lo_ss(X.v[2].z, (int)b.y, s0); s1 = dp2a_hi_ss(X.v[2].w, (int)b.y, s1);
  s0 = dp2a_lo_ss(X.v[3].x, (int)b.z, s0); s1 = dp2a_hi_ss(X.v[3].y, (int)b.z, s1);
  s0 = dp2a_lo_ss(X.v[3].z, (int)b.w, s0); s1 = dp2a_hi_ss(X.v[3].w, (int)b.w, s1);
  return d * (X.xs * (float)(s0 + s1));
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// Shared-memory ring of weight stages: `ns` slots of `slot_bytes`, one full
// and one empty mbarrier per slot.  The producer and the consumers each keep
// their own copy of the (slot, phase) position and advance it once per stage;
// a ring may carry the stages of several GEMVs back to back.
struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int ns, slot_bytes;
  int slot = 0;
  uint32_t phase = 0;
  int used = 0;  // stages issued so far, saturating at ns (producer only)
  __device__ __forceinline__ uint8_t* slot_ptr() const { return base + (size_t)slot * slot_bytes; }
  __device__ __forceinline__ void advance() {
    if (used < ns) ++used;
    if (++slot == ns) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// The CTA's stages of one GEMV, chunk-major: for chunk c = 0..C-1, the 8-row
// groups [gb, ge) taken NR at a time (SwiGLU: one group, gate tile + up
// tile).  Iterated with counters only (no division in the loop).
template <int NR, bool PAIR>
struct StageIter {
  int gb, ge, C;
  int c = 0, g = 0;
  __device__ __forceinline__ StageIter(int gb_, int ge_, int C_) : gb(gb_), ge(ge_), C(C_) { g = gb; }
  __device__ __forceinline__ bool done() const { return c >= C || gb >= ge; }
  __device__ __forceinline__ int ntiles() const { return PAIR ? 2 : ((NR == 2 && g + 1 < ge) ? 2 : 1); }
  __device__ __forceinline__ void next() {
    g += (PAIR || NR == 1) ? 1 : 2;
    if (g >= ge) {
      g = gb;
      ++c;
    }
  }
};

// Producer (one thread): bulk-copy the CTA's tiles of groups [gb, ge) of
// `w` (and `w2`, SwiGLU) into the ring.  Returns false if a wait for a free
// slot gave up (the consumers stopped); the caller then stops producing.
template <int NR, bool PAIR>
__device__ __forceinline__ bool produce_gemv(Ring& rg, const WeightDev& w, const WeightDev& w2, int gb,
                                             int ge) {
  const TileLayout& L = w.L;
  const uint32_t tb = (uint32_t)tile_bytes(L);
  for (StageIter<NR, PAIR> it(gb, ge, L.C); !it.done(); it.next()) {
    if (rg.used >= rg.ns && !mbar_wait_bounded(&rg.empty[rg.slot], rg.phase ^ 1u)) return false;
    const int nt = it.ntiles();
    uint64_t* fb = &rg.full[rg.slot];
    mbar_arrive_expect_tx(fb, tb * nt);
    uint8_t* sl = rg.slot_ptr();
    const int64_t t0 = (int64_t)it.g * L.C + it.c;
    bulk_g2s(sl, w.base + t0 * tb, tb, fb);
    if (PAIR) bulk_g2s(sl + tb, w2.base + t0 * tb, tb, fb);
    else if (nt == 2) bulk_g2s(sl + tb, w.base + (t0 + L.C) * tb, tb, fb);
    rg.advance();
  }
  return true;
}

// Consumers (warps 0..15): the row partials of the CTA's stages of one
// GEMV, accumulated into the shared-memory row accumulators
// racc[h][tile i][row][t] (h = unit half; i = gate/up for SwiGLU).  The
// accumulators are zeroed here; the caller runs the epilogue after the
// trailing consumer_sync.  `ok` turns false if a wait gave up.  DT: the GGML
// type when known at compile time, or -1 to dispatch on L.dtype.
template <int MT, int NR, bool PAIR, int DT = -1>
__device__ __forceinline__ void consume_gemv(Ring& rg, const TileLayout& L, int gb, int ge, int rows_cap,
                                             const SX& sx, bool& ok, float* racc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tb = (uint32_t)tile_bytes(L);
  const int p = warp >> 1, hf = warp & 1;  // row p of every tile; unit half hf
  constexpr int NW = PAIR ? 2 : 1;
  const int dt = DT >= 0 ? DT : L.dtype;
  for (int i = threadIdx.x; i < 2 * NW * rows_cap * MT; i += kGemvConsumerWarps * 32) racc[i] = 0.0f;
  consumer_sync();

  const XPhase xp = make_xphase(lane);
  const int lane0 = lane + 32 * hf;
  const int csel = lane & 3;  // u & 3 for every unit of this lane (KC % 8 == 0)
  XUnit X[MT];
  int cur_c = -1;
  bool uok = false;
  int ul = 0;
  for (StageIter<NR, PAIR> it(gb, ge, L.C); !it.done(); it.next()) {
    if (it.c != cur_c) {  // new chunk pass: this lane's activations
      cur_c = it.c;
      ul = lane0;
      const int u = it.c * L.KC + ul;
      uok = ul < L.KC && u < L.U;
      if (uok && ok) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if (dt == kQ4_K || dt == kQ5_K) xload_q4k(X[t], sx, t, u, xp.f4);
          else if (dt == kQ6_K) xload_q6k(X[t], sx, t, u, xp.f6a, xp.f6b);
          else if (dt == kQ4_0) xload_q40(X[t], sx, t, u, xp.f8);
          else xload_q80(X[t], sx, t, u, xp.f8);
        }
      }
    }
    if (ok) ok = mbar_wait_bounded(&rg.full[rg.slot], rg.phase);
    const int nt = it.ntiles();
    float part[NR][MT];
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int t = 0; t < MT; ++t) part[i][t] = 0.0f;
    if (ok && uok) {
      const uint8_t* sl = rg.slot_ptr() + p * L.rc;
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        if (i >= nt) break;
        const uint8_t* rc = sl + i * tb;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if (dt == kQ4_K) part[i][t] = row_q4k(rc, L.KC, L.o_aux, ul, csel, X[t]);
          else if (dt == kQ6_K) part[i][t] = row_q6k(rc, L.KC, L.o_aux, L.o_aux2, ul, X[t]);
          else if (dt == kQ5_K) part[i][t] = row_q5k(rc, L.KC, L.o_aux, L.o_aux2, ul, csel, X[t]);
          else if (dt == kQ4_0) part[i][t] = row_q40(rc, L.o_aux, ul, X[t]);
          else part[i][t] = row_q80(rc, L.KC, L.o_aux, ul, X[t]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rg.empty[rg.slot]);  // the stage may be refilled
    rg.advance();
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int t = 0; t < MT; ++t) part[i][t] = warp_sum(part[i][t]);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        if (i >= nt) break;
        // PAIR: tile 0 = gate, tile 1 = up, same row; else tile i = group g + i
        const int wsel = PAIR ? i : 0;
        const int r = (PAIR ? (it.g - gb) : (it.g + i - gb)) * 8 + p;
        float* dst = racc + ((hf * NW + wsel) * rows_cap + r) * MT;
#pragma unroll
        for (int t = 0; t < MT; ++t) dst[t] += part[i][t];
      }
    }
  }
  consumer_sync();
}

// Final value of local row r, token t, weight wsel (SwiGLU: 0 gate, 1 up).
template <int MT, bool PAIR>
__device__ __forceinline__ float racc_value(const float* racc, int rows_cap, int r, int t, int wsel) {
  constexpr int NW = PAIR ? 2 : 1;
  return racc[((0 * NW + wsel) * rows_cap + r) * MT + t] + racc[((1 * NW + wsel) * rows_cap + r) * MT + t];
}

// Epilogue: y for every (row, token) of rows [8 gb, 8 ge) (rows >= n skipped).
template <int MT, int EPI>
__device__ __forceinline__ void gemv_epilogue(const float* racc, int rows_cap, int gb, int ge, int n, float* y,
                                              int ldy, bool ok) {
  constexpr bool kPair = EPI == kEpiSwiglu;
  if (!ok) return;
  const int row0 = gb * 8;
  const int nrows = (ge - gb) * 8;
  for (int idx = threadIdx.x; idx < nrows * MT; idx += kGemvConsumerWarps * 32) {
    const int r = idx / MT, t = idx % MT;
    const int row = row0 + r;
    if (row >= n) continue;
    const float v = racc_value<MT, kPair>(racc, rows_cap, r, t, 0);
    float* yp = y + (int64_t)t * ldy + row;
    if (kPair) *yp = silu_f(v) * racc_value<MT, kPair>(racc, rows_cap, r, t, 1);
    else if (EPI == kEpiAdd) *yp = __ldcg(yp) + v;  // y may be written by other CTAs
    else *yp = v;
  }
}

template <int MT, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full_bar[kGemvMaxStages], empty_bar[kGemvMaxStages], x_bar;
  constexpr bool kPair = EPI == kEpiSwiglu;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // segment of this CTA and its contiguous range of 8-row groups
  int s = 0;
#pragma unroll
  for (int q = 1; q < kMaxSegs; ++q)
    if (q < a.nseg && (int)blockIdx.x >= a.seg[q].cta0) s = q;
  const GemvSeg& sg = a.seg[s];
  const TileLayout& L = sg.w.L;
  const int ci = blockIdx.x - sg.cta0;
  const int gb = (int)((int64_t)L.G * ci / sg.ncta);
  const int ge = (int)((int64_t)L.G * (ci + 1) / sg.ncta);
  const int NS = a.ns;

  const int kp = a.kpad;
  if (kChecks) {  // uniform over the CTA: every thread leaves before any barrier
    const size_t need = gemv_x_bytes(kp, MT) + (size_t)NS * a.slot_bytes;
    if (!b2q_check(ci >= 0 && ci < sg.ncta && 0 <= gb && gb <= ge && ge <= L.G && NS <= kGemvMaxStages &&
                       need <= dyn_smem_bytes(),
                   kChkGemv))
      return;
  }
  uint8_t* stages = smem + gemv_x_bytes(kp, MT);
  float* racc = reinterpret_cast<float*>(stages + (size_t)NS * a.slot_bytes);
  SX sx;
  sx.q = reinterpret_cast<const int16_t*>(smem);
  sx.scale = reinterpret_cast<const float*>(smem + (size_t)MT * kp * 2);
  sx.s16 = reinterpret_cast<const int32_t*>(sx.scale + MT * (kp / 64));
  sx.kpad = kp;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kGemvConsumerWarps);
    }
    mbar_init(&x_bar, 1);
    fence_mbar_init();
    // let the next kernel launch now: its CTAs take each SM as soon as this
    // grid's CTA there exits, and stream their weights while the rest of this
    // grid finishes.  Its reads of this kernel's outputs still wait for the
    // whole grid (griddepcontrol.wait in every kernel launched dependent).
    pdl_launch_dependents();
  }
  __syncthreads();
  Ring rg;
  rg.base = stages;
  rg.full = full_bar;
  rg.empty = empty_bar;
  rg.ns = NS;
  rg.slot_bytes = a.slot_bytes;

  if (warp == kGemvConsumerWarps) {
    // producer: weights never depend on the previous kernel
    if (lane == 0) {
      if (kPair) produce_gemv<2, true>(rg, sg.w, sg.w2, gb, ge);
      else if (sg.nr == 2) produce_gemv<2, false>(rg, sg.w, sg.w2, gb, ge);
      else produce_gemv<1, false>(rg, sg.w, sg.w2, gb, ge);
    }
    return;
  }

  if (threadIdx.x == 0) {
    pdl_wait();  // the activations come from the previous kernel
    const uint32_t bq = (uint32_t)(MT * kp * 2), bs = (uint32_t)(MT * (kp / 64) * 4),
                   b16 = (uint32_t)(MT * (kp / 16) * 4);
    mbar_arrive_expect_tx(&x_bar, bq + bs + b16);
    bulk_g2s((void*)sx.q, a.xq + (int64_t)a.t0 * kp, bq, &x_bar);
    bulk_g2s((void*)sx.scale, a.xscale + (int64_t)a.t0 * (kp / 64), bs, &x_bar);
    bulk_g2s((void*)sx.s16, a.xs16 + (int64_t)a.t0 * (kp / 16), b16, &x_bar);
  }
  bool ok = mbar_wait_bounded(&x_bar, 0);
  if (kPair) consume_gemv<MT, 2, true>(rg, L, gb, ge, a.rows_cap, sx, ok, racc);
  else if (sg.nr == 2) consume_gemv<MT, 2, false>(rg, L, gb, ge, a.rows_cap, sx, ok, racc);
  else consume_gemv<MT, 1, false>(rg, L, gb, ge, a.rows_cap, sx, ok, racc);
  gemv_epilogue<MT, EPI>(racc, a.rows_cap, gb, ge, L.n, sg.y, sg.ldy, ok);
}

}  // namespace b2q
