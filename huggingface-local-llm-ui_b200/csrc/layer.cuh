// layer.cuh -- the per-layer operations around the GEMVs in the Llama
// block (StandardNativeEngine::forward, inference.rs:2695-2860): RMSNorm,
// NeoX RoPE, KV-cache append, GQA attention, and greedy argmax.
#pragma once

#include "quant.cuh"

namespace b2q {

constexpr int kAttnTile = 64;  // key tokens per attention split
// One split partial: {max, sum, O[128]} padded to 132 floats (528 bytes, a
// multiple of 16, so a head's partials can be moved with one bulk copy).
constexpr int kPartStride = 132;
constexpr int kHeadDim = 128;

// RMSNorm of each row (rms_norm_rows, inference.rs:1501-1512) fused with the
// int16 quantisation the next GEMV consumes.  One CTA of 1024 threads per
// row; each warp normalises and quantises whole 64-element blocks (lane i:
// elements 64j + i and 64j + 32 + i).  `y` (optional) receives the f32 row.
__global__ void __launch_bounds__(1024) rmsnorm_quant_kernel(
    const float* __restrict__ x, int row_stride, int row0, const float* __restrict__ w, int dim,
    float eps, XQ xq, float* __restrict__ y) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float part[32];
  const int t = blockIdx.x;
  const float* xr = x + (int64_t)(row0 + t) * row_stride;
  float ss = 0.0f;
  for (int e = threadIdx.x; e < dim; e += blockDim.x) ss = fmaf(xr[e], xr[e], ss);
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.0f;
    v = warp_sum(v);
    if (lane == 0) part[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(part[0] / (float)dim + eps);
  const int nw = blockDim.x >> 5;
  for (int e0 = warp * 64; e0 < xq.kpad; e0 += nw * 64) {
    const int ea = e0 + lane, eb = e0 + 32 + lane;
    // (x * inv) * w, two separate roundings as the reference computes it
    const float va = ea < dim ? __fmul_rn(__fmul_rn(xr[ea], inv), w[ea]) : 0.0f;
    const float vb = eb < dim ? __fmul_rn(__fmul_rn(xr[eb], inv), w[eb]) : 0.0f;
    if (y != nullptr) {
      if (ea < dim) y[(int64_t)t * dim + ea] = va;
      if (eb < dim) y[(int64_t)t * dim + eb] = vb;
    }
    xq_store_block(va, vb, lane, t, e0 >> 6, xq);
  }
}

// NeoX half-split RoPE on q (in place) and k, plus the f16 KV-cache append
// (inference.rs:2755-2780).  qkv [m][(H + 2*KV) * hd] as written by the QKV
// GEMV group; cache layout [KV][cap][hd] per layer.  `pos_dev` holds the
// start position (device scalar, so a captured graph can be replayed).
__global__ void rope_kv_kernel(float* __restrict__ qkv, int m, int H, int KV, int hd,
                               const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                               const int* __restrict__ pos_dev, int cap, __half* __restrict__ kc,
                               __half* __restrict__ vc, const float* __restrict__ q_bias,
                               const float* __restrict__ k_bias, const float* __restrict__ v_bias) {
  pdl_wait();
  pdl_launch_dependents();
  const int s = blockIdx.x;
  const int start = *pos_dev;
  const int p_abs = start + s;
  const int p_rope = p_abs < 8191 ? p_abs : 8191;
  const int half = hd / 2;
  const int width = (H + 2 * KV) * hd;
  float* row = qkv + (int64_t)s * width;
  const float* cs = rope_cos + (int64_t)p_rope * half;
  const float* sn = rope_sin + (int64_t)p_rope * half;
  // q and k: rotate pairs (j, j + half)
  for (int idx = threadIdx.x; idx < (H + KV) * half; idx += blockDim.x) {
    const int h = idx / half, j = idx % half;
    float* b = row + h * hd;
    const float* bias = h < H ? q_bias : k_bias;
    const int bo = h < H ? h * hd : (h - H) * hd;
    float x0 = b[j], x1 = b[half + j];
    if (bias != nullptr) { x0 += bias[bo + j]; x1 += bias[bo + half + j]; }
    const float c = cs[j], sv = sn[j];
    const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv));
    const float y1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sv));
    if (h < H) {
      b[j] = y0;
      b[half + j] = y1;
    } else if (p_abs < cap) {
      const int kh = h - H;
      __half* dst = kc + ((int64_t)kh * cap + p_abs) * hd;
      dst[j] = __float2half_rn(y0);
      dst[half + j] = __float2half_rn(y1);
    }
  }
  // v: append as is
  for (int idx = threadIdx.x; idx < KV * hd; idx += blockDim.x) {
    const int kh = idx / hd, d = idx % hd;
    float v = row[(H + KV) * hd + idx];
    if (v_bias != nullptr) v += v_bias[idx];
    if (p_abs < cap) vc[((int64_t)kh * cap + p_abs) * hd + d] = __float2half_rn(v);
  }
}

// ---------------------------------------------------------------------------
// Split GQA attention over the f16 KV cache (inference.rs:2782-2820).  The
// cached keys of a query are cut into splits of kAttnTile tokens; one item =
// (KV head g, split z) on kAttnThreads threads computes, for the G query
// heads of g, the split's softmax partial (max, sum, unnormalised P*V).  The
// K and V rows of a tile are brought into shared memory by TMA (one round
// trip to HBM), then everything runs from shared memory.  The same item code serves the per-kernel path
// (attn_split_kernel) and the persistent decode kernel, so both give the
// same bits.
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 512;

// The two products of a tile, q K^T and P V, run on the warp-level tensor
// cores (mma.sync m16n8k16, f16 operands, f32 accumulation).  The f16 K and
// V rows of the cache enter exactly; the f32 queries and probabilities are
// carried as two f16 parts each, hi = f16(v) toward zero and lo = f16(v -
// hi), as rows h (hi) and G + h (lo) of the A operand (A rows 2G..15, G < 8,
// repeat rows 0..2G-1 and their products are dropped), so one MMA gives both
// halves of each product; their sum carries the f32 operand to ~2^-22
// relative.  The probabilities enter scaled by 2^15 (out of the f16
// subnormal range; the P*V sums are scaled back exactly).  Queries must stay
// below the f16 maximum, 65504, in magnitude.
//
// Shared-memory layouts, all chosen so that the eight 16-byte rows of every
// ldmatrix phase sit on distinct banks:
//  * K and V tiles arrive by TMA with the 128-byte swizzle: two boxes of
//    64 rows x 64 dims (128 bytes) per tile, dims 0..63 then 64..127, and
//    the 16-byte chunk c of row r of a box stored at chunk c ^ (r & 7)
//    (kv_off); each tile buffer starts on a 1024-byte boundary, the period
//    of the swizzle.
//  * the query image [2G rows][128 dims] and the probability image (over
//    the score rows) store the chunk c of image row i at c ^ (i & 7).
constexpr float kPScale = 32768.0f;
constexpr uint32_t kAttnTileBytes = 2u * kAttnTile * kHeadDim * 2u;  // K + V of one tile
constexpr int kAttnAlignPad = 1024 - 16;  // worst-case padding of a tile buffer to 1024 bytes

template <int G>
struct AttnTile {
  __half k[kAttnTile * kHeadDim];  // tile rows (kv_off layout), then the P*V output [G][128] f32
  __half v[kAttnTile * kHeadDim];
  __half qimg[2 * G * kHeadDim];   // rotated queries: hi rows 0..G-1, lo rows G..2G-1
  float sp[G][kAttnTile];          // scores; then, over each head's own row, the probability
                                   // image: hi parts in chunks 0..7, lo parts in chunks 8..15
  float m[G], l[G];                // softmax max and sum per head
  __half kcur[kHeadDim];           // the current token's rotated k and its v, copied into
  __half vcur[kHeadDim];           // the tile that holds the token once its copy has landed
};

// element offset (halves) of row r, dim d in a K or V tile buffer
__device__ __forceinline__ int kv_off(int r, int d) {
  return (d >> 6) * (kAttnTile * 64) + r * 64 + ((d & 63) ^ ((r & 7) << 3));
}
// element offset of column c in an image row keyed i (halves; 128 per row)
__device__ __forceinline__ int img_col(int i, int c) { return c ^ ((i & 7) << 3); }

// the 1024-byte aligned address at or after p (shared memory); computed
// where it is used (volatile: never hoisted into a long-lived register)
__device__ __forceinline__ uint8_t* smem_align1024(uint8_t* p) {
  uint32_t pad;
  asm volatile("{\n\t.reg .u32 t;\n\tneg.s32 t, %1;\n\tand.b32 %0, t, 1023;\n\t}" : "=r"(pad) : "r"(smem_u32(p)));
  return p + pad;
}

__device__ __forceinline__ __half f16_hi(float v) { return __float2half_rz(v); }
__device__ __forceinline__ __half f16_lo(float v, __half hi) { return __float2half_rn(v - __half2float(hi)); }

template <int G>
__device__ __forceinline__ void attn_set_q(AttnTile<G>& T, int h, int d, float v) {
  const __half hi = f16_hi(v);
  T.qimg[h * kHeadDim + img_col(h, d)] = hi;
  T.qimg[(G + h) * kHeadDim + img_col(G + h, d)] = f16_lo(v, hi);
}

// Image row (head h + G * part, part 0 hi / 1 lo) behind A-operand row r
// (0..15) of an m16n8k16 product
template <int G>
__device__ __forceinline__ int attn_arow(int r) { return G == 8 ? r : r % (2 * G); }

// ldmatrix from a shared-memory address (32-bit)
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// d += a * b, m16n8k16, f16 x f16 -> f32
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Issue the TMA copies of the K and V tile whose first cache row (KV head
// times capacity plus token) is row0: four boxes of 64 rows x 64 dims into
// kb / vb (1024-byte aligned shared memory; one thread); completes on `bar`
// (expect_tx included).  Rows past the cache's end read as zeros; rows past
// the valid tokens are read as they are and masked by the caller.
__device__ __forceinline__ void attn_rows_load(__half* kb, __half* vb, const void* tmk, const void* tmv, int row0,
                                               uint64_t* bar) {
  mbar_arrive_expect_tx(bar, kAttnTileBytes);
  tma_load_2d(kb, tmk, 0, row0, bar);
  tma_load_2d(kb + kAttnTile * 64, tmk, 64, row0, bar);
  tma_load_2d(vb, tmv, 0, row0, bar);
  tma_load_2d(vb + kAttnTile * 64, tmv, 64, row0, bar);
}

// Key tiles per attention group.  A query's nz tiles of kAttnTile keys are
// cut into groups of consecutive tiles, one work item per (KV head, group),
// so that a single-token step has about `grid` items whatever the context:
// at short contexts one tile per group, at 8192 keys and 8 KV heads eight.
// The persistent kernel and the per-kernel path use the same grouping, so
// their partials and merges are the same bits.
__host__ __device__ __forceinline__ int attn_group_tiles(int nz, int KV, int grid) {
  const int ng = max(1, grid / max(1, KV));
  return (nz + ng - 1) / ng;
}

// Running softmax state of one attention group, for the (head, dim)
// elements i = tid + kAttnThreads * r a thread owns: max, sum and the
// unnormalised P*V of the tiles seen so far.  Folding tile partial (m_t, l_t,
// O_t) in: M = max(m, m_t); l = l * e^(m - M) + l_t * e^(m_t - M); O likewise
// (the first tile is taken as is, so a one-tile group is that tile's partial
// bit for bit).
template <int R>
struct AttnRun {
  float m[R], l[R], o[R];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int r = 0; r < R; ++r) { m[r] = -INFINITY; l[r] = 0.0f; o[r] = 0.0f; }
  }
  __device__ __forceinline__ void fold(int r, float mt, float lt, float ot) {
    if (m[r] == -INFINITY) { m[r] = mt; l[r] = lt; o[r] = ot; return; }
    const float M = fmaxf(m[r], mt);
    const float a = expf(m[r] - M), b = expf(mt - M);
    l[r] = fmaf(lt, b, l[r] * a);
    o[r] = fmaf(ot, b, o[r] * a);
    m[r] = M;
  }
};

// The softmax partial of one tile on kAttnThreads threads; the query image
// and the first `nv` rows of kb / vb (T.k / T.v, or a second tile buffer) are
// in place.  `sync` is the item's barrier.  For
// every (head, dim) element i = h * 128 + d of the G heads of head group g a
// thread owns (i = tid + kAttnThreads * r), calls emit(r, h, d, max, sum, O).
template <int G, class Sync, class Emit>
__device__ __forceinline__ void attn_tile_compute_emit(AttnTile<G>& T, const __half* kb, const __half* vb, int nv,
                                                       float scale, Sync sync, Emit emit) {
  constexpr int HD = kHeadDim;
  // the thread index through a volatile read: the per-lane operand addresses
  // below are then formed here, per tile, and never hoisted by the compiler
  // into registers held across a persistent kernel's other phases
  uint32_t tix;
  asm volatile("mov.u32 %0, %%tid.x;" : "=r"(tix));
  const int tid = (int)tix & (kAttnThreads - 1), lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3, l16 = lane & 15;
  // the A-operand image row and column half (hb) an ldmatrix.x4 lane
  // addresses; the head a lane's D row g holds and the sum of its two parts.
  // Every swizzled chunk index below is (2 ks) ^ (lane constant), so each
  // operand address is one per-lane base XOR / plus an immediate per slice.
  const int ar = attn_arow<G>((lane & 7) + ((lane >> 3) & 1) * 8), hb = lane >> 4;
  auto parts = [&](float hi_or_g, float g8) {
    return G == 8 ? hi_or_g + g8 : hi_or_g + __shfl_xor_sync(B2Q_FULL, hi_or_g, 4 * G);
  };
  if (w < 8) {
    // scores: warp w takes keys 8w..8w+7 over the 128 dims (8 k16 slices)
    // q image row ar: chunk 2 ks + hb at (2 ks) ^ (hb ^ (ar & 7)); K row
    // 8w + (l16 & 7) of box ks / 4: chunk 2 (ks & 3) + (l16 >> 3) at
    // (2 (ks & 3)) ^ ((l16 >> 3) ^ (l16 & 7))
    const uint32_t qa = smem_u32(T.qimg) + ar * 256 + ((hb ^ (ar & 7)) << 4);
    const uint32_t ka = smem_u32(kb) + (8 * w + (l16 & 7)) * 128 + ((((l16 >> 3) ^ l16) & 7) << 4);
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4], b0, b1;
      ldsm_x4(a, qa ^ (uint32_t)(ks << 5));
      ldsm_x2(b0, b1, (ka ^ (uint32_t)((ks & 3) << 5)) + (ks >> 2) * (kAttnTile * 128));
      mma_16816(d, a, b0, b1);
    }
    const float s0 = parts(d[0], d[2]), s1 = parts(d[1], d[3]);
    if (g < G) {
      T.sp[g][8 * w + 2 * t] = s0;
      T.sp[g][8 * w + 2 * t + 1] = s1;
    }
  } else if (nv < kAttnTile) {
    // V rows past the valid tokens hold whatever the cache or an earlier
    // tile left: zero them (rows nv.. of both boxes), so that a zero
    // probability never meets an inf or NaN there
    uint32_t* vz = reinterpret_cast<uint32_t*>(const_cast<__half*>(vb));
    const int per = (kAttnTile - nv) * 32;  // words per box
    for (int i = tid - 256; i < 2 * per; i += kAttnThreads - 256) {
      const int bx = i >= per ? 1 : 0;
      vz[bx * (kAttnTile * 32) + nv * 32 + (i - bx * per)] = 0u;
    }
  }
  sync();
  // softmax: warp h takes head h; lane holds tokens lane, lane + 32.  The
  // probability parts overwrite the head's score row after the warp's
  // reductions, so every lane has read its scores by then.
  if (w < G) {
    const int h = w, t0 = lane, t1 = lane + 32;
    const float s0 = t0 < nv ? T.sp[h][t0] * scale : -INFINITY;
    const float s1 = t1 < nv ? T.sp[h][t1] * scale : -INFINITY;
    const float mx = warp_max(fmaxf(s0, s1));
    const float p0 = t0 < nv ? expf(s0 - mx) : 0.0f;
    const float p1 = t1 < nv ? expf(s1 - mx) : 0.0f;
    const float sum = warp_sum(p0 + p1);
    __half* pr = reinterpret_cast<__half*>(T.sp[h]);
    const __half h0 = f16_hi(p0 * kPScale), h1 = f16_hi(p1 * kPScale);
    pr[img_col(h, t0)] = h0;
    pr[img_col(h, t1)] = h1;
    pr[img_col(G + h, kAttnTile + t0)] = f16_lo(p0 * kPScale, h0);
    pr[img_col(G + h, kAttnTile + t1)] = f16_lo(p1 * kPScale, h1);
    if (lane == 0) { T.m[h] = mx; T.l[h] = sum; }
  }
  sync();
  // P * V: warp w takes dims 8w..8w+7 over the 64 keys (4 k16 slices); the
  // output [G][HD] goes over the K rows, no longer read
  float* o = reinterpret_cast<float*>(const_cast<__half*>(kb));
  {
    // probability image row ar (score row ar % G): chunk 8 part + 2 ks + hb
    // at (8 part) ^ (2 ks) ^ (hb ^ (ar & 7)); V rows 16 ks + l16, dims 8w..
    // (box w / 8, chunk w & 7 at (w ^ l16) & 7)
    const uint32_t pa = smem_u32(T.sp[ar % G]) + ((((ar / G) << 3) ^ (hb ^ (ar & 7))) << 4);
    const uint32_t va = smem_u32(vb) + (w >> 3) * (kAttnTile * 128) + l16 * 128 + (((w ^ l16) & 7) << 4);
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < kAttnTile / 16; ++ks) {
      uint32_t a[4], b0, b1;
      ldsm_x4(a, pa ^ (uint32_t)(ks << 5));
      ldsm_x2_t(b0, b1, va + ks * (16 * 128));
      mma_16816(d, a, b0, b1);
    }
    const float o0 = parts(d[0], d[2]), o1 = parts(d[1], d[3]);
    if (g < G) {
      o[g * HD + 8 * w + 2 * t] = o0 * (1.0f / kPScale);
      o[g * HD + 8 * w + 2 * t + 1] = o1 * (1.0f / kPScale);
    }
  }
  sync();
  constexpr int R = (G * HD + kAttnThreads - 1) / kAttnThreads;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = tid + kAttnThreads * r;
    if (i >= G * HD) break;
    const int h = i / HD, d = i % HD;
    emit(r, h, d, T.m[h], T.l[h], o[h * HD + d]);
  }
}

// Write a group partial: part[(h * nsplit + j) * kPartStride] = {max, sum,
// O[128]} for head h = g*G + (element's head).
__device__ __forceinline__ void attn_store_partial(float* part, int g, int G, int j, int nsplit, int h, int d,
                                                   float m, float l, float o) {
  if (!b2q_check(h >= 0 && h < G && j >= 0 && j < nsplit && d >= 0 && d < kHeadDim, kChkPart)) return;
  float* pp = part + ((int64_t)(g * G + h) * nsplit + j) * kPartStride;
  if (d == 0) { pp[0] = m; pp[1] = l; }
  pp[2 + d] = o;
}

// Per-kernel path: grid (KV, m, nsplit), kAttnThreads threads,
// sizeof(AttnTile<G>) + kAttnAlignPad bytes of dynamic shared memory; tmk /
// tmv are the TMA descriptors of the layer's K and V caches (global memory).  Query s sits at
// position start+s and sees keys t < start+s+1 (causal); q was rotated in
// place by rope_kv_kernel.  Block (g, s, j) folds the key tiles of group j
// (attn_group_tiles with `grid` = the SM count) into one partial.
template <int G>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(
    const float* __restrict__ qkv, int m, int H, int KV, const int* __restrict__ pos_dev, int cap,
    const void* tmk, const void* tmv, float scale, int nsplit, float* __restrict__ part, int grid) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ uint64_t bar;
  AttnTile<G>& T = *reinterpret_cast<AttnTile<G>*>(smem_align1024(attn_smem));
  pdl_wait();
  pdl_launch_dependents();
  constexpr int HD = kHeadDim;
  constexpr int R = (G * HD + kAttnThreads - 1) / kAttnThreads;
  const int g = blockIdx.x, s = blockIdx.y, j = blockIdx.z;
  const int start = *pos_dev;
  const int valid = min(start + s + 1, cap);
  const int nz = (valid + kAttnTile - 1) / kAttnTile;
  const int tpg = attn_group_tiles(nz, KV, grid);
  const int z0 = j * tpg, z1 = min(nz, z0 + tpg);
  float* ps = part + (int64_t)s * H * nsplit * kPartStride;
  if (z0 >= nz) {
    if (threadIdx.x < G) {
      float* p = ps + ((int64_t)(g * G + threadIdx.x) * nsplit + j) * kPartStride;
      p[0] = -INFINITY;
      p[1] = 0.0f;
    }
    return;
  }
  if (kChecks && !b2q_check(g < KV && (z1 - 1) * kAttnTile < cap &&
                                smem_u32(&T) + sizeof(AttnTile<G>) <= smem_u32(attn_smem) + dyn_smem_bytes(),
                            kChkAttnRows))
    return;  // (uniform over the CTA)
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    attn_rows_load(T.k, T.v, tmk, tmv, g * cap + z0 * kAttnTile, &bar);
  }
  const int width = (H + 2 * KV) * HD;
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) attn_set_q(T, i / HD, i % HD, qkv[(int64_t)s * width + g * G * HD + i]);
  AttnRun<R> run;
  run.init();
  for (int z = z0; z < z1; ++z) {
    const int t_begin = z * kAttnTile, nv = min(kAttnTile, valid - t_begin);
    __syncthreads();  // q in place / the previous tile's shared-memory reads are done
    if (z > z0 && threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      attn_rows_load(T.k, T.v, tmk, tmv, g * cap + t_begin, &bar);
    }
    mbar_wait_bounded(&bar, (uint32_t)((z - z0) & 1));  // a timeout is recorded in the device error word
    attn_tile_compute_emit<G>(T, T.k, T.v, nv, scale, [] { __syncthreads(); },
                              [&](int r, int, int, float mt, float lt, float ot) { run.fold(r, mt, lt, ot); });
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = threadIdx.x + kAttnThreads * r;
    if (i < G * HD) attn_store_partial(ps, g, G, j, nsplit, i / HD, i % HD, run.m[r], run.l[r], run.o[r]);
  }
}

// Merge the split partials of every head, normalise (inv_sum =
// 1/max(sum, 1e-12), inference.rs:2816), write attn [m][H*hd] and quantise it
// for the o-projection.  grid (KV, m), G*128 threads (one per output dim).
__global__ void attn_combine_kernel(const float* __restrict__ part, int m, int H, int G,
                                    const int* __restrict__ pos_dev, int cap, int nsplit,
                                    float* __restrict__ out, XQ xq, int grid) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int HD = kHeadDim;
  __shared__ float vals[8 * HD];
  const int g = blockIdx.x, s = blockIdx.y;
  const int h = g * G + threadIdx.x / HD, d = threadIdx.x % HD;
  const int start = *pos_dev;
  const int valid = min(start + s + 1, cap);
  const int nz = (valid + kAttnTile - 1) / kAttnTile;
  const int tpg = attn_group_tiles(nz, H / G, grid);
  const int ns = min(nsplit, (nz + tpg - 1) / tpg);  // groups
  const float* pp = part + ((int64_t)s * H + h) * nsplit * kPartStride;
  float M = -INFINITY;
  for (int z = 0; z < ns; ++z) M = fmaxf(M, pp[z * kPartStride]);
  float L = 0.0f, O = 0.0f;
  for (int z = 0; z < ns; ++z) {
    const float mz = pp[z * kPartStride];
    const float f = mz == -INFINITY ? 0.0f : expf(mz - M);
    L = fmaf(f, pp[z * kPartStride + 1], L);
    O = fmaf(f, pp[z * kPartStride + 2 + d], O);
  }
  const float v = O * (1.0f / fmaxf(L, 1e-12f));
  const int col0 = g * G * HD;
  out[(int64_t)s * H * HD + col0 + threadIdx.x] = v;
  vals[threadIdx.x] = v;
  __syncthreads();
  // quantise: warp w < 2G takes the 64-element block w of this KV group
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < 2 * G)
    xq_store_block(vals[64 * warp + lane], vals[64 * warp + 32 + lane], lane, s, (col0 >> 6) + warp, xq);
}

// ---------------------------------------------------------------------------
// Prompt-pass attention (m >= 16 queries, the tensor-core projection path):
// one CTA of 4 warps takes 64 query rows -- 64 / G consecutive tokens times
// the G query heads of KV head g, row r = token (r / G), head (r % G) -- and
// runs over the key tiles up to its last token with a running softmax
// (inference.rs:2782-2833 for each query: scores q.k * scale over the keys
// t <= position, softmax, P.V, normalised by 1/max(sum, 1e-12)).  K and V
// tiles arrive by TMA (the decode tiles' 128-byte-swizzled layout, two
// buffers, the next tile in flight); the products run on mma.sync
// m16n8k16 with the f32 queries and probabilities each split into f16 hi
// and lo fragments (two MMAs per product, ~2^-22 relative) and the f16 K/V
// entering exactly.  Warp w owns rows 16w..16w+15: its S tile (16 x 64) and
// its output (16 x 128) stay in registers; the S accumulator fragments of
// two adjacent key octets are the A fragment of the P.V k-slice.
// grid (KV, ceil(m / (64 / G))), 128 threads, kAttnPrefillSmem bytes of
// dynamic shared memory.
// ---------------------------------------------------------------------------
constexpr int kAttnPrefillSmem = 2 * (int)kAttnTileBytes + 1024;

__device__ __forceinline__ void f16_split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half ha = f16_hi(a), hb = f16_hi(b);
  const __half la = f16_lo(a, ha), lb = f16_lo(b, hb);
  hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
  lo = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}

template <int G>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const float* __restrict__ qkv, int m, int H, int KV,
                                                            const int* __restrict__ pos_dev, int cap,
                                                            const void* tmk, const void* tmv, float scale,
                                                            float* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ uint64_t bars[2];
  constexpr int HD = kHeadDim, QT = 64 / G;  // tokens per CTA
  pdl_wait();
  pdl_launch_dependents();
  const int g = blockIdx.x, s0 = blockIdx.y * QT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
  const int start = *pos_dev;
  const int s_last = min(m, s0 + QT) - 1;
  const int nkeys = min(start + s_last + 1, cap);  // keys of the block's last query
  const int ntiles = (nkeys + kAttnTile - 1) / kAttnTile;
  uint8_t* base = smem_align1024(attn_smem);
  __half* kb[2] = {reinterpret_cast<__half*>(base), reinterpret_cast<__half*>(base + kAttnTileBytes)};
  if (kChecks && !b2q_check(g < KV && smem_u32(base) + 2 * kAttnTileBytes <= smem_u32(attn_smem) + dyn_smem_bytes(),
                            kChkAttnRows))
    return;  // (uniform over the CTA)
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    attn_rows_load(kb[0], kb[0] + kAttnTile * HD, tmk, tmv, g * cap, &bars[0]);
  }
  // this thread's two rows (gq and gq + 8 of the warp's 16) and their query positions
  const int width = (H + 2 * KV) * HD;
  const int r0 = 16 * warp + gq, r1 = r0 + 8;
  const int tok0 = s0 + r0 / G, tok1 = s0 + r1 / G;
  const int qp0 = start + tok0, qp1 = start + tok1;
  // Q fragments (hi, lo) for the 8 k16 slices of the 128 dims
  uint32_t qh[8][4], ql[8][4];
  {
    const float* q0 = qkv + (int64_t)min(tok0, m - 1) * width + (g * G + r0 % G) * HD;
    const float* q1 = qkv + (int64_t)min(tok1, m - 1) * width + (g * G + r1 % G) * HD;
    const bool v0 = tok0 < m, v1 = tok1 < m;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int c = 16 * ks + 2 * t;
      const float2 a = v0 ? *reinterpret_cast<const float2*>(q0 + c) : make_float2(0.f, 0.f);
      const float2 b = v1 ? *reinterpret_cast<const float2*>(q1 + c) : make_float2(0.f, 0.f);
      const float2 cc = v0 ? *reinterpret_cast<const float2*>(q0 + c + 8) : make_float2(0.f, 0.f);
      const float2 d = v1 ? *reinterpret_cast<const float2*>(q1 + c + 8) : make_float2(0.f, 0.f);
      f16_split2(a.x, a.y, qh[ks][0], ql[ks][0]);
      f16_split2(b.x, b.y, qh[ks][1], ql[ks][1]);
      f16_split2(cc.x, cc.y, qh[ks][2], ql[ks][2]);
      f16_split2(d.x, d.y, qh[ks][3], ql[ks][3]);
    }
  }
  __syncthreads();  // the barriers are initialised
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float mx0 = -INFINITY, mx1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const int l16 = lane & 15;
  for (int z = 0; z < ntiles; ++z) {
    const int b = z & 1;
    if (threadIdx.x == 0 && z + 1 < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      attn_rows_load(kb[b ^ 1], kb[b ^ 1] + kAttnTile * HD, tmk, tmv, g * cap + (z + 1) * kAttnTile, &bars[b ^ 1]);
    }
    mbar_wait_bounded(&bars[b], (uint32_t)((z >> 1) & 1));  // a timeout is recorded in the device error word
    const __half* K = kb[b];
    const __half* V = kb[b] + kAttnTile * HD;
    // S = Q K^T: 16 rows x 64 keys, 8 key octets
    float sc[8][4];
    const uint32_t ka = smem_u32(K) + (l16 & 7) * 128 + ((((l16 >> 3) ^ l16) & 7) << 4);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        uint32_t b0, b1;
        ldsm_x2(b0, b1, ((ka + nt * 8 * 128) ^ (uint32_t)((ks & 3) << 5)) + (ks >> 2) * (kAttnTile * 128));
        mma_16816(sc[nt], qh[ks], b0, b1);
        mma_16816(sc[nt], ql[ks], b0, b1);
      }
    }
    // scale, causal mask, running max
    const int kp0 = z * kAttnTile;
    float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = kp0 + 8 * nt + 2 * t + e;
        sc[nt][e] = kp <= qp0 && kp < nkeys ? sc[nt][e] * scale : -INFINITY;
        sc[nt][2 + e] = kp <= qp1 && kp < nkeys ? sc[nt][2 + e] * scale : -INFINITY;
        tm0 = fmaxf(tm0, sc[nt][e]);
        tm1 = fmaxf(tm1, sc[nt][2 + e]);
      }
    }
    tm0 = fmaxf(tm0, __shfl_xor_sync(B2Q_FULL, tm0, 1));
    tm0 = fmaxf(tm0, __shfl_xor_sync(B2Q_FULL, tm0, 2));
    tm1 = fmaxf(tm1, __shfl_xor_sync(B2Q_FULL, tm1, 1));
    tm1 = fmaxf(tm1, __shfl_xor_sync(B2Q_FULL, tm1, 2));
    const float nm0 = fmaxf(mx0, tm0), nm1 = fmaxf(mx1, tm1);
    // rows with no key yet keep m = -inf and contribute nothing
    const float al0 = nm0 == -INFINITY ? 1.0f : expf(mx0 - nm0), al1 = nm1 == -INFINITY ? 1.0f : expf(mx1 - nm1);
    mx0 = nm0;
    mx1 = nm1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    // P = exp(S - m) (scaled by 2^15 out of the f16 subnormal range) as A
    // fragments of the 4 key slices, then O += P V
#pragma unroll
    for (int ks = 0; ks < kAttnTile / 16; ++ks) {
      uint32_t ph[4], pl[4];
      float p[2][4];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float sv = sc[2 * ks + hh][e];
          const float pe = sv == -INFINITY ? 0.0f : expf(sv - (e < 2 ? nm0 : nm1));
          p[hh][e] = pe;
          if (e < 2) l0 += pe;
          else l1 += pe;
        }
      f16_split2(p[0][0] * kPScale, p[0][1] * kPScale, ph[0], pl[0]);
      f16_split2(p[0][2] * kPScale, p[0][3] * kPScale, ph[1], pl[1]);
      f16_split2(p[1][0] * kPScale, p[1][1] * kPScale, ph[2], pl[2]);
      f16_split2(p[1][2] * kPScale, p[1][3] * kPScale, ph[3], pl[3]);
      const uint32_t va = smem_u32(V) + (16 * ks + l16) * 128;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        uint32_t b0, b1;
        ldsm_x2_t(b0, b1, va + (n >> 3) * (kAttnTile * 128) + (((n ^ l16) & 7) << 4));
        mma_16816(o[n], ph, b0, b1);
        mma_16816(o[n], pl, b0, b1);
      }
    }
    __syncthreads();  // buffer b is free for the tile after next
  }
  // row sums across the quad, normalise, store
  l0 += __shfl_xor_sync(B2Q_FULL, l0, 1);
  l0 += __shfl_xor_sync(B2Q_FULL, l0, 2);
  l1 += __shfl_xor_sync(B2Q_FULL, l1, 1);
  l1 += __shfl_xor_sync(B2Q_FULL, l1, 2);
  const float i0 = (1.0f / kPScale) * (1.0f / fmaxf(l0, 1e-12f)), i1 = (1.0f / kPScale) * (1.0f / fmaxf(l1, 1e-12f));
  float* o0 = out + (int64_t)tok0 * H * HD + (g * G + r0 % G) * HD;
  float* o1 = out + (int64_t)tok1 * H * HD + (g * G + r1 % G) * HD;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = 8 * n + 2 * t;
    if (tok0 < m) *reinterpret_cast<float2*>(o0 + d) = make_float2(o[n][0] * i0, o[n][1] * i0);
    if (tok1 < m) *reinterpret_cast<float2*>(o1 + d) = make_float2(o[n][2] * i1, o[n][3] * i1);
  }
}

// Seeded synthetic KV rows (benchmark set-up: a long context without a
// prompt pass).  Element e of the K (kv = 0) or V (kv = 1) row of global KV
// head h at position t in layer l is u * scale, u in [-1, 1) from a 64-bit
// mix (splitmix64 finaliser) of (seed, l, kv, h, t, e), rounded to f16; the
// global head index makes a tensor-parallel rank's rows those of one GPU.
// grid (positions, local KV heads), block kHeadDim.
__global__ void kv_fill_kernel(__half* __restrict__ kc, __half* __restrict__ vc, int max_seq, int t0,
                               int layer, int head0, uint64_t seed, float scale) {
  const int t = t0 + (int)blockIdx.x, g = (int)blockIdx.y, e = (int)threadIdx.x;
  const int64_t off = ((int64_t)g * max_seq + t) * kHeadDim + e;
  for (int kv = 0; kv < 2; ++kv) {
    uint64_t z = seed ^ ((uint64_t)layer << 48) ^ ((uint64_t)kv << 47) ^ ((uint64_t)(head0 + g) << 38) ^
                 ((uint64_t)t << 8) ^ (uint64_t)e;
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    z ^= z >> 31;
    const float u = (float)(z >> 40) * (1.0f / 8388608.0f) - 1.0f;  // 24 bits -> [-1, 1)
    (kv ? vc : kc)[off] = __float2half_rn(u * scale);
  }
}

// Step inputs written by a kernel (parameters are captured at launch), so
// asynchronous callers never race on a reused host staging slot.
__global__ void set_step_kernel(int* __restrict__ pos_dev, int pos, uint32_t* __restrict__ tokens_dev,
                                const uint32_t* __restrict__ src, int n, int vocab) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *pos_dev = pos;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t t = src[i];
    tokens_dev[i] = t < (uint32_t)vocab ? t : 0u;
  }
}

// Greedy argmax over [n] logits: first index of the maximum, as the
// reference's strict `>` scan (inference.rs:1621-1629).  One CTA.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ v, int n,
                                                      uint32_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float bv[32];
  __shared__ int bi[32];
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x > best) { best = x; idx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(B2Q_FULL, best, o);
    const int oi = __shfl_xor_sync(B2Q_FULL, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? bv[lane] : -INFINITY;
    idx = lane < nw ? bi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(B2Q_FULL, best, o);
      const int oi = __shfl_xor_sync(B2Q_FULL, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) *out = idx == 0x7fffffff ? 0u : (uint32_t)idx;
  }
}

}  // namespace b2q
