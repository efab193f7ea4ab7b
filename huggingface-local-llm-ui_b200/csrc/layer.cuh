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
  pdl_launch_dependents();
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
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Split GQA attention over the f16 KV cache (inference.rs:2782-2820).  The
// cached keys of a query are cut into splits of kAttnTile tokens; one item =
// (KV head g, split z) on kAttnThreads threads computes, for the G query
// heads of g, the split's softmax partial (max, sum, unnormalised P*V).  The
// K and V rows of the split are brought into shared memory with two bulk
// async copies (one round trip to HBM), then everything runs from shared
// memory.  The same item code serves the per-kernel path
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
constexpr int kQImgStride = kHeadDim + 8;   // halves per query image row (ldmatrix rows on distinct banks)
constexpr int kSpStride = kAttnTile + 4;    // floats per score row
constexpr float kPScale = 32768.0f;

template <int G>
struct AttnTile {
  __half k[kAttnTile * kHeadDim];  // rows t_begin.. of the split (then the P*V output)
  __half v[kAttnTile * kHeadDim];
  __half qimg[2 * G * kQImgStride];  // rotated queries: hi rows 0..G-1, lo rows G..2G-1
  float sp[G][kSpStride];            // scores; then the probabilities' hi (bytes 0..127) and lo
                                     // (bytes 128..255) f16 parts, over each head's own row
  float m[G], l[G];                  // softmax max and sum per head
  __half kcur[kHeadDim];             // the current token's rotated k and its v (persistent
  __half vcur[kHeadDim];             // kernel: copied into the tile that holds the token)
};

__device__ __forceinline__ __half f16_hi(float v) { return __float2half_rz(v); }
__device__ __forceinline__ __half f16_lo(float v, __half hi) { return __float2half_rn(v - __half2float(hi)); }

template <int G>
__device__ __forceinline__ void attn_set_q(AttnTile<G>& T, int h, int d, float v) {
  const __half hi = f16_hi(v);
  T.qimg[h * kQImgStride + d] = hi;
  T.qimg[(G + h) * kQImgStride + d] = f16_lo(v, hi);
}

// Image row (head h + G * part, part 0 hi / 1 lo) behind A-operand row r
// (0..15) of an m16n8k16 product
template <int G>
__device__ __forceinline__ int attn_arow(int r) { return G == 8 ? r : r % (2 * G); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
// d += a * b, m16n8k16, f16 x f16 -> f32
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Issue the bulk copies of K/V rows [t0, t0 + rows) of KV head g into kb /
// vb (shared memory; one thread); completes on `bar` (expect_tx included).
__device__ __forceinline__ void attn_rows_load(__half* kb, __half* vb, const __half* kc, const __half* vc, int g,
                                               int cap, int t0, int rows, uint64_t* bar) {
  const uint32_t bytes = (uint32_t)rows * kHeadDim * 2;
  mbar_arrive_expect_tx(bar, 2 * bytes);
  bulk_g2s(kb, kc + ((int64_t)g * cap + t0) * kHeadDim, bytes, bar);
  bulk_g2s(vb, vc + ((int64_t)g * cap + t0) * kHeadDim, bytes, bar);
}

template <int G>
__device__ __forceinline__ void attn_tile_load(AttnTile<G>& T, const __half* kc, const __half* vc, int g, int cap,
                                               int t0, int rows, uint64_t* bar) {
  attn_rows_load(T.k, T.v, kc, vc, g, cap, t0, rows, bar);
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
// and the first `nv` rows of kb / vb (T.k / T.v, or a second tile buffer; vb
// must follow kb directly) are in place.  `sync` is the item's barrier.  For
// every (head, dim) element i = h * 128 + d of the G heads of head group g a
// thread owns (i = tid + kAttnThreads * r), calls emit(r, h, d, max, sum, O).
template <int G, class Sync, class Emit>
__device__ __forceinline__ void attn_tile_compute_emit(AttnTile<G>& T, const __half* kb, const __half* vb, int nv,
                                                       float scale, Sync sync, Emit emit) {
  constexpr int HD = kHeadDim;
  const int tid = threadIdx.x & (kAttnThreads - 1), lane = threadIdx.x & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3, l16 = lane & 15;
  // the A-operand row (as head and part) and column half an ldmatrix.x4 lane
  // addresses; the head a lane's D row g holds and the sum of its two parts
  const int ar = attn_arow<G>((lane & 7) + ((lane >> 3) & 1) * 8), acol = (lane >> 4) * 8;
  auto parts = [&](float hi_or_g, float g8) {
    return G == 8 ? hi_or_g + g8 : hi_or_g + __shfl_xor_sync(B2Q_FULL, hi_or_g, 4 * G);
  };
  if (w < 8) {
    // scores: warp w takes keys 8w..8w+7 over the 128 dims (8 k16 slices)
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4], b0, b1;
      ldsm_x4(a, T.qimg + ar * kQImgStride + 16 * ks + acol);
      ldsm_x2(b0, b1, kb + (8 * w + (l16 & 7)) * HD + 16 * ks + (l16 >> 3) * 8);
      mma_16816(d, a, b0, b1);
    }
    const float s0 = parts(d[0], d[2]), s1 = parts(d[1], d[3]);
    if (g < G) {
      T.sp[g][8 * w + 2 * t] = s0;
      T.sp[g][8 * w + 2 * t + 1] = s1;
    }
  } else if (nv < kAttnTile) {
    // V rows past the tile's end hold stale shared memory: zero them, so that
    // a zero probability never meets an inf or NaN there
    uint32_t* vz = reinterpret_cast<uint32_t*>(const_cast<__half*>(vb) + nv * HD);
    for (int i = tid - 256; i < (kAttnTile - nv) * HD / 2; i += kAttnThreads - 256) vz[i] = 0u;
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
    pr[t0] = h0;
    pr[t1] = h1;
    pr[kAttnTile + t0] = f16_lo(p0 * kPScale, h0);
    pr[kAttnTile + t1] = f16_lo(p1 * kPScale, h1);
    if (lane == 0) { T.m[h] = mx; T.l[h] = sum; }
  }
  sync();
  // P * V: warp w takes dims 8w..8w+7 over the 64 keys (4 k16 slices); the
  // output [G][HD] goes over the K rows, no longer read
  float* o = reinterpret_cast<float*>(const_cast<__half*>(kb));
  {
    const __half* pa = reinterpret_cast<const __half*>(T.sp[ar % G]) + (ar / G) * kAttnTile + acol;
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < kAttnTile / 16; ++ks) {
      uint32_t a[4], b0, b1;
      ldsm_x4(a, pa + 16 * ks);
      ldsm_x2_t(b0, b1, vb + (16 * ks + l16) * HD + 8 * w);
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
  float* pp = part + ((int64_t)(g * G + h) * nsplit + j) * kPartStride;
  if (d == 0) { pp[0] = m; pp[1] = l; }
  pp[2 + d] = o;
}

// Per-kernel path: grid (KV, m, nsplit), kAttnThreads threads,
// sizeof(AttnTile<G>) bytes of dynamic shared memory.  Query s sits at
// position start+s and sees keys t < start+s+1 (causal); q was rotated in
// place by rope_kv_kernel.  Block (g, s, j) folds the key tiles of group j
// (attn_group_tiles with `grid` = the SM count) into one partial.
template <int G>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(
    const float* __restrict__ qkv, int m, int H, int KV, const int* __restrict__ pos_dev, int cap,
    const __half* __restrict__ kc, const __half* __restrict__ vc, float scale, int nsplit,
    float* __restrict__ part, int grid) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ uint64_t bar;
  AttnTile<G>& T = *reinterpret_cast<AttnTile<G>*>(attn_smem);
  pdl_wait();
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
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    attn_tile_load(T, kc, vc, g, cap, z0 * kAttnTile, min(kAttnTile, valid - z0 * kAttnTile), &bar);
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
      attn_tile_load(T, kc, vc, g, cap, t_begin, nv, &bar);
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
  pdl_launch_dependents();
}

// Merge the split partials of every head, normalise (inv_sum =
// 1/max(sum, 1e-12), inference.rs:2816), write attn [m][H*hd] and quantise it
// for the o-projection.  grid (KV, m), G*128 threads (one per output dim).
__global__ void attn_combine_kernel(const float* __restrict__ part, int m, int H, int G,
                                    const int* __restrict__ pos_dev, int cap, int nsplit,
                                    float* __restrict__ out, XQ xq, int grid) {
  pdl_wait();
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
  pdl_launch_dependents();
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
  pdl_launch_dependents();
}

}  // namespace b2q
