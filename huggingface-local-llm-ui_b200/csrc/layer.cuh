// layer.cuh -- the per-layer operations around the GEMVs in the Llama
// block (StandardNativeEngine::forward, inference.rs:2695-2860): RMSNorm,
// NeoX RoPE, KV-cache append, GQA attention, and greedy argmax.
#pragma once

#include "quant.cuh"

namespace b2q {

constexpr int kAttnTile = 128;  // tokens per attention split (4 warps x 32)
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
  for (int e = threadIdx.x; e < dim; e += blockDim.x) ss += xr[e] * xr[e];
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

// Split-T GQA attention for queries at positions start+s (causal: keys
// t < start+s+1).  grid (KV, m, nsplit), 128 threads.  One lane per key
// token for the scores, one lane per 4 head dims for P*V, an online softmax
// per warp, merged across the CTA's 4 warps; the split partials
// (max, sum, out[hd]) go to `part` and are merged by attn_combine_kernel.
template <int G>
__global__ void __launch_bounds__(128) attn_split_kernel(
    const float* __restrict__ qkv, int m, int H, int KV, const int* __restrict__ pos_dev, int cap,
    const __half* __restrict__ kc, const __half* __restrict__ vc, float scale, int nsplit,
    float* __restrict__ part) {
  pdl_wait();
  constexpr int HD = kHeadDim;
  __shared__ float qs[G][HD];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wo[4][G][HD];
  const int g = blockIdx.x, s = blockIdx.y, z = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int start = *pos_dev;
  const int valid = min(start + s + 1, cap);
  const int t_begin = z * kAttnTile;
  const int width = (H + 2 * KV) * HD;
  float* pm = part + (((int64_t)s * H + g * G) * nsplit + z) * (HD + 2);
  if (t_begin >= valid) {
    if (threadIdx.x < G) {
      float* p = part + (((int64_t)s * H + g * G + threadIdx.x) * nsplit + z) * (HD + 2);
      p[0] = -INFINITY;
      p[1] = 0.0f;
    }
    return;
  }
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x)
    qs[i / HD][i % HD] = qkv[(int64_t)s * width + (g * G) * HD + i];
  __syncthreads();

  const int t = t_begin + warp * 32 + lane;
  const bool tv = t < valid;
  float sc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) sc[h] = 0.0f;
  if (tv) {
    const uint4* kr = reinterpret_cast<const uint4*>(kc + ((int64_t)g * cap + t) * HD);
#pragma unroll 4
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 pk = kr[c];
      const __half2* h2 = reinterpret_cast<const __half2*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kf = __half22float2(h2[e]);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          sc[h] = fmaf(qs[h][c * 8 + 2 * e], kf.x, sc[h]);
          sc[h] = fmaf(qs[h][c * 8 + 2 * e + 1], kf.y, sc[h]);
        }
      }
    }
  }
  float mx[G], l[G], p[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float sv = tv ? sc[h] * scale : -INFINITY;
    mx[h] = warp_max(sv);
    p[h] = tv ? expf(sv - mx[h]) : 0.0f;
    l[h] = warp_sum(p[h]);
  }
  // P * V over this warp's 32 tokens; lane owns dims 4*lane .. 4*lane+3
  float o[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[h][e] = 0.0f;
  const int nt = min(32, valid - (t_begin + warp * 32));
  for (int src = 0; src < nt; ++src) {
    const int ts = t_begin + warp * 32 + src;
    const uint2 pv = *reinterpret_cast<const uint2*>(vc + ((int64_t)g * cap + ts) * HD + 4 * lane);
    const __half2* v2 = reinterpret_cast<const __half2*>(&pv);
    const float2 va = __half22float2(v2[0]), vb = __half22float2(v2[1]);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float ph = __shfl_sync(B2Q_FULL, p[h], src);
      o[h][0] = fmaf(ph, va.x, o[h][0]);
      o[h][1] = fmaf(ph, va.y, o[h][1]);
      o[h][2] = fmaf(ph, vb.x, o[h][2]);
      o[h][3] = fmaf(ph, vb.y, o[h][3]);
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) { wm[warp][h] = mx[h]; wl[warp][h] = l[h]; }
  }
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) wo[warp][h][4 * lane + e] = o[h][e];
  __syncthreads();
  // merge the 4 warps: thread handles (h, d) pairs
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < 4; ++w2) M = fmaxf(M, wm[w2][h]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < 4; ++w2) {
      const float f = wm[w2][h] == -INFINITY ? 0.0f : expf(wm[w2][h] - M);
      L += f * wl[w2][h];
      O += f * wo[w2][h][d];
    }
    float* pp = pm + (int64_t)h * nsplit * (HD + 2);
    if (d == 0) { pp[0] = M; pp[1] = L; }
    pp[2 + d] = O;
  }
  pdl_launch_dependents();
}

// Merge the split partials of every head, normalise (inv_sum =
// 1/max(sum, 1e-12), inference.rs:2816), write attn [m][H*hd] and quantise it
// for the o-projection.  grid (KV, m), G*128 threads (one per output dim).
__global__ void attn_combine_kernel(const float* __restrict__ part, int m, int H, int G,
                                    const int* __restrict__ pos_dev, int cap, int nsplit,
                                    float* __restrict__ out, XQ xq) {
  pdl_wait();
  constexpr int HD = kHeadDim;
  __shared__ float vals[8 * HD];
  const int g = blockIdx.x, s = blockIdx.y;
  const int h = g * G + threadIdx.x / HD, d = threadIdx.x % HD;
  const int start = *pos_dev;
  const int valid = min(start + s + 1, cap);
  const int ns = min(nsplit, (valid + kAttnTile - 1) / kAttnTile);
  const float* pp = part + ((int64_t)s * H + h) * nsplit * (HD + 2);
  float M = -INFINITY;
  for (int z = 0; z < ns; ++z) M = fmaxf(M, pp[z * (HD + 2)]);
  float L = 0.0f, O = 0.0f;
  for (int z = 0; z < ns; ++z) {
    const float mz = pp[z * (HD + 2)];
    const float f = mz == -INFINITY ? 0.0f : expf(mz - M);
    L += f * pp[z * (HD + 2) + 1];
    O += f * pp[z * (HD + 2) + 2 + d];
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
