// gdn.cuh -- the Gated DeltaNet state update of the reference's Qwen3.5
// hybrid model (src/inference.rs:2281-2374 with ssm_head_step_avx2,
// :1535-1583), one token at a time.
//
// Per token, after the quad projection (attn_qkv, attn_gate = z, ssm_alpha,
// ssm_beta):
//   conv:  c_out[c] = silu(sum_k state[c][k] * w[c][k] + x[c] * w[c][K-1]),
//          then the channel's history shifts by one (x appended);
//   q, k:  the first 2 * n_k_heads * d_k channels, L2-normalised per head
//          (x / sqrt(sum x^2 + eps));
//   head vh (k head vh % n_k_heads): beta = sigmoid(beta_raw),
//          g = exp(softplus(alpha + dt_bias) * a); for every row i of the
//          state S [d_v][d_k]: d = (v_i - g * (S_i . k)) * beta,
//          S_i = g * S_i + d * k, o_i = (S_i . q) / sqrt(d_k);
//   out:   y = o * rsqrt(mean(o^2) + eps) * ssm_norm * silu(z).
// gdn_conv_kernel does the convolution (one thread per channel); the head
// step runs one CTA per value head, a warp per state row at a time (lane:
// four consecutive columns, the row read and written as float4, the two dot
// products as warp reductions).  The state stays in HBM between tokens
// (n_v_heads * d_v * d_k f32, 2 MB at 32 x 128 x 128; it lives in L2 while
// a token's layers run).
#pragma once

#include "common.cuh"

namespace b2q {

constexpr int kGdnThreads = 256;  // 8 warps per value head

__device__ __forceinline__ float gdn_silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gdn_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float gdn_softplus(float x) {
  return x > 20.0f ? x : x < -20.0f ? expf(x) : logf(1.0f + expf(x));
}

// x: [channels] this token's qkv projection; state: [channels][K-1];
// w: [channels][K]; out: [channels].
__global__ void gdn_conv_kernel(const float* __restrict__ x, float* __restrict__ state,
                                const float* __restrict__ w, int channels, int K, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= channels) return;
  const int hist = K - 1;
  float* st = state + (size_t)c * hist;
  const float* wc = w + (size_t)c * K;
  float acc = 0.0f;
  for (int k = 0; k < hist; ++k) acc = __fadd_rn(acc, __fmul_rn(st[k], wc[k]));
  acc = __fadd_rn(acc, __fmul_rn(x[c], wc[hist]));
  out[c] = gdn_silu(acc);
  for (int k = 0; k + 1 < hist; ++k) st[k] = st[k + 1];
  if (hist > 0) st[hist - 1] = x[c];
}

// One CTA per value head.  conv: [channels] (q | k | v); S: [n_v][d_v][d_k];
// z: [n_v * d_v]; y: [n_v * d_v].  d_k must be 128 (one float4 per lane).
__global__ void __launch_bounds__(kGdnThreads) gdn_head_kernel(
    const float* __restrict__ conv, float* __restrict__ S, const float* __restrict__ z,
    const float* __restrict__ alpha, const float* __restrict__ beta_raw, const float* __restrict__ ssm_a,
    const float* __restrict__ dt_bias, const float* __restrict__ ssm_norm, int n_k, int d_k, int d_v, float eps,
    float* __restrict__ y) {
  __shared__ float4 qs[32], ks[32];
  __shared__ float red[kGdnThreads / 32];
  __shared__ float o_sh[512];
  const int vh = blockIdx.x, kh = vh % n_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qsrc = conv + (size_t)kh * d_k;
  const float* ksrc = conv + (size_t)n_k * d_k + (size_t)kh * d_k;
  const float* vsrc = conv + (size_t)2 * n_k * d_k + (size_t)vh * d_v;
  // L2-normalised q (warp 0) and k (warp 1)
  if (warp < 2) {
    const float4 v = reinterpret_cast<const float4*>(warp == 0 ? qsrc : ksrc)[lane];
    float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss + eps);
    const float4 n = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
    if (warp == 0) qs[lane] = n;
    else ks[lane] = n;
  }
  __syncthreads();
  const float beta = gdn_sigmoid(beta_raw[vh]);
  const float g = expf(gdn_softplus(alpha[vh] + dt_bias[vh]) * ssm_a[vh]);
  const float scale = 1.0f / sqrtf((float)d_k);
  const float4 q4 = qs[lane], k4 = ks[lane];
  float* Sh = S + (size_t)vh * d_v * d_k;
  for (int i = warp; i < d_v; i += kGdnThreads / 32) {
    float4* row = reinterpret_cast<float4*>(Sh + (size_t)i * d_k);
    float4 s = row[lane];
    const float sk = warp_sum(s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w);
    const float d = (vsrc[i] - g * sk) * beta;
    s.x = fmaf(d, k4.x, g * s.x);
    s.y = fmaf(d, k4.y, g * s.y);
    s.z = fmaf(d, k4.z, g * s.z);
    s.w = fmaf(d, k4.w, g * s.w);
    row[lane] = s;
    const float o = warp_sum(s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w);
    if (lane == 0) o_sh[i] = o * scale;
  }
  __syncthreads();
  // RMS norm over the head's outputs, times ssm_norm and silu(z)
  float ss = 0.0f;
  for (int i = threadIdx.x; i < d_v; i += kGdnThreads) ss += o_sh[i] * o_sh[i];
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < kGdnThreads / 32; ++w) tot += red[w];
  const float inv = 1.0f / sqrtf(tot / (float)d_v + eps);
  for (int i = threadIdx.x; i < d_v; i += kGdnThreads) {
    const size_t o = (size_t)vh * d_v + i;
    y[o] = o_sh[i] * inv * ssm_norm[i] * gdn_silu(z[o]);
  }
}

}  // namespace b2q
