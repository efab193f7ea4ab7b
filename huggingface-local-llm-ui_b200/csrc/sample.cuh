// sample.cuh -- temperature / top-p sampling of the next token on the device
// (SelfMadeSampler::sample, src/inference.rs:1619-1681).
//
// The reference keeps the candidates within 14 * temperature of the max
// logit, weighs them p = exp((v - max) / T), sorts them by p (descending),
// keeps the shortest prefix whose mass reaches top_p * sum, and walks that
// prefix with r = u * min(prefix mass, sum), u from its xorshift64 state.
// One CTA does the same without sorting: the prefix of a descending order
// is a threshold on p, so the cut and the element r falls on are both
// found by bisection over the bit patterns of p (positive floats order like
// their bits), with ties at a threshold taken in index order.  Masses are
// tree sums, not the reference's running sums, and exp is the device's:
// the token equals the reference's except when r falls within rounding of a
// boundary between two candidates.  The random number u is drawn on the
// host (the state never leaves it); out[1] tells whether it was used.
#pragma once

#include <cfloat>

#include "common.cuh"

namespace b2q {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
  return warp_sum(v);
}

__device__ __forceinline__ int block_sum_i(int v, int* red) {
  v = __reduce_add_sync(B2Q_FULL, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0;
  return __reduce_add_sync(B2Q_FULL, v);
}

// Mass of the candidates with p >= t (bit pattern tb), and of those with p > t.
__device__ __forceinline__ void mass_ge(const float* p, int n, uint32_t tb, float* red, float* ge, float* gt) {
  float a = 0.0f, b = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = p[i];
    const uint32_t vb = __float_as_uint(v);
    if (v >= 0.0f && vb >= tb) a += v;
    if (v >= 0.0f && vb > tb) b += v;
  }
  *ge = block_sum_f(a, red);
  *gt = block_sum_f(b, red);
}

// Largest threshold bit pattern t with mass(p >= t) >= want (0 if none).
__device__ __forceinline__ uint32_t bisect_mass(const float* p, int n, float want, float* red) {
  uint32_t lo = 0u, hi = 0x7F800001u;  // mass(>= lo) >= want holds at lo = 0; never at hi (above +inf)
  while (hi - lo > 1u) {
    const uint32_t mid = lo + (hi - lo) / 2u;
    float ge, gt;
    mass_ge(p, n, mid, red, &ge, &gt);
    if (ge >= want) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Index of the j-th (1-based) candidate whose p has bit pattern tb, in index order.
__device__ __forceinline__ int nth_tie(const float* p, int n, uint32_t tb, int j, int* redi) {
  __shared__ int s_found;
  if (threadIdx.x == 0) s_found = -1;
  int seen = 0;  // ties before this chunk
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool tie = i < n && p[i] >= 0.0f && __float_as_uint(p[i]) == tb;
    // rank of this tie within the chunk
    const unsigned bal = __ballot_sync(B2Q_FULL, tie);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) redi[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      if (w < warp) before += redi[w];
      total += redi[w];
    }
    before += __popc(bal & ((1u << lane) - 1u));
    if (tie && seen + before + 1 == j) s_found = i;
    seen += total;
    __syncthreads();
    if (s_found >= 0) break;
  }
  __syncthreads();
  return s_found;
}

// out[0] = token, out[1] = 1 if the random number was used.  scratch: [n] floats.
__global__ void __launch_bounds__(kSampleThreads) sample_top_p_kernel(const float* __restrict__ logits, int n,
                                                                       float temperature, float top_p,
                                                                       float u, float* __restrict__ p,
                                                                       uint32_t* __restrict__ out) {
  __shared__ float red[32];
  __shared__ int redi[32];
  // max logit (NaN never wins a strict '>')
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (logits[i] > mx) mx = logits[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(B2Q_FULL, mx, o);
    if (m2 > mx) mx = m2;
  }
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(B2Q_FULL, mx, o);
      if (m2 > mx) mx = m2;
    }
  }
  const float inv_temp = 1.0f / temperature;
  const float cutoff = mx - 14.0f * temperature;
  float s = 0.0f;
  int cnt = 0, first = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = logits[i];
    float w = -1.0f;  // not a candidate
    if (v >= cutoff) {
      w = expf((v - mx) * inv_temp);
      s += w;
      ++cnt;
      first = min(first, i);
    }
    p[i] = w;
  }
  __syncthreads();
  const float sum = block_sum_f(s, red);
  cnt = block_sum_i(cnt, redi);
  if (cnt == 0 || sum <= 0.0f) {  // as the reference: token 0, no draw
    if (threadIdx.x == 0) { out[0] = 0u; out[1] = 0u; }
    return;
  }
  if (!(sum == sum)) {  // NaN weights (all logits -inf): the reference draws and returns its first candidate
    first = __reduce_min_sync(B2Q_FULL, first);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) redi[warp] = first;
    __syncthreads();
    if (threadIdx.x == 0) {
      int f = 0x7fffffff;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) f = min(f, redi[w]);
      out[0] = (uint32_t)f;
      out[1] = 1u;
    }
    return;
  }
  // the kept prefix: every p > t_keep, and the first j_keep candidates with p == t_keep
  const float target = sum * top_p;
  // a mass of 0 (top_p 0, or u 0 below) still selects the first candidate
  const uint32_t tk = bisect_mass(p, n, fmaxf(target, FLT_MIN), red);
  float ge, gt;
  mass_ge(p, n, tk, red, &ge, &gt);
  const float tkv = __uint_as_float(tk);
  int j_keep = tkv > 0.0f ? (int)ceilf((target - gt) / tkv) : 1;
  if (j_keep < 1) j_keep = 1;
  const float cum = gt + (float)j_keep * tkv;
  const float r = u * fminf(cum, sum);
  // the element r falls on, walking the prefix in descending p
  uint32_t tr = bisect_mass(p, n, fmaxf(r, FLT_MIN), red);
  if (tr < tk) tr = tk;  // never past the kept prefix
  float ge2, gt2;
  mass_ge(p, n, tr, red, &ge2, &gt2);
  const float trv = __uint_as_float(tr);
  int j = trv > 0.0f ? (int)ceilf((r - gt2) / trv) : 1;
  if (j < 1) j = 1;
  if (tr == tk && j > j_keep) j = j_keep;
  int tok = nth_tie(p, n, tr, j, redi);
  if (tok < 0) tok = nth_tie(p, n, tr, 1, redi);  // rounding left j past the ties: the first of them
  if (threadIdx.x == 0) {
    out[0] = (uint32_t)(tok < 0 ? 0 : tok);
    out[1] = 1u;
  }
}

}  // namespace b2q
