// gemm_tc.cuh -- multi-token matmul (prompt prefill) on the 5th-generation
// tensor cores: Y[t][r] = sum_k W[r][k] * X[t][k] for many tokens t.
//
// The batched path of MmapWeight::matmul_batched (src/inference.rs:589-760,
// m > 1) and of the prompt pass of StandardNativeEngine::forward.  With
// hundreds of tokens per weight row the work is tensor-core bound, not
// HBM-bound, so the weights are dequantised once per CTA tile into f16 in
// shared memory and multiplied by tcgen05.mma with the accumulator in TMEM.
//
// Per CTA: 128 weight rows (the UMMA M) x N tokens (the UMMA N, a multiple
// of 16, <= 256) x a range of k-stages of 64 elements (split-K over
// gridDim.z).  Warp roles:
//   warps 0-15  dequantise the weight tile of each stage: thread (row r,
//               quarter q) reads its bytes straight from the GEMV tile layout
//               (quant.cuh), computes the f32 value bit-exactly as
//               dequantize_slice does and rounds it to f16, and writes the
//               no-swizzle K-major core-matrix layout UMMA reads;
//   warp 16     streams the activation stage (pre-arranged in global memory
//               in the same layout, f16) with one 1-D bulk copy per stage;
//   warp 17     allocates TMEM and issues the MMAs (one thread), committing
//               each stage back to its producers;
//   warps 0-3   after the last stage, read the accumulator out of TMEM
//               (tcgen05.ld, one weight row per thread) and store f32 partial
//               sums [split][token][row] for tc_reduce_kernel.
// Precision: every f32 operand v is carried as two f16 values, hi = f16(v)
// and lo = f16(v - hi), and each k16 slice is three MMAs, hi*hi + lo*hi +
// hi*lo (the lo*lo term, ~2^-22 relative, is dropped): the products are
// those of f32 operands to ~2^-21, so the matmul holds the decode path's
// fp64 tolerance where single f16 operands (2^-11 per weight and per
// activation) do not.  Activations are scaled per token by a power of two
// so that the largest |x| of the token lies in [2^13, 2^14): no overflow,
// no subnormal hi parts (the scale is undone exactly in the reduce).  Weight
// values are the f32 of dequantize_slice before the split.  All waits are
// bounded; on a timeout the kernel records an error, drains the work it
// issued and frees its TMEM.
#pragma once

#include "gemv.cuh"

namespace b2q {

constexpr int kTcM = 128;          // weight rows per tile (UMMA M)
constexpr int kTcK = 64;           // k per pipeline stage
constexpr int kTcStagesMax = 4;
constexpr int kTcNMax = 256;       // tokens per tile (UMMA N)
constexpr int kTcDequantWarps = 16;  // 512 threads: (tile row, quarter) -> 16 weights per stage
constexpr int kTcThreads = (kTcDequantWarps + 2) * 32;
constexpr int kTcABytes = kTcM * kTcK * 2;  // one f16 image of the weight tile: 16 KB
constexpr int kTcMinTokens = 16;   // below this the GEMV path is used
constexpr int kTcSmemBudget = 200 * 1024;
constexpr int kTcPrefetch = 3;     // stages of raw weight bytes loaded ahead (registers)

// Bytes of the activation stage (hi and lo images of N tokens x 64 k).
__host__ __device__ inline int tc_b_bytes(int N) { return 2 * N * kTcK * 2; }
__host__ __device__ inline int tc_stage_bytes(int N) { return 2 * kTcABytes + tc_b_bytes(N); }
__host__ __device__ inline int tc_stages(int N) {
  const int s = kTcSmemBudget / tc_stage_bytes(N);
  return s < kTcStagesMax ? s : kTcStagesMax;
}
__host__ __device__ inline int tc_tmem_cols(int N) {
  int c = 32;
  while (c < N) c <<= 1;
  return c;
}

// Offset (in f16 elements) of element (row, kk) of a stage image with `rows`
// rows (a multiple of 8) and 64 k: [k16 slice][8-row group][8-k chunk][row][8].
__host__ __device__ inline int tc_img_off(int row, int kk, int rows) {
  return (((kk >> 4) * (rows >> 3) + (row >> 3)) * 2 + ((kk >> 3) & 1)) * 64 + (row & 7) * 8 + (kk & 7);
}

// UMMA shared-memory descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored contiguously; `lbo` = bytes between the two 8-k
// halves of a k16 slice, `sbo` = bytes between 8-row groups; version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of tcgen05.mma.kind::f16: D f32, A and B f16,
// both K-major, M = 128, N tokens.
__host__ __device__ inline uint32_t umma_idesc_f16(int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
}

constexpr int kTcMaxSegs = 3;

// Up to kTcMaxSegs weights with the same k (q, k, v) in one launch: segment
// i owns row tiles [rt[i], rt[i+1]) of gridDim.x and columns [c0[i], c0[i] +
// n of weight i) of the partial sums.
struct TcArgs {
  WeightDev w[kTcMaxSegs];
  int rt[kTcMaxSegs + 1];
  int c0[kTcMaxSegs];
  int nseg;
  const __half* xh;    // activation images [token tile][k-stage][N * 64]
  int KS;              // k-stages of the whole row (kpad / 64)
  int N;               // tokens per tile (multiple of 16, <= 256)
  int m;               // valid tokens
  int ncol;            // columns of the partial sums (all segments)
  int splits;          // split-K factor (gridDim.z)
  float* part;         // [split][mpad][ncol] partial sums (scaled activations)
  int mpad;            // token tiles * N
  int stages;          // pipeline depth (<= kTcStagesMax)
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint4 ldg_nc128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_nc32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// hi = f16(v), lo = f16(v - hi) of two values, as packed f16 pairs.
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 f = __half22float2(h);
  const __half2 l = __floats2half2_rn(a - f.x, b - f.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Write 8 values (k = kk..kk+7 of image row `row`, `rows` rows) as hi and lo
// f16 into the two images of a stage (lo image `lo_off` bytes after hi).
__device__ __forceinline__ void st_img8(uint8_t* img, int lo_off, int row, int kk, int rows, const float (&v)[8]) {
  uint4 h, l;
  split_h2(v[0], v[1], h.x, l.x);
  split_h2(v[2], v[3], h.y, l.y);
  split_h2(v[4], v[5], h.z, l.z);
  split_h2(v[6], v[7], h.w, l.w);
  uint8_t* p = img + 2 * tc_img_off(row, kk, rows);
  *reinterpret_cast<uint4*>(p) = h;
  *reinterpret_cast<uint4*>(p + lo_off) = l;
}

__device__ __forceinline__ void zero_img8(uint8_t* img, int lo_off, int row, int kk) {
  uint8_t* p = img + 2 * tc_img_off(row, kk, kTcM);
  *reinterpret_cast<uint4*>(p) = make_uint4(0, 0, 0, 0);
  *reinterpret_cast<uint4*>(p + lo_off) = make_uint4(0, 0, 0, 0);
}

// Raw bytes of one thread's 16 weights of a stage, loaded ahead of use.
// Thread (tile row r, quarter qq): half hf = qq >> 1 of the unit pair or
// plane pair, and bytes 8*(qq & 1) .. +7 of each 16-byte plane it reads.
struct TcRaw {
  uint2 a, b, c;   // Q4_K / Q5_K: qs bytes, header words 0-1, 2-3; Q6_K: ql lo, ql hi, qh;
                   // Q8_0: codes 0-15 part, 16-31 part; Q4_0: qs bytes
  uint32_t s, d;   // Q6_K: sub-scale word, d word; Q8_0 / Q4_0: d word; Q5_K: fifth-bit words
  bool live;
};

// Unit of tile row r's half `hf` in stage ks (Q4_K / Q6_K: 64-weight
// units, Q8_0: 32-weight blocks).
__device__ __forceinline__ int tc_unit(int dt, int ks, int hf) {
  if (dt == kQ8_0 || dt == kQ4_0) return 2 * ks + hf;
  if (dt == kQ6_K) return 4 * (ks >> 2) + 2 * ((ks & 3) >> 1) + hf;
  return ks;
}

__device__ __forceinline__ uint2 ldg_nc64(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

template <int DT>
__device__ __forceinline__ TcRaw tc_load(const WeightDev& w, int64_t R, int qq, int ks) {
  const TileLayout& L = w.L;
  constexpr int dt = DT;
  const int hf = qq >> 1, e8 = 8 * (qq & 1);
  const int u = tc_unit(dt, ks, hf);
  TcRaw x;
  x.live = R < (int64_t)L.G * 8 && u < L.U;
  if (!x.live) return x;
  const int c = u / L.KC, ul = u - c * L.KC;
  const uint8_t* rc = w.base + (((R >> 3) * L.C + c) * 8 + (R & 7)) * (int64_t)L.rc;
  if (dt == kQ4_K || dt == kQ5_K) {
    x.a = ldg_nc64(rc + 16 * (hf * L.KC + ul) + e8);
    const uint4 hb = ldg_nc128(rc + (dt == kQ5_K ? L.o_aux2 : L.o_aux) + 16 * (ul >> 2));
    x.b = make_uint2(hb.x, hb.y);
    x.c = make_uint2(hb.z, hb.w);
    if (dt == kQ5_K) {
      const uint2 m = ldg_nc64(rc + L.o_aux + 8 * ul);
      x.s = m.x;
      x.d = m.y;
    }
  } else if (dt == kQ4_0) {
    x.a = ldg_nc64(rc + 16 * ul + e8);
    x.d = ldg_nc32(rc + L.o_aux + 4 * (ul >> 1));
  } else if (dt == kQ6_K) {
    x.a = ldg_nc64(rc + 16 * ul + e8);
    x.b = ldg_nc64(rc + 16 * (L.KC + ul) + e8);
    x.c = ldg_nc64(rc + 16 * (2 * L.KC + ul) + e8);
    x.s = ldg_nc32(rc + L.o_aux + 4 * ul);
    x.d = ldg_nc32(rc + L.o_aux2 + 4 * (ul >> 3));
  } else {
    x.a = ldg_nc64(rc + 16 * ul + e8);
    x.b = ldg_nc64(rc + 16 * (L.KC + ul) + e8);
    x.d = ldg_nc32(rc + L.o_aux + 4 * (ul >> 1));
  }
  return x;
}

// Exact float of a small non-negative integer held in the low bits of
// `bits` (< 2^23): 2^23 + q is built by OR-ing q into the exponent pattern
// of 2^23, then 2^23 is subtracted (full-rate ALU + FADD, no I2F).
__device__ __forceinline__ float small_uint_f(uint32_t bits) {
  return __uint_as_float(0x4B000000u | bits) - 8388608.0f;
}

// Dequantise one thread's 16 weights of stage `ks` (tile row r, quarter qq)
// from its raw bytes into the A images (hi at img, lo at img + kTcABytes):
// two runs of 8 consecutive k.  The block formats of dequantize_slice
// (inference.rs:1367-1458); each value is d*sc*q - dmin*m with the products
// d*sc, dmin*m in f32 as the reference forms them and the last step fused
// (one rounding), which the hi/lo split then carries to ~2^-22.  Integer
// fields become floats by exponent-pattern arithmetic (small_uint_f), the
// f16 scales by the hardware conversion (exact for finite values).
template <int DT>
__device__ __forceinline__ void tc_convert(const TcRaw& x, int r, int qq, int ks, uint8_t* img) {
  constexpr int dt = DT;
  const int hf = qq >> 1, e8 = 8 * (qq & 1);
  const int u = tc_unit(dt, ks, hf);
  // k offsets (within the stage) of the two 8-element outputs
  int k0, k1;
  if (dt == kQ8_0 || dt == kQ4_0) { k0 = 32 * hf + e8; k1 = 32 * hf + 16 + e8; }
  else { k0 = 16 * hf + e8; k1 = 32 + 16 * hf + e8; }
  if (!x.live) {
    zero_img8(img, kTcABytes, r, k0);
    zero_img8(img, kTcABytes, r, k1);
    return;
  }
  float v0[8], v1[8];
  if (dt == kQ4_K || dt == kQ5_K) {
    const uint4 hb = make_uint4(x.b.x, x.b.y, x.c.x, x.c.y);
    const uint32_t sel = u & 3;  // KC is a multiple of 8: u & 3 == ul & 3
    const uint32_t h = sel == 0 ? hb.x : sel == 1 ? hb.y : sel == 2 ? hb.z : hb.w;
    const uint32_t dd = __byte_perm(__byte_perm(hb.x, hb.y, 0x0073), __byte_perm(hb.z, hb.w, 0x0073), 0x5410);
    const float d = f16_bits_fast(dd & 0xffffu), dmin = f16_bits_fast(dd >> 16);
    const float d1 = d * small_uint_f(h & 63u), m1 = dmin * small_uint_f((h >> 12) & 63u);
    const float d2 = d * small_uint_f((h >> 6) & 63u), m2 = dmin * small_uint_f((h >> 18) & 63u);
    const uint32_t wd[2] = {x.a.x, x.a.y};
    const bool q5 = dt == kQ5_K;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = wd[i >> 2] >> (8 * (i & 3));
      // Q5_K: fifth bit of element l of each sub-block at bit 8*(l & 3) + (l >> 2)
      const int l = 16 * hf + e8 + i;
      const uint32_t sh = 8 * (l & 3) + (l >> 2);
      const uint32_t b5a = q5 ? ((x.s >> sh) & 1u) << 4 : 0u, b5b = q5 ? ((x.d >> sh) & 1u) << 4 : 0u;
      v0[i] = fmaf(d1, small_uint_f((b & 15u) | b5a), -m1);
      v1[i] = fmaf(d2, small_uint_f(((b >> 4) & 15u) | b5b), -m2);
    }
  } else if (dt == kQ6_K) {
    // u & 7 == ul & 7 (KC a multiple of 8): the d of block ul >> 2 is half (ul >> 2) & 1 of the word
    const float d = f16_bits_fast(((u >> 2) & 1) ? x.d >> 16 : x.d & 0xffffu);
    const int hi = (ks & 1);  // groups 2,3 (high nibbles) or 0,1 (low nibbles)
    const float s0 = d * (small_uint_f(((x.s >> (8 * (2 * hi))) & 0xffu) ^ 0x80u) - 128.0f);
    const float s1 = d * (small_uint_f(((x.s >> (8 * (2 * hi + 1))) & 0xffu) ^ 0x80u) - 128.0f);
    const uint32_t wa[2] = {x.a.x, x.a.y}, wb[2] = {x.b.x, x.b.y}, wh[2] = {x.c.x, x.c.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sh = 8 * (i & 3);
      const uint32_t a = (wa[i >> 2] >> sh) & 0xffu, b = (wb[i >> 2] >> sh) & 0xffu;
      const uint32_t hh = (wh[i >> 2] >> sh) & 0xffu;
      uint32_t q0, q1;  // unsigned codes 0..63; the -32 offset is exact in f32
      if (hi) {
        q0 = (a >> 4) | (((hh >> 4) & 3u) << 4);
        q1 = (b >> 4) | (((hh >> 6) & 3u) << 4);
      } else {
        q0 = (a & 15u) | ((hh & 3u) << 4);
        q1 = (b & 15u) | (((hh >> 2) & 3u) << 4);
      }
      v0[i] = s0 * (small_uint_f(q0) - 32.0f);
      v1[i] = s1 * (small_uint_f(q1) - 32.0f);
    }
  } else if (dt == kQ4_0) {  // u & 1 == ul & 1 (KC even)
    const float d = f16_bits_fast((u & 1) ? x.d >> 16 : x.d & 0xffffu);
    const uint32_t wd[2] = {x.a.x, x.a.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = wd[i >> 2] >> (8 * (i & 3));
      v0[i] = d * (small_uint_f(b & 15u) - 8.0f);
      v1[i] = d * (small_uint_f((b >> 4) & 15u) - 8.0f);
    }
  } else {  // Q8_0: u & 1 == ul & 1 (KC even)
    const float d = f16_bits_fast((u & 1) ? x.d >> 16 : x.d & 0xffffu);
    const uint32_t wa[2] = {x.a.x, x.a.y}, wb[2] = {x.b.x, x.b.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sh = 8 * (i & 3);
      // int8 code c: (c ^ 0x80) = c + 128 as an unsigned byte
      v0[i] = d * (small_uint_f(((wa[i >> 2] >> sh) & 0xffu) ^ 0x80u) - 128.0f);
      v1[i] = d * (small_uint_f(((wb[i >> 2] >> sh) & 0xffu) ^ 0x80u) - 128.0f);
    }
  }
  st_img8(img, kTcABytes, r, k0, kTcM, v0);
  st_img8(img, kTcABytes, r, k1, kTcM, v1);
}

// The dequantising warps' loop: raw bytes of the next kTcPrefetch stages are
// in flight in registers while the current one is converted.
template <int DT>
__device__ __forceinline__ void tc_produce(const WeightDev& w, int row0, int ks0, int nst, int S, uint8_t* As,
                                           uint64_t* empty, uint64_t* a_full, volatile int* s_ok) {
  const int d = threadIdx.x, lane = threadIdx.x & 31;
  // a warp takes eight tile rows and all four quarters of each, so its raw
  // loads cover eight rows with whole 32-byte sectors; lanes 8q..8q+7 take
  // quarter q of the eight rows, so each 8-lane phase of an image store
  // writes one 128-byte core matrix (eight rows, distinct banks)
  const int qq = (d >> 3) & 3, r = ((d >> 5) << 3) | (d & 7);
  const int64_t R = (int64_t)row0 + r;
  TcRaw raw[kTcPrefetch];
#pragma unroll
  for (int j = 0; j < kTcPrefetch; ++j)
    if (j < nst) raw[j] = tc_load<DT>(w, R, qq, ks0 + j);
  for (int i0 = 0; i0 < nst; i0 += kTcPrefetch) {
#pragma unroll
    for (int j = 0; j < kTcPrefetch; ++j) {
      const int i = i0 + j;
      if (i >= nst || !*s_ok) break;
      const int s = i % S;
      if (i >= S && !mbar_wait_bounded(&empty[s], ((i / S) - 1) & 1)) {
        *s_ok = 0;
        break;
      }
      tc_convert<DT>(raw[j], r, qq, ks0 + i, As + (size_t)s * 2 * kTcABytes);
      if (i + kTcPrefetch < nst) raw[j] = tc_load<DT>(w, R, qq, ks0 + i + kTcPrefetch);
      fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
  }
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t a_full[kTcStagesMax], b_full[kTcStagesMax], empty[kTcStagesMax], done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int s_ok_;
  volatile int* s_ok = &s_ok_;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = a.N;
  const int S = a.stages;
  const int bb = tc_b_bytes(N);
  uint8_t* As = smem;                                 // per stage: hi, lo weight images
  uint8_t* Bs = smem + (size_t)S * 2 * kTcABytes;     // per stage: hi, lo activation images
  int sg = 0;
#pragma unroll
  for (int q = 1; q < kTcMaxSegs; ++q)
    if (q < a.nseg && (int)blockIdx.x >= a.rt[q]) sg = q;
  const WeightDev& W = a.w[sg];
  const int row0 = ((int)blockIdx.x - a.rt[sg]) * kTcM;
  const int tile = blockIdx.y;
  const int z = blockIdx.z;
  const int ks0 = (int)((int64_t)a.KS * z / a.splits), ks1 = (int)((int64_t)a.KS * (z + 1) / a.splits);
  const int nst = ks1 - ks0;
  const int ncols = tc_tmem_cols(N);
  if (kChecks && !b2q_check(S >= 1 && S <= kTcStagesMax && N >= 16 && N <= kTcNMax && (N & 15) == 0 &&
                                (size_t)S * tc_stage_bytes(N) <= dyn_smem_bytes() && ks0 >= 0 && ks1 <= a.KS &&
                                row0 >= 0,
                            kChkTcStage))
    return;  // (uniform over the CTA, before any barrier or TMEM allocation)

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&a_full[s], kTcDequantWarps);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done_bar, 1);
    *s_ok = 1;
    fence_mbar_init();
  }
  if (warp == kTcDequantWarps + 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp < kTcDequantWarps) {
    // ---- weight producers (one instantiation per GGML type) ----
    switch (W.L.dtype) {
      case kQ4_K: tc_produce<kQ4_K>(W, row0, ks0, nst, S, As, empty, a_full, s_ok); break;
      case kQ6_K: tc_produce<kQ6_K>(W, row0, ks0, nst, S, As, empty, a_full, s_ok); break;
      case kQ8_0: tc_produce<kQ8_0>(W, row0, ks0, nst, S, As, empty, a_full, s_ok); break;
      case kQ5_K: tc_produce<kQ5_K>(W, row0, ks0, nst, S, As, empty, a_full, s_ok); break;
      default: tc_produce<kQ4_0>(W, row0, ks0, nst, S, As, empty, a_full, s_ok); break;
    }
  } else if (warp == kTcDequantWarps) {
    // ---- activation producer ----
    if (lane == 0) {
      pdl_wait();  // the activation images come from the previous kernel
      const uint8_t* xt = reinterpret_cast<const uint8_t*>(a.xh) + (size_t)tile * a.KS * bb;
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait_bounded(&empty[s], ((i / S) - 1) & 1)) {
          *s_ok = 0;
          break;
        }
        mbar_arrive_expect_tx(&b_full[s], (uint32_t)bb);
        bulk_g2s(Bs + (size_t)s * bb, xt + (size_t)(ks0 + i) * bb, (uint32_t)bb, &b_full[s]);
        ++issued;
      }
      // copies in flight must land before the CTA may exit
      for (int i = max(0, issued - S); i < issued; ++i)
        if (!mbar_wait_bounded(&b_full[i % S], (i / S) & 1)) *s_ok = 0;
    }
  } else {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(N);
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait_bounded(&a_full[s], ph) || !mbar_wait_bounded(&b_full[s], ph)) {
          *s_ok = 0;
          break;
        }
        tc_fence_after();
        const uint32_t ahi = smem_u32(As + (size_t)s * 2 * kTcABytes), alo = ahi + kTcABytes;
        const uint32_t bhi = smem_u32(Bs + (size_t)s * bb), blo = bhi + bb / 2;
#pragma unroll
        for (int j = 0; j < kTcK / 16; ++j) {
          const uint32_t ao = j * (kTcM / 8) * 256, bo = j * (N / 8) * 256;
          // hi*hi, lo*hi, hi*lo
          const uint64_t ad[3] = {umma_desc(ahi + ao, 128, 256), umma_desc(alo + ao, 128, 256),
                                  umma_desc(ahi + ao, 128, 256)};
          const uint64_t bd[3] = {umma_desc(bhi + bo, 128, 256), umma_desc(bhi + bo, 128, 256),
                                  umma_desc(blo + bo, 128, 256)};
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            const uint32_t acc = (i > 0 || j > 0 || q > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
                "l"(ad[q]), "l"(bd[q]), "r"(idesc), "r"(acc)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
        ++issued;
      }
      // everything issued has completed once done_bar flips
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&done_bar))
                   : "memory");
      if (issued < nst) *s_ok = 0;
    }
  }

  // ---- epilogue: warps 0-3 read rows 32w..32w+31 of the accumulator ----
  if (warp < 4) {
    pdl_wait();  // the partial-sum buffer is read by an earlier kernel's reduce
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&done_bar, 0)) && *s_ok;
    tc_fence_after();
    if (ok && nst > 0) {
      const int r = warp * 32 + lane;
      const int64_t R = (int64_t)row0 + r;
      const int t0 = tile * N;
      float* outp = a.part + ((size_t)z * a.mpad) * a.ncol + a.c0[sg];
      const int64_t nrow = W.L.n;
      for (int c0 = 0; c0 < N; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
            "%13, %14, %15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15])
            : "r"(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (R < nrow) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = t0 + c0 + j;
            if (t < a.m) outp[(size_t)t * a.ncol + R] = __uint_as_float(v[j]);
          }
        }
      }
    } else if (!ok) {
      if (lane == 0) atomicExch(&g_b2q_device_error, 5);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcDequantWarps + 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// X f32 [m][ldx] (k valid columns) -> f16 stage images [token tile][k-stage]
// [hi, lo][N * 64] (zero beyond m and k) and the per-token inverse scales
// inv[t] = 2^(e-14), amax(x_t) = f * 2^e, f in [0.5, 1).  One block per token
// (padding tokens write zeros): the row is read twice, coalesced (float4 when
// the rows are 16-byte aligned), for its maximum and for the image.
__global__ void tc_act_kernel(const float* __restrict__ x, int ldx, int m, int k, int KS, int N,
                              __half* __restrict__ img, float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[32];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool live = t < m;
  const float* xr = x + (size_t)(live ? t : 0) * ldx;
  const bool v4 = ((reinterpret_cast<uintptr_t>(x) | ((size_t)ldx * 4)) & 15) == 0;
  float mx = 0.0f;
  if (live) {
    if (v4) {
      for (int i = 4 * threadIdx.x; i < k; i += 4 * blockDim.x) {
        const float4 q = *reinterpret_cast<const float4*>(xr + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
      }
    } else {
      for (int i = threadIdx.x; i < k; i += blockDim.x) mx = fmaxf(mx, fabsf(xr[i]));
    }
  }
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
  mx = warp_max(mx);
  float sc = 1.0f, iv = 1.0f;
  if (mx > 0.0f && mx <= 3.0e38f) {
    int e;
    frexpf(mx, &e);
    sc = ldexpf(1.0f, 14 - e);
    iv = ldexpf(1.0f, e - 14);
  }
  if (threadIdx.x == 0 && live) inv[t] = iv;
  const int tile = t / N, tt = t - tile * N;
  // chunks of 8 k: (stage ks, k8 index 0..7)
  for (int ch = threadIdx.x; ch < KS * 8; ch += blockDim.x) {
    const int ks = ch >> 3, kk = (ch & 7) * 8, k0 = ks * kTcK + kk;
    float v[8];
    if (live && v4 && k0 + 8 <= k) {
      const float4 a = *reinterpret_cast<const float4*>(xr + k0), b = *reinterpret_cast<const float4*>(xr + k0 + 4);
      v[0] = a.x * sc; v[1] = a.y * sc; v[2] = a.z * sc; v[3] = a.w * sc;
      v[4] = b.x * sc; v[5] = b.y * sc; v[6] = b.z * sc; v[7] = b.w * sc;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (live && k0 + e < k) ? xr[k0 + e] * sc : 0.0f;
    }
    // a NaN element contributes nothing (the quantised paths' rule, after
    // quantize_row_q8_k); the maximum above already ignores it
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] != v[e] ? 0.0f : v[e];
    uint8_t* stage = reinterpret_cast<uint8_t*>(img) + ((size_t)tile * KS + ks) * (size_t)tc_b_bytes(N);
    st_img8(stage, N * kTcK * 2, tt, kk, N, v);
  }
}

// RMSNorm of x's rows (rms_norm_rows, inference.rs:1501-1512) written
// straight into the activation images: rmsnorm_quant_kernel's f32 values
// (the same reduction order, (x * inv) * w with two roundings), then
// tc_act_kernel's per-token power-of-two scaling and hi/lo split, so the
// images hold the bits the two kernels in sequence give, without the f32 row
// going through global memory.  One block of 1024 threads per token
// (padding tokens write zeros); k floats of dynamic shared memory.
__global__ void __launch_bounds__(1024) tc_rmsnorm_act_kernel(const float* __restrict__ x, int ldx,
                                                              const float* __restrict__ w, float eps, int m, int k,
                                                              int KS, int N, __half* __restrict__ img,
                                                              float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float vrow[];
  __shared__ float part[32];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const bool live = t < m;
  const float* xr = x + (size_t)(live ? t : 0) * ldx;
  float ss = 0.0f;
  if (live)
    for (int e = threadIdx.x; e < k; e += blockDim.x) ss = fmaf(xr[e], xr[e], ss);
  ss = warp_sum(ss);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < nw ? part[lane] : 0.0f;
    v = warp_sum(v);
    if (lane == 0) part[0] = v;
  }
  __syncthreads();
  const float rinv = 1.0f / sqrtf(part[0] / (float)k + eps);
  float mx = 0.0f;  // fmaxf leaves NaN out
  for (int e = threadIdx.x; e < k; e += blockDim.x) {
    const float v = live ? __fmul_rn(__fmul_rn(xr[e], rinv), w[e]) : 0.0f;
    vrow[e] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  __syncthreads();  // part[0] read by every thread above
  if (lane == 0) part[warp] = mx;
  __syncthreads();
  mx = lane < nw ? part[lane] : 0.0f;
  mx = warp_max(mx);
  float sc = 1.0f, iv = 1.0f;
  if (mx > 0.0f && mx <= 3.0e38f) {
    int e;
    frexpf(mx, &e);
    sc = ldexpf(1.0f, 14 - e);
    iv = ldexpf(1.0f, e - 14);
  }
  if (threadIdx.x == 0 && live) inv[t] = iv;
  const int tile = t / N, tt = t - tile * N;
  for (int ch = threadIdx.x; ch < KS * 8; ch += blockDim.x) {
    const int ks = ch >> 3, kk = (ch & 7) * 8, k0 = ks * kTcK + kk;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float u = k0 + e < k ? vrow[k0 + e] * sc : 0.0f;
      v[e] = u != u ? 0.0f : u;  // a NaN element contributes nothing
    }
    uint8_t* stage = reinterpret_cast<uint8_t*>(img) + ((size_t)tile * KS + ks) * (size_t)tc_b_bytes(N);
    st_img8(stage, N * kTcK * 2, tt, kk, N, v);
  }
}

// y[t][col0 + r] = epi(inv[t] * sum_s part[s][t][r]) for t < m, r < n;
// partial rows have stride ldp.  EPI kEpiStore / kEpiAdd (y +=) /
// kEpiSwiglu (part2 = up partials: silu(g) * u).
// Grid (column blocks, m tokens): token t = blockIdx.y; each thread takes V
// consecutive columns (V = 4: 16-byte loads and stores, used when every row
// start is 16-byte aligned).  Per element the splits are added in order s =
// 0, 1, ..., as one thread per element would.
template <int EPI, int V>
__global__ void tc_reduce_kernel(const float* __restrict__ part, const float* __restrict__ part2, int splits,
                                 int mpad, int m, int n, int ldp, const float* __restrict__ inv,
                                 float* __restrict__ y, int ldy, int col0) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const float it = inv[t];
  float* yr = y + (size_t)t * ldy + col0;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) * V; r < n; r += gridDim.x * blockDim.x * V) {
    float g[V], u[V];
#pragma unroll
    for (int j = 0; j < V; ++j) g[j] = u[j] = 0.0f;
    for (int s = 0; s < splits; ++s) {
      const size_t off = ((size_t)s * mpad + t) * ldp + r;
      if (V == 4) {
        const float4 a = *reinterpret_cast<const float4*>(part + off);
        g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w;
        if (EPI == kEpiSwiglu) {
          const float4 b = *reinterpret_cast<const float4*>(part2 + off);
          u[0] += b.x; u[1] += b.y; u[2] += b.z; u[3] += b.w;
        }
      } else {
        g[0] += part[off];
        if (EPI == kEpiSwiglu) u[0] += part2[off];
      }
    }
    float o[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float gg = g[j] * it;
      if (EPI == kEpiSwiglu) o[j] = silu_f(gg) * (u[j] * it);
      else o[j] = gg;
    }
    if (V == 4) {
      float4* yp = reinterpret_cast<float4*>(yr + r);
      if (EPI == kEpiAdd) {
        const float4 prev = *yp;
        *yp = make_float4(prev.x + o[0], prev.y + o[1], prev.z + o[2], prev.w + o[3]);
      } else {
        *yp = make_float4(o[0], o[1], o[2], o[3]);
      }
    } else {
      if (EPI == kEpiAdd) yr[r] += o[0];
      else yr[r] = o[0];
    }
  }
}

}  // namespace b2q
