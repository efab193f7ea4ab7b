// quant.cuh -- activation quantisation, bit-exact dequantisation and the
// load-time repack of GGUF blocks into the GEMV stream layout.
#pragma once

#include "common.cuh"

namespace b2q {

enum : int {
  kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14, kBF16 = 30
};

// Activation format consumed by the GEMV kernels.  Each f32 vector of k
// values is cut into 32-element blocks; block j is stored as 16-bit integers
// q in [-16383, 16383] with x ~= q * scale[j] (scale = max|x| / 16383), plus
// per-block sums used by the formats with an offset or a min term:
//   s16[2j], s16[2j+1] = sum of q over the two 16-element halves,
//   fsum[j]            = scale[j] * (s16[2j] + s16[2j+1]).
// Rows are padded to kpad (a multiple of 256) with zeros.  The int16 range is
// limited to +-16383 so that every integer partial sum the GEMV forms stays
// inside int32 (Q6_K: 4 groups x 16 x 32 x 16383 x 64 < 2^31).
constexpr int kXMax = 16383;

struct XQ {
  int16_t* q;    // [m][kpad]
  float* scale;  // [m][kpad/32]
  float* fsum;   // [m][kpad/32]
  int32_t* s16;  // [m][kpad/16]
  int kpad;
};

__host__ __device__ inline int round_up_int(int a, int b) { return (a + b - 1) / b * b; }

// One warp per 32-element block.  x [m][ldx] f32 (first k columns used).
__device__ __forceinline__ void quantize_block_warp(const float* x, int k, int t, int j, int lane,
                                                    const XQ& xq) {
  const int pos = j * 32 + lane;
  const float v = pos < k ? x[pos] : 0.0f;
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(B2Q_FULL, amax, o));
  int q = 0;
  float scale = 0.0f;
  if (amax > 0.0f && amax <= 3.0e38f) {
    scale = amax / (float)kXMax;
    const float inv = (float)kXMax / amax;
    q = __float2int_rn(v * inv);
    q = max(-kXMax, min(kXMax, q));
  }
  const int kp = xq.kpad;
  xq.q[(size_t)t * kp + pos] = (int16_t)q;
  int s = q;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(B2Q_FULL, s, o);  // within 16-lane halves
  const int s_other = __shfl_xor_sync(B2Q_FULL, s, 16);
  if (lane == 0) {
    xq.s16[(size_t)t * (kp / 16) + 2 * j] = s;
    xq.scale[(size_t)t * (kp / 32) + j] = scale;
    xq.fsum[(size_t)t * (kp / 32) + j] = scale * (float)(s + s_other);
  } else if (lane == 16) {
    xq.s16[(size_t)t * (kp / 16) + 2 * j + 1] = s;
  }
}

// x [m][k] f32 -> XQ (all kpad/32 blocks of every row, zero tail).
__global__ void quantize_x_kernel(const float* __restrict__ x, int m, int k, XQ xq) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int nblk = xq.kpad / 32;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int idx = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; idx < m * nblk; idx += warps) {
    const int t = idx / nblk, j = idx % nblk;
    quantize_block_warp(x + (size_t)t * k, k, t, j, lane, xq);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Bit-exact dequantisation of raw GGUF bytes (dequantize_slice,
// inference.rs:1347-1474).  The f32 multiply/subtract are issued with
// explicit round-to-nearest intrinsics so nvcc cannot contract them into an
// FMA, which would change the bits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t rd16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// One thread per "slot": Q4_K/Q5_K/Q6_K slot = (block, l in 0..127) writing
// 2 values; Q8_0/Q4_0 slot = (block, i in 0..31 / 0..15); F32/F16/BF16 slot
// = one element.
__device__ __forceinline__ void dequant_slot(const uint8_t* raw, int dtype, int64_t slot, float* out) {
  switch (dtype) {
    case kF32: {
      out[slot] = __uint_as_float((uint32_t)raw[4 * slot] | ((uint32_t)raw[4 * slot + 1] << 8) |
                                  ((uint32_t)raw[4 * slot + 2] << 16) |
                                  ((uint32_t)raw[4 * slot + 3] << 24));
      break;
    }
    case kF16: out[slot] = f16_bits_exact(rd16(raw + 2 * slot)); break;
    case kBF16: out[slot] = __uint_as_float(rd16(raw + 2 * slot) << 16); break;
    case kQ4_K:
    case kQ5_K: {
      const int64_t blk = slot >> 7;
      const int l = (int)(slot & 127);
      const int chunk = l >> 5, li = l & 31;
      const uint8_t* b = raw + blk * (dtype == kQ4_K ? 144 : 176);
      const float d = f16_bits_exact(rd16(b));
      const float dmin = f16_bits_exact(rd16(b + 2));
      const uint8_t* s = b + 4;
      const int j0 = 2 * chunk, j1 = 2 * chunk + 1;
      // decode_q4k_scales (inference.rs:988-1000) for the two sub-blocks
      int sc0, m0, sc1, m1;
      if (j0 < 4) {
        sc0 = s[j0] & 63; m0 = s[j0 + 4] & 63;
        sc1 = s[j1] & 63; m1 = s[j1 + 4] & 63;
      } else {
        sc0 = (s[j0 + 4] & 0x0F) | ((s[j0 - 4] >> 6) << 4);
        m0 = (s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4);
        sc1 = (s[j1 + 4] & 0x0F) | ((s[j1 - 4] >> 6) << 4);
        m1 = (s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4);
      }
      const float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
      const float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
      int v0, v1;
      if (dtype == kQ4_K) {
        const uint8_t q = b[16 + chunk * 32 + li];
        v0 = q & 0x0F; v1 = q >> 4;
      } else {
        const uint8_t q = b[48 + chunk * 32 + li];
        const uint8_t h = b[16 + li];
        v0 = (q & 0x0F) | (((h >> (2 * chunk)) & 1) << 4);
        v1 = (q >> 4) | (((h >> (2 * chunk + 1)) & 1) << 4);
      }
      float* dst = out + blk * 256 + chunk * 64;
      dst[li] = __fsub_rn(__fmul_rn(d1, (float)v0), mm1);
      dst[32 + li] = __fsub_rn(__fmul_rn(d2, (float)v1), mm2);
      break;
    }
    case kQ6_K: {
      const int64_t blk = slot >> 7;
      const int l = (int)(slot & 127);
      const int half = l >> 6, r = l & 63;  // r: 0..31 -> (q1,q3), 32..63 -> (q2,q4)
      const uint8_t* b = raw + blk * 210;
      const float d = f16_bits_exact(rd16(b + 208));
      const uint8_t* qlh = b + half * 64;
      const uint8_t* qhh = b + 128 + half * 32;
      const int8_t* sch = (const int8_t*)(b + 192 + half * 8);
      const int li = r & 31;
      const int is = li >> 4;
      float* dh = out + blk * 256 + half * 128;
      if (r < 32) {
        const int q1 = ((qlh[li] & 0x0F) | (((qhh[li] >> 0) & 3) << 4)) - 32;
        const int q3 = ((qlh[li] >> 4) | (((qhh[li] >> 4) & 3) << 4)) - 32;
        dh[li] = __fmul_rn(__fmul_rn(d, (float)sch[is]), (float)q1);
        dh[li + 64] = __fmul_rn(__fmul_rn(d, (float)sch[is + 4]), (float)q3);
      } else {
        const int q2 = ((qlh[li + 32] & 0x0F) | (((qhh[li] >> 2) & 3) << 4)) - 32;
        const int q4 = ((qlh[li + 32] >> 4) | (((qhh[li] >> 6) & 3) << 4)) - 32;
        dh[li + 32] = __fmul_rn(__fmul_rn(d, (float)sch[is + 2]), (float)q2);
        dh[li + 96] = __fmul_rn(__fmul_rn(d, (float)sch[is + 6]), (float)q4);
      }
      break;
    }
    case kQ8_0: {
      const int64_t blk = slot >> 5;
      const int i = (int)(slot & 31);
      const uint8_t* b = raw + blk * 34;
      out[slot] = __fmul_rn(f16_bits_exact(rd16(b)), (float)(int8_t)b[2 + i]);
      break;
    }
    case kQ4_0: {
      const int64_t blk = slot >> 4;
      const int i = (int)(slot & 15);
      const uint8_t* b = raw + blk * 18;
      const float d = f16_bits_exact(rd16(b));
      out[blk * 32 + i] = __fmul_rn(d, (float)((int)(b[2 + i] & 0x0F) - 8));
      out[blk * 32 + i + 16] = __fmul_rn(d, (float)((int)(b[2 + i] >> 4) - 8));
      break;
    }
    default: break;
  }
}

__host__ __device__ inline int64_t dequant_slots(int dtype, int64_t n_elems) {
  switch (dtype) {
    case kQ4_K: case kQ5_K: case kQ6_K: return n_elems / 2;
    case kQ4_0: return n_elems / 2;
    default: return n_elems;
  }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ raw, int dtype, int64_t n_elems,
                               float* __restrict__ out) {
  const int64_t slots = dequant_slots(dtype, n_elems);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < slots;
       s += (int64_t)gridDim.x * blockDim.x)
    dequant_slot(raw, dtype, s, out);
}

// Token-embedding lookup (MmapWeight::get_row_f32, inference.rs:575-582):
// dequantise row tokens[t] of a raw GGUF [vocab][k] tensor into x[t][k].
__global__ void embed_rows_kernel(const uint8_t* __restrict__ raw, int dtype, int64_t row_bytes,
                                  int k, int vocab, const uint32_t* __restrict__ tokens,
                                  float* __restrict__ x) {
  pdl_wait();
  const int t = blockIdx.y;
  uint32_t tok = tokens[t];
  if (tok >= (uint32_t)vocab) tok = 0;  // out-of-range ids are rejected on the host
  const uint8_t* row = raw + (int64_t)tok * row_bytes;
  float* out = x + (int64_t)t * k;
  const int64_t slots = dequant_slots(dtype, k);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < slots;
       s += (int64_t)gridDim.x * blockDim.x)
    dequant_slot(row, dtype, s, out);
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Load-time repack into the GEMV stream layout.  All byte values are moved,
// never recomputed, so the dequantised values stay bit-exact.
//
//   Q4_K (U = k/64 units of 64 weights per row; unit u = 4*block + chunk):
//     qs  [n][2][U][16]  half 0: qs bytes 32c..32c+15, half 1: 32c+16..32c+31
//     hdr [n][U] u32     sc(2c) | sc(2c+1)<<6 | m(2c)<<12 | m(2c+1)<<18 |
//                        byte c of (d | dmin<<16) << 24
//   Q6_K (U = k/64; unit u = 4*block + 2*half + sub, sub covers l = 16*sub..):
//     qs  [n][3][U][16]  ql[64h+16s..], ql[64h+32+16s..], qh[32h+16s..]
//     scw [n][U] u32     int8 scales sc[8h+s+2i], i = 0..3, byte i
//     d   [n][nb] u16
//   Q8_0 (U = k/32; unit = block):
//     qs  [n][2][U][16]  codes 0..15 / 16..31
//     d   [n][U] u16
// Every stream row is 16-byte aligned when k is a multiple of 32.
// ---------------------------------------------------------------------------
__global__ void repack_q4k_kernel(const uint8_t* __restrict__ raw, int64_t n, int nb,
                                  uint8_t* __restrict__ qs, uint32_t* __restrict__ hdr) {
  const int U = nb * 4;
  const int64_t total = n * U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / U;
    const int u = (int)(idx % U);
    const int blk = u >> 2, c = u & 3;
    const uint8_t* b = raw + (row * nb + blk) * 144;
    const uint4* src = reinterpret_cast<const uint4*>(b + 16 + 32 * c);
    uint4* dst0 = reinterpret_cast<uint4*>(qs + row * (int64_t)U * 32 + (int64_t)u * 16);
    uint4* dst1 = reinterpret_cast<uint4*>(qs + row * (int64_t)U * 32 + (int64_t)(U + u) * 16);
    *dst0 = src[0];
    *dst1 = src[1];
    const uint8_t* s = b + 4;
    const int j0 = 2 * c, j1 = 2 * c + 1;
    uint32_t sc0, m0, sc1, m1;
    if (j0 < 4) {
      sc0 = s[j0] & 63; m0 = s[j0 + 4] & 63; sc1 = s[j1] & 63; m1 = s[j1 + 4] & 63;
    } else {
      sc0 = (s[j0 + 4] & 0x0F) | ((s[j0 - 4] >> 6) << 4);
      m0 = (s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4);
      sc1 = (s[j1 + 4] & 0x0F) | ((s[j1 - 4] >> 6) << 4);
      m1 = (s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4);
    }
    const uint32_t dd = rd16(b) | (rd16(b + 2) << 16);
    hdr[row * U + u] = sc0 | (sc1 << 6) | (m0 << 12) | (m1 << 18) | (((dd >> (8 * c)) & 0xffu) << 24);
  }
}

__global__ void repack_q6k_kernel(const uint8_t* __restrict__ raw, int64_t n, int nb,
                                  uint8_t* __restrict__ qs, uint32_t* __restrict__ scw,
                                  uint16_t* __restrict__ dd) {
  const int U = nb * 4;
  const int64_t total = n * U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / U;
    const int u = (int)(idx % U);
    const int blk = u >> 2, h = (u >> 1) & 1, s = u & 1;
    const uint8_t* b = raw + (row * nb + blk) * 210;
    uint8_t* base = qs + row * (int64_t)U * 48;
    // raw Q6_K blocks are only 2-byte aligned: copy bytewise
    const uint8_t* src0 = b + 64 * h + 16 * s;
    const uint8_t* src1 = b + 64 * h + 32 + 16 * s;
    const uint8_t* src2 = b + 128 + 32 * h + 16 * s;
    uint8_t* d0 = base + (int64_t)u * 16;
    uint8_t* d1 = base + (int64_t)(U + u) * 16;
    uint8_t* d2 = base + (int64_t)(2 * U + u) * 16;
#pragma unroll
    for (int i = 0; i < 16; i++) { d0[i] = src0[i]; d1[i] = src1[i]; d2[i] = src2[i]; }
    const uint8_t* sc = b + 192 + 8 * h + s;
    scw[row * U + u] = (uint32_t)sc[0] | ((uint32_t)sc[2] << 8) | ((uint32_t)sc[4] << 16) |
                       ((uint32_t)sc[6] << 24);
    if ((u & 3) == 0) dd[row * nb + blk] = (uint16_t)rd16(b + 208);
  }
}

__global__ void repack_q80_kernel(const uint8_t* __restrict__ raw, int64_t n, int nb,
                                  uint8_t* __restrict__ qs, uint16_t* __restrict__ dd) {
  const int U = nb;
  const int64_t total = n * U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / U;
    const int u = (int)(idx % U);
    const uint8_t* b = raw + (row * nb + u) * 34;
    uint8_t* base = qs + row * (int64_t)U * 32;
    uint8_t* d0 = base + (int64_t)u * 16;
    uint8_t* d1 = base + (int64_t)(U + u) * 16;
#pragma unroll
    for (int i = 0; i < 16; i++) { d0[i] = b[2 + i]; d1[i] = b[18 + i]; }
    dd[row * U + u] = (uint16_t)rd16(b);
  }
}

}  // namespace b2q
