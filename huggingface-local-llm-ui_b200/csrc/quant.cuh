// quant.cuh -- activation quantisation, bit-exact dequantisation and the
// load-time repack of GGUF blocks into the GEMV stream layout.
#pragma once

#include "common.cuh"

namespace b2q {

enum : int {
  kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14, kBF16 = 30
};

// Activation format consumed by the GEMV kernels.  Each f32 vector of k
// values is cut into 64-element blocks; block j is stored as 16-bit integers
// q in [-16383, 16383] with x ~= q * scale[j] (scale = max|x| / 16383; the q
// row is stored in the bank-swizzled order of xswz below), plus the sums of
// q over each 16-element quarter, s16[4j .. 4j+3], used by the formats with
// an offset (Q6_K) or a min term (Q4_K).  Rows are padded to kpad (a
// multiple of 256) with zeros.  The int16 range is limited to +-16383 so that
// every integer partial sum the GEMV forms stays inside int32 (the largest,
// Q6_K: 2 groups x 16 x 32 x 16383 x 64 < 2^31).
constexpr int kXMax = 16383;
constexpr int kXBlock = 64;

struct XQ {
  int16_t* q;     // [m][kpad]
  float* scale;   // [m][kpad/64]
  int32_t* s16;   // [m][kpad/16]
  int kpad;
};

__host__ __device__ inline int round_up_int(int a, int b) { return (a + b - 1) / b * b; }

// Shared-memory bank swizzle of the int16 activation rows.  A row is cut into
// 64-element groups (128 bytes = all 32 banks); 16-byte chunk c of group g is
// stored at chunk position c ^ f(g), f(g) = g's low three bits with bits 0
// and 1 exchanged.  Every GEMV lane pattern (Q4_K: 8 lanes read chunk c of 8
// consecutive groups; Q6_K / Q8_0: pairs of lanes share a group and read
// chunks 2 or 4 apart) then hits 8 distinct chunk positions per 8-lane phase.
__host__ __device__ inline int xswz_f(int g) { return ((g >> 1) & 1) | ((g & 1) << 1) | (g & 4); }
__host__ __device__ inline int xswz_chunk(int g, int c) { return (g << 6) | ((c ^ xswz_f(g)) << 3); }
__host__ __device__ inline int xswz(int pos) { return xswz_chunk(pos >> 6, (pos >> 3) & 7) | (pos & 7); }

// Quantise one 64-element block held two values per lane (lane i holds
// elements 64*j + i and 64*j + 32 + i of row t) and store it into `xq`.
// All 32 lanes call it.  The block maximum of |x| is a warp reduction of
// the float bit patterns (for non-negative floats the integer order is the
// float order), the quarter sums are integer reductions: single redux.sync
// instructions, exact, so every ordering gives the same bits.  A NaN
// element is left out of the maximum and quantises to 0 (the float to int
// conversion maps NaN to 0), as quantize_row_q8_k treats it
// (inference.rs:933-962: NaN never wins the |x| scan, and `NaN as i8` is 0).
__device__ __forceinline__ int xq_quant(float v, float inv) {
  return max(-kXMax, min(kXMax, __float2int_rn(v * inv)));
}

// |v| as an ordered bit pattern, NaN as 0
__device__ __forceinline__ uint32_t xq_abs_bits(float v) {
  const uint32_t b = __float_as_uint(fabsf(v));
  return b > 0x7F800000u ? 0u : b;
}

__device__ __forceinline__ void xq_store_block(float v0, float v1, int lane, int t, int j, const XQ& xq) {
  const uint32_t mbits = __reduce_max_sync(B2Q_FULL, max(xq_abs_bits(v0), xq_abs_bits(v1)));
  const float amax = __uint_as_float(mbits);
  int q0 = 0, q1 = 0;
  float scale = 0.0f;
  if (amax > 0.0f && amax <= 3.0e38f) {
    scale = amax / (float)kXMax;
    const float inv = (float)kXMax / amax;
    q0 = xq_quant(v0, inv);
    q1 = xq_quant(v1, inv);
  }
  const int kp = xq.kpad;
  int16_t* qr = xq.q + (int64_t)t * kp;
  qr[xswz(j * 64 + lane)] = (int16_t)q0;
  qr[xswz(j * 64 + 32 + lane)] = (int16_t)q1;
  const bool lo = lane < 16;
  const int s0 = __reduce_add_sync(B2Q_FULL, lo ? q0 : 0), s1 = __reduce_add_sync(B2Q_FULL, lo ? 0 : q0);
  const int s2 = __reduce_add_sync(B2Q_FULL, lo ? q1 : 0), s3 = __reduce_add_sync(B2Q_FULL, lo ? 0 : q1);
  if (lane == 0) {
    int32_t* sr = xq.s16 + (int64_t)t * (kp / 16) + 4 * j;
    *reinterpret_cast<int4*>(sr) = make_int4(s0, s1, s2, s3);
    xq.scale[(int64_t)t * (kp / 64) + j] = scale;
  }
}

// The same for up to N blocks at once (block i = j0 + i * jstride, skipped
// when >= nb; warp-uniform), so that the reductions of the blocks overlap.
template <int N>
__device__ __forceinline__ void xq_store_blocks(const float (&v0)[N], const float (&v1)[N], int lane, int t, int j0,
                                                int jstride, int nb, const XQ& xq) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (j0 + i * jstride < nb) xq_store_block(v0[i], v1[i], lane, t, j0 + i * jstride, xq);
}

// The same values with 8 lanes per block: lanes 8b..8b+7 of a warp hold
// block j (each lane one 16-byte chunk c = lane & 7, elements 8c..8c+7), so
// the block maximum and the quarter sums need only lane-local work and four
// shuffles, and each lane writes its chunk with one 16-byte store.  The
// values are those of xq_store_block (exact reductions, same scale).
// `valid`: this lane group's block exists (all lanes call it).
__device__ __forceinline__ void xq_store_chunk8(const float (&v)[8], int lane, int t, int j, bool valid,
                                                const XQ& xq) {
  uint32_t mb = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) mb = max(mb, xq_abs_bits(v[i]));
  mb = max(mb, __shfl_xor_sync(B2Q_FULL, mb, 1));
  mb = max(mb, __shfl_xor_sync(B2Q_FULL, mb, 2));
  mb = max(mb, __shfl_xor_sync(B2Q_FULL, mb, 4));
  const float amax = __uint_as_float(mb);
  const bool nz = amax > 0.0f && amax <= 3.0e38f;
  const float inv = nz ? (float)kXMax / amax : 0.0f;
  int q[8], s8 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    q[i] = nz ? xq_quant(v[i], inv) : 0;
    s8 += q[i];
  }
  const int s16 = s8 + __shfl_xor_sync(B2Q_FULL, s8, 1);
  if (!valid) return;
  const int c = lane & 7, kp = xq.kpad;
  int4 pk;
  pk.x = (q[0] & 0xffff) | (q[1] << 16);
  pk.y = (q[2] & 0xffff) | (q[3] << 16);
  pk.z = (q[4] & 0xffff) | (q[5] << 16);
  pk.w = (q[6] & 0xffff) | (q[7] << 16);
  *reinterpret_cast<int4*>(xq.q + (int64_t)t * kp + xswz_chunk(j, c)) = pk;
  if ((c & 1) == 0) xq.s16[(int64_t)t * (kp / 16) + 4 * j + (c >> 1)] = s16;
  if (c == 0) xq.scale[(int64_t)t * (kp / 64) + j] = nz ? amax / (float)kXMax : 0.0f;
}

// x [m][k] f32 -> XQ (all kpad/64 blocks of every row, zero tail).
__global__ void quantize_x_kernel(const float* __restrict__ x, int m, int k, XQ xq) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int nblk = xq.kpad / 64;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int idx = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; idx < m * nblk; idx += warps) {
    const int t = idx / nblk, j = idx % nblk;
    const int p0 = j * 64 + lane, p1 = p0 + 32;
    const float* xr = x + (size_t)t * k;
    xq_store_block(p0 < k ? xr[p0] : 0.0f, p1 < k ? xr[p1] : 0.0f, lane, t, j, xq);
  }
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
  pdl_launch_dependents();
  const int t = blockIdx.y;
  uint32_t tok = tokens[t];
  if (tok >= (uint32_t)vocab) tok = 0;  // out-of-range ids are rejected on the host
  const uint8_t* row = raw + (int64_t)tok * row_bytes;
  float* out = x + (int64_t)t * k;
  const int64_t slots = dequant_slots(dtype, k);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < slots;
       s += (int64_t)gridDim.x * blockDim.x)
    dequant_slot(row, dtype, s, out);
}

// ---------------------------------------------------------------------------
// Load-time repack into the tiled GEMV layout.  All byte values are moved,
// never recomputed, so the dequantised values stay bit-exact.
//
// A row of k weights is U units (Q4_K, Q6_K: 64 weights; Q8_0: 32), cut into
// C k-chunks of KC <= 64 units (C = ceil(U / 64); KC a multiple of 8, of 16
// for Q8_0, so that a GEMV lane always sees the same activation-swizzle
// phase, see gemv.cuh).  Rows are
// grouped by 8.  Tile (g, c) = rows 8g..8g+7, chunk c, stored as 8
// consecutive row-chunks of rc bytes; tiles are ordered (g, c) row-group
// major, so one pipeline stage of the GEMV is one contiguous bulk copy.
// Row-chunk content (ul = unit index within the chunk):
//   Q4_K  [16 B x KC: qs bytes 32c'..32c'+15 of unit ul = 4*block + c']
//         [16 B x KC: qs bytes 32c'+16..32c'+31]
//         [ 4 B x KC: sc(2c') | sc(2c'+1)<<6 | m(2c')<<12 | m(2c'+1)<<18 |
//                     byte c' of (d | dmin<<16) << 24]
//   Q6_K  (unit ul = 4*block + 2*half + s covers l = 16s..16s+15 of a half)
//         [16 B x KC: ql[64h+16s..]] [16 B x KC: ql[64h+32+16s..]]
//         [16 B x KC: qh[32h+16s..]] [4 B x KC: int8 sc[8h+s+2i], i=0..3]
//         [2 B x KC/4: d per block, padded to 16 B]
//   Q8_0  [16 B x KC: codes 0..15] [16 B x KC: codes 16..31]
//         [2 B x KC: d, padded to 16 B]
//   Q5_K  as Q4_K, plus [8 B x KC: the fifth bits of the unit's two
//         sub-blocks, two words; element 4j+i of a sub-block at bit 8i+j]
//         before the header words: [16 x KC][16 x KC][8 x KC][4 x KC]
//   Q4_0  (unit = one block of 32) [16 B x KC: the 16 nibble bytes]
//         [2 B x KC: d, padded to 16 B]
// Padding units (u >= U) and rows (>= n) are zero and never read.
// ---------------------------------------------------------------------------
struct TileLayout {
  int dtype, n, k;
  int U, nb;    // units per row, GGUF blocks per row
  int KC, C;    // units per chunk, chunks per row
  int G;        // groups of 8 rows
  int rc;       // bytes per row-chunk
  int o_aux;    // offset of the per-unit scale words / d in a row-chunk
  int o_aux2;   // Q6_K: offset of the per-block d
};

__host__ __device__ inline int64_t tile_bytes(const TileLayout& L) { return 8LL * L.rc; }

__host__ inline TileLayout make_tile_layout(int dtype, int64_t n, int64_t k) {
  TileLayout L;
  L.dtype = dtype;
  L.n = (int)n;
  L.k = (int)k;
  const bool b32 = dtype == kQ8_0 || dtype == kQ4_0;  // units are whole 32-element blocks
  const int qk = b32 ? 32 : 256;
  L.nb = (int)(k / qk);
  L.U = b32 ? L.nb : (int)(k / 64);
  L.C = (L.U + 63) / 64;
  L.KC = round_up_int((L.U + L.C - 1) / L.C, b32 ? 16 : 8);
  L.G = (int)((n + 7) / 8);
  const int kc = L.KC;
  if (dtype == kQ4_K) {
    L.o_aux = 32 * kc;
    L.o_aux2 = 0;
    L.rc = 36 * kc;
  } else if (dtype == kQ6_K) {
    L.o_aux = 48 * kc;
    L.o_aux2 = 52 * kc;
    L.rc = 52 * kc + round_up_int(kc / 2, 16);
  } else if (dtype == kQ5_K) {
    L.o_aux = 32 * kc;   // fifth-bit words
    L.o_aux2 = 40 * kc;  // header words
    L.rc = 44 * kc;
  } else if (dtype == kQ4_0) {
    L.o_aux = 16 * kc;
    L.o_aux2 = 0;
    L.rc = 16 * kc + round_up_int(2 * kc, 16);
  } else {
    L.o_aux = 32 * kc;
    L.o_aux2 = 0;
    L.rc = 32 * kc + round_up_int(2 * kc, 16);
  }
  return L;
}

__device__ __forceinline__ uint8_t* tile_row_chunk(uint8_t* base, const TileLayout& L, int64_t row, int c) {
  const int64_t g = row >> 3;
  return base + ((g * L.C + c) * 8 + (row & 7)) * (int64_t)L.rc;
}

__global__ void repack_q4k_kernel(const uint8_t* __restrict__ raw, TileLayout L, uint8_t* __restrict__ out) {
  const int64_t total = (int64_t)L.n * L.U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / L.U;
    const int u = (int)(idx % L.U);
    const int c = u / L.KC, ul = u % L.KC;
    const int blk = u >> 2, cc = u & 3;
    const uint8_t* b = raw + (row * L.nb + blk) * 144;
    uint8_t* rcp = tile_row_chunk(out, L, row, c);
    const uint4* src = reinterpret_cast<const uint4*>(b + 16 + 32 * cc);
    *reinterpret_cast<uint4*>(rcp + 16 * ul) = src[0];
    *reinterpret_cast<uint4*>(rcp + 16 * (L.KC + ul)) = src[1];
    const uint8_t* s = b + 4;
    const int j0 = 2 * cc, j1 = 2 * cc + 1;
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
    *reinterpret_cast<uint32_t*>(rcp + L.o_aux + 4 * ul) =
        sc0 | (sc1 << 6) | (m0 << 12) | (m1 << 18) | (((dd >> (8 * cc)) & 0xffu) << 24);
  }
}

__global__ void repack_q6k_kernel(const uint8_t* __restrict__ raw, TileLayout L, uint8_t* __restrict__ out) {
  const int64_t total = (int64_t)L.n * L.U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / L.U;
    const int u = (int)(idx % L.U);
    const int c = u / L.KC, ul = u % L.KC;
    const int blk = u >> 2, h = (u >> 1) & 1, s = u & 1;
    const uint8_t* b = raw + (row * L.nb + blk) * 210;
    uint8_t* rcp = tile_row_chunk(out, L, row, c);
    // raw Q6_K blocks are only 2-byte aligned: copy bytewise
    const uint8_t* src0 = b + 64 * h + 16 * s;
    const uint8_t* src1 = b + 64 * h + 32 + 16 * s;
    const uint8_t* src2 = b + 128 + 32 * h + 16 * s;
    uint8_t* d0 = rcp + 16 * ul;
    uint8_t* d1 = rcp + 16 * (L.KC + ul);
    uint8_t* d2 = rcp + 16 * (2 * L.KC + ul);
#pragma unroll
    for (int i = 0; i < 16; i++) { d0[i] = src0[i]; d1[i] = src1[i]; d2[i] = src2[i]; }
    const uint8_t* sc = b + 192 + 8 * h + s;
    *reinterpret_cast<uint32_t*>(rcp + L.o_aux + 4 * ul) =
        (uint32_t)sc[0] | ((uint32_t)sc[2] << 8) | ((uint32_t)sc[4] << 16) | ((uint32_t)sc[6] << 24);
    if ((ul & 3) == 0) *reinterpret_cast<uint16_t*>(rcp + L.o_aux2 + 2 * (ul >> 2)) = (uint16_t)rd16(b + 208);
  }
}

// Q4_K / Q5_K header word of unit cc of a block (scales at b + 4, d|dmin at b).
__device__ __forceinline__ uint32_t kquant_header_word(const uint8_t* b, int cc) {
  const uint8_t* s = b + 4;
  const int j0 = 2 * cc, j1 = 2 * cc + 1;
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
  return sc0 | (sc1 << 6) | (m0 << 12) | (m1 << 18) | (((dd >> (8 * cc)) & 0xffu) << 24);
}

// Q5_K block: d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48
// (dequantize_slice, inference.rs:1418-1447).
__global__ void repack_q5k_kernel(const uint8_t* __restrict__ raw, TileLayout L, uint8_t* __restrict__ out) {
  const int64_t total = (int64_t)L.n * L.U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / L.U;
    const int u = (int)(idx % L.U);
    const int c = u / L.KC, ul = u % L.KC;
    const int blk = u >> 2, cc = u & 3;
    const uint8_t* b = raw + (row * L.nb + blk) * 176;
    uint8_t* rcp = tile_row_chunk(out, L, row, c);
    const uint8_t* qs = b + 48 + 32 * cc;
    for (int i = 0; i < 16; ++i) { rcp[16 * ul + i] = qs[i]; rcp[16 * (L.KC + ul) + i] = qs[16 + i]; }
    const uint8_t* qh = b + 16;
    uint32_t mlo = 0, mhi = 0;
    for (int l = 0; l < 32; ++l) {
      const uint32_t pos = 8 * (l & 3) + (l >> 2);
      mlo |= ((uint32_t)(qh[l] >> (2 * cc)) & 1u) << pos;
      mhi |= ((uint32_t)(qh[l] >> (2 * cc + 1)) & 1u) << pos;
    }
    *reinterpret_cast<uint2*>(rcp + L.o_aux + 8 * ul) = make_uint2(mlo, mhi);
    *reinterpret_cast<uint32_t*>(rcp + L.o_aux2 + 4 * ul) = kquant_header_word(b, cc);
  }
}

// Q4_0 block: d @0, qs[16] @2 (element i: low nibble, i + 16: high nibble)
// (dequantize_slice, inference.rs:1459-1469).
__global__ void repack_q40_kernel(const uint8_t* __restrict__ raw, TileLayout L, uint8_t* __restrict__ out) {
  const int64_t total = (int64_t)L.n * L.U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / L.U;
    const int u = (int)(idx % L.U);
    const int c = u / L.KC, ul = u % L.KC;
    const uint8_t* b = raw + (row * L.nb + u) * 18;
    uint8_t* rcp = tile_row_chunk(out, L, row, c);
    for (int i = 0; i < 16; ++i) rcp[16 * ul + i] = b[2 + i];
    *reinterpret_cast<uint16_t*>(rcp + L.o_aux + 2 * ul) = (uint16_t)rd16(b);
  }
}

__global__ void repack_q80_kernel(const uint8_t* __restrict__ raw, TileLayout L, uint8_t* __restrict__ out) {
  const int64_t total = (int64_t)L.n * L.U;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / L.U;
    const int u = (int)(idx % L.U);
    const int c = u / L.KC, ul = u % L.KC;
    const uint8_t* b = raw + (row * L.nb + u) * 34;
    uint8_t* rcp = tile_row_chunk(out, L, row, c);
    uint8_t* d0 = rcp + 16 * ul;
    uint8_t* d1 = rcp + 16 * (L.KC + ul);
#pragma unroll
    for (int i = 0; i < 16; i++) { d0[i] = b[2 + i]; d1[i] = b[18 + i]; }
    *reinterpret_cast<uint16_t*>(rcp + L.o_aux + 2 * ul) = (uint16_t)rd16(b);
  }
}

}  // namespace b2q
