// common.cuh -- device helpers shared by the sm_100a kernels of libb2q.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B2Q_FULL 0xffffffffu

// Device error word: set by a kernel whose bounded wait gave up
// (B2Q_ETIMEOUT = 5), or by the persistent decode kernel when its shared
// memory is not laid out as planned (B2Q_ECUDA = 3).  Read and cleared by
// b2q_check_device_error() and by the blocking forward entry points.
// libb2q is a single translation unit (b2q_api.cu includes the rest).
__device__ int g_b2q_device_error = 0;

// Debug-bounds build (compiled with -DB2Q_CHECKS; build.py --checks makes
// libb2q_checks.so): index and layout checks in front of the accesses that
// a wrong plan, layout or argument could send astray -- ring offsets, staged
// input sizes, attention tile rows, tagged-vector and partial-sum indices,
// tensor-core stage offsets, GEMV row groups.  A failed check
// records its site (the first one wins) in g_b2q_check_site, sets the device
// error word to B2Q_ECUDA (3) and skips the access it guards; the host reads
// the site with b2q_debug_check_site().  Without the flag every check is the
// constant true and compiles away.
enum CheckSite : int {
  kChkRing = 1,       // a ring stage lies inside the ring
  kChkAttnRows = 2,   // an attention tile's first cache row
  kChkAttnTok = 3,    // the current token's row inside its tile
  kChkStage = 4,      // a phase input fits the staging region
  kChkTag = 5,        // a tagged-vector index
  kChkTpSlot = 6,     // a tensor-parallel partial-sum slot
  kChkPart = 7,       // an attention partial index
  kChkTcStage = 8,    // a tensor-core pipeline stage
  kChkGemv = 9,       // a standalone GEMV's row groups and shared-memory plan
};
__device__ int g_b2q_check_site = 0;
#ifdef B2Q_CHECKS
constexpr bool kChecks = true;
__device__ __noinline__ void b2q_check_fail(int site) {
  atomicCAS(&g_b2q_check_site, 0, site);
  atomicExch(&g_b2q_device_error, 3);
}
__device__ __forceinline__ bool b2q_check(bool ok, int site) {
  if (!ok) b2q_check_fail(site);
  return ok;
}
#else
constexpr bool kChecks = false;
__device__ __forceinline__ constexpr bool b2q_check(bool, int) { return true; }
#endif

// Bytes of dynamic shared memory this CTA was launched with.
__device__ __forceinline__ uint32_t dyn_smem_bytes() {
  uint32_t v;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}

// Upper bound for any spin (an mbarrier, a grid or all-rank barrier, a
// tagged hand-off), in SM clock cycles: 4e9 (~2 s at 1.965 GHz) unless the
// host lowers it with b2q_set_wait_limit_cycles().  Read only on the slow
// path of a wait, so the common case costs no load.
constexpr long long kSpinLimitCycles = 4000000000ll;
__device__ long long g_b2q_wait_limit = kSpinLimitCycles;

__device__ __forceinline__ long long wait_limit() { return *(volatile long long*)&g_b2q_wait_limit; }

// ---------------------------------------------------------------------------
// Global loads.  Weights are read once per token and never reused by the
// same kernel: non-coherent, no L1 allocation, evict-first in L2 so that the
// small activations and the KV cache keep their L2 residency.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t make_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint4 ldg_stream128(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ldg_stream32(const void* p, uint64_t pol) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ldg_stream16(const void* p, uint64_t pol) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;"
               : "=h"(r)
               : "l"(p), "l"(pol));
  return r;
}

// ---------------------------------------------------------------------------
// Integer dot products.  dp2a: two signed 16-bit activations times two bytes
// of the weight word (low or high half), accumulated in s32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int dp2a_lo_ss(int a, int b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_ss(int a, int b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// unsigned weight bytes (0..255)
__device__ __forceinline__ int dp2a_lo_su(int a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_su(int a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---------------------------------------------------------------------------
// f16 -> f32.  The bit construction of the reference's f16_to_f32
// (inference.rs:868-890), written with integer ops so that inf/NaN keep
// their payload exactly; used where bit-exactness is the contract.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float f16_bits_exact(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      // normalise: shift the leading one of the 10-bit mantissa to bit 10
      int lz = __clz(man) - 21;  // leading zeros within the 11-bit field
      uint32_t ee = 113u - (uint32_t)lz;
      bits = sign | (ee << 23) | (((man << lz) & 0x3ffu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (man << 13);
  }
  return __uint_as_float(bits);
}

// Hardware conversion: exact for every finite f16 (including subnormals).
__device__ __forceinline__ float f16_bits_fast(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

// ---------------------------------------------------------------------------
// mbarrier, 1-D bulk async copies and 2-D tiled tensor copies (TMA engine, no
// multicast).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and raises the device error word) if the
// phase did not complete within the wait limit (g_b2q_wait_limit cycles).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case: no clock reads
  const long long t0 = clock64(), lim = wait_limit();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > lim) {
      atomicExch(&g_b2q_device_error, 5);
      return false;
    }
  }
  return true;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Tiled 2-D TMA copy of the box at element coordinates (x, y) of the tensor
// map at `tmap` (global memory) into shared memory at dst; completes on `bar`.
// x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: wait for the producer grid's memory, and
// let the next grid start its prologue early.  No-ops without the launch
// attribute.  Every kernel launched with the attribute calls pdl_wait()
// before it touches memory an earlier kernel writes, so a kernel may fire
// pdl_launch_dependents() as early as it likes: the kernels here fire it
// right after their own wait (the GEMV at its start), and the next grid's
// CTAs take SMs, and its weight streams start, while this grid still runs.
// griddepcontrol.wait returns only once the whole producer grid has
// completed and its memory is visible.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(B2Q_FULL, v, o);
  return v;
}
// Sums of a and b over the warp with two halves of one reduction tree:
// lane 0 returns the sum of a, lane 16 the sum of b, each with the bits of
// warp_sum (the same additions in the same order), in 5 shuffles for both.
__device__ __forceinline__ float warp_sum2(float a, float b, int lane) {
  const bool lo = lane < 16;
  float v = (lo ? a : b) + __shfl_xor_sync(B2Q_FULL, lo ? b : a, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(B2Q_FULL, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(B2Q_FULL, v, o));
  return v;
}
