// decode.cuh -- the whole single-token decode step (StandardNativeEngine::
// forward with one token, inference.rs:2695-2860) as ONE persistent kernel.
//
// One CTA per SM, launched cooperatively (all CTAs resident).  The kernel
// keeps the GEMV kernel's warp roles for its whole life:
//  * warp 16 (producer) streams every weight tile this CTA needs for the
//    whole token -- for each layer its rows of q/k/v, attn_output, the
//    ffn_gate/ffn_up pair and ffn_down, then its rows of the output head --
//    into one shared-memory ring of variable-size stages (byte-packed, so
//    the ring holds as many bytes in flight as there is shared memory,
//    whatever the tile sizes).  Weights never depend on activations, so the
//    stream runs ahead across phase boundaries: while the consumers wait at a
//    grid barrier or compute attention, the ring fills with the next phase's
//    tiles.  Weight copies carry an L2 evict-first hint so that the small,
//    re-read data (activations, KV cache, norm weights) keeps its L2 lines.
//  * warps 0..15 (consumers) walk the phases of the Llama block, separated by
//    grid barriers where every output depends on every input:
//      stage rmsnorm(x)            -> QKV GEMV            -> barrier
//      RoPE + KV append + attention (split over the cached tokens, the last
//      split of a KV head to finish merges the partials)  -> barrier
//      stage attn                  -> O GEMV (+= x)       -> barrier
//      stage rmsnorm(x)            -> gate/up + SwiGLU    -> barrier
//      stage h                     -> down GEMV (+= x)    -> barrier
//    then the final norm, the output head and a two-level greedy argmax.
//    "stage" = each CTA normalises / quantises the whole input vector (read
//    from L2) into its own shared memory, which replaces a separate kernel
//    and a barrier.  Each CTA's view of every phase (its rows, the tile
//    layout) is loaded into shared memory once, at kernel start: under a
//    saturated HBM every dependent global load on the consumers' path costs
//    microseconds.
// Every value is computed with the same operations in the same order as the
// per-kernel path (layer.cuh, gemv.cuh), so the logits are bit-identical to
// it.  Cross-CTA data (x, qkv, attn, h, attention partials) is read with
// L2-coherent loads (ld.global.cg) after the barriers.  Every wait is bounded
// (kSpinLimitCycles); a CTA whose wait gave up raises the device error word
// and skips its remaining barrier waits, so the kernel always ends.
#pragma once

#include "gemv.cuh"
#include "layer.cuh"

namespace b2q {

constexpr int kDecSegs = 3;
enum : int { kPhQKV = 0, kPhO = 1, kPhGU = 2, kPhDown = 3, kDecPhases = 4 };
constexpr int kRingSlots = 16;  // mbarrier pairs of the byte ring (stages in flight)

// Producer view of a phase: which CTAs own which weight (segment).
struct DecSeg {
  WeightDev w;   // weight (gate for SwiGLU)
  WeightDev w2;  // up (SwiGLU only)
  int cta0, ncta;
  int nr;        // 8-row tiles per stage (1 or 2)
  int ycol;      // first output column of this segment
};

struct DecPhase {
  DecSeg seg[kDecSegs];
  int nseg;
  int pair;      // gate/up with the SwiGLU epilogue
};

struct DecLayer {
  DecPhase ph[kDecPhases];
  const float* attn_norm;
  const float* ffn_norm;
  const float* qb;  // optional q/k/v biases
  const float* kb;
  const float* vb;
  __half* kc;       // f16 KV cache [KV][max_seq][128]
  __half* vc;
};

// Consumer view of one phase for one CTA (32 bytes; table [grid][phases]).
struct CtaPhase {
  int gb, ge;     // 8-row groups [gb, ge); gb == ge: no rows in this phase
  int dtype_nr;   // GGML type | tiles per stage << 8
  int KC, C, U;   // tile layout (quant.cuh TileLayout)
  int n;          // rows of the weight
  int ycol;       // first output column
};

// Synchronisation words (zeroed at set-up; every complete launch leaves
// them consistent: the barrier count stays a multiple of the grid size and
// the arrival counters return to zero).
struct DecSync {
  unsigned long long bar;  // grid barrier arrivals (monotonic)
  unsigned int head_cnt;   // CTAs done with their argmax candidate
  unsigned int pad;
  unsigned int attn_cnt[64];  // per KV head: attention splits finished
};

struct DecodeArgs {
  const DecLayer* layers;  // [n_layers], device
  DecPhase head;
  const CtaPhase* ctab;    // [grid][nph], nph = 4 n_layers + 1
  int nph;
  int n_layers, E, H, KV, F, V;
  float eps, scale;
  int max_seq;
  const float* out_norm;
  const uint8_t* tok_raw;
  int tok_dtype;
  int64_t tok_row_bytes;
  const float* rope_cos;
  const float* rope_sin;
  const uint32_t* token;  // this step's token id (device)
  int pos;                // its position
  float* x;               // [E] residual stream
  float* qkv;             // [(H + 2 KV) * 128]
  float* attn;            // [H * 128]
  float* h;               // [F]
  float* logits;          // [V]
  float* part;            // [H][nsplit][130] attention split partials
  int nsplit;
  DecSync* sync;
  int2* cand;             // [grid] per-CTA argmax candidate (value bits, index)
  uint32_t* argmax;       // model's argmax word
  uint32_t* argmax2;      // optional caller's copy
  // shared memory: [ring cap][staging stage_bytes][accumulators racc_bytes][phase table]
  int cap;
  int stage_bytes;
  int racc_bytes;
  int tile_bytes;         // one attention tile (AttnTile<G>), 128-byte multiple
  int ngrp;               // attention items processed at once per CTA (<= 4)
};

// Row-chunk bytes and aux offsets of a tile layout (make_tile_layout).
struct RcGeom {
  int rc, o_aux, o_aux2;
};
__host__ __device__ __forceinline__ RcGeom rc_geom(int dtype, int kc) {
  RcGeom g;
  if (dtype == kQ4_K) { g.o_aux = 32 * kc; g.o_aux2 = 0; g.rc = 36 * kc; }
  else if (dtype == kQ6_K) { g.o_aux = 48 * kc; g.o_aux2 = 52 * kc; g.rc = 52 * kc + round_up_int(kc / 2, 16); }
  else { g.o_aux = 32 * kc; g.o_aux2 = 0; g.rc = 32 * kc + round_up_int(2 * kc, 16); }
  return g;
}

// ---------------------------------------------------------------------------
// Developer timeline (compiled only with -DB2Q_DECODE_TRACE): %globaltimer
// stamps of thread 0 of every CTA at each step boundary (consumers: step
// start, input staged, outputs written; producer: last stage of a phase
// issued), read back with b2q_debug_decode_trace().
// ---------------------------------------------------------------------------
#ifdef B2Q_DECODE_TRACE
constexpr int kTraceSlots = 512;
__device__ unsigned long long g_dec_trace[2 * 160 * kTraceSlots];
__device__ __forceinline__ void dec_trace(int slot, bool producer) {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (blockIdx.x < 160 && slot < kTraceSlots)
    g_dec_trace[((producer ? 160 : 0) + blockIdx.x) * kTraceSlots + slot] = t;
}
#define B2Q_TRACE(slot) do { if (threadIdx.x == 0) dec_trace((slot), false); } while (0)
#define B2Q_PTRACE(slot) dec_trace((slot), true)
__device__ int g_dec_dbg[2 * 160 * 160 * 4];
#define B2Q_DBG(prod, ph, v0, v1, v2, v3)                                                   \
  do {                                                                                     \
    if (blockIdx.x < 160 && (ph) < 160) {                                                 \
      int* d_ = g_dec_dbg + ((((prod) ? 160 : 0) + blockIdx.x) * 160 + (ph)) * 4;          \
      d_[0] = (v0); d_[1] = (v1); d_[2] = (v2); d_[3] = (v3);                              \
    }                                                                                      \
  } while (0)
#else
#define B2Q_DBG(prod, ph, v0, v1, v2, v3) do { } while (0)
#define B2Q_TRACE(slot) do { } while (0)
#define B2Q_PTRACE(slot) do { } while (0)
#endif

// ---------------------------------------------------------------------------
// synchronisation
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Barrier over the consumer warps of every CTA.  `s_ok` (shared) turns 0
// when this CTA's wait gave up; later barriers are then skipped.
__device__ __forceinline__ void grid_sync(unsigned long long* bar, volatile int* s_ok) {
  consumer_sync();
  if (threadIdx.x == 0 && *s_ok) {
    __threadfence();
    const unsigned long long n = gridDim.x;
    const unsigned long long old = atomicAdd(bar, 1ull);
    const unsigned long long target = (old / n + 1ull) * n;
    const long long t0 = clock64();
    while (ld_acquire_u64(bar) < target) {
      if (clock64() - t0 > kSpinLimitCycles) {
        atomicExch(&g_b2q_device_error, 5);
        *s_ok = 0;
        break;
      }
    }
    __threadfence();
  }
  consumer_sync();
}

// 128-thread group g (warps 4g..4g+3) of the consumers.
__device__ __forceinline__ void group_sync(int g) {
  asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory");
}

// ---------------------------------------------------------------------------
// activation staging (consumers): the quantised GEMV input in shared memory,
// in the layout gemv_kernel stages (quant.cuh XQ, one row).  Loads are
// issued in batches ahead of their use; the quantisation reductions of a
// batch are interleaved (xq_store_blocks).
// ---------------------------------------------------------------------------
constexpr int kStageBatch = 8;  // 64-element blocks per warp per batch

__device__ __forceinline__ XQ smem_xq(uint8_t* xs, int kpad) {
  XQ q;
  q.q = reinterpret_cast<int16_t*>(xs);
  q.scale = reinterpret_cast<float*>(xs + (size_t)kpad * 2);
  q.s16 = reinterpret_cast<int32_t*>(q.scale + kpad / 64);
  q.kpad = kpad;
  return q;
}

__device__ __forceinline__ SX smem_sx(const XQ& q) {
  SX s;
  s.q = q.q;
  s.scale = q.scale;
  s.s16 = q.s16;
  s.kpad = q.kpad;
  return s;
}

__host__ __device__ __forceinline__ size_t xq_smem_bytes(int kpad) { return (gemv_x_bytes(kpad, 1) + 127) / 128 * 128; }

// RMSNorm of x [dim] times w, quantised.  x is read once (into shared memory
// after the quantised row, `xs`).  The sum of squares follows the reduction
// order of rmsnorm_quant_kernel's 1024-thread CTA exactly (consumer thread i
// plays threads i and i + 512), so the values are the same bits.
__device__ __forceinline__ void stage_rmsnorm(const float* x, const float* w, int dim, float eps, const XQ& q,
                                              float* xs, float* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float sa = 0.0f, sb = 0.0f;
  for (int e0 = 0; e0 < dim; e0 += 1024 * kStageBatch) {
    float va[kStageBatch], vb[kStageBatch];
#pragma unroll
    for (int i = 0; i < kStageBatch; ++i) {
      const int ea = e0 + 1024 * i + tid, eb = ea + 512;
      va[i] = ea < dim ? __ldcg(x + ea) : 0.0f;
      vb[i] = eb < dim ? __ldcg(x + eb) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < kStageBatch; ++i) {
      const int ea = e0 + 1024 * i + tid, eb = ea + 512;
      if (ea < dim) { sa = fmaf(va[i], va[i], sa); xs[ea] = va[i]; }
      if (eb < dim) { sb = fmaf(vb[i], vb[i], sb); xs[eb] = vb[i]; }
    }
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  if (lane == 0) {
    red[warp] = sa;
    red[warp + 16] = sb;
  }
  consumer_sync();
  const float tot = warp_sum(red[lane]);
  const float inv = 1.0f / sqrtf(tot / (float)dim + eps);
  const int nb = q.kpad >> 6;
  for (int j0 = warp; j0 < nb; j0 += kGemvConsumerWarps * kStageBatch) {
    float va[kStageBatch], vb[kStageBatch];
#pragma unroll
    for (int i = 0; i < kStageBatch; ++i) {
      const int ea = (j0 + kGemvConsumerWarps * i) * 64 + lane, eb = ea + 32;
      // (x * inv) * w, two separate roundings as the reference computes it
      va[i] = ea < dim ? __fmul_rn(__fmul_rn(xs[ea], inv), w[ea]) : 0.0f;
      vb[i] = eb < dim ? __fmul_rn(__fmul_rn(xs[eb], inv), w[eb]) : 0.0f;
    }
    xq_store_blocks<kStageBatch>(va, vb, lane, 0, j0, kGemvConsumerWarps, nb, q);
  }
  consumer_sync();
}

// Plain quantisation of src [dim] (quantize_x_kernel's values).
__device__ __forceinline__ void stage_plain(const float* src, int dim, const XQ& q) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = q.kpad >> 6;
  for (int j0 = warp; j0 < nb; j0 += kGemvConsumerWarps * kStageBatch) {
    float xa[kStageBatch], xb[kStageBatch];
#pragma unroll
    for (int i = 0; i < kStageBatch; ++i) {
      const int ea = (j0 + kGemvConsumerWarps * i) * 64 + lane, eb = ea + 32;
      xa[i] = ea < dim ? __ldcg(src + ea) : 0.0f;
      xb[i] = eb < dim ? __ldcg(src + eb) : 0.0f;
    }
    xq_store_blocks<kStageBatch>(xa, xb, lane, 0, j0, kGemvConsumerWarps, nb, q);
  }
  consumer_sync();
}

// ---------------------------------------------------------------------------
// byte ring: stage j occupies [off_j, off_j + size_j) of the ring; stages
// are placed back to back and restart at offset 0 when one would not fit
// before the end.  Stage j completes on full[j % kRingSlots] (use j /
// kRingSlots) and is released on empty[j % kRingSlots].  Producer and
// consumers walk the same stage sequence, so they place every stage at the
// same offset without exchanging it.
// ---------------------------------------------------------------------------
struct ByteRing {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int cap;
};

// bulk copy with an L2 cache policy (weights: evict first)
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// producer (one thread)
// ---------------------------------------------------------------------------
struct Producer {
  ByteRing R;
  uint64_t pol;
  int j = 0;       // next stage
  int wo = 0;      // next write offset
  int oldest = 0;  // oldest stage not known to be released
  int* qs;         // [kRingSlots] start offset of the stage in each slot (shared)
  int* qe;         // [kRingSlots] end offset

  // Place a stage of `size` bytes; false if a wait gave up.  Consumers
  // release stages in order, so it suffices to wait for the newest earlier
  // stage that overlaps the new one (or that holds its barrier slot).
  __device__ __forceinline__ bool alloc(int size, int& off) {
    int o = wo;
    if (o + size > R.cap) o = 0;
    int need = j - kRingSlots;  // the previous user of this barrier slot
    for (int k = max(oldest, need + 1); k < j; ++k) {
      const int s = k & (kRingSlots - 1);
      if (o < qe[s] && qs[s] < o + size) need = k;
    }
    if (need >= oldest) {
      if (!mbar_wait_bounded(&R.empty[need & (kRingSlots - 1)], (uint32_t)((need / kRingSlots) & 1))) return false;
      oldest = need + 1;
    }
    const int s = j & (kRingSlots - 1);
    qs[s] = o;
    qe[s] = o + size;
    off = o;
    wo = o + size;
    return true;
  }

  template <int NR, bool PAIR>
  __device__ __forceinline__ bool gemv(const WeightDev& w, const WeightDev& w2, int gb, int ge) {
    const TileLayout& L = w.L;
    const uint32_t tb = (uint32_t)tile_bytes(L);
    for (StageIter<NR, PAIR> it(gb, ge, L.C); !it.done(); it.next()) {
      const int nt = it.ntiles();
      int off;
      if (!alloc((int)tb * nt, off)) return false;
      uint64_t* fb = &R.full[j & (kRingSlots - 1)];
      mbar_arrive_expect_tx(fb, tb * nt);
      uint8_t* sl = R.base + off;
      const int64_t t0 = (int64_t)it.g * L.C + it.c;
      bulk_g2s_hint(sl, w.base + t0 * tb, tb, fb, pol);
      if (PAIR) bulk_g2s_hint(sl + tb, w2.base + t0 * tb, tb, fb, pol);
      else if (nt == 2) bulk_g2s_hint(sl + tb, w.base + (t0 + L.C) * tb, tb, fb, pol);
      ++j;
    }
    return true;
  }
};

// This CTA's segment of a phase and its 8-row groups [gb, ge); false if it
// owns no rows.
__device__ __forceinline__ bool cta_range(const DecPhase& ph, int& s, int& gb, int& ge) {
  const int b = blockIdx.x;
  for (s = 0; s < ph.nseg; ++s) {
    const DecSeg& sg = ph.seg[s];
    if (b >= sg.cta0 && b < sg.cta0 + sg.ncta) {
      const int ci = b - sg.cta0;
      const int G = sg.w.L.G;
      gb = (int)((int64_t)G * ci / sg.ncta);
      ge = (int)((int64_t)G * (ci + 1) / sg.ncta);
      return gb < ge;
    }
  }
  return false;
}

__device__ __forceinline__ bool produce_phase(Producer& P, const DecPhase& ph) {
  int s, gb, ge;
  if (!cta_range(ph, s, gb, ge)) return true;
  const DecSeg& sg = ph.seg[s];
  if (ph.pair) return P.gemv<2, true>(sg.w, sg.w2, gb, ge);
  if (sg.nr == 2) return P.gemv<2, false>(sg.w, sg.w2, gb, ge);
  return P.gemv<1, false>(sg.w, sg.w2, gb, ge);
}

__device__ __noinline__ void decode_producer(const DecodeArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             int* qs, int* qe) {
  Producer P;
  P.R.base = ring;
  P.R.full = full;
  P.R.empty = empty;
  P.R.cap = a.cap;
  P.pol = make_evict_first_policy();
  P.qs = qs;
  P.qe = qe;
  for (int l = 0; l < a.n_layers; ++l) {
    const DecLayer& Ly = a.layers[l];
#pragma unroll 1
    for (int p = 0; p < kDecPhases; ++p) {
      if (!produce_phase(P, Ly.ph[p])) return;
      B2Q_PTRACE(l * kDecPhases + p);
      B2Q_DBG(true, l * kDecPhases + p, P.j, P.wo, P.oldest, 0);
    }
  }
  produce_phase(P, a.head);
  B2Q_PTRACE(a.n_layers * kDecPhases);
  B2Q_DBG(true, a.n_layers * kDecPhases, P.j, P.wo, P.oldest, 0);
}

// ---------------------------------------------------------------------------
// consumers: one GEMV phase (this CTA's rows), activations already staged.
// A single copy of the consume loop serves every phase: the SwiGLU pairing,
// the tiles per stage and the GGML type are runtime values (uniform across
// the CTA).  Per row the partials are accumulated in the same order as
// gemv_kernel's (chunk by chunk, then the two unit halves), so the outputs
// are the same bits.  racc layout: [unit half][w][rows], w = 1 for the up
// projection of the SwiGLU pair; rows = this phase's row count.
// ---------------------------------------------------------------------------
struct Consumer {
  ByteRing R;
  int j = 0;   // next stage
  int ro = 0;  // next read offset
};

__device__ __forceinline__ void consume_phase(Consumer& cs, const CtaPhase& ph, bool pair, const SX& sx, bool& ok,
                                              float* racc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = warp >> 1, hf = warp & 1;  // row p of every tile; unit half hf
  const int gb = ph.gb, ge = ph.ge;
  const int dt = ph.dtype_nr & 0xff, nr = ph.dtype_nr >> 8;
  const int KC = ph.KC, C = ph.C, U = ph.U;
  const RcGeom geo = rc_geom(dt, KC);
  const int tb = 8 * geo.rc;
  const int rows = (ge - gb) * 8;
  const int nw = pair ? 2 : 1;
  for (int i = threadIdx.x; i < 2 * nw * rows; i += kGemvConsumerWarps * 32) racc[i] = 0.0f;
  consumer_sync();
  const int step = (pair || nr == 1) ? 1 : 2;
  const bool two = pair || nr == 2;
  const XPhase xp = make_xphase(lane);
  const int ul = lane + 32 * hf;
  const int csel = lane & 3;
  float* acc = racc + hf * nw * rows + p;  // this warp's row p, half hf
  XUnit X;
  bool uok = false;
  for (int c = 0, g = gb; c < C && gb < ge;) {
    if (g == gb) {  // new chunk pass: this lane's activations
      const int u = c * KC + ul;
      uok = ul < KC && u < U;
      if (uok && ok) {
        if (dt == kQ4_K) xload_q4k(X, sx, 0, u, xp.f4);
        else if (dt == kQ6_K) xload_q6k(X, sx, 0, u, xp.f6a, xp.f6b);
        else xload_q80(X, sx, 0, u, xp.f8);
      }
    }
    const bool nt2 = two && (pair || g + 1 < ge);
    int off = cs.ro;
    const int size = nt2 ? 2 * tb : tb;
    if (off + size > cs.R.cap) off = 0;
    cs.ro = off + size;
    const int slot = cs.j & (kRingSlots - 1);
    if (ok) ok = mbar_wait_bounded(&cs.R.full[slot], (uint32_t)((cs.j / kRingSlots) & 1));
    float p0 = 0.0f, p1 = 0.0f;
    if (ok && uok) {
      const uint8_t* rc = cs.R.base + off + p * geo.rc;
      if (dt == kQ4_K) {
        p0 = row_q4k(rc, KC, geo.o_aux, ul, csel, X);
        if (nt2) p1 = row_q4k(rc + tb, KC, geo.o_aux, ul, csel, X);
      } else if (dt == kQ6_K) {
        p0 = row_q6k(rc, KC, geo.o_aux, geo.o_aux2, ul, X);
        if (nt2) p1 = row_q6k(rc + tb, KC, geo.o_aux, geo.o_aux2, ul, X);
      } else {
        p0 = row_q80(rc, KC, geo.o_aux, ul, X);
        if (nt2) p1 = row_q80(rc + tb, KC, geo.o_aux, ul, X);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&cs.R.empty[slot]);  // the stage may be refilled
    ++cs.j;
    p0 = warp_sum(p0);
    if (nt2) p1 = warp_sum(p1);
    if (lane == 0) {
      const int r = (g - gb) * 8;
      acc[r] += p0;
      if (nt2) {
        if (pair) acc[rows + r] += p1;  // up tile, same row
        else acc[r + 8] += p1;          // next 8-row group
      }
    }
    g += step;
    if (g >= ge) {
      g = gb;
      ++c;
    }
  }
  consumer_sync();
}

// Epilogue of a phase: rows [8 gb, min(8 ge, n)) of y.  Thread i handles
// rows i and i + 512 first; `xr` holds their residual (prefetched).
__device__ __forceinline__ float dec_racc(const float* racc, int rows, int nw, int r, int w) {
  return racc[w * rows + r] + racc[(nw + w) * rows + r];
}

// ---------------------------------------------------------------------------
// attention item (KV head g, split z) on a 128-thread group: the work of
// rope_kv_kernel (for this head group) + attn_split_kernel + (last split of
// head g to finish) attn_combine_kernel, with the same arithmetic.  The
// split holding `pos` takes this token's k/v from registers (and appends
// them to the cache); the other rows arrive by bulk copy.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int G>
__device__ __noinline__ void attn_item(const DecodeArgs& a, const DecLayer& Ly, int g, int z, int nz,
                                       AttnTile<G>& T, int grp, uint64_t* bar, int* uses, int* s_last) {
  constexpr int HD = kHeadDim, HALF = kHeadDim / 2;
  const int gt = threadIdx.x & 127;
  const int pos = a.pos, cap = a.max_seq;
  const int H = a.H, KV = a.KV;
  const int t_begin = z * kAttnTile;
  const int nv = min(kAttnTile, pos + 1 - t_begin);
  const bool last = z == nz - 1;
  const int nload = last ? nv - 1 : nv;
  if (gt == 0 && nload > 0) {
    fence_proxy_async_smem();  // earlier generic accesses to this region come first
    attn_tile_load(T, Ly.kc, Ly.vc, g, cap, t_begin, nload, bar);
  }
  const int p_rope = pos < 8191 ? pos : 8191;
  const float* cs = a.rope_cos + (int64_t)p_rope * HALF;
  const float* sn = a.rope_sin + (int64_t)p_rope * HALF;
  const float* row = a.qkv;
  for (int idx = gt; idx < G * HALF; idx += 128) {
    const int hh = idx / HALF, j = idx % HALF;
    const int h = g * G + hh;
    float x0 = __ldcg(row + h * HD + j), x1 = __ldcg(row + h * HD + HALF + j);
    if (Ly.qb != nullptr) { x0 += Ly.qb[h * HD + j]; x1 += Ly.qb[h * HD + HALF + j]; }
    const float c = cs[j], sv = sn[j];
    T.q[hh][j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv));
    T.q[hh][HALF + j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sv));
  }
  if (last) {  // this token's k (rotated) and v: into the tile and the cache
    const int r = nv - 1;
    for (int j = gt; j < HALF; j += 128) {
      const float* kr = row + (H + g) * HD;
      float x0 = __ldcg(kr + j), x1 = __ldcg(kr + HALF + j);
      if (Ly.kb != nullptr) { x0 += Ly.kb[g * HD + j]; x1 += Ly.kb[g * HD + HALF + j]; }
      const float c = cs[j], sv = sn[j];
      const __half y0 = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv)));
      const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sv)));
      __half* dst = Ly.kc + ((int64_t)g * cap + pos) * HD;
      dst[j] = y0;
      dst[HALF + j] = y1;
      T.k[r * HD + j] = y0;
      T.k[r * HD + HALF + j] = y1;
    }
    for (int d = gt; d < HD; d += 128) {
      float v = __ldcg(row + (H + KV) * HD + g * HD + d);
      if (Ly.vb != nullptr) v += Ly.vb[g * HD + d];
      const __half hv = __float2half_rn(v);
      Ly.vc[((int64_t)g * cap + pos) * HD + d] = hv;
      T.v[r * HD + d] = hv;
    }
  }
  if (nload > 0) {
    mbar_wait_bounded(bar, (uint32_t)(*uses & 1));  // a timeout is recorded in the device error word
    ++*uses;
  }
  group_sync(grp);
  attn_tile_compute<G>(T, nv, a.scale, a.part, g, z, a.nsplit, [grp] { group_sync(grp); });
  // the last split of this KV head to finish merges all of them
  group_sync(grp);
  if (gt == 0) {
    __threadfence();
    const unsigned int old = atomicAdd(&a.sync->attn_cnt[g], 1u);
    *s_last = old == (unsigned int)(nz - 1);
  }
  group_sync(grp);
  if (*s_last) {
    // merge (attn_combine_kernel's arithmetic): the partials of all splits
    // are staged into the idle tile with independent loads, then reduced in
    // split order from shared memory
    __threadfence();
    const int nsplit = a.nsplit;
    float* ml = reinterpret_cast<float*>(T.v);  // [G][nz] x {max, sum}
    float* ob = reinterpret_cast<float*>(T.k);  // [zc][G][HD] O chunk
    constexpr int kZc = (kAttnTile * HD / 2) / (G * HD);  // splits per O chunk (T.k as floats)
    for (int i = gt; i < G * nz; i += 128) {
      const int hh = i / nz, zz = i % nz;
      const float* pp = a.part + ((int64_t)(g * G + hh) * nsplit + zz) * (HD + 2);
      ml[2 * i] = __ldcg(pp);
      ml[2 * i + 1] = __ldcg(pp + 1);
    }
    group_sync(grp);
    float M[(G * HD + 127) / 128], Ls[(G * HD + 127) / 128], O[(G * HD + 127) / 128];
#pragma unroll
    for (int r = 0; r < (G * HD + 127) / 128; ++r) {
      const int i = gt + 128 * r, hh = i / HD;
      float mx = -INFINITY;
      if (i < G * HD)
        for (int zz = 0; zz < nz; ++zz) mx = fmaxf(mx, ml[2 * (hh * nz + zz)]);
      M[r] = mx;
      Ls[r] = 0.0f;
      O[r] = 0.0f;
    }
    for (int z0 = 0; z0 < nz; z0 += kZc) {
      const int zn = min(kZc, nz - z0);
      group_sync(grp);  // previous chunk consumed
      for (int i = gt; i < zn * G * HD; i += 128) {
        const int zz = i / (G * HD), rem = i % (G * HD), hh = rem / HD, d = rem % HD;
        ob[i] = __ldcg(a.part + ((int64_t)(g * G + hh) * nsplit + z0 + zz) * (HD + 2) + 2 + d);
      }
      group_sync(grp);
#pragma unroll
      for (int r = 0; r < (G * HD + 127) / 128; ++r) {
        const int i = gt + 128 * r, hh = i / HD, d = i % HD;
        if (i >= G * HD) continue;
        for (int zz = 0; zz < zn; ++zz) {
          const float mz = ml[2 * (hh * nz + z0 + zz)];
          const float f = mz == -INFINITY ? 0.0f : expf(mz - M[r]);
          Ls[r] = fmaf(f, ml[2 * (hh * nz + z0 + zz) + 1], Ls[r]);
          O[r] = fmaf(f, ob[(zz * G + hh) * HD + d], O[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < (G * HD + 127) / 128; ++r) {
      const int i = gt + 128 * r;
      if (i < G * HD) a.attn[(g * G + i / HD) * HD + i % HD] = O[r] * (1.0f / fmaxf(Ls[r], 1e-12f));
    }
    if (gt == 0) a.sync->attn_cnt[g] = 0u;
  }
  group_sync(grp);  // the tile and s_last are reused by the group's next item
}

// ---------------------------------------------------------------------------
// argmax helpers: first index of the maximum (strict '>' scan); NaN never
// wins; an all -inf / NaN vector gives index 0 (argmax_kernel's semantics).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void argmax_merge(float& best, int& idx, float ob, int oi) {
  if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
}

__device__ __forceinline__ void warp_argmax(float& best, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(B2Q_FULL, best, o);
    const int oi = __shfl_xor_sync(B2Q_FULL, idx, o);
    argmax_merge(best, idx, ob, oi);
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(kGemvThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full_bar[kRingSlots], empty_bar[kRingSlots];
  __shared__ int ring_qs[kRingSlots], ring_qe[kRingSlots];
  __shared__ float red[32];
  __shared__ int s_ok;
  __shared__ float s_bv[kGemvConsumerWarps];
  __shared__ int s_bi[kGemvConsumerWarps];
  __shared__ int s_last;
  __shared__ uint64_t attn_bar[4];
  __shared__ int attn_last[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // [ring][activation staging][row accumulators][phase table]; an attention
  // tile spans the staging and accumulator regions, both idle during
  // attention
  uint8_t* ring = smem;
  uint8_t* xs = smem + a.cap;
  float* racc = reinterpret_cast<float*>(xs + a.stage_bytes);
  CtaPhase* tab = reinterpret_cast<CtaPhase*>(xs + a.stage_bytes + a.racc_bytes);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRingSlots; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kGemvConsumerWarps);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&attn_bar[i], 1);
    fence_mbar_init();
    s_ok = 1;
  }
  __syncthreads();
  if (warp == kGemvConsumerWarps) {
    if (lane == 0) decode_producer(a, ring, full_bar, empty_bar, ring_qs, ring_qe);
    return;
  }

  // ---- consumers ----
  volatile int* okp = &s_ok;
  bool ok = true;
  Consumer cs;
  cs.R.base = ring;
  cs.R.full = full_bar;
  cs.R.empty = empty_bar;
  cs.R.cap = a.cap;
  unsigned long long* bar = &a.sync->bar;

  // this CTA's phase table, and the token embedding (embed_rows_kernel's
  // values) spread over the grid
  {
    const int4* src = reinterpret_cast<const int4*>(a.ctab + (size_t)blockIdx.x * a.nph);
    int4* dst = reinterpret_cast<int4*>(tab);
    for (int i = threadIdx.x; i < a.nph * 2; i += kGemvConsumerWarps * 32) dst[i] = __ldcg(src + i);
    uint32_t tok = a.token[0];
    if (tok >= (uint32_t)a.V) tok = 0;
    const uint8_t* rowp = a.tok_raw + (int64_t)tok * a.tok_row_bytes;
    const int64_t slots = dequant_slots(a.tok_dtype, a.E);
    for (int64_t sl = (int64_t)blockIdx.x * 512 + threadIdx.x; sl < slots; sl += (int64_t)gridDim.x * 512)
      dequant_slot(rowp, a.tok_dtype, sl, a.x);
  }
  grid_sync(bar, okp);

  const int nz = a.pos / kAttnTile + 1;
  const int grp = warp >> 2;
  int attn_uses = 0;  // completed phases of this group's attention mbarrier
  const int kp_e = round_up_int(a.E, 256);
  float* xcopy = reinterpret_cast<float*>(xs + xq_smem_bytes(kp_e));
  float best = -INFINITY;
  int idx = 0x7fffffff;
  // steps: per layer QKV, attention, O, gate/up, down; then the head
  for (int l = 0, k = 0; l <= a.n_layers; ++k) {
    if (k == 5) {
      k = 0;
      ++l;
      if (l > a.n_layers) break;
    }
    const bool head = l == a.n_layers;
    if (head && k > 0) break;
    const int tslot = (l * 5 + k) * 3;
    B2Q_TRACE(tslot);
    if (k == 1) {  // RoPE, KV append, attention
      const DecLayer& Ly = a.layers[l];
      if (grp < a.ngrp) {
        AttnTile<G>& T = *reinterpret_cast<AttnTile<G>*>(xs + (size_t)grp * a.tile_bytes);
        for (int it = blockIdx.x + gridDim.x * grp; it < a.KV * nz; it += gridDim.x * a.ngrp)
          attn_item<G>(a, Ly, it / nz, it % nz, nz, T, grp, &attn_bar[grp], &attn_uses, &attn_last[grp]);
      }
      B2Q_TRACE(tslot + 2);
      grid_sync(bar, okp);
      continue;
    }
    const CtaPhase& ph = tab[head ? 4 * a.n_layers : 4 * l + (k == 0 ? 0 : k - 1)];
    if (ph.gb < ph.ge) {
      const bool add = k == 2 || k == 4;
      const int row0 = ph.gb * 8, nrows = min(ph.ge * 8, ph.n) - row0;
      // residual rows of this CTA, fetched while the input is staged
      float xr0 = 0.0f, xr1 = 0.0f;
      if (add) {
        if (threadIdx.x < nrows) xr0 = __ldcg(a.x + row0 + threadIdx.x);
        if (threadIdx.x + 512 < nrows) xr1 = __ldcg(a.x + row0 + threadIdx.x + 512);
      }
      // stage the input: rmsnorm(x) for QKV, gate/up and the head; attn; h
      XQ q;
      if (k == 2) {
        q = smem_xq(xs, round_up_int(a.H * kHeadDim, 256));
        stage_plain(a.attn, a.H * kHeadDim, q);
      } else if (k == 4) {
        q = smem_xq(xs, round_up_int(a.F, 256));
        stage_plain(a.h, a.F, q);
      } else {
        q = smem_xq(xs, kp_e);
        const float* nw = head ? a.out_norm : (k == 0 ? a.layers[l].attn_norm : a.layers[l].ffn_norm);
        stage_rmsnorm(a.x, nw, a.E, a.eps, q, xcopy, red);
      }
      B2Q_TRACE(tslot + 1);
      const bool pair = k == 3;
      consume_phase(cs, ph, pair, smem_sx(q), ok, racc);
      // epilogue
      if (ok) {
        const int rows = (ph.ge - ph.gb) * 8, nw = pair ? 2 : 1;
        float* y = (head ? a.logits : k == 0 ? a.qkv : pair ? a.h : a.x) + ph.ycol + row0;
        for (int r = threadIdx.x; r < nrows; r += kGemvConsumerWarps * 32) {
          const float v = dec_racc(racc, rows, nw, r, 0);
          if (pair) y[r] = silu_f(v) * dec_racc(racc, rows, nw, r, 1);
          else if (add) y[r] = (r < 512 ? xr0 : r < 1024 ? xr1 : __ldcg(y + r)) + v;
          else y[r] = v;
          if (head && v > best) { best = v; idx = row0 + r; }
        }
      }
      B2Q_TRACE(tslot + 2);
#ifdef B2Q_DECODE_TRACE
      if (threadIdx.x == 0) {
        float cks = 0.0f;
        for (int r = 0; r < nrows; ++r) cks += dec_racc(racc, (ph.ge - ph.gb) * 8, pair ? 2 : 1, r, 0);
        B2Q_DBG(false, head ? 4 * a.n_layers : 4 * l + (k == 0 ? 0 : k - 1), cs.j, cs.ro, __float_as_int(cks),
                __float_as_int(q.scale[0]));
      }
#endif
    }
    if (!head) grid_sync(bar, okp);
  }
  warp_argmax(best, idx);
  if (lane == 0) { s_bv[warp] = best; s_bi[warp] = idx; }
  consumer_sync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kGemvConsumerWarps; ++w) argmax_merge(best, idx, s_bv[w], s_bi[w]);
    a.cand[blockIdx.x] = make_int2(__float_as_int(best), idx);
    __threadfence();
    const unsigned int old = atomicAdd(&a.sync->head_cnt, 1u);
    s_last = old == gridDim.x - 1;
  }
  consumer_sync();
  if (s_last && warp == 0) {
    __threadfence();
    best = -INFINITY;
    idx = 0x7fffffff;
    for (int c = lane; c < (int)gridDim.x; c += 32) {
      const int2 cv = __ldcg(a.cand + c);
      argmax_merge(best, idx, __int_as_float(cv.x), cv.y);
    }
    warp_argmax(best, idx);
    if (lane == 0) {
      const uint32_t r = idx == 0x7fffffff ? 0u : (uint32_t)idx;
      *a.argmax = r;
      if (a.argmax2 != nullptr) *a.argmax2 = r;
      a.sync->head_cnt = 0u;
    }
  }
}

}  // namespace b2q
