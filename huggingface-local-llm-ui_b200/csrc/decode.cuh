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
// it.  Cross-CTA data is read from L2 after the barriers: on one GPU x, q|k|v
// and the attention output as tagged 8-byte words (value and hand-off tag in
// one store, see DecodeArgs), behind relaxed barriers; h, the attention
// partials and, under tensor parallelism, everything else with L2-coherent
// loads (ld.global.cg) behind release/acquire barriers.  Every wait is bounded
// (g_b2q_wait_limit cycles); a CTA whose wait gave up raises the device error word
// and skips its remaining barrier waits, so the kernel always ends.
#pragma once

#include "gemv.cuh"
#include "layer.cuh"

namespace b2q {

constexpr int kDecSegs = 3;
enum : int { kPhQKV = 0, kPhO = 1, kPhGU = 2, kPhDown = 3, kDecPhases = 4 };
constexpr int kRingSlots = 16;  // mbarrier pairs of the byte ring (stages in flight)
constexpr int kMaxTp = 8;       // tensor-parallel ranks of one box

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
  const void* tmk;  // TMA descriptors of kc and vc (global memory)
  const void* tmv;
};

// Consumer view of one phase for one CTA (32 bytes; table [grid][phases]).
struct CtaPhase {
  int gb, ge;     // 8-row groups [gb, ge); gb == ge: no rows in this phase
  int dtype_nr;   // GGML type | tiles per stage << 8
  int KC, C, U;   // tile layout (quant.cuh TileLayout)
  int n;          // rows of the weight
  int ycol;       // first output column
};

// Synchronisation words (zeroed at set-up).
struct DecSync {
  unsigned long long bar;  // grid barrier arrivals (monotonic)
  unsigned int head_cnt;   // CTAs done with their argmax candidate
  unsigned int pad;
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
  const uint32_t* token;  // this step's token id (device), or nullptr: token_imm
  uint32_t token_imm;     // the token id by value (a host caller's token)
  int pos;                // its position
  float* part;            // [H][nsplit][kPartStride] attention split partials
  int nsplit;
  unsigned long long* attnpll;  // [H][attn_ngmax][kPartStride] tagged group partials (G >= 8)
  int attn_ngmax;               // groups per KV head at most: max(1, grid / KV)
  DecSync* sync;
  // [n_layers][KV] attention splits finished per layer and KV head (the
  // last split to finish merges and returns the word to zero; the next use
  // is the same layer of the next launch)
  unsigned int* attn_cnt;
  // The vectors that cross CTAs between phases -- the residual x, q/k/v and
  // the attention output -- are stored tagged, value | tag << 32 in one
  // 8-byte store, with tag = tag0 + 5 * layer + hand-off (0: x into QKV, 1:
  // q/k/v, 2: attention output, 3: x into gate/up).  A reader that sees the
  // tag sees the value, so no release fence sits between a phase's last
  // store and the barrier in front of the next phase: that barrier is a
  // relaxed gate that only keeps readers from polling early, and each reader
  // polls (bounded) for the tag.  The SwiGLU output h, the attention
  // partials and the argmax candidates keep plain stores behind
  // release/acquire synchronisation.
  unsigned long long* xll;     // [E]
  unsigned long long* qkvll;   // [(H + 2 KV) * 128] this rank's heads
  unsigned long long* attnll;  // [H * 128] this rank's heads
  uint32_t tag0;
  uint32_t* argmax;       // model's argmax word
  uint32_t* argmax2;      // optional caller's copy
  // Tensor parallelism: this is rank `rank` of `tp` (tp = 1 on one GPU).  H,
  // KV are this rank's heads, Fl its SwiGLU rows.  Attention and the SwiGLU
  // output stay local; attn_output and ffn_down hold this rank's columns
  // (the K split), so their epilogues produce partial sums of every row.  The
  // CTA owning a row stores its partial, tagged (tag0 + 5 * layer + 2 for O,
  // + 4 for down), into every rank's slot partll[p][(set * tp + rank) * E +
  // row] (set 0: O, 1: down) over NVLink, then waits (bounded) for the other
  // ranks' partials of the same row in its own slots and forms x + p_0 + p_1
  // + ... in rank order -- the sum the per-kernel path forms after its NCCL
  // all-gather -- so every rank holds the same residual and no per-layer
  // all-rank barrier is needed: a slot is rewritten only after every rank
  // has consumed its previous contents, which the data dependencies between
  // layers guarantee.  logitsg[p], candg[p] are rank p's copies of the
  // vocabulary slices and argmax candidates (one all-rank barrier per
  // token, at the head).  Pointers for p != rank are peer memory over NVLink.
  int tp, rank;
  int Hg;                 // query heads over all ranks
  int Fl;                 // this rank's SwiGLU rows
  int v_off;              // first vocabulary row of this rank's head slice
  float* hg[kMaxTp];      // [Fl] SwiGLU output of this rank's rows (local)
  unsigned long long* partll[kMaxTp];  // [2][tp][E] tagged partial O / down sums from every rank
  float* logitsg[kMaxTp]; // [V]
  int2* candg[kMaxTp];    // [tp * grid] per-CTA argmax candidates (value bits, global row)
  unsigned long long* xflagg[kMaxTp];  // [kMaxTp] per-source-rank barrier epochs
  // this launch's grid-barrier counter base and all-rank epoch base (the
  // counter and the epochs only grow)
  unsigned long long lbase, xepoch;
  // shared memory: [ring cap][staging stage_bytes][accumulators racc_bytes][phase table];
  // the staging region starts on a 1024-byte boundary
  int attn_dbuf;  // the staging + accumulator regions hold a second K/V tile buffer
  int* probe;     // set-up only: receives the shared-memory address of the dynamic region, nothing else runs
  int cap;
  int stage_bytes;
  int racc_bytes;
};

// Row-chunk bytes and aux offsets of a tile layout (make_tile_layout).
struct RcGeom {
  int rc, o_aux, o_aux2;
};
__host__ __device__ __forceinline__ RcGeom rc_geom(int dtype, int kc) {
  RcGeom g;
  if (dtype == kQ4_K) { g.o_aux = 32 * kc; g.o_aux2 = 0; g.rc = 36 * kc; }
  else if (dtype == kQ6_K) { g.o_aux = 48 * kc; g.o_aux2 = 52 * kc; g.rc = 52 * kc + round_up_int(kc / 2, 16); }
  else if (dtype == kQ5_K) { g.o_aux = 32 * kc; g.o_aux2 = 40 * kc; g.rc = 44 * kc; }
  else if (dtype == kQ4_0) { g.o_aux = 16 * kc; g.o_aux2 = 0; g.rc = 16 * kc + round_up_int(2 * kc, 16); }
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
#ifndef B2Q_TRACE_SLOTS
#define B2Q_TRACE_SLOTS 512
#endif
constexpr int kTraceSlots = B2Q_TRACE_SLOTS;
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
// fine stamps of one layer: [cta][32]
__device__ unsigned long long g_dec_fine[160 * 32];
__device__ int g_dec_fine_layer = 1;
// per CTA per phase: cycles warp 0 spent waiting for full stages, cycles of the whole consume
__device__ long long g_dec_wait[160 * 160 * 2];
#define B2Q_FTRACE(layer, i)                                                                  \
  do {                                                                                        \
    if (threadIdx.x % 128 == 0 && (layer) == g_dec_fine_layer && blockIdx.x < 160) {          \
      unsigned long long t_;                                                                  \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                  \
      g_dec_fine[blockIdx.x * 32 + (i)] = t_;                                                 \
    }                                                                                         \
  } while (0)
#define B2Q_DBG(prod, ph, v0, v1, v2, v3)                                                   \
  do {                                                                                     \
    if (blockIdx.x < 160 && (ph) < 160) {                                                 \
      int* d_ = g_dec_dbg + ((((prod) ? 160 : 0) + blockIdx.x) * 160 + (ph)) * 4;          \
      d_[0] = (v0); d_[1] = (v1); d_[2] = (v2); d_[3] = (v3);                              \
    }                                                                                      \
  } while (0)
#else
#define B2Q_DBG(prod, ph, v0, v1, v2, v3) do { } while (0)
#define B2Q_FTRACE(layer, i) do { } while (0)
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

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

// Tagged hand-offs (one GPU, see DecodeArgs): value | tag << 32, one
// single-copy-atomic 8-byte store.
__device__ __forceinline__ void ll_store(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// The value of `first` (an earlier load of p) once p carries `tag`.  A
// timeout raises the device error word and clears *s_ok, after which this
// CTA polls no more (the value is then whatever was read).
__device__ __forceinline__ float ll_value(const unsigned long long* p, unsigned long long first, uint32_t tag,
                                          volatile int* s_ok) {
  unsigned long long v = first;
  if ((uint32_t)(v >> 32) != tag) {
    // polls (rare: the value was stored but not yet visible) are bounded by
    // the wait limit in clock cycles
    const long long t0 = clock64(), lim = wait_limit();
    while ((uint32_t)(v >> 32) != tag && *s_ok && clock64() - t0 <= lim) {
      __nanosleep(32);
      v = ld_relaxed_u64(p);
    }
    if ((uint32_t)(v >> 32) != tag && *s_ok) {
      atomicExch(&g_b2q_device_error, 5);
      *s_ok = 0;
    }
  }
  return __uint_as_float((uint32_t)v);
}

// Tagged words crossing GPUs (tensor-parallel partial sums): system-scope
// 8-byte stores into a peer's memory and loads of the words peers wrote here.
__device__ __forceinline__ void ll_store_sys(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

// ll_value for words written by other GPUs (bounded polling, system scope).
__device__ __forceinline__ float ll_value_sys(const unsigned long long* p, unsigned long long first, uint32_t tag,
                                              volatile int* s_ok) {
  unsigned long long v = first;
  if ((uint32_t)(v >> 32) != tag) {
    const long long t0 = clock64(), lim = wait_limit();
    while ((uint32_t)(v >> 32) != tag && *s_ok && clock64() - t0 <= lim) {
      __nanosleep(64);
      v = ld_relaxed_sys_u64(p);
    }
    if ((uint32_t)(v >> 32) != tag && *s_ok) {
      atomicExch(&g_b2q_device_error, 5);
      *s_ok = 0;
    }
  }
  return __uint_as_float((uint32_t)v);
}

// consumer_sync that also returns whether `v` was true on any consumer thread
__device__ __forceinline__ bool consumer_sync_or(bool v) {
  unsigned r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 512, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((unsigned)v)
      : "memory");
  return r != 0;
}

// Barrier over the consumer warps of every CTA of this GPU.  The counter
// only grows: barrier number k of a launch completes at base + (k + 1) *
// gridDim.x arrivals (base: the count every earlier launch left).  The
// arrival is a release reduction that does not wait for a reply; `relaxed`
// (a gate in front of tagged hand-offs): a relaxed reduction and relaxed
// polling, no fence.  `s_ok` (shared) turns 0 when this CTA's wait gave up;
// later waits are skipped.
__device__ __forceinline__ void grid_sync(unsigned long long* bar, unsigned long long base, int& k,
                                          volatile int* s_ok, bool sys = false, bool relaxed = false) {
  consumer_sync();
  if (threadIdx.x == 0 && *s_ok) {
    // sys: the release also orders this CTA's stores into peer memory
    if (sys) asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
    else if (relaxed) asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
    else asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
    const unsigned long long target = base + (unsigned long long)(k + 1) * gridDim.x;
    const long long t0 = clock64(), lim = wait_limit();
    while ((relaxed ? ld_relaxed_u64(bar) : ld_acquire_u64(bar)) < target) {
      if (clock64() - t0 > lim) {
        atomicExch(&g_b2q_device_error, 5);
        *s_ok = 0;
        break;
      }
    }
  }
  ++k;
  consumer_sync();
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Barrier over every CTA of every rank, in two levels so that no address
// takes more than one write per rank over NVLink: the CTAs of this GPU meet
// at a grid barrier whose arrivals are system-scope releases (ordering their
// stores into peer memory); then on CTA 0 lane p of warp 0 publishes the
// barrier's epoch into peer p's flag slot for this rank (a system-scope
// release), and on every CTA lane p polls peer p's slot in its own memory
// (system-scope acquires) until it carries the epoch.  The lanes work in
// parallel, so the cost does not grow with the number of ranks.  One GPU:
// the grid barrier alone.
__device__ __forceinline__ void xgrid_sync(const DecodeArgs& a, unsigned long long* bar, int& k, int& kx,
                                           volatile int* s_ok, bool relaxed = false) {
  grid_sync(bar, a.lbase, k, s_ok, a.tp > 1, relaxed && a.tp == 1);
  if (a.tp == 1) return;
  const unsigned long long epoch = a.xepoch + (unsigned long long)(++kx);
  const int p = threadIdx.x;
  if (p < a.tp && p != a.rank && *s_ok) {
    if (blockIdx.x == 0) st_release_sys_u64(a.xflagg[p] + a.rank, epoch);
    const unsigned long long* slot = a.xflagg[a.rank] + p;
    const long long t0 = clock64(), lim = wait_limit();
    while (ld_acquire_sys_u64(slot) < epoch) {
      if (clock64() - t0 > lim) {
        atomicExch(&g_b2q_device_error, 5);
        *s_ok = 0;
        break;
      }
    }
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
constexpr int kStageBatch = 4;  // x elements per thread per load batch / 1024

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
// after the quantised row, `xs`); the norm weights are loaded together with
// x, so the staging costs one round trip per 4096 elements.  The sum of
// squares follows the reduction order of rmsnorm_quant_kernel's 1024-thread
// CTA exactly (consumer thread i plays threads i and i + 512), so the values
// are the same bits.  Quantisation: 8 lanes per block (xq_store_chunk8),
// warp w takes blocks 4w..4w+3, then 4w+64.. .  x is read from its tagged
// copy `xll`, whose elements must carry `tag` (polled for, bounded, in the
// rare case that some element is not yet visible).
__device__ __forceinline__ void stage_rmsnorm(const unsigned long long* xll, const float* w, int dim, float eps,
                                              const XQ& q, float* xs, float* red, int tl, int tb, uint32_t tag,
                                              volatile int* s_ok) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = q.kpad >> 6;
  float sa = 0.0f, sb = 0.0f;
  uint32_t bad = 0u;  // nonzero: some tagged element read here was not yet visible
  for (int e0 = 0; e0 < dim; e0 += 1024 * kStageBatch) {
    float va[kStageBatch], vb[kStageBatch];
    {  // every load of the batch in flight; the tags are checked in bulk below
      unsigned long long ua[kStageBatch], ub[kStageBatch];
#pragma unroll
      for (int i = 0; i < kStageBatch; ++i) {
        const int ea = e0 + 1024 * i + tid, eb = ea + 512;
        ua[i] = ea < dim ? ld_relaxed_u64(xll + ea) : (unsigned long long)tag << 32;
        ub[i] = eb < dim ? ld_relaxed_u64(xll + eb) : (unsigned long long)tag << 32;
      }
#pragma unroll
      for (int i = 0; i < kStageBatch; ++i) {
        bad |= ((uint32_t)(ua[i] >> 32) ^ tag) | ((uint32_t)(ub[i] >> 32) ^ tag);
        va[i] = __uint_as_float((uint32_t)ua[i]);
        vb[i] = __uint_as_float((uint32_t)ub[i]);
      }
    }
    if (e0 == 0) {  // norm weights towards L1 while x is in flight (one 128-byte line per thread)
      const int e = tid * 32;
      if (e < dim) asm volatile("prefetch.global.L1 [%0];" ::"l"(w + e));
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
  B2Q_FTRACE(tl, tb + 0);
  if (lane == 0) {
    red[warp] = sa;
    red[warp + 16] = sb;
  }
  if (consumer_sync_or(bad != 0u)) {
    // rare: read x again, polling for the tag, and redo the sums in the same order
    sa = sb = 0.0f;
    for (int e0 = 0; e0 < dim; e0 += 1024 * kStageBatch)
#pragma unroll
      for (int i = 0; i < kStageBatch; ++i) {
        const int ea = e0 + 1024 * i + tid, eb = ea + 512;
        if (ea < dim) {
          const float v = ll_value(xll + ea, ld_relaxed_u64(xll + ea), tag, s_ok);
          sa = fmaf(v, v, sa);
          xs[ea] = v;
        }
        if (eb < dim) {
          const float v = ll_value(xll + eb, ld_relaxed_u64(xll + eb), tag, s_ok);
          sb = fmaf(v, v, sb);
          xs[eb] = v;
        }
      }
    sa = warp_sum(sa);
    sb = warp_sum(sb);
    if (lane == 0) {
      red[warp] = sa;
      red[warp + 16] = sb;
    }
    consumer_sync();
  }
  B2Q_FTRACE(tl, tb + 1);
  const float tot = warp_sum(red[lane]);
  const float inv = 1.0f / sqrtf(tot / (float)dim + eps);
  B2Q_FTRACE(tl, tb + 2);
  for (int jq = 4 * warp; jq < nb; jq += 4 * kGemvConsumerWarps) {
    const int j = jq + (lane >> 3), e = j * 64 + (lane & 7) * 8;
    const bool in = e < dim;
    const float4 x0 = *reinterpret_cast<const float4*>(xs + e), x1 = *reinterpret_cast<const float4*>(xs + e + 4);
    const float4 w0 = in ? *reinterpret_cast<const float4*>(w + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 w1 = in ? *reinterpret_cast<const float4*>(w + e + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const float wvv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)  // (x * inv) * w, two separate roundings as the reference computes it
      v[i] = e + i < dim ? __fmul_rn(__fmul_rn(xv[i], inv), wvv[i]) : 0.0f;
    xq_store_chunk8(v, lane, 0, j, j < nb, q);
  }
  B2Q_FTRACE(tl, tb + 3);
  consumer_sync();
}

// Plain quantisation of src [dim] (quantize_x_kernel's values).
__device__ __forceinline__ void stage_plain(const float* src, int dim, const XQ& q) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = q.kpad >> 6;
  constexpr int kQ = 2;  // block quads per warp per batch
  for (int j0 = 4 * warp; j0 < nb; j0 += 4 * kGemvConsumerWarps * kQ) {
    float4 xv[kQ][2];
#pragma unroll
    for (int it = 0; it < kQ; ++it) {
      const int j = j0 + 4 * kGemvConsumerWarps * it + (lane >> 3), e = j * 64 + (lane & 7) * 8;
      const bool in = j < nb && e < dim;
      xv[it][0] = in ? __ldcg(reinterpret_cast<const float4*>(src + e)) : make_float4(0.f, 0.f, 0.f, 0.f);
      xv[it][1] = in ? __ldcg(reinterpret_cast<const float4*>(src + e + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int it = 0; it < kQ; ++it) {
      const int jq = j0 + 4 * kGemvConsumerWarps * it;
      if (jq >= nb) break;
      const int j = jq + (lane >> 3), e = j * 64 + (lane & 7) * 8;
      float v[8] = {xv[it][0].x, xv[it][0].y, xv[it][0].z, xv[it][0].w, xv[it][1].x, xv[it][1].y, xv[it][1].z, xv[it][1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (e + i >= dim) v[i] = 0.0f;
      xq_store_chunk8(v, lane, 0, j, j < nb, q);
    }
  }
  consumer_sync();
}

// Plain quantisation of a tagged vector (one GPU): its elements are read with
// coalesced 8-byte loads (polling for `tag`) into `xs` (shared memory, dim
// floats, rounded up to 8), then quantised from there -- the values of
// stage_plain.
__device__ __forceinline__ void stage_plain_ll(const unsigned long long* src, int dim, const XQ& q, float* xs,
                                               uint32_t tag, volatile int* s_ok) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = q.kpad >> 6;
  constexpr int kB = 2 * kStageBatch;  // loads in flight per thread
  uint32_t bad = 0u;
  for (int e0 = 0; e0 < dim; e0 += 512 * kB) {
    unsigned long long u[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int e = e0 + 512 * i + tid;
      u[i] = e < dim ? ld_relaxed_u64(src + e) : (unsigned long long)tag << 32;
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int e = e0 + 512 * i + tid;
      bad |= (uint32_t)(u[i] >> 32) ^ tag;
      if (e < dim) xs[e] = __uint_as_float((uint32_t)u[i]);
    }
  }
  if (consumer_sync_or(bad != 0u)) {  // rare: read again, polling for the tag
    for (int e = tid; e < dim; e += 512) xs[e] = ll_value(src + e, ld_relaxed_u64(src + e), tag, s_ok);
    consumer_sync();
  }
  for (int jq = 4 * warp; jq < nb; jq += 4 * kGemvConsumerWarps) {
    const int j = jq + (lane >> 3), e = j * 64 + (lane & 7) * 8;
    float v[8];
    if (e < dim) {
      const float4 x0 = *reinterpret_cast<const float4*>(xs + e), x1 = *reinterpret_cast<const float4*>(xs + e + 4);
      const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = e + i < dim ? xv[i] : 0.0f;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    xq_store_chunk8(v, lane, 0, j, true, q);
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
  // this CTA's attention work items (the consumers' grouping)
  const int nz = a.pos / kAttnTile + 1;
  const int tpg = attn_group_tiles(nz, a.KV, (int)gridDim.x), ng = (nz + tpg - 1) / tpg;
  for (int l = 0; l < a.n_layers; ++l) {
    const DecLayer& Ly = a.layers[l];
#pragma unroll 1
    for (int p = 0; p < kDecPhases; ++p) {
      if (p == 1 && tpg == 1) {
        // short contexts (one key tile per attention item), once the layer's
        // q/k/v weights are issued: the cached K/V tile of each of this
        // CTA's attention items into L2, so the copy that opens the item
        // finds it there (the K and the V rows of a 64-key tile are 16 KB
        // each, contiguous; the current token's row is written by the item
        // itself).  Measured +0.6 % at 512 keys (8B).  With several tiles
        // per item (8192 keys, 70B) prefetching all of them cost 1 % and the
        // first one alone 0.35 %: those groups copy each tile one ahead.
        for (int it = blockIdx.x; it < a.KV * ng; it += gridDim.x) {
          const int g = it / ng, zb = (it % ng) * tpg, ze = min(nz, zb + 1);
          for (int z = zb; z < ze; ++z) {
            const int rows = min(kAttnTile, a.max_seq - z * kAttnTile);  // inside this head's rows
            if (rows <= 0) break;
            const int64_t r0 = ((int64_t)g * a.max_seq + z * kAttnTile) * kHeadDim;
            const uint32_t bytes = (uint32_t)rows * kHeadDim * 2;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(Ly.kc + r0), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(Ly.vc + r0), "r"(bytes) : "memory");
          }
        }
      }
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

// The stage loop (DT: the GGML type, or < 0 to read it from the phase; one
// runtime-typed copy keeps the kernel within its registers).  DT == -1
// takes Q4_K, Q6_K and Q8_0 rows (the Q4_K_M / Q6_K / Q8_0 models); DT ==
// -2 adds Q5_K and Q4_0, in a separate kernel instance, so that the common
// loop carries no branch for them.  Software-pipelined: the warp
// reductions and accumulator updates of stage j are issued after the dot
// products of stage j + 1 have started, in the same straight-line block, so
// the shuffle latency overlaps integer work.
template <int DT>
__device__ __forceinline__ void consume_loop(Consumer& cs, const CtaPhase& ph, bool pair, const SX& sx, bool& ok,
                                             float* racc, long long& wsum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = warp >> 1, hf = warp & 1;  // row p of every tile; unit half hf
  const int gb = ph.gb, ge = ph.ge;
  const int nr = ph.dtype_nr >> 8;
  const int KC = ph.KC, C = ph.C, U = ph.U;
  const int dt = DT >= 0 ? DT : (ph.dtype_nr & 0xff);  // uniform over the CTA
  constexpr bool kAll = DT == -2;
  const RcGeom geo = rc_geom(dt, KC);
  const int tb = 8 * geo.rc;
  const int rows = (ge - gb) * 8;
  const int nw = pair ? 2 : 1;
  const int step = (pair || nr == 1) ? 1 : 2;
  const bool two = pair || nr == 2;
  const XPhase xp = make_xphase(lane);
  const int ul = lane + 32 * hf;
  const int csel = lane & 3;
  float* acc = racc + hf * nw * rows + p;  // this warp's row p, half hf
  XUnit X;
  bool uok = false;
  float q0 = 0.0f, q1 = 0.0f;  // previous stage's lane partials
  int d0 = 0, d1 = -1;         // their accumulator offsets (-1: none)
  for (int c = 0, g = gb; c < C && gb < ge;) {
    if (g == gb) {  // new chunk pass: this lane's activations
      const int u = c * KC + ul;
      uok = ul < KC && u < U;
      if (uok && ok) {
        if (dt == kQ4_K || (kAll && dt == kQ5_K)) xload_q4k(X, sx, 0, u, xp.f4);
        else if (dt == kQ6_K) xload_q6k(X, sx, 0, u, xp.f6a, xp.f6b);
        else if (kAll && dt == kQ4_0) xload_q40(X, sx, 0, u, xp.f8);
        else xload_q80(X, sx, 0, u, xp.f8);
      }
    }
    const bool nt2 = two && (pair || g + 1 < ge);
    int off = cs.ro;
    const int size = nt2 ? 2 * tb : tb;
    if (off + size > cs.R.cap) off = 0;
    if (!b2q_check(off + size <= cs.R.cap, kChkRing)) ok = false;  // outputs withheld
    cs.ro = off + size;
    const int slot = cs.j & (kRingSlots - 1);
#ifdef B2Q_DECODE_TRACE
    const long long tw0 = clock64();
#endif
    if (ok) ok = mbar_wait_bounded(&cs.R.full[slot], (uint32_t)((cs.j / kRingSlots) & 1));
#ifdef B2Q_DECODE_TRACE
    wsum += clock64() - tw0;
#endif
    // both rows unconditionally (the second re-reads the first tile when the
    // stage has one; lanes past the chunk compute on padding), masked after
    const uint8_t* rc = cs.R.base + off + p * geo.rc;
    const uint8_t* rc2 = nt2 ? rc + tb : rc;
    float p0, p1;
    if (dt == kQ4_K) {
      p0 = row_q4k(rc, KC, geo.o_aux, ul, csel, X);
      p1 = row_q4k(rc2, KC, geo.o_aux, ul, csel, X);
    } else if (dt == kQ6_K) {
      p0 = row_q6k(rc, KC, geo.o_aux, geo.o_aux2, ul, X);
      p1 = row_q6k(rc2, KC, geo.o_aux, geo.o_aux2, ul, X);
    } else if (kAll && dt == kQ5_K) {
      p0 = row_q5k(rc, KC, geo.o_aux, geo.o_aux2, ul, csel, X);
      p1 = row_q5k(rc2, KC, geo.o_aux, geo.o_aux2, ul, csel, X);
    } else if (kAll && dt == kQ4_0) {
      p0 = row_q40(rc, geo.o_aux, ul, X);
      p1 = row_q40(rc2, geo.o_aux, ul, X);
    } else {
      p0 = row_q80(rc, KC, geo.o_aux, ul, X);
      p1 = row_q80(rc2, KC, geo.o_aux, ul, X);
    }
    // the previous stage: reduce across the warp and accumulate (lane 0:
    // first row, lane 16: second row, when the stage had one)
    {
      const float sum = warp_sum2(q0, q1, lane);
      if (lane == 0) acc[d0] += sum;
      if (lane == 16 && d1 >= 0) acc[d1] += sum;
    }
    const bool live = ok && uok;
    q0 = live ? p0 : 0.0f;
    q1 = live && nt2 ? p1 : 0.0f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&cs.R.empty[slot]);  // the stage may be refilled
    ++cs.j;
    const int r = (g - gb) * 8;
    d0 = r;
    d1 = !nt2 ? -1 : pair ? rows + r : r + 8;  // up tile (same row) / next 8-row group
    g += step;
    if (g >= ge) {
      g = gb;
      ++c;
    }
  }
  {
    const float sum = warp_sum2(q0, q1, lane);
    if (lane == 0) acc[d0] += sum;
    if (lane == 16 && d1 >= 0) acc[d1] += sum;
  }
}

template <bool kAllTypes>
__device__ __forceinline__ void consume_phase(Consumer& cs, const CtaPhase& ph, bool pair, const SX& sx, bool& ok,
                                              float* racc, int tph = -1) {
  long long wsum = 0;
#ifdef B2Q_DECODE_TRACE
  const long long tc0 = clock64();
#endif
  const int rows = (ph.ge - ph.gb) * 8;
  const int nw = pair ? 2 : 1;
  for (int i = threadIdx.x; i < 2 * nw * rows; i += kGemvConsumerWarps * 32) racc[i] = 0.0f;
  consumer_sync();
  consume_loop<kAllTypes ? -2 : -1>(cs, ph, pair, sx, ok, racc, wsum);
#ifdef B2Q_DECODE_TRACE
  if (threadIdx.x == 0 && tph >= 0 && tph < 160 && blockIdx.x < 160) {
    g_dec_wait[(blockIdx.x * 160 + tph) * 2] = wsum;
    g_dec_wait[(blockIdx.x * 160 + tph) * 2 + 1] = clock64() - tc0;
  }
#endif
  (void)wsum;
  (void)tph;
  consumer_sync();
}

// Epilogue of a phase: rows [8 gb, min(8 ge, n)) of y.  Thread i handles
// rows i and i + 512 first; `xr` holds their residual (prefetched).
__device__ __forceinline__ float dec_racc(const float* racc, int rows, int nw, int r, int w) {
  return racc[w * rows + r] + racc[(nw + w) * rows + r];
}

// ---------------------------------------------------------------------------
// attention item (KV head g, group j of tpg consecutive key tiles) on the 16
// consumer warps: the work of rope_kv_kernel (for this head group) +
// attn_split_kernel + (last group of head g to finish) attn_combine_kernel,
// with the same arithmetic.  The tiles of the group are folded one after the
// other into a running softmax partial (AttnRun); the tile holding `pos`
// takes this token's k/v from registers (which are also appended to the
// cache), the other rows arrive by bulk copy.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int G>
__device__ __forceinline__ void attn_item(const DecodeArgs& a, const DecLayer& Ly, int g, int j, int ng, int tpg,
                                          int nz, AttnTile<G>& T, __half* kb2, uint64_t* bar, int& uses,
                                          uint64_t* bar2, int& uses2, int* s_last, int tl, volatile int* s_ok) {
  constexpr int HD = kHeadDim, HALF = kHeadDim / 2;
  constexpr int R = (G * HD + kAttnThreads - 1) / kAttnThreads;
  const int gt = threadIdx.x;  // 0..511
  const int pos = a.pos, cap = a.max_seq;
  const int H = a.H, KV = a.KV;
  const int z0 = j * tpg, z1 = min(nz, z0 + tpg);
  const bool last = z1 == nz;  // this group holds the tile with the current token
  // K/V tile z by TMA into buffer b (0: T.k / T.v, 1: the second buffer
  // kb2, when the region holds one: the group's tiles are then
  // double-buffered, tile z + 1 in flight while tile z is computed).  The
  // current token's row is copied in from T.kcur / T.vcur once its tile has
  // landed; a tile with no other row is not loaded.  (Double buffering is
  // compiled in for eight query heads per KV head only, the widths whose
  // staging region holds the second buffer; the other instances keep their
  // registers.)
  const bool dbuf = G >= 8 && kb2 != nullptr;
  auto kbuf = [&](int b) { return b ? kb2 : T.k; };
  auto vbuf = [&](int b) { return b ? kb2 + kAttnTile * HD : T.v; };
  auto load = [&](int z, int b) {
    const int nv = min(kAttnTile, pos + 1 - z * kAttnTile);
    int nload = z == nz - 1 ? nv - 1 : nv;
    if (!b2q_check(g >= 0 && g < KV && z >= 0 && z * kAttnTile < cap, kChkAttnRows)) nload = 0;  // (uniform)
    if (gt == 0 && nload > 0) {
      fence_proxy_async_smem();  // earlier generic accesses to this region come first
      attn_rows_load(kbuf(b), vbuf(b), Ly.tmk, Ly.tmv, g * cap + z * kAttnTile, b ? bar2 : bar);
    }
    return nload;
  };
  int nl[2] = {load(z0, 0), 0};
  const int p_rope = pos < 8191 ? pos : 8191;
  const float* cs = a.rope_cos + (int64_t)p_rope * HALF;
  const float* sn = a.rope_sin + (int64_t)p_rope * HALF;
  // work index w < G*64: one q pair; [G*64, G*64 + 64): a k pair of this
  // token (last group); [G*64 + 64, G*64 + 192): a v value.  RW indices per
  // thread (one up to four query heads per KV head), all loads issued first.
  constexpr int RW = (G * HALF + HALF + HD + kAttnThreads - 1) / kAttnThreads;
  const int qn = G * HALF, nwork = qn + (last ? HALF + HD : 0);
  float x0[RW], x1[RW], c[RW], sv[RW];
  int o0[RW], o1[RW];  // offsets of the thread's inputs in q|k|v (-1: none)
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int w = gt + kAttnThreads * r;
    c[r] = sv[r] = 0.0f;
    o0[r] = o1[r] = -1;
    if (w < qn) {
      const int hh = w / HALF, jj = w % HALF, h = g * G + hh;
      o0[r] = h * HD + jj;
      o1[r] = o0[r] + HALF;
      c[r] = cs[jj];
      sv[r] = sn[jj];
    } else if (w < qn + HALF && w < nwork) {
      const int jj = w - qn;
      o0[r] = (H + g) * HD + jj;
      o1[r] = o0[r] + HALF;
      c[r] = cs[jj];
      sv[r] = sn[jj];
    } else if (w < nwork) {
      o0[r] = (H + KV) * HD + g * HD + (w - qn - HALF);
    }
  }
  {  // tagged q|k|v
    const uint32_t tq = a.tag0 + (uint32_t)(5 * tl + 1);
    unsigned long long u0[RW], u1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      u0[r] = o0[r] >= 0 ? ld_relaxed_u64(a.qkvll + o0[r]) : 0ull;
      u1[r] = o1[r] >= 0 ? ld_relaxed_u64(a.qkvll + o1[r]) : 0ull;
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      x0[r] = o0[r] >= 0 ? ll_value(a.qkvll + o0[r], u0[r], tq, s_ok) : 0.0f;
      x1[r] = o1[r] >= 0 ? ll_value(a.qkvll + o1[r], u1[r], tq, s_ok) : 0.0f;
    }
  }
  // optional biases: q rows h*HD + j, k rows (H + g)*HD + j, v rows
  // (H + KV + g)*HD + j of q|k|v map to offset o - {0, H*HD, (H+KV)*HD} of
  // the layer's q, k, v bias vectors
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    if (o0[r] < 0) continue;
    const float* b = o0[r] < H * HD ? Ly.qb : o0[r] < (H + KV) * HD ? Ly.kb : Ly.vb;
    if (b == nullptr) continue;
    const int bo = o0[r] < H * HD ? o0[r] : o0[r] < (H + KV) * HD ? o0[r] - H * HD : o0[r] - (H + KV) * HD;
    x0[r] += b[bo];
    if (o1[r] >= 0) x1[r] += b[bo + HALF];
  }
  // rotated q into the tile; this token's rotated k and its v into the cache
  // and into T.kcur / T.vcur (copied into its tile in the tile loop)
  __half* const krow = T.kcur;
  __half* const vrow = T.vcur;
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int w = gt + kAttnThreads * r;
    if (w < qn) {
      const int hh = w / HALF, jj = w % HALF;
      attn_set_q(T, hh, jj, __fsub_rn(__fmul_rn(x0[r], c[r]), __fmul_rn(x1[r], sv[r])));
      attn_set_q(T, hh, HALF + jj, __fadd_rn(__fmul_rn(x1[r], c[r]), __fmul_rn(x0[r], sv[r])));
    } else if (w < qn + HALF && w < nwork) {
      const int jj = w - qn;
      const __half y0 = __float2half_rn(__fsub_rn(__fmul_rn(x0[r], c[r]), __fmul_rn(x1[r], sv[r])));
      const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1[r], c[r]), __fmul_rn(x0[r], sv[r])));
      __half* dst = Ly.kc + ((int64_t)g * cap + pos) * HD;
      dst[jj] = y0;
      dst[HALF + jj] = y1;
      krow[jj] = y0;
      krow[HALF + jj] = y1;
    } else if (w < nwork) {
      const int jj = w - qn - HALF;
      const __half hv = __float2half_rn(x0[r]);
      Ly.vc[((int64_t)g * cap + pos) * HD + jj] = hv;
      vrow[jj] = hv;
    }
  }
  B2Q_FTRACE(tl, 10);
  AttnRun<R> run;
  run.init();
  for (int z = z0; z < z1; ++z) {
    const int nv = min(kAttnTile, pos + 1 - z * kAttnTile);
    const int b = dbuf ? (z - z0) & 1 : 0;
    if (z > z0) {
      consumer_sync();  // the previous tile's shared-memory reads are done
      if (!dbuf) nl[0] = load(z, 0);
    }
    if (dbuf && z + 1 < z1) nl[b ^ 1] = load(z + 1, b ^ 1);  // into the buffer tile z - 1 has left
    if (nl[b] > 0) {  // a timeout is recorded in the device error word
      if (b) mbar_wait_bounded(bar2, (uint32_t)(uses2++ & 1));
      else mbar_wait_bounded(bar, (uint32_t)(uses++ & 1));
    }
    if (z == nz - 1) {  // the current token's row, over what the copy brought
      if (z == z0) consumer_sync();  // T.kcur / T.vcur written above
      if (gt < HD && b2q_check(nv >= 1 && nv <= kAttnTile, kChkAttnTok)) {
        kbuf(b)[kv_off(nv - 1, gt)] = T.kcur[gt];
        vbuf(b)[kv_off(nv - 1, gt)] = T.vcur[gt];
      }
    }
    consumer_sync();
    attn_tile_compute_emit<G>(T, kbuf(b), vbuf(b), nv, a.scale, [] { consumer_sync(); },
                              [&](int r, int, int, float mt, float lt, float ot) { run.fold(r, mt, lt, ot); });
  }
  B2Q_FTRACE(tl, 11);
  if constexpr (G >= 8) {
    // long-context widths (eight query heads per KV head, many groups per
    // head): the group partials {max, sum, O[128]} are stored tagged, and
    // the ng groups of the head each finalise a slice of its G*128 outputs
    // from every group's partial (polled, bounded) -- no counter, no fence,
    // no serial merge.  attn_combine_kernel's arithmetic, same group order.
    const uint32_t tp = a.tag0 + (uint32_t)(5 * tl + 2);
    const int ngm = a.attn_ngmax;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = gt + kAttnThreads * r;
      if (i < G * HD && b2q_check(j < ngm, kChkPart)) {
        const int h = i / HD, d = i % HD;
        unsigned long long* pp = a.attnpll + ((int64_t)(g * G + h) * ngm + j) * kPartStride;
        if (d == 0) {
          ll_store(pp, run.m[r], tp);
          ll_store(pp + 1, run.l[r], tp);
        }
        ll_store(pp + 2 + d, run.o[r], tp);
      }
    }
    B2Q_FTRACE(tl, 12);
    consumer_sync();  // the tile buffers are free for the gathered partials
    const int n = G * HD;
    const int e0 = n * j / ng, ne = n * (j + 1) / ng - e0, np = ne * ng;
    float* sm_m = reinterpret_cast<float*>(T.k);
    float* sm_l = sm_m + np;
    float* sm_o = sm_l + np;
    for (int i = gt; i < np; i += kAttnThreads) {
      const int el = i / ng, z = i - el * ng, e = e0 + el;
      const unsigned long long* pw = a.attnpll + ((int64_t)(g * G + e / HD) * ngm + z) * kPartStride;
      const unsigned long long u0 = ld_relaxed_u64(pw), u1 = ld_relaxed_u64(pw + 1),
                               u2 = ld_relaxed_u64(pw + 2 + e % HD);
      sm_m[i] = ll_value(pw, u0, tp, s_ok);
      sm_l[i] = ll_value(pw + 1, u1, tp, s_ok);
      sm_o[i] = ll_value(pw + 2 + e % HD, u2, tp, s_ok);
    }
    consumer_sync();
    B2Q_FTRACE(tl, 13);
    for (int el = gt; el < ne; el += kAttnThreads) {
      const float* m = sm_m + el * ng;
      float M = -INFINITY;
      for (int z = 0; z < ng; ++z) M = fmaxf(M, m[z]);
      float L = 0.0f, O = 0.0f;
      for (int z = 0; z < ng; ++z) {
        const float f = m[z] == -INFINITY ? 0.0f : expf(m[z] - M);
        L = fmaf(f, sm_l[el * ng + z], L);
        O = fmaf(f, sm_o[el * ng + z], O);
      }
      const int oi = g * n + e0 + el;  // this rank's heads, local
      if (b2q_check(oi < a.H * HD, kChkTag)) ll_store(a.attnll + oi, O * (1.0f / fmaxf(L, 1e-12f)), tp);
    }
    B2Q_FTRACE(tl, 14);
  } else {
  #pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = gt + kAttnThreads * r;
      if (i < G * HD) attn_store_partial(a.part, g, G, j, a.nsplit, i / HD, i % HD, run.m[r], run.l[r], run.o[r]);
    }
    // the last group of this KV head to finish merges all of them
    consumer_sync();
    B2Q_FTRACE(tl, 12);
    if (gt == 0) {
      // one acquire-release arrival: it releases this CTA's partials (the
      // stores of every thread, ordered before it by the CTA barrier) and,
      // for the last arrival, acquires every other group's
      unsigned int old;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                   : "=r"(old)
                   : "l"(&a.attn_cnt[tl * KV + g])
                   : "memory");
      *s_last = old == (unsigned int)(ng - 1);
    }
    consumer_sync();
    B2Q_FTRACE(tl, 13);
    if (*s_last) {
      // merge (attn_combine_kernel's arithmetic, same order): the partials of
      // up to kZc groups per head are brought into the idle tile with bulk
      // copies (one round trip), then reduced in group order
      const int nsplit = a.nsplit;
      constexpr int kZc = (2 * kAttnTile * HD / 2) / (G * kPartStride);  // splits per chunk (T.k + T.v)
      float* pb = reinterpret_cast<float*>(T.k);                          // [G][zc][kPartStride]
      float M[R], Ls[R], O[R];
  #pragma unroll
      for (int r = 0; r < R; ++r) {
        M[r] = -INFINITY;
        Ls[r] = 0.0f;
        O[r] = 0.0f;
      }
      if (ng > kZc) {  // many groups: the maxima of every partial first, 8 loads in flight
  #pragma unroll
        for (int r = 0; r < R; ++r) {
          const int i = gt + kAttnThreads * r;
          if (i >= G * HD) continue;
          const float* ph = a.part + (int64_t)(g * G + i / HD) * nsplit * kPartStride;
          for (int zz0 = 0; zz0 < ng; zz0 += 8) {
            float mv[8];
  #pragma unroll
            for (int u = 0; u < 8; ++u) mv[u] = zz0 + u < ng ? __ldcg(ph + (zz0 + u) * kPartStride) : -INFINITY;
  #pragma unroll
            for (int u = 0; u < 8; ++u) M[r] = fmaxf(M[r], mv[u]);
          }
        }
      }
      for (int z0 = 0; z0 < ng; z0 += kZc) {
        const int zn = min(kZc, ng - z0);
        if (gt == 0) {
          asm volatile("fence.proxy.async.global;" ::: "memory");
          fence_proxy_async_smem();
          const uint32_t bytes = (uint32_t)zn * kPartStride * 4;
          mbar_arrive_expect_tx(bar, bytes * G);
          for (int h = 0; h < G; ++h)
            bulk_g2s(pb + h * zn * kPartStride, a.part + ((int64_t)(g * G + h) * nsplit + z0) * kPartStride, bytes, bar);
        }
        mbar_wait_bounded(bar, (uint32_t)(uses & 1));
        ++uses;
  #pragma unroll
        for (int r = 0; r < R; ++r) {
          const int i = gt + kAttnThreads * r;
          if (i >= G * HD) continue;
          const int h = i / HD, d = i % HD;
          const float* ph = pb + h * zn * kPartStride;
          if (ng <= kZc)  // one chunk holds every partial: maxima from shared memory
            for (int zz = 0; zz < zn; ++zz) M[r] = fmaxf(M[r], ph[zz * kPartStride]);
          for (int zz = 0; zz < zn; ++zz) {
            const float m = ph[zz * kPartStride];
            const float f = m == -INFINITY ? 0.0f : expf(m - M[r]);
            Ls[r] = fmaf(f, ph[zz * kPartStride + 1], Ls[r]);
            O[r] = fmaf(f, ph[zz * kPartStride + 2 + d], O[r]);
          }
        }
        consumer_sync();  // chunk consumed before the next copy lands
      }
  #pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = gt + kAttnThreads * r;
        if (i < G * HD) {
          const float v = O[r] * (1.0f / fmaxf(Ls[r], 1e-12f));
          const int oi = (g * G + i / HD) * HD + i % HD;  // this rank's heads, local
          if (b2q_check(oi < a.H * HD, kChkTag)) ll_store(a.attnll + oi, v, a.tag0 + (uint32_t)(5 * tl + 2));
        }
      }
      if (gt == 0) a.attn_cnt[tl * KV + g] = 0u;
      B2Q_FTRACE(tl, 14);
    }
  }
  consumer_sync();  // the tile (and s_last) are reused by the next item
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
// G: query heads per KV head; kAllTypes: the stage loop also takes Q5_K and
// Q4_0 rows.
template <int G, bool kAllTypes>
__global__ void __launch_bounds__(kGemvThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  if (a.probe != nullptr) {  // layout query
    if (blockIdx.x == 0 && threadIdx.x == 0) *a.probe = (int)smem_u32(smem);
    return;
  }
  __shared__ uint64_t full_bar[kRingSlots], empty_bar[kRingSlots];
  __shared__ int ring_qs[kRingSlots], ring_qe[kRingSlots];
  __shared__ float red[32];
  __shared__ int s_ok;
  __shared__ float s_bv[kGemvConsumerWarps];
  __shared__ int s_bi[kGemvConsumerWarps];
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
  if ((smem_u32(xs) & 1023u) != 0u) {  // the layout the host planned (never expected to differ)
    if (threadIdx.x == 0) atomicExch(&g_b2q_device_error, 3);
    return;  // every CTA alike, before any exchange
  }
  if (kChecks && !b2q_check((size_t)a.cap + a.stage_bytes + a.racc_bytes + (size_t)a.nph * sizeof(CtaPhase) <=
                                dyn_smem_bytes(),
                            kChkStage))
    return;  // (uniform, before any exchange)

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
  int nbar = 0, nxbar = 0;  // this-GPU and all-rank barriers passed
  const int kp_e = round_up_int(a.E, 256);
  float* xcopy = reinterpret_cast<float*>(xs + xq_smem_bytes(kp_e));

  // this CTA's phase table, and the token embedding (embed_rows_kernel's
  // values): every CTA dequantises the row into shared memory and stores its
  // slice of x, tagged
  {
    const int4* src = reinterpret_cast<const int4*>(a.ctab + (size_t)blockIdx.x * a.nph);
    int4* dst = reinterpret_cast<int4*>(tab);
    for (int i = threadIdx.x; i < a.nph * 2; i += kGemvConsumerWarps * 32) dst[i] = __ldcg(src + i);
    uint32_t tok = a.token != nullptr ? a.token[0] : a.token_imm;
    if (tok >= (uint32_t)a.V) tok = 0;
    const uint8_t* rowp = a.tok_raw + (int64_t)tok * a.tok_row_bytes;
    const int64_t slots = dequant_slots(a.tok_dtype, a.E);
    for (int64_t sl = threadIdx.x; sl < slots; sl += kGemvConsumerWarps * 32) dequant_slot(rowp, a.tok_dtype, sl, xcopy);
    consumer_sync();
    const int e0 = (int)((int64_t)a.E * blockIdx.x / gridDim.x), e1 = (int)((int64_t)a.E * (blockIdx.x + 1) / gridDim.x);
    for (int e = e0 + threadIdx.x; e < e1; e += kGemvConsumerWarps * 32) ll_store(a.xll + e, xcopy[e], a.tag0);
  }
  grid_sync(bar, a.lbase, nbar, okp, false, true);

  const int nz = a.pos / kAttnTile + 1;  // key tiles of this step
  const int tpg = attn_group_tiles(nz, a.KV, (int)gridDim.x), ng = (nz + tpg - 1) / tpg;
  int attn_uses = 0, attn_uses2 = 0;  // completed phases of the two attention mbarriers
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
    (void)tslot;
    B2Q_TRACE(tslot);
    B2Q_FTRACE(l, 16 + k);
    if (k == 1) {  // RoPE, KV append, attention
      const DecLayer& Ly = a.layers[l];
      // [second K/V buffer (double buffering, eight query heads per KV head
      // only)][AttnTile], from a 1024-byte boundary of the staging region
      const bool dbuf = G >= 8 && a.attn_dbuf;
      uint8_t* ab = xs;
      __half* kb2 = dbuf ? reinterpret_cast<__half*>(ab) : nullptr;
      AttnTile<G>& T = *reinterpret_cast<AttnTile<G>*>(ab + (dbuf ? kAttnTileBytes : 0u));
      for (int it = blockIdx.x; it < a.KV * ng; it += gridDim.x)
        attn_item<G>(a, Ly, it / ng, it % ng, ng, tpg, nz, T, kb2, &attn_bar[0], attn_uses, &attn_bar[1],
                     attn_uses2, &attn_last[0], l, okp);
      B2Q_TRACE(tslot + 2);
      grid_sync(bar, a.lbase, nbar, okp, false, true);  // the O projection reads this rank's heads
      continue;
    }
    const CtaPhase& ph = tab[head ? 4 * a.n_layers : 4 * l + (k == 0 ? 0 : k - 1)];
    if (ph.gb < ph.ge) {
      const bool add = k == 2 || k == 4;  // O / down: the residual update
      const int row0 = ph.gb * 8, nrows = min(ph.ge * 8, ph.n) - row0;
      const int rows = (ph.ge - ph.gb) * 8;
      // global row of local row 0 (head: vocabulary rows of this rank)
      const int grow0 = row0 + (head ? a.v_off : 0);
      // residual rows of this CTA (tagged): copied (L2 -> shared,
      // asynchronously) behind the accumulators while the input is staged;
      // the epilogue checks each tag (and polls x for it if the copy was
      // early, which only a CTA that staged no input of the previous phase
      // can meet)
      unsigned long long* resid = reinterpret_cast<unsigned long long*>(racc + 2 * rows);
      if (add)
        for (int r2 = threadIdx.x; 2 * r2 < nrows; r2 += kGemvConsumerWarps * 32)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(resid + 2 * r2)),
                       "l"(a.xll + grow0 + 2 * r2)
                       : "memory");
      // stage the input: rmsnorm(x) for QKV, gate/up and the head; attn; h
      bool stage_ok = true;
      if (kChecks) {
        const size_t need = k == 2 ? xq_smem_bytes(round_up_int(a.H * kHeadDim, 256)) +
                                         (size_t)4 * round_up_int(a.H * kHeadDim, 8)
                            : k == 4 ? xq_smem_bytes(round_up_int(a.Fl, 256))
                                     : xq_smem_bytes(kp_e) + (size_t)4 * a.E;
        stage_ok = b2q_check(need <= (size_t)a.stage_bytes, kChkStage);
        if (!stage_ok) ok = false;  // nothing staged, outputs withheld
      }
      XQ q;
      if (!stage_ok) {
        q = smem_xq(xs, kp_e);
      } else if (k == 2) {
        const int kp_a = round_up_int(a.H * kHeadDim, 256);
        q = smem_xq(xs, kp_a);
        stage_plain_ll(a.attnll, a.H * kHeadDim, q, reinterpret_cast<float*>(xs + xq_smem_bytes(kp_a)),
                       a.tag0 + (uint32_t)(5 * l + 2), okp);
      } else if (k == 4) {
        q = smem_xq(xs, round_up_int(a.Fl, 256));
        stage_plain(a.hg[a.rank], a.Fl, q);
      } else {
        q = smem_xq(xs, kp_e);
        const float* nw = head ? a.out_norm : (k == 0 ? a.layers[l].attn_norm : a.layers[l].ffn_norm);
        stage_rmsnorm(a.xll, nw, a.E, a.eps, q, xcopy, red, l, k == 0 ? 0 : 4,
                      a.tag0 + (uint32_t)(5 * l + (k == 0 ? 0 : 3)), okp);
      }
      B2Q_TRACE(tslot + 1);
      B2Q_FTRACE(l, 21 + k);
      const bool pair = k == 3;
      consume_phase<kAllTypes>(cs, ph, pair, smem_sx(q), ok, racc, head ? 4 * a.n_layers : 4 * l + (k == 0 ? 0 : k - 1));
      // epilogue
      if (add) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        consumer_sync();
      }
      if (ok && add && a.tp > 1) {
        // x + p_0 + p_1 + ... (rank order), tagged for the next phase.  v is
        // this rank's partial sum of a row (its columns of attn_output /
        // ffn_down); it goes, tagged, into every rank's slot for this rank
        // over NVLink, and the row's other partials arrive in this rank's
        // slots the same way.  Three passes, the partials gathered through
        // shared memory behind the accumulators and residual rows.
        const uint32_t tp_tag = a.tag0 + (uint32_t)(5 * l + (k == 2 ? 2 : 4));
        const size_t set = (size_t)(k == 2 ? 0 : 1) * a.tp;
        float* pv = racc + 4 * rows;  // [tp][rows]
        for (int r = threadIdx.x; r < nrows; r += kGemvConsumerWarps * 32) {
          const float v = dec_racc(racc, rows, 1, r, 0);
          if (b2q_check(grow0 + r < a.E && a.rank < a.tp, kChkTpSlot))
            for (int p = 0; p < a.tp; ++p) ll_store_sys(a.partll[p] + (set + a.rank) * a.E + grow0 + r, v, tp_tag);
          pv[a.rank * rows + r] = v;
        }
        for (int i = threadIdx.x; i < a.tp * nrows; i += kGemvConsumerWarps * 32) {
          const int p = i / nrows, r = i - p * nrows;
          if (p == a.rank) continue;
          const unsigned long long* w = a.partll[a.rank] + (set + p) * a.E + grow0 + r;
          pv[p * rows + r] = ll_value_sys(w, ld_relaxed_sys_u64(w), tp_tag, okp);
        }
        consumer_sync();
        for (int r = threadIdx.x; r < nrows; r += kGemvConsumerWarps * 32) {
          float sum = ll_value(a.xll + grow0 + r, resid[r], a.tag0 + (uint32_t)(5 * l + (k == 2 ? 0 : 3)), okp);
          for (int p = 0; p < a.tp; ++p) sum += pv[p * rows + r];
          if (b2q_check(grow0 + r < a.E, kChkTag))
            ll_store(a.xll + grow0 + r, sum, a.tag0 + (uint32_t)(k == 2 ? 5 * l + 3 : 5 * (l + 1)));
        }
      } else if (ok) {
        const int nw = pair ? 2 : 1;
        for (int r = threadIdx.x; r < nrows; r += kGemvConsumerWarps * 32) {
          const float v = dec_racc(racc, rows, nw, r, 0);
          if (k == 0 && !head) {  // q/k/v: this rank's heads, local
            if (b2q_check(ph.ycol + row0 + r < (a.H + 2 * a.KV) * kHeadDim, kChkTag))
              ll_store(a.qkvll + ph.ycol + row0 + r, v, a.tag0 + (uint32_t)(5 * l + 1));
            continue;
          }
          if (pair) {  // SwiGLU rows of this rank, local
            a.hg[a.rank][row0 + r] = silu_f(v) * dec_racc(racc, rows, nw, r, 1);
            continue;
          }
          if (add) {  // one GPU: x += v, tagged for the next phase (gate/up, or the next layer's QKV)
            const float xr = ll_value(a.xll + grow0 + r, resid[r], a.tag0 + (uint32_t)(5 * l + (k == 2 ? 0 : 3)), okp);
            if (b2q_check(grow0 + r < a.E, kChkTag))
              ll_store(a.xll + grow0 + r, xr + v, a.tag0 + (uint32_t)(k == 2 ? 5 * l + 3 : 5 * (l + 1)));
            continue;
          }
          // the head: this rank's vocabulary slice into every rank's logits
          for (int p = 0; p < a.tp; ++p) a.logitsg[p][grow0 + r] = v;
          if (v > best) { best = v; idx = grow0 + r; }
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
    if (head) break;
    // gates in front of tagged data (relaxed), except h after gate/up
    grid_sync(bar, a.lbase, nbar, okp, false, k != 3);
  }
  warp_argmax(best, idx);
  if (lane == 0) { s_bv[warp] = best; s_bi[warp] = idx; }
  consumer_sync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kGemvConsumerWarps; ++w) argmax_merge(best, idx, s_bv[w], s_bi[w]);
    const int2 cv = make_int2(__float_as_int(best), idx);
    for (int p = 0; p < a.tp; ++p) a.candg[p][a.rank * gridDim.x + blockIdx.x] = cv;
  }
  xgrid_sync(a, bar, nbar, nxbar, okp);  // every CTA's candidate, every rank's logits
  if (blockIdx.x == 0 && warp == 0) {
    best = -INFINITY;
    idx = 0x7fffffff;
    const int2* cand = a.candg[a.rank];
    for (int c = lane; c < a.tp * (int)gridDim.x; c += 32) {
      const int2 cv = __ldcg(cand + c);
      argmax_merge(best, idx, __int_as_float(cv.x), cv.y);
    }
    warp_argmax(best, idx);
    if (lane == 0) {
      const uint32_t r = idx == 0x7fffffff ? 0u : (uint32_t)idx;
      *a.argmax = r;
      if (a.argmax2 != nullptr) *a.argmax2 = r;
    }
  }
}

}  // namespace b2q
