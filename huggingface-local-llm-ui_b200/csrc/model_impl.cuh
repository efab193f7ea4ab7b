// model_impl.cuh -- the Llama forward on the device (StandardNativeEngine,
// inference.rs:2406-2860), with the activations and the f16 KV cache kept in
// HBM for the whole step, and the single-token decode step captured as one
// CUDA graph.  Included by b2q_api.cu (single translation unit).
#pragma once

#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <cuda.h>  // CUtensorMap and its enums (the encoder comes from the driver at run time)

#include "internal.h"
#include "tp.h"

namespace b2q {

struct LayerW {
  b2q_weight *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  b2q_weight *gate = nullptr, *up = nullptr, *down = nullptr;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
  float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
  __half *kc = nullptr, *vc = nullptr;
  const CUtensorMap *tmk = nullptr, *tmv = nullptr;  // TMA descriptors of kc / vc (device)
};

// cuTensorMapEncodeTiled, resolved through the runtime's driver entry point
// (no link-time dependency on the driver library)
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static TmapEncodeFn tmap_encoder() {
  static TmapEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TmapEncodeFn>(p);
  });
  return fn;
}

// TMA descriptor of one KV cache, `rows` rows of kHeadDim f16: boxes of
// kAttnTile rows x 64 dims (128 bytes) with the 128-byte swizzle, the layout
// attn_rows_load and kv_off expect; rows past the end read as zeros.
static bool kv_tensor_map(CUtensorMap* out, void* base, uint64_t rows) {
  const TmapEncodeFn enc = tmap_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * sizeof(__half)};
  const cuuint32_t box[2] = {64u, (cuuint32_t)kAttnTile};
  const cuuint32_t estr[2] = {1u, 1u};
  return enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kPrefillChunk = 256;  // tokens per forward pass of a long prompt (one tensor-core N tile)

}  // namespace b2q

struct b2q_model {
  b2q_engine* eng = nullptr;
  b2q_model_config c{};
  cudaStream_t st = nullptr;
  // weights
  void* tok_raw = nullptr;  // raw GGUF token_embd for the row lookup
  int tok_dtype = 0;
  int64_t tok_row_bytes = 0;
  b2q_weight* output = nullptr;
  float* output_norm = nullptr;
  std::vector<b2q::LayerW> L;
  size_t weight_bytes = 0;
  // tensor-parallel shard sizes (local)
  int H_loc = 0, KV_loc = 0, F_loc = 0, V_loc = 0;
  b2q::TpComm tp;
  // activations
  float* x = nullptr;       // [mmax][E] residual stream
  float* qkv = nullptr;     // [mmax][(H_loc + 2 KV_loc) hd]
  float* attn = nullptr;    // [mmax][H hd] (gathered under TP)
  float* attn_loc = nullptr;
  float* hbuf = nullptr;    // [mmax][F] (gathered under TP)
  float* h_loc = nullptr;
  float* y_loc = nullptr;   // [mmax][E_loc] local o-proj / down rows (TP)
  float* logits = nullptr;  // [V]
  float* logits_loc = nullptr;
  float* part = nullptr;    // attention split partials
  CUtensorMap* kv_maps = nullptr;  // [n_layers][K, V] TMA descriptors of the KV caches
  uint32_t* tokens = nullptr;
  uint32_t* argmax = nullptr;
  int* pos = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  b2q::XQBuf xq_e, xq_a, xq_f;
  int nsplit = 0;
  int mmax = b2q::kPrefillChunk;
  // host staging (pinned) for b2q_forward's token ids, and the device error
  // word read back by the blocking forward entry points
  uint32_t* h_tok = nullptr;
  int* h_err = nullptr;
  // decode graph (m = 1)
  cudaGraphExec_t graph = nullptr;
  uint64_t graph_kernels = 0;
  // persistent decode kernel (m = 1, one GPU)
  b2q::DecLayer* dec_layers = nullptr;
  b2q::CtaPhase* dec_tab = nullptr;
  void* dec_xblock = nullptr;              // exchanged vectors of this rank (see DecodeArgs)
  void* dec_peer[b2q::kMaxTp] = {nullptr};  // peers' blocks (IPC-mapped), tensor parallelism
  float* dec_logits = nullptr;
  uint64_t dec_launches = 0;
  const float* last_logits = nullptr;       // where the last forward left its logits
  b2q::DecSync* dec_sync = nullptr;
  unsigned int* dec_attn_cnt = nullptr;      // [n_layers][KV_loc] attention split arrivals
  unsigned long long* dec_ll = nullptr;      // tagged x | q|k|v | attention output
  size_t dec_ll_words = 0;
  b2q::DecodeArgs dec{};
  size_t dec_smem = 0;
  int dec_G = 0;
  bool dec_all = false;  // the persistent kernel instance that also takes Q5_K / Q4_0 rows
  bool dec_on = false;
  bool finalized = false;
  std::map<std::string, bool> have;
};

namespace b2q {

static b2q_status model_cuda(cudaError_t e, const char* what) { return cuda_error(e, what); }

// Zeroed device allocation.  The memset is synchronous (legacy stream, then
// a device sync) so no later work on a non-blocking stream can overtake it.
template <class T>
static cudaError_t dalloc(T** p, size_t count) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T));
  if (e == cudaSuccess) e = cudaMemset(*p, 0, std::max<size_t>(count, 1) * sizeof(T));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e;
}

static cudaLaunchConfig_t lcfg(dim3 g, dim3 b, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr,
                               bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

// Split the rows of an [n][...] tensor for tensor parallelism.
//  attn_q / attn_k / attn_v: by KV head groups (whole heads per rank)
//  ffn_gate/up, output: contiguous row ranges
//  attn_output, ffn_down: every row (they are split by columns instead, see
//  col_range_cfg), norms and token_embd: every row
static bool col_split_role(const std::string& role) { return role == "attn_output" || role == "ffn_down"; }

static void shard_range_cfg(const b2q_model_config& c, const std::string& role, int64_t n, int64_t* b,
                            int64_t* e) {
  const int r = c.tp_rank, P = c.tp_size;
  if (P <= 1 || col_split_role(role)) {
    *b = 0;
    *e = n;
    return;
  }
  int64_t unit = 1;
  if (role == "attn_q" || role == "attn_k" || role == "attn_v" || role == "attn_q.bias" ||
      role == "attn_k.bias" || role == "attn_v.bias")
    unit = c.head_dim;
  const int64_t units = n / unit;
  const int64_t per = units / P;
  *b = per * r * unit;
  *e = per * (r + 1) * unit;
}

static void shard_range(const b2q_model* m, const std::string& role, int64_t n, int64_t* b, int64_t* e) {
  shard_range_cfg(m->c, role, n, b, e);
}

// Columns [b, e) of attn_output ([E][H*hd]: this rank's query heads) and
// ffn_down ([E][F]: this rank's SwiGLU rows) that the rank keeps: the K
// split that pairs with the head / row split of attention and gate/up, so
// that attention output and SwiGLU output never leave the GPU.
static void col_range_cfg(const b2q_model_config& c, const std::string& role, int64_t k, int64_t* b,
                          int64_t* e) {
  const int r = c.tp_rank, P = c.tp_size;
  if (P <= 1 || !col_split_role(role)) {
    *b = 0;
    *e = k;
    return;
  }
  const int64_t unit = role == "attn_output" ? c.head_dim : 1;
  const int64_t per = k / unit / P;
  *b = per * r * unit;
  *e = per * (r + 1) * unit;
}

static std::string role_of(const std::string& name, int* layer) {
  *layer = -1;
  std::string base = name;
  if (base.size() > 7 && base.compare(base.size() - 7, 7, ".weight") == 0)
    base = base.substr(0, base.size() - 7);
  if (base.compare(0, 4, "blk.") == 0) {
    const size_t dot = base.find('.', 4);
    if (dot == std::string::npos) return "";
    *layer = atoi(base.substr(4, dot - 4).c_str());
    return base.substr(dot + 1);
  }
  return base;
}

static b2q_status upload_f32(const void* host, size_t count, float** out) {
  cudaError_t e = dalloc(out, count);
  if (e == cudaSuccess) e = cudaMemcpy(*out, host, count * 4, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? B2Q_OK : cuda_error(e, "upload f32 tensor");
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

// One pass of `m` tokens (m <= mmax) whose ids are in M->tokens and whose
// start position is in M->pos.  Writes logits of the last token.
static cudaError_t forward_pass(b2q_model* M, int m, bool pdl, cudaStream_t st) {
  b2q_engine* e = M->eng;
  const b2q_model_config& c = M->c;
  const int E = c.n_embd, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads;
  const int Hl = M->H_loc, KVl = M->KV_loc, Fl = M->F_loc;
  const int G = H / KV;
  const int P = c.tp_size;
  cudaLaunchAttribute attr[1];
  cudaError_t err;

  // token embedding (raw GGUF rows, bit-exact dequant)
  {
    const int64_t slots = dequant_slots(M->tok_dtype, E);
    const int bx = (int)std::min<int64_t>((slots + 255) / 256, 64);
    cudaLaunchConfig_t cfg = lcfg(dim3(bx, m), dim3(256), 0, st, attr, pdl);
    launch_counted(e, 1);
    err = cudaLaunchKernelEx(&cfg, embed_rows_kernel, (const uint8_t*)M->tok_raw, M->tok_dtype,
                             M->tok_row_bytes, E, c.n_vocab, (const uint32_t*)M->tokens, M->x);
    if (err != cudaSuccess) return err;
  }
  const float scale = 1.0f / sqrtf((float)hd);
  const int width_loc = (Hl + 2 * KVl) * hd;
  // prompt passes of kTcMinTokens or more tokens run their projections on
  // the tensor cores (gemm_tc.cuh); shorter passes and single-token steps
  // stream the weights through the GEMV
  const bool tc = m >= kTcMinTokens;
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& Lw = M->L[l];
    // attention norm + quantise (on the tensor-core path the norm is fused
    // into the projection's activation images)
    if (!tc) {
      cudaLaunchConfig_t cfg = lcfg(dim3(m), dim3(1024), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, (const float*)M->x, E, 0,
                               (const float*)Lw.attn_norm, E, c.rms_eps, M->xq_e.x, (float*)nullptr);
      if (err != cudaSuccess) return err;
    }
    // q, k, v projections (one launch, outputs interleaved per token)
    if (tc) {
      const b2q_weight* ws[3] = {Lw.q, Lw.k, Lw.v};
      const int col0[3] = {0, (int)Lw.q->n, (int)(Lw.q->n + Lw.k->n)};
      err = tc_matmul(e, M->x, E, m, E, ws, 3, kEpiStore, M->qkv, width_loc, col0, st, pdl, Lw.attn_norm,
                      c.rms_eps);
      if (err != cudaSuccess) return err;
    } else {
      GemvSeg segs[3];
      memset(segs, 0, sizeof segs);
      b2q_weight* ws[3] = {Lw.q, Lw.k, Lw.v};
      int off = 0;
      for (int i = 0; i < 3; ++i) {
        segs[i].w = ws[i]->view;
        segs[i].w2 = ws[i]->view;
        segs[i].y = M->qkv + off;
        segs[i].ldy = width_loc;
        segs[i].rows_out = (int)ws[i]->n;
        off += (int)ws[i]->n;
      }
      err = run_gemv(e, segs, 3, M->xq_e, m, kEpiStore, st, pdl);
      if (err != cudaSuccess) return err;
    }
    // RoPE + KV append
    {
      cudaLaunchConfig_t cfg = lcfg(dim3(m), dim3(256), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg, rope_kv_kernel, M->qkv, m, Hl, KVl, hd,
                               (const float*)M->rope_cos, (const float*)M->rope_sin,
                               (const int*)M->pos, c.max_seq, Lw.kc, Lw.vc,
                               (const float*)Lw.q_bias, (const float*)Lw.k_bias,
                               (const float*)Lw.v_bias);
      if (err != cudaSuccess) return err;
    }
    // attention: prompt chunks on the tensor-core path take the 64-row
    // prompt kernel (its float output feeds the tensor-core O projection);
    // fewer tokens take the split + combine/quantise kernels of the decode
    // path (their quantised output feeds the GEMV)
    if (tc) {
      float* aout = P > 1 ? M->attn_loc : M->attn;
      const int qt = 64 / G;
      cudaLaunchConfig_t cfg = lcfg(dim3(KVl, (m + qt - 1) / qt), dim3(128), kAttnPrefillSmem, st, attr, pdl);
      launch_counted(e, 1);
      auto kern = G == 4 ? attn_prefill_kernel<4> : G == 8 ? attn_prefill_kernel<8>
                : G == 2 ? attn_prefill_kernel<2> : attn_prefill_kernel<1>;
      err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnPrefillSmem);
      if (err == cudaSuccess)
        err = cudaLaunchKernelEx(&cfg, kern, (const float*)M->qkv, m, Hl, KVl, (const int*)M->pos, c.max_seq,
                                 (const void*)Lw.tmk, (const void*)Lw.tmv, scale, aout);
      if (err != cudaSuccess) return err;
    } else {
      float* aout = P > 1 ? M->attn_loc : M->attn;
      const size_t tile = kAttnAlignPad + (G == 4 ? sizeof(AttnTile<4>) : G == 8 ? sizeof(AttnTile<8>)
                                           : G == 2 ? sizeof(AttnTile<2>) : sizeof(AttnTile<1>));
      cudaLaunchConfig_t cfg = lcfg(dim3(KVl, m, M->nsplit), dim3(kAttnThreads), tile, st, attr, pdl);
      launch_counted(e, 1);
      if (G == 4)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<4>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const void*)Lw.tmk,
                                 (const void*)Lw.tmv, scale, M->nsplit, M->part, e->num_sms);
      else if (G == 8)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<8>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const void*)Lw.tmk,
                                 (const void*)Lw.tmv, scale, M->nsplit, M->part, e->num_sms);
      else if (G == 2)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<2>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const void*)Lw.tmk,
                                 (const void*)Lw.tmv, scale, M->nsplit, M->part, e->num_sms);
      else
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<1>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const void*)Lw.tmk,
                                 (const void*)Lw.tmv, scale, M->nsplit, M->part, e->num_sms);
      if (err != cudaSuccess) return err;
      cudaLaunchConfig_t cfg2 = lcfg(dim3(KVl, m), dim3(G * kHeadDim), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg2, attn_combine_kernel, (const float*)M->part, m, Hl, G,
                               (const int*)M->pos, c.max_seq, M->nsplit, aout, M->xq_a.x, e->num_sms);
      if (err != cudaSuccess) return err;
      // under tensor parallelism the attention output of this rank's heads
      // stays local: attn_output holds the matching columns (K split)
    }
    // o-projection + residual (tensor parallelism: partial sums over this
    // rank's heads, added across ranks in rank order)
    if (tc) {
      const int col0 = 0;
      const b2q_weight* wo = Lw.o;
      err = P > 1 ? tc_matmul(e, M->attn_loc, Hl * hd, m, Hl * hd, &wo, 1, kEpiStore, M->y_loc, E, &col0, st, pdl)
                  : tc_matmul(e, M->attn, H * hd, m, H * hd, &wo, 1, kEpiAdd, M->x, E, &col0, st, pdl);
      if (err == cudaSuccess && P > 1) err = tp_allreduce_add(M->tp, M->y_loc, M->x, m, E, st);
      if (err != cudaSuccess) return err;
    } else {
      GemvSeg sg;
      memset(&sg, 0, sizeof sg);
      sg.w = Lw.o->view;
      sg.w2 = Lw.o->view;
      sg.rows_out = (int)Lw.o->n;
      if (P > 1) {
        sg.y = M->y_loc;
        sg.ldy = E;
        err = run_gemv(e, &sg, 1, M->xq_a, m, kEpiStore, st, pdl);
        if (err == cudaSuccess) err = tp_allreduce_add(M->tp, M->y_loc, M->x, m, E, st);
      } else {
        sg.y = M->x;
        sg.ldy = E;
        err = run_gemv(e, &sg, 1, M->xq_a, m, kEpiAdd, st, pdl);
      }
      if (err != cudaSuccess) return err;
    }
    // FFN norm + quantise (fused into the images on the tensor-core path)
    if (!tc) {
      cudaLaunchConfig_t cfg = lcfg(dim3(m), dim3(1024), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, (const float*)M->x, E, 0,
                               (const float*)Lw.ffn_norm, E, c.rms_eps, M->xq_e.x, (float*)nullptr);
      if (err != cudaSuccess) return err;
    }
    // gate/up with fused SwiGLU, per token
    {
      float* hout = P > 1 ? M->h_loc : M->hbuf;
      if (tc) {
        const b2q_weight* ws[2] = {Lw.gate, Lw.up};
        const int col0 = 0;
        err = tc_matmul(e, M->x, E, m, E, ws, 2, kEpiSwiglu, hout, Fl, &col0, st, pdl, Lw.ffn_norm, c.rms_eps);
        if (err != cudaSuccess) return err;
      }
      for (int t = 0; t < (tc ? 0 : m); ++t) {
        GemvArgs a;
        memset(&a, 0, sizeof a);
        a.nseg = 1;
        a.seg[0].w = Lw.gate->view;
        a.seg[0].w2 = Lw.up->view;
        a.seg[0].y = hout + (int64_t)t * Fl;
        a.seg[0].ldy = Fl;
        a.seg[0].rows_out = Fl;
        a.xq = M->xq_e.x.q;
        a.xscale = M->xq_e.x.scale;
        a.xs16 = M->xq_e.x.s16;
        a.kpad = M->xq_e.kpad;
        a.t0 = t;
        err = launch_gemv(e, a, kEpiSwiglu, 1, st, pdl);
        if (err != cudaSuccess) return err;
      }
      // under tensor parallelism the SwiGLU rows stay local: ffn_down holds the matching columns
      if (!tc) err = launch_quantize(e, hout, m, Fl, M->xq_f, st, pdl);
      if (err != cudaSuccess) return err;
    }
    // down projection + residual
    if (tc) {
      const int col0 = 0;
      const b2q_weight* wd = Lw.down;
      err = P > 1 ? tc_matmul(e, M->h_loc, Fl, m, Fl, &wd, 1, kEpiStore, M->y_loc, E, &col0, st, pdl)
                  : tc_matmul(e, M->hbuf, c.n_ff, m, c.n_ff, &wd, 1, kEpiAdd, M->x, E, &col0, st, pdl);
      if (err == cudaSuccess && P > 1) err = tp_allreduce_add(M->tp, M->y_loc, M->x, m, E, st);
      if (err != cudaSuccess) return err;
    } else {
      GemvSeg sg;
      memset(&sg, 0, sizeof sg);
      sg.w = Lw.down->view;
      sg.w2 = Lw.down->view;
      sg.rows_out = (int)Lw.down->n;
      if (P > 1) {
        sg.y = M->y_loc;
        sg.ldy = E;
        err = run_gemv(e, &sg, 1, M->xq_f, m, kEpiStore, st, pdl);
        if (err == cudaSuccess) err = tp_allreduce_add(M->tp, M->y_loc, M->x, m, E, st);
      } else {
        sg.y = M->x;
        sg.ldy = E;
        err = run_gemv(e, &sg, 1, M->xq_f, m, kEpiAdd, st, pdl);
      }
      if (err != cudaSuccess) return err;
    }
  }
  // final norm of the last token + output head
  {
    cudaLaunchConfig_t cfg = lcfg(dim3(1), dim3(1024), 0, st, attr, pdl);
    launch_counted(e, 1);
    err = cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, (const float*)M->x, E, m - 1,
                             (const float*)M->output_norm, E, c.rms_eps, M->xq_e.x, (float*)nullptr);
    if (err != cudaSuccess) return err;
    GemvSeg sg;
    memset(&sg, 0, sizeof sg);
    sg.w = M->output->view;
    sg.w2 = M->output->view;
    sg.rows_out = (int)M->output->n;
    sg.y = P > 1 ? M->logits_loc : M->logits;
    sg.ldy = (int)M->output->n;
    err = run_gemv(e, &sg, 1, M->xq_e, 1, kEpiStore, st, pdl);
    if (err != cudaSuccess) return err;
    if (P > 1) {
      err = tp_allgather_rows(M->tp, M->logits_loc, M->logits, 1, M->V_loc, st);
      if (err != cudaSuccess) return err;
    }
    cudaLaunchConfig_t cfg2 = lcfg(dim3(1), dim3(1024), 0, st, attr, pdl);
    launch_counted(e, 1);
    err = cudaLaunchKernelEx(&cfg2, argmax_kernel, (const float*)M->logits, c.n_vocab, M->argmax);
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

static cudaError_t build_decode_graph(b2q_model* M) {
  if (M->graph) {
    cudaGraphExecDestroy(M->graph);
    M->graph = nullptr;
  }
  const uint64_t before = M->eng->launches.load();
  cudaGraph_t g = nullptr;
  cudaError_t err = cudaStreamBeginCapture(M->st, cudaStreamCaptureModeRelaxed);
  if (err != cudaSuccess) return err;
  cudaError_t ferr = forward_pass(M, 1, /*pdl=*/true, M->st);
  err = cudaStreamEndCapture(M->st, &g);
  if (ferr != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return ferr;
  }
  if (err != cudaSuccess) return err;
  err = cudaGraphInstantiate(&M->graph, g, 0);
  cudaGraphDestroy(g);
  M->graph_kernels = M->eng->launches.load() - before;
  // capture does not launch anything
  M->eng->launches.fetch_sub(M->graph_kernels);
  return err;
}

// ---------------------------------------------------------------------------
// persistent decode kernel (decode.cuh): plan and launch
// ---------------------------------------------------------------------------

// One phase of the persistent kernel: the grid (one CTA per SM) is split
// over the phase's weights in proportion to their bytes, as launch_gemv_t
// splits its grid, but never beyond the grid.
constexpr int kDecStageMax = 56 * 1024;  // two tiles per stage when they fit

static void plan_dec_phase(DecPhase* ph, b2q_weight* const* ws, const b2q_weight* w2, int nw, const int* ycol,
                           bool pair, int grid, int* stage_max) {
  memset(ph, 0, sizeof *ph);
  ph->nseg = nw;
  ph->pair = pair ? 1 : 0;
  double bytes[kDecSegs], total = 0.0;
  for (int s = 0; s < nw; ++s) {
    const TileLayout& L = ws[s]->view.L;
    const int tb = (int)tile_bytes(L);
    DecSeg& sg = ph->seg[s];
    sg.w = ws[s]->view;
    sg.w2 = pair ? w2->view : ws[s]->view;
    sg.nr = (pair || 2 * tb <= kDecStageMax) ? 2 : 1;
    sg.ycol = ycol[s];
    *stage_max = std::max(*stage_max, tb * sg.nr);
    bytes[s] = (double)L.G * L.C * tb * (pair ? 2 : 1);
    total += bytes[s];
  }
  int n[kDecSegs], sum = 0;
  for (int s = 0; s < nw; ++s) {
    n[s] = (int)((double)grid * bytes[s] / total + 0.5);
    n[s] = std::max(1, std::min(n[s], ph->seg[s].w.L.G));
    sum += n[s];
  }
  while (sum > grid) {
    int big = 0;
    for (int s = 1; s < nw; ++s)
      if (n[s] > n[big]) big = s;
    if (n[big] <= 1) break;
    --n[big];
    --sum;
  }
  int cta = 0;
  for (int s = 0; s < nw; ++s) {
    ph->seg[s].cta0 = cta;
    ph->seg[s].ncta = n[s];
    cta += n[s];
  }
}

// The consumers' view of a phase for CTA b (cta_range in decode.cuh).
static CtaPhase cta_phase(const DecPhase& ph, int b) {
  CtaPhase r;
  memset(&r, 0, sizeof r);
  for (int s = 0; s < ph.nseg; ++s) {
    const DecSeg& sg = ph.seg[s];
    if (b < sg.cta0 || b >= sg.cta0 + sg.ncta) continue;
    const TileLayout& L = sg.w.L;
    const int ci = b - sg.cta0;
    r.gb = (int)((int64_t)L.G * ci / sg.ncta);
    r.ge = (int)((int64_t)L.G * (ci + 1) / sg.ncta);
    r.dtype_nr = L.dtype | ((ph.pair ? 2 : sg.nr) << 8);
    r.KC = L.KC;
    r.C = L.C;
    r.U = L.U;
    r.n = L.n;
    r.ycol = sg.ycol;
    break;
  }
  return r;
}

template <int G>
static void* decode_kernel_for(bool all) {
  return all ? reinterpret_cast<void*>(decode_kernel<G, true>) : reinterpret_cast<void*>(decode_kernel<G, false>);
}

// all: the model has Q5_K or Q4_0 weights (the kernel instance whose stage
// loop takes every supported type)
static void* decode_kernel_ptr(int G, bool all, size_t* attn_smem) {
  switch (G) {
    case 1: *attn_smem = sizeof(AttnTile<1>); return decode_kernel_for<1>(all);
    case 2: *attn_smem = sizeof(AttnTile<2>); return decode_kernel_for<2>(all);
    case 4: *attn_smem = sizeof(AttnTile<4>); return decode_kernel_for<4>(all);
    case 8: *attn_smem = sizeof(AttnTile<8>); return decode_kernel_for<8>(all);
    default: return nullptr;
  }
}

static size_t round128(size_t v) { return (v + 127) / 128 * 128; }

// One rank's block of the vectors every rank needs whole (DecodeArgs xg,
// attng, hg, logitsg, candg, xbarg): one allocation, so that one IPC handle
// maps it into the peers.
struct XBlock {
  size_t part, h, logits, cand, bar, total;
};
static XBlock xblock_layout(int E, int Hhd, int F, int V, int tp, int grid) {
  (void)Hhd;
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  XBlock b;
  size_t o = 0;
  b.part = o;  // [2][tp][E] tagged partial O / down sums from every rank (8 bytes each)
  o += al((size_t)2 * tp * E * 8);
  b.h = o;
  o += al((size_t)F * 4);
  b.logits = o;
  o += al((size_t)V * 4);
  b.cand = o;
  o += al((size_t)tp * grid * sizeof(int2));
  b.bar = o;  // kMaxTp 64-bit epoch slots, one per source rank
  o += 256;
  b.total = o;
  return b;
}

// Builds the persistent decode plan.  Leaves dec_on false (single-token
// steps then use the captured graph) when the model does not fit it: more
// ranks than kMaxTp, an unsupported head grouping, or too little shared
// memory for two pipeline stages.
static cudaError_t setup_decode(b2q_model* M) {
  const b2q_model_config& c = M->c;
  b2q_engine* e = M->eng;
  M->dec_on = false;
  // at most 64 KV heads per rank; ranks within the peer tables
  const int P = c.tp_size, rk = c.tp_rank;
  if (M->KV_loc > 64 || P > kMaxTp) return cudaSuccess;
  const int H = M->H_loc, KV = M->KV_loc, G = H / KV, hd = c.head_dim;
  // the persistent kernel's stage loop takes Q4_K, Q6_K and Q8_0 rows, and
  // in a second instance also Q5_K and Q4_0; models with other weight types
  // step through the captured graph
  bool all = false;
  {
    auto common = [](const b2q_weight* w) { return w->dtype == kQ4_K || w->dtype == kQ6_K || w->dtype == kQ8_0; };
    auto other = [](const b2q_weight* w) { return w->dtype == kQ5_K || w->dtype == kQ4_0; };
    std::vector<const b2q_weight*> ws{M->output};
    for (int l = 0; l < c.n_layers; ++l) {
      const LayerW& w = M->L[l];
      ws.insert(ws.end(), {w.q, w.k, w.v, w.o, w.gate, w.up, w.down});
    }
    for (const b2q_weight* w : ws) {
      if (other(w)) all = true;
      else if (!common(w)) return cudaSuccess;
    }
  }
  size_t attn_one = 0;
  void* kern = decode_kernel_ptr(G, all, &attn_one);
  if (!kern) return cudaSuccess;
  // the split merge stages {max, sum} of every split of a head group in one tile
  if (2 * G * M->nsplit > kAttnTile * kHeadDim / 2) return cudaSuccess;
  const int grid = e->num_sms;
  int stage_max = 0;
  std::vector<DecLayer> host((size_t)c.n_layers);
  std::vector<const DecPhase*> phases;
  const int y0[1] = {0};
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& w = M->L[l];
    DecLayer& d = host[(size_t)l];
    memset(&d, 0, sizeof d);
    b2q_weight* qkv[3] = {w.q, w.k, w.v};
    const int yc[3] = {0, H * hd, (H + KV) * hd};
    plan_dec_phase(&d.ph[kPhQKV], qkv, nullptr, 3, yc, false, grid, &stage_max);
    b2q_weight* o[1] = {w.o};
    plan_dec_phase(&d.ph[kPhO], o, nullptr, 1, y0, false, grid, &stage_max);
    b2q_weight* gt[1] = {w.gate};
    plan_dec_phase(&d.ph[kPhGU], gt, w.up, 1, y0, true, grid, &stage_max);
    b2q_weight* dn[1] = {w.down};
    plan_dec_phase(&d.ph[kPhDown], dn, nullptr, 1, y0, false, grid, &stage_max);
    d.attn_norm = w.attn_norm;
    d.ffn_norm = w.ffn_norm;
    d.qb = w.q_bias;
    d.kb = w.k_bias;
    d.vb = w.v_bias;
    d.kc = w.kc;
    d.vc = w.vc;
    d.tmk = w.tmk;
    d.tmv = w.tmv;
  }
  DecodeArgs& a = M->dec;
  memset(&a, 0, sizeof a);
  b2q_weight* hw[1] = {M->output};
  plan_dec_phase(&a.head, hw, nullptr, 1, y0, false, grid, &stage_max);
  for (auto& d : host)
    for (int p = 0; p < kDecPhases; ++p) phases.push_back(&d.ph[p]);
  phases.push_back(&a.head);
  const int nph = (int)phases.size();
  // per-CTA phase tables and the accumulator size
  std::vector<CtaPhase> tab((size_t)grid * nph);
  size_t racc = 128;
  for (int b = 0; b < grid; ++b)
    for (int p = 0; p < nph; ++p) {
      const CtaPhase r = cta_phase(*phases[(size_t)p], b);
      tab[(size_t)b * nph + p] = r;
      // accumulators [2][nw][rows]; O and down also keep their residual rows
      const bool add = p < 4 * c.n_layers && (p % 4 == kPhO || p % 4 == kPhDown);
      // (the residual rows are tagged 8-byte words; under tensor parallelism
      // every rank's partial of each row follows them)
      const size_t per_row = phases[(size_t)p]->pair ? 4 : add ? 4 + (size_t)P : 2;
      racc = std::max(racc, per_row * (r.ge - r.gb) * 8 * sizeof(float));
    }
  racc = round128(racc);
  // shared memory: [ring][staging][accumulators][phase table]; attention
  // tiles overlay staging + accumulators (idle during attention)
  const int kp_e = round_up_int(c.n_embd, 256);
  const int kpmax = std::max({kp_e, round_up_int(H * hd, 256), round_up_int(c.n_ff, 256)});
  const size_t tile = round128(attn_one);
  // staging: the largest quantised input; the RMSNorm copy of x behind the
  // quantised x; the float copy of the tagged attention output behind the
  // quantised attention output (one GPU)
  const int kp_a = round_up_int(H * hd, 256);
  size_t stage = std::max({xq_smem_bytes(kpmax), xq_smem_bytes(kp_e) + (size_t)4 * c.n_embd,
                           xq_smem_bytes(kp_a) + (size_t)4 * round_up_int(H * hd, 8)});
  if (stage + racc < tile) stage = tile - racc;
  stage = round128(stage);
  const size_t tabb = round128((size_t)nph * sizeof(CtaPhase));
  cudaFuncAttributes fa;
  cudaError_t err = cudaFuncGetAttributes(&fa, kern);
  if (err != cudaSuccess) return err;
  const size_t budget = (size_t)232448 - fa.sharedSizeBytes;
  if (stage + racc + tabb + 2 * (size_t)stage_max > budget) return cudaSuccess;
  const size_t cap = (budget - stage - racc - tabb) / 128 * 128;
  const size_t smem = cap + stage + racc + tabb;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) return cudaSuccess;
  err = dalloc(&M->dec_layers, host.size());
  if (err == cudaSuccess)
    err = cudaMemcpy(M->dec_layers, host.data(), host.size() * sizeof(DecLayer), cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = dalloc(&M->dec_tab, tab.size());
  if (err == cudaSuccess)
    err = cudaMemcpy(M->dec_tab, tab.data(), tab.size() * sizeof(CtaPhase), cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = dalloc(&M->dec_sync, 1);
  if (err == cudaSuccess) err = dalloc(&M->dec_attn_cnt, (size_t)c.n_layers * KV);
  // tagged vectors: x (rounded up to even: the residual copy reads pairs),
  // q|k|v and the attention output of this rank's heads, and (eight query
  // heads per KV head) the attention group partials of its heads, at most
  // max(1, grid / KV) groups per head
  const int ngmax = std::max(1, grid / KV);
  const size_t ll_x = (size_t)round_up_int(c.n_embd, 2), ll_qkv = (size_t)(H + 2 * KV) * hd, ll_attn = (size_t)H * hd;
  const size_t ll_part = G >= 8 ? (size_t)H * ngmax * kPartStride : 0;
  if (err == cudaSuccess) err = dalloc(&M->dec_ll, ll_x + ll_qkv + ll_attn + ll_part);
  M->dec_ll_words = ll_x + ll_qkv + ll_attn + ll_part;
  const XBlock xl = xblock_layout(c.n_embd, c.n_heads * hd, c.n_ff, c.n_vocab, P, grid);
  if (err == cudaSuccess) err = dalloc(reinterpret_cast<uint8_t**>(&M->dec_xblock), xl.total);
  if (err != cudaSuccess) return err;
  M->dec_peer[rk] = M->dec_xblock;
  if (P > 1) {
    // map every rank's block into this process: IPC handles gathered over NCCL
    cudaIpcMemHandle_t mine;
    err = cudaIpcGetMemHandle(&mine, M->dec_xblock);
    uint8_t* hb = nullptr;
    if (err == cudaSuccess) err = dalloc(&hb, sizeof(cudaIpcMemHandle_t) * (size_t)(P + 1));
    if (err == cudaSuccess) err = cudaMemcpy(hb, &mine, sizeof mine, cudaMemcpyHostToDevice);
    if (err == cudaSuccess) err = tp_allgather_bytes(M->tp, hb, hb + sizeof mine, sizeof mine, M->st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
    std::vector<cudaIpcMemHandle_t> all((size_t)P);
    if (err == cudaSuccess) err = cudaMemcpy(all.data(), hb + sizeof mine, sizeof mine * P, cudaMemcpyDeviceToHost);
    if (hb) cudaFree(hb);
    for (int p = 0; p < P && err == cudaSuccess; ++p)
      if (p != rk) err = cudaIpcOpenMemHandle(&M->dec_peer[p], all[(size_t)p], cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return err;
  }
  a.layers = M->dec_layers;
  a.ctab = M->dec_tab;
  a.nph = nph;
  a.n_layers = c.n_layers;
  a.E = c.n_embd;
  a.H = H;
  a.KV = KV;
  a.Hg = c.n_heads;
  a.F = c.n_ff;
  a.V = c.n_vocab;
  a.eps = c.rms_eps;
  a.scale = 1.0f / sqrtf((float)hd);
  a.max_seq = c.max_seq;
  a.out_norm = M->output_norm;
  a.tok_raw = static_cast<const uint8_t*>(M->tok_raw);
  a.tok_dtype = M->tok_dtype;
  a.tok_row_bytes = M->tok_row_bytes;
  a.rope_cos = M->rope_cos;
  a.rope_sin = M->rope_sin;
  a.part = M->part;
  a.nsplit = M->nsplit;
  a.sync = M->dec_sync;
  a.attn_cnt = M->dec_attn_cnt;
  a.xll = M->dec_ll;
  a.qkvll = M->dec_ll + ll_x;
  a.attnll = M->dec_ll + ll_x + ll_qkv;
  a.attnpll = M->dec_ll + ll_x + ll_qkv + ll_attn;
  a.attn_ngmax = ngmax;
  a.argmax = M->argmax;
  a.tp = P;
  a.rank = rk;
  a.Fl = M->F_loc;
  a.v_off = rk * M->V_loc;
  for (int p = 0; p < P; ++p) {
    uint8_t* base = static_cast<uint8_t*>(M->dec_peer[p]);
    a.partll[p] = reinterpret_cast<unsigned long long*>(base + xl.part);
    a.hg[p] = reinterpret_cast<float*>(base + xl.h);
    a.logitsg[p] = reinterpret_cast<float*>(base + xl.logits);
    a.candg[p] = reinterpret_cast<int2*>(base + xl.cand);
    a.xflagg[p] = reinterpret_cast<unsigned long long*>(base + xl.bar);
  }
  M->dec_logits = a.logitsg[rk];
  a.stage_bytes = (int)stage;
  a.racc_bytes = (int)racc;
  // where the kernel's dynamic shared memory starts (fixed per kernel: its
  // static shared memory comes first); the ring ends where the staging
  // region, and with it the attention tile buffers, start on a 1024-byte
  // boundary (the ring gives up less than 1 KB)
  {
    int* d_base = nullptr;
    err = cudaMalloc(&d_base, sizeof(int));
    if (err != cudaSuccess) return err;
    DecodeArgs q{};
    q.probe = d_base;
    void* qargs[] = {&q};
    err = cudaLaunchKernel(kern, dim3(1), dim3(kGemvThreads), qargs, smem, M->st);
    int base = 0;
    if (err == cudaSuccess) err = cudaMemcpyAsync(&base, d_base, sizeof(int), cudaMemcpyDeviceToHost, M->st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
    cudaFree(d_base);
    if (err != cudaSuccess) return err;
    a.cap = (int)(cap - (((size_t)base + cap) & 1023u));
  }
  // a second K/V tile buffer (long contexts: the tiles of an attention group
  // double-buffered) where the staging and accumulator regions already hold
  // it; never grown for it (the ring would shrink)
  a.attn_dbuf = stage + racc >= (size_t)kAttnTileBytes + attn_one ? 1 : 0;
#ifdef B2Q_DECODE_TRACE
  fprintf(stderr, "decode smem: ring %d stage %zu racc %zu table %zu attention tile %zu double buffer %d\n", a.cap,
          stage, racc, tabb, attn_one, a.attn_dbuf);
#endif
  M->dec_smem = smem;
  M->dec_G = G;
  M->dec_all = all;
  M->dec_on = true;
  return cudaSuccess;
}

// One single-token step: token id at `tok` (device), position `pos`.
// `tok`: the token id in device memory, or nullptr and the id `tok_imm` by
// value in the launch arguments (a host caller's token: no copy).
static cudaError_t launch_decode(b2q_model* M, const uint32_t* tok, uint32_t tok_imm, int pos, uint32_t* argmax2,
                                 cudaStream_t st) {
  DecodeArgs a = M->dec;
  a.token = tok;
  a.token_imm = tok_imm;
  a.pos = pos;
  a.argmax2 = argmax2;
  // every earlier launch passed 5L + 2 grid barriers (the last one the
  // first level of the head's all-rank barrier) and one all-rank epoch
  const unsigned long long seq = M->dec_launches++, grid = (unsigned long long)M->eng->num_sms;
  // tags of this launch: 5 per layer plus the head's input, counted from
  // the launch sequence, so the ranks of a tensor-parallel model agree on
  // them; re-arming clears every tagged word and restarts the sequence
  // (wrap-around is harmless: every launch rewrites every tagged element)
  a.tag0 = (uint32_t)(1ull + seq * (5ull * a.n_layers + 5ull));
  a.lbase = seq * (5ull * a.n_layers + 2ull) * grid;
  a.xepoch = seq;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M->eng->num_sms);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = M->dec_smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  launch_counted(M->eng, 1);
  if (M->dec_all) switch (M->dec_G) {
      case 1: return cudaLaunchKernelEx(&cfg, decode_kernel<1, true>, a);
      case 2: return cudaLaunchKernelEx(&cfg, decode_kernel<2, true>, a);
      case 4: return cudaLaunchKernelEx(&cfg, decode_kernel<4, true>, a);
      default: return cudaLaunchKernelEx(&cfg, decode_kernel<8, true>, a);
    }
  switch (M->dec_G) {
    case 1: return cudaLaunchKernelEx(&cfg, decode_kernel<1, false>, a);
    case 2: return cudaLaunchKernelEx(&cfg, decode_kernel<2, false>, a);
    case 4: return cudaLaunchKernelEx(&cfg, decode_kernel<4, false>, a);
    default: return cudaLaunchKernelEx(&cfg, decode_kernel<8, false>, a);
  }
}

}  // namespace b2q
