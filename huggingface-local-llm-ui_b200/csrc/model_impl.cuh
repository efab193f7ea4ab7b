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

#include "internal.h"
#include "tp.h"

namespace b2q {

struct LayerW {
  b2q_weight *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  b2q_weight *gate = nullptr, *up = nullptr, *down = nullptr;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
  float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
  __half *kc = nullptr, *vc = nullptr;
};

constexpr int kPrefillChunk = 64;  // tokens per forward pass of a long prompt

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
  uint32_t* tokens = nullptr;
  uint32_t* argmax = nullptr;
  int* pos = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  b2q::XQBuf xq_e, xq_a, xq_f;
  int nsplit = 0;
  int mmax = b2q::kPrefillChunk;
  // host staging (pinned) for b2q_forward's token ids
  uint32_t* h_tok = nullptr;
  // decode graph (m = 1)
  cudaGraphExec_t graph = nullptr;
  uint64_t graph_kernels = 0;
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
//  attn_output, ffn_gate/up/down, output: contiguous row ranges
static void shard_range(const b2q_model* m, const std::string& role, int64_t n, int64_t* b,
                        int64_t* e) {
  const int r = m->c.tp_rank, P = m->c.tp_size;
  if (P <= 1) {
    *b = 0;
    *e = n;
    return;
  }
  int64_t unit = 1;
  if (role == "attn_q" || role == "attn_k" || role == "attn_v" || role == "attn_q.bias" ||
      role == "attn_k.bias" || role == "attn_v.bias")
    unit = m->c.head_dim;
  const int64_t units = n / unit;
  const int64_t per = units / P;
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
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& Lw = M->L[l];
    // attention norm + quantise
    {
      cudaLaunchConfig_t cfg = lcfg(dim3(m), dim3(1024), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, (const float*)M->x, E, 0,
                               (const float*)Lw.attn_norm, E, c.rms_eps, M->xq_e.x, (float*)nullptr);
      if (err != cudaSuccess) return err;
    }
    // q, k, v projections (one launch, outputs interleaved per token)
    {
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
    // attention (split over the cached tokens) + combine/quantise
    {
      float* aout = P > 1 ? M->attn_loc : M->attn;
      cudaLaunchConfig_t cfg = lcfg(dim3(KVl, m, M->nsplit), dim3(128), 0, st, attr, pdl);
      launch_counted(e, 1);
      if (G == 4)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<4>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const __half*)Lw.kc,
                                 (const __half*)Lw.vc, scale, M->nsplit, M->part);
      else if (G == 8)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<8>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const __half*)Lw.kc,
                                 (const __half*)Lw.vc, scale, M->nsplit, M->part);
      else if (G == 2)
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<2>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const __half*)Lw.kc,
                                 (const __half*)Lw.vc, scale, M->nsplit, M->part);
      else
        err = cudaLaunchKernelEx(&cfg, attn_split_kernel<1>, (const float*)M->qkv, m, Hl, KVl,
                                 (const int*)M->pos, c.max_seq, (const __half*)Lw.kc,
                                 (const __half*)Lw.vc, scale, M->nsplit, M->part);
      if (err != cudaSuccess) return err;
      cudaLaunchConfig_t cfg2 = lcfg(dim3(KVl, m), dim3(G * kHeadDim), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg2, attn_combine_kernel, (const float*)M->part, m, Hl, G,
                               (const int*)M->pos, c.max_seq, M->nsplit, aout, M->xq_a.x);
      if (err != cudaSuccess) return err;
      if (P > 1) {
        err = tp_allgather_rows(M->tp, M->attn_loc, M->attn, m, Hl * hd, st);
        if (err != cudaSuccess) return err;
        err = launch_quantize(e, M->attn, m, H * hd, M->xq_a, st, pdl);
        if (err != cudaSuccess) return err;
      }
    }
    // o-projection + residual
    {
      GemvSeg sg;
      memset(&sg, 0, sizeof sg);
      sg.w = Lw.o->view;
      sg.w2 = Lw.o->view;
      sg.rows_out = (int)Lw.o->n;
      if (P > 1) {
        sg.y = M->y_loc;
        sg.ldy = (int)Lw.o->n;
        err = run_gemv(e, &sg, 1, M->xq_a, m, kEpiStore, st, pdl);
        if (err == cudaSuccess) err = tp_allgather_add_rows(M->tp, M->y_loc, M->x, m, (int)Lw.o->n, E, st);
      } else {
        sg.y = M->x;
        sg.ldy = E;
        err = run_gemv(e, &sg, 1, M->xq_a, m, kEpiAdd, st, pdl);
      }
      if (err != cudaSuccess) return err;
    }
    // FFN norm + quantise
    {
      cudaLaunchConfig_t cfg = lcfg(dim3(m), dim3(1024), 0, st, attr, pdl);
      launch_counted(e, 1);
      err = cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, (const float*)M->x, E, 0,
                               (const float*)Lw.ffn_norm, E, c.rms_eps, M->xq_e.x, (float*)nullptr);
      if (err != cudaSuccess) return err;
    }
    // gate/up with fused SwiGLU, per token
    {
      float* hout = P > 1 ? M->h_loc : M->hbuf;
      for (int t = 0; t < m; ++t) {
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
      if (P > 1) {
        err = tp_allgather_rows(M->tp, M->h_loc, M->hbuf, m, Fl, st);
        if (err != cudaSuccess) return err;
      }
      err = launch_quantize(e, M->hbuf, m, c.n_ff, M->xq_f, st, pdl);
      if (err != cudaSuccess) return err;
    }
    // down projection + residual
    {
      GemvSeg sg;
      memset(&sg, 0, sizeof sg);
      sg.w = Lw.down->view;
      sg.w2 = Lw.down->view;
      sg.rows_out = (int)Lw.down->n;
      if (P > 1) {
        sg.y = M->y_loc;
        sg.ldy = (int)Lw.down->n;
        err = run_gemv(e, &sg, 1, M->xq_f, m, kEpiStore, st, pdl);
        if (err == cudaSuccess)
          err = tp_allgather_add_rows(M->tp, M->y_loc, M->x, m, (int)Lw.down->n, E, st);
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

}  // namespace b2q
