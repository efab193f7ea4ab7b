// model_api.cuh -- C ABI of the whole-model forward (b2q_model_*), included
// by b2q_api.cu after model_impl.cuh.
#pragma once

#include "model_impl.cuh"

using namespace b2q;

extern "C" {

b2q_status b2q_tp_unique_id(unsigned char out[128]) {
  if (!out) return set_error(B2Q_EINVAL, "b2q_tp_unique_id: out is NULL");
  return tp_unique_id(out);
}

b2q_status b2q_set_tp_init_timeout_ms(int ms) {
  if (ms <= 0) return set_error(B2Q_EINVAL, "b2q_set_tp_init_timeout_ms: %d ms", ms);
  tp_timeout_ms() = ms;
  return B2Q_OK;
}

b2q_status b2q_model_create(b2q_engine* e, const b2q_model_config* cfg, const unsigned char* tp_id,
                            b2q_model** out) {
  if (!e || !cfg || !out) return set_error(B2Q_EINVAL, "b2q_model_create: NULL argument");
  *out = nullptr;
  const b2q_model_config& c = *cfg;
  if (c.n_layers <= 0 || c.n_embd <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_ff <= 0 ||
      c.n_vocab <= 0 || c.max_seq <= 0)
    return set_error(B2Q_EINVAL, "b2q_model_create: all sizes must be positive");
  if (c.head_dim != kHeadDim)
    return set_error(B2Q_EUNSUP, "b2q_model_create: head_dim %d (only %d is built)", c.head_dim, kHeadDim);
  if (c.n_heads % c.n_kv_heads != 0)
    return set_error(B2Q_EINVAL, "b2q_model_create: n_heads %% n_kv_heads != 0");
  const int G = c.n_heads / c.n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(B2Q_EUNSUP, "b2q_model_create: GQA ratio %d not built (1, 2, 4, 8)", G);
  const int P = c.tp_size < 1 ? 1 : c.tp_size;
  if (c.tp_rank < 0 || c.tp_rank >= P) return set_error(B2Q_EINVAL, "b2q_model_create: bad tp_rank");
  if (c.n_kv_heads % P || c.n_embd % P || c.n_ff % P || c.n_vocab % P)
    return set_error(B2Q_EINVAL,
                     "b2q_model_create: tp_size %d must divide n_kv_heads, n_embd, n_ff and n_vocab", P);
  if (c.n_embd % 256 || c.n_ff % 256 || (c.n_heads * c.head_dim) % 256)
    return set_error(B2Q_EUNSUP, "b2q_model_create: n_embd, n_ff and n_heads*head_dim must be multiples of 256");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  b2q_model* M = new b2q_model();
  M->eng = e;
  M->c = c;
  M->c.tp_size = P;
  M->L.resize(c.n_layers);
  M->H_loc = c.n_heads / P;
  M->KV_loc = c.n_kv_heads / P;
  M->F_loc = c.n_ff / P;
  M->V_loc = c.n_vocab / P;
  cudaError_t err = cudaStreamCreateWithFlags(&M->st, cudaStreamNonBlocking);
  if (err != cudaSuccess) {
    delete M;
    return cuda_error(err, "model stream");
  }
  if (P > 1) {
    const size_t stage = (size_t)P * M->mmax * std::max({c.n_embd, c.n_ff, c.n_heads * c.head_dim}) +
                         (size_t)c.n_vocab;
    b2q_status s = tp_init(M->tp, tp_id, c.tp_rank, P, stage);
    if (s != B2Q_OK) {
      tp_destroy(M->tp);
      cudaStreamDestroy(M->st);
      delete M;
      return s;
    }
  }
  *out = M;
  return B2Q_OK;
}

b2q_status b2q_tp_shard_rows(const b2q_model_config* cfg, const char* name, int64_t n, int64_t* b, int64_t* e) {
  if (!cfg || !name || !b || !e) return set_error(B2Q_EINVAL, "b2q_tp_shard_rows: NULL argument");
  if (cfg->tp_size < 1 || cfg->tp_rank < 0 || cfg->tp_rank >= cfg->tp_size)
    return set_error(B2Q_EINVAL, "b2q_tp_shard_rows: tp_rank %d of tp_size %d", cfg->tp_rank, cfg->tp_size);
  int layer = -1;
  std::string role = role_of(name, &layer);
  if (role == "token_embd" || role == "output_norm" || role == "attn_norm" || role == "ffn_norm") {
    *b = 0;
    *e = n;
    return B2Q_OK;
  }
  shard_range_cfg(*cfg, role, n, b, e);
  return B2Q_OK;
}

b2q_status b2q_tp_shard_cols(const b2q_model_config* cfg, const char* name, int64_t k, int64_t* b, int64_t* e) {
  if (!cfg || !name || !b || !e) return set_error(B2Q_EINVAL, "b2q_tp_shard_cols: NULL argument");
  if (cfg->tp_size < 1 || cfg->tp_rank < 0 || cfg->tp_rank >= cfg->tp_size)
    return set_error(B2Q_EINVAL, "b2q_tp_shard_cols: tp_rank %d of tp_size %d", cfg->tp_rank, cfg->tp_size);
  int layer = -1;
  col_range_cfg(*cfg, role_of(name, &layer), k, b, e);
  return B2Q_OK;
}

b2q_status b2q_model_shard_rows(b2q_model* M, const char* name, int64_t n, int64_t* b, int64_t* e) {
  if (!M || !name || !b || !e) return set_error(B2Q_EINVAL, "b2q_model_shard_rows: NULL argument");
  return b2q_tp_shard_rows(&M->c, name, n, b, e);
}

static b2q_status set_tensor_impl(b2q_model* M, const char* name, int dtype, const int64_t* dims,
                                  int nd, int64_t rb, int64_t re, const void* bytes, size_t len) {
  if (!M || !name || !dims || nd < 1 || !bytes)
    return set_error(B2Q_EINVAL, "b2q_model_set_tensor: NULL argument");
  if (M->finalized) return set_error(B2Q_EINVAL, "b2q_model_set_tensor: model already finalized");
  int layer = -1;
  const std::string role = role_of(name, &layer);
  const b2q_model_config& c = M->c;
  if (layer >= c.n_layers) return set_error(B2Q_EINVAL, "tensor %s: layer out of range", name);
  const int64_t k = dims[nd - 1];
  const int64_t n = nd > 1 ? dims[0] : 1;
  for (int i = 1; i < nd - 1; ++i)
    if (dims[i] != 1) return set_error(B2Q_EUNSUP, "tensor %s: more than 2 non-trivial dims", name);
  const int bs = dtype_block(dtype), ts = dtype_size(dtype);
  if (bs == 0) return set_error(B2Q_EUNSUP, "tensor %s: GGML type %d not supported", name, dtype);
  if (k % bs) return set_error(B2Q_EINVAL, "tensor %s: inner dim %lld not a multiple of %d", name, (long long)k, bs);
  const int64_t row_bytes = k / bs * ts;
  if (rb < 0 || re > n || rb >= re) return set_error(B2Q_EINVAL, "tensor %s: bad row range", name);
  if ((int64_t)len != (re - rb) * row_bytes)
    return set_error(B2Q_EINVAL, "tensor %s: %zu bytes for %lld rows of %lld bytes", name, len,
                     (long long)(re - rb), (long long)row_bytes);
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  const uint8_t* src = static_cast<const uint8_t*>(bytes);

  // 1-D f32 tensors (norms, biases): dequantised on the host side by the
  // reference too (tensor_f32_1d, inference.rs:494-500); here only F32 is taken
  auto take_vec = [&](float** dst, int64_t want_b, int64_t want_e) -> b2q_status {
    if (dtype != kF32) return set_error(B2Q_EUNSUP, "tensor %s: 1-D tensors must be F32", name);
    if (rb > want_b || re < want_e) return set_error(B2Q_EINVAL, "tensor %s: shard rows missing", name);
    const float* f = reinterpret_cast<const float*>(src) + (want_b - rb) * k;
    M->have[name] = true;
    return upload_f32(f, (size_t)(want_e - want_b) * k, dst);
  };
  auto take_weight = [&](b2q_weight** dst) -> b2q_status {
    int64_t sb, se;
    shard_range(M, role, n, &sb, &se);
    if (rb > sb || re < se)
      return set_error(B2Q_EINVAL, "tensor %s: rows [%lld, %lld) of this rank were not supplied", name,
                       (long long)sb, (long long)se);
    if (!gemv_supported(dtype))
      return set_error(B2Q_EUNSUP, "tensor %s: GGML type %d has no GEMV kernel", name, dtype);
    int64_t cb, ce;
    col_range_cfg(c, role, k, &cb, &ce);
    b2q_status s;
    if (cb == 0 && ce == k) {
      M->eng->mu.unlock();
      s = b2q_upload_weight(M->eng, src + (sb - rb) * row_bytes, (size_t)((se - sb) * row_bytes), dtype, se - sb,
                            k, dst);
      M->eng->mu.lock();
    } else {
      // this rank's columns: whole blocks of every row, gathered on the host
      if (cb % bs || ce % bs || (ce - cb) % 64)
        return set_error(B2Q_EUNSUP, "tensor %s: column split [%lld, %lld) is not block aligned", name,
                         (long long)cb, (long long)ce);
      const int64_t lb = (ce - cb) / bs * ts, off = cb / bs * ts;
      std::vector<uint8_t> cols((size_t)((se - sb) * lb));
      for (int64_t r = sb; r < se; ++r)
        memcpy(cols.data() + (r - sb) * lb, src + (r - rb) * row_bytes + off, (size_t)lb);
      M->eng->mu.unlock();
      s = b2q_upload_weight(M->eng, cols.data(), cols.size(), dtype, se - sb, ce - cb, dst);
      M->eng->mu.lock();
    }
    if (s == B2Q_OK) {
      M->weight_bytes += (*dst)->gguf_bytes;
      M->have[name] = true;
    }
    return s;
  };

  if (role == "token_embd") {
    if (n != c.n_vocab || k != c.n_embd) return set_error(B2Q_EINVAL, "token_embd: wrong shape");
    if (rb != 0 || re != n) return set_error(B2Q_EINVAL, "token_embd: every rank needs all rows");
    cudaError_t err = cudaMalloc(&M->tok_raw, len);
    if (err == cudaSuccess) err = cudaMemcpy(M->tok_raw, src, len, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return cuda_error(err, "token_embd upload");
    M->tok_dtype = dtype;
    M->tok_row_bytes = row_bytes;
    M->weight_bytes += len;
    M->have[name] = true;
    // tied output head (inference.rs:2560-2562) unless output.weight comes
    if (!M->output && dtype_block(dtype) > 1 && gemv_supported(dtype)) {
      int64_t sb, se;
      shard_range(M, "output", n, &sb, &se);
      M->eng->mu.unlock();
      b2q_status s = b2q_upload_weight(M->eng, src + sb * row_bytes, (size_t)((se - sb) * row_bytes),
                                       dtype, se - sb, k, &M->output);
      M->eng->mu.lock();
      if (s != B2Q_OK) return s;
      M->have["output.tied"] = true;
    }
    return B2Q_OK;
  }
  if (role == "output") {
    if (n != c.n_vocab || k != c.n_embd) return set_error(B2Q_EINVAL, "output: wrong shape");
    if (M->output) {
      b2q_weight_free(M->output);
      M->output = nullptr;
    }
    M->have.erase("output.tied");
    return take_weight(&M->output);
  }
  if (role == "output_norm") return take_vec(&M->output_norm, 0, 1);
  if (layer < 0) return set_error(B2Q_EINVAL, "tensor %s: unknown name", name);
  LayerW& Lw = M->L[layer];
  const int hd = c.head_dim;
  if (role == "attn_norm") return take_vec(&Lw.attn_norm, 0, 1);
  if (role == "ffn_norm") return take_vec(&Lw.ffn_norm, 0, 1);
  if (role == "attn_q.bias" || role == "attn_k.bias" || role == "attn_v.bias") {
    // 1-D [n] biases: dims = [n]; shard by heads
    const int64_t nn = k;
    int64_t sb, se;
    shard_range(M, role, nn, &sb, &se);
    if (dtype != kF32) return set_error(B2Q_EUNSUP, "tensor %s: biases must be F32", name);
    float** dst = role == "attn_q.bias" ? &Lw.q_bias : role == "attn_k.bias" ? &Lw.k_bias : &Lw.v_bias;
    M->have[name] = true;
    return upload_f32(reinterpret_cast<const float*>(src) + sb, (size_t)(se - sb), dst);
  }
  struct { const char* r; b2q_weight** w; int64_t n, k; } tab[] = {
      {"attn_q", &Lw.q, (int64_t)c.n_heads * hd, c.n_embd},
      {"attn_k", &Lw.k, (int64_t)c.n_kv_heads * hd, c.n_embd},
      {"attn_v", &Lw.v, (int64_t)c.n_kv_heads * hd, c.n_embd},
      {"attn_output", &Lw.o, c.n_embd, (int64_t)c.n_heads * hd},
      {"ffn_gate", &Lw.gate, c.n_ff, c.n_embd},
      {"ffn_up", &Lw.up, c.n_ff, c.n_embd},
      {"ffn_down", &Lw.down, c.n_embd, c.n_ff},
  };
  for (auto& t : tab) {
    if (role == t.r) {
      if (n != t.n || k != t.k)
        return set_error(B2Q_EINVAL, "tensor %s: shape [%lld, %lld], expected [%lld, %lld]", name,
                         (long long)n, (long long)k, (long long)t.n, (long long)t.k);
      if (*t.w) {
        b2q_weight_free(*t.w);
        *t.w = nullptr;
      }
      return take_weight(t.w);
    }
  }
  return set_error(B2Q_EINVAL, "tensor %s: unknown name", name);
}

b2q_status b2q_model_set_tensor(b2q_model* M, const char* name, int dtype, const int64_t* dims, int nd,
                                const void* bytes, size_t len) {
  if (!dims || nd < 1) return set_error(B2Q_EINVAL, "b2q_model_set_tensor: no dims");
  const int64_t n = nd > 1 ? dims[0] : 1;
  return set_tensor_impl(M, name, dtype, dims, nd, 0, n, bytes, len);
}

b2q_status b2q_model_set_tensor_rows(b2q_model* M, const char* name, int dtype, const int64_t* dims,
                                     int nd, int64_t rb, int64_t re, const void* bytes, size_t len) {
  return set_tensor_impl(M, name, dtype, dims, nd, rb, re, bytes, len);
}

b2q_status b2q_model_finalize(b2q_model* M) {
  if (!M) return set_error(B2Q_EINVAL, "b2q_model_finalize: NULL model");
  if (M->finalized) return B2Q_OK;
  const b2q_model_config& c = M->c;
  if (!M->tok_raw) return set_error(B2Q_EINVAL, "missing tensor token_embd.weight");
  if (!M->output) return set_error(B2Q_EINVAL, "missing tensor output.weight");
  if (!M->output_norm) return set_error(B2Q_EINVAL, "missing tensor output_norm.weight");
  for (int l = 0; l < c.n_layers; ++l) {
    const LayerW& w = M->L[l];
    const char* miss = !w.attn_norm ? "attn_norm" : !w.ffn_norm ? "ffn_norm" : !w.q ? "attn_q"
                     : !w.k ? "attn_k" : !w.v ? "attn_v" : !w.o ? "attn_output" : !w.gate ? "ffn_gate"
                     : !w.up ? "ffn_up" : !w.down ? "ffn_down" : nullptr;
    if (miss) return set_error(B2Q_EINVAL, "missing tensor blk.%d.%s.weight", l, miss);
    if (w.gate->dtype != w.up->dtype)
      return set_error(B2Q_EUNSUP, "blk.%d: ffn_gate and ffn_up must share a GGML type", l);
  }
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  const int E = c.n_embd, hd = c.head_dim, H = c.n_heads;
  const int mm = M->mmax;
  M->nsplit = (c.max_seq + kAttnTile - 1) / kAttnTile;
  cudaError_t err = cudaSuccess;
  const size_t kv = (size_t)M->KV_loc * c.max_seq * hd;
  for (int l = 0; l < c.n_layers && err == cudaSuccess; ++l) {
    err = dalloc(&M->L[l].kc, kv);
    if (err == cudaSuccess) err = dalloc(&M->L[l].vc, kv);
  }
  if (err == cudaSuccess) {  // the caches' TMA descriptors
    std::vector<CUtensorMap> maps((size_t)2 * c.n_layers);
    for (int l = 0; l < c.n_layers; ++l)
      for (int kv2 = 0; kv2 < 2; ++kv2)
        if (!kv_tensor_map(&maps[(size_t)2 * l + kv2], kv2 ? M->L[l].vc : M->L[l].kc,
                           (uint64_t)M->KV_loc * c.max_seq))
          return set_error(B2Q_ECUDA, "cuTensorMapEncodeTiled failed for the KV cache of layer %d", l);
    err = dalloc(&M->kv_maps, maps.size());
    if (err == cudaSuccess)
      err = cudaMemcpy(M->kv_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    for (int l = 0; l < c.n_layers && err == cudaSuccess; ++l) {
      M->L[l].tmk = M->kv_maps + 2 * l;
      M->L[l].tmv = M->kv_maps + 2 * l + 1;
    }
  }
  if (err == cudaSuccess) err = dalloc(&M->x, (size_t)mm * E);
  if (err == cudaSuccess) err = dalloc(&M->qkv, (size_t)mm * (M->H_loc + 2 * M->KV_loc) * hd);
  if (err == cudaSuccess) err = dalloc(&M->attn, (size_t)mm * H * hd);
  if (err == cudaSuccess) err = dalloc(&M->attn_loc, (size_t)mm * M->H_loc * hd);
  if (err == cudaSuccess) err = dalloc(&M->hbuf, (size_t)mm * c.n_ff);
  if (err == cudaSuccess) err = dalloc(&M->h_loc, (size_t)mm * M->F_loc);
  if (err == cudaSuccess) err = dalloc(&M->y_loc, (size_t)mm * E);
  if (err == cudaSuccess) err = dalloc(&M->logits, (size_t)c.n_vocab);
  if (err == cudaSuccess) err = dalloc(&M->logits_loc, (size_t)M->V_loc);
  if (err == cudaSuccess) err = dalloc(&M->part, (size_t)mm * M->H_loc * M->nsplit * kPartStride);
  if (err == cudaSuccess) err = dalloc(&M->tokens, (size_t)2 * mm);  // ids + host staging
  if (err == cudaSuccess) err = dalloc(&M->argmax, 1);
  if (err == cudaSuccess) err = dalloc(&M->pos, 1);
  if (err == cudaSuccess) err = xq_alloc(&M->xq_e, mm, E);
  if (err == cudaSuccess) err = xq_alloc(&M->xq_a, mm, H * hd);
  if (err == cudaSuccess) err = xq_alloc(&M->xq_f, mm, c.n_ff);
  if (err == cudaSuccess) err = cudaMallocHost(&M->h_tok, sizeof(uint32_t) * mm);
  if (err == cudaSuccess) err = cudaMallocHost(&M->h_err, sizeof(int));
  if (err != cudaSuccess) return cuda_error(err, "b2q_model_finalize: allocation");
  // RoPE tables: freq = 1/theta^(2j/hd) in f32 powf, angle in f32, f32 cos/sin
  // (inference.rs:2538-2549), for positions 0..8191
  {
    const int half = hd / 2, NP = 8192;
    std::vector<float> cs((size_t)NP * half), sn((size_t)NP * half);
    for (int p = 0; p < NP; ++p)
      for (int j = 0; j < half; ++j) {
        const float freq = 1.0f / powf(c.rope_theta, (float)(2 * j) / (float)hd);
        const float angle = (float)p * freq;
        cs[(size_t)p * half + j] = cosf(angle);
        sn[(size_t)p * half + j] = sinf(angle);
      }
    b2q_status s = upload_f32(cs.data(), cs.size(), &M->rope_cos);
    if (s == B2Q_OK) s = upload_f32(sn.data(), sn.size(), &M->rope_sin);
    if (s != B2Q_OK) return s;
  }
  err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return cuda_error(err, "b2q_model_finalize: sync");
  if (c.no_graph == 0) {
    err = setup_decode(M);
    if (err != cudaSuccess) return cuda_error(err, "b2q_model_finalize: persistent decode set-up");
  }
  if ((c.no_graph == 0 && !M->dec_on) || c.no_graph == 2) {
    err = build_decode_graph(M);
    if (err != cudaSuccess) return cuda_error(err, "b2q_model_finalize: decode graph capture");
  }
  M->finalized = true;
  return B2Q_OK;
}

// `argmax_dev` (optional): a device word that a single-token step on the
// persistent kernel writes directly; *argmax_done tells the caller so.
static b2q_status forward_impl(b2q_model* M, const uint32_t* tokens, bool tok_on_dev, int n, int start,
                               cudaStream_t st, uint32_t* argmax_dev = nullptr, bool* argmax_done = nullptr) {
  if (argmax_done) *argmax_done = false;
  const b2q_model_config& c = M->c;
  if (n <= 0) return set_error(B2Q_EINVAL, "forward: no tokens");
  if (start < 0 || start + n > c.max_seq)
    return set_error(B2Q_EINVAL, "forward: positions [%d, %d) exceed the KV capacity %d", start,
                     start + n, c.max_seq);
  if (!tok_on_dev)
    for (int i = 0; i < n; ++i)
      if (tokens[i] >= (uint32_t)c.n_vocab)
        return set_error(B2Q_EINVAL, "forward: token id %u >= vocab %d", tokens[i], c.n_vocab);
  // Under stream capture a single-token step takes the per-kernel path: the
  // persistent kernel's barrier bases and hand-off tags are host counters
  // baked into each launch's arguments, so a replayed launch would reuse
  // them (stale tags would pass, barrier targets would not match).
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t err = cudaStreamIsCapturing(st, &cap);
  if (err != cudaSuccess) return cuda_error(err, "forward: cudaStreamIsCapturing");
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  for (int off = 0; off < n && err == cudaSuccess; off += M->mmax) {
    const int m = std::min(M->mmax, n - off);
    const uint32_t* src = tokens + off;
    if (m == 1 && M->dec_on && !capturing) {
      // one persistent kernel for the whole step (validates the id itself); a
      // host token goes by value in the launch arguments
      err = launch_decode(M, tok_on_dev ? src : nullptr, tok_on_dev ? 0u : tokens[off], start + off, argmax_dev, st);
      M->last_logits = M->dec_logits;
      if (err == cudaSuccess && argmax_done) *argmax_done = argmax_dev != nullptr;
      continue;
    }
    if (!tok_on_dev) {
      // host tokens: stage through the pinned buffer (synchronous callers only)
      memcpy(M->h_tok, tokens + off, sizeof(uint32_t) * m);
      err = cudaMemcpyAsync(M->tokens + M->mmax, M->h_tok, sizeof(uint32_t) * m, cudaMemcpyHostToDevice, st);
      if (err != cudaSuccess) break;
      src = M->tokens + M->mmax;
    }
    launch_counted(M->eng, 1);
    set_step_kernel<<<1, 64, 0, st>>>(M->pos, start + off, M->tokens, src, m, c.n_vocab);
    err = cudaGetLastError();
    if (err != cudaSuccess) break;
    if (m == 1 && M->graph && !capturing) {
      err = cudaGraphLaunch(M->graph, st);
      M->eng->launches.fetch_add(M->graph_kernels);
    } else {
      err = forward_pass(M, m, false, st);
    }
    M->last_logits = M->logits;
    // the pinned staging is reused by the next chunk: wait for its copy
    if (err == cudaSuccess && !tok_on_dev && off + m < n) err = cudaStreamSynchronize(st);
  }
  if (err != cudaSuccess) return cuda_error(err, "forward");
  return B2Q_OK;
}

b2q_status b2q_forward_dev(b2q_model* M, const uint32_t* tokens_dev, int n, int start, float* logits_dev,
                           uint32_t* argmax_dev, void* stream) {
  if (!M || !tokens_dev) return set_error(B2Q_EINVAL, "b2q_forward_dev: NULL argument");
  if (!M->finalized) return set_error(B2Q_EINVAL, "b2q_forward_dev: model not finalized");
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : M->st;
  bool argmax_done = false;
  b2q_status s = forward_impl(M, tokens_dev, true, n, start, st, argmax_dev, &argmax_done);
  if (s != B2Q_OK) return s;
  cudaError_t err = cudaSuccess;
  if (logits_dev)
    err = cudaMemcpyAsync(logits_dev, M->last_logits, sizeof(float) * M->c.n_vocab, cudaMemcpyDeviceToDevice, st);
  if (err == cudaSuccess && argmax_dev && !argmax_done)
    err = cudaMemcpyAsync(argmax_dev, M->argmax, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st);
  if (err != cudaSuccess) return cuda_error(err, "b2q_forward_dev: copy out");
  return B2Q_OK;
}

// Re-arm the persistent kernel's synchronisation state: the grid-barrier
// counter, the attention split counters, this rank's all-rank epoch slots and
// the host's launch sequence (the barrier bases and epochs of the next launch
// start from zero again).  A step whose bounded wait gave up leaves them
// inconsistent.  Caller holds the engine lock; synchronous on M->st.
static cudaError_t rearm_decode(b2q_model* M) {
  if (!M->dec_sync) return cudaSuccess;
  cudaError_t err = cudaMemsetAsync(M->dec_sync, 0, sizeof(b2q::DecSync), M->st);
  if (err == cudaSuccess)
    err = cudaMemsetAsync(M->dec_attn_cnt, 0, sizeof(unsigned int) * M->c.n_layers * M->KV_loc, M->st);
  const b2q::XBlock xl = b2q::xblock_layout(M->c.n_embd, M->c.n_heads * M->c.head_dim, M->c.n_ff,
                                            M->c.n_vocab, M->c.tp_size, M->eng->num_sms);
  if (err == cudaSuccess)
    err = cudaMemsetAsync(static_cast<uint8_t*>(M->dec_xblock) + xl.bar, 0, 8 * b2q::kMaxTp, M->st);
  // every tagged word back to tag 0 (never a live tag): the tags of the next
  // launches restart from the launch sequence, on every rank alike
  if (err == cudaSuccess) err = cudaMemsetAsync(M->dec_ll, 0, sizeof(unsigned long long) * M->dec_ll_words, M->st);
  if (err == cudaSuccess)
    err = cudaMemsetAsync(static_cast<uint8_t*>(M->dec_xblock) + xl.part, 0,
                          sizeof(unsigned long long) * 2 * (size_t)M->c.tp_size * M->c.n_embd, M->st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
  M->dec_launches = 0;
  return err;
}

// Queue the read-back of the device error word behind a blocking forward's
// work on M->st (into pinned M->h_err; no extra synchronisation).
static cudaError_t queue_error_readback(b2q_model* M) {
  return cudaMemcpyFromSymbolAsync(M->h_err, g_b2q_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, M->st);
}

// After M->st has been synchronised: a nonzero device error word means a
// bounded wait gave up during the step, so its outputs are not valid.  The
// word is cleared and B2Q_ETIMEOUT returned.  On one GPU the persistent
// kernel's synchronisation state is re-armed here, so the next step runs
// normally; under tensor parallelism every rank must call b2q_clear_state
// (together, followed by a host barrier across the ranks) before the next
// step, since a rank cannot re-arm its peers' epoch slots on its own.
static b2q_status forward_error_check(b2q_model* M, const char* what) {
  const int v = *M->h_err;
  if (v == 0) return B2Q_OK;
  *M->h_err = 0;
  const int zero = 0;
  cudaError_t err = cudaMemcpyToSymbolAsync(g_b2q_device_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, M->st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
  if (err == cudaSuccess && M->c.tp_size == 1) err = rearm_decode(M);
  if (err != cudaSuccess) return cuda_error(err, what);
  if (v == 3)
    return set_error(B2Q_ECUDA, "%s: the decode kernel's shared-memory layout differs from the planned one; the "
                     "step's outputs are invalid", what);
  return set_error(B2Q_ETIMEOUT, "%s: a device-side bounded wait gave up (code %d); the step's outputs are invalid%s",
                   what, v, M->c.tp_size > 1 ? "; every rank must call b2q_clear_state" : "");
}

b2q_status b2q_forward(b2q_model* M, const uint32_t* tokens, int n, int start, float* logits,
                       uint32_t* argmax) {
  if (!M || !tokens) return set_error(B2Q_EINVAL, "b2q_forward: NULL argument");
  if (!M->finalized) return set_error(B2Q_EINVAL, "b2q_forward: model not finalized");
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  b2q_status s = forward_impl(M, tokens, false, n, start, M->st);
  if (s != B2Q_OK) return s;
  cudaError_t err = cudaSuccess;
  if (logits)
    err = cudaMemcpyAsync(logits, M->last_logits, sizeof(float) * M->c.n_vocab, cudaMemcpyDeviceToHost, M->st);
  if (err == cudaSuccess && argmax)
    err = cudaMemcpyAsync(argmax, M->argmax, sizeof(uint32_t), cudaMemcpyDeviceToHost, M->st);
  if (err == cudaSuccess) err = queue_error_readback(M);
  if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
  if (err != cudaSuccess) return cuda_error(err, "b2q_forward");
  return forward_error_check(M, "b2q_forward");
}

b2q_status b2q_forward_sample(b2q_model* M, const uint32_t* tokens, int n, int start, float temperature,
                              float top_p, uint64_t* rng_state, uint32_t* token) {
  if (!M || !tokens || !rng_state || !token) return set_error(B2Q_EINVAL, "b2q_forward_sample: NULL argument");
  if (!M->finalized) return set_error(B2Q_EINVAL, "b2q_forward_sample: model not finalized");
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  b2q_status s = forward_impl(M, tokens, false, n, start, M->st);
  if (s != B2Q_OK) return s;
  cudaError_t err = queue_error_readback(M);
  if (err != cudaSuccess) return cuda_error(err, "b2q_forward_sample");
  // the sampler synchronises M->st, which also completes the read-back; a
  // step whose wait gave up reports that instead of its (invalid) token
  const uint64_t rng0 = *rng_state;
  s = sample_core(M->eng, M->last_logits, M->c.n_vocab, temperature, top_p, rng_state, token, M->st);
  if (s != B2Q_OK) return s;
  s = forward_error_check(M, "b2q_forward_sample");
  if (s != B2Q_OK) *rng_state = rng0;
  return s;
}

b2q_status b2q_model_fill_kv(b2q_model* M, int start, int n, uint64_t seed, float scale) {
  if (!M || !M->finalized) return set_error(B2Q_EINVAL, "b2q_model_fill_kv: model not finalized");
  if (start < 0 || n <= 0 || start + n > M->c.max_seq)
    return set_error(B2Q_EINVAL, "b2q_model_fill_kv: positions [%d, %d) outside the KV capacity %d", start,
                     start + n, M->c.max_seq);
  std::lock_guard<std::mutex> lk(M->eng->mu);
  cudaSetDevice(M->eng->device);
  const int head0 = M->c.tp_rank * M->KV_loc;
  cudaError_t err = cudaSuccess;
  for (int l = 0; l < M->c.n_layers && err == cudaSuccess; ++l) {
    launch_counted(M->eng, 1);
    kv_fill_kernel<<<dim3(n, M->KV_loc), kHeadDim, 0, M->st>>>(M->L[l].kc, M->L[l].vc, M->c.max_seq, start, l,
                                                               head0, seed, scale);
    err = cudaGetLastError();
  }
  if (err == cudaSuccess) err = cudaStreamSynchronize(M->st);
  if (err != cudaSuccess) return cuda_error(err, "b2q_model_fill_kv");
  return B2Q_OK;
}

b2q_status b2q_model_debug_desync(b2q_model* M) {
  if (!M || !M->finalized) return set_error(B2Q_EINVAL, "b2q_model_debug_desync: model not finalized");
  if (!M->dec_on) return set_error(B2Q_EUNSUP, "b2q_model_debug_desync: the model has no persistent decode step");
  std::lock_guard<std::mutex> lk(M->eng->mu);
  ++M->dec_launches;
  return B2Q_OK;
}

b2q_status b2q_clear_state(b2q_model* M) {
  // The KV cache is indexed by absolute position, so clearing only resets
  // what the caller considers the current position; entries past it are
  // never read (attention reads keys t < start + s + 1).
  if (!M) return set_error(B2Q_EINVAL, "b2q_clear_state: NULL model");
  if (M->dec_sync) {
    // (all ranks of a tensor-parallel model call it together)
    std::lock_guard<std::mutex> lk(M->eng->mu);
    cudaSetDevice(M->eng->device);
    cudaError_t err = rearm_decode(M);
    if (err != cudaSuccess) return cuda_error(err, "b2q_clear_state");
  }
  return B2Q_OK;
}

size_t b2q_model_weight_bytes(const b2q_model* M) { return M ? M->weight_bytes : 0; }

int b2q_model_step_path(const b2q_model* M) {
  if (!M || !M->finalized) return -1;
  return M->dec_on ? 0 : M->graph ? 2 : 1;
}

b2q_status b2q_model_destroy(b2q_model* M) {
  if (!M) return B2Q_OK;
  cudaSetDevice(M->eng->device);
  cudaStreamSynchronize(M->st);
  if (M->graph) cudaGraphExecDestroy(M->graph);
  tp_destroy(M->tp);
  for (auto& l : M->L) {
    b2q_weight* ws[7] = {l.q, l.k, l.v, l.o, l.gate, l.up, l.down};
    for (auto* w : ws) b2q_weight_free(w);
    float* fs[5] = {l.attn_norm, l.ffn_norm, l.q_bias, l.k_bias, l.v_bias};
    for (auto* f : fs)
      if (f) cudaFree(f);
    if (l.kc) cudaFree(l.kc);
    if (l.vc) cudaFree(l.vc);
  }
  b2q_weight_free(M->output);
  void* ps[] = {M->tok_raw, M->output_norm, M->x, M->qkv, M->attn, M->attn_loc, M->hbuf, M->h_loc,
                M->y_loc, M->logits, M->logits_loc, M->part, M->tokens, M->argmax, M->pos,
                M->rope_cos, M->rope_sin, M->dec_layers, M->dec_tab, M->dec_sync, M->dec_xblock,
                M->dec_attn_cnt, M->dec_ll, M->kv_maps};
  for (int p = 0; p < b2q::kMaxTp; ++p)
    if (M->dec_peer[p] && p != M->c.tp_rank) cudaIpcCloseMemHandle(M->dec_peer[p]);
  for (void* p : ps)
    if (p) cudaFree(p);
  xq_free(&M->xq_e);
  xq_free(&M->xq_a);
  xq_free(&M->xq_f);
  if (M->h_tok) cudaFreeHost(M->h_tok);
  if (M->h_err) cudaFreeHost(M->h_err);
  cudaStreamDestroy(M->st);
  delete M;
  return B2Q_OK;
}

}  // extern "C"
