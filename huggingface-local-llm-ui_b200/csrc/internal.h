// internal.h -- types shared by the translation units of libb2q.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/b2q.h"
#include "gemv.cuh"
#include "layer.cuh"
#include "decode.cuh"
#include "gemm_tc.cuh"
#include "sample.cuh"
#include "gdn.cuh"

namespace b2q {

struct XQBuf {
  void* mem = nullptr;
  XQ x{};
  int m = 0, k = 0, kpad = 0;
};

// Scratch of the tensor-core multi-token matmul (grown on demand).
struct TcScratch {
  __half* img = nullptr;   // f16 activation images
  float* inv = nullptr;    // per-token inverse scales
  float* part = nullptr;   // split-K partials (the weights of one launch side by side)
  size_t img_cap = 0, inv_cap = 0, part_cap = 0;  // bytes
};

b2q_status set_error(b2q_status st, const char* fmt, ...);
b2q_status cuda_error(cudaError_t e, const char* what);
int dtype_block(int t);
int dtype_size(int t);
bool gemv_supported(int dtype);
cudaError_t xq_alloc(XQBuf* b, int m, int k);
void xq_free(XQBuf* b);

}  // namespace b2q

struct b2q_engine {
  int device = 0;
  int num_sms = 148;
  int l2_bytes = 0;
  char name[256] = {0};
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::atomic<uint64_t> launches{0};
  // workspace of the host-pointer matvec entry points
  float* ws_x = nullptr;
  float* ws_y = nullptr;
  float* ws_h = nullptr;
  size_t ws_x_cap = 0, ws_y_cap = 0, ws_h_cap = 0;
  b2q::XQBuf ws_xq, ws_hq;
  b2q::TcScratch tc;
  float* ws_gdn = nullptr;          // [channels] Gated DeltaNet convolution output
  size_t ws_gdn_cap = 0;
  float* ws_sample = nullptr;       // [n] candidate weights of the sampler
  uint32_t* ws_sample_out = nullptr; // token, drew
  size_t ws_sample_cap = 0;
};

struct b2q_weight {
  b2q_engine* eng = nullptr;
  int dtype = 0;
  int64_t n = 0, k = 0;
  size_t gguf_bytes = 0;
  void* mem = nullptr;
  size_t mem_bytes = 0;
  b2q::WeightDev view{};
};

namespace b2q {
cudaError_t launch_counted(b2q_engine* e, uint64_t n);
cudaError_t launch_gemv(b2q_engine* e, GemvArgs& a, int epi, int mt, cudaStream_t st, bool pdl);
cudaError_t run_gemv(b2q_engine* e, const GemvSeg* segs, int nseg, const XQBuf& xq, int m, int epi,
                     cudaStream_t st, bool pdl);
cudaError_t launch_quantize(b2q_engine* e, const float* x, int m, int k, XQBuf& xq, cudaStream_t st,
                            bool pdl);
// Multi-token matmul on the tensor cores (gemm_tc.cuh): for weight i of
// `ws`, y[t][col0[i] + r] = (X W_i^T)[t][r] (epi kEpiStore / kEpiAdd), or
// with ws = {gate, up} and epi kEpiSwiglu, y[t][col0[0] + r] =
// silu(g) * u.  x is [m][ldx] f32 on the device, m >= kTcMinTokens.  With
// norm_w, x is taken through RMSNorm (weights norm_w, epsilon eps) first,
// fused into the activation images.
cudaError_t tc_matmul(b2q_engine* e, const float* x, int ldx, int m, int k, const b2q_weight* const* ws,
                      int nw, int epi, float* y, int ldy, const int* col0, cudaStream_t st, bool pdl,
                      const float* norm_w = nullptr, float eps = 0.0f);
void tc_free(b2q_engine* e);
// Next token from logits_dev [n] (SelfMadeSampler::sample); *rng_state is
// advanced when the sampler draws.  Synchronous on `st`.
b2q_status sample_core(b2q_engine* e, const float* logits_dev, int n, float temperature, float top_p,
                       uint64_t* rng_state, uint32_t* token, cudaStream_t st);
}  // namespace b2q
