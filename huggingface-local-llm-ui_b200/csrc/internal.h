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

namespace b2q {

struct XQBuf {
  void* mem = nullptr;
  XQ x{};
  int m = 0, k = 0, kpad = 0;
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
}  // namespace b2q
