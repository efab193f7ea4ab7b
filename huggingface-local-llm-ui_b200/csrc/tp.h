// tp.h -- tensor-parallel plumbing: NCCL all-gathers of row-sharded outputs.
//
// Every weight [n][k] is split by output rows over the ranks; each rank
// computes its contiguous slice of y and an all-gather rebuilds the full
// vector that the next operation consumes (attention output, o-proj output,
// SwiGLU output, down output, logits).  NCCL is resolved at run time with
// dlopen("libnccl.so.2"), so a process that already loaded NCCL (through
// torch.distributed) shares that copy and single-GPU use needs no NCCL.
#pragma once

#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstring>

#include "internal.h"

namespace b2q {

typedef int nccl_result_t;
typedef void* nccl_comm_t;
struct nccl_unique_id { char internal[128]; };
constexpr int kNcclUint8 = 1;
constexpr int kNcclFloat32 = 7;

struct NcclApi {
  void* h = nullptr;
  nccl_result_t (*get_unique_id)(nccl_unique_id*) = nullptr;
  nccl_result_t (*comm_init_rank)(nccl_comm_t*, int, nccl_unique_id, int) = nullptr;
  nccl_result_t (*all_gather)(const void*, void*, size_t, int, nccl_comm_t, cudaStream_t) = nullptr;
  nccl_result_t (*comm_destroy)(nccl_comm_t) = nullptr;
  const char* (*error_string)(nccl_result_t) = nullptr;
};

inline NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    api.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (api.h) {
      api.get_unique_id = (decltype(api.get_unique_id))dlsym(api.h, "ncclGetUniqueId");
      api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(api.h, "ncclCommInitRank");
      api.all_gather = (decltype(api.all_gather))dlsym(api.h, "ncclAllGather");
      api.comm_destroy = (decltype(api.comm_destroy))dlsym(api.h, "ncclCommDestroy");
      api.error_string = (decltype(api.error_string))dlsym(api.h, "ncclGetErrorString");
      if (!api.get_unique_id || !api.comm_init_rank || !api.all_gather || !api.comm_destroy) {
        dlclose(api.h);
        api.h = nullptr;
      }
    }
  }
  return api;
}

struct TpComm {
  nccl_comm_t comm = nullptr;
  int rank = 0, size = 1;
  float* stage = nullptr;  // [P][m][n_loc] gather staging
  size_t stage_cap = 0;
};

inline b2q_status tp_unique_id(unsigned char out[128]) {
  NcclApi& a = nccl();
  if (!a.h) return set_error(B2Q_ENCCL, "libnccl.so.2 could not be loaded");
  nccl_unique_id id;
  nccl_result_t r = a.get_unique_id(&id);
  if (r != 0) return set_error(B2Q_ENCCL, "ncclGetUniqueId: %s", a.error_string ? a.error_string(r) : "?");
  memcpy(out, id.internal, 128);
  return B2Q_OK;
}

inline b2q_status tp_init(TpComm& t, const unsigned char* id, int rank, int size, size_t stage_floats) {
  t.rank = rank;
  t.size = size;
  if (size <= 1) return B2Q_OK;
  NcclApi& a = nccl();
  if (!a.h) return set_error(B2Q_ENCCL, "libnccl.so.2 could not be loaded");
  if (!id) return set_error(B2Q_EINVAL, "tensor parallelism needs the NCCL unique id");
  nccl_unique_id uid;
  memcpy(uid.internal, id, 128);
  nccl_result_t r = a.comm_init_rank(&t.comm, size, uid, rank);
  if (r != 0) return set_error(B2Q_ENCCL, "ncclCommInitRank: %s", a.error_string ? a.error_string(r) : "?");
  cudaError_t e = cudaMalloc(&t.stage, stage_floats * sizeof(float));
  if (e != cudaSuccess) return cuda_error(e, "tp staging buffer");
  t.stage_cap = stage_floats;
  return B2Q_OK;
}

inline void tp_destroy(TpComm& t) {
  if (t.comm) nccl().comm_destroy(t.comm);
  t.comm = nullptr;
  if (t.stage) cudaFree(t.stage);
  t.stage = nullptr;
}

// [P][m][n_loc] -> [m][P*n_loc] (add = 1: accumulate into dst)
__global__ void tp_scatter_rows_kernel(const float* __restrict__ stage, float* __restrict__ dst,
                                       int P, int m, int n_loc, int add) {
  pdl_wait();
  const int64_t total = (int64_t)P * m * n_loc;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / ((int64_t)m * n_loc));
    const int64_t r = i % ((int64_t)m * n_loc);
    const int t = (int)(r / n_loc), c = (int)(r % n_loc);
    float* d = dst + (int64_t)t * P * n_loc + (int64_t)p * n_loc + c;
    if (add) *d += stage[i];
    else *d = stage[i];
  }
  pdl_launch_dependents();
}

inline cudaError_t tp_gather_core(TpComm& t, const float* loc, float* full, int m, int n_loc, int add,
                                  cudaStream_t st) {
  NcclApi& a = nccl();
  const size_t cnt = (size_t)m * n_loc;
  if (cnt * t.size > t.stage_cap) return cudaErrorInvalidValue;
  float* dst = (m == 1 && !add) ? full : t.stage;
  nccl_result_t r = a.all_gather(loc, dst, cnt, kNcclFloat32, t.comm, st);
  if (r != 0) return cudaErrorUnknown;
  if (dst == full) return cudaSuccess;
  const int64_t total = (int64_t)cnt * t.size;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
  tp_scatter_rows_kernel<<<blocks, 256, 0, st>>>(t.stage, full, t.size, m, n_loc, add);
  return cudaGetLastError();
}

// Every rank's `bytes` bytes at send (device) -> recv [P][bytes] (device).
inline cudaError_t tp_allgather_bytes(TpComm& t, const void* send, void* recv, size_t bytes, cudaStream_t st) {
  nccl_result_t r = nccl().all_gather(send, recv, bytes, kNcclUint8, t.comm, st);
  return r == 0 ? cudaSuccess : cudaErrorUnknown;
}

inline cudaError_t tp_allgather_rows(TpComm& t, const float* loc, float* full, int m, int n_loc,
                                     cudaStream_t st) {
  return tp_gather_core(t, loc, full, m, n_loc, 0, st);
}

// x[t][i] += part_0[t][i] + part_1[t][i] + ... (rank order) for a K-split
// projection: every rank's partial sums [m][n] gathered to [P][m][n], then
// summed in the same order on every rank, so all ranks hold the same x.
__global__ void tp_sum_add_kernel(const float* __restrict__ stage, float* __restrict__ x, int P, int64_t cnt) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt; i += (int64_t)gridDim.x * blockDim.x) {
    float v = x[i];
    for (int p = 0; p < P; ++p) v += stage[(int64_t)p * cnt + i];
    x[i] = v;
  }
  pdl_launch_dependents();
}

inline cudaError_t tp_allreduce_add(TpComm& t, const float* part, float* x, int m, int n, cudaStream_t st) {
  const size_t cnt = (size_t)m * n;
  if (cnt * t.size > t.stage_cap) return cudaErrorInvalidValue;
  nccl_result_t r = nccl().all_gather(part, t.stage, cnt, kNcclFloat32, t.comm, st);
  if (r != 0) return cudaErrorUnknown;
  const int blocks = (int)std::min<int64_t>(((int64_t)cnt + 255) / 256, 1024);
  tp_sum_add_kernel<<<blocks, 256, 0, st>>>(t.stage, x, t.size, (int64_t)cnt);
  return cudaGetLastError();
}

inline cudaError_t tp_allgather_add_rows(TpComm& t, const float* loc, float* x, int m, int n_loc,
                                         int n_full, cudaStream_t st) {
  (void)n_full;
  return tp_gather_core(t, loc, x, m, n_loc, 1, st);
}

}  // namespace b2q
