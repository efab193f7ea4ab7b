// tp.h -- tensor-parallel plumbing over NCCL for the per-kernel forward path.
//
// Sharding (model_impl.cuh): attn_q/k/v by whole KV-head groups, ffn_gate/up
// and the output head by rows, attn_output and ffn_down by the matching
// columns (the K split).  Attention output and SwiGLU output therefore stay on
// their rank; the two K-split projections produce partial sums of every row,
// which one NCCL all-gather per projection brings to every rank, where they
// are added to the residual in rank order (tp_allreduce_add), so all ranks
// hold bit-identical residuals.  The logits slices are all-gathered.  The
// persistent single-token kernel (decode.cuh) does not use NCCL on its data
// path: it stores its partial sums straight into the peers' memory; NCCL only
// exchanges its IPC handles at set-up.
//
// NCCL is resolved at run time with dlopen("libnccl.so.2"), so a process that
// already loaded NCCL (through torch.distributed) shares that copy and
// single-GPU use needs no NCCL.  Types and result codes come from the system
// nccl.h; the functions are looked up by name.  Communicators are created in
// non-blocking mode (ncclCommInitRankConfig, blocking = 0) and polled with a
// host-side timeout, so a rank that never joins ends the set-up with
// B2Q_ETIMEOUT after ncclCommAbort instead of hanging the process.
#pragma once

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "internal.h"

namespace b2q {

typedef ncclResult_t nccl_result_t;
typedef ncclComm_t nccl_comm_t;
typedef ncclUniqueId nccl_unique_id;

struct NcclApi {
  void* h = nullptr;
  nccl_result_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  nccl_result_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  nccl_result_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  nccl_result_t (*comm_abort)(ncclComm_t) = nullptr;
  nccl_result_t (*comm_finalize)(ncclComm_t) = nullptr;
  nccl_result_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  nccl_result_t (*comm_destroy)(ncclComm_t) = nullptr;
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
      api.comm_init_rank_config = (decltype(api.comm_init_rank_config))dlsym(api.h, "ncclCommInitRankConfig");
      api.get_async_error = (decltype(api.get_async_error))dlsym(api.h, "ncclCommGetAsyncError");
      api.comm_abort = (decltype(api.comm_abort))dlsym(api.h, "ncclCommAbort");
      api.comm_finalize = (decltype(api.comm_finalize))dlsym(api.h, "ncclCommFinalize");
      api.all_gather = (decltype(api.all_gather))dlsym(api.h, "ncclAllGather");
      api.comm_destroy = (decltype(api.comm_destroy))dlsym(api.h, "ncclCommDestroy");
      api.error_string = (decltype(api.error_string))dlsym(api.h, "ncclGetErrorString");
      if (!api.get_unique_id || !api.comm_init_rank_config || !api.get_async_error || !api.comm_abort ||
          !api.all_gather || !api.comm_destroy) {
        dlclose(api.h);
        api.h = nullptr;
      }
    }
  }
  return api;
}

// Host-side bound of the communicator set-up and of any NCCL call that
// reports ncclInProgress (b2q_set_tp_init_timeout_ms; default 120 s).
inline int& tp_timeout_ms() {
  static int ms = 120000;
  return ms;
}

inline const char* nccl_str(nccl_result_t r) {
  NcclApi& a = nccl();
  return a.error_string ? a.error_string(r) : "?";
}

// Poll a non-blocking communicator until its pending operation completes:
// ncclSuccess, an error, or ncclInProgress if the timeout ran out.
inline nccl_result_t nccl_wait(ncclComm_t comm) {
  NcclApi& a = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    nccl_result_t r = a.get_async_error(comm, &st);
    if (r != ncclSuccess) return r;
    if (st != ncclInProgress) return st;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > tp_timeout_ms()) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// A collective's return code: a non-blocking communicator may answer
// ncclInProgress while it sets up connections; wait for that to finish.
inline nccl_result_t nccl_done(ncclComm_t comm, nccl_result_t r) {
  return r == ncclInProgress ? nccl_wait(comm) : r;
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
  ncclUniqueId id;
  nccl_result_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) return set_error(B2Q_ENCCL, "ncclGetUniqueId: %s", nccl_str(r));
  memcpy(out, id.internal, 128);
  return B2Q_OK;
}

inline void tp_destroy(TpComm& t) {
  if (t.comm) {
    // (NCCL is loaded only when a communicator exists: a one-GPU model must
    // not pull libnccl into the process, whose copy would then shadow the
    // one a later import of torch brings)
    NcclApi& a = nccl();
    // non-blocking communicator: finalize (flushes pending work), wait, destroy
    if (a.comm_finalize && nccl_done(t.comm, a.comm_finalize(t.comm)) == ncclSuccess)
      a.comm_destroy(t.comm);
    else
      a.comm_abort(t.comm);
  }
  t.comm = nullptr;
  if (t.stage) cudaFree(t.stage);
  t.stage = nullptr;
}

// Create this rank's communicator (every rank calls it with the same id).
// Non-blocking: the set-up is polled for at most tp_timeout_ms(); a rank
// that never joins makes it end with B2Q_ETIMEOUT after ncclCommAbort.
inline b2q_status tp_init(TpComm& t, const unsigned char* id, int rank, int size, size_t stage_floats) {
  t.rank = rank;
  t.size = size;
  if (size <= 1) return B2Q_OK;
  NcclApi& a = nccl();
  if (!a.h) return set_error(B2Q_ENCCL, "libnccl.so.2 could not be loaded");
  if (!id) return set_error(B2Q_EINVAL, "tensor parallelism needs the NCCL unique id");
  ncclUniqueId uid;
  memcpy(uid.internal, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  nccl_result_t r = a.comm_init_rank_config(&comm, size, uid, rank, &cfg);
  if (r == ncclInProgress || (r == ncclSuccess && comm)) r = nccl_wait(comm);
  if (r != ncclSuccess) {
    if (comm) a.comm_abort(comm);
    if (r == ncclInProgress)
      return set_error(B2Q_ETIMEOUT, "ncclCommInitRankConfig: rank %d of %d: the other ranks did not join within %d ms",
                       rank, size, tp_timeout_ms());
    return set_error(B2Q_ENCCL, "ncclCommInitRankConfig: %s", nccl_str(r));
  }
  t.comm = comm;
  cudaError_t e = cudaMalloc(&t.stage, stage_floats * sizeof(float));
  if (e != cudaSuccess) return cuda_error(e, "tp staging buffer");
  t.stage_cap = stage_floats;
  return B2Q_OK;
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
  nccl_result_t r = nccl_done(t.comm, a.all_gather(loc, dst, cnt, ncclFloat32, t.comm, st));
  if (r != ncclSuccess) return cudaErrorUnknown;
  if (dst == full) return cudaSuccess;
  const int64_t total = (int64_t)cnt * t.size;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
  tp_scatter_rows_kernel<<<blocks, 256, 0, st>>>(t.stage, full, t.size, m, n_loc, add);
  return cudaGetLastError();
}

// Every rank's `bytes` bytes at send (device) -> recv [P][bytes] (device).
inline cudaError_t tp_allgather_bytes(TpComm& t, const void* send, void* recv, size_t bytes, cudaStream_t st) {
  nccl_result_t r = nccl_done(t.comm, nccl().all_gather(send, recv, bytes, ncclUint8, t.comm, st));
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
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
  nccl_result_t r = nccl_done(t.comm, nccl().all_gather(part, t.stage, cnt, ncclFloat32, t.comm, st));
  if (r != ncclSuccess) return cudaErrorUnknown;
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
