// tc_host.cuh -- launch planning of the tensor-core multi-token matmul
// (gemm_tc.cuh), included by b2q_api.cu.
#pragma once

namespace b2q {

struct TcPlan {
  int N, tiles, mpad, KS, rowtiles, splits;
};

// Token tiles of at most 256 (balanced), k-stages of 64, and a split-K
// factor of one split per 16 stages (at most 8).  The split depends on k
// only, so every output element is summed in the same order whatever the
// number of rows (a tensor-parallel shard gives the same bits as the whole
// weight) or tokens.
static TcPlan tc_plan(int m, int64_t n, int64_t k, int num_sms) {
  (void)num_sms;
  TcPlan p;
  p.tiles = (m + kTcNMax - 1) / kTcNMax;
  p.N = round_up_int((m + p.tiles - 1) / p.tiles, 16);
  p.mpad = p.tiles * p.N;
  p.KS = (int)((k + kTcK - 1) / kTcK);
  p.rowtiles = (int)((n + kTcM - 1) / kTcM);
  p.splits = std::max(1, std::min(8, p.KS / 16));
  return p;
}

static cudaError_t tc_grow(void** p, size_t* cap, size_t bytes, cudaStream_t st) {
  if (*cap >= bytes) return cudaSuccess;
  cudaError_t err = cudaStreamSynchronize(st);  // the old buffer may be in use
  if (err != cudaSuccess) return err;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  bytes = align_up(bytes, (size_t)1 << 20);
  err = cudaMalloc(p, bytes);
  if (err == cudaSuccess) *cap = bytes;
  return err;
}

void tc_free(b2q_engine* e) {
  TcScratch& t = e->tc;
  if (t.img) cudaFree(t.img);
  if (t.inv) cudaFree(t.inv);
  if (t.part) cudaFree(t.part);
  if (t.part2) cudaFree(t.part2);
  t = TcScratch{};
}

static cudaError_t tc_launch_gemm(b2q_engine* e, const b2q_weight* w, const TcPlan& p, int m, float* part,
                                  cudaStream_t st, bool pdl) {
  if (p.N < 16 || p.N > kTcNMax || p.N % 16 != 0) return cudaErrorInvalidValue;
  TcArgs a;
  a.w = w->view;
  a.xh = e->tc.img;
  a.KS = p.KS;
  a.N = p.N;
  a.m = m;
  a.n = (int)w->n;
  a.splits = p.splits;
  a.part = part;
  a.mpad = p.mpad;
  a.stages = tc_stages(p.N);
  if (a.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)a.stages * tc_stage_bytes(p.N);
  cudaError_t err = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.rowtiles, p.tiles, p.splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  (void)pdl;  // the kernel reads the image from its first instruction: no early launch
  launch_counted(e, 1);
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, a);
}

template <int EPI>
static cudaError_t tc_launch_reduce(b2q_engine* e, const TcPlan& p, int m, int n, float* y, int ldy, int col0,
                                    cudaStream_t st) {
  const int64_t total = (int64_t)m * n;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)e->num_sms * 8);
  launch_counted(e, 1);
  tc_reduce_kernel<EPI><<<blocks, 256, 0, st>>>(e->tc.part, e->tc.part2, p.splits, p.mpad, m, n, e->tc.inv, y,
                                                ldy, col0);
  return cudaGetLastError();
}

cudaError_t tc_matmul(b2q_engine* e, const float* x, int ldx, int m, int k, const b2q_weight* const* ws, int nw,
                      int epi, float* y, int ldy, const int* col0, cudaStream_t st, bool pdl) {
  if (m < 1 || nw < 1 || (epi == kEpiSwiglu && nw != 2)) return cudaErrorInvalidValue;
  for (int i = 0; i < nw; ++i)
    if (ws[i]->k != k || !gemv_supported(ws[i]->dtype))
      return cudaErrorInvalidValue;
  TcScratch& t = e->tc;
  // scratch: image and scales for these tokens, partials for the largest weight
  const TcPlan p0 = tc_plan(m, ws[0]->n, k, e->num_sms);
  size_t part_need = 0;
  for (int i = 0; i < nw; ++i) {
    const TcPlan p = tc_plan(m, ws[i]->n, k, e->num_sms);
    part_need = std::max(part_need, (size_t)p.splits * p.mpad * ws[i]->n * sizeof(float));
  }
  cudaError_t err = tc_grow(reinterpret_cast<void**>(&t.img), &t.img_cap,
                            (size_t)p0.tiles * p0.KS * tc_b_bytes(p0.N), st);
  if (err == cudaSuccess) err = tc_grow(reinterpret_cast<void**>(&t.inv), &t.inv_cap, (size_t)p0.mpad * 4, st);
  if (err == cudaSuccess) err = tc_grow(reinterpret_cast<void**>(&t.part), &t.part_cap, part_need, st);
  if (err == cudaSuccess && epi == kEpiSwiglu)
    err = tc_grow(reinterpret_cast<void**>(&t.part2), &t.part2_cap, part_need, st);
  if (err != cudaSuccess) return err;
  {
    launch_counted(e, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p0.mpad);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    err = cudaLaunchKernelEx(&cfg, tc_act_kernel, x, ldx, m, k, p0.KS, p0.N, t.img, t.inv);
    if (err != cudaSuccess) return err;
  }
  if (epi == kEpiSwiglu) {
    const TcPlan p = tc_plan(m, ws[0]->n, k, e->num_sms);
    err = tc_launch_gemm(e, ws[0], p, m, t.part, st, pdl);
    if (err == cudaSuccess) err = tc_launch_gemm(e, ws[1], p, m, t.part2, st, pdl);
    if (err == cudaSuccess) err = tc_launch_reduce<kEpiSwiglu>(e, p, m, (int)ws[0]->n, y, ldy, col0[0], st);
    return err;
  }
  for (int i = 0; i < nw && err == cudaSuccess; ++i) {
    const TcPlan p = tc_plan(m, ws[i]->n, k, e->num_sms);
    err = tc_launch_gemm(e, ws[i], p, m, t.part, st, pdl);
    if (err != cudaSuccess) break;
    err = epi == kEpiAdd ? tc_launch_reduce<kEpiAdd>(e, p, m, (int)ws[i]->n, y, ldy, col0[i], st)
                         : tc_launch_reduce<kEpiStore>(e, p, m, (int)ws[i]->n, y, ldy, col0[i], st);
  }
  return err;
}

}  // namespace b2q
