// tc_host.cuh -- launch planning of the tensor-core multi-token matmul
// (gemm_tc.cuh), included by b2q_api.cu.
#pragma once

namespace b2q {

struct TcPlan {
  int N, tiles, mpad, KS, rowtiles, splits;
};

// Token tiles of at most 256 (balanced), k-stages of 64, and a split-K
// factor of about one split per 24 stages (at most 16): long enough k-ranges
// to keep a CTA's pipeline full, few enough partial sums.  The split depends
// on k only, so every output element is summed in the same order whatever
// the number of rows (a tensor-parallel shard gives the same bits as the
// whole weight) or tokens.
static TcPlan tc_plan(int m, int64_t n, int64_t k, int num_sms) {
  (void)num_sms;
  TcPlan p;
  p.tiles = (m + kTcNMax - 1) / kTcNMax;
  p.N = round_up_int((m + p.tiles - 1) / p.tiles, 16);
  p.mpad = p.tiles * p.N;
  p.KS = (int)((k + kTcK - 1) / kTcK);
  p.rowtiles = (int)((n + kTcM - 1) / kTcM);
  p.splits = std::max(1, std::min(16, (p.KS + 12) / 24));
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
  t = TcScratch{};
}

// One launch over the weights ws[0..nw) (same k): weight i's rows go to
// columns c0[i].. of partial sums with ncol columns.
static cudaError_t tc_launch_gemm(b2q_engine* e, const b2q_weight* const* ws, const int* c0, int nw,
                                  const TcPlan& p, int m, float* part, int ncol, cudaStream_t st, bool pdl) {
  if (p.N < 16 || p.N > kTcNMax || p.N % 16 != 0 || nw < 1 || nw > kTcMaxSegs) return cudaErrorInvalidValue;
  TcArgs a;
  memset(&a, 0, sizeof a);
  a.nseg = nw;
  int rt = 0;
  for (int i = 0; i < nw; ++i) {
    a.w[i] = ws[i]->view;
    a.rt[i] = rt;
    a.c0[i] = c0[i];
    rt += (int)((ws[i]->n + kTcM - 1) / kTcM);
  }
  a.rt[nw] = rt;
  a.xh = e->tc.img;
  a.KS = p.KS;
  a.N = p.N;
  a.m = m;
  a.ncol = ncol;
  a.splits = p.splits;
  a.part = part;
  a.mpad = p.mpad;
  a.stages = tc_stages(p.N);
  if (a.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)a.stages * tc_stage_bytes(p.N);
  cudaError_t err = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rt, p.tiles, p.splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  // dependent launch: the weight-dequantising warps and the TMEM allocation
  // start while the previous kernel runs; the activation copies and the
  // partial-sum stores wait for it (griddepcontrol.wait).  Two GEMM grids
  // never overlap: the split-K reduce between them is a plain launch.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  launch_counted(e, 1);
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, a);
}

template <int EPI>
static cudaError_t tc_launch_reduce(b2q_engine* e, const TcPlan& p, int m, int n, int ldp, const float* part2,
                                    float* y, int ldy, int col0, cudaStream_t st) {
  // 16-byte vectors when every row of the partials and of y starts aligned
  const bool v4 = n % 4 == 0 && ldp % 4 == 0 && ldy % 4 == 0 && col0 % 4 == 0 &&
                  ((reinterpret_cast<uintptr_t>(e->tc.part) | reinterpret_cast<uintptr_t>(part2) |
                    reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const int per = 256 * (v4 ? 4 : 1);
  const dim3 grid((unsigned)std::min(64, (n + per - 1) / per), (unsigned)m);
  launch_counted(e, 1);
  if (v4)
    tc_reduce_kernel<EPI, 4><<<grid, 256, 0, st>>>(e->tc.part, part2, p.splits, p.mpad, m, n, ldp, e->tc.inv, y,
                                                   ldy, col0);
  else
    tc_reduce_kernel<EPI, 1><<<grid, 256, 0, st>>>(e->tc.part, part2, p.splits, p.mpad, m, n, ldp, e->tc.inv, y,
                                                   ldy, col0);
  return cudaGetLastError();
}

cudaError_t tc_matmul(b2q_engine* e, const float* x, int ldx, int m, int k, const b2q_weight* const* ws, int nw,
                      int epi, float* y, int ldy, const int* col0, cudaStream_t st, bool pdl, const float* norm_w,
                      float eps) {
  if (m < 1 || nw < 1 || (epi == kEpiSwiglu && nw != 2)) return cudaErrorInvalidValue;
  for (int i = 0; i < nw; ++i)
    if (ws[i]->k != k || !gemv_supported(ws[i]->dtype)) return cudaErrorInvalidValue;
  TcScratch& t = e->tc;
  const TcPlan p = tc_plan(m, ws[0]->n, k, e->num_sms);  // tiles, stages and splits depend on m and k only
  // weights whose outputs are adjacent columns (q | k | v), and the gate/up
  // pair, run as one launch; partial sums of all of them side by side
  bool fused = nw <= kTcMaxSegs;
  int64_t ncol = 0;
  for (int i = 0; i < nw; ++i) {
    if (epi != kEpiSwiglu && col0[i] != col0[0] + ncol) fused = false;
    ncol += ws[i]->n;
  }
  size_t part_need = 0;
  if (fused) part_need = (size_t)p.splits * p.mpad * ncol * sizeof(float);
  else
    for (int i = 0; i < nw; ++i) part_need = std::max(part_need, (size_t)p.splits * p.mpad * ws[i]->n * sizeof(float));
  cudaError_t err = tc_grow(reinterpret_cast<void**>(&t.img), &t.img_cap,
                            (size_t)p.tiles * p.KS * tc_b_bytes(p.N), st);
  if (err == cudaSuccess) err = tc_grow(reinterpret_cast<void**>(&t.inv), &t.inv_cap, (size_t)p.mpad * 4, st);
  if (err == cudaSuccess) err = tc_grow(reinterpret_cast<void**>(&t.part), &t.part_cap, part_need, st);
  if (err != cudaSuccess) return err;
  {
    launch_counted(e, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.mpad);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (norm_w != nullptr) {  // x is the residual: RMSNorm fused into the images
      cfg.blockDim = dim3(1024);
      cfg.dynamicSmemBytes = (size_t)k * sizeof(float);
      err = cudaLaunchKernelEx(&cfg, tc_rmsnorm_act_kernel, x, ldx, norm_w, eps, m, k, p.KS, p.N, t.img, t.inv);
    } else {
      err = cudaLaunchKernelEx(&cfg, tc_act_kernel, x, ldx, m, k, p.KS, p.N, t.img, t.inv);
    }
    if (err != cudaSuccess) return err;
  }
  if (fused) {
    int c[kTcMaxSegs];
    int64_t o = 0;
    for (int i = 0; i < nw; ++i) {
      c[i] = (int)o;
      o += ws[i]->n;
    }
    err = tc_launch_gemm(e, ws, c, nw, p, m, t.part, (int)ncol, st, pdl);
    if (err != cudaSuccess) return err;
    if (epi == kEpiSwiglu)
      return tc_launch_reduce<kEpiSwiglu>(e, p, m, (int)ws[0]->n, (int)ncol, t.part + ws[0]->n, y, ldy, col0[0], st);
    if (epi == kEpiAdd) return tc_launch_reduce<kEpiAdd>(e, p, m, (int)ncol, (int)ncol, nullptr, y, ldy, col0[0], st);
    return tc_launch_reduce<kEpiStore>(e, p, m, (int)ncol, (int)ncol, nullptr, y, ldy, col0[0], st);
  }
  for (int i = 0; i < nw && err == cudaSuccess; ++i) {
    const int z0 = 0, n = (int)ws[i]->n;
    err = tc_launch_gemm(e, &ws[i], &z0, 1, p, m, t.part, n, st, pdl);
    if (err != cudaSuccess) break;
    err = epi == kEpiAdd ? tc_launch_reduce<kEpiAdd>(e, p, m, n, n, nullptr, y, ldy, col0[i], st)
                         : tc_launch_reduce<kEpiStore>(e, p, m, n, n, nullptr, y, ldy, col0[i], st);
  }
  return err;
}

}  // namespace b2q
