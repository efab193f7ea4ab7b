// b2q_api.cu -- the C ABI of include/b2q.h: engine, weights, matvec entry
// points and error handling.  The whole-model forward (model_impl.cuh,
// model_api.cuh) is included at the end: libb2q is one translation unit.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b2q.h"
#include "internal.h"

namespace b2q {

static thread_local std::string t_last_error;

b2q_status set_error(b2q_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return st;
}

b2q_status cuda_error(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return set_error(B2Q_ENOMEM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(B2Q_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool gemv_supported(int dtype) {
  return dtype == kQ4_K || dtype == kQ6_K || dtype == kQ8_0 || dtype == kQ5_K || dtype == kQ4_0;
}

int dtype_block(int t) {
  switch (t) {
    case kF32: case kF16: case kBF16: return 1;
    case kQ4_0: case kQ8_0: return 32;
    case kQ4_K: case kQ5_K: case kQ6_K: return 256;
    default: return 0;
  }
}
int dtype_size(int t) {
  switch (t) {
    case kF32: return 4;
    case kF16: case kBF16: return 2;
    case kQ4_0: return 18;
    case kQ8_0: return 34;
    case kQ4_K: return 144;
    case kQ5_K: return 176;
    case kQ6_K: return 210;
    default: return 0;
  }
}

cudaError_t launch_counted(b2q_engine* e, uint64_t n) {
  e->launches.fetch_add(n, std::memory_order_relaxed);
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// XQ workspace
// ---------------------------------------------------------------------------
cudaError_t xq_alloc(XQBuf* b, int m, int k) {
  b->m = m;
  b->k = k;
  b->kpad = round_up_int(k, 256);
  const size_t nq = (size_t)m * b->kpad;
  const size_t bq = align_up(nq * 2, 256), bs = align_up(nq / 64 * 4, 256),
               b16 = align_up(nq / 16 * 4, 256);
  cudaError_t err = cudaMalloc(&b->mem, bq + bs + b16);
  if (err != cudaSuccess) return err;
  err = cudaMemset(b->mem, 0, bq + bs + b16);
  // the memset runs on the legacy stream, which does not order with the
  // library's non-blocking streams: finish it before anyone uses the buffer
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return err;
  uint8_t* p = static_cast<uint8_t*>(b->mem);
  b->x.q = reinterpret_cast<int16_t*>(p);
  b->x.scale = reinterpret_cast<float*>(p + bq);
  b->x.s16 = reinterpret_cast<int32_t*>(p + bq + bs);
  b->x.kpad = b->kpad;
  return cudaSuccess;
}

void xq_free(XQBuf* b) {
  if (b->mem) cudaFree(b->mem);
  b->mem = nullptr;
}

// ---------------------------------------------------------------------------
// GEMV launch planning
// ---------------------------------------------------------------------------
constexpr int kStageMax = 40 * 1024;  // two tiles per stage when they fit

template <int MT, int EPI>
static cudaError_t launch_gemv_t(b2q_engine* e, GemvArgs& a, cudaStream_t st, bool pdl) {
  constexpr bool kPair = EPI == kEpiSwiglu;
  // bytes per segment -> share of the persistent grid (one CTA per SM)
  double total = 0.0;
  double bytes[kMaxSegs];
  int slot = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const TileLayout& L = a.seg[s].w.L;
    const int tb = (int)tile_bytes(L);
    a.seg[s].nr = (kPair || 2 * tb <= kStageMax) ? 2 : 1;
    slot = std::max(slot, tb * a.seg[s].nr);
    bytes[s] = (double)L.G * L.C * tb * (kPair ? 2 : 1);
    total += bytes[s];
  }
  int cta = 0, rows_cap = 8;
  for (int s = 0; s < a.nseg; ++s) {
    GemvSeg& g = a.seg[s];
    int n = (int)((double)e->num_sms * bytes[s] / total + 0.5);
    n = std::max(1, std::min(n, g.w.L.G));
    g.cta0 = cta;
    g.ncta = n;
    cta += n;
    rows_cap = std::max(rows_cap, gemv_rows_cap(g.w.L.G, n));
  }
  if (cta == 0) return cudaSuccess;
  a.rows_cap = rows_cap;
  const size_t xb = gemv_x_bytes(a.kpad, MT);
  const size_t rb = (size_t)2 * (kPair ? 2 : 1) * rows_cap * MT * sizeof(float);
  if (xb + rb + 2 * (size_t)slot > kGemvSmemBudget) return cudaErrorInvalidConfiguration;
  const int ns = (int)std::min<size_t>(kGemvMaxStages, (kGemvSmemBudget - xb - rb) / (size_t)slot);
  a.ns = ns;
  a.slot_bytes = slot;
  const size_t smem = xb + (size_t)ns * slot + rb;
  auto kern = gemv_kernel<MT, EPI>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cta);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  launch_counted(e, 1);
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_gemv(b2q_engine* e, GemvArgs& a, int epi, int mt, cudaStream_t st, bool pdl) {
  if (epi == kEpiSwiglu) return launch_gemv_t<1, kEpiSwiglu>(e, a, st, pdl);
  if (epi == kEpiStore) return mt == 1 ? launch_gemv_t<1, kEpiStore>(e, a, st, pdl)
                                       : launch_gemv_t<2, kEpiStore>(e, a, st, pdl);
  return mt == 1 ? launch_gemv_t<1, kEpiAdd>(e, a, st, pdl) : launch_gemv_t<2, kEpiAdd>(e, a, st, pdl);
}

b2q_status sample_core(b2q_engine* e, const float* logits_dev, int n, float temperature, float top_p,
                       uint64_t* rng_state, uint32_t* token, cudaStream_t st) {
  if (n <= 0) return set_error(B2Q_EINVAL, "sample: no logits");
  cudaError_t err = cudaSuccess;
  if (!e->ws_sample_out) err = cudaMalloc(&e->ws_sample_out, 2 * sizeof(uint32_t));
  if (err == cudaSuccess && e->ws_sample_cap < (size_t)n) {
    if (e->ws_sample) cudaFree(e->ws_sample);
    e->ws_sample = nullptr;
    e->ws_sample_cap = 0;
    err = cudaMalloc(&e->ws_sample, sizeof(float) * (size_t)n);
    if (err == cudaSuccess) e->ws_sample_cap = (size_t)n;
  }
  if (err != cudaSuccess) return cuda_error(err, "sample: workspace");
  uint32_t out[2] = {0u, 0u};
  if (temperature <= 1e-5f) {  // greedy: first index of the maximum, no draw
    launch_counted(e, 1);
    argmax_kernel<<<1, 1024, 0, st>>>(logits_dev, n, e->ws_sample_out);
  } else {
    // the draw the reference's next_f32 makes, kept only if the sampler uses it
    uint64_t x = *rng_state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    const float u = (float)(uint32_t)(x >> 40) / (float)(1u << 24);
    launch_counted(e, 1);
    sample_top_p_kernel<<<1, kSampleThreads, 0, st>>>(logits_dev, n, temperature, top_p, u, e->ws_sample,
                                                       e->ws_sample_out);
    err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaMemcpyAsync(out, e->ws_sample_out, sizeof out, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) return cuda_error(err, "sample");
    if (out[1]) *rng_state = x;
    *token = out[0];
    return B2Q_OK;
  }
  err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaMemcpyAsync(out, e->ws_sample_out, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_error(err, "sample");
  *token = out[0];
  return B2Q_OK;
}

}  // namespace b2q
#include "tc_host.cuh"
namespace b2q {

// Largest token count per GEMV pass: each consumer lane keeps the
// activations of every token of the pass in registers (32 per token), so
// passes carry at most two tokens; larger prompts loop over passes.
int gemv_max_mt(int kpad) {
  const size_t budget = kGemvSmemBudget - 4 * (size_t)(8 * 3360);
  return gemv_x_bytes(kpad, 2) <= budget ? 2 : 1;
}

// Run y = W x for all m tokens of an XQ buffer, in passes of MT tokens.
// `segs` carry w / y / ldy / rows_out; y pointers are for token 0.
cudaError_t run_gemv(b2q_engine* e, const GemvSeg* segs, int nseg, const XQBuf& xq, int m,
                     int epi, cudaStream_t st, bool pdl) {
  int t = 0;
  const int mtmax = (epi == kEpiSwiglu) ? 1 : gemv_max_mt(xq.kpad);
  while (t < m) {
    const int mt = (mtmax >= 2 && m - t >= 2) ? 2 : 1;
    GemvArgs a;
    memset(&a, 0, sizeof a);
    a.nseg = nseg;
    for (int s = 0; s < nseg; ++s) {
      a.seg[s] = segs[s];
      a.seg[s].y = segs[s].y + (int64_t)t * segs[s].ldy;
    }
    a.xq = xq.x.q;
    a.xscale = xq.x.scale;
    a.xs16 = xq.x.s16;
    a.kpad = xq.kpad;
    a.t0 = t;
    cudaError_t err = launch_gemv(e, a, epi, mt, st, pdl);
    if (err != cudaSuccess) return err;
    t += mt;
  }
  return cudaSuccess;
}

cudaError_t launch_quantize(b2q_engine* e, const float* x, int m, int k, XQBuf& xq, cudaStream_t st,
                            bool pdl) {
  const int blocks = std::max(1, std::min(e->num_sms * 4, (m * (xq.kpad / 32) + 7) / 8));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  launch_counted(e, 1);
  return cudaLaunchKernelEx(&cfg, quantize_x_kernel, x, m, k, xq.x);
}

}  // namespace b2q

using namespace b2q;

// ===========================================================================
// Allocation-free matvec scratch.
//
// b2q_matmul_noalloc_dev serves callers that must not allocate device
// memory -- code running where cudaMalloc is forbidden or unsafe (inside a
// memory pool that has to stay fixed for the life of a process, on a
// real-time path that cannot afford an allocation's synchronisation, or
// in a host whose allocator is owned by someone else).  Its only scratch,
// the quantised activations, lives in this file-scope array, which every GPU
// that loads the library holds until the process exits.
// ===========================================================================
namespace {

// int16 codes of m*kpad activations + one f32 scale per 64 + one int32 sum
// per 16: 2 + 4/64 + 4/16 bytes per element.
constexpr int64_t kNoAllocMaxElems = 262144;  // m * round_up(k, 256) limit
constexpr size_t kNoAllocQBytes = (size_t)kNoAllocMaxElems * 2;
constexpr size_t kNoAllocScaleBytes = (size_t)kNoAllocMaxElems / 64 * 4;
constexpr size_t kNoAllocSumBytes = (size_t)kNoAllocMaxElems / 16 * 4;
constexpr size_t kNoAllocBytes = kNoAllocQBytes + kNoAllocScaleBytes + kNoAllocSumBytes;  // 606,208

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device.  The host-side
// name g_noalloc_scratch is only a stand-in for the symbol; the address a
// kernel can use comes from cudaGetSymbolAddress, looked up once per device.
b2q_status noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) return set_error(B2Q_EINVAL, "noalloc: device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) return cuda_error(err, "noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return B2Q_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* b2q_last_error(void) { return t_last_error.c_str(); }
const char* b2q_version(void) { return "b2q 0.1 (sm_100a)"; }

b2q_status b2q_init(int device, b2q_engine** out) {
  if (!out) return set_error(B2Q_EINVAL, "b2q_init: out is NULL");
  *out = nullptr;
  int ndev = 0;
  cudaError_t err = cudaGetDeviceCount(&ndev);
  if (err != cudaSuccess) return cuda_error(err, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev)
    return set_error(B2Q_EINVAL, "b2q_init: device %d out of range (%d devices)", device, ndev);
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_error(err, "cudaSetDevice");
  cudaDeviceProp prop;
  err = cudaGetDeviceProperties(&prop, device);
  if (err != cudaSuccess) return cuda_error(err, "cudaGetDeviceProperties");
  if (prop.major < 10)
    return set_error(B2Q_EUNSUP, "b2q_init: %s is sm_%d%d; this library is built for sm_100a",
                     prop.name, prop.major, prop.minor);
  b2q_engine* e = new b2q_engine();
  e->device = device;
  e->num_sms = prop.multiProcessorCount;
  e->l2_bytes = prop.l2CacheSize;
  snprintf(e->name, sizeof e->name, "%s", prop.name);
  err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  if (err != cudaSuccess) {
    delete e;
    return cuda_error(err, "cudaStreamCreate");
  }
  *out = e;
  return B2Q_OK;
}

static void ws_free(b2q_engine* e) {
  if (e->ws_x) cudaFree(e->ws_x);
  if (e->ws_y) cudaFree(e->ws_y);
  if (e->ws_h) cudaFree(e->ws_h);
  xq_free(&e->ws_xq);
  xq_free(&e->ws_hq);
  tc_free(e);
  if (e->ws_gdn) cudaFree(e->ws_gdn);
  e->ws_gdn = nullptr;
  e->ws_gdn_cap = 0;
  if (e->ws_sample) cudaFree(e->ws_sample);
  if (e->ws_sample_out) cudaFree(e->ws_sample_out);
  e->ws_sample = nullptr;
  e->ws_sample_out = nullptr;
  e->ws_sample_cap = 0;
  e->ws_x = e->ws_y = e->ws_h = nullptr;
  e->ws_x_cap = e->ws_y_cap = e->ws_h_cap = 0;
}

b2q_status b2q_engine_destroy(b2q_engine* e) {
  if (!e) return B2Q_OK;
  cudaSetDevice(e->device);
  cudaStreamSynchronize(e->stream);
  ws_free(e);
  cudaStreamDestroy(e->stream);
  delete e;
  return B2Q_OK;
}

b2q_status b2q_device_info(b2q_engine* e, char* name, size_t name_len, size_t* free_bytes,
                           size_t* total_bytes) {
  if (!e) return set_error(B2Q_EINVAL, "engine is NULL");
  cudaSetDevice(e->device);
  if (name && name_len) snprintf(name, name_len, "%s", e->name);
  size_t f = 0, t = 0;
  cudaError_t err = cudaMemGetInfo(&f, &t);
  if (err != cudaSuccess) return cuda_error(err, "cudaMemGetInfo");
  if (free_bytes) *free_bytes = f;
  if (total_bytes) *total_bytes = t;
  return B2Q_OK;
}

int b2q_can_alloc(b2q_engine* e, size_t bytes, size_t reserve) {
  if (!e) return 0;
  cudaSetDevice(e->device);
  size_t f = 0, t = 0;
  if (cudaMemGetInfo(&f, &t) != cudaSuccess) return 0;
  return f > bytes + reserve ? 1 : 0;
}

size_t b2q_weight_bytes(const b2q_weight* w) { return w ? w->gguf_bytes : 0; }

b2q_status b2q_upload_weight(b2q_engine* e, const void* bytes, size_t len, int dtype, int64_t n,
                             int64_t k, b2q_weight** out) {
  if (!e || !bytes || !out) return set_error(B2Q_EINVAL, "b2q_upload_weight: NULL argument");
  *out = nullptr;
  if (!gemv_supported(dtype))
    return set_error(B2Q_EUNSUP, "b2q_upload_weight: GGML type %d has no GEMV kernel", dtype);
  const int bs = dtype_block(dtype), ts = dtype_size(dtype);
  if (n <= 0 || k <= 0 || k % bs != 0 || k % 64 != 0)
    return set_error(B2Q_EINVAL, "b2q_upload_weight: bad shape [%lld, %lld] for type %d",
                     (long long)n, (long long)k, dtype);
  if (n > (int64_t)INT32_MAX / 2 || k > (1 << 24))
    return set_error(B2Q_EINVAL, "b2q_upload_weight: shape too large");
  const int64_t nb = k / bs;
  const size_t need = (size_t)(n * nb * ts);
  if (len != need)
    return set_error(B2Q_EINVAL, "b2q_upload_weight: %zu bytes given, [%lld, %lld] type %d needs %zu",
                     len, (long long)n, (long long)k, dtype, need);
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  b2q_weight* w = new b2q_weight();
  w->eng = e;
  w->dtype = dtype;
  w->n = n;
  w->k = k;
  w->gguf_bytes = need;
  WeightDev& v = w->view;
  v.L = make_tile_layout(dtype, n, k);
  const size_t total = (size_t)v.L.G * v.L.C * (size_t)tile_bytes(v.L);
  cudaError_t err = cudaMalloc(&w->mem, total);
  if (err != cudaSuccess) {
    delete w;
    return cuda_error(err, "b2q_upload_weight: cudaMalloc");
  }
  cudaMemsetAsync(w->mem, 0, total, e->stream);  // padding units / rows stay zero
  w->mem_bytes = total;
  uint8_t* base = static_cast<uint8_t*>(w->mem);
  v.base = base;
  // stage the raw bytes on the device, then repack
  cudaPointerAttributes pa;
  const bool is_dev = cudaPointerGetAttributes(&pa, bytes) == cudaSuccess &&
                      pa.type == cudaMemoryTypeDevice;
  cudaGetLastError();
  void* raw = nullptr;
  if (is_dev) {
    raw = const_cast<void*>(bytes);
  } else {
    err = cudaMalloc(&raw, need);
    if (err != cudaSuccess) {
      cudaFree(w->mem);
      delete w;
      return cuda_error(err, "b2q_upload_weight: staging cudaMalloc");
    }
    err = cudaMemcpyAsync(raw, bytes, need, cudaMemcpyHostToDevice, e->stream);
  }
  if (err == cudaSuccess) {
    const int64_t units = n * (int64_t)v.L.U;
    const int blocks = (int)std::min<int64_t>((units + 255) / 256, 65535);
    const uint8_t* r8 = static_cast<const uint8_t*>(raw);
    if (dtype == kQ4_K)
      repack_q4k_kernel<<<blocks, 256, 0, e->stream>>>(r8, v.L, base);
    else if (dtype == kQ6_K)
      repack_q6k_kernel<<<blocks, 256, 0, e->stream>>>(r8, v.L, base);
    else if (dtype == kQ5_K)
      repack_q5k_kernel<<<blocks, 256, 0, e->stream>>>(r8, v.L, base);
    else if (dtype == kQ4_0)
      repack_q40_kernel<<<blocks, 256, 0, e->stream>>>(r8, v.L, base);
    else
      repack_q80_kernel<<<blocks, 256, 0, e->stream>>>(r8, v.L, base);
    launch_counted(e, 1);
    err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  }
  if (!is_dev && raw) cudaFree(raw);
  if (err != cudaSuccess) {
    cudaFree(w->mem);
    delete w;
    return cuda_error(err, "b2q_upload_weight: repack");
  }
  *out = w;
  return B2Q_OK;
}

b2q_status b2q_weight_free(b2q_weight* w) {
  if (!w) return B2Q_OK;
  cudaSetDevice(w->eng->device);
  if (w->mem) cudaFree(w->mem);
  delete w;
  return B2Q_OK;
}

// --- workspace for the host-pointer entry points ---------------------------
static cudaError_t ws_reserve(float** p, size_t* cap, size_t bytes) {
  if (*cap >= bytes) return cudaSuccess;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t err = cudaMalloc(p, bytes);
  if (err == cudaSuccess) *cap = bytes;
  return err;
}

static cudaError_t ws_xq(XQBuf* b, int m, int k) {
  const int kpad = round_up_int(k, 256);
  if (b->mem && b->m >= m && b->kpad >= kpad) {
    // same buffer, but the quantiser writes exactly kpad columns per row
    b->kpad = kpad;
    b->x.kpad = kpad;
    b->k = k;
    return cudaSuccess;
  }
  xq_free(b);
  return xq_alloc(b, std::max(m, 1), std::max(k, 256));
}

static b2q_status check_weight(const b2q_weight* w, int n, int k, const char* what) {
  if (!w) return set_error(B2Q_EINVAL, "%s: weight is NULL", what);
  if (w->n != n || w->k != k)
    return set_error(B2Q_EINVAL, "%s: weight is [%lld, %lld], call asks for [%d, %d]", what,
                     (long long)w->n, (long long)w->k, n, k);
  return B2Q_OK;
}

static GemvSeg make_seg(const b2q_weight* w, float* y, int ldy) {
  GemvSeg s;
  memset(&s, 0, sizeof s);
  s.w = w->view;
  s.w2 = w->view;
  s.y = y;
  s.ldy = ldy;
  s.rows_out = (int)w->n;
  return s;
}

// y = W x with x, y device pointers
static b2q_status matmul_group_core(b2q_engine* e, const b2q_weight* const* ws, const int* ns,
                                   int count, const float* x_dev, int m, int k, float* y_dev,
                                   cudaStream_t st) {
  if (count <= 0) return set_error(B2Q_EINVAL, "matmul_group: count must be positive");
  if (m <= 0 || k <= 0) return set_error(B2Q_EINVAL, "matmul: m and k must be positive");
  for (int i = 0; i < count; ++i) {
    b2q_status s = check_weight(ws[i], ns[i], k, "matmul");
    if (s != B2Q_OK) return s;
  }
  if (m >= kTcMinTokens) {
    // many tokens per weight row: tensor cores
    int64_t off = 0;
    for (int i = 0; i < count; ++i) {
      const int col0 = 0;
      cudaError_t err = tc_matmul(e, x_dev, k, m, k, &ws[i], 1, kEpiStore, y_dev + off, ns[i], &col0, st, false);
      if (err != cudaSuccess) return cuda_error(err, "matmul: tensor-core launch");
      off += (int64_t)m * ns[i];
    }
    return B2Q_OK;
  }
  cudaError_t err = ws_xq(&e->ws_xq, m, k);
  if (err != cudaSuccess) return cuda_error(err, "matmul: workspace");
  err = launch_quantize(e, x_dev, m, k, e->ws_xq, st, false);
  if (err != cudaSuccess) return cuda_error(err, "matmul: quantize launch");
  // outputs are concatenated per weight, each [m][n_i]
  int64_t off = 0;
  for (int i0 = 0; i0 < count; i0 += kMaxSegs) {
    GemvSeg segs[kMaxSegs];
    const int c = std::min(kMaxSegs, count - i0);
    for (int j = 0; j < c; ++j) {
      segs[j] = make_seg(ws[i0 + j], y_dev + off, ns[i0 + j]);
      off += (int64_t)m * ns[i0 + j];
    }
    err = run_gemv(e, segs, c, e->ws_xq, m, kEpiStore, st, false);
    if (err != cudaSuccess) return cuda_error(err, "matmul: gemv launch");
  }
  return B2Q_OK;
}

b2q_status b2q_matmul_group_dev(b2q_engine* e, const b2q_weight* const* ws, const int* ns, int count,
                                const float* x_dev, int m, int k, float* y_dev, void* stream) {
  if (!e || !ws || !ns || !x_dev || !y_dev) return set_error(B2Q_EINVAL, "matmul_group_dev: NULL argument");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  return matmul_group_core(e, ws, ns, count, x_dev, m, k, y_dev,
                           stream ? (cudaStream_t)stream : e->stream);
}

b2q_status b2q_matmul_dev(b2q_engine* e, const b2q_weight* w, const float* x_dev, float* y_dev, int m,
                          int n, int k, void* stream) {
  const b2q_weight* ws[1] = {w};
  int ns[1] = {n};
  return b2q_matmul_group_dev(e, ws, ns, 1, x_dev, m, k, y_dev, stream);
}

b2q_status b2q_matmul_group(b2q_engine* e, const b2q_weight* const* ws, const int* ns, int count,
                            const float* x, int m, int k, float* y_flat) {
  if (!e || !ws || !ns || !x || !y_flat) return set_error(B2Q_EINVAL, "matmul_group: NULL argument");
  if (count <= 0 || m <= 0 || k <= 0) return set_error(B2Q_EINVAL, "matmul_group: bad sizes");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  int64_t total_n = 0;
  for (int i = 0; i < count; ++i) total_n += ns[i];
  const size_t xb = (size_t)m * k * 4, yb = (size_t)m * total_n * 4;
  cudaError_t err = ws_reserve(&e->ws_x, &e->ws_x_cap, xb);
  if (err == cudaSuccess) err = ws_reserve(&e->ws_y, &e->ws_y_cap, yb);
  if (err != cudaSuccess) return cuda_error(err, "matmul_group: workspace");
  err = cudaMemcpyAsync(e->ws_x, x, xb, cudaMemcpyHostToDevice, e->stream);
  if (err != cudaSuccess) return cuda_error(err, "matmul_group: H2D");
  b2q_status s = matmul_group_core(e, ws, ns, count, e->ws_x, m, k, e->ws_y, e->stream);
  if (s != B2Q_OK) return s;
  err = cudaMemcpyAsync(y_flat, e->ws_y, yb, cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return cuda_error(err, "matmul_group: D2H");
  return B2Q_OK;
}

b2q_status b2q_matmul(b2q_engine* e, const b2q_weight* w, const float* x, float* y, int m, int n, int k) {
  const b2q_weight* ws[1] = {w};
  int ns[1] = {n};
  return b2q_matmul_group(e, ws, ns, 1, x, m, k, y);
}

static b2q_status ffn_core(b2q_engine* e, const b2q_weight* gate, const b2q_weight* up,
                           const b2q_weight* down, const float* x_dev, int m, int n_embd,
                           int ffn_inter, float* y_dev, cudaStream_t st) {
  b2q_status s = check_weight(gate, ffn_inter, n_embd, "ffn_swiglu(gate)");
  if (s == B2Q_OK) s = check_weight(up, ffn_inter, n_embd, "ffn_swiglu(up)");
  if (s == B2Q_OK) s = check_weight(down, n_embd, ffn_inter, "ffn_swiglu(down)");
  if (s != B2Q_OK) return s;
  if (gate->dtype != up->dtype)
    return set_error(B2Q_EUNSUP, "ffn_swiglu: gate and up must share a GGML type");
  if (m >= kTcMinTokens) {
    cudaError_t err = ws_reserve(&e->ws_h, &e->ws_h_cap, (size_t)m * ffn_inter * 4);
    const b2q_weight* gu[2] = {gate, up};
    const int col0 = 0;
    if (err == cudaSuccess)
      err = tc_matmul(e, x_dev, n_embd, m, n_embd, gu, 2, kEpiSwiglu, e->ws_h, ffn_inter, &col0, st, false);
    if (err == cudaSuccess)
      err = tc_matmul(e, e->ws_h, ffn_inter, m, ffn_inter, &down, 1, kEpiStore, y_dev, n_embd, &col0, st, false);
    if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: tensor-core launch");
    return B2Q_OK;
  }
  cudaError_t err = ws_xq(&e->ws_xq, m, n_embd);
  if (err == cudaSuccess) err = ws_xq(&e->ws_hq, m, ffn_inter);
  if (err == cudaSuccess) err = ws_reserve(&e->ws_h, &e->ws_h_cap, (size_t)m * ffn_inter * 4);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: workspace");
  err = launch_quantize(e, x_dev, m, n_embd, e->ws_xq, st, false);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: quantize");
  for (int t = 0; t < m; ++t) {
    GemvSeg sg = make_seg(gate, e->ws_h + (int64_t)t * ffn_inter, ffn_inter);
    sg.w2 = up->view;
    GemvArgs a;
    memset(&a, 0, sizeof a);
    a.nseg = 1;
    a.seg[0] = sg;
    a.xq = e->ws_xq.x.q;
    a.xscale = e->ws_xq.x.scale;
    a.xs16 = e->ws_xq.x.s16;
    a.kpad = e->ws_xq.kpad;
    a.t0 = t;
    err = launch_gemv(e, a, kEpiSwiglu, 1, st, false);
    if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: gate/up gemv");
  }
  err = launch_quantize(e, e->ws_h, m, ffn_inter, e->ws_hq, st, false);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: quantize h");
  GemvSeg sd = make_seg(down, y_dev, n_embd);
  err = run_gemv(e, &sd, 1, e->ws_hq, m, kEpiStore, st, false);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: down gemv");
  return B2Q_OK;
}

b2q_status b2q_ffn_swiglu_dev(b2q_engine* e, const b2q_weight* gate, const b2q_weight* up,
                              const b2q_weight* down, const float* x_dev, int m, int n_embd,
                              int ffn_inter, float* y_dev, void* stream) {
  if (!e || !x_dev || !y_dev) return set_error(B2Q_EINVAL, "ffn_swiglu_dev: NULL argument");
  if (m <= 0) return set_error(B2Q_EINVAL, "ffn_swiglu_dev: m must be positive");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  return ffn_core(e, gate, up, down, x_dev, m, n_embd, ffn_inter, y_dev,
                  stream ? (cudaStream_t)stream : e->stream);
}

b2q_status b2q_ffn_swiglu(b2q_engine* e, const b2q_weight* gate, const b2q_weight* up,
                          const b2q_weight* down, const float* x, int m, int n_embd, int ffn_inter,
                          float* y) {
  if (!e || !x || !y) return set_error(B2Q_EINVAL, "ffn_swiglu: NULL argument");
  if (m <= 0 || n_embd <= 0 || ffn_inter <= 0) return set_error(B2Q_EINVAL, "ffn_swiglu: bad sizes");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  const size_t xb = (size_t)m * n_embd * 4;
  cudaError_t err = ws_reserve(&e->ws_x, &e->ws_x_cap, xb);
  if (err == cudaSuccess) err = ws_reserve(&e->ws_y, &e->ws_y_cap, xb);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: workspace");
  err = cudaMemcpyAsync(e->ws_x, x, xb, cudaMemcpyHostToDevice, e->stream);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: H2D");
  b2q_status s = ffn_core(e, gate, up, down, e->ws_x, m, n_embd, ffn_inter, e->ws_y, e->stream);
  if (s != B2Q_OK) return s;
  err = cudaMemcpyAsync(y, e->ws_y, xb, cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return cuda_error(err, "ffn_swiglu: D2H");
  return B2Q_OK;
}

b2q_status b2q_dequantize_dev(b2q_engine* e, const void* raw_dev, int dtype, int64_t n_elems,
                              float* out_dev, void* stream) {
  if (!e || !raw_dev || !out_dev) return set_error(B2Q_EINVAL, "dequantize_dev: NULL argument");
  const int bs = dtype_block(dtype);
  if (bs == 0) return set_error(B2Q_EUNSUP, "dequantize_dev: GGML type %d not supported", dtype);
  if (n_elems < 0 || n_elems % bs != 0)
    return set_error(B2Q_EINVAL, "dequantize_dev: %lld elements is not a whole number of blocks",
                     (long long)n_elems);
  if (n_elems == 0) return B2Q_OK;
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  const int64_t slots = dequant_slots(dtype, n_elems);
  const int blocks = (int)std::min<int64_t>((slots + 255) / 256, (int64_t)e->num_sms * 16);
  dequant_kernel<<<blocks, 256, 0, stream ? (cudaStream_t)stream : e->stream>>>(
      static_cast<const uint8_t*>(raw_dev), dtype, n_elems, out_dev);
  launch_counted(e, 1);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "dequantize_dev launch");
  return B2Q_OK;
}

b2q_status b2q_time_gemv(b2q_engine* e, const b2q_weight* const* ws, int count, const float* x_dev,
                         int k, int reps, void* stream, float* avg_ms, int chained) {
  if (!e || !ws || count <= 0 || !x_dev || reps <= 0 || !avg_ms)
    return set_error(B2Q_EINVAL, "b2q_time_gemv: bad argument");
  int64_t nmax = 0;
  for (int i = 0; i < count; ++i) {
    if (!ws[i] || ws[i]->k != k) return set_error(B2Q_EINVAL, "b2q_time_gemv: weight %d has k != %d", i, k);
    nmax = std::max(nmax, ws[i]->n);
  }
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : e->stream;
  cudaError_t err = ws_xq(&e->ws_xq, 1, k);
  if (err == cudaSuccess) err = ws_reserve(&e->ws_y, &e->ws_y_cap, (size_t)nmax * 4);
  if (err != cudaSuccess) return cuda_error(err, "b2q_time_gemv: workspace");
  err = launch_quantize(e, x_dev, 1, k, e->ws_xq, st, false);
  if (err != cudaSuccess) return cuda_error(err, "b2q_time_gemv: quantize");
  cudaEvent_t ev0, ev1;
  cudaEventCreate(&ev0);
  cudaEventCreate(&ev1);
  cudaEventRecord(ev0, st);
  for (int r = 0; r < reps && err == cudaSuccess; ++r)
    for (int i = 0; i < count && err == cudaSuccess; ++i) {
      GemvSeg sg = make_seg(ws[i], e->ws_y, (int)ws[i]->n);
      // chained: programmatic dependent launch, as the per-kernel decode
      // path launches its GEMVs (the next launch streams its weights while
      // this one drains; it reads the activations only after this one ends)
      err = run_gemv(e, &sg, 1, e->ws_xq, 1, kEpiStore, st, chained != 0);
    }
  cudaEventRecord(ev1, st);
  if (err == cudaSuccess) err = cudaEventSynchronize(ev1);
  float ms = 0.0f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, ev0, ev1);
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  if (err != cudaSuccess) return cuda_error(err, "b2q_time_gemv");
  *avg_ms = ms / (float)(reps * count);
  return B2Q_OK;
}

b2q_status b2q_matmul_noalloc_dev(const b2q_weight* w, const float* x_dev, float* y_dev, int m, int n, int k,
                                  void* stream) {
  if (!w || !x_dev || !y_dev) return set_error(B2Q_EINVAL, "matmul_noalloc_dev: NULL argument");
  if (m <= 0 || n <= 0 || k <= 0) return set_error(B2Q_EINVAL, "matmul_noalloc_dev: m, n and k must be positive");
  b2q_status s = check_weight(w, n, k, "matmul_noalloc_dev");
  if (s != B2Q_OK) return s;
  const int kpad = round_up_int(k, 256);
  if ((int64_t)m * kpad > kNoAllocMaxElems)
    return set_error(B2Q_EINVAL,
                     "matmul_noalloc_dev: m * round_up(k, 256) = %lld exceeds the fixed scratch of %lld "
                     "activations (use b2q_matmul_dev)",
                     (long long)m * kpad, (long long)kNoAllocMaxElems);
  b2q_engine* e = w->eng;
  cudaError_t err = cudaSetDevice(e->device);
  if (err != cudaSuccess) return cuda_error(err, "matmul_noalloc_dev: cudaSetDevice");
  void* base = nullptr;
  s = noalloc_scratch(e->device, &base);
  if (s != B2Q_OK) return s;
  // carve the quantised-activation buffer out of the static array; the
  // quantiser rewrites every element the GEMV reads, so nothing in it has
  // to start at zero
  XQBuf xq;
  uint8_t* p = static_cast<uint8_t*>(base);
  xq.m = m;
  xq.k = k;
  xq.kpad = kpad;
  xq.x.kpad = kpad;
  xq.x.q = reinterpret_cast<int16_t*>(p);
  xq.x.scale = reinterpret_cast<float*>(p + kNoAllocQBytes);
  xq.x.s16 = reinterpret_cast<int32_t*>(p + kNoAllocQBytes + kNoAllocScaleBytes);
  cudaStream_t st = stream ? (cudaStream_t)stream : e->stream;
  err = launch_quantize(e, x_dev, m, k, xq, st, false);
  if (err != cudaSuccess) return cuda_error(err, "matmul_noalloc_dev: quantize launch");
  GemvSeg sg = make_seg(w, y_dev, n);
  err = run_gemv(e, &sg, 1, xq, m, kEpiStore, st, false);
  if (err != cudaSuccess) return cuda_error(err, "matmul_noalloc_dev: gemv launch");
  return B2Q_OK;
}

uint64_t b2q_kernel_launch_count(b2q_engine* e) { return e ? e->launches.load() : 0; }

#ifdef B2Q_DECODE_TRACE
// Developer build only: copy the persistent decode kernel's timeline out.
int b2q_debug_decode_trace(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, b2q::g_dec_trace, std::min(bytes, sizeof(b2q::g_dec_trace))) == cudaSuccess ? 0 : 1;
}
int b2q_debug_decode_wait(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, b2q::g_dec_wait, std::min(bytes, sizeof(b2q::g_dec_wait))) == cudaSuccess ? 0 : 1;
}
int b2q_debug_decode_fine(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, b2q::g_dec_fine, std::min(bytes, sizeof(b2q::g_dec_fine))) == cudaSuccess ? 0 : 1;
}
int b2q_debug_decode_dbg(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, b2q::g_dec_dbg, std::min(bytes, sizeof(b2q::g_dec_dbg))) == cudaSuccess ? 0 : 1;
}
#endif

b2q_status b2q_gdn_step_dev(b2q_engine* e, const b2q_gdn_config* cfg, int n_tokens, const float* qkv,
                            const float* z, const float* alpha, const float* beta, const float* conv_w,
                            const float* ssm_a, const float* dt_bias, const float* ssm_norm, float* conv_state,
                            float* ssm_state, float* y, void* stream) {
  if (!e || !cfg || !qkv || !z || !alpha || !beta || !conv_w || !ssm_a || !dt_bias || !ssm_norm || !conv_state ||
      !ssm_state || !y)
    return set_error(B2Q_EINVAL, "b2q_gdn_step_dev: NULL argument");
  const b2q_gdn_config c = *cfg;
  if (n_tokens <= 0) return set_error(B2Q_EINVAL, "b2q_gdn_step_dev: n_tokens must be positive");
  if (c.d_k != 128) return set_error(B2Q_EUNSUP, "b2q_gdn_step_dev: d_k %d (128 is supported)", c.d_k);
  if (c.d_v <= 0 || c.d_v > 512 || c.n_k_heads <= 0 || c.n_v_heads <= 0 || c.n_v_heads % c.n_k_heads ||
      c.conv_kernel < 1)
    return set_error(B2Q_EINVAL, "b2q_gdn_step_dev: bad shape (n_k %d, n_v %d, d_v %d, kernel %d)", c.n_k_heads,
                     c.n_v_heads, c.d_v, c.conv_kernel);
  if (reinterpret_cast<uintptr_t>(ssm_state) % 16)
    return set_error(B2Q_EINVAL, "b2q_gdn_step_dev: ssm_state must be 16-byte aligned");
  const int channels = 2 * c.n_k_heads * c.d_k + c.n_v_heads * c.d_v;
  const int vdim = c.n_v_heads * c.d_v;
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : e->stream;
  cudaError_t err = cudaSuccess;
  if (e->ws_gdn_cap < (size_t)channels) {
    if (e->ws_gdn) {
      err = cudaStreamSynchronize(st);
      cudaFree(e->ws_gdn);
    }
    e->ws_gdn = nullptr;
    e->ws_gdn_cap = 0;
    if (err == cudaSuccess) err = cudaMalloc(&e->ws_gdn, sizeof(float) * (size_t)channels);
    if (err != cudaSuccess) return cuda_error(err, "b2q_gdn_step_dev: workspace");
    e->ws_gdn_cap = (size_t)channels;
  }
  // the recurrence runs token by token
  for (int t = 0; t < n_tokens && err == cudaSuccess; ++t) {
    launch_counted(e, 2);
    gdn_conv_kernel<<<(channels + 255) / 256, 256, 0, st>>>(qkv + (size_t)t * channels, conv_state, conv_w,
                                                            channels, c.conv_kernel, e->ws_gdn);
    gdn_head_kernel<<<c.n_v_heads, kGdnThreads, 0, st>>>(e->ws_gdn, ssm_state, z + (size_t)t * vdim,
                                                          alpha + (size_t)t * c.n_v_heads,
                                                          beta + (size_t)t * c.n_v_heads, ssm_a, dt_bias, ssm_norm,
                                                          c.n_k_heads, c.d_k, c.d_v, c.eps, y + (size_t)t * vdim);
    err = cudaGetLastError();
  }
  if (err != cudaSuccess) return cuda_error(err, "b2q_gdn_step_dev");
  return B2Q_OK;
}

uint64_t b2q_sampler_state(uint64_t seed) { return seed == 0 ? 0x853C49E6748FEA9Bull : seed; }

b2q_status b2q_sample_dev(b2q_engine* e, const float* logits_dev, int n, float temperature, float top_p,
                          uint64_t* rng_state, uint32_t* token, void* stream) {
  if (!e || !logits_dev || !rng_state || !token) return set_error(B2Q_EINVAL, "b2q_sample_dev: NULL argument");
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  return sample_core(e, logits_dev, n, temperature, top_p, rng_state, token,
                     stream ? (cudaStream_t)stream : e->stream);
}

b2q_status b2q_set_wait_limit_cycles(b2q_engine* e, long long cycles) {
  if (!e) return set_error(B2Q_EINVAL, "engine is NULL");
  if (cycles <= 0) cycles = kSpinLimitCycles;
  std::lock_guard<std::mutex> lk(e->mu);
  cudaSetDevice(e->device);
  cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_b2q_wait_limit, &cycles, sizeof cycles);
  if (err != cudaSuccess) return cuda_error(err, "b2q_set_wait_limit_cycles");
  return B2Q_OK;
}

b2q_status b2q_check_device_error(b2q_engine* e) {
  if (!e) return set_error(B2Q_EINVAL, "engine is NULL");
  cudaSetDevice(e->device);
  cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return cuda_error(err, "check_device_error: stream");
  int v = 0, zero = 0;
  err = cudaMemcpyFromSymbol(&v, g_b2q_device_error, sizeof v);
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_b2q_device_error, &zero, sizeof zero);
  if (err != cudaSuccess) return cuda_error(err, "check_device_error: symbol");
  if (v == 3) return set_error(B2Q_ECUDA, "a device-side layout or bounds check failed (b2q_debug_check_site)");
  if (v != 0) return set_error((b2q_status)v, "a device-side bounded wait gave up (code %d)", v);
  return B2Q_OK;
}

int b2q_debug_checks_enabled(void) { return kChecks ? 1 : 0; }

b2q_status b2q_debug_check_site(b2q_engine* e, int* site) {
  if (!e || !site) return set_error(B2Q_EINVAL, "b2q_debug_check_site: NULL argument");
  cudaSetDevice(e->device);
  cudaError_t err = cudaStreamSynchronize(e->stream);
  int zero = 0;
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(site, g_b2q_check_site, sizeof(int));
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_b2q_check_site, &zero, sizeof zero);
  if (err != cudaSuccess) return cuda_error(err, "b2q_debug_check_site");
  return B2Q_OK;
}

}  // extern "C"

#include "model_api.cuh"
#include "gguf_api.cuh"
