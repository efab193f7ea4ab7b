/*
 * b2q.h -- C ABI of the B200 GGUF dequant-GEMV decode library (libb2q.so).
 *
 * Drop-in boundary for the reference engine's GPU accelerator
 * (roblar658/huggingface-Local-LLM-UI, src/gpu.rs `CudaEngine`) and for its
 * model forward (src/inference.rs `StandardNativeEngine`).  Plain pointers,
 * sizes and status codes only; no C++ or framework types cross the ABI.
 *
 * Conventions
 *  - Every call returns a b2q_status; B2Q_OK is 0.  On failure
 *    b2q_last_error() returns a thread-local description.  There is no CPU
 *    fallback: the reference returned None and silently ran on the CPU
 *    (inference.rs:600-606); a caller of this ABI maps a non-OK status to
 *    its own error.
 *  - GGUF tensors are passed as their raw on-disk block bytes, `n` rows of
 *    `k` elements ([n][k] row-major, the order the reference's parser
 *    produces after reversing GGML's dims, inference.rs:403).  The library
 *    may repack blocks at upload; dequantised values stay bit-exact.
 *  - Activations are f32.  Entry points without a suffix take HOST pointers
 *    and return after the result is on the host, as the reference's
 *    synchronous memcpy path did.  `_dev` entry points take DEVICE pointers
 *    and a cudaStream_t (passed as void*) and are asynchronous.
 *  - The library's kernels let the next launch on their stream start early
 *    (programmatic dependent launch).  A caller's kernel launched right
 *    after a `_dev` call WITHOUT the programmatic-serialisation attribute
 *    waits for it as usual; one launched WITH it must call
 *    cudaGridDependencySynchronize() (griddepcontrol.wait) before it reads
 *    the call's outputs or writes its inputs.
 *  - One engine per CUDA device; handles are internally locked.
 */
#ifndef B2Q_H
#define B2Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B2Q_OK = 0,
  B2Q_EINVAL = 1,   /* bad dtype, shape, pointer or argument */
  B2Q_ENOMEM = 2,   /* device allocation failed */
  B2Q_ECUDA = 3,    /* CUDA runtime / kernel error */
  B2Q_ENCCL = 4,    /* NCCL error */
  B2Q_ETIMEOUT = 5, /* a bounded device-side wait gave up */
  B2Q_EUNSUP = 6    /* dtype or feature not supported */
} b2q_status;

/* GGML type ids (GgmlDType::from_u32, inference.rs:136-155). */
enum {
  B2Q_F32 = 0, B2Q_F16 = 1, B2Q_Q4_0 = 2, B2Q_Q8_0 = 8,
  B2Q_Q4_K = 12, B2Q_Q5_K = 13, B2Q_Q6_K = 14, B2Q_BF16 = 30
};

typedef struct b2q_engine b2q_engine; /* CudaEngine (gpu.rs:183-207) */
typedef struct b2q_weight b2q_weight; /* CudaWeightBuffer (gpu.rs:212-238) */
typedef struct b2q_model b2q_model;   /* StandardNativeEngine (inference.rs:2498-2510) */

/* Thread-local text of the last failure on this thread. */
const char* b2q_last_error(void);

/* Library version string. */
const char* b2q_version(void);

/* ---- engine ---------------------------------------------------------- */

/* Replaces CudaEngine::global / init_internal (gpu.rs:238-385): bind the
 * device, create the stream and workspace.  Kernels are compiled into the
 * library for sm_100a; nothing is JIT-loaded. */
b2q_status b2q_init(int device, b2q_engine** out);
b2q_status b2q_engine_destroy(b2q_engine* eng);

/* Device name and memory (the reference's device_name / cuMemGetInfo). */
b2q_status b2q_device_info(b2q_engine* eng, char* name, size_t name_len,
                           size_t* free_bytes, size_t* total_bytes);

/* Replaces CudaEngine::can_safely_alloc (gpu.rs:403-437): true (1) if
 * `bytes` more can be allocated while keeping `reserve_bytes` free. */
int b2q_can_alloc(b2q_engine* eng, size_t bytes, size_t reserve_bytes);

/* ---- weights --------------------------------------------------------- */

/* Replaces CudaEngine::try_upload_weight (gpu.rs:468-507): copy the raw GGUF
 * bytes of an [n][k] tensor (`len` must equal n * row_bytes) to the device,
 * repacked into the GEMV layout.  `bytes` may be a host or device pointer. */
b2q_status b2q_upload_weight(b2q_engine* eng, const void* bytes, size_t len,
                             int ggml_type, int64_t n, int64_t k, b2q_weight** out);

/* Drop for CudaWeightBuffer (gpu.rs:222-238). */
b2q_status b2q_weight_free(b2q_weight* w);

/* Device bytes held by a weight (equals the GGUF byte length). */
size_t b2q_weight_bytes(const b2q_weight* w);

/* ---- matvec entry points --------------------------------------------- */

/* Replaces CudaEngine::matmul_batched (gpu.rs:557-589) and the kernels
 * matmul_{q4k,q6k,q8_0,...} it launched (gpu.rs:510-555):
 * y[t][r] = sum_c dequant(W)[r][c] * x[t][c], x [m][k], y [m][n], f32.
 * m < 16: the bandwidth-bound GEMV; m >= 16: the tensor-core GEMM
 * (tcgen05, f16 hi/lo operand split, f32 accumulation). */
b2q_status b2q_matmul(b2q_engine* eng, const b2q_weight* w, const float* x, float* y,
                      int m, int n, int k);
b2q_status b2q_matmul_dev(b2q_engine* eng, const b2q_weight* w, const float* x_dev,
                          float* y_dev, int m, int n, int k, void* stream);

/* No counterpart in the reference.  y = W x for callers that must not
 * allocate device memory (a fixed memory pool, a real-time path that cannot
 * take an allocation's implicit synchronisation, a host that owns the
 * allocator): this entry point calls no cudaMalloc, cudaFree or allocating
 * library routine.  It always runs the GEMV path (the quantiser and the
 * bandwidth-bound GEMV, in passes of one or two tokens), so below 16 tokens
 * its output is bit-identical to b2q_matmul_dev's; from 16 tokens on,
 * b2q_matmul_dev uses the tensor cores instead, and the two agree within
 * the matvec tolerance (rel-L2 1e-3 of fp64) rather than bit for bit, while
 * this call re-streams the weights once per pass.  Its scratch (the
 * quantised activations) is a fixed array inside the library, about 0.6 MB
 * per GPU that loads the library, held until the process exits; calls with
 * m * round_up(k, 256) > 262144 are rejected with B2Q_EINVAL.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  Every call shares the
 * array: calls that overlap on the GPU (different streams, no ordering)
 * race and must be serialised by the caller.  x_dev / y_dev are device
 * pointers; asynchronous on `stream` (NULL: the engine's stream). */
b2q_status b2q_matmul_noalloc_dev(const b2q_weight* w, const float* x_dev, float* y_dev, int m, int n,
                                  int k, void* stream);

/* Replaces CudaEngine::matmul_group_same_input (gpu.rs:593-650): `count`
 * weights sharing the input x [m][k]; outputs are concatenated in order,
 * each as its own [m][n_i] block, into y_flat (gpu.rs:617-646). */
b2q_status b2q_matmul_group(b2q_engine* eng, const b2q_weight* const* ws, const int* ns,
                            int count, const float* x, int m, int k, float* y_flat);
b2q_status b2q_matmul_group_dev(b2q_engine* eng, const b2q_weight* const* ws, const int* ns,
                                int count, const float* x_dev, int m, int k, float* y_flat_dev,
                                void* stream);

/* Replaces CudaEngine::ffn_swiglu_fused (gpu.rs:657-734) and the swiglu_f32
 * kernel: y = W_down * (silu(W_gate * x) .* (W_up * x)); x [m][n_embd],
 * y [m][n_embd]. */
b2q_status b2q_ffn_swiglu(b2q_engine* eng, const b2q_weight* gate, const b2q_weight* up,
                          const b2q_weight* down, const float* x, int m, int n_embd,
                          int ffn_inter, float* y);
b2q_status b2q_ffn_swiglu_dev(b2q_engine* eng, const b2q_weight* gate, const b2q_weight* up,
                              const b2q_weight* down, const float* x_dev, int m, int n_embd,
                              int ffn_inter, float* y_dev, void* stream);

/* Replaces dequantize_slice (inference.rs:1347-1474) on the device: raw GGUF
 * bytes (device pointer) of `n_elems` elements to f32, bit-exact. */
b2q_status b2q_dequantize_dev(b2q_engine* eng, const void* raw_dev, int ggml_type,
                              int64_t n_elems, float* out_dev, void* stream);

/* ---- whole model (keeps activations and the KV cache on the device) ---- */

typedef struct {
  int n_layers;      /* {arch}.block_count */
  int n_embd;        /* {arch}.embedding_length */
  int n_heads;       /* {arch}.attention.head_count */
  int n_kv_heads;    /* {arch}.attention.head_count_kv */
  int head_dim;      /* {arch}.attention.key_length */
  int n_ff;          /* rows of ffn_gate */
  int n_vocab;       /* rows of output / token_embd */
  float rms_eps;     /* {arch}.attention.layer_norm_rms_epsilon, default 1e-5 */
  float rope_theta;  /* {arch}.rope.freq_base, default 1e4 */
  int max_seq;       /* KV capacity in tokens; positions clamp at 8191 for RoPE */
  int tp_rank;       /* tensor-parallel rank of this process (0 for 1 GPU) */
  int tp_size;       /* tensor-parallel world size (1 for 1 GPU) */
  int no_graph;      /* single-token steps: 0 (default) one persistent kernel per
                        token, on one GPU or across the tensor-parallel ranks
                        (the captured graph where the model does not fit it);
                        1 the per-layer kernels launched eagerly; 2 the
                        captured CUDA graph of those kernels.  The three give
                        bit-identical logits. */
} b2q_model_config;

/* Unique id for NCCL communicator setup (ncclGetUniqueId); rank 0 creates
 * it and the caller broadcasts the 128 bytes to the other ranks. */
b2q_status b2q_tp_unique_id(unsigned char out[128]);

/* Host-side bound (milliseconds, default 120000) of the NCCL communicator
 * set-up in b2q_model_create under tensor parallelism, and of any NCCL call
 * that answers "in progress".  Communicators are created non-blocking; when
 * the other ranks do not join in time the set-up is aborted
 * (ncclCommAbort) and b2q_model_create returns B2Q_ETIMEOUT instead of
 * hanging.  No counterpart in the reference (it had no multi-GPU path). */
b2q_status b2q_set_tp_init_timeout_ms(int ms);

/* Replaces StandardNativeEngine::from_gguf (inference.rs:2513-2620):
 * create an empty model; tensors are then added by GGUF name. */
b2q_status b2q_model_create(b2q_engine* eng, const b2q_model_config* cfg,
                            const unsigned char* tp_unique_id, b2q_model** out);

/* Add one tensor by its GGUF name ("token_embd.weight", "output_norm.weight",
 * "output.weight", "blk.{i}.attn_norm.weight", "blk.{i}.attn_q.weight",
 * ".attn_k", ".attn_v", ".attn_output", ".ffn_norm", ".ffn_gate", ".ffn_up",
 * ".ffn_down", optional ".attn_{q,k,v}.bias").  dims are [outer.., inner]
 * as the reference stores them (inference.rs:403).  Under tensor
 * parallelism each rank passes the FULL tensor; the library keeps its
 * shard.  `bytes` is a host pointer. */
b2q_status b2q_model_set_tensor(b2q_model* m, const char* name, int ggml_type,
                                const int64_t* dims, int n_dims, const void* bytes, size_t len);

/* Same, but the caller passes only rows [row_begin, row_end) of an [n][k]
 * tensor (its own shard, for sharded loading of large models). */
b2q_status b2q_model_set_tensor_rows(b2q_model* m, const char* name, int ggml_type,
                                     const int64_t* dims, int n_dims, int64_t row_begin,
                                     int64_t row_end, const void* bytes, size_t len);

/* Row range of an [n][...] tensor this rank must supply for `name`. */
b2q_status b2q_model_shard_rows(b2q_model* m, const char* name, int64_t n,
                                int64_t* row_begin, int64_t* row_end);

/* The same range from a configuration alone (cfg->tp_rank of cfg->tp_size),
   without a device: attn_q/k/v are split by whole heads (rank r owns KV heads
   [r*KV/P, (r+1)*KV/P) and their query heads), ffn_gate/up and output by
   contiguous rows; attn_output and ffn_down are split by columns instead
   (b2q_tp_shard_cols), so every rank supplies all their rows; norms and
   token_embd are replicated.  Loader-side counterpart of the reference's
   per-tensor placement in from_gguf (inference.rs:2605-2616), which has no
   tensor parallelism. */
b2q_status b2q_tp_shard_rows(const b2q_model_config* cfg, const char* name, int64_t n,
                             int64_t* row_begin, int64_t* row_end);

/* Columns [col_begin, col_end) of an [n][k] tensor this rank keeps: for
   attn_output the columns of its query heads, for ffn_down those of its
   ffn_gate/up rows (so attention and SwiGLU outputs stay on the rank and the
   two projections produce partial sums that the ranks add in rank order);
   [0, k) for every other tensor.  The library cuts the columns itself from
   the full rows passed to b2q_model_set_tensor(_rows). */
b2q_status b2q_tp_shard_cols(const b2q_model_config* cfg, const char* name, int64_t k,
                             int64_t* col_begin, int64_t* col_end);

/* Validate that every tensor is present, allocate the KV cache and build
 * the decode graphs. */
b2q_status b2q_model_finalize(b2q_model* m);

/* Replaces StandardNativeEngine::forward (inference.rs:2695-2860): run
 * `n_tokens` tokens starting at `start_pos`, appending to the KV cache, and
 * write the logits of the LAST position ([n_vocab] f32) to `logits` (host
 * pointer, may be NULL).  If `argmax` is non-NULL the greedy next token
 * (SelfMadeSampler at temperature <= 1e-5, inference.rs:1620-1630) is
 * written there too.  Returns B2Q_ETIMEOUT (and clears the device error
 * word) when a bounded device-side wait gave up during the step: its outputs
 * are then invalid.  On one GPU the persistent kernel's synchronisation
 * state is re-armed before returning, so the step can simply be repeated;
 * under tensor parallelism every rank must call b2q_clear_state, followed by
 * a host barrier across the ranks, first.  (The reference fell back to the
 * CPU on any GPU failure, inference.rs:600-606; there is no fallback here.) */
b2q_status b2q_forward(b2q_model* m, const uint32_t* tokens, int n_tokens, int start_pos,
                       float* logits, uint32_t* argmax);

/* Device-pointer form: tokens_dev / logits_dev / argmax_dev are device
 * pointers (any may be NULL except tokens_dev); asynchronous on `stream`
 * (NULL: the model's own stream).  It does not synchronise, so it cannot see
 * a bounded wait that gave up: call b2q_check_device_error to learn that.
 * Stream capture: when `stream` is capturing, a single-token step runs the
 * per-kernel path (no persistent kernel, no nested graph), because the
 * persistent kernel's barrier bases and hand-off tags are host counters
 * baked into each launch and a replayed launch would reuse them. */
b2q_status b2q_forward_dev(b2q_model* m, const uint32_t* tokens_dev, int n_tokens,
                           int start_pos, float* logits_dev, uint32_t* argmax_dev, void* stream);

/* The forward followed by SelfMadeSampler::sample (inference.rs:1619-1681)
 * on the device: temperature <= 1e-5 is the greedy first maximum; otherwise
 * the candidates within 14 * temperature of the max logit, weighed
 * exp((v - max) / temperature), the smallest set of largest weights whose
 * mass reaches top_p of the total, and a draw from it.  *rng_state is the
 * sampler's xorshift64 state (b2q_sampler_state(seed) to start), advanced
 * by one draw when the sampler draws; the next token goes to *token.  The
 * token equals the reference's except when the draw falls within rounding
 * of a boundary between two candidates (device exp, tree sums).  Under
 * tensor parallelism every rank calls it with the same state. */
b2q_status b2q_forward_sample(b2q_model* m, const uint32_t* tokens, int n_tokens, int start_pos,
                              float temperature, float top_p, uint64_t* rng_state, uint32_t* token);

/* Initial sampler state of SelfMadeSampler::new(seed) (inference.rs:1601-1607). */
uint64_t b2q_sampler_state(uint64_t seed);

/* The sampling step alone, on logits already on the device ([n] f32). */
b2q_status b2q_sample_dev(b2q_engine* eng, const float* logits_dev, int n, float temperature, float top_p,
                          uint64_t* rng_state, uint32_t* token, void* stream);

/* ---- Gated DeltaNet state update (the reference's Qwen3.5 hybrid model) ---- */
typedef struct {
  int n_k_heads;   /* qwen35.ssm.group_count: q/k heads */
  int n_v_heads;   /* qwen35.ssm.time_step_rank: value heads (a multiple of n_k_heads) */
  int d_k;         /* qwen35.ssm.state_size (128) */
  int d_v;         /* qwen35.ssm.inner_size / n_v_heads (<= 512) */
  int conv_kernel; /* qwen35.ssm.conv_kernel */
  float eps;       /* the model's RMS epsilon (also the L2-norm epsilon) */
} b2q_gdn_config;

/* The Gated DeltaNet mixer core of Qwen35Mixer::GatedDeltaNet
 * (inference.rs:2281-2374, ssm_head_step_avx2 :1535-1583) for n_tokens
 * tokens in order, on the device: causal convolution with state and SiLU
 * over the attn_qkv output, L2 norm of q and k per head, the per-head state
 * update S = g S + ((v - g S k) beta) k^T with o = S q / sqrt(d_k), then
 * RMS norm * ssm_norm * silu(z).  Inputs per token: qkv [2 n_k d_k + n_v d_v],
 * z [n_v d_v], alpha / beta [n_v] (the quad projection's outputs, token-major);
 * weights conv_w [channels][conv_kernel], ssm_a / dt_bias [n_v], ssm_norm
 * [d_v]; state conv_state [channels][conv_kernel - 1] and ssm_state
 * [n_v][d_v][d_k] (16-byte aligned) are read and updated; y [n_tokens][n_v d_v].
 * All device pointers; asynchronous on `stream`. */
b2q_status b2q_gdn_step_dev(b2q_engine* eng, const b2q_gdn_config* cfg, int n_tokens, const float* qkv,
                            const float* z, const float* alpha, const float* beta, const float* conv_w,
                            const float* ssm_a, const float* dt_bias, const float* ssm_norm, float* conv_state,
                            float* ssm_state, float* y, void* stream);

/* Replaces StandardNativeEngine::clear_state (inference.rs:2688-2693).
 * Also re-arms the persistent decode kernel's barrier counters and all-rank
 * epoch slots (tensor parallelism: every rank calls it, then the ranks meet
 * at a host barrier before the next step). */
b2q_status b2q_clear_state(b2q_model* m);

/* Benchmark set-up, no counterpart in the reference: writes seeded synthetic
 * K and V rows (uniform in [-scale, scale), rounded to f16) for positions
 * [start, start + n) of every layer's KV cache, for this rank's KV heads, so
 * that single-token steps can be timed at a long context without a prompt
 * pass.  The values depend only on (seed, layer, K or V, global KV head,
 * position, element), so tensor-parallel ranks hold the rows one GPU would.
 * Synchronous. */
b2q_status b2q_model_fill_kv(b2q_model* m, int start, int n, uint64_t seed, float scale);

/* Test hook, no counterpart in the reference: advances the model's
 * persistent-kernel launch sequence on the host without launching, which is
 * what a launch skipped by a peer looks like from this GPU: the next step's
 * barrier targets lie beyond the arrivals it will see, so its bounded waits
 * give up and the blocking forward returns B2Q_ETIMEOUT.  Used to test the
 * failure path without faulting or hanging a GPU (lower the wait limit
 * first with b2q_set_wait_limit_cycles). */
b2q_status b2q_model_debug_desync(b2q_model* m);

/* ---- GGUF files (GgufModelFile, inference.rs:235-510) ----
 * A read-only POSIX mapping of the file, parsed as GgufModelFile::open
 * does (inference.rs:343-446): versions 1..3, metadata types 0..12, dims
 * reversed to [outer.., inner], data section aligned to general.alignment
 * (default 32), every tensor checked to end inside the file; a tensor
 * whose element count overflows 64 bits is rejected.  Names and
 * string values returned below point into the handle and stay valid until
 * b2q_gguf_close.  Errors are B2Q_EINVAL with the reason in
 * b2q_last_error() (the reference's anyhow messages). */
typedef struct b2q_gguf b2q_gguf;

/* GgufModelFile::open (inference.rs:343-446). */
b2q_status b2q_gguf_open(const char* path, b2q_gguf** out);
/* Drop of GgufModelFile: unmaps the file. */
b2q_status b2q_gguf_close(b2q_gguf* g);
int b2q_gguf_version(const b2q_gguf* g);
int64_t b2q_gguf_n_tensors(const b2q_gguf* g);
/* Metadata keys in file order; value_type is the GGUF value type (0..12). */
int64_t b2q_gguf_n_kv(const b2q_gguf* g);
b2q_status b2q_gguf_kv_key(const b2q_gguf* g, int64_t index, const char** key, int* value_type);
/* GgufTensorDesc (inference.rs:236-244) of tensor `index` (file order):
 * dims has room for 8 entries, [outer.., inner]; abs_offset is
 * data_offset + the tensor's relative offset; byte_len is
 * elements / block_size * type_size.  Any pointer may be NULL. */
b2q_status b2q_gguf_tensor_info(const b2q_gguf* g, int64_t index, const char** name, int* ggml_type,
                                int* n_dims, int64_t* dims, uint64_t* abs_offset, uint64_t* byte_len);
/* Index of tensor `name`; B2Q_EINVAL "tensor '...' not found in GGUF". */
b2q_status b2q_gguf_find_tensor(const b2q_gguf* g, const char* name, int64_t* index);
/* Host pointer to the tensor's bytes inside the mapping (NULL if out of range). */
const void* b2q_gguf_tensor_data(const b2q_gguf* g, int64_t index);
/* GgufModelFile::get_usize / get_f32 (inference.rs:447-460) with
 * GgufValue::as_usize / as_f32 (:203-223): u8/u16/u32/u64 and non-negative
 * i32/i64 read as integers; f32, f64, u32 and i32 read as floats. */
b2q_status b2q_gguf_get_usize(const b2q_gguf* g, const char* key, uint64_t* out);
b2q_status b2q_gguf_get_f32(const b2q_gguf* g, const char* key, float* out);
/* A string value (not NUL-terminated): pointer into the mapping and length. */
b2q_status b2q_gguf_get_str(const b2q_gguf* g, const char* key, const char** s, size_t* len);

/* Hyperparameters of StandardNativeEngine::from_gguf (inference.rs:2513-2537):
 * "{arch}." keys, or "llama." when "{arch}.block_count" is absent
 * (arch NULL means "llama"); head_count_kv defaults to head_count,
 * key_length to embedding_length / head_count, the RMS epsilon to 1e-5,
 * rope.freq_base to 10000; n_ff and n_vocab are the row counts of
 * blk.0.ffn_gate.weight and token_embd.weight.  Fills those fields of
 * *cfg and leaves max_seq, tp_rank, tp_size and no_graph as the caller set
 * them. */
b2q_status b2q_gguf_llama_config(const b2q_gguf* g, const char* arch, b2q_model_config* cfg);

/* Tensor loading of from_gguf (inference.rs:2551-2587) into a model made by
 * b2q_model_create: token_embd, output_norm, output (tied to token_embd when
 * the file has none), and for every block attn_norm, attn_q/k/v, the
 * optional attn_{q,k,v}.bias, attn_output, ffn_norm, ffn_gate/up/down.  Each
 * rank uploads only its tensor-parallel rows, read from the mapping;
 * 1-D F16/BF16 tensors are widened to F32 on the host.  Call
 * b2q_model_finalize afterwards. */
b2q_status b2q_model_load_gguf(b2q_model* m, const b2q_gguf* g);

/* Device bytes held by the model's weights on this rank. */
size_t b2q_model_weight_bytes(const b2q_model* m);

/* How a finalized model runs a single-token step: 0 = the persistent decode
 * kernel, 1 = eager per-kernel launches, 2 = the captured per-kernel graph
 * (-1 before b2q_model_finalize). */
int b2q_model_step_path(const b2q_model* m);

b2q_status b2q_model_destroy(b2q_model* m);

/* Kernel timing for benchmarks: quantise x (device, [k] f32) once, then
 * launch the GEMV of each of the `count` weights (same k) `reps` times in
 * turn on `stream`, writing y to scratch, and return the average device
 * time of one GEMV launch in *avg_ms (CUDA events on `stream`).  Rotating
 * through weights that together exceed the L2 cache times HBM streaming.
 * chained != 0: each launch is a programmatic dependent launch of the
 * previous one, as the per-kernel decode path chains its GEMVs, so a
 * launch's weight stream starts while the previous launch drains; 0: plain
 * back-to-back launches (each launch's ring fill exposed). */
b2q_status b2q_time_gemv(b2q_engine* eng, const b2q_weight* const* ws, int count,
                         const float* x_dev, int k, int reps, void* stream, float* avg_ms, int chained);

/* Launch statistics: number of library kernels launched so far on this
 * engine (graph replays count every kernel node). */
uint64_t b2q_kernel_launch_count(b2q_engine* eng);

/* Read and clear the device-side error word (B2Q_ETIMEOUT when a bounded
 * wait gave up; B2Q_ECUDA when the persistent decode kernel found its shared
 * memory laid out otherwise than planned, or, in the debug-bounds build, a
 * bounds check failed); synchronises the engine's stream. */
b2q_status b2q_check_device_error(b2q_engine* eng);

/* Debug-bounds build (libb2q_checks.so, compiled with -DB2Q_CHECKS): 1 when
 * this library has the kernels' index and layout checks compiled in, else 0.
 * No counterpart in the reference (its kernels are a PTX image, gpu.rs:6,301);
 * it stands in for a memory checker. */
int b2q_debug_checks_enabled(void);

/* Site of the first failed check since the last call (0: none; 1 ring stage,
 * 2 attention tile rows, 3 current token row, 4 staged input size, 5
 * tagged-vector index, 6 tensor-parallel slot, 7 attention partial index, 8
 * tensor-core stage plan, 9 standalone GEMV plan), then cleared.  Always 0
 * in the regular build.  Synchronises the engine's stream. */
b2q_status b2q_debug_check_site(b2q_engine* eng, int* site);

/* Upper bound of every device-side wait of this engine's GPU (mbarriers,
 * grid and all-rank barriers, tagged hand-offs), in SM clock cycles;
 * cycles <= 0 restores the default 4e9 (~2 s).  A wait that reaches it sets
 * the device error word and lets its kernel finish.  No counterpart in the
 * reference, which had no device-side waits of its own. */
b2q_status b2q_set_wait_limit_cycles(b2q_engine* eng, long long cycles);

#ifdef __cplusplus
}
#endif

#endif /* B2Q_H */
