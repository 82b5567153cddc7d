/*
 * ib_cuda.h -- C ABI of the B200 (sm_100a) backend for inference.cpp's
 * quantized-weight path.
 *
 * This library replaces the reference's CUDA backend loader
 * (src/ops/cuda_backend.cpp: dlopen of libcuda.so.1, cuModuleLoadData of
 * clang-built sm_75 PTX, cuLaunchKernel by name) with kernels compiled for
 * sm_100a and called through plain C functions.  Every function returns an int
 * status (IB_OK on success); on failure ib_last_error() gives a message in the
 * reference's style ("CUDA: <what> failed: <reason>").  All pointers named
 * `dev`/device below are device pointers; `host` pointers are host memory.
 * `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream,
 * which is what the reference launches on, cuda_backend.cpp:180-181).
 *
 * Tensor layout matches the reference after its dimension reversal
 * (src/models/transformer.cpp:160-161,200): a weight is row-major [rows, cols]
 * with rows = output features; a GGUF block-quantised weight is the file's
 * bytes unchanged, i.e. rows * (cols / block_elems) consecutive blocks.
 */
#ifndef IB_CUDA_H
#define IB_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define IB_OK 0
#define IB_ERR_INVALID 1     /* bad argument (null pointer, size, type) */
#define IB_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define IB_ERR_UNSUPPORTED 3 /* type/shape not supported by this path */
#define IB_ERR_OOM 4         /* device memory exhausted */
#define IB_ERR_TIMEOUT 5     /* a bounded wait expired */
#define IB_ERR_COMM 6        /* collective / communicator failure */

/* ---- GGUF tensor types (reference include/core/tensor.hpp:16-37) ------------ */
#define IB_TYPE_F32 0
#define IB_TYPE_F16 1
#define IB_TYPE_Q4_0 2
#define IB_TYPE_Q5_0 6
#define IB_TYPE_Q5_1 7
#define IB_TYPE_Q8_0 8
#define IB_TYPE_Q4_K 12
#define IB_TYPE_Q6_K 14
#define IB_TYPE_I16 17
/* Sized by the reference (include/core/tensor.hpp:204-262) but not decoded by it
 * (src/gguf/quantization.cpp:201-204 throw); here decoded from the published GGUF
 * layouts by ib_dequant_f32 / ib_dequant_i16 / ib_embedding_q / ib_gemv_q / ib_gemm_q
 * and usable as model weights (the per-operation decode step). */
#define IB_TYPE_Q4_1 3
#define IB_TYPE_Q2_K 10
#define IB_TYPE_Q3_K 11
#define IB_TYPE_Q5_K 13

/* Message of the last failed call on this thread ("" if none). */
const char* ib_last_error(void);

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int ib_version(void);

/* Elements and bytes per block of a type (reference type_nbytes_per_block /
 * block_size, include/core/tensor.hpp:204-262). */
int ib_type_info(int type, int64_t* block_elems, int64_t* block_bytes);

/* ---- lifecycle (replaces inference::cuda::available, device_name, total_memory,
 *      free_memory, sync, shutdown: include/ops/cuda_backend.hpp:17-22) ------- */
int ib_init(int device);                        /* select device; idempotent */
int ib_available(void);                         /* 1 if a usable sm_100 device exists, else 0 */
int ib_device_name(char* buf, size_t len);
int ib_memory_info(size_t* free_bytes, size_t* total_bytes);
int ib_sync(void);                              /* device-wide synchronise */
/* Every wait inside a pipelined kernel is bounded; an expired wait makes the
 * kernel record a code and return early instead of hanging.  This reads and
 * clears that record on the current device: IB_ERR_TIMEOUT (and *code != 0)
 * means results since the previous check are invalid. */
int ib_check_fault(int* code);
int ib_shutdown(void);                          /* no-op: buffers stay valid to exit */

/* ---- memory (replaces alloc, release, upload, download:
 *      include/ops/cuda_backend.hpp:25-28; the reference copies synchronously) -- */
int ib_alloc(void** dev, size_t bytes);
int ib_free(void* dev);
int ib_upload(void* dev, const void* host, size_t bytes, void* stream);
int ib_download(void* host, const void* dev, size_t bytes, void* stream);
int ib_memset(void* dev, int value, size_t bytes, void* stream);

/* ---- block-quantised weights (the hot path) -------------------------------- */

/* Dequantise a packed [rows, cols] tensor to FP32, bit-exact with the reference
 * dequantize() (src/gguf/quantization.cpp:250-267; Q4_0 :33, Q8_0 :59, Q5_0 :83,
 * Q5_1 :112, Q4_K :161, Q6_K :211).  F16 and F32 inputs are converted/copied as
 * load_tensor does (src/models/transformer.cpp:176-199). */
int ib_dequant_f32(int type, const void* dev_blocks, float* dev_out, int64_t rows,
                   int64_t cols, void* stream);

/* Dequantise and requantise each row to symmetric INT16 with one FP32 scale per
 * row, bit-exact with make_weight (src/models/transformer.cpp:208-251) and
 * quantize_i16 (src/models/model_cuda.cpp:62-99). */
int ib_dequant_i16(int type, const void* dev_blocks, int16_t* dev_q, float* dev_row_scale,
                   int64_t rows, int64_t cols, void* stream);

/* Fused dequant + GEMV on packed blocks: y[r] = sum_c W[r, c] * x[c], FP32
 * activations and accumulation.  Replaces gemv / gemv_i16
 * (include/ops/cuda_backend.hpp:31-34; kernels src/ops/cuda_kernels.cu:62-95) for
 * weights kept in GGUF form.  W is never expanded in memory. */
int ib_gemv_q(int type, const void* dev_W, const float* dev_x, float* dev_y, int64_t rows,
              int64_t cols, void* stream);

/* ib_gemv_q without any device allocation.  No counterpart in the reference: it
 * exists for callers that must not allocate device memory during a call (a host
 * whose allocator is owned by another runtime, a memory-budgeted process).  The
 * activation-limb scratch is a static device array of 144 KiB, which caps cols at
 * IB_NOALLOC_MAX_COLS; larger cols return IB_ERR_INVALID with a message naming the
 * limit.  The first call on each device resolves that array's address and prepares
 * the kernels of all six formats (set-up); make it before any stream capture.  The
 * resolved address belongs to the device's primary context: do not call this entry
 * point again after cudaDeviceReset (or any other teardown of that context) in the
 * same process.  The scratch needs no zeroing.  Calls overlapping in time on one
 * device share the scratch and race: order them on one stream.  The weight pointer
 * must meet the format's alignment (16 bytes for Q4_K, 8 for Q5_1, 2 otherwise) and
 * x 16 bytes; all six block formats are accepted. */
#define IB_NOALLOC_MAX_COLS 32768
int ib_gemv_q_noalloc(int type, const void* dev_W, const float* dev_x, float* dev_y,
                      int64_t rows, int64_t cols, void* stream);

/* ib_gemv_q in two steps, for an activation shared by several GEMVs: the exact int8
 * limb split of x ("limb slab", ib_slab_bytes bytes, 16-byte aligned) is computed once
 * by ib_limb_slab for the weight family of `type` (K-quants or 32-element blocks), and
 * ib_gemv_q_slab runs the GEMV kernel on it.  No counterpart in the reference (its
 * GEMV takes FP32 x directly). */
int ib_slab_bytes(int type, int64_t cols, size_t* bytes);
int ib_limb_slab(int type, const float* dev_x, int64_t cols, void* dev_slab, void* stream);
int ib_gemv_q_slab(int type, const void* dev_W, const void* dev_slab, float* dev_y, int64_t rows,
                   int64_t cols, void* stream);
/* ib_gemv_q_slab launched as a link of a chain (programmatic dependent launch): it may
 * start, and stream its weights, while the previous kernel on the stream still runs;
 * it reads the slab and writes y only after that kernel has completed.  For chains
 * whose weights no earlier kernel on the stream writes (the decode step's case). */
int ib_gemv_q_slab_chained(int type, const void* dev_W, const void* dev_slab, float* dev_y,
                           int64_t rows, int64_t cols, void* stream);

/* Batched product on packed blocks: Y[T, rows] = X[T, cols] @ W^T.  Replaces
 * gemm / gemm_i16 (include/ops/cuda_backend.hpp:35-38; kernels
 * src/ops/cuda_kernels.cu:279-346). */
int ib_gemm_q(int type, const void* dev_W, const float* dev_X, float* dev_Y, int64_t T,
              int64_t rows, int64_t cols, void* stream);
/* Which kernel ib_gemm_q runs (process-wide).  Both tensor-core kernels use tcgen05 with
 * FP32 accumulation in tensor memory and operands as FP16 hi/lo pairs:
 *   0  automatic (default): for T >= 128 the packed weights are decoded once into FP16
 *      planes and a TMA-fed kernel (128 x 256 tiles) multiplies them; shorter prompts
 *      decode each weight tile inside the kernel (128 x 128 tiles); shapes neither takes
 *      (cols % 64 != 0) run on CUDA cores
 *   1  CUDA-core FP32 tiles
 *   2  the in-kernel-decode tensor-core kernel where it applies
 *   3  the planes kernel where it applies
 * No counterpart in the reference. */
int ib_gemm_set_path(int path);
/* Prepared weights for repeated prompt GEMMs: the packed [rows, cols] weights decoded
 * once (bit-exact values) into FP16 hi/lo planes of ib_gemm_planes_bytes(rows, cols)
 * bytes (4 per weight) at a 16-byte aligned dev_planes, then Y[T, rows] = X Wᵀ on them
 * with the tcgen05 kernel of ib_gemm_q's automatic path (same result bit for bit, without
 * the per-call decoding).  cols % 32 == 0. */
size_t ib_gemm_planes_bytes(int64_t rows, int64_t cols);
int ib_gemm_prepare_planes(int type, const void* dev_W, int64_t rows, int64_t cols,
                           void* dev_planes, void* stream);
int ib_gemm_planes(const void* dev_planes, const float* dev_X, float* dev_Y, int64_t T,
                   int64_t rows, int64_t cols, void* stream);

/* Embedding gather with dequantisation: out[t, :] = dequant(table[ids[t], :]).
 * Replaces embedding / embedding_batch (include/ops/cuda_backend.hpp:44-50) for a
 * packed table; ids outside [0, vocab) read row 0 as Model::forward does
 * (src/models/model.cpp:259). */
int ib_embedding_q(int type, const void* dev_table, const int32_t* dev_ids, float* dev_out,
                   int T, int64_t vocab, int64_t dim, void* stream);

/* ---- FP32 / INT16 operators with the reference's argument meaning
 *      (include/ops/cuda_backend.hpp:31-64; all tensors FP32 row-major) ------- */
int ib_gemv(const float* W, const float* x, float* y, int M, int N, void* stream);
int ib_gemv_i16(const int16_t* W, const float* row_scale, const float* x, float* y, int M,
                int N, void* stream);
int ib_gemm(const float* W, const float* X, float* Y, int T, int M, int K, void* stream);
int ib_gemm_i16(const int16_t* W, const float* row_scale, const float* X, float* Y, int T,
                int M, int K, void* stream);
int ib_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps,
               void* stream);
int ib_silu(float* x, int n, void* stream);
int ib_mul(float* a, const float* b, int n, void* stream);
int ib_add(float* a, const float* b, int n, void* stream);
int ib_embedding(const float* table, int id, float* out, int dim, void* stream);
int ib_embedding_i16(const int16_t* table, const float* row_scale, int id, float* out,
                     int dim, void* stream);
int ib_embedding_batch(const float* table, const int32_t* ids, float* out, int T, int dim,
                       void* stream);
int ib_embedding_batch_i16(const int16_t* table, const float* row_scale, const int32_t* ids,
                           float* out, int T, int dim, void* stream);
int ib_kv_write(float* kc, float* vc, const float* k, const float* v, int n_heads,
                int head_dim, int max_seq, int pos, void* stream);
int ib_kv_write_batch(float* kc, float* vc, const float* k, const float* v, int n_heads,
                      int head_dim, int max_seq, int start, int T, void* stream);
int ib_rope(float* q, float* k, const float* table, int n_heads, int n_kv_heads,
            int head_dim, int pos, void* stream);
int ib_rope_batch(float* q, float* k, const float* table, int n_heads, int n_kv_heads,
                  int head_dim, int start, int T, void* stream);
int ib_attention(const float* q, const float* kc, const float* vc, float* out, int n_heads,
                 int n_kv_heads, int head_dim, int max_seq, int pos, float scale,
                 void* stream);
int ib_attention_batch(const float* q, const float* kc, const float* vc, float* out,
                       int n_heads, int n_kv_heads, int head_dim, int max_seq, int start,
                       int T, float scale, void* stream);

/* Decode attention as the native runner's decode step runs it: one kernel of
 * (kv head, split) CTAs whose last CTA per kv head combines the splits, with the
 * position read from device memory (*pos_dev) so the call can sit in a CUDA graph.
 * Same result contract as ib_attention (reference attention_kernel,
 * src/ops/cuda_kernels.cu:216-267).  Needs head_dim % 4 == 0, head_dim <= 128,
 * n_heads / n_kv_heads <= 8 and 16-byte aligned q, kc, vc, out.  part: scratch of
 * ib_attention_split_part_bytes(n_heads, head_dim) bytes; counters: n_kv_heads
 * int32 that are zero on entry and are left at zero. */
size_t ib_attention_split_part_bytes(int n_heads, int head_dim);
int ib_attention_split(const float* q, const float* kc, const float* vc, float* out,
                       int n_heads, int n_kv_heads, int head_dim, int max_seq,
                       const int32_t* pos_dev, float scale, float* part, int32_t* counters,
                       void* stream);

/* Index of the first maximum of x[0..n) (reference sample_argmax,
 * src/ops/ops.cpp:424-438), written to *dev_out. */
int ib_argmax(const float* x, int n, int32_t* dev_out, void* stream);

/* ---- native Llama runner on packed weights ----------------------------------
 * Replaces the reference's GPU model driver (src/models/model_cuda.cpp:
 * upload_weights :138-212, prefill :293-368, forward_token :372-407,
 * generate_cuda :442-495; API include/models/cuda_model.hpp:9-32).  Weights
 * stay in GGUF block form in HBM (precision NATIVE), or are converted on the
 * GPU to the reference's symmetric INT16 (INT16, --gpu-precision int16) or to
 * FP32 (FP32, --gpu-precision fp32).  Decoding is greedy (temperature 0,
 * repetition penalty 1), the argmax runs on the device. */
#define IB_PRECISION_NATIVE 0
#define IB_PRECISION_INT16 1
#define IB_PRECISION_FP32 2

typedef struct {
    int32_t n_layers, dim, n_heads, n_kv_heads, ffn, vocab, max_seq;
    float rope_theta, rms_eps;
    int32_t precision;
} ib_model_config;

/* GenerationStats (include/models/cuda_model.hpp:12-17). */
typedef struct {
    double init_ms, prefill_ms, decode_ms;
    int32_t generated;
} ib_generation_stats;

int ib_model_create(const ib_model_config* cfg, int device, void** model);
/* Tensor by its GGUF name ("token_embd.weight", "blk.3.attn_q.weight", ...),
 * shape [rows, cols] (rows = output features), data in host or device memory. */
int ib_model_set_tensor(void* model, const char* gguf_name, int type, int64_t rows,
                        int64_t cols, const void* data, int data_on_device);
/* Checks every tensor is set, allocates the FP32 KV cache and activations,
 * builds the RoPE table (VRAM preflight as model_cuda.cpp:243-252). */
int ib_model_finalize(void* model);
/* Reads a GGUF file (metadata as src/models/transformer.cpp:139-154) and uploads
 * its tensors unchanged; max_seq <= 0 takes llama.context_length. */
int ib_model_load_gguf(const char* path, int precision, int device, int max_seq, void** model);
int ib_model_free(void* model);
/* Batched prompt prefill at positions start..start+T-1 (fills the KV cache);
 * logits of the last position to host_logits (may be NULL), greedy id to *next. */
int ib_model_prefill(void* model, const int32_t* host_ids, int T, int start,
                     float* host_logits, int32_t* next);
/* One decode step of `token` at `pos`; logits (optional) and greedy next id. */
int ib_model_decode(void* model, int32_t token, int pos, float* host_logits, int32_t* next);
/* Greedy generation: out = prompt + up to max_tokens ids (stops at eos_token_id
 * when >= 0 or at the context end); *n_out = ids written. */
int ib_model_generate(void* model, const int32_t* prompt, int n_prompt, int max_tokens,
                      int32_t eos_token_id, int32_t* out, int* n_out, ib_generation_stats* stats);
/* n_steps greedy steps on the device from `token` at `pos`, each argmax fed back
 * as the next input without a host round trip; ids to host_tokens[0..n_steps). */
int ib_model_decode_loop(void* model, int32_t token, int pos, int n_steps, int32_t* host_tokens);
/* Capture the decode step in a CUDA graph (default on) or launch it directly. */
int ib_model_set_graph(void* model, int enabled);
/* Fused decode kernels (default on): per layer one QKV GEMV with RMSNorm, RoPE and
 * the KV write, attention, one wo GEMV with the residual add, one gate+up GEMV with
 * SwiGLU and one down GEMV with the residual add, chained by programmatic dependent
 * launch.  Used only when every weight's format and shape has a fused kernel. */
int ib_model_set_fused(void* model, int enabled);
/* *fused = 1 when decode steps run on the fused kernels (either decode path below). */
int ib_model_uses_fused(void* model, int* fused);
/* Persistent decode step (default off): one kernel launch runs the whole step -- the
 * fused kernels' work as a task list claimed in dependency order by a persistent grid,
 * weights streaming across layer boundaries, attention splits and limb slabs published
 * through per-slice readiness counters.  Used on one GPU when the fused kernels are in
 * use and the shapes fit (head_dim 32, 64 or 128, at most 8 query heads per kv head);
 * otherwise the fused per-operation kernels run.  No counterpart in the reference. */
int ib_model_set_persistent(void* model, int enabled);
#define IB_DECODE_SEPARATE 0
#define IB_DECODE_FUSED 1
#define IB_DECODE_PERSISTENT 2
/* Which decode step runs: IB_DECODE_SEPARATE / _FUSED / _PERSISTENT. */
int ib_model_decode_path(void* model, int* path);
/* The stream the model launches on (a cudaStream_t), e.g. for event timing. */
int ib_model_stream(void* model, void** stream);
/* KV cache element type of the native runner: IB_TYPE_F32 (the default, the
 * reference's FP32 cache, src/models/model_cuda.cpp:204-211) or IB_TYPE_F16 (half the
 * cache bytes per position; K and V rounded to nearest when written, every attention
 * kernel reads them back as FP32).  On a finalized model the caches are replaced by
 * empty ones (positions must be prefilled again) and the persistent decode step is
 * disabled with FP16 (the fused per-operation step runs). */
int ib_model_set_kv_type(void* model, int type);
/* enabled != 0: keep every packed linear of the layers decoded once as FP16 hi/lo planes
 * (ib_gemm_prepare_planes; 4 bytes per weight, 28 GB for the Llama-3-8B shape) so prompt
 * GEMMs of 128 tokens and more skip the per-call decoding (same results); IB_ERR_OOM
 * when they do not fit.  0 releases them.  On a finalized model. */
int ib_model_set_prefill_planes(void* model, int enabled);
int ib_model_kv_type(void* model, int* type);
/* Number of kernels one decode step launches. */
int ib_model_step_kernels(void* model, int* n_kernels);
/* Bytes of weights held on the device. */
int ib_model_weight_bytes(void* model, size_t* bytes);
/* The model's configuration (the whole model's shapes under tensor parallelism). */
int ib_model_get_config(void* model, ib_model_config* cfg);

/* ---- tensor parallelism (no counterpart in the reference, which runs on one GPU) ----
 * One process per GPU.  Rank 0 creates an id (ib_comm_unique_id), every rank receives
 * it out of band and calls ib_comm_init.  NCCL (libnccl.so.2) is opened at run time;
 * without it these calls return IB_ERR_COMM and the rest of the library works. */
int ib_comm_unique_id(uint8_t* id128);
/* The communicator runs in NCCL's non-blocking mode: initialisation and every later
 * NCCL call settle within timeout_ms (ib_comm_init: IB_COMM_DEFAULT_TIMEOUT_MS), or the
 * call returns IB_ERR_TIMEOUT (IB_ERR_COMM on an NCCL error) and the communicator is
 * aborted -- ncclCommAbort, which also ends NCCL kernels still waiting for a rank that
 * never arrived -- so a rank that never joins (or dies) leaves the others with an error,
 * not a hang.  Every later call on an aborted communicator fails at once. */
#define IB_COMM_DEFAULT_TIMEOUT_MS 300000
int ib_comm_init(int rank, int world, const uint8_t* id128, int device, void** comm);
int ib_comm_init_timeout(int rank, int world, const uint8_t* id128, int device,
                         int64_t timeout_ms, void** comm);
/* In-place sum over the ranks (FP32), on `stream`. */
int ib_comm_allreduce_f32(void* comm, float* dev_buf, int64_t n, void* stream);
/* *failed = 1 once the communicator has been aborted (after a failed or expired call,
 * or ib_comm_abort). */
int ib_comm_failed(void* comm, int* failed);
/* Aborts the communicator (ncclCommAbort); ib_comm_free still releases the handle. */
int ib_comm_abort(void* comm);
int ib_comm_free(void* comm);
/* The tensor-parallel model's peer-memory set-up (inside ib_model_finalize) is a
 * two-round protocol in which every rank fails together: round 1 gathers each rank's
 * status and IPC handle, round 2 the status of mapping the others' buffers; a rank that
 * failed earlier in its set-up still joins both rounds.  This runs that protocol with a
 * stand-in IPC layer (no device memory: a rank's handle is its rank number) over the
 * caller's all-gather, for host-side tests of the failure paths: local_status != 0
 * marks this rank as failed before the set-up, and on rank fail_rank the step
 * fail_step (1 = export the handle, 2 = map a peer) fails.  Returns what the set-up
 * returns on this rank (IB_OK or IB_ERR_COMM, the message names the failing rank);
 * *opened / *closed count the stand-in mappings made and released. */
typedef int (*ib_gather_fn)(void* ctx, const uint8_t* mine, uint8_t* all, size_t bytes);
int ib_peer_setup_check(int rank, int world, int local_status, int fail_rank, int fail_step,
                        ib_gather_fn gather, void* gather_ctx, int* opened, int* closed);
/* Host-side shard of a packed [rows, cols] tensor: axis 0 = the rank's contiguous
 * rows/world rows, axis 1 = the rank's contiguous (cols/block)/world blocks of every
 * row (the split of an input dimension on block boundaries). */
int ib_tp_shard(int type, const void* host_src, int64_t rows, int64_t cols, int axis, int rank,
                int world, void* host_dst);
/* A model whose layers are split over the communicator's ranks (Megatron split):
 * attn_q/k/v, ffn_gate/up and output rows by head / FFN column / vocabulary row,
 * attn_output and ffn_down input columns on block boundaries, token_embd and the
 * norms whole.  cfg and ib_model_set_tensor take the WHOLE model's shapes and
 * tensors; each rank uploads only its shard.  n_kv_heads, ffn and vocab must divide
 * by the world size.  Every rank makes the same calls in the same order (prefill,
 * decode, generate), including the same host_logits null-ness, since the steps hold
 * collectives; each rank then gets the same ids and logits. */
int ib_model_create_tp(const ib_model_config* cfg, int device, void* comm, void** model);
/* Self-test of the exchange's bounded wait on one GPU: rank 0 and a stand-in rank 1
 * whose rows are sent only when peer_sends != 0.  *fault = 0 and *x_out = 0.75 when
 * they arrive; otherwise the receiving kernel gives up after 2 s and *fault = 21 (the
 * code ib_check_fault would report), and the context stays usable. */
int ib_tp_wait_selftest(int peer_sends, int* fault, float* x_out);
int ib_model_load_gguf_tp(const char* path, int precision, int device, int max_seq, void* comm,
                          void** model);
/* Device time of one exchange round of the fused tensor-parallel decode step, measured
 * in isolation: every rank's rows of the model's dimension sent to every rank over peer
 * memory, then received, summed in rank order and turned into the next GEMV's limb slab
 * (zero rows, so the model's state is unchanged).  The step holds one round after each
 * row-split projection (attn_output, ffn_down).  Collective: every rank calls it with the
 * same `rounds`; IB_ERR_TIMEOUT when a peer's rows did not arrive within the exchange's
 * bounded wait. */
int ib_model_tp_exchange_time(void* model, int rounds, float* us_per_round);

/* ---- seeded synthetic weights (test and benchmark data, not a timed path) ---
 * Fills a [rows, cols] tensor of `type` with blocks encoding N(0, std) values
 * drawn from a counter-based stream keyed by `seed`.  The host and device
 * versions produce identical bytes. */
int ib_synth_host(int type, int64_t rows, int64_t cols, uint64_t seed, float stdv,
                  void* host_out, int n_threads);
int ib_synth_device(int type, int64_t rows, int64_t cols, uint64_t seed, float stdv,
                    void* dev_out, void* stream);
/* The FP32 values behind ib_synth_* (before quantisation). */
int ib_synth_values_host(int64_t n, uint64_t seed, float stdv, float* host_out);

#ifdef __cplusplus
}
#endif

#endif /* IB_CUDA_H */
