/*
 * nexus_gpu.h -- C ABI of libnexus_gpu.so, the B200 (sm_100a) implementation
 * of NexusLLM's fused quantized GEMV path.
 *
 * Plain C types only (pointers, sizes, integers); no CUDA or torch types in
 * any signature.  CUDA streams are passed as `void*` (a cudaStream_t; NULL
 * means the legacy default stream).
 *
 * Three layers, each replacing one reference interface:
 *
 *  1. Drop-in kernels with the reference's own signatures and semantics:
 *     host pointers in, host pointers out, synchronous, `void` return.
 *     They replace nexus::QuantizationKernel::fused_gemv_* and
 *     dequantize_gguf_* (include/quantization.hpp:80-153) and follow the C ABI
 *     precedent nexus_fused_gemv_int4/fp8 (include/nexus_abi.h:136-150,
 *     src/nexus_abi.cpp:462-480).  Weight matrices are uploaded once and kept
 *     in a device cache keyed by (host pointer, dtype, rows, cols); see
 *     nexus_gpu_weight_cache_invalidate.  On error they print one line to
 *     stderr and leave y untouched, as a void function must.
 *
 *  2. The backend hook INexusComputeBackend::gemv_dispatch
 *     (include/nexus_backend.hpp:55-62; CUDABackend at
 *     src/nexus_backend.cpp:239-367) plus the backend's device-memory calls
 *     (allocate_device_memory / copy_*_async / synchronize,
 *     include/nexus_backend.hpp:46-52).  Same argument meaning; returns a
 *     NexusStatus value instead of void.
 *
 *  3. The device-pointer API, asynchronous on a caller's stream, for callers
 *     that keep weights and activations resident in HBM (batched M >= 1,
 *     fp32 or bf16 activations).  New in this library; no reference
 *     counterpart (the reference has no device memory and no batched GEMV).
 *
 * Status codes are NexusStatus values (include/nexus_common.hpp:329-340),
 * extended with NEXUS_GPU_ERROR_* below for conditions the reference has no
 * code for.
 */
#ifndef NEXUS_GPU_H
#define NEXUS_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEXUS_GPU_API __attribute__((visibility("default")))

/* nexus::DataType values (include/nexus_common.hpp:244-260) accepted here. */
enum {
    NEXUS_GPU_FP32 = 0,      /* activations only */
    NEXUS_GPU_FP16 = 1,
    NEXUS_GPU_BF16 = 2,      /* activations only */
    NEXUS_GPU_GGUF_Q4_0 = 7,
    NEXUS_GPU_GGUF_Q8_0 = 9,
    NEXUS_GPU_GGUF_Q5_K = 11,
    NEXUS_GPU_GGUF_Q6_K = 12
};

/* NexusStatus (include/nexus_common.hpp:329-340) */
enum {
    NEXUS_GPU_SUCCESS = 0,
    NEXUS_GPU_ERROR_OUT_OF_HOST_MEMORY = -1,
    NEXUS_GPU_ERROR_OUT_OF_TIER0_MEMORY = -2, /* cudaMalloc failed */
    NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED = -3,
    NEXUS_GPU_ERROR_SHAPE_MISMATCH = -5,      /* cols not a whole number of blocks */
    NEXUS_GPU_ERROR_INVALID_ARGUMENT = -9,
    /* no NexusStatus equivalent: */
    NEXUS_GPU_ERROR_CUDA = -100,              /* a CUDA runtime call failed */
    NEXUS_GPU_ERROR_NO_DEVICE = -101,
    NEXUS_GPU_ERROR_WORKSPACE = -102,         /* workspace too small (and cannot grow now) */
    NEXUS_GPU_ERROR_TIMEOUT = -103            /* a bounded device-side wait expired */
};

/* ---------------------------------------------------------------- layer 1 */

/* QuantizationKernel::fused_gemv_q4_0 (include/quantization.hpp:116-120):
 * y[rows] = W[rows, cols] . x[cols]; W is rows*cols/32 BlockQ4_0 (18 B). */
NEXUS_GPU_API void nexus_fused_gemv_q4_0(const void* W_q4, const float* x, float* y, size_t rows, size_t cols);
/* QuantizationKernel::fused_gemv_q8_0 (include/quantization.hpp:122-126); BlockQ8_0 (34 B). */
NEXUS_GPU_API void nexus_fused_gemv_q8_0(const void* W_q8, const float* x, float* y, size_t rows, size_t cols);
/* QuantizationKernel::fused_gemv_fp16 (include/quantization.hpp:128-132); W is rows*cols halves,
 * decoded with the reference's fp16_to_fp32 (include/quantization.hpp:59-70). */
NEXUS_GPU_API void nexus_fused_gemv_fp16(const uint16_t* W_fp16, const float* x, float* y, size_t rows,
                                         size_t cols);
/* QuantizationKernel::fused_gemv_q5_k (include/quantization.hpp:143-147); BlockQ5_K (176 B). */
NEXUS_GPU_API void nexus_fused_gemv_q5_k(const void* W_q5_k, const float* x, float* y, size_t rows, size_t cols);
/* QuantizationKernel::fused_gemv_q6_k (include/quantization.hpp:149-153); BlockQ6_K (210 B). */
NEXUS_GPU_API void nexus_fused_gemv_q6_k(const void* W_q6_k, const float* x, float* y, size_t rows, size_t cols);

/* QuantizationKernel::dequantize_gguf_q4_0 / _q5_k / _q6_k (include/quantization.hpp:80-83,135-141):
 * host blocks in, host floats out (32 or 256 per block), bit-exact. */
NEXUS_GPU_API void nexus_dequantize_gguf_q4_0(const void* blocks, float* output, size_t num_blocks);
NEXUS_GPU_API void nexus_dequantize_gguf_q5_k(const void* blocks, float* output, size_t num_blocks);
NEXUS_GPU_API void nexus_dequantize_gguf_q6_k(const void* blocks, float* output, size_t num_blocks);

/* QuantizationKernel::fused_gemv_int4 (include/quantization.hpp:99-106; ABI
 * nexus_fused_gemv_int4, include/nexus_abi.h:136-143): INT4-AWQ, W_packed is
 * rows x cols/8 uint32 (column c = nibble c % 8 of word c / 8), scales and
 * zeros are rows x cols/group_size floats (zeros may be NULL), w = (q - zero)
 * * scale.  Needs cols % 8 == 0 and cols % group_size == 0 (the reference
 * reads past a row otherwise). */
NEXUS_GPU_API void nexus_fused_gemv_int4(const uint32_t* W_packed, const float* x, const float* scales,
                                         const float* zeros, float* y, size_t rows, size_t cols, size_t group_size);
/* QuantizationKernel::fused_gemv_fp8 (include/quantization.hpp:108-113; ABI
 * nexus_fused_gemv_fp8, include/nexus_abi.h:145-150): FP8-E4M3 bytes, the
 * reference's decoder (NaN codes 0x7F/0xFF -> 0) times one scale. */
NEXUS_GPU_API void nexus_fused_gemv_fp8(const uint8_t* W_fp8, const float* x, float* y, size_t rows, size_t cols,
                                        float scale);
/* QuantizationKernel::dequantize_int4_awq / dequantize_fp8_e4m3
 * (include/quantization.hpp:72-90): host in, host floats out, bit-exact. */
NEXUS_GPU_API void nexus_dequantize_int4_awq(const uint32_t* packed, const float* scales, const float* zeros,
                                             float* output, size_t count, size_t group_size);
NEXUS_GPU_API void nexus_dequantize_fp8_e4m3(const uint8_t* input, float* output, size_t count, float scale);

/* ---------------------------------------------------------------- layer 2 */

/* INexusComputeBackend::gemv_dispatch (include/nexus_backend.hpp:55-62) on the
 * CUDA device: host W (cached on the device), host x and y, synchronous.
 * W == NULL is a no-op returning SUCCESS, like TransformerOps::matmul_vec_dispatch
 * (include/transformer_ops.hpp:158).  FP32 weights are not handled here
 * (FORMAT_UNSUPPORTED): the reference's FP32 path is TransformerOps::matmul_vec. */
NEXUS_GPU_API int32_t nexus_gpu_gemv_dispatch(const void* W, uint32_t dtype, const float* x, float* y, size_t rows,
                                              size_t cols);

/* INexusComputeBackend::allocate_device_memory / free_device_memory /
 * copy_host_to_device_async / copy_device_to_host_async / synchronize
 * (include/nexus_backend.hpp:46-52) for the current CUDA device. */
NEXUS_GPU_API void* nexus_gpu_allocate_device_memory(size_t bytes);
NEXUS_GPU_API void nexus_gpu_free_device_memory(void* ptr);
NEXUS_GPU_API int32_t nexus_gpu_copy_host_to_device_async(void* dst_device, const void* src_host, size_t bytes,
                                                           void* stream);
NEXUS_GPU_API int32_t nexus_gpu_copy_device_to_host_async(void* dst_host, const void* src_device, size_t bytes,
                                                           void* stream);
NEXUS_GPU_API int32_t nexus_gpu_synchronize(void* stream);

/* Drop the cached device copy of a host weight buffer (call when the host
 * buffer is reused for another tensor, e.g. a recycled tier-0 slot,
 * src/memory_tier.cpp:341-356).  NULL drops every cached weight of the
 * current device.  The cache also re-uploads by itself when the host bytes'
 * fingerprint changes.  The fingerprint is checked at every call:
 *  - by default it covers the first and last 64 bytes and 16 bytes of every
 *    64 KiB.  A new tensor that matches the old one at all of those bytes
 *    goes undetected, so only this call is a guarantee;
 *  - with the environment variable NEXUS_GPU_WEIGHT_CHECK=full it hashes
 *    every byte (about 1 ms per 10 MB on one host thread), so any change is
 *    detected, up to a 64-bit hash collision. */
NEXUS_GPU_API int32_t nexus_gpu_weight_cache_invalidate(const void* host_W);
/* Bytes of device memory currently held by the weight cache. */
NEXUS_GPU_API size_t nexus_gpu_weight_cache_bytes(void);

/* ---------------------------------------------------------------- layer 3 */

/* Exact weight bytes of a rows x cols matrix in `dtype` (0 if unsupported). */
NEXUS_GPU_API size_t nexus_gpu_weight_bytes(uint32_t dtype, size_t rows, size_t cols);

/* Y[M, rows] = X[M, cols] . W[rows, cols]^T on the device, asynchronous on
 * `stream`.  dW, dX, dY are device pointers; X and Y are row-major with
 * leading dimensions cols and rows.  x_dtype is NEXUS_GPU_FP32 or
 * NEXUS_GPU_BF16.  Scratch space comes from a per-(device, stream) workspace
 * that the library grows with cudaMalloc when needed; it never grows while
 * the stream is capturing a CUDA graph (WORKSPACE is returned instead: make
 * one uncaptured call with the same shapes first, or use nexus_gpu_gemv_ws). */
NEXUS_GPU_API int32_t nexus_gpu_gemv(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype, float* dY,
                                     size_t M, size_t rows, size_t cols, void* stream);

/* Scratch bytes nexus_gpu_gemv_ws needs for these shapes. */
NEXUS_GPU_API size_t nexus_gpu_gemv_workspace_size(uint32_t dtype, size_t M, size_t rows, size_t cols);

/* nexus_gpu_gemv with caller-owned scratch (device memory, 256-byte aligned,
 * at least nexus_gpu_gemv_workspace_size bytes).  Never allocates. */
NEXUS_GPU_API int32_t nexus_gpu_gemv_ws(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype, float* dY,
                                        size_t M, size_t rows, size_t cols, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* nexus_gpu_gemv without any allocation.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: engines that assign all device
 * memory to weights and KV cache at start-up and forbid allocations on the
 * decode path, code that must not trigger the device-wide synchronisation a
 * cudaMalloc/cudaFree can cause, and callers with no workspace of their own to
 * hand to nexus_gpu_gemv_ws.  Same arguments and results as nexus_gpu_gemv.
 *
 * Its scratch (the quantized activations) is a fixed 1 MiB array inside the
 * library, held by every GPU that loads the library until the process exits.
 * Shapes needing more than that -- M * cols / 32 * 80 bytes (plus alignment)
 * above 1 MiB, e.g. M = 1 with cols above about 409,000 -- are rejected with
 * NEXUS_GPU_ERROR_WORKSPACE and a message naming the limit.  FP16 weights need
 * no scratch.  The first call on a device looks up the array's device address
 * for that device (cudaGetSymbolAddress, with the device current); make that
 * first call before any stream capture.  All calls share the one array and
 * every call rewrites the part it reads, so nothing needs clearing between
 * calls, but calls that overlap on the GPU (different streams, no ordering
 * between them) race on it: serialise them. */
NEXUS_GPU_API int32_t nexus_gpu_gemv_noalloc(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype,
                                             float* dY, size_t M, size_t rows, size_t cols, void* stream);

/* ------------------------------------------------------------ GEMV stacks */

/* One GEMV of a stack: y[rows] = W[rows, cols] . x (device pointers).  x is
 * the stack input (x_source = -1) or the y of an earlier task x_source.
 * `after` (-1 for none) names an earlier task that must have completed before
 * this one starts -- the ordering a decode step has between layers even when
 * the data does not flow directly. */
typedef struct {
    const void* W;
    uint64_t rows, cols;
    float* y;
    int32_t x_source;
    int32_t after;
} NexusGpuStackTask;

/* A sequence of GEMVs run by ONE persistent, cooperative kernel launch: the
 * GEMVs of a decode step (src/forward_pass.cpp:504-585 runs them one call at a
 * time).  Weights stream through the SMs back to back across tasks; each task
 * waits only for its own input.  Results equal nexus_gpu_gemv on the same
 * inputs bit for bit.  Integer GGUF formats; every task's shape must be inside
 * the fast kernel's limits.  No counterpart in the reference. */
NEXUS_GPU_API int32_t nexus_gpu_stack_create(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                             uint64_t input_cols, void** out_stack);
/* Run the stack on `stream` with input dX (fp32, input_cols, 16-byte aligned).
 * Graph-capturable: one kernel launch.  Runs of one stack must not overlap.
 * Counters are cumulative over runs (a device-side run counter sets each
 * run's targets), so a run needs no reset.  After a run reported a timeout
 * through nexus_gpu_device_status the stack is poisoned: destroy it. */
NEXUS_GPU_API int32_t nexus_gpu_stack_run(void* stack, const float* dX, void* stream);
NEXUS_GPU_API int32_t nexus_gpu_stack_destroy(void* stack);

/* A stack for `tokens` activation vectors per run: batched decode of that
 * many requests.  Every weight is read from HBM once per run, not once per
 * token; the reference decodes the requests one after another
 * (src/forward_pass.cpp:633-667).  The tasks are those of
 * nexus_gpu_stack_create; each tasks[i].y holds tokens * rows floats (token t
 * at y + t * rows, 16-byte aligned), and nexus_gpu_stack_run's dX holds
 * tokens * input_cols floats (token t at dX + t * input_cols).  Unsharded.
 *  - tokens 2..4: CUDA cores, integer GGUF formats.  Each token's outputs are
 *    within the GEMV tolerance of the single-token stack on that token (same
 *    arithmetic, another fixed summation order).
 *  - tokens 16..64: tcgen05 tensor cores, GGUF Q4_0, every task's cols a
 *    multiple of 256; one persistent launch whose CTAs meet at grid barriers
 *    where a task's input changes.  Each task's outputs are within 1e-6 of
 *    nexus_gpu_gemv with `tokens` rows on the same input.
 *  - tokens 5..15: ceil(tokens / 4) multi-token stacks of 2..4 tokens over
 *    the same tasks, launched one after another by each run (so every weight
 *    is read ceil(tokens / 4) times a run); each token's outputs as above.
 *  - tokens = 1 is nexus_gpu_stack_create; other counts are refused.
 * No counterpart in the reference. */
NEXUS_GPU_API int32_t nexus_gpu_stack_create_tokens(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                                    uint64_t input_cols, uint32_t tokens, void** out_stack);

/* Row-sharded GEMV stacks over `world` GPUs (2..8) of one node, one process
 * (or thread) per GPU, each holding the full x.  Row sharding of the
 * reference's GEMVs (src/forward_pass.cpp:504-585) with the all-gather fused
 * into the kernel: rank r computes rows [rows*r/world, rows*(r+1)/world) of
 * every task and writes them straight into every peer's copy of the output
 * over NVLink (peer stores); a task that another task depends on also writes
 * each row as a tagged 32-bit word (the run's parity in its lowest mantissa
 * bit), which the dependent task's readers check,
 * so no fence or counter sits between ranks inside a run.  No counterpart in
 * the reference.
 *   tasks[i].rows = the FULL row count; tasks[i].W = this rank's row slice
 *   (contiguous GGUF rows); tasks[i].y must be NULL: outputs belong to the
 *   stack (full-length on every rank, nexus_gpu_stack_output).
 * Every rank builds the same task list, then:
 *   nexus_gpu_stack_export  -> this rank's blob (CUDA IPC handle + checks);
 *   exchange the blobs between ranks (any host channel);
 *   nexus_gpu_stack_connect -> all `world` blobs in rank order.
 * Every rank must run the stack the same number of times. */
NEXUS_GPU_API int32_t nexus_gpu_stack_create_sharded(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                                     uint64_t input_cols, uint32_t world, uint32_t rank,
                                                     void** out_stack);
/* A stack task with the operations around the GEMV fused into it, so that a
 * stack can run the reference's decode layer (src/forward_pass.cpp:504-562:
 * RMSNorm -> q,k,v; o + residual; RMSNorm -> gate, up; SwiGLU -> down +
 * residual) in one launch.  Fields as NexusGpuStackTask, plus:
 *   x_source2       -1, or an earlier task: the GEMV input is
 *                   silu(x_source's output) * x_source2's output (SwiGLU,
 *                   include/transformer_ops.hpp:86-95);
 *   norm_weight     NULL, or cols fp32 weights on the device (16-byte aligned):
 *                   the input is RMSNorm(x) * norm_weight with norm_eps
 *                   (TransformerOps::rmsnorm, include/transformer_ops.hpp:23-44),
 *                   applied after the SwiGLU when both are given;
 *   residual_source -2 none, -1 the stack input, or an earlier task with as
 *                   many rows: y = GEMV + that vector (the residual adds of
 *                   src/forward_pass.cpp:539-541,558-561);
 *   W_up            NULL, or a second matrix of the same shape and format
 *                   (16-byte aligned; sharded: this rank's row slice, like W):
 *                   the task is the gate+up pair with its SwiGLU epilogue,
 *                   y = silu(W.x) * (W_up.x) (src/forward_pass.cpp:544-547), and
 *                   a down task reads it as its plain x_source.
 * world == 1 builds an unsharded stack (y required); world > 1 a sharded one
 * (y NULL, then export / connect as for nexus_gpu_stack_create_sharded). */
typedef struct {
    const void* W;
    uint64_t rows, cols;
    float* y;
    int32_t x_source;
    int32_t after;
    int32_t x_source2;
    int32_t residual_source;
    const float* norm_weight;
    float norm_eps;
    const void* W_up;
} NexusGpuStackTaskEx;
NEXUS_GPU_API int32_t nexus_gpu_stack_create_ex(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n_tasks,
                                                uint64_t input_cols, uint32_t world, uint32_t rank, void** out_stack);
/* Blob size when blob == NULL; else writes *blob_bytes (>= that size) bytes. */
NEXUS_GPU_API int32_t nexus_gpu_stack_export(void* stack, void* blob, uint64_t* blob_bytes);
NEXUS_GPU_API int32_t nexus_gpu_stack_connect(void* stack, const void* blobs, uint64_t blobs_bytes);
/* Connect the `n_stacks` ranks of one sharded stack that live in THIS process
 * (stacks[r] = rank r's handle; one thread or loop driving several GPUs, or
 * several ranks on one GPU): peers are reached by device pointer, with peer
 * access enabled between distinct devices.  Replaces export / connect. */
NEXUS_GPU_API int32_t nexus_gpu_stack_connect_local(void* const* stacks, uint32_t n_stacks);
/* Limit, in nanoseconds, of the stack's waits for rows of other CTAs and ranks
 * (0: the default, 2 s).  A wait that runs out sets the timeout bit of
 * nexus_gpu_device_status and poisons the stack. */
NEXUS_GPU_API int32_t nexus_gpu_stack_set_wait_limit(void* stack, uint64_t limit_ns);
/* Synchronize `stream`, then report NEXUS_GPU_ERROR_TIMEOUT if a bounded wait
 * of the stack expired (the reference's status convention,
 * include/nexus_common.hpp:329-340); the stack must then be destroyed. */
NEXUS_GPU_API int32_t nexus_gpu_stack_wait(void* stack, void* stream);
/* Device pointer to task `task`'s output on this rank (the caller's y for an
 * unsharded stack). */
NEXUS_GPU_API int32_t nexus_gpu_stack_output(void* stack, uint32_t task, float** y);

/* Bit-exact dequantization of `count` elements (a whole number of blocks)
 * from device blocks to device floats, asynchronous on `stream`. */
NEXUS_GPU_API int32_t nexus_gpu_dequantize(const void* dW, uint32_t dtype, float* dOut, size_t count, void* stream);

/* ------------------------------------------------ GGUF file -> device upload
 *
 * The on-disk side of the path: UniversalModelLoader::load_gguf
 * (src/model_loader.cpp:416-836) memory-maps a GGUF v2/v3 file and registers
 * every tensor; these calls do the same parse (host only, no device needed)
 * and then copy chosen tensors into ONE caller-owned device allocation.
 * Differences from the reference, on purpose:
 *   - ggml types map one to one (model_loader.cpp:735-746 maps Q4_1 onto
 *     Q4_0, Q5_1 onto Q5_0, Q8_1 onto Q8_0 and every type >= 24 onto BF16);
 *     types without a NexusLLM DataType get dtype -1 and are not uploaded;
 *   - byte sizes are the true block sizes (TensorShape::total_bytes,
 *     include/nexus_common.hpp:262-281, over-counts Q4_0 and Q6_K);
 *   - rows/cols follow GGUF's dimension order, cols = dims[0] (the row
 *     length) and rows = dims[1] * ... (src/forward_pass.cpp:581 takes the
 *     LM head's dims[0] as the vocabulary size, which is the hidden size);
 *   - a tensor that ends past the end of the file is skipped, as the
 *     reference skips one that starts past it (model_loader.cpp:728-731).
 * Metadata (NexusGpuGgufModel) follows model_loader.cpp:538-653 and its
 * fallbacks at 803-824: the same keys, defaults and inferences. */
typedef struct {
    char architecture[64];
    uint32_t version, alignment;
    uint64_t tensor_count;   /* tensors registered (skipped ones excluded) */
    uint64_t skipped;        /* tensors outside the file */
    uint64_t data_offset;    /* file offset of the tensor data section */
    uint32_t vocab_size, hidden_size, intermediate_size, num_hidden_layers;
    uint32_t num_attention_heads, num_key_value_heads, max_position_embeddings;
    float rms_norm_eps, rope_theta;
    uint32_t is_moe, num_experts, num_experts_per_tok;
} NexusGpuGgufModel;

typedef struct {
    char name[128];          /* truncated to 127 bytes; nexus_gpu_gguf_find matches the full name */
    uint32_t ggml_type;      /* as stored in the file */
    int32_t dtype;           /* NexusLLM DataType (NEXUS_GPU_* values), or -1 */
    uint32_t served;         /* 1: nexus_gpu_gemv takes this dtype (Q4_0, Q8_0, Q5_K, Q6_K, FP16) */
    uint32_t n_dims;
    uint64_t dims[4];        /* GGUF order: dims[0] is the row length */
    uint64_t rows, cols;     /* rows = dims[1] * dims[2] * dims[3], cols = dims[0] */
    uint64_t file_offset;    /* absolute offset of the data in the file */
    uint64_t bytes;          /* true size in the file (0 when the type's block size is unknown) */
} NexusGpuGgufTensor;

/* Opens and parses `path` (memory-mapped, read-only).  Host only. */
NEXUS_GPU_API int32_t nexus_gpu_gguf_open(const char* path, void** out_file);
NEXUS_GPU_API int32_t nexus_gpu_gguf_close(void* file);
NEXUS_GPU_API int32_t nexus_gpu_gguf_model(void* file, NexusGpuGgufModel* out);
NEXUS_GPU_API int32_t nexus_gpu_gguf_tensor(void* file, uint64_t index, NexusGpuGgufTensor* out);
/* Index of the tensor `name`: that name, else the first tensor with the same
 * canonical key in the reference's alias classes (register_aliases,
 * model_loader.cpp:60-302: e.g. "layers.0.wq" finds "blk.0.attn_q.weight" or
 * "model.layers.0.self_attn.q_proj.weight"; MTP-head aliases are not kept),
 * else, for the LM head, the token embedding when the file has no LM head
 * (tied weights, model_loader.cpp:793-801).  NEXUS_GPU_ERROR_INVALID_ARGUMENT
 * if absent. */
NEXUS_GPU_API int32_t nexus_gpu_gguf_find(void* file, const char* name, uint64_t* index);
/* Device bytes that nexus_gpu_gguf_upload needs for these tensors: each one
 * starts on a 256-byte boundary of the image. */
NEXUS_GPU_API uint64_t nexus_gpu_gguf_upload_size(void* file, const uint64_t* indices, uint64_t n);
/* Copies the tensors into d_dst (dst_bytes >= nexus_gpu_gguf_upload_size),
 * each at the offset it returns in offsets[i], through pinned staging
 * buffers filled by host threads, on `stream`.  Returns when the bytes are on
 * the device.  Tensors with dtype -1 or unknown size are refused. */
NEXUS_GPU_API int32_t nexus_gpu_gguf_upload(void* file, const uint64_t* indices, uint64_t n, void* d_dst,
                                            uint64_t dst_bytes, uint64_t* offsets, void* stream);

/* ------------------------------------------------------------- diagnostics */

/* INT4-AWQ / FP8-E4M3 on device pointers, stream-ordered (the layer-1 calls
 * above on device memory).  nexus_gpu_gemv_int4 quantizes x into a workspace
 * of nexus_gpu_gemv_int4_workspace_size(cols) bytes: the caller's (workspace,
 * workspace_bytes), or the library's per-stream workspace when workspace is
 * NULL.  Returns a NEXUS_GPU_* status. */
NEXUS_GPU_API size_t nexus_gpu_gemv_int4_workspace_size(size_t cols);
NEXUS_GPU_API int32_t nexus_gpu_gemv_int4(const void* dW, const float* dScales, const float* dZeros, const float* dX,
                                          float* dY, size_t rows, size_t cols, size_t group_size, void* workspace,
                                          size_t workspace_bytes, void* stream);
NEXUS_GPU_API int32_t nexus_gpu_gemv_fp8(const void* dW, const float* dX, float* dY, size_t rows, size_t cols,
                                         float scale, void* stream);
NEXUS_GPU_API int32_t nexus_gpu_dequantize_int4_awq(const void* dPacked, const float* dScales, const float* dZeros,
                                                    float* dOut, size_t count, size_t group_size, void* stream);
NEXUS_GPU_API int32_t nexus_gpu_dequantize_fp8_e4m3(const void* dIn, float* dOut, size_t count, float scale,
                                                    void* stream);

/* Message of the last error on the calling thread ("" if none). */
NEXUS_GPU_API const char* nexus_gpu_last_error(void);
/* Reads and clears the device-side status word of the current device
 * (bit 0: a bounded wait expired).  Synchronizes the device. */
NEXUS_GPU_API int32_t nexus_gpu_device_status(uint32_t* out_bits);
/* Name of the device, SM count and compute capability of the current device. */
NEXUS_GPU_API int32_t nexus_gpu_device_info(char* name, size_t name_len, int* sm_count, int* cc_major,
                                            int* cc_minor);
/* Library version string. */
NEXUS_GPU_API const char* nexus_gpu_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NEXUS_GPU_H */
