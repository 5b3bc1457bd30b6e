/*
 * bramha_cuda.h -- C ABI of the B200 (sm_100a) quantized linear-layer plane.
 *
 * This is the drop-in boundary for the GPU arm of the reference's compute
 * layer (akshaybhlrp/bramha): it replaces `WgpuComputePlane`
 * (src/compute/wgpu_backend.rs:100-1728) and the dead GPU dispatch inside
 * `matvec_mul` (src/inference/cpu_engine.rs:380-454), and adds the prefill
 * GEMM that `gemm_cpu` (src/inference/cpu_engine.rs:565-912) computes on the
 * host.  Plain C types only: a Rust `extern "C"` block, ctypes or cgo can bind
 * it without CUDA or torch headers.  Streams are passed as `void*` holding a
 * `cudaStream_t` (NULL = the context's own stream).
 *
 * Conventions (mirroring the reference):
 *  - every call returns BRAMHA_OK (0) or a negative BRAMHA_ERR_* status and
 *    never aborts; no C++ exception crosses this boundary;
 *  - the message of the last failure on the calling thread is returned by
 *    bramha_cuda_last_error() (the reference returns `Err(String)`);
 *  - size mismatches are errors (wgpu_backend.rs:1096-1104); N == 0 or K == 0
 *    returns zeros (wgpu_backend.rs:1092-1095);
 *  - weights are copied once into a persistent device buffer keyed by
 *    "model:layer" (get_or_create_op, wgpu_backend.rs:603-722) and evicted in
 *    least-recently-used order above a device-memory cap (ModelBuffers,
 *    wgpu_backend.rs:25-82);
 *  - the registry is thread-safe; host-buffer calls are synchronous (they
 *    return once the result is in host memory), like the reference's
 *    `device.poll(Wait)` round trip (wgpu_backend.rs:1244).
 *
 * Weight formats (row-major, one fp32 scale per output row):
 *  - BRAMHA_FMT_F32   : f32 [N][K]                          (matvec_mul, wgpu_backend.rs:734)
 *  - BRAMHA_FMT_W8    : i8  [N][K], w = q * s_row           (quantize_to_int8, src/models/quantization.rs:7-38)
 *  - BRAMHA_FMT_W4ZP8 : u8  [N][K/2], even column in the high nibble,
 *                       w = (nibble - 8) * s_row            (quantize_to_int4, quantization.rs:41-83)
 *  - BRAMHA_FMT_LOG4  : u8  [N][K/2], high nibble first,
 *                       w = (2^code - 1) * s_row            (dequantize_log4, spanda-engine/src/lib.rs:332-342)
 */
#ifndef BRAMHA_CUDA_H
#define BRAMHA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BRAMHA_CUDA_ABI_VERSION 1

#if defined(__GNUC__)
#define BRAMHA_API __attribute__((visibility("default")))
#else
#define BRAMHA_API
#endif

enum bramha_format {
    BRAMHA_FMT_F32 = 0,
    BRAMHA_FMT_W8 = 1,
    BRAMHA_FMT_W4ZP8 = 2,
    BRAMHA_FMT_LOG4 = 3,
    /* 2:4 structured-sparse weights (registered through the sparse24 calls
     * below, never through bramha_cuda_register_weight): two kept codes of
     * each group of four columns, of F32, W8 or W4ZP8. */
    BRAMHA_FMT_SP24_F32 = 4,
    BRAMHA_FMT_SP24_W8 = 5,
    BRAMHA_FMT_SP24_W4ZP8 = 6
};

enum bramha_dtype { BRAMHA_DTYPE_F32 = 0, BRAMHA_DTYPE_BF16 = 1 };

enum bramha_status {
    BRAMHA_OK = 0,
    BRAMHA_ERR_INVALID = -1,     /* null pointer, bad enum, negative size   */
    BRAMHA_ERR_SIZE = -2,        /* buffer length does not match the shape  */
    BRAMHA_ERR_CUDA = -3,        /* a CUDA runtime call failed              */
    BRAMHA_ERR_OOM = -4,         /* device memory exhausted / above the cap */
    BRAMHA_ERR_UNSUPPORTED = -5, /* shape or format this build cannot run   */
    BRAMHA_ERR_NOT_FOUND = -6,   /* unknown weight key                      */
    BRAMHA_ERR_TIMEOUT = -7,     /* a bounded device-side wait gave up      */
    BRAMHA_ERR_NCCL = -8         /* a collective failed                     */
};

typedef struct bramha_ctx bramha_ctx;
typedef struct bramha_weight bramha_weight;

/* ---------------------------------------------------------------- context */

/* Replaces WgpuComputePlane::new (wgpu_backend.rs:121) / get_wgpu_plane
 * (wgpu_backend.rs:1710-1728): binds `device`, creates the context stream and
 * the weight registry, and allocates the context's GEMV scratch (32 MB of
 * K-split partial results and a ticket array, kept for the context's life).
 * GEMV calls on one context share that scratch, so GEMVs of one context must
 * not run concurrently on different streams (use one context per stream for
 * that).  Fails with BRAMHA_ERR_UNSUPPORTED on a device that is not sm_100
 * (the kernels are built for sm_100a only). */
BRAMHA_API int bramha_cuda_init(int device, bramha_ctx** out);

/* Frees every registered weight and the context. */
BRAMHA_API int bramha_cuda_destroy(bramha_ctx* ctx);

/* Message of the last failed call on this thread ("" if none).  The
 * reference's `Err(String)` payloads (wgpu_backend.rs:1096-1104). */
BRAMHA_API const char* bramha_cuda_last_error(void);

BRAMHA_API int bramha_cuda_abi_version(void);

/* Device-memory cap for registered weights, in bytes (ModelBuffers::new,
 * wgpu_backend.rs:41-56; the reference caps at 3 GB). 0 = no cap. */
BRAMHA_API int bramha_cuda_set_memory_cap(bramha_ctx* ctx, size_t bytes);
BRAMHA_API int bramha_cuda_memory_used(bramha_ctx* ctx, size_t* bytes);

/* Which GEMV kernel the context's calls use for the quantized formats.
 * AUTO (default): at batch 1, launches with rows of at most 1024 columns and at
 * most 8 MB of packed weights run on the CUDA cores (latency-bound: weights
 * preloaded before the launch dependency, fp32 multiply-adds), all others and
 * batches > 1 on the tensor cores.  TENSOR_CORE / CUDA_CORE pin one kernel (CUDA_CORE applies at batch 1;
 * other batches stay on the tensor cores).  Both compute y = s * sum x * code
 * within the path's 1e-3 tolerance of the reference. */
#define BRAMHA_GEMV_AUTO 0
#define BRAMHA_GEMV_TENSOR_CORE 1
#define BRAMHA_GEMV_CUDA_CORE 2
BRAMHA_API int bramha_cuda_set_gemv_kernel(bramha_ctx* ctx, int kind);

/* Bound on every device-side wait of the tensor-core kernels, in nanoseconds
 * of %globaltimer (default 2 s; 0 restores it).  A kernel whose wait runs out
 * records BRAMHA_ERR_TIMEOUT, drains the copies and MMAs it issued, frees its
 * TMEM and returns; the host-buffer calls and bramha_cuda_stream_sync then
 * return BRAMHA_ERR_TIMEOUT (the reference reports a failed GPU call as
 * `Err(String)`, wgpu_backend.rs:1096-1104, and falls back to the CPU).  Set it
 * while no work of the context is in flight. */
BRAMHA_API int bramha_cuda_set_wait_timeout(bramha_ctx* ctx, uint64_t ns);

/* TEST ONLY (no counterpart in the reference): makes CTA 0 of every later
 * tensor-core GEMV (kind BRAMHA_TEST_FAULT_GEMV) or tensor-core GEMM (kind
 * BRAMHA_TEST_FAULT_GEMM) launch of this context withhold one weight copy, so
 * the consumers' bounded waits run out and the call reports
 * BRAMHA_ERR_TIMEOUT without hanging or faulting the GPU.  Kind 0 turns it off.
 * Use a short bramha_cuda_set_wait_timeout with it. */
#define BRAMHA_TEST_FAULT_NONE 0
#define BRAMHA_TEST_FAULT_GEMV 1
#define BRAMHA_TEST_FAULT_GEMM 2
BRAMHA_API int bramha_cuda_test_fault(bramha_ctx* ctx, int kind);

/* L2 prefetch of the tensor-core GEMV (tuning; no counterpart in the
 * reference).  lookahead_bytes: how far ahead of its shared-memory copies each
 * CTA asks HBM for its weight stream (default 0 = off).  next_launch_bytes: in
 * a GEMV chain, how many of the next launch's weight bytes the current launch
 * requests into L2 once its own copies are issued (default 8 MB; 0 = off).
 * Prefetching reads no memory outside the weights and changes no result. */
BRAMHA_API int bramha_cuda_set_prefetch(bramha_ctx* ctx, int64_t lookahead_bytes, int64_t next_launch_bytes);

/* Tensor-core GEMV tuning (no counterpart in the reference; results do not
 * change): LOOKAHEAD_BYTES / NEXT_LAUNCH_BYTES as bramha_cuda_set_prefetch;
 * EVICT_FIRST (default 0): weight copies are marked first to be evicted from
 * L2; SPLIT_COST (default 240): what the K-split plan charges for splitting a
 * launch's K range, in eighths of one 64-column weight block;
 * PROGRAM_LOOKAHEAD_BYTES (default 0 = off): how far ahead of its shared-memory
 * copies each CTA of a GEMV program requests its weight stream into L2, so the
 * stream continues while an op waits for the previous op's output.
 * CC_SPLIT_DEPTH (default 4, 1..64): the CUDA-core GEMV (batch 1, K <= 1024)
 * splits K until its CTAs cover the SMs this many deep; the split changes only
 * the grouping of the fp32 sums (the partials are added in split order). */
#define BRAMHA_TUNE_LOOKAHEAD_BYTES 1
#define BRAMHA_TUNE_NEXT_LAUNCH_BYTES 2
#define BRAMHA_TUNE_EVICT_FIRST 3
#define BRAMHA_TUNE_SPLIT_COST 4
#define BRAMHA_TUNE_PROGRAM_LOOKAHEAD_BYTES 5
#define BRAMHA_TUNE_CC_SPLIT_DEPTH 6
BRAMHA_API int bramha_cuda_set_gemv_tuning(bramha_ctx* ctx, int what, int64_t value);

/* ---------------------------------------------------------------- weights */

/* get_or_create_op (wgpu_backend.rs:603-722): copies the packed weight and
 * its per-row scales from HOST memory into a persistent device buffer under
 * `key`.  Idempotent per key: a second call with the same key returns the
 * cached weight and refreshes its LRU position.  `scales` may be NULL for
 * BRAMHA_FMT_F32.  q_bytes must equal N*K*4 (F32), N*K (W8) or N*(K/2)
 * (W4ZP8, LOG4); n_scales must equal N. */
BRAMHA_API int bramha_cuda_register_weight(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                const void* q, size_t q_bytes, const float* scales, size_t n_scales,
                                bramha_weight** out);

/* Same, from DEVICE memory (device-to-device copy on `stream`). */
BRAMHA_API int bramha_cuda_register_weight_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                    const void* q_dev, size_t q_bytes, const float* scales_dev,
                                    size_t n_scales, void* stream, bramha_weight** out);

/* Looks up a registered weight (refreshes its LRU position). */
BRAMHA_API int bramha_cuda_lookup_weight(bramha_ctx* ctx, const char* key, bramha_weight** out);

/* Evicts one key, or all (clear_persistent_buffers, wgpu_backend.rs:725-731). */
BRAMHA_API int bramha_cuda_evict_weight(bramha_ctx* ctx, const char* key);
BRAMHA_API int bramha_cuda_clear(bramha_ctx* ctx);

/* Shape / format / device footprint of a registered weight. */
BRAMHA_API int bramha_cuda_weight_info(const bramha_weight* w, int* fmt, int64_t* N, int64_t* K, size_t* device_bytes);

/* -------------------------------------------------------- decode GEMV path */

/* matvec_mul_int4 / matvec_mul_int8 / matvec_mul (wgpu_backend.rs:1083, 906,
 * 734) in one entry point: y[b][j] = sum_i x[b][i] * dq(w[j][i]) for
 * b < batch, host buffers, synchronous.  `x_host` is [batch][K] f32,
 * `y_host` is [batch][N] f32. */
BRAMHA_API int bramha_cuda_gemv(bramha_ctx* ctx, const bramha_weight* w, const float* x_host, int64_t batch,
                     float* y_host);

/* Device-pointer, stream-ordered variant (asynchronous). */
BRAMHA_API int bramha_cuda_gemv_dev(bramha_ctx* ctx, const bramha_weight* w, const float* x_dev, int64_t batch,
                         float* y_dev, void* stream);

/* fused_qkv_mul_into (cpu_engine.rs:3342-3354) generalised: several weights
 * that share one input x (same K), computed by ONE kernel launch.  y_devs[i]
 * is [batch][N_i]. At most 8 weights. */
BRAMHA_API int bramha_cuda_gemv_multi_dev(bramha_ctx* ctx, int n_weights, const bramha_weight* const* ws,
                               const float* x_dev, int64_t batch, float* const* y_devs, void* stream);

/* The down projection of a SwiGLU MLP in one launch: y[b] = W (silu(gate[b]) *
 * up[b]) with silu(g) = g * (1 / (1 + exp(-g))), the activation formed while the
 * tensor-core GEMV stages it (run_mlp_into's dense branch, cpu_engine.rs:
 * 2023-2029, as bramha_cuda_op_silu_mul followed by bramha_cuda_gemv_dev, with
 * the same rounding).  LOG4, W4ZP8 and W8 weights; gate and up [batch][K] f32,
 * 16-byte aligned; y [batch][N]; stream-ordered. */
BRAMHA_API int bramha_cuda_gemv_swiglu_dev(bramha_ctx* ctx, const bramha_weight* w, const float* gate_dev,
                                           const float* up_dev, int64_t batch, float* y_dev, void* stream);

/* A pre-norm block's RMSNorm and the GEMVs that read it, batch 1: with
 * r = x + delta (delta may be NULL: r = x), h = rms_norm(r) * norm_w exactly as
 * bramha_cuda_op_rmsnorm computes it (rms_norm, cpu_engine.rs:1292-1302, with
 * the residual add of the decode loop, :2819-3064), then y_i = W_i h for each
 * weight (fused_qkv_mul_into / the gate and up projections, :3342-3354).  r is
 * stored to x_out_dev when it is non-NULL (x_out_dev must not overlap x_dev or
 * delta_dev: the residual stream is double-buffered); h is not stored.  When
 * the CUDA-core GEMV takes the weights (batch-1 launches of short rows, see
 * bramha_cuda_set_gemv_kernel) the RMSNorm is formed inside that one launch,
 * every CTA reducing the whole r in the RMSNorm kernel's order; otherwise the
 * RMSNorm kernel runs first (stream-ordered scratch).  Either way the outputs
 * equal bramha_cuda_op_rmsnorm followed by bramha_cuda_gemv_multi_dev bit for
 * bit.  1..8 weights of one tiled format and K; device pointers; stream-ordered. */
BRAMHA_API int bramha_cuda_gemv_rmsnorm_dev(bramha_ctx* ctx, int n_weights, const bramha_weight* const* ws,
                                            const float* x_dev, const float* delta_dev, const float* norm_w_dev,
                                            float eps, float* x_out_dev, float* const* y_devs, void* stream);

/* A chain of dependent GEMVs: the reference's decode loop calls
 * matvec_mul_into back to back (fused_qkv_mul_into, o_proj, run_mlp_into's
 * gate / up / down, lm_head; cpu_engine.rs:2873-2976), each GEMV reading what
 * the previous steps wrote.  ops[i] is one launch of 1..8 weights sharing x
 * (same format and K), run after ops[i-1] in stream order; while it runs it
 * also requests the first weights of ops[i+1] from HBM into L2, so the
 * weight stream does not pause at the launch boundary.  x_up non-NULL makes
 * the activation silu(x) * x_up (the down projection of a SwiGLU MLP, as
 * bramha_cuda_gemv_swiglu_dev).  Results equal one bramha_cuda_gemv_multi_dev
 * (or _swiglu_dev) call per op. */
typedef struct bramha_gemv_op {
    int n_weights;                         /* 1..8 */
    const bramha_weight* const* weights;   /* n_weights handles */
    const float* x;                        /* [batch][K] */
    const float* x_up;                     /* NULL, or [batch][K] (SwiGLU) */
    float* const* y;                       /* y[i] is [batch][N_i] */
} bramha_gemv_op;

/* Device pointers, stream-ordered (x 16-byte aligned, as gemv_multi_dev). */
BRAMHA_API int bramha_cuda_gemv_chain_dev(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                                          void* stream);

/* Host buffers (any alignment), synchronous: every op's x is copied to the
 * device, the chain runs, every y is copied back, and the call returns once
 * they are in host memory (one wait for the whole chain, which also reports a
 * device-side failure).  The copies run on two streams of the context beside
 * its launch stream, in blocks of ops (1, 2, 4, 8, 16, ..., 16, 8, 4, 2, 1):
 * a block's launches wait only for its own inputs, and its outputs are copied
 * back while the later blocks run, so with pinned host buffers the copies hide
 * behind the launches.  Pageable buffers work too (the driver stages them). */
BRAMHA_API int bramha_cuda_gemv_chain(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch);

/* A host-buffer chain bound once and run many times (no counterpart in the
 * reference, whose host calls each stand alone): the op list -- weights and
 * the x, x_up and y host pointers -- is copied at creation, the chain gets its
 * own device staging, and when every x, x_up and y is page-locked host memory
 * the copies and launches of bramha_cuda_gemv_chain are recorded once into a
 * CUDA graph that each run replays (otherwise each run enqueues them as
 * bramha_cuda_gemv_chain does).  A run is synchronous, reads the host inputs'
 * current contents and reports a device-side failure like
 * bramha_cuda_gemv_chain.  The host buffers must stay allocated and, when
 * recorded, page-locked while the chain exists; the weights must stay
 * registered (each run checks).  The launch choices in force at creation (GEMV
 * kernel, tuning keys) are kept.  Create a chain while no other thread enqueues
 * work on the context's own stream (the recording captures that stream).
 * With sharded weights in the list each run is a bramha_cuda_gemv_chain call
 * on the bound ops (staged in the shard arena, not recorded). */
typedef struct bramha_host_chain bramha_host_chain;
BRAMHA_API int bramha_cuda_host_chain_create(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                                             bramha_host_chain** out);
BRAMHA_API int bramha_cuda_host_chain_run(bramha_ctx* ctx, bramha_host_chain* chain);
/* *out = 1 when the chain replays a recorded CUDA graph, 0 when it runs eagerly. */
BRAMHA_API int bramha_cuda_host_chain_uses_graph(bramha_ctx* ctx, const bramha_host_chain* chain, int* out);
BRAMHA_API int bramha_cuda_host_chain_destroy(bramha_ctx* ctx, bramha_host_chain* chain);

/* The same chain as ONE persistent launch (no counterpart in the reference,
 * which runs one GEMV at a time).  One CTA per SM runs every op: the weight
 * stream and its decoding continue across op boundaries, and op i+1 reads its
 * input only after every CTA has finished op i (a bounded wait on a per-op
 * counter), so op i+1 may read op i's output.  A program binds its ops --
 * weights, x, x_up and y pointers -- at creation and can be run any number of
 * times (also from a CUDA graph); the weights must stay registered while it
 * exists.  Requirements: every op LOG4, or every op W4ZP8, or every op W8;
 * batch 1..8; every weight with N > 0 and K > 0; device pointers as for
 * bramha_cuda_gemv_chain_dev; no sharded weights.  Results: W8 and W4ZP8
 * equal the op-by-op chain within fp32 rounding of sum(x); LOG4 within fp32
 * rounding (the chain's slots are grouped differently among the four MMA
 * accumulators); all within the path's 1e-3 of the reference.  A program
 * shares its context's K-split workspace: run one program or GEMV of a
 * context at a time. */
typedef struct bramha_gemv_program bramha_gemv_program;
BRAMHA_API int bramha_cuda_gemv_program_create(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                                               bramha_gemv_program** out);
BRAMHA_API int bramha_cuda_gemv_program_run_dev(bramha_ctx* ctx, bramha_gemv_program* prog, void* stream);
BRAMHA_API int bramha_cuda_gemv_program_destroy(bramha_ctx* ctx, bramha_gemv_program* prog);

/* Tracing of a program (the GPU counterpart of the reference's scoped
 * profiler, src/inference/profiler.rs:57-153): with `on`, each later run
 * records, per op and CTA, eight %globaltimer stamps in nanoseconds -- the op
 * is reached, every CTA has finished the previous op, this CTA's MMAs of it
 * are done, the activations are loaded, the activation terms are built, the
 * last accumulator is ready, the outputs are stored, the completion is
 * published.  read_trace copies [n_ops][grid][8] stamps (at most `n`) into
 * host memory after a run; *grid receives the CTA count. */
BRAMHA_API int bramha_cuda_gemv_program_trace(bramha_ctx* ctx, bramha_gemv_program* prog, int on);
BRAMHA_API int bramha_cuda_gemv_program_read_trace(bramha_ctx* ctx, bramha_gemv_program* prog, uint64_t* out,
                                                   size_t n, int* grid);

/* The reference's keyed one-shot call, e.g.
 * `matvec_mul_int4(h, q_weight, scales, out_features, model_name, layer_name)`
 * (wgpu_backend.rs:1083-1091): when both names are non-NULL the weight is
 * cached under "model:layer"; otherwise it is uploaded for this call only.
 * K is the length of h; out is [N]. */
BRAMHA_API int bramha_cuda_matvec(bramha_ctx* ctx, int fmt, const float* h, int64_t K, const void* q_weight,
                       size_t q_bytes, const float* scales, size_t n_scales, int64_t N,
                       const char* model_name, const char* layer_name, float* out);

/* ------------------------------------------------- 2:4 structured sparsity */

/* The reference's 2:4 sparse GEMVs (spanda-engine/src/sparse.rs:19-138 and
 * sparse_matvec_mul_2_4_tensor_into, cpu_engine.rs:1532-1640) keep, in every
 * group of four consecutive columns of a row, two weights and sum their
 * products with x.  Registered 2:4 weights (formats BRAMHA_FMT_SP24_*) run
 * through bramha_cuda_gemv / _gemv_dev / _gemv_multi_dev / _gemm like any
 * other weight (f32 activations; one launch per activation row), computing
 *   y[j] = s_j * (sum over groups of the two kept products + the products of
 *          the K % 4 trailing columns)
 * in fp32 (s_j = 1 for F32 weights).  Device bytes per group of four
 * columns: 8.5 (F32), 2.5 (W8), 1.5 (W4ZP8). */

/* Registers a dense F32, W8 or W4ZP8 weight (the layouts and size rules of
 * bramha_cuda_register_weight; W4ZP8 needs an even K, as the reference's int4
 * arm panics otherwise) as 2:4: each group of four keeps the two codes of
 * largest magnitude, ties to the lower column, the selection
 * sparse_matvec_mul_2_4_tensor_into makes on every call (cpu_engine.rs:
 * 1539-1552, 1568-1581, 1606-1623) made here once on the device.  The K % 4
 * trailing columns stay dense (cpu_engine.rs:1558-1561).  Idempotent per key
 * (a key registered with another format or shape is an error). */
BRAMHA_API int bramha_cuda_register_sparse24(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                             const void* q, size_t q_bytes, const float* scales, size_t n_scales,
                                             bramha_weight** out);
BRAMHA_API int bramha_cuda_register_sparse24_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                                 const void* q_dev, size_t q_bytes, const float* scales_dev,
                                                 size_t n_scales, void* stream, bramha_weight** out);

/* Registers a compressed 2:4 tensor (the .spanda BlockSparse2_4 variant,
 * spanda-engine/src/lib.rs:89-93): masks [rows][cols / 4] u16, low 4 bits =
 * kept columns of the group; values consumed in column order from index
 * 2 * r * (cols / 4) for row r while any remain (sparse.rs:109-125).  Columns
 * past the last whole group are ignored (sparse.rs:128-132).  Fails with
 * BRAMHA_ERR_SIZE when masks holds fewer than rows * (cols / 4) entries and
 * BRAMHA_ERR_UNSUPPORTED when a group would consume more than two values. */
BRAMHA_API int bramha_cuda_register_sparse24_compressed(bramha_ctx* ctx, const char* key, int64_t rows,
                                                        int64_t cols, const uint16_t* masks, size_t n_masks,
                                                        const float* values, size_t n_values, bramha_weight** out);

/* sparse_matvec_mul_2_4 (sparse.rs:19, F32) / sparse_matvec_mul_2_4_tensor_into
 * (cpu_engine.rs:1532; F32, W8, W4ZP8) as a keyed one-shot call with the
 * conventions of bramha_cuda_matvec: h [K] host, out [N] host, synchronous;
 * cached under "model:layer" when both names are given. */
BRAMHA_API int bramha_cuda_sparse_matvec_2_4(bramha_ctx* ctx, int fmt, const float* h, int64_t K,
                                             const void* q_weight, size_t q_bytes, const float* scales,
                                             size_t n_scales, int64_t N, const char* model_name,
                                             const char* layer_name, float* out);

/* sparse_matvec_2_4_compressed (sparse.rs:100): x [cols] host, out [rows]
 * host, synchronous; cached under "model:layer" when both names are given. */
BRAMHA_API int bramha_cuda_sparse_matvec_2_4_compressed(bramha_ctx* ctx, const float* x, int64_t cols,
                                                        const uint16_t* masks, size_t n_masks, const float* values,
                                                        size_t n_values, int64_t rows, const char* model_name,
                                                        const char* layer_name, float* out);

/* ------------------------------------------------------- MoE expert MLP */

/* The MoE branch of run_mlp_into (src/inference/cpu_engine.rs:1799-1989) for a
 * batch of T decode tokens: per token, p = softmax(logits[t]) (sequential, as
 * the reference), the first top_k experts of a stable descending sort (equal
 * probabilities keep the lower expert first; no renormalisation; experts with
 * p <= 0 skipped), and
 *   out[t] = sum over the kept experts, in that order, of p_e * down_e(silu(gate_e x) * up_e x)
 * with silu(g) = g / (1 + exp(-g)).  Tokens are grouped by expert so each
 * expert's weights are read once per call (grouped tcgen05 GEMMs, f32
 * activations split into bf16 hi + lo, fp32 accumulation: within ~1e-3
 * normwise of the reference).
 * Weights, registered with bramha_cuda_register_weight in one of LOG4, W4ZP8,
 * W8 (both the same):
 *   gate_up: [E * 2I][H], expert e's gate rows then its up rows at rows
 *            [2I e, 2I e + I) and [2I e + I, 2I (e + 1));
 *   down:    [E * H][I], expert e at rows [H e, H (e + 1)).
 * 2I and H must be multiples of 128; T * min(top_k, E) <= 16384; E <= 1024.
 * x [T][H], logits [T][E] (the router's output: a GEMV with the router weight,
 * cpu_engine.rs:1801-1803, is a bramha_cuda_gemv call), out [T][H] f32;
 * selected [T][min(top_k, E)] receives the sorted expert ids (skipped ones
 * included), or pass NULL.  Scratch comes from the stream-ordered pool. */
BRAMHA_API int bramha_cuda_moe_mlp_dev(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down,
                                       int num_experts, int top_k, const float* x_dev, const float* logits_dev,
                                       int64_t T, float* out_dev, int32_t* selected_dev, void* stream);
/* The two halves of that layer for expert parallelism, where the experts of a
 * layer are spread over several GPUs and each token's activation is sent to the
 * GPUs holding its experts:
 *  - moe_route_dev: the routing alone -- ids [T][min(top_k, E)] (int32) and
 *    weights (the probabilities, f32) of the first top_k experts of the stable
 *    descending order, as above; a weight <= 0 means the expert is skipped;
 *  - moe_experts_dev: y[r] = down_e(silu(gate_e x[r]) * up_e x[r]) for e =
 *    ids[r] (int32, an index into the E experts of the given weights; a row
 *    with an id outside [0, E) gives 0), x and y [R][H], R <= 16384.
 * Combining sum_j weight[t][j] * y(t, j) in j order (one rounding per product
 * and per sum, starting from 0) reproduces bramha_cuda_moe_mlp_dev. */
BRAMHA_API int bramha_cuda_moe_route_dev(bramha_ctx* ctx, const float* logits_dev, int64_t T, int num_experts,
                                         int top_k, int32_t* ids_dev, float* weights_dev, void* stream);
BRAMHA_API int bramha_cuda_moe_experts_dev(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down,
                                           int num_experts, const float* x_dev, const int32_t* ids_dev, int64_t R,
                                           float* y_dev, void* stream);
/* Same with host buffers, synchronous. */
BRAMHA_API int bramha_cuda_moe_mlp(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down,
                                   int num_experts, int top_k, const float* x_host, const float* logits_host,
                                   int64_t T, float* out_host, int32_t* selected_host);

/* ------------------------------------------------------- prefill GEMM path */

/* gemm_cpu (cpu_engine.rs:565-912): out[m][j] = sum_i h[m][i] * dq(w[j][i]),
 * h_block [M][K] f32 host, out [M][N] f32 host, synchronous. */
BRAMHA_API int bramha_cuda_gemm(bramha_ctx* ctx, const bramha_weight* w, const float* h_host, int64_t M,
                     float* out_host);

/* Device variant, stream-ordered: x_dev is [M][K] of `x_dtype`.  BF16 input
 * runs one tcgen05 pass (bf16 tiles, fp32 accumulation); F32 input is split
 * into bf16 hi + lo parts and runs two accumulating passes (~2^-16 relative).
 * Weights are dequantized exactly (int4 -> q-8, int8 -> q, log4 -> 2^c), so
 * the activation rounding is the only approximation. */
BRAMHA_API int bramha_cuda_gemm_dev(bramha_ctx* ctx, const bramha_weight* w, const void* x_dev, int x_dtype, int64_t M,
                         float* y_dev, void* stream);

/* Allocation-free variant of bramha_cuda_gemm_dev, for callers that cannot let
 * a library allocate device memory during a call -- for example an engine that
 * reserves all of HBM for its own weight and KV-cache pools at start-up and
 * must not grow the CUDA memory pool afterwards, or a latency-bound serving
 * path where a pool growth could block.  It has no counterpart in the
 * reference.  Same computation as bramha_cuda_gemm_dev with BF16 activations:
 * x_dev is bf16 [M][K] (16-byte aligned, K a multiple of 8), y_dev f32 [M][N],
 * stream-ordered.  Its only scratch (the per-token activation sums of the log4
 * correction) lives in a fixed device array compiled into the library, sized
 * for at most 16384 tokens: larger M is rejected with BRAMHA_ERR_UNSUPPORTED.
 * The array is held by every GPU that loads the library until exit.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture.  All calls share the one
 * array (each call overwrites the sums it reads, nothing needs to start at
 * zero): calls whose work overlaps on the GPU race with each other, so order
 * them on one stream.  Int4 and int8 weights use no scratch at all. */
BRAMHA_API int bramha_cuda_gemm_noalloc_dev(bramha_ctx* ctx, const bramha_weight* w, const void* x_dev, int64_t M,
                                            float* y_dev, void* stream);

/* Waits for `stream` (NULL = the context stream) and reports a failure that a
 * kernel recorded on the device: the tensor-core GEMV and GEMM bound every
 * wait and return BRAMHA_ERR_TIMEOUT here instead of hanging.  Host-buffer
 * calls (bramha_cuda_gemv, _matvec, _gemm, _gemv_chain, _moe_mlp, ...) check
 * this before returning. */
BRAMHA_API int bramha_cuda_stream_sync(bramha_ctx* ctx, void* stream);

/* ------------------------------------------- column sharding over several GPUs
 *
 * The reference runs every linear on one device (matvec_mul_into,
 * cpu_engine.rs:1307-1444); here a linear's output rows (its out_features)
 * can be split across the GPUs of one node, one process and one context per
 * GPU.  Each rank holds rows [N*rank/world, N*(rank+1)/world) of a sharded
 * weight; a GEMV on sharded weights (bramha_cuda_gemv_dev, _gemv_multi_dev,
 * _gemv_chain_dev, _gemv_chain; tensor-core formats LOG4, W4ZP8, W8, batch
 * 1..8) computes this rank's rows and stores them, over NVLink, straight into
 * every rank's copy of the full output -- the all-gather is part of the GEMV's
 * epilogue -- and then publishes the launch to every rank.  Before a sharded
 * GEMV reads its input it waits until every rank has published the previous
 * sharded GEMV, so a sharded GEMV may read the output of the one before it.
 * Outputs of sharded GEMVs live in a symmetric arena: every rank allocates the
 * same sizes in the same order (bramha_cuda_shard_malloc), so an output has
 * the same offset on every rank.  All ranks must issue the same sequence of
 * sharded GEMVs.  Waits are bounded (bramha_cuda_set_wait_timeout); after a
 * BRAMHA_ERR_TIMEOUT the group is unusable and must be re-created.  An output
 * buffer may be written again only after every rank has finished reading it,
 * which the ordering above guarantees for reads by the next sharded GEMV.
 * No multicast and no collective library: plain peer loads and stores.
 *
 * Set-up: each rank calls bramha_cuda_shard_handle (allocates its arena and
 * returns an IPC handle), the caller exchanges the handles between the ranks
 * (for example with torch.distributed), and each rank calls
 * bramha_cuda_shard_init with all of them. */
typedef struct bramha_ipc_handle {
    unsigned char bytes[64];
} bramha_ipc_handle;

BRAMHA_API int bramha_cuda_shard_handle(bramha_ctx* ctx, size_t arena_bytes, bramha_ipc_handle* out);

/* handles[r] is rank r's handle (world <= 8); opens the peers' arenas. */
BRAMHA_API int bramha_cuda_shard_init(bramha_ctx* ctx, int world, int rank, const bramha_ipc_handle* handles);

/* Symmetric allocation from the arena (256-byte aligned; same sizes and
 * order on every rank); *out is this rank's device pointer. */
BRAMHA_API int bramha_cuda_shard_malloc(bramha_ctx* ctx, size_t bytes, void** out);

/* Registers this rank's rows of the full packed weight (the layout and size
 * rules of bramha_cuda_register_weight, for the whole N x K weight).  A rank
 * may hold no rows (N < world). */
BRAMHA_API int bramha_cuda_register_weight_shard(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                                 const void* q, size_t q_bytes, const float* scales, size_t n_scales,
                                                 bramha_weight** out);
BRAMHA_API int bramha_cuda_register_weight_shard_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                                     const void* q_dev, size_t q_bytes, const float* scales_dev,
                                                     size_t n_scales, void* stream, bramha_weight** out);

/* First row and row count of this rank's shard of an N-row weight. */
BRAMHA_API int bramha_cuda_shard_rows(bramha_ctx* ctx, int64_t N, int64_t* row0, int64_t* rows);

/* Stream-ordered: work after it sees every rank's rows of every sharded GEMV
 * this rank has issued (a bounded wait on the ranks' publications). */
BRAMHA_API int bramha_cuda_shard_sync_dev(bramha_ctx* ctx, void* stream);

/* ------------------------------------------------------------ packers (GPU) */

/* quantize_to_int8 / quantize_to_int4 (src/models/quantization.rs:7-83) and
 * the log4 encoder this project defines, on the device, bit-exact with the
 * reference's rounding (half away from zero) and nibble order.  w_dev is
 * f32 [N][K]; q_dev receives the packed bytes, scales_dev [N] the scales. */
BRAMHA_API int bramha_cuda_quantize_dev(bramha_ctx* ctx, int fmt, int64_t N, int64_t K, const float* w_dev, void* q_dev,
                             float* scales_dev, void* stream);

/* ------------------------------------------- decode-step operations (GPU)
 *
 * The per-token operations of the reference's single-token decode
 * (src/inference/cpu_engine.rs:2819-3064) around the quantized GEMVs, so that
 * a whole decode step -- these calls and bramha_cuda_gemv_multi_dev -- can be
 * captured once in a CUDA graph and replayed token after token.  The current
 * token id and position are int32 values in device memory (token_dev,
 * pos_dev), read by the kernels when they run.  All pointers are device
 * pointers; stream NULL = the context stream; calls are asynchronous. */

/* x = table[token mod vocab] (cpu_engine.rs:2821-2825); table f32 [vocab][hidden]. */
BRAMHA_API int bramha_cuda_op_embed(bramha_ctx* ctx, const float* table_dev, int64_t vocab, int64_t hidden,
                                    const int32_t* token_dev, float* x_dev, void* stream);

/* RMSNorm (rms_norm_into, cpu_engine.rs:1292-1302): if delta_dev is given,
 * x += delta first (the residual connection, :2937-2939 / :2966-2968), then
 * out = x * (1 / sqrt(mean(x^2) + eps)) * weight.  n <= 2^24. */
BRAMHA_API int bramha_cuda_op_rmsnorm(bramha_ctx* ctx, float* x_dev, const float* delta_dev, const float* weight_dev,
                                      int64_t n, float eps, float* out_dev, void* stream);

/* q, k, v (+ optional biases, :2895-2897), half-split RoPE of q and k at the
 * position *pos_dev (apply_rope_cpu :1682-1698, theta_i = 1/base^(2i/hd)),
 * then k and v stored as row *pos_dev of the caches [max_ctx][kv_heads *
 * head_dim] (:2909).  q is rotated in place. */
BRAMHA_API int bramha_cuda_op_qkv_rope(bramha_ctx* ctx, float* q_dev, const float* k_dev, const float* v_dev,
                                       const float* bq_dev, const float* bk_dev, const float* bv_dev, int num_q_heads,
                                       int num_kv_heads, int head_dim, float rope_theta, const int32_t* pos_dev,
                                       int64_t max_ctx, float* k_cache_dev, float* v_cache_dev, void* stream);

/* Single-token grouped-query attention over cache rows 0 .. *pos_dev
 * (flash_attention_single_into, cpu_engine.rs:1450-1509); head_dim <= 128,
 * max_ctx <= 51200; out [num_q_heads * head_dim].  The tokens are split over
 * up to 64 CTAs per head (about 20 tokens of max_ctx each) whose softmax
 * statistics are combined in a fixed order; the
 * combine uses the context's GEMV workspace, so like a GEMV it runs one at a
 * time per context (stream-ordered). */
BRAMHA_API int bramha_cuda_op_attention(bramha_ctx* ctx, const float* q_dev, const float* k_cache_dev,
                                        const float* v_cache_dev, const int32_t* pos_dev, int num_q_heads,
                                        int num_kv_heads, int head_dim, int64_t max_ctx, float* out_dev, void* stream);

/* bramha_cuda_op_qkv_rope followed by bramha_cuda_op_attention in one launch
 * (same arithmetic): each query head's CTA rotates its own q and the current
 * token's k, attends over cache rows 0 .. *pos_dev - 1 plus that new row, and
 * the new k / v row is stored at row *pos_dev.  q is not modified. */
BRAMHA_API int bramha_cuda_op_rope_attention(bramha_ctx* ctx, const float* q_dev, const float* k_dev,
                                             const float* v_dev, const float* bq_dev, const float* bk_dev,
                                             const float* bv_dev, int num_q_heads, int num_kv_heads, int head_dim,
                                             float rope_theta, const int32_t* pos_dev, int64_t max_ctx,
                                             float* k_cache_dev, float* v_cache_dev, float* out_dev, void* stream);

/* out = silu(g) * u (run_mlp_into, cpu_engine.rs:2023-2026). */
BRAMHA_API int bramha_cuda_op_silu_mul(bramha_ctx* ctx, const float* g_dev, const float* u_dev, int64_t n,
                                       float* out_dev, void* stream);

/* Token selection (cpu_engine.rs:2985-3031).  greedy != 0: the repetition
 * penalty over every entry of generated[0 .. *count) (logit > 0 ? logit /
 * penalty : logit * penalty, in place), then the first maximum becomes
 * *token_dev and is appended to generated (while *count < max_generated).
 * greedy == 0 (teacher forcing: the caller writes the next token): only the
 * position advances.  Either way *pos_dev += 1. */
BRAMHA_API int bramha_cuda_op_select(bramha_ctx* ctx, float* logits_dev, int64_t vocab, int32_t* generated_dev,
                                     int32_t* count_dev, int64_t max_generated, float penalty, int greedy,
                                     int32_t* token_dev, int32_t* pos_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BRAMHA_CUDA_H */
