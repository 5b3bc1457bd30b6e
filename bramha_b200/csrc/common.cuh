// common.cuh -- definitions shared by the kernels and the C-ABI host code.
//
// Device weight layout (HBM), one buffer per registered weight:
//  * quantized formats (int8, int4, log4): TILE-MAJOR (repack.cu) -- 128-row
//    tiles cut into k-steps of 64 columns; block (tile t, step s) holds the 128
//    row slices of those columns contiguously (32 bytes per row for 4-bit, 64
//    for int8), so each pipeline stage is one contiguous 4 KB / 8 KB read.
//    4-bit words are rearranged (even columns in bits 0-15, odd in 16-31).
//    Rows past N and columns past K are zero.
//  * dense f32: row-major, rows padded to a 16-byte pitch.
//  * 2:4 sparse (BRAMHA_FMT_SP24_*): kept code pairs, 4-bit column pairs and
//    the K % 4 tail, row-major (sparse24.cu).
// Scales: f32 [N], one per output row.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/bramha_cuda.h"

namespace bramha {

constexpr int kMaxGemvBatch = 8;     // GEMV kernels take batch 1..8 per launch
constexpr int kMaxSegments = 8;      // weights fused into one GEMV launch

// Device status block of a context.  Kernels are handed `int* err` = &err (the
// first member); the tensor-core kernels also read the bound on their mbarrier
// waits and the test-only fault switch from the same block.
struct DevStatus {
    int err;                        // 0 = ok, else the BRAMHA_ERR_* a kernel recorded
    int fault;                      // kFault* (tests only; 0 in normal use)
    unsigned long long timeout_ns;  // bound on every mbarrier wait
};
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // 2 s
// Test-only faults: CTA 0 of the next tensor-core GEMV (or GEMM) launches
// withholds one weight copy, so the consumers' bounded waits run out.
constexpr int kFaultNone = 0;
constexpr int kFaultGemvWithholdCopy = 1;
constexpr int kFaultGemmWithholdCopy = 2;

// Bytes of one packed row (without padding) for a format.
inline int64_t row_bytes_of(int fmt, int64_t K) {
    switch (fmt) {
        case BRAMHA_FMT_F32: return K * 4;
        case BRAMHA_FMT_W8: return K;
        case BRAMHA_FMT_W4ZP8:
        case BRAMHA_FMT_LOG4: return K / 2;
        default: return -1;
    }
}
inline int64_t pitch_of(int64_t row_bytes) { return (row_bytes + 15) / 16 * 16; }

// Tile-major layout of the quantized formats.
constexpr int kTileRows = 128;   // rows per tile (= UMMA M)
constexpr int kTileK = 64;       // columns per k-step
__host__ __device__ constexpr int tile_slice_bytes(int fmt) {
    return fmt == BRAMHA_FMT_W8 ? 64 : (fmt == BRAMHA_FMT_W4ZP8 || fmt == BRAMHA_FMT_LOG4) ? 32 : 0;
}
// K here is the number of columns the packed rows hold.
__host__ __device__ constexpr int64_t k_steps(int64_t K) { return (K + kTileK - 1) / kTileK; }
__host__ __device__ constexpr int64_t row_tiles(int64_t N) { return (N + kTileRows - 1) / kTileRows; }
inline int64_t tiled_bytes(int fmt, int64_t N, int64_t K) {
    return row_tiles(N) * k_steps(K) * kTileRows * tile_slice_bytes(fmt);
}
inline bool is_tiled(int fmt) { return tile_slice_bytes(fmt) > 0; }
// Columns held by a packed row: K/2 bytes of 4-bit codes cover 2*(K/2) columns.
inline int64_t held_columns(int fmt, int64_t K) {
    return (fmt == BRAMHA_FMT_W4ZP8 || fmt == BRAMHA_FMT_LOG4) ? (K / 2) * 2 : K;
}

// 2:4 sparse formats: BRAMHA_FMT_SP24_X keeps the codes of BRAMHA_FMT_X.
inline bool is_sp24(int fmt) { return fmt >= BRAMHA_FMT_SP24_F32 && fmt <= BRAMHA_FMT_SP24_W4ZP8; }
inline int sp24_base(int fmt) { return fmt - BRAMHA_FMT_SP24_F32 + BRAMHA_FMT_F32; }

// Device view of a 2:4 sparse weight (layout in sparse24.cu).
struct Sp24Weight {
    uint8_t* vals;    // [N][ldv] kept code pairs
    int64_t ldv;      // bytes per row = Cp * sp24_value_bytes
    uint32_t* idx;    // [N][ldi] 4-bit column-pair ids, 8 groups per word
    int64_t ldi;      // words per row = Cp / 8
    float* tail;      // [N][4] codes of the K % 4 trailing columns, or null
    const float* scales;
    int64_t N, K, Cp; // Cp = groups of 4 columns per row, rounded up to 8
};
inline int64_t sp24_groups_padded(int64_t K) { return (K / 4 + 7) / 8 * 8; }
// Column pairs (a < b) of a group of four and their ids 0..5:
// (0,1) (0,2) (0,3) (1,2) (1,3) (2,3).
__host__ __device__ constexpr int sp24_pair_a(int p) { return p < 3 ? 0 : p < 5 ? 1 : 2; }
__host__ __device__ constexpr int sp24_pair_b(int p) { return p < 3 ? p + 1 : p < 5 ? p - 1 : 3; }
__host__ __device__ constexpr int sp24_pair_id(int a, int b) { return a == 0 ? b - 1 : a == 1 ? b + 1 : 5; }

// Column-shard group of a tensor-core GEMV launch (world > 1; one process per
// GPU).  The launch computes rows [row0, row0 + N) of each segment's output
// and stores them in every rank's copy of that output (peer pointers into the
// ranks' symmetric arenas, plain stores over NVLink).  Every CTA, once its
// stores are done, makes them visible system-wide (one fence) and adds 1 to
// its rank's arrival counter in every rank's arena.  Before a launch reads its
// activations it waits (bounded) until each rank's counter here has reached
// the total CTA count of that rank's sharded launches so far (`expected`,
// advanced by each launch's last CTA with every rank's grid size).
constexpr int kMaxShardWorld = 8;
struct ShardArgs {
    int world;                                    // 0 or 1: not sharded
    int rank;
    float* peer_y[kMaxSegments][kMaxShardWorld];  // segment s: rank p's copy of the full output
    int64_t row0[kMaxSegments];                   // first output row of this rank's shard
    int grid_of[kMaxShardWorld];                  // CTAs of this launch on rank p
    unsigned* arrive;                             // this rank's arrive[world]: CTAs of rank p done here
    unsigned* peer_arrive[kMaxShardWorld];        // rank p's arrive array
    unsigned* expected;                           // this rank's expected[world] (through the last launch)
    unsigned* done;                               // CTAs of the running launch that have finished
};

// One weight inside a (possibly fused) GEMV launch.
struct GemvSeg {
    const uint8_t* q;      // device weight: tile-major (quantized) or rows of pitch ldq (f32)
    const float* scales;   // [N]
    float* y;              // [batch][ldy]
    int64_t ldq;
    int64_t ldy;
    int N;
    int tile_begin;        // first tile index of this segment
};

struct GemvArgs {
    GemvSeg seg[kMaxSegments];
    const float* x;        // [batch][ldx]
    int64_t ldx;
    // Non-null: the activation is silu(x) * x_up (x_up [batch][ldx]), formed
    // while the tensor-core GEMV stages it (the SwiGLU before a down projection).
    const float* x_up;
    int nseg;
    int K;                 // activation length (columns covered by the packed row)
    int batch;
    int ldq_min;           // smallest pitch among segments (all equal for one K/format)
    int nsteps;            // vector steps per row
    int ntiles;            // tiles over all segments
    uint32_t mul[8];       // log4: powers of two moving each code to bit 23 (set by the launcher)
    int* err;              // device error word for bounded waits (tensor-core kernels)
    // K-split combine of the tensor-core GEMV (context-owned): per-split
    // partial results and per-tile arrival tickets (zero between launches)
    float* split_ws;
    int64_t split_ws_floats;
    int* split_tickets;
    int split_tickets_n;
    // L2 prefetch of the tensor-core GEMV: pf_ahead = slot pairs (even) that
    // the bulk-copy producers request from HBM into L2 ahead of their copies
    // (0 = none); pf_next_* = the weight buffers of the NEXT launch of a chain,
    // whose first pf_next_total bytes the CTAs prefetch (a slice each) once
    // their own copies are issued, so HBM keeps streaming across the launch
    // boundary.
    int pf_ahead;
    // Non-null norm_w (CUDA-core GEMV, batch 1): the activation is the RMSNorm
    // of r = x + delta (delta may be null) with weight norm_w and epsilon eps,
    // computed exactly as launch_rmsnorm does; r is also stored to x_out (when
    // non-null; it must not overlap x or delta).
    const float* norm_w;
    const float* delta;
    float* x_out;
    float eps;
    int pf_next_n;
    const uint8_t* pf_next_ptr[kMaxSegments];
    int64_t pf_next_bytes[kMaxSegments];
    int64_t pf_next_total;
    int evict_first;       // weight copies marked first to be evicted from L2
    int split_cost;        // K-split plan: cost of a split launch, in eighths of a 64-column block
    int cc_depth;          // CUDA-core GEMV: CTAs per SM its K split aims for (1 = no split unless tiles are few)
    ShardArgs shard;       // column-shard group (shard.world > 1), tensor-core GEMV only
};

constexpr int64_t kSplitWsFloats = 8 << 20;   // 32 MB of partial results per context
constexpr int kSplitTickets = 1 << 18;         // K-split arrival counters (4 per tile of a launch)

// CUDA-core GEMV for dense f32 weights (gemv_f32.cu).
cudaError_t launch_gemv_f32(const GemvArgs& a, int num_sms, cudaStream_t stream);

// Reference row-major packed rows (row_bytes per row) -> tile-major device
// layout of tiled_bytes(fmt, N, held_columns(fmt, K)) bytes (repack.cu).
cudaError_t launch_tile_weights(int fmt, const uint8_t* src, int64_t row_bytes, int64_t N, int64_t K, uint8_t* dst,
                                cudaStream_t stream);

// Prefill GEMM on tcgen05 (gemm_tcgen05.cu).  K = columns held by the packed
// rows; x is bf16 (x_is_f32 = 0) or f32 (split into bf16 hi + lo).  GEMMs with
// fewer tiles than SMs are K-split through ws / tickets (NULL = never).
cudaError_t launch_gemm_tcgen05(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N, int64_t K,
                                const void* x, int x_is_f32, int64_t ldx, int64_t M, float* y, int64_t ldy, int* err,
                                float* ws, int64_t ws_floats, int* tickets, int64_t n_tickets, cudaStream_t stream);

// Several weights (same format, same K) applied to one x: the activation
// copy and per-token sums are prepared once for all of them.
struct GemmOut {
    const uint8_t* q;      // tile-major weight
    const float* scales;
    int64_t N;
    float* y;              // [M][ldy]
    int64_t ldy;
};
cudaError_t launch_gemm_tcgen05_multi(int fmt, int n, const GemmOut* outs, int64_t K, const void* x, int x_is_f32,
                                      int64_t ldx, int64_t M, int* err, float* ws, int64_t ws_floats, int* tickets,
                                      int64_t n_tickets, cudaStream_t stream);

// bf16-activation GEMM that allocates nothing: the log4 per-token sums go to
// `rowsum_scratch` (at least M floats, caller-owned); x must be 16-byte
// aligned with a row pitch that is a multiple of 8 elements.
cudaError_t launch_gemm_tcgen05_bf16_noalloc(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N,
                                             int64_t K, const void* x, int64_t ldx, int64_t M, float* y,
                                             int64_t ldy, int* err, float* rowsum_scratch, cudaStream_t stream);

// Fixed scratch of bramha_cuda_gemm_noalloc_dev (noalloc.cu).
constexpr int64_t kNoAllocMaxTokens = 16384;
cudaError_t noalloc_rowsum_scratch(int device, float** out);

// CUDA-core batch-1 GEMV of the tiled formats for latency-bound (small)
// launches (gemv_cc.cu); eligible() says whether a launch should take it.
bool gemv_cc_eligible(int fmt, const GemvArgs& a);
cudaError_t launch_gemv_cc(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream);

// A chain of dependent tensor-core GEMVs in one persistent cooperative launch
// (gemv_chain.cu): ops[j] describes launch j as launch_gemv_tc would take it
// (one format and batch for the whole chain); the program owns its device op
// table and per-op completion counters and uses the caller's K-split
// workspace and tickets.
struct ChainProgram;
cudaError_t chain_program_create(int fmt, int batch, int nops, const GemvArgs* ops, int num_sms, int split_cost,
                                 float* ws, int64_t ws_floats, int* tickets, int n_tickets, ChainProgram** out);
cudaError_t chain_program_run(ChainProgram* prog, int* err, int64_t lookahead_bytes, cudaStream_t stream);
void chain_program_destroy(ChainProgram* prog);
// Per-op, per-CTA %globaltimer stamps of the next runs ([nops][grid][4]).
cudaError_t chain_program_trace(ChainProgram* prog, int on);
cudaError_t chain_program_read_trace(ChainProgram* prog, unsigned long long* out, size_t n, int* grid);

// Tensor-core GEMV for the quantized formats, batch 1..8 (gemv_tc.cu).
cudaError_t launch_gemv_tc(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream);
// Shard-group bookkeeping without a GEMV (gemv_tc.cu): publish = 1 takes part
// in a sharded launch in which this rank has no rows (one CTA: waits for the
// previous launch, then arrives); publish = 0 waits until every rank's CTAs of
// every sharded launch so far have arrived, so later work sees every shard.
cudaError_t launch_shard_signal(const ShardArgs& s, int* err, int publish, cudaStream_t stream);
// CTAs a tensor-core GEMV launch of `ntiles` 128-row tiles over K columns uses
// (the grid a rank's sharded launch will have; gemv_tc.cu).
int gemv_tc_grid(int fmt, int batch, int ntiles, int K, int num_sms, int split_cost, int64_t split_ws_floats,
                 int split_tickets_n);

// Decode-step operations (decode.cu); token and position live in device memory.
cudaError_t launch_embed(const float* table, int64_t vocab, int64_t hidden, const int32_t* token, float* x,
                         cudaStream_t stream);
cudaError_t launch_rmsnorm(float* x, const float* delta, const float* w, int64_t n, float eps, float* out,
                           cudaStream_t stream);
cudaError_t launch_qkv_rope(float* q, const float* k, const float* v, const float* bq, const float* bk,
                            const float* bv, int nq, int nkv, int hd, float rope_theta, const int32_t* pos,
                            int64_t max_ctx, float* k_cache, float* v_cache, cudaStream_t stream);
// (ws / tickets: the context's K-split workspace and tickets, for the per-head
// combine of the attention's token splits; tickets are left at zero)
cudaError_t launch_attention(const float* q, const float* k_cache, const float* v_cache, const int32_t* pos, int nq,
                             int nkv, int hd, int64_t max_ctx, float* ws, int64_t ws_floats, int* tickets,
                             int64_t n_tickets, float* out, cudaStream_t stream);
cudaError_t launch_rope_attention(const float* q, const float* k, const float* v, const float* bq, const float* bk,
                                  const float* bv, float rope_theta, const int32_t* pos, int64_t max_ctx,
                                  float* k_cache, float* v_cache, int nq, int nkv, int hd, float* ws,
                                  int64_t ws_floats, int* tickets, int64_t n_tickets, float* out,
                                  cudaStream_t stream);
cudaError_t launch_silu_mul(const float* g, const float* u, int64_t n, float* out, cudaStream_t stream);
cudaError_t launch_select(float* logits, int64_t vocab, int32_t* generated, int32_t* count, int64_t max_gen,
                          float penalty, int greedy, int32_t* token, int32_t* pos, cudaStream_t stream);

// 2:4 sparse GEMV of one activation row x (16-byte aligned) into y, and the
// registration-time selection from a reference-layout weight (sparse24.cu).
int sp24_value_bytes(int base_fmt);
cudaError_t launch_sp24_gemv(int base_fmt, const Sp24Weight& w, const float* x, float* y, float* ws,
                             int64_t ws_floats, int* tickets, int n_tickets, int num_sms, cudaStream_t stream);
cudaError_t launch_sp24_prune(int base_fmt, const uint8_t* src, int64_t row_bytes, const Sp24Weight& w,
                              cudaStream_t stream);

// Grouped tcgen05 GEMM over a device tile table (gemm_tcgen05.cu); the MoE
// path (moe.cu) builds the tables with kGemmGroupTok tokens per tile.
constexpr int kGemmGroupTok = 64;
cudaError_t launch_gemm_tcgen05_grouped(int fmt, const uint8_t* q, const float* scales, int64_t N_group, int64_t K,
                                        const float* x, int64_t ldx, int64_t M, float* y, int64_t ldy,
                                        const int4* tiles, const int* ntiles_dev, int64_t max_tiles, int* err,
                                        cudaStream_t stream);

// MoE expert MLP of T tokens (moe.cu): routing (softmax, stable top-k),
// gather, grouped gate+up GEMM, SiLU * up, grouped down GEMM, weighted
// combine.  gate_up: tile-major [E][2I][H] (gate rows then up rows per
// expert), down: [E][H][I]; 2I and H multiples of 128.
struct MoeWeights {
    int fmt;
    const uint8_t* gate_up;
    const float* gate_up_scales;
    const uint8_t* down;
    const float* down_scales;
    int64_t E, H, I;
};
cudaError_t launch_moe_mlp(const MoeWeights& w, int top_k, const float* x, const float* logits, int64_t T, float* out,
                           int32_t* selected, int* err, cudaStream_t stream);
// Expert outputs of rows routed by the caller (ids[r] in [0, E); others give 0),
// and the routing alone (sorted expert ids and probabilities, [T][min(k, E)]).
cudaError_t launch_moe_experts(const MoeWeights& w, const float* x, const int32_t* ids, int64_t R, float* y, int* err,
                               cudaStream_t stream);
cudaError_t launch_moe_route(const float* logits, int64_t T, int64_t E, int top_k, int32_t* ids, float* weights,
                             cudaStream_t stream);
constexpr int64_t kMoeMaxAssignments = 16384;  // T * top_k per call (routing state in shared memory)
constexpr int64_t kMoeMaxExperts = 1024;

// GPU packers (quant.cu).
cudaError_t launch_quantize(int fmt, int64_t N, int64_t K, const float* w, uint8_t* q, float* scales,
                            cudaStream_t stream);

}  // namespace bramha
