// gemv_cc.cu -- batch-1 GEMV of the tiled quantized formats on the CUDA cores,
// for weights small enough that a launch is latency-bound (the decode-step
// linears of small models, the q|k|v and o projections of 7B-class layers).
//
// Same result definition as the reference's matvec_mul_into
// (src/inference/cpu_engine.rs:1307-1444), y_j = s_j * sum_k x_k * code(w_jk):
//   int4 (quantize_to_int4)  code = q - 8
//   int8 (quantize_to_int8)  code = q
//   log4 (dequantize_log4)   code = 2^c - 1
// accumulated in fp32 (the tensor-core GEMV carries the activations as 8-bit
// terms instead; both are within the path's 1e-3 tolerance of the oracle).
//
// A CTA takes one 128-row tile and one K range (a "split") of nb 64-column
// blocks; two threads per row each own 32 columns of every block.  The CTA's
// packed weights do not depend on the previous kernel, so they are loaded into
// registers before the programmatic-launch dependency wait; after it the CTA
// only stages its activations, multiplies and adds.  With more than one split
// each CTA writes its row partials to the context workspace and takes a tile
// ticket; the last split of a tile adds the partials in split order and writes
// y (deterministic), then resets the ticket.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {

constexpr int kCcThreads = 256;  // 2 threads per row of a 128-row tile
constexpr int kCcNormMaxK = 1024;  // a fused RMSNorm keeps the whole residual in shared memory
constexpr int kCcMaxBlocks = 16;  // 64-column blocks per CTA (registers: 4-bit 4 words/block, int8 8)

struct CcParams {
    GemvSeg seg[kMaxSegments];
    const float* x;
    int nseg;
    int K;         // columns held by the packed rows
    int ksteps;    // 64-column blocks per row
    int ntiles;
    int ksplit;    // splits per tile
    int bps;       // blocks per split
    float* ws;     // [ntiles][ksplit][128] partials (ksplit > 1)
    int* tickets;  // [ntiles], zero between launches
    // RMSNorm of r = x + delta as the activation (GemvArgs::norm_w); r -> x_out
    const float* norm_w;
    const float* delta;
    float* x_out;
    float eps;
};

template <int FMT>
struct CcFmt {
    static constexpr int kSlice = FMT == BRAMHA_FMT_W8 ? 64 : 32;  // bytes per row per block
    static constexpr int kWords = kSlice / 8;                       // words per thread per block (half a row)
};

__device__ __forceinline__ float nib_float(uint32_t n) {  // exact float of a 4-bit code
    return __uint_as_float(0x4B000000u | n) - 8388608.0f;
}
__device__ __forceinline__ float pow2_minus1(uint32_t c) {  // 2^c - 1, exact for c <= 15
    return __uint_as_float((c + 127u) << 23) - 1.0f;
}

template <int FMT>
__device__ __forceinline__ float block_dot(const uint32_t (&w)[CcFmt<FMT>::kWords], const float* xs, int half,
                                           int row) {
    float acc = 0.f;
    if constexpr (FMT == BRAMHA_FMT_W8) {
        // the thread's 32 columns: chunks 2*half and 2*half + 1 of the row (16 columns each)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float* xc = xs + 16 * (2 * half + c);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t v = w[4 * c + j];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float q = (float)(int8_t)(v >> (8 * b));
                    acc = fmaf(xc[4 * j + b], q, acc);
                }
            }
        }
    } else {
        // word j of the half-row covers columns 32*half + 8j .. +7: nibble i of the low
        // half is column 2i, nibble i of the high half column 2i + 1
        const float* xc = xs + 32 * half;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t v = w[j];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t lo = (v >> (4 * i)) & 0xFu, hi = (v >> (16 + 4 * i)) & 0xFu;
                float a, b;
                if constexpr (FMT == BRAMHA_FMT_LOG4) {
                    a = pow2_minus1(lo);
                    b = pow2_minus1(hi);
                } else {
                    a = nib_float(lo) - 8.0f;
                    b = nib_float(hi) - 8.0f;
                }
                acc = fmaf(xc[8 * j + 2 * i], a, acc);
                acc = fmaf(xc[8 * j + 2 * i + 1], b, acc);
            }
        }
    }
    (void)row;
    return acc;
}

// 1 / sqrt(mean(r^2) + eps) of r = x + delta over the K (<= 1024) columns,
// with the additions in exactly the order of the RMSNorm kernel (launch_rmsnorm,
// 1024 threads: thread t sums columns t, t + 1024, ..., warp trees, then a tree
// over the 32 warp sums): thread t of this CTA stands for threads t + 256j of
// that kernel.  r is left in rs[] for the staging.  Every thread returns the
// same value.
__device__ float rms_inv(const CcParams& p, float* red, float* rs) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 1024 / kCcThreads; ++j) {
        const int vt = threadIdx.x + kCcThreads * j;
        float ss = 0.f;
        if (vt < p.K) {
            float v = __ldcg(p.x + vt);
            if (p.delta) v = __fadd_rn(v, __ldcg(p.delta + vt));
            rs[vt] = v;
            ss = __fadd_rn(ss, __fmul_rn(v, v));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[vt >> 5] = ss;
    }
    __syncthreads();
    float v = red[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float var = v / (float)p.K;
    return 1.0f / sqrtf(__fadd_rn(var, p.eps));
}

template <int FMT>
__device__ __forceinline__ void load_block(const uint8_t* blk, int row, int half, uint32_t (&w)[CcFmt<FMT>::kWords]) {
    if constexpr (FMT == BRAMHA_FMT_W8) {
        // 16-byte chunk j of a row is stored at chunk j ^ ((row >> 1) & 3) (repack.cu)
        const int sw = (row >> 1) & 3;
        const uint8_t* r = blk + row * 64;
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(r + 16 * ((2 * half) ^ sw)));
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(r + 16 * ((2 * half + 1) ^ sw)));
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
        w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(blk + row * 32 + 16 * half));
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    }
}

template <int FMT, bool NORM>
__global__ void __launch_bounds__(kCcThreads) cc_gemv_kernel(const __grid_constant__ CcParams p) {
    using Fm = CcFmt<FMT>;
    __shared__ float xs[kCcMaxBlocks * kTileK];
    __shared__ float red[32];
    __shared__ float rs[NORM ? kCcNormMaxK : 1];  // fused RMSNorm: the residual r = x + delta
    __shared__ int last;
    const int tile = blockIdx.x / p.ksplit, split = blockIdx.x - tile * p.ksplit;
    const int row = threadIdx.x >> 1, half = threadIdx.x & 1;
    int si = 0;
    while (si + 1 < p.nseg && p.seg[si + 1].tile_begin <= tile) ++si;
    const GemvSeg& sg = p.seg[si];
    const int grow = (tile - sg.tile_begin) * kTileRows + row;
    const int b0 = split * p.bps;
    const int nb = min(p.bps, p.ksteps - b0);
    const uint8_t* base = sg.q + ((int64_t)(tile - sg.tile_begin) * p.ksteps + b0) * (kTileRows * Fm::kSlice);
    constexpr int kBlockBytes = kTileRows * Fm::kSlice;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // weights (immutable) before the dependency wait
    uint32_t w[kCcMaxBlocks][Fm::kWords];
    const int n0 = min(nb, kCcMaxBlocks);
#pragma unroll
    for (int i = 0; i < kCcMaxBlocks; ++i)
        if (i < n0) load_block<FMT>(base + (int64_t)i * kBlockBytes, row, half, w[i]);
    const float sc = grow < sg.N ? __ldg(sg.scales + grow) : 0.f;
    // fused RMSNorm: this thread's norm weights of the staging loop below (one
    // chunk: K <= 1024), also immutable
    constexpr int kNw = NORM ? kCcNormMaxK / kCcThreads : 1;
    float nwr[kNw];
#pragma unroll
    for (int u = 0; u < kNw; ++u) {
        const int j = threadIdx.x + u * kCcThreads, col = b0 * kTileK + j;
        nwr[u] = NORM && j < n0 * kTileK && col < p.K ? __ldg(p.norm_w + col) : 0.f;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float rinv = 0.f;
    if constexpr (NORM) rinv = rms_inv(p, red, rs);  // (its barrier also publishes rs)

    float acc = 0.f;
    for (int c0 = 0; c0 < nb; c0 += kCcMaxBlocks) {
        const int cn = min(nb - c0, kCcMaxBlocks);
        const int col0 = (b0 + c0) * kTileK;
        if (c0 > 0) {
            __syncthreads();  // the previous chunk's activations are no longer read
#pragma unroll
            for (int i = 0; i < kCcMaxBlocks; ++i)
                if (i < cn) load_block<FMT>(base + (int64_t)(c0 + i) * kBlockBytes, row, half, w[i]);
        }
#pragma unroll 4
        for (int u = 0, j = threadIdx.x; j < cn * kTileK; ++u, j += kCcThreads) {
            const int col = col0 + j;
            float v = 0.f;
            if (col < p.K) {
                if constexpr (NORM) {  // r = x + delta, then r * rinv * w as the RMSNorm kernel rounds it
                    v = rs[col];   // (one chunk: u < kNw)
                    if (p.x_out && tile == 0) p.x_out[col] = v;  // each column once: the splits of tile 0
                    float w = 0.f;
#pragma unroll
                    for (int q = 0; q < kNw; ++q)
                        if (q == u) w = nwr[q];
                    v = __fmul_rn(__fmul_rn(v, rinv), w);
                } else {
                    v = __ldcg(p.x + col);  // written by the previous kernel: L2, not L1
                }
            }
            xs[j] = v;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kCcMaxBlocks; ++i)
            if (i < cn) acc += block_dot<FMT>(w[i], xs + i * kTileK, half, row);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);  // the row's two halves

    if (p.ksplit == 1) {
        if (half == 0 && grow < sg.N) sg.y[grow] = acc * sc;
        return;
    }
    float* part = p.ws + (int64_t)tile * p.ksplit * kTileRows;
    if (half == 0) part[split * kTileRows + row] = acc;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&p.tickets[tile], 1) == p.ksplit - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (half == 0) {
        // partials added in split order, 16 loads in flight (at most 16 splits)
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = k < p.ksplit ? __ldcg(part + k * kTileRows + row) : 0.f;
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (k < p.ksplit) s += v[k];
        if (grow < sg.N) sg.y[grow] = s * sc;
    }
    if (threadIdx.x == 0) p.tickets[tile] = 0;  // ready for the next launch
}

template <int FMT>
cudaError_t launch_fmt(const CcParams& p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)(p.ntiles * p.ksplit));
    cfg.blockDim = dim3(kCcThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.norm_w) return cudaLaunchKernelEx(&cfg, cc_gemv_kernel<FMT, true>, p);
    return cudaLaunchKernelEx(&cfg, cc_gemv_kernel<FMT, false>, p);
}

}  // namespace

// AUTO takes the CUDA-core GEMV at batch 1 for short rows (K <= 1024) and at
// most 8 MB of packed weights per launch.  Measured on B200 (graph of 20
// dependent launches, log4): the Qwen2-0.5B q|k|v 4.5 vs 5.8 us (tensor cores),
// o 4.6 vs 5.5, gate|up 8.0 vs 14.3; with long rows (0.5B down, K = 4864: 8.2 vs
// 5.8) and at 7B sizes (q 9.7 vs 7.3) the tensor-core GEMV is faster.
constexpr int64_t kCcMaxBytes = 8ll << 20;
constexpr int kCcMaxK = 1024;
constexpr int kCcMaxSplit = 16;  // the last CTA of a tile adds the partials (16 loads in flight)
static_assert(kCcMaxSplit <= 16, "the combine loads at most 16 partials at once");

bool gemv_cc_eligible(int fmt, const GemvArgs& a) {
    if (!is_tiled(fmt) || a.batch != 1 || a.nseg < 1 || a.K > kCcMaxK) return false;
    int64_t tiles = 0;
    for (int i = 0; i < a.nseg; ++i) tiles += row_tiles(a.seg[i].N);
    const int64_t bytes = tiles * k_steps(a.K) * kTileRows * tile_slice_bytes(fmt);
    return bytes <= kCcMaxBytes && a.split_ws && a.split_tickets && tiles <= a.split_tickets_n;
}

// Splits: enough CTAs to cover the SMs a.cc_depth deep (default 4; CTAs are
// small), at least one block per split and at most kCcMaxSplit; a workspace
// slot per (tile, split, row).
cudaError_t launch_gemv_cc(int fmt, const GemvArgs& a, int num_sms, cudaStream_t st) {
    CcParams p = {};
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        if ((reinterpret_cast<uintptr_t>(a.seg[i].q) & 15) != 0) return cudaErrorInvalidValue;
        p.seg[i] = a.seg[i];
        p.seg[i].tile_begin = ntiles;
        ntiles += (int)row_tiles(a.seg[i].N);
    }
    if (ntiles <= 0 || a.K <= 0) return cudaErrorInvalidValue;
    p.x = a.x;
    p.nseg = a.nseg;
    p.K = a.K;
    p.ksteps = (int)k_steps(a.K);
    p.ntiles = ntiles;
    const int64_t want = (int64_t)(a.cc_depth > 0 ? a.cc_depth : 4) * num_sms;
    int ks = (int)((want + ntiles - 1) / ntiles);
    if (ks > p.ksteps) ks = p.ksteps;
    if (ks > kCcMaxSplit) ks = kCcMaxSplit;
    if (ks < 1) ks = 1;
    const int64_t max_ks = a.split_ws_floats / ((int64_t)ntiles * kTileRows);
    if (ks > max_ks) ks = (int)(max_ks < 1 ? 1 : max_ks);
    p.bps = (p.ksteps + ks - 1) / ks;
    p.ksplit = (p.ksteps + p.bps - 1) / p.bps;
    p.ws = a.split_ws;
    p.tickets = a.split_tickets;
    if (a.norm_w && a.K > kCcNormMaxK) return cudaErrorInvalidValue;
    p.norm_w = a.norm_w;
    p.delta = a.delta;
    p.x_out = a.x_out;
    p.eps = a.eps;
    switch (fmt) {
        case BRAMHA_FMT_LOG4: return launch_fmt<BRAMHA_FMT_LOG4>(p, st);
        case BRAMHA_FMT_W4ZP8: return launch_fmt<BRAMHA_FMT_W4ZP8>(p, st);
        case BRAMHA_FMT_W8: return launch_fmt<BRAMHA_FMT_W8>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bramha
