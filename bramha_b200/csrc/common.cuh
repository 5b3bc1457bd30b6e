// common.cuh -- definitions shared by the kernels and the C-ABI host code.
//
// Device weight layout (HBM): one buffer per registered weight, rows in the
// reference's order, each row padded to a pitch `ldq` that is a multiple of 16
// bytes so every 16-byte vector load is aligned.  Padding bytes are zero; the
// kernels read the matching activation columns as zero, so padding contributes
// nothing.  Int8 and f32 rows keep the reference's byte layout; the two 4-bit
// formats are rearranged inside each 32-bit word (repack.cu): even columns in
// bits 0-15, odd columns in bits 16-31.  Scales: f32 [N], one per output row.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/bramha_cuda.h"

namespace bramha {

constexpr int kMaxGemvBatch = 8;     // CUDA-core GEMV handles batch 1..8
constexpr int kMaxSegments = 8;      // weights fused into one GEMV launch

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

// One weight inside a (possibly fused) GEMV launch.
struct GemvSeg {
    const uint8_t* q;      // device rows, pitch ldq
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
    int nseg;
    int K;                 // activation length (columns covered by the packed row)
    int batch;
    int ldq_min;           // smallest pitch among segments (all equal for one K/format)
    int nsteps;            // vector steps per row
    int ntiles;            // tiles over all segments
    uint32_t mul[8];       // log4: powers of two moving each code to bit 23 (set by the launcher)
};

// Launch a GEMV over the segments; chooses the tiling from the shape.
cudaError_t launch_gemv(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream);

// Rearranges 4-bit rows into the device word layout, in place (repack.cu).
cudaError_t launch_repack_nibbles(uint8_t* q, int64_t nbytes, cudaStream_t stream);

// Prefill GEMM on tcgen05 (gemm_tcgen05.cu).  K = columns held by the packed
// rows; x is bf16 (x_is_f32 = 0) or f32 (split into two bf16 passes).
cudaError_t launch_gemm_tcgen05(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N, int64_t K,
                                const void* x, int x_is_f32, int64_t ldx, int64_t M, float* y, int64_t ldy, int* err,
                                cudaStream_t stream);

// bf16-activation GEMM that allocates nothing: the log4 per-token sums go to
// `rowsum_scratch` (at least M floats, caller-owned); x must be 16-byte
// aligned with a row pitch that is a multiple of 8 elements.
cudaError_t launch_gemm_tcgen05_bf16_noalloc(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N,
                                             int64_t K, const void* x, int64_t ldx, int64_t M, float* y,
                                             int64_t ldy, int* err, float* rowsum_scratch, cudaStream_t stream);

// Fixed scratch of bramha_cuda_gemm_noalloc_dev (noalloc.cu).
constexpr int64_t kNoAllocMaxTokens = 16384;
cudaError_t noalloc_rowsum_scratch(int device, float** out);

// GPU packers (quant.cu).
cudaError_t launch_quantize(int fmt, int64_t N, int64_t K, const float* w, uint8_t* q, float* scales,
                            cudaStream_t stream);

}  // namespace bramha
