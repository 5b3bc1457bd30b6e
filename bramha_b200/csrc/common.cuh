// common.cuh -- definitions shared by the kernels and the C-ABI host code.
//
// Device weight layout (HBM): one buffer per registered weight, rows in the
// reference's order and byte layout (src/models/quantization.rs:41-83 for
// nibbles: byte i of a row = column 2i in the high nibble, column 2i+1 in the
// low nibble), each row padded to a pitch `ldq` that is a multiple of 16 bytes
// so every 16-byte vector load is aligned.  Padding bytes are zero; the kernels
// read the matching activation columns as zero, so padding contributes nothing.
// Scales: f32 [N], one per output row.
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
};

// Launch a GEMV over the segments; chooses the tiling from the shape.
cudaError_t launch_gemv(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream);

// GPU packers (quant.cu).
cudaError_t launch_quantize(int fmt, int64_t N, int64_t K, const float* w, uint8_t* q, float* scales,
                            cudaStream_t stream);

}  // namespace bramha
