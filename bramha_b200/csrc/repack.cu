// repack.cu -- device layout of the quantized formats (done once, at registration).
//
// The reference stores a quantized weight row-major: row j, then row j+1, with
// two 4-bit codes per byte, column 2i in the high nibble and column 2i+1 in the
// low nibble (src/models/quantization.rs:74-78, spanda-engine/src/lib.rs:335-339),
// or one int8 per byte (quantization.rs:7-38).
//
// On the device the weight is TILE-MAJOR: 128-row tiles, each cut into k-steps
// of 64 columns, and each (tile, k-step) block stored as 128 consecutive row
// slices:
//     block(t, s) = rows 128t .. 128t+127, columns 64s .. 64s+63
//     offset      = (t * ksteps + s) * 128 * slice,  slice = 32 B (4-bit) / 64 B (int8)
// so every pipeline stage of the kernels is ONE contiguous 4 KB (8 KB) read:
// a single bulk copy, sequential DRAM pages.  Rows past N and columns past K
// are zero (the kernels drop those rows and see zero activations there).
//
// 4-bit words are also rearranged inside each 32-bit word (columns c0..c7):
// even columns c0,c2,c4,c6 in bits 0-15, odd columns c1,c3,c5,c7 in bits 16-31,
// nibble j of each half = column 2j / 2j+1.  A column pair is then 16 bits
// apart: one shift and one logic op give a bf16x2 pair; one mask gives four
// codes as bytes (c0, c4, c1, c5) / (c2, c6, c3, c7).
//
// int8 row slices (64 B) are stored in the tensor cores' 64-byte-swizzle
// order, so a block is an MMA operand as it lands in shared memory: the
// 16-byte chunk j of row r sits at chunk position j ^ ((r >> 1) & 3).
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {

__host__ __device__ inline uint32_t to_device_word(uint32_t w) {
    const uint32_t ev = (w >> 4) & 0x0F0F0F0Fu;  // byte k low nibble = column 2k
    const uint32_t od = w & 0x0F0F0F0Fu;         // byte k low nibble = column 2k+1
    const uint32_t e = (ev | (ev >> 4));
    const uint32_t o = (od | (od >> 4));
    const uint32_t e16 = (e & 0xFFu) | ((e >> 8) & 0xFF00u);
    const uint32_t o16 = (o & 0xFFu) | ((o >> 8) & 0xFF00u);
    return e16 | (o16 << 16);
}

// One thread per 32-bit word of the tiled buffer.  `src` is the reference
// row-major layout with `row_bytes` bytes per row (no alignment assumed).
__global__ void tile_kernel(const uint8_t* __restrict__ src, int64_t row_bytes, int64_t N, int64_t ksteps,
                            int slice, int nibbles, uint32_t* __restrict__ dst, int64_t nwords) {
    const int words_per_slice = slice / 4;
    for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < nwords; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t wi = o % words_per_slice;
        const int64_t row_in_tile = (o / words_per_slice) % kTileRows;
        const int64_t block = o / (words_per_slice * kTileRows);
        const int64_t tile = block / ksteps, step = block % ksteps;
        const int64_t row = tile * kTileRows + row_in_tile;
        int64_t b0 = step * slice + wi * 4;  // source byte offset in the row
        if (!nibbles) {                      // int8: chunk position p holds chunk p ^ ((r >> 1) & 3)
            const int64_t j = (wi >> 2) ^ ((row_in_tile >> 1) & 3);
            b0 = step * slice + j * 16 + (wi & 3) * 4;
        }
        uint32_t w = 0;
        if (row < N) {
            const uint8_t* r = src + row * row_bytes;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (b0 + i < row_bytes) w |= (uint32_t)r[b0 + i] << (8 * i);
        }
        dst[o] = nibbles ? to_device_word(w) : w;
    }
}

}  // namespace

cudaError_t launch_tile_weights(int fmt, const uint8_t* src, int64_t row_bytes, int64_t N, int64_t K, uint8_t* dst,
                                cudaStream_t st) {
    const int slice = tile_slice_bytes(fmt);
    if (slice <= 0) return cudaErrorInvalidValue;
    const int64_t nbytes = tiled_bytes(fmt, N, K);
    if (nbytes == 0) return cudaSuccess;
    const int64_t nwords = nbytes / 4;
    const int64_t blocks = (nwords + 255) / 256;
    tile_kernel<<<(unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8), 256, 0, st>>>(
        src, row_bytes, N, k_steps(K), slice, fmt != BRAMHA_FMT_W8, reinterpret_cast<uint32_t*>(dst), nwords);
    return cudaGetLastError();
}

}  // namespace bramha
