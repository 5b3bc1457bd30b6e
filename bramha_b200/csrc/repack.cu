// repack.cu -- device word layout of the 4-bit formats.
//
// The reference packs two codes per byte, column 2i in the high nibble and
// column 2i+1 in the low nibble (src/models/quantization.rs:74-78,
// spanda-engine/src/lib.rs:335-339).  At registration each 32-bit word
// (columns c0..c7) is rearranged in place so that the even columns c0,c2,c4,c6
// occupy bits 0-15 and the odd columns c1,c3,c5,c7 bits 16-31, nibble j of
// each half holding column 2j / 2j+1.  Column pairs (2j, 2j+1) are then 16 bits
// apart, which lets the kernels build two dequantized values with one shift
// and one logic operation (a bf16x2 pair for the tensor-core GEMM).  The
// transform is a bijection on words; padding words (zero) stay zero.
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

__global__ void repack_kernel(uint32_t* __restrict__ q, int64_t nwords) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords; i += (int64_t)gridDim.x * blockDim.x)
        q[i] = to_device_word(q[i]);
}

}  // namespace

cudaError_t launch_repack_nibbles(uint8_t* q, int64_t nbytes, cudaStream_t st) {
    if (nbytes <= 0) return cudaSuccess;
    if (nbytes % 4) return cudaErrorInvalidValue;  // rows are padded to 16 bytes
    const int64_t nwords = nbytes / 4;
    const int64_t blocks = (nwords + 255) / 256;
    repack_kernel<<<(unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8), 256, 0, st>>>(reinterpret_cast<uint32_t*>(q),
                                                                                      nwords);
    return cudaGetLastError();
}

}  // namespace bramha
