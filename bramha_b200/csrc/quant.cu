// quant.cu -- device packers, bit-exact with the reference quantizers.
//
//  quantize_to_int8  src/models/quantization.rs:7-38
//  quantize_to_int4  src/models/quantization.rs:41-83
//  log4 encoder      defined by this project (the reference only has the
//                    decoder, spanda-engine/src/lib.rs:332-342): per-row scale
//                    max|w| / 32767, nearest code, ties to the lower code.
//
// One CTA per row.  All arithmetic uses explicitly rounded intrinsics
// (__fdiv_rn, __fmul_rn, __fsub_rn) so no multiply-add is ever contracted and
// every value is the IEEE result the reference's f32 code produces.  Rounding
// is half away from zero, like Rust's f32::round.
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {

constexpr int kThreads = 256;

// Rust `f32 as u8` / `as i8`: saturating, NaN -> 0.
__device__ __forceinline__ uint32_t rust_as_u8(float v) {
    if (isnan(v) || v <= 0.f) return 0u;
    if (v >= 255.f) return 255u;
    return (uint32_t)v;
}
__device__ __forceinline__ int rust_as_i8(float v) {
    if (isnan(v)) return 0;
    if (v <= -128.f) return -128;
    if (v >= 127.f) return 127;
    return (int)v;
}
// Rust f32::round: nearest integer, halves away from zero.  Built from the
// exact primitives trunc and subtract (x - trunc(x) is exact in fp32), so
// values just below a half (e.g. 0.49999997) can never round up.
__device__ __forceinline__ float round_half_away(float x) {
    float t = truncf(x);
    const float d = __fsub_rn(x, t);
    if (fabsf(d) >= 0.5f) t = __fadd_rn(t, copysignf(1.0f, x));
    return t;
}
// Rust f32::clamp (NaN passes through).
__device__ __forceinline__ float rclamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

// max |w| over a row; NaN never wins, as in `if abs > max_abs`.
__device__ float row_max_abs(const float* row, int64_t K) {
    float m = 0.f;
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x) {
        const float a = fabsf(row[i]);
        if (a > m) m = a;
    }
    __shared__ float red[kThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, m, o);
        if (t > m) m = t;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) {
            const float t = __shfl_xor_sync(0xffffffffu, m, o);
            if (t > m) m = t;
        }
        if (threadIdx.x == 0) red[0] = m;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kThreads) quant_int8_kernel(const float* __restrict__ w, int64_t K,
                                                              int8_t* __restrict__ q, float* __restrict__ scales) {
    const int64_t j = blockIdx.x;
    const float* row = w + j * K;
    const float m = row_max_abs(row, K);
    const float scale = (m == 0.f) ? 1.0f : __fdiv_rn(m, 127.0f);
    if (threadIdx.x == 0) scales[j] = scale;
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x)
        q[j * K + i] = (int8_t)rust_as_i8(rclamp(round_half_away(__fdiv_rn(row[i], scale)), -127.f, 127.f));
}

__global__ void __launch_bounds__(kThreads) quant_int4_kernel(const float* __restrict__ w, int64_t K,
                                                              uint8_t* __restrict__ q, float* __restrict__ scales) {
    const int64_t j = blockIdx.x;
    const int64_t half = K / 2;
    const float* row = w + j * K;
    const float m = row_max_abs(row, K);
    const float scale = (m == 0.f) ? 1.0f : __fdiv_rn(m, 7.0f);
    if (threadIdx.x == 0) scales[j] = scale;
    for (int64_t i = threadIdx.x; i < half; i += blockDim.x) {
        const uint32_t q1 = rust_as_u8(__fadd_rn(rclamp(round_half_away(__fdiv_rn(row[2 * i], scale)), -7.f, 7.f), 8.0f));
        const uint32_t q2 =
            rust_as_u8(__fadd_rn(rclamp(round_half_away(__fdiv_rn(row[2 * i + 1], scale)), -7.f, 7.f), 8.0f));
        q[j * half + i] = (uint8_t)(((q1 << 4) & 0xFFu) | (q2 & 0x0Fu));
    }
}

__device__ __forceinline__ uint32_t log4_code(float a, const float* d) {
    uint32_t best = 0;
    float best_err = fabsf(__fsub_rn(a, d[0]));
#pragma unroll
    for (uint32_t c = 1; c < 16; ++c) {
        const float e = fabsf(__fsub_rn(a, d[c]));
        if (e < best_err) {
            best = c;
            best_err = e;
        }
    }
    return best;
}

__global__ void __launch_bounds__(kThreads) quant_log4_kernel(const float* __restrict__ w, int64_t K,
                                                              uint8_t* __restrict__ q, float* __restrict__ scales) {
    const int64_t j = blockIdx.x;
    const int64_t half = K / 2;
    const float* row = w + j * K;
    const float m = row_max_abs(row, K);
    const float s = (m == 0.f) ? 1.0f : __fdiv_rn(m, 32767.0f);
    if (threadIdx.x == 0) scales[j] = s;
    float d[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) d[c] = __fmul_rn(__fmul_rn(1.0f, __fsub_rn((float)(1u << c), 1.0f)), s);
    for (int64_t i = threadIdx.x; i < half; i += blockDim.x) {
        const uint32_t c0 = log4_code(fabsf(row[2 * i]), d);
        const uint32_t c1 = log4_code(fabsf(row[2 * i + 1]), d);
        q[j * half + i] = (uint8_t)((c0 << 4) | c1);
    }
}

}  // namespace

cudaError_t launch_quantize(int fmt, int64_t N, int64_t K, const float* w, uint8_t* q, float* scales,
                            cudaStream_t st) {
    if (N <= 0) return cudaSuccess;
    if (N > 0x7fffffffLL) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)N);
    switch (fmt) {
        case BRAMHA_FMT_W8: quant_int8_kernel<<<grid, kThreads, 0, st>>>(w, K, reinterpret_cast<int8_t*>(q), scales); break;
        case BRAMHA_FMT_W4ZP8: quant_int4_kernel<<<grid, kThreads, 0, st>>>(w, K, q, scales); break;
        case BRAMHA_FMT_LOG4: quant_log4_kernel<<<grid, kThreads, 0, st>>>(w, K, q, scales); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace bramha
