#pragma once
// gemv_impl.cuh -- dequantize-fused GEMV for decode (batch 1..8), CUDA cores, sm_100a.
//
// Replaces the decode GEMV of the reference: `matvec_mul_into`
// (src/inference/cpu_engine.rs:1307-1444) and the WGSL shaders it would have
// dispatched to (src/compute/shaders/gemm_int4.wgsl, gemm_int8.wgsl, gemm.wgsl).
// y[b][j] = s_j * sum_i x[b][i] * code(w_ji), fp32 accumulation.
//
// Bandwidth-bound design (no tensor cores):
//  * one warp owns R consecutive rows; per step each lane streams VEC bytes of
//    each row with one 128/64/32-bit non-allocating load, so every warp load
//    is one contiguous 32*VEC-byte run of a row;
//  * the lane's activation slice is loaded once per step (L1-resident) and
//    reused for all R rows;
//  * KS warps of a CTA split the steps of the same rows and combine partial
//    sums through shared memory (named barriers per warp group);
//  * dequantization is bit construction, not table lookups:
//      - int4 / int8: the code is masked IN PLACE (w & (0xF << p)); read as a
//        float, those bits are the subnormal code * 2^(p-149), exactly, for
//        p + width <= 24.  The activation is pre-scaled by 2^(85-p), so the
//        product is x * code * 2^-64 and the zero point is folded out:
//        y = s * (2^64 * sum(x*code) - zp * sum(x)).  Requires no FTZ.
//      - log4: the code is shifted into the exponent field of a float,
//        (c << 23) | (112 << 23) = 2^(c-15), so y = s*(2^15*sum(x*2^(c-15)) - sum(x)),
//        matching w = (2^c - 1) * s (spanda-engine/src/lib.rs:332-342);
//  * products accumulate with packed f32x2 FMAs (FFMA2), two columns at once.
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {  // internal linkage: each per-format TU gets its own copy

template <int VEC>
struct VecT;
template <>
struct VecT<16> { using T = uint4; };
template <>
struct VecT<8> { using T = uint2; };
template <>
struct VecT<4> { using T = uint32_t; };

// Streaming load: weights are touched once per GEMV; keep them out of L1.
__device__ __forceinline__ void ldw(const uint8_t* p, uint4& v) {
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
}
__device__ __forceinline__ void ldw(const uint8_t* p, uint2& v) {
    asm("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
}
__device__ __forceinline__ void ldw(const uint8_t* p, uint32_t& v) {
    asm("ld.global.nc.L1::no_allocate.L2::256B.u32 %0, [%1];" : "=r"(v) : "l"(p));
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t word_of(const uint2& v, int i) { return i == 0 ? v.x : v.y; }
__device__ __forceinline__ uint32_t word_of(const uint32_t& v, int) { return v; }

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float bits(uint32_t u) { return __uint_as_float(u); }

// Columns covered by one 32-bit word of packed weights.
template <int FMT>
struct Fmt;

// ---- int4, zero point 8 (quantize_to_int4) --------------------------------
template <>
struct Fmt<BRAMHA_FMT_W4ZP8> {
    static constexpr int kColsPerWord = 8;
    static constexpr int kColsPerByte = 2;
    // Pre-scale exponent per column of a word (see file comment):
    // col 2b (high nibble, bit 8b+4) and col 2b+1 (low nibble, bit 8b);
    // byte 3 is read from w >> 8, i.e. at bits 16 / 20.
    __device__ __forceinline__ static float prescale(int c) {
        constexpr float s0 = 2.4178516392292583e+24f;   // 2^81
        constexpr float s1 = 3.8685626227668134e+25f;   // 2^85
        constexpr float s2 = 9.4447329657392904e+21f;   // 2^73
        constexpr float s3 = 1.5111572745182865e+23f;   // 2^77
        constexpr float s4 = 3.6893488147419103e+19f;   // 2^65
        constexpr float s5 = 5.9029581035870565e+20f;   // 2^69
        const float t[8] = {s0, s1, s2, s3, s4, s5, s4, s5};
        return t[c];
    }
    __device__ __forceinline__ static void acc(uint32_t w, const float* xp, float2& a0, float2& a1) {
        const uint32_t w3 = w >> 8;
        a0 = __ffma2_rn(f2(xp[0], xp[1]), f2(bits(w & 0x000000F0u), bits(w & 0x0000000Fu)), a0);
        a1 = __ffma2_rn(f2(xp[2], xp[3]), f2(bits(w & 0x0000F000u), bits(w & 0x00000F00u)), a1);
        a0 = __ffma2_rn(f2(xp[4], xp[5]), f2(bits(w & 0x00F00000u), bits(w & 0x000F0000u)), a0);
        a1 = __ffma2_rn(f2(xp[6], xp[7]), f2(bits(w3 & 0x00F00000u), bits(w3 & 0x000F0000u)), a1);
    }
    // dot = 2^64 * acc - 8 * sum(x)
    __device__ __forceinline__ static float finish(float acc, float sx) {
        return fmaf(acc, 1.8446744073709552e+19f, -8.0f * sx);
    }
};

// ---- int8 (quantize_to_int8): bytes XOR 0x80 -> q + 128 ------------------
template <>
struct Fmt<BRAMHA_FMT_W8> {
    static constexpr int kColsPerWord = 4;
    static constexpr int kColsPerByte = 1;
    __device__ __forceinline__ static float prescale(int c) {
        constexpr float s0 = 3.8685626227668134e+25f;   // 2^85 (bits 0..7)
        constexpr float s1 = 1.5111572745182865e+23f;   // 2^77 (bits 8..15)
        constexpr float s2 = 5.9029581035870565e+20f;   // 2^69 (bits 16..23)
        const float t[4] = {s0, s1, s2, s2};
        return t[c];
    }
    __device__ __forceinline__ static void acc(uint32_t w, const float* xp, float2& a0, float2& a1) {
        const uint32_t u = w ^ 0x80808080u;
        const uint32_t u3 = u >> 8;
        a0 = __ffma2_rn(f2(xp[0], xp[1]), f2(bits(u & 0x000000FFu), bits(u & 0x0000FF00u)), a0);
        a1 = __ffma2_rn(f2(xp[2], xp[3]), f2(bits(u & 0x00FF0000u), bits(u3 & 0x00FF0000u)), a1);
    }
    __device__ __forceinline__ static float finish(float acc, float sx) {
        return fmaf(acc, 1.8446744073709552e+19f, -128.0f * sx);
    }
};

// ---- log4 (dequantize_log4): 2^c built in the exponent field -------------
template <>
struct Fmt<BRAMHA_FMT_LOG4> {
    static constexpr int kColsPerWord = 8;
    static constexpr int kColsPerByte = 2;
    __device__ __forceinline__ static float prescale(int) { return 1.0f; }
    __device__ __forceinline__ static uint32_t e(uint32_t t) { return (t & 0x07800000u) | 0x38000000u; }
    __device__ __forceinline__ static void acc(uint32_t w, const float* xp, float2& a0, float2& a1) {
        // column 2b is the high nibble of byte b (bit 8b+4), column 2b+1 the low one (bit 8b)
        a0 = __ffma2_rn(f2(xp[0], xp[1]), f2(bits(e(w << 19)), bits(e(w << 23))), a0);
        a1 = __ffma2_rn(f2(xp[2], xp[3]), f2(bits(e(w << 11)), bits(e(w << 15))), a1);
        a0 = __ffma2_rn(f2(xp[4], xp[5]), f2(bits(e(w << 3)), bits(e(w << 7))), a0);
        a1 = __ffma2_rn(f2(xp[6], xp[7]), f2(bits(e(w >> 5)), bits(e(w >> 1))), a1);
    }
    // dot = 2^15 * acc - sum(x)   since  (2^c - 1) = 2^15 * 2^(c-15) - 1
    __device__ __forceinline__ static float finish(float acc, float sx) { return fmaf(acc, 32768.0f, -sx); }
};

// ---- dense f32 (matvec_mul on f32 weights) -------------------------------
template <>
struct Fmt<BRAMHA_FMT_F32> {
    static constexpr int kColsPerWord = 1;
    static constexpr int kColsPerByte = 0;  // 4 bytes per column
    __device__ __forceinline__ static float prescale(int) { return 1.0f; }
    __device__ __forceinline__ static float finish(float acc, float) { return acc; }
};

template <int FMT>
__device__ __forceinline__ int64_t col_of_byte(int64_t b) {
    if constexpr (FMT == BRAMHA_FMT_F32) return b >> 2;
    else return b * Fmt<FMT>::kColsPerByte;
}

// Named barrier over the KS warps of one group (ids 1..8; 0 is __syncthreads).
__device__ __forceinline__ void group_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int FMT, int B, int R, int KS, int VEC>
__global__ void __launch_bounds__(256) gemv_kernel(const __grid_constant__ GemvArgs a) {
    using V = typename VecT<VEC>::T;
    constexpr int kWords = VEC / 4;
    constexpr int kCols = (FMT == BRAMHA_FMT_F32) ? VEC / 4 : VEC * Fmt<FMT>::kColsPerByte;
    constexpr int G = 8 / KS;  // row groups per CTA

    __shared__ float red[8][B][R + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = warp / KS, kw = warp % KS;
    const int K = a.K;
    const int64_t step_bytes = 32 * VEC;

    // sum(x) over the columns this lane ever touches: fixed per warp, so
    // computed once and reused for every tile.
    float sx[B];
#pragma unroll
    for (int b = 0; b < B; ++b) sx[b] = 0.f;
    if constexpr (FMT != BRAMHA_FMT_F32) {
        for (int s = kw; s < a.nsteps; s += KS) {
            const int64_t c0 = col_of_byte<FMT>(s * step_bytes + lane * VEC);
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float* xr = a.x + b * a.ldx;
#pragma unroll
                for (int c = 0; c < kCols; ++c) {
                    const int64_t k = c0 + c;
                    sx[b] += (k < K) ? __ldg(xr + k) : 0.f;
                }
            }
        }
    }

    for (int tile = blockIdx.x * G + group; tile < a.ntiles; tile += gridDim.x * G) {
        int si = 0;
#pragma unroll 1
        for (int i = 1; i < a.nseg; ++i)
            if (tile >= a.seg[i].tile_begin) si = i;
        const GemvSeg& sg = a.seg[si];
        const int row0 = (tile - sg.tile_begin) * R;
        const int nrows = min(R, sg.N - row0);

        float2 acc[R][B][2];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][b][0] = acc[r][b][1] = f2(0.f, 0.f);

        const uint8_t* qrow = sg.q + (int64_t)row0 * sg.ldq;
#pragma unroll 2
        for (int s = kw; s < a.nsteps; s += KS) {
            const int64_t bo = s * step_bytes + lane * VEC;
            const bool valid = bo < sg.ldq;
            V wv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (valid && r < nrows) ldw(qrow + r * sg.ldq + bo, wv[r]);
                else wv[r] = V{};
            }
            const int64_t c0 = col_of_byte<FMT>(bo);
            float xs[B][kCols];
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float* xr = a.x + b * a.ldx + c0;
                if (c0 + kCols <= K) {
#pragma unroll
                    for (int c = 0; c < kCols; c += 4) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
                        xs[b][c] = v.x; xs[b][c + 1] = v.y; xs[b][c + 2] = v.z; xs[b][c + 3] = v.w;
                    }
                } else if constexpr (kCols >= 4) {
#pragma unroll
                    for (int c = 0; c < kCols; ++c) xs[b][c] = (c0 + c < K) ? __ldg(xr + c) : 0.f;
                } else {
                    xs[b][0] = (c0 < K) ? __ldg(xr) : 0.f;
                }
#pragma unroll
                for (int c = 0; c < kCols; ++c) xs[b][c] *= Fmt<FMT>::prescale(c % Fmt<FMT>::kColsPerWord);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int i = 0; i < kWords; ++i) {
                    const uint32_t w = word_of(wv[r], i);
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        if constexpr (FMT == BRAMHA_FMT_F32) {
                            acc[r][b][i & 1].x = fmaf(xs[b][i], __uint_as_float(w), acc[r][b][i & 1].x);
                        } else {
                            Fmt<FMT>::acc(w, &xs[b][i * Fmt<FMT>::kColsPerWord], acc[r][b][0], acc[r][b][1]);
                        }
                    }
                }
            }
        }

        // Reduce over the 32 lanes, then over the KS warps of the group.
        float part[R][B];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) {
                float v = (acc[r][b][0].x + acc[r][b][0].y) + (acc[r][b][1].x + acc[r][b][1].y);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                part[r][b] = v;
            }
        float sxr[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float v = sx[b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            sxr[b] = v;
        }
        if constexpr (KS > 1) {
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
#pragma unroll
                    for (int r = 0; r < R; ++r) red[warp][b][r] = part[r][b];
                    red[warp][b][R] = sxr[b];
                }
            }
            group_sync(1 + group, KS * 32);
            if (kw == 0 && lane == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float v = 0.f;
#pragma unroll
                        for (int k2 = 0; k2 < KS; ++k2) v += red[group * KS + k2][b][r];
                        part[r][b] = v;
                    }
                    float v = 0.f;
#pragma unroll
                    for (int k2 = 0; k2 < KS; ++k2) v += red[group * KS + k2][b][R];
                    sxr[b] = v;
                }
            }
            group_sync(1 + group, KS * 32);
        }
        // Lane 0 of the group's first warp holds the totals (every lane does
        // when KS == 1); broadcast them and let lane r store row r.
        if (kw == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    part[r][b] = __shfl_sync(0xffffffffu, part[r][b], 0);
                }
#pragma unroll
            for (int b = 0; b < B; ++b) sxr[b] = __shfl_sync(0xffffffffu, sxr[b], 0);
            if (lane < nrows) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (r == lane) {
                        const float s = (FMT == BRAMHA_FMT_F32) ? 1.0f : __ldg(sg.scales + row0 + r);
#pragma unroll
                        for (int b = 0; b < B; ++b)
                            sg.y[b * sg.ldy + row0 + r] = Fmt<FMT>::finish(part[r][b], sxr[b]) * s;
                    }
                }
            }
        }
    }
}

template <int FMT, int B, int R, int KS, int VEC>
cudaError_t launch_t(const GemvArgs& a, int num_sms, cudaStream_t st) {
    constexpr int G = 8 / KS;
    // Resident CTAs per SM, queried once per instantiation (and outside any
    // stream capture: the first call happens on the first launch).
    static const int per_sm = [] {
        int v = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, gemv_kernel<FMT, B, R, KS, VEC>, 256, 0) !=
                cudaSuccess ||
            v < 1)
            v = 1;
        return v;
    }();
    const int need = (a.ntiles + G - 1) / G;
    const int grid = need < num_sms * per_sm ? need : num_sms * per_sm;
    gemv_kernel<FMT, B, R, KS, VEC><<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

template <int FMT, int B>
cudaError_t pick_tiling(GemvArgs a, int num_sms, cudaStream_t st) {
    constexpr int R = 4;
    constexpr int VEC = (FMT == BRAMHA_FMT_F32) ? 16 : 16;
    const int64_t step_bytes = 32 * VEC;
    a.nsteps = (int)((a.ldq_min + step_bytes - 1) / step_bytes);
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        a.seg[i].tile_begin = ntiles;
        ntiles += (a.seg[i].N + R - 1) / R;
    }
    a.ntiles = ntiles;
    // Enough warps in flight to cover HBM latency: ~16 warps per SM.
    const int64_t target = (int64_t)num_sms * 16;
    if ((int64_t)ntiles >= target || a.nsteps < 2) return launch_t<FMT, B, R, 1, VEC>(a, num_sms, st);
    if ((int64_t)ntiles * 2 >= target || a.nsteps < 4) return launch_t<FMT, B, R, 2, VEC>(a, num_sms, st);
    if ((int64_t)ntiles * 4 >= target || a.nsteps < 8) return launch_t<FMT, B, R, 4, VEC>(a, num_sms, st);
    return launch_t<FMT, B, R, 8, VEC>(a, num_sms, st);
}


// Batch sizes with their own instantiation; other sizes are split into these.
template <int FMT>
cudaError_t dispatch_batch(const GemvArgs& a, int num_sms, cudaStream_t st) {
    switch (a.batch) {
        case 1: return pick_tiling<FMT, 1>(a, num_sms, st);
        case 2: return pick_tiling<FMT, 2>(a, num_sms, st);
        case 4: return pick_tiling<FMT, 4>(a, num_sms, st);
        case 8: return pick_tiling<FMT, 8>(a, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace
}  // namespace bramha
