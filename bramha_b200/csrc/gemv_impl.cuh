#pragma once
// gemv_impl.cuh -- dequantize-fused GEMV for decode (batch 1..8), CUDA cores, sm_100a.
//
// Replaces the decode GEMV of the reference: `matvec_mul_into`
// (src/inference/cpu_engine.rs:1307-1444) and the WGSL shaders it would have
// dispatched to (src/compute/shaders/gemm_int4.wgsl, gemm_int8.wgsl, gemm.wgsl).
// y[b][j] = s_j * sum_i x[b][i] * code(w_ji), fp32 accumulation.
//
// Bandwidth-bound design (no tensor cores):
//  * persistent CTAs (occupancy x SMs); each CTA first stages the activations
//    in shared memory, pre-scaled, in natural order with an XOR swizzle that
//    makes both the coalesced staging stores and the per-lane 16-byte loads
//    conflict-free, and sums them once (the zero-point / log offset
//    correction needs sum(x)); the first weights are in flight meanwhile;
//  * a warp owns R consecutive rows; per step each lane streams 16 bytes of
//    each row (one non-allocating 128-bit load per row, so a warp load is one
//    contiguous 512-byte run) and prefetches the next step's bytes;
//  * KS warps of a CTA split the steps of the same rows and combine partial
//    sums through shared memory (named barrier per warp group);
//  * dequantization is bit construction in registers, no tables:
//      - int4 / int8: the code is masked IN PLACE (w & (0xF << p)); read as a
//        float those bits are the subnormal value code * 2^(p-149), exactly,
//        for bit positions below 24.  The activation is pre-scaled by
//        2^(85-p), so each product is x * code * 2^-64 and the zero point is
//        folded out: y = s * (2^64 * sum(x*code) - zp * sum(x)).  Needs
//        subnormals (no flush-to-zero; the library is built with -ftz=false).
//      - log4: x * 2^c is formed by adding c << 23 to the bits of x (one
//        integer multiply-add on the FMA pipe), so y = s * (sum(x * 2^c) - sum(x)), matching
//        w = (2^c - 1) * s (spanda-engine/src/lib.rs:332-342).  A zero x
//        contributes 2^(c-127) <= 2^-112 instead of 0; a NaN/Inf in x makes
//        sum(x), and so y, NaN/Inf.
//  * products accumulate with packed f32x2 instructions, two columns at once.
//
// Device word layout of the 4-bit formats (set up at registration,
// repack.cu): the 32-bit word holding columns c0..c7 keeps the even columns
// c0,c2,c4,c6 in bits 0-15 and the odd ones c1,c3,c5,c7 in bits 16-31
// (nibble j of each half = column 2j / 2j+1), so column pairs (c0,c1),
// (c2,c3), ... sit 16 bits apart.
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {  // internal linkage: each per-format TU gets its own copy

constexpr int kThreads = 256;
constexpr int kVec = 16;                       // bytes per lane per step
constexpr int kStepBytes = 32 * kVec;          // bytes per warp per step (one row)

__device__ __forceinline__ void ldw(const uint8_t* p, uint4& v) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float bits(uint32_t u) { return __uint_as_float(u); }
template <int FMT>
struct Fmt;

// ---- int4, zero point 8 (quantize_to_int4), device word layout ------------
template <>
struct Fmt<BRAMHA_FMT_W4ZP8> {
    static constexpr int kColsPerWord = 8;
    static constexpr int kColsPerLane = 32;  // per 16-byte step
    // pre-scale exponent 85 - p for the bit position p each column is read at
    // (c5 / c7 are read from w >> 8, at 16 / 20)
    // p / 4 for c0..c7 = {0, 4, 1, 5, 2, 4, 3, 5}, one nibble each
    __device__ __forceinline__ static float prescale(int c) {
        const int p = 4 * (int)((0x53425140u >> (4 * c)) & 0xFu);
        return __uint_as_float((uint32_t)(85 - p + 127) << 23);
    }
    __device__ __forceinline__ static void acc(uint32_t w, const float4& xa, const float4& xb, float2& a0,
                                               float2& a1) {
        const uint32_t w8 = w >> 8;
        a0 = __ffma2_rn(f2(xa.x, xa.y), f2(bits(w & 0x0000000Fu), bits(w & 0x000F0000u)), a0);
        a1 = __ffma2_rn(f2(xa.z, xa.w), f2(bits(w & 0x000000F0u), bits(w & 0x00F00000u)), a1);
        a0 = __ffma2_rn(f2(xb.x, xb.y), f2(bits(w & 0x00000F00u), bits(w8 & 0x000F0000u)), a0);
        a1 = __ffma2_rn(f2(xb.z, xb.w), f2(bits(w & 0x0000F000u), bits(w8 & 0x00F00000u)), a1);
    }
    // dot = 2^64 * acc - 8 * sum(x)
    __device__ __forceinline__ static float finish(float acc, float sx) {
        return fmaf(acc, 1.8446744073709552e+19f, -8.0f * sx);
    }
};

// ---- log4 (dequantize_log4), device word layout ---------------------------
// mul[] = {2^23, 2^7, 2^19, 2^3, 2^15, 2^7, 2^11, 2^3}: moves the code of
// column c0..c7 (even columns at bits 0,4,8,12; odd at 16,20 and, read from
// w >> 8, 16,20) to bit 23.  They arrive as kernel parameters so the compiler
// cannot turn the multiply-adds into shifts on the (half-rate) ALU pipe.
template <>
struct Fmt<BRAMHA_FMT_LOG4> {
    static constexpr int kColsPerWord = 8;
    static constexpr int kColsPerLane = 32;
    __device__ __forceinline__ static float prescale(int) { return 1.0f; }
    __device__ __forceinline__ static float madx(uint32_t m, uint32_t mul, float x) {
        return __uint_as_float(m * mul + __float_as_uint(x));
    }
    __device__ __forceinline__ static void acc(uint32_t w, const float4& xa, const float4& xb, const uint32_t* mul,
                                               float2& a0, float2& a1) {
        const uint32_t w8 = w >> 8;
        a0 = __fadd2_rn(a0, f2(madx(w & 0x0000000Fu, mul[0], xa.x), madx(w & 0x000F0000u, mul[1], xa.y)));
        a1 = __fadd2_rn(a1, f2(madx(w & 0x000000F0u, mul[2], xa.z), madx(w & 0x00F00000u, mul[3], xa.w)));
        a0 = __fadd2_rn(a0, f2(madx(w & 0x00000F00u, mul[4], xb.x), madx(w8 & 0x000F0000u, mul[5], xb.y)));
        a1 = __fadd2_rn(a1, f2(madx(w & 0x0000F000u, mul[6], xb.z), madx(w8 & 0x00F00000u, mul[7], xb.w)));
    }
    // dot = sum(x * 2^c) - sum(x)  since  w / s = 2^c - 1
    __device__ __forceinline__ static float finish(float acc, float sx) { return acc - sx; }
};

// ---- int8 (quantize_to_int8): bytes XOR 0x80 -> q + 128 ------------------
template <>
struct Fmt<BRAMHA_FMT_W8> {
    static constexpr int kColsPerWord = 4;
    static constexpr int kColsPerLane = 16;
    // bit position of byte c0..c3: 0, 8, 16 and (read from u >> 8) 16
    __device__ __forceinline__ static float prescale(int c) {
        const int p = c == 3 ? 16 : 8 * c;
        return __uint_as_float((uint32_t)(85 - p + 127) << 23);
    }
    __device__ __forceinline__ static void acc(uint32_t w, const float4& x, float2& a0, float2& a1) {
        const uint32_t u = w ^ 0x80808080u;
        const uint32_t u8 = u >> 8;
        a0 = __ffma2_rn(f2(x.x, x.y), f2(bits(u & 0x000000FFu), bits(u & 0x0000FF00u)), a0);
        a1 = __ffma2_rn(f2(x.z, x.w), f2(bits(u & 0x00FF0000u), bits(u8 & 0x00FF0000u)), a1);
    }
    __device__ __forceinline__ static float finish(float acc, float sx) {
        return fmaf(acc, 1.8446744073709552e+19f, -128.0f * sx);
    }
};

// ---- dense f32 (matvec_mul on f32 weights) -------------------------------
template <>
struct Fmt<BRAMHA_FMT_F32> {
    static constexpr int kColsPerWord = 1;
    static constexpr int kColsPerLane = 4;
    __device__ __forceinline__ static float prescale(int) { return 1.0f; }
    __device__ __forceinline__ static float finish(float acc, float) { return acc; }
};

// Named barrier over the KS warps of one group (ids 1..8; 0 is __syncthreads).
__device__ __forceinline__ void group_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Shared-memory bytes for the staged activations of `batch` rows.
template <int FMT>
__host__ __device__ constexpr int64_t xs_bytes(int nsteps, int batch) {
    return (int64_t)batch * nsteps * 32 * Fmt<FMT>::kColsPerLane * 4;
}

// Shared-memory slot of activation float4 number n: natural order with the
// float4 index inside each 128-byte group XOR-swizzled by the group index,
// so the staging stores (consecutive n) and the per-lane loads (lane l reads
// group l of a step) are both bank-conflict free.
__device__ __forceinline__ int xs_slot(int n) { return (n & ~7) | ((n ^ (n >> 3)) & 7); }

template <int FMT, int B, int R, int KS>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int kCols = Fmt<FMT>::kColsPerLane;  // activation columns per lane per step
    constexpr int kC4 = kCols / 4;                  // float4 per lane per step
    constexpr int G = 8 / KS;                       // row groups per CTA
    extern __shared__ float4 xs[];                  // [B][nsteps * 32 * kC4], swizzled
    __shared__ float sx_sh[B];
    __shared__ float red[8][B][R];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = warp / KS, kw = warp % KS;
    const int K = a.K, nsteps = a.nsteps;
    const int n4row = nsteps * 32 * kC4;            // float4 per staged activation row

    // Per-tile state; the first tile's first weights are requested before the
    // activations are staged so the two overlap.
    int tile = blockIdx.x * G + group;
    const GemvSeg* sg = nullptr;
    int row0 = 0, nrows = 0;
    const uint8_t* rows[R];
    auto setup_tile = [&](int t) {
        int si = 0;
#pragma unroll 1
        for (int i = 1; i < a.nseg; ++i)
            if (t >= a.seg[i].tile_begin) si = i;
        sg = &a.seg[si];
        row0 = (t - sg->tile_begin) * R;
        nrows = min(R, sg->N - row0);
#pragma unroll
        for (int r = 0; r < R; ++r)  // rows past the end re-read the last row; results are dropped
            rows[r] = sg->q + (int64_t)(row0 + min(r, nrows - 1)) * sg->ldq + lane * kVec;
    };
    // steps whose 16 bytes lie inside the row pitch for every lane
    uint4 cur[R], nxt[R];
    auto load = [&](uint4 (&dst)[R], int s, int64_t ldq) {
        const int64_t bo = (int64_t)s * kStepBytes;
        if (bo + kStepBytes <= ldq) {
#pragma unroll
            for (int r = 0; r < R; ++r) ldw(rows[r] + bo, dst[r]);
        } else {
            const bool valid = bo + lane * kVec < ldq;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (valid) ldw(rows[r] + bo, dst[r]);
                else dst[r] = make_uint4(0, 0, 0, 0);
            }
        }
    };
    if (tile < a.ntiles) {
        setup_tile(tile);
        if (kw < nsteps) load(cur, kw, sg->ldq);
    }

    // ---- prologue: stage pre-scaled activations, sum(x) per batch row
    {
        if (threadIdx.x < B) sx_sh[threadIdx.x] = 0.f;
        __syncthreads();
#pragma unroll 1
        for (int b = 0; b < B; ++b) {
            const float* xr = a.x + (int64_t)b * a.ldx;
            float4* xsb = xs + (int64_t)b * n4row;
            float part = 0.f;
            for (int i = threadIdx.x; i < n4row; i += kThreads) {
                const int col0 = 4 * i;
                float4 v;
                if (col0 + 3 < K) {
                    v = __ldg(reinterpret_cast<const float4*>(xr + col0));
                } else {
                    v.x = col0 < K ? __ldg(xr + col0) : 0.f;
                    v.y = col0 + 1 < K ? __ldg(xr + col0 + 1) : 0.f;
                    v.z = col0 + 2 < K ? __ldg(xr + col0 + 2) : 0.f;
                    v.w = col0 + 3 < K ? __ldg(xr + col0 + 3) : 0.f;
                }
                part += (v.x + v.y) + (v.z + v.w);
                if constexpr (FMT == BRAMHA_FMT_W4ZP8 || FMT == BRAMHA_FMT_W8) {
                    const int p0 = col0 % Fmt<FMT>::kColsPerWord;
                    v.x *= Fmt<FMT>::prescale(p0);
                    v.y *= Fmt<FMT>::prescale(p0 + 1);
                    v.z *= Fmt<FMT>::prescale(p0 + 2);
                    v.w *= Fmt<FMT>::prescale(p0 + 3);
                }
                xsb[xs_slot(i)] = v;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0) atomicAdd(&sx_sh[b], part);
        }
        __syncthreads();
    }

    const uint32_t* mul = a.mul;  // log4 multipliers (2^k), opaque to the compiler so they stay IMADs
    for (; tile < a.ntiles; tile += gridDim.x * G) {
        const int64_t ldq = sg->ldq;
        float2 acc[R][B][2];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][b][0] = acc[r][b][1] = f2(0.f, 0.f);

        auto compute = [&](const uint4 (&wv)[R], int s) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int n0 = (s * 32 + lane) * kC4;  // first float4 of this lane's chunk
                const float4* xrow = xs + (int64_t)b * n4row;
                if constexpr (FMT == BRAMHA_FMT_F32) {
                    const float4 x = xrow[xs_slot(n0)];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        acc[r][b][0] = __ffma2_rn(f2(x.x, x.y), f2(bits(wv[r].x), bits(wv[r].y)), acc[r][b][0]);
                        acc[r][b][1] = __ffma2_rn(f2(x.z, x.w), f2(bits(wv[r].z), bits(wv[r].w)), acc[r][b][1]);
                    }
                } else if constexpr (FMT == BRAMHA_FMT_W8) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 x = xrow[xs_slot(n0 + i)];
#pragma unroll
                        for (int r = 0; r < R; ++r) Fmt<FMT>::acc(word_of(wv[r], i), x, acc[r][b][0], acc[r][b][1]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 xa = xrow[xs_slot(n0 + 2 * i)], xc = xrow[xs_slot(n0 + 2 * i + 1)];
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            if constexpr (FMT == BRAMHA_FMT_LOG4)
                                Fmt<FMT>::acc(word_of(wv[r], i), xa, xc, mul, acc[r][b][0], acc[r][b][1]);
                            else
                                Fmt<FMT>::acc(word_of(wv[r], i), xa, xc, acc[r][b][0], acc[r][b][1]);
                        }
                    }
                }
            }
        };
#pragma unroll 2
        for (int s = kw; s < nsteps; s += KS) {
            if (s + KS < nsteps) load(nxt, s + KS, ldq);
            compute(cur, s);
#pragma unroll
            for (int r = 0; r < R; ++r) cur[r] = nxt[r];
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
        if constexpr (KS > 1) {
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) red[warp][b][r] = part[r][b];
            }
            group_sync(1 + group, KS * 32);
            if (kw == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float v = 0.f;
#pragma unroll
                        for (int k2 = 0; k2 < KS; ++k2) v += red[group * KS + k2][b][r];
                        part[r][b] = v;
                    }
            }
            group_sync(1 + group, KS * 32);
        }
        if (kw == 0) {
            // lane (r, b) stores y[b][row0 + r]
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b)
                    if (lane == r * B + b && r < nrows) {
                        const float s = (FMT == BRAMHA_FMT_F32) ? 1.0f : __ldg(sg->scales + row0 + r);
                        sg->y[(int64_t)b * sg->ldy + row0 + r] = Fmt<FMT>::finish(part[r][b], sx_sh[b]) * s;
                    }
        }
        // next tile: set up its rows and request its first step
        const int nt = tile + gridDim.x * G;
        if (nt < a.ntiles) {
            setup_tile(nt);
            if (kw < nsteps) load(cur, kw, sg->ldq);
        }
    }
}

template <int FMT, int B, int R, int KS>
cudaError_t launch_t(const GemvArgs& a, int num_sms, size_t smem, cudaStream_t st) {
    constexpr int G = 8 / KS;
    auto kern = gemv_kernel<FMT, B, R, KS>;
    static int configured_smem = 0;  // dynamic shared memory already allowed for this instantiation
    if ((int)smem > configured_smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured_smem = (int)smem;
    }
    static size_t cached_smem = ~size_t(0);  // last occupancy query (benign race: both threads compute the same)
    static int cached_per_sm = 0;
    int per_sm = cached_per_sm;
    if (cached_smem != smem) {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
        if (e != cudaSuccess) return e;
        cached_per_sm = per_sm;
        cached_smem = smem;
    }
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int need = (a.ntiles + G - 1) / G;
    const int grid = need < num_sms * per_sm ? need : num_sms * per_sm;
    kern<<<grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <int FMT, int B>
cudaError_t pick_tiling(GemvArgs a, int num_sms, cudaStream_t st) {
    constexpr int R = (B <= 2) ? 4 : (B <= 4 ? 2 : 1);
    a.nsteps = (a.ldq_min + kStepBytes - 1) / kStepBytes;
    const uint32_t mul[8] = {1u << 23, 1u << 7, 1u << 19, 1u << 3, 1u << 15, 1u << 7, 1u << 11, 1u << 3};
    for (int i = 0; i < 8; ++i) a.mul[i] = mul[i];
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        a.seg[i].tile_begin = ntiles;
        ntiles += (a.seg[i].N + R - 1) / R;
    }
    a.ntiles = ntiles;
    const size_t smem = (size_t)xs_bytes<FMT>(a.nsteps, B);
    // Enough warps in flight to cover HBM latency: ~16 warps per SM.
    const int64_t target = (int64_t)num_sms * 16;
    if ((int64_t)ntiles >= target || a.nsteps < 2) return launch_t<FMT, B, R, 1>(a, num_sms, smem, st);
    if ((int64_t)ntiles * 2 >= target || a.nsteps < 4) return launch_t<FMT, B, R, 2>(a, num_sms, smem, st);
    if ((int64_t)ntiles * 4 >= target || a.nsteps < 8) return launch_t<FMT, B, R, 4>(a, num_sms, smem, st);
    return launch_t<FMT, B, R, 8>(a, num_sms, smem, st);
}

// Largest batch chunk (1, 2, 4 or 8, at most `left`) whose staged activations
// fit in `max_smem` bytes; 0 if even one row does not fit.
template <int FMT>
int max_batch_chunk(int nsteps, int left, int64_t max_smem) {
    for (int b = 8; b >= 1; b >>= 1)
        if (b <= left && xs_bytes<FMT>(nsteps, b) <= max_smem) return b;
    return 0;
}

// Splits the batch into chunks whose staged activations fit in shared
// memory (each chunk re-reads the weights) and launches one kernel per chunk.
template <int FMT>
cudaError_t run_gemv(const GemvArgs& a, int num_sms, cudaStream_t st) {
    const int nsteps = (a.ldq_min + kStepBytes - 1) / kStepBytes;
    constexpr int64_t kMaxSmem = 200 * 1024;
    GemvArgs part = a;
    int done = 0;
    while (done < a.batch) {
        const int bc = max_batch_chunk<FMT>(nsteps, a.batch - done, kMaxSmem);
        if (bc == 0) return cudaErrorInvalidValue;  // K too large to stage one activation row
        part.batch = bc;
        part.x = a.x + (int64_t)done * a.ldx;
        for (int i = 0; i < a.nseg; ++i) part.seg[i].y = a.seg[i].y + (int64_t)done * a.seg[i].ldy;
        cudaError_t e;
        switch (bc) {
            case 1: e = pick_tiling<FMT, 1>(part, num_sms, st); break;
            case 2: e = pick_tiling<FMT, 2>(part, num_sms, st); break;
            case 4: e = pick_tiling<FMT, 4>(part, num_sms, st); break;
            default: e = pick_tiling<FMT, 8>(part, num_sms, st); break;
        }
        if (e != cudaSuccess) return e;
        done += bc;
    }
    return cudaSuccess;
}

}  // namespace
}  // namespace bramha
