// gemv_f32.cu -- GEMV for dense f32 weights (batch 1..8), CUDA cores.
//
// The reference's `matvec_mul` on `WeightTensor::Float` (src/inference/cpu_engine.rs:
// 1311-1335, wgpu arm src/compute/wgpu_backend.rs:734).  Dense f32 weights are not
// a quantized format of this path, but the compute plane keeps the same call
// surface.  At 4 bytes per weight one FMA per 4 bytes is far from any compute
// limit, so the kernel is a plain streaming one:
//  * a warp owns R consecutive rows; per step each lane reads 16 bytes (4
//    columns) of each row with a non-allocating 128-bit load, so a warp load is
//    one contiguous 512-byte run, and the next step's bytes are prefetched;
//  * the activation slice is read from L1 (it is shared by all rows);
//  * KS warps of a CTA split the steps of the same rows (shared-memory reduce).
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {

constexpr int kThreads = 256;
constexpr int kStepBytes = 512;  // 32 lanes x 16 bytes

__device__ __forceinline__ void ldw(const uint8_t* p, float4& v) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
}

template <int B, int R, int KS>
__global__ void __launch_bounds__(kThreads) gemv_f32_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int G = 8 / KS;  // row groups per CTA
    __shared__ float red[8][B][R];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = warp / KS, kw = warp % KS;
    const int K = a.K, nsteps = a.nsteps;

    for (int tile = blockIdx.x * G + group; tile < a.ntiles; tile += gridDim.x * G) {
        int si = 0;
        for (int i = 1; i < a.nseg; ++i)
            if (tile >= a.seg[i].tile_begin) si = i;
        const GemvSeg& sg = a.seg[si];
        const int row0 = (tile - sg.tile_begin) * R;
        const int nrows = min(R, sg.N - row0);
        const int64_t ldq = sg.ldq;
        const uint8_t* rows[R];
#pragma unroll
        for (int r = 0; r < R; ++r)  // rows past the end re-read the last row; results are dropped
            rows[r] = sg.q + (int64_t)(row0 + min(r, nrows - 1)) * ldq + lane * 16;

        float acc[R][B];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][b] = 0.f;

        auto load = [&](float4 (&dst)[R], int s) {
            const int64_t bo = (int64_t)s * kStepBytes;
            const bool valid = bo + lane * 16 < ldq;  // the pitch is a multiple of 16 bytes
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (valid) ldw(rows[r] + bo, dst[r]);
                else dst[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        float4 cur[R], nxt[R];
        if (kw < nsteps) load(cur, kw);
#pragma unroll 2
        for (int s = kw; s < nsteps; s += KS) {
            if (s + KS < nsteps) load(nxt, s + KS);
            const int c0 = s * (kStepBytes / 4) + lane * 4;  // first column of this lane
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float* xr = a.x + (int64_t)b * a.ldx + c0;
                float4 x;
                if (c0 + 3 < K) {
                    x = __ldg(reinterpret_cast<const float4*>(xr));
                } else {
                    x.x = c0 < K ? __ldg(xr) : 0.f;
                    x.y = c0 + 1 < K ? __ldg(xr + 1) : 0.f;
                    x.z = c0 + 2 < K ? __ldg(xr + 2) : 0.f;
                    x.w = c0 + 3 < K ? __ldg(xr + 3) : 0.f;
                }
#pragma unroll
                for (int r = 0; r < R; ++r)
                    acc[r][b] = fmaf(x.x, cur[r].x, fmaf(x.y, cur[r].y, fmaf(x.z, cur[r].z, fmaf(x.w, cur[r].w, acc[r][b]))));
            }
#pragma unroll
            for (int r = 0; r < R; ++r) cur[r] = nxt[r];
        }
        // reduce over lanes, then over the KS warps of the group
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], o);
        if constexpr (KS > 1) {
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) red[warp][b][r] = acc[r][b];
            asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(KS * 32) : "memory");
            if (kw == 0)
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float v = 0.f;
#pragma unroll
                        for (int k2 = 0; k2 < KS; ++k2) v += red[group * KS + k2][b][r];
                        acc[r][b] = v;
                    }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(KS * 32) : "memory");
        }
        if (kw == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b)
                    if (lane == r * B + b && r < nrows) sg.y[(int64_t)b * sg.ldy + row0 + r] = acc[r][b];
        }
    }
}

template <int B, int R, int KS>
cudaError_t launch_t(const GemvArgs& a, int num_sms, cudaStream_t st) {
    constexpr int G = 8 / KS;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_f32_kernel<B, R, KS>, kThreads, 0);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int need = (a.ntiles + G - 1) / G;
    const int grid = need < num_sms * per_sm ? need : num_sms * per_sm;
    gemv_f32_kernel<B, R, KS><<<grid, kThreads, 0, st>>>(a);
    return cudaGetLastError();
}

template <int B>
cudaError_t pick(GemvArgs a, int num_sms, cudaStream_t st) {
    constexpr int R = B <= 2 ? 4 : B <= 4 ? 2 : 1;
    a.nsteps = (a.ldq_min + kStepBytes - 1) / kStepBytes;
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        a.seg[i].tile_begin = ntiles;
        ntiles += (a.seg[i].N + R - 1) / R;
    }
    a.ntiles = ntiles;
    const int64_t target = (int64_t)num_sms * 16;  // ~16 warps in flight per SM
    if ((int64_t)ntiles >= target || a.nsteps < 2) return launch_t<B, R, 1>(a, num_sms, st);
    if ((int64_t)ntiles * 2 >= target || a.nsteps < 4) return launch_t<B, R, 2>(a, num_sms, st);
    if ((int64_t)ntiles * 4 >= target || a.nsteps < 8) return launch_t<B, R, 4>(a, num_sms, st);
    return launch_t<B, R, 8>(a, num_sms, st);
}

}  // namespace

cudaError_t launch_gemv_f32(const GemvArgs& a, int num_sms, cudaStream_t st) {
    switch (a.batch) {
        case 1: return pick<1>(a, num_sms, st);
        case 2: return pick<2>(a, num_sms, st);
        case 3: return pick<3>(a, num_sms, st);
        case 4: return pick<4>(a, num_sms, st);
        case 5: return pick<5>(a, num_sms, st);
        case 6: return pick<6>(a, num_sms, st);
        case 7: return pick<7>(a, num_sms, st);
        case 8: return pick<8>(a, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bramha
