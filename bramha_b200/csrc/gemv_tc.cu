// gemv_tc.cu -- decode GEMV for the quantized formats (batch 1..8) with the
// multiply-accumulate on the tensor cores and only the dequantization on the
// CUDA cores.
//
// Same result as `matvec_mul_into` (src/inference/cpu_engine.rs:1307-1444) on
// int4 (quantize_to_int4, src/models/quantization.rs:41-83), int8
// (quantize_to_int8, :7-38) or log4 (dequantize_log4,
// spanda-engine/src/lib.rs:332-342) weights.
//
// Why tensor cores for a bandwidth-bound GEMV: dequantizing on CUDA cores and
// accumulating with FMAs costs >= 2.6 issue slots per 4-bit code for log4,
// which at full HBM bandwidth is ~94% of an SM's issue rate (ncu measured 4.4
// on the CUDA-core kernel).  Here the CUDA cores only turn two codes into a
// bf16 pair (one shift + one logic op), the pairs go to TMEM with tcgen05.st,
// and tcgen05.mma (A = weights in TMEM, B = activations in shared memory)
// does the products, so the decode costs ~1 issue slot per code.
//
// Exactness: weights are exact in bf16 (log4 -> 2^(c-15), int4 -> 128 + q,
// both corrected in the epilogue with sum(x)); each activation is split into
// bf16 hi + lo (x = hi + lo to ~2^-16), so batch row b uses B columns 2b and
// 2b+1 of the N = 16 MMA and results match fp32 to ~1e-5.
//
// Tile: 128 weight rows x a K-range.  grid = (tiles over all fused weights,
// ksplit); with ksplit > 1 the partial results of a tile are added into y
// (zeroed first) with fp32 atomics.
//   warp 0      bulk copy: one contiguous (tile, k-step) block of the tile-major
//               weight per step (4 KB 4-bit / 8 KB int8) into a 64 KB ring
//   warp 1      TMEM alloc; lane 0 issues tcgen05.mma (kind::f16, M=128, N=16)
//   warp 2      activations: f32 -> bf16 hi/lo B tile (128-byte swizzle), sum(x)
//   warps 4-11  dequantize: two groups take alternate steps; per row 64 codes
//               -> 32 bf16 pairs -> tcgen05.st (store wait overlapped)
//   warps 4-7   epilogue: tcgen05.ld of the accumulator, scale, store
// All mbarrier waits are bounded (tc_common.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

constexpr int TM = 128;                  // weight rows per tile (UMMA M)
constexpr int TK = 64;                   // K per step (4 x UMMA K=16)
constexpr int TN = 16;                   // UMMA N: x_hi / x_lo for up to 8 batch rows
constexpr int kRingBytes = 64 * 1024;    // packed weight ring in shared memory
constexpr int kSX = 8;                   // activation stages
constexpr int kSA = 6;                   // dequantized stages in TMEM (32 columns each)
constexpr int kDCol = 0;                 // accumulator columns [0, 16)
constexpr int kACol = 32;                // A stages from column 32
constexpr int kTmemCols = 256;
constexpr int kThreads = 384;            // 12 warps

struct TcSeg {
    const uint8_t* q;      // tile-major weight (repack.cu)
    const float* scales;
    float* y;              // [B][ldy]
    int64_t ldy;
    int N;
    int tile_begin;
};

struct TcGemvParams {
    TcSeg seg[kMaxSegments];
    const float* x;        // [B][ldx] f32
    int64_t ldx;
    int* err;
    int nseg;
    int ntiles;
    int K;                 // columns held by the packed rows
    int ksteps;            // ceil(K / 64)
    int steps_per_split;
    int atomic_out;        // 1 when gridDim.y > 1
};

// Per-format stage geometry: one stage = one (tile, k-step) block of the
// tile-major layout, read with a single bulk copy.
template <int FMT>
struct Geo {
    static constexpr int kSlice = tile_slice_bytes(FMT);  // bytes per row per step
    static constexpr int kStage = TM * kSlice;            // 4 KB (4-bit) / 8 KB (int8)
    static constexpr int kSW = kRingBytes / kStage;       // ring depth
};

template <int FMT>
struct TcSmem {
    uint8_t w[Geo<FMT>::kSW][Geo<FMT>::kStage];
    uint8_t x[kSX][TN * 128];            // 2 KB each, SW128 K-major (rows 2B..15 stay zero)
    uint64_t w_full[Geo<FMT>::kSW], w_empty[Geo<FMT>::kSW];
    uint64_t x_full[kSX], x_empty[kSX];
    uint64_t a_full[kSA], a_empty[kSA];
    uint64_t acc_full, sx_ready;
    float sx[8];
    uint32_t tmem;
    int abort_flag;
};

// Every lane polls; the warp proceeds only if all lanes saw the phase (so the
// .sync.aligned TMEM instructions that follow stay warp-uniform on timeout).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
    const bool ok = mbar_wait(bar, parity, abort_flag, err);
    return __all_sync(0xffffffffu, ok);
}

// Two 4-bit codes per bf16x2 pair (device word layout, repack.cu): even
// columns in bits 0-15, odd in 16-31.  log4 -> 2^(c-15); int4 -> 128 + q.
template <int FMT>
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t* o) {
    if constexpr (FMT == BRAMHA_FMT_LOG4) {
        constexpr uint32_t M = 0x07800780u, E = 0x38003800u;
        o[0] = ((w << 7) & M) | E;
        o[1] = ((w << 3) & M) | E;
        o[2] = ((w >> 1) & M) | E;
        o[3] = ((w >> 5) & M) | E;
    } else {
        constexpr uint32_t M = 0x000F000Fu, E = 0x43004300u;
        o[0] = (w & M) | E;
        o[1] = ((w >> 4) & M) | E;
        o[2] = ((w >> 8) & M) | E;
        o[3] = ((w >> 12) & M) | E;
    }
}

// int8 -> bf16 pair: bytes of u are q + 128; 0x4B000000 | byte is 2^23 + q + 128.
__device__ __forceinline__ uint32_t i8_pair(uint32_t u, uint32_t sel_lo, uint32_t sel_hi) {
    const float a = __uint_as_float(__byte_perm(u, 0x4Bu, sel_lo)) - 8388736.0f;
    const float b = __uint_as_float(__byte_perm(u, 0x4Bu, sel_hi)) - 8388736.0f;
    __nv_bfloat162 r = __floats2bfloat162_rn(a, b);  // |q| <= 127: exact
    return *reinterpret_cast<uint32_t*>(&r);
}

// A row's 64 codes of one step -> 32 bf16 pairs.
template <int FMT>
__device__ __forceinline__ void dq_row(const uint8_t* slice, uint32_t (&v)[32]) {
    if constexpr (FMT == BRAMHA_FMT_W8) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const uint4 p = *reinterpret_cast<const uint4*>(slice + 16 * h);
            const uint32_t wv[4] = {p.x ^ 0x80808080u, p.y ^ 0x80808080u, p.z ^ 0x80808080u, p.w ^ 0x80808080u};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[8 * h + 2 * i] = i8_pair(wv[i], 0x4550, 0x4551);
                v[8 * h + 2 * i + 1] = i8_pair(wv[i], 0x4552, 0x4553);
            }
        }
    } else {
        const uint4 p0 = *reinterpret_cast<const uint4*>(slice);
        const uint4 p1 = *reinterpret_cast<const uint4*>(slice + 16);
        dq_word<FMT>(p0.x, v + 0);
        dq_word<FMT>(p0.y, v + 4);
        dq_word<FMT>(p0.z, v + 8);
        dq_word<FMT>(p0.w, v + 12);
        dq_word<FMT>(p1.x, v + 16);
        dq_word<FMT>(p1.y, v + 20);
        dq_word<FMT>(p1.z, v + 24);
        dq_word<FMT>(p1.w, v + 28);
    }
}

template <int FMT, int B>
__global__ void __launch_bounds__(kThreads, 2) tc_gemv_kernel(const __grid_constant__ TcGemvParams p) {
    extern __shared__ uint8_t smem_raw[];
    using G = Geo<FMT>;
    constexpr int kSW = G::kSW;
    TcSmem<FMT>& S = *reinterpret_cast<TcSmem<FMT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* abort_flag = &S.abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    int si = 0;
    for (int i = 1; i < p.nseg; ++i)
        if (tile >= p.seg[i].tile_begin) si = i;
    const TcSeg& sg = p.seg[si];
    const int row0 = (tile - sg.tile_begin) * TM;  // first row inside weight si
    const int step0 = blockIdx.y * p.steps_per_split;
    const int nsteps = min(p.steps_per_split, p.ksteps - step0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSW; ++s) {
            mbar_init(&S.w_full[s], 1);
            mbar_init(&S.w_empty[s], 4);
        }
        for (int s = 0; s < kSX; ++s) {
            mbar_init(&S.x_full[s], 1);
            mbar_init(&S.x_empty[s], 1);
        }
        for (int s = 0; s < kSA; ++s) {
            mbar_init(&S.a_full[s], 4);
            mbar_init(&S.a_empty[s], 1);
        }
        mbar_init(&S.acc_full, 1);
        mbar_init(&S.sx_ready, 1);
        S.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // zero the activation tiles once: rows >= 2B are never written again
    for (int i = threadIdx.x; i < kSX * TN * 128 / 16; i += kThreads)
        reinterpret_cast<uint4*>(&S.x[0][0])[i] = make_uint4(0, 0, 0, 0);
    if (warp == 1) tmem_alloc(&S.tmem, kTmemCols);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;

    if (warp == 0) {
        // ---------------- bulk-copy producer: one contiguous block per step
        if (lane == 0) {
            const uint8_t* src = sg.q + ((int64_t)(tile - sg.tile_begin) * p.ksteps + step0) * G::kStage;
            int it = 0;
            for (; it < nsteps; ++it) {
                const int s = it % kSW;
                if (it >= kSW && !mbar_wait(&S.w_empty[s], ((it / kSW) & 1) ^ 1, abort_flag, p.err)) break;
                mbar_expect_tx(&S.w_full[s], G::kStage);
                bulk_load(&S.w[s][0], src + (int64_t)it * G::kStage, G::kStage, &S.w_full[s]);
            }
            for (int j = (it > kSW ? it - kSW : 0); j < it; ++j)
                mbar_wait(&S.w_full[j % kSW], (j / kSW) & 1, abort_flag, p.err);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16<TM, TN>();
            for (int it = 0; it < nsteps; ++it) {
                const int sa = it % kSA, sx = it % kSX;
                if (!mbar_wait(&S.a_full[sa], (it / kSA) & 1, abort_flag, p.err)) break;
                if (!mbar_wait(&S.x_full[sx], (it / kSX) & 1, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t xb = smem_u32(&S.x[sx][0]);
#pragma unroll
                for (int kk = 0; kk < TK / 16; ++kk)
                    umma_bf16_ts(tmem + kDCol, tmem + kACol + sa * 32 + kk * 8, sw128_desc(xb + kk * 32), idesc,
                                 (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&S.a_empty[sa]);
                umma_commit(&S.x_empty[sx]);
            }
            umma_commit(&S.acc_full);
        }
    } else if (warp == 2) {
        // ---------------- activations: hi/lo bf16 B tile per step, sum(x)
        // The loads for PF steps are issued together so one L2 round trip
        // covers several steps (a step's tile is needed every few hundred cycles).
        constexpr int PF = B <= 1 ? 8 : B <= 2 ? 4 : B <= 4 ? 2 : 1;  // steps per round trip
        float sxp[B];
#pragma unroll
        for (int b = 0; b < B; ++b) sxp[b] = 0.f;
        const int chunk = lane >> 2, within = (lane & 3) * 4;
        bool ok = true;
        for (int base = 0; base < nsteps && ok; base += PF) {
            float2 v[PF][B];
#pragma unroll
            for (int j = 0; j < PF; ++j) {
                const int k = (step0 + base + j) * TK + 2 * lane;
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float* xr = p.x + (int64_t)b * p.ldx;
                    v[j][b].x = (base + j < nsteps && k < p.K) ? __ldg(xr + k) : 0.f;
                    v[j][b].y = (base + j < nsteps && k + 1 < p.K) ? __ldg(xr + k + 1) : 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < PF; ++j) {
                const int it = base + j;
                if (it >= nsteps) break;
                const int sx = it % kSX;
                if (it >= kSX && !warp_wait(&S.x_empty[sx], ((it / kSX) & 1) ^ 1, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
                uint8_t* tile_x = &S.x[sx][0];
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const __nv_bfloat162 hi = __floats2bfloat162_rn(v[j][b].x, v[j][b].y);
                    const float2 hf = __bfloat1622float2(hi);
                    const __nv_bfloat162 lo = __floats2bfloat162_rn(v[j][b].x - hf.x, v[j][b].y - hf.y);
                    const float2 lf = __bfloat1622float2(lo);
                    sxp[b] += (hf.x + lf.x) + (hf.y + lf.y);
                    const int rh = 2 * b, rl = 2 * b + 1;
                    *reinterpret_cast<__nv_bfloat162*>(tile_x + rh * 128 + ((chunk ^ (rh & 7)) << 4) + within) = hi;
                    *reinterpret_cast<__nv_bfloat162*>(tile_x + rl * 128 + ((chunk ^ (rl & 7)) << 4) + within) = lo;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.x_full[sx]);
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float v = sxp[b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) S.sx[b] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.sx_ready);
    } else if (warp >= 4) {
        // ---------------- dequantize into TMEM
        // Two groups of four warps (one warp per TMEM lane quarter) take
        // alternate steps; each thread turns its row's 64 codes into 32 bf16
        // pairs.  The wait for a step's tcgen05.st is deferred until the next
        // step's codes are decoded, so the store latency overlaps work.
        const int q4 = warp & 3;               // TMEM lane quarter of this warp
        const int grp = (warp - 4) >> 2;       // steps grp, grp + 2, ...
        const int row = q4 * 32 + lane;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        int pending = -1;                      // stage whose store is not yet published
        for (int it = grp; it < nsteps; it += 2) {
            const int sw = it % kSW, sa = it % kSA;
            if (!warp_wait(&S.w_full[sw], (it / kSW) & 1, abort_flag, p.err)) break;
            uint32_t v[32];
            dq_row<FMT>(&S.w[sw][row * G::kSlice], v);
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.w_empty[sw]);
            if (pending >= 0) {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.a_full[pending]);
                pending = -1;
            }
            if (it >= kSA && !warp_wait(&S.a_empty[sa], ((it / kSA) & 1) ^ 1, abort_flag, p.err)) break;
            tmem_st32(tmem + lane_base + kACol + sa * 32, v);
            pending = sa;
        }
        if (pending >= 0) {
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.a_full[pending]);
        }
        // ---------------- epilogue (warps 4-7: one per lane quarter)
        if (grp == 0) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&S.acc_full, 0, abort_flag, p.err) && mbar_wait(&S.sx_ready, 0, abort_flag, p.err);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (ok) {
                tc_fence_after();
                uint32_t d[16];
                tmem_ld16(tmem + lane_base + kDCol, d);
                const int grow = row0 + row;
                if (grow < sg.N) {
                    const float sc = __ldg(sg.scales + grow);
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        const float acc = __uint_as_float(d[2 * b]) + __uint_as_float(d[2 * b + 1]);
                        float dot;
                        if constexpr (FMT == BRAMHA_FMT_LOG4) dot = fmaf(acc, 32768.0f, -S.sx[b]);
                        else if constexpr (FMT == BRAMHA_FMT_W4ZP8) dot = fmaf(-136.0f, S.sx[b], acc);
                        else dot = acc;  // int8 weights are exact in bf16
                        float* dst = sg.y + (int64_t)b * sg.ldy + grow;
                        if (p.atomic_out) atomicAdd(dst, dot * sc);
                        else *dst = dot * sc;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <int FMT, int B>
cudaError_t launch_b(const TcGemvParams& p, int ksplit, cudaStream_t st) {
    auto kern = tc_gemv_kernel<FMT, B>;
    constexpr int smem = (int)sizeof(TcSmem<FMT>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3((unsigned)p.ntiles, (unsigned)ksplit), kThreads, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace

// Tensor-core GEMV over up to 8 fused quantized weights sharing x (batch 1..8).
// `segs` carry the tile-major device weights, scales and outputs.
cudaError_t launch_gemv_tc(int fmt, const GemvArgs& a, int num_sms, cudaStream_t st) {
    if (!is_tiled(fmt)) return cudaErrorInvalidValue;
    if (a.batch < 1 || a.batch > 8 || a.nseg < 1 || a.nseg > kMaxSegments || a.K <= 0) return cudaErrorInvalidValue;
    TcGemvParams p;
    memset(&p, 0, sizeof(p));
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        const GemvSeg& s = a.seg[i];
        if ((reinterpret_cast<uintptr_t>(s.q) & 15) != 0) return cudaErrorInvalidValue;
        p.seg[i].q = s.q;
        p.seg[i].scales = s.scales;
        p.seg[i].y = s.y;
        p.seg[i].ldy = s.ldy;
        p.seg[i].N = s.N;
        p.seg[i].tile_begin = ntiles;
        ntiles += (int)row_tiles(s.N);
    }
    p.x = a.x;
    p.ldx = a.ldx;
    p.err = a.err;
    p.nseg = a.nseg;
    p.ntiles = ntiles;
    p.K = a.K;
    p.ksteps = (int)k_steps(a.K);
    // split K until ~2 CTAs per SM are busy (each split keeps >= 8 steps)
    int ksplit = 1;
    while (ksplit < 16 && (int64_t)ntiles * ksplit < 2LL * num_sms && p.ksteps / (ksplit * 2) >= 8) ksplit *= 2;
    p.steps_per_split = (p.ksteps + ksplit - 1) / ksplit;
    ksplit = (p.ksteps + p.steps_per_split - 1) / p.steps_per_split;
    p.atomic_out = ksplit > 1;
    if (p.atomic_out)
        for (int i = 0; i < a.nseg; ++i) {
            cudaError_t e = cudaMemsetAsync(a.seg[i].y, 0, sizeof(float) * (size_t)a.seg[i].ldy * a.batch, st);
            if (e != cudaSuccess) return e;
        }
#define BRAMHA_TC_B(n)                                                                     \
    case n:                                                                                \
        return fmt == BRAMHA_FMT_LOG4    ? launch_b<BRAMHA_FMT_LOG4, n>(p, ksplit, st)     \
               : fmt == BRAMHA_FMT_W4ZP8 ? launch_b<BRAMHA_FMT_W4ZP8, n>(p, ksplit, st)    \
                                         : launch_b<BRAMHA_FMT_W8, n>(p, ksplit, st);
    switch (a.batch) {
        BRAMHA_TC_B(1)
        BRAMHA_TC_B(2)
        BRAMHA_TC_B(3)
        BRAMHA_TC_B(4)
        BRAMHA_TC_B(5)
        BRAMHA_TC_B(6)
        BRAMHA_TC_B(7)
        BRAMHA_TC_B(8)
        default: return cudaErrorInvalidValue;
    }
#undef BRAMHA_TC_B
}

}  // namespace bramha
