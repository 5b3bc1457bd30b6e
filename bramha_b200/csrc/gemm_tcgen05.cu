// gemm_tcgen05.cu -- prefill dequant-GEMM on the 5th-generation tensor cores.
//
// Replaces `gemm_cpu` (src/inference/cpu_engine.rs:565-912; the sequential
// branch at :576-706 is what the reference runs):
//     y[m][j] = s_j * sum_k x[m][k] * code(w_jk)
// with bf16 activations and the weights dequantized EXACTLY to bf16:
//     int4 (quantize_to_int4):  q - 8        in [-8, 7]
//     int8 (quantize_to_int8):  q            in [-127, 127]
//     log4 (dequantize_log4) :  2^(c - 15)   and y = s * (2^15 * acc - sum_k x[m][k])
// so the only rounding is the fp32 accumulation in TMEM.
//
// One CTA computes a 128 (weight rows) x BN (tokens) tile: D = W_tile * X_tile^T
// ("weights as the M operand"), looping over K in steps of 64.
//   warp 0      TMA producer: X tile (bf16, 128-byte swizzle, tensor map) and
//               the packed weight block (one contiguous bulk copy from the
//               tile-major layout) per stage, mbarrier complete_tx.
//   warp 1      allocates TMEM (BN fp32 columns), one lane issues tcgen05.mma
//               (M=128, N=BN, K=16, both operands K-major SW128 in shared
//               memory) and tcgen05.commit to release stages.
//   warps 2-5   dequantize: thread t owns weight row t of the tile, reads its
//               packed bytes, writes 8 x 16-byte bf16 chunks in the swizzled
//               K-major layout the MMA descriptor describes; then the epilogue
//               (tcgen05.ld of its TMEM lane, scale, store fp32).
// Every mbarrier wait is bounded (~2 s of %globaltimer): on timeout the kernel
// records BRAMHA_ERR_TIMEOUT in an error word, drains, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

constexpr int BM = 128;          // weight rows per tile (UMMA M)
constexpr int BK = 64;           // K per stage: 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;    // 6 warps

struct GemmArgs {
    const uint8_t* q;      // tile-major weight (repack.cu)
    const float* scales;   // [N]
    const float* rowsum;   // [M] sum of the bf16 activations (log4 only)
    float* y;              // [M][ldy]
    int64_t ldy;
    int M, N, K;
    int k_steps;
    int accumulate;        // 0: y = result, 1: y += result (second half of a hi/lo split)
    int* err;              // device error word (0 = ok)
};

// Packed weight bytes per row per stage.
template <int FMT>
constexpr int packed_bytes() {
    return FMT == BRAMHA_FMT_W8 ? BK : BK / 2;
}

// ---- dequantization of one 8-column chunk into 4 bf16x2 words ------------
// 4-bit device word: even columns in bits 0-15, odd in 16-31 (repack.cu), so
// the pair (2j, 2j+1) is nibble j of each half.
__device__ __forceinline__ uint4 dq_log4(uint32_t w) {
    // shift nibble j of each half to bits 7-10 / 23-26, then exponent base 112:
    // bf16 value 2^(c - 15), exact.
    constexpr uint32_t M = 0x07800780u, E = 0x38003800u;
    uint4 o;
    o.x = ((w << 7) & M) | E;
    o.y = ((w << 3) & M) | E;
    o.z = ((w >> 1) & M) | E;
    o.w = ((w >> 5) & M) | E;
    return o;
}
__device__ __forceinline__ uint32_t bf2_sub136(uint32_t v) {
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&v);
    const __nv_bfloat162 c = __floats2bfloat162_rn(136.0f, 136.0f);
    a = __hsub2(a, c);  // (128 + n) - 136 = n - 8, exact
    return *reinterpret_cast<uint32_t*>(&a);
}
__device__ __forceinline__ uint4 dq_int4(uint32_t w) {
    // nibble at bits 0-3 of each half OR'ed into bf16 128.0 -> 128 + n
    constexpr uint32_t M = 0x000F000Fu, E = 0x43004300u;
    uint4 o;
    o.x = bf2_sub136((w & M) | E);
    o.y = bf2_sub136(((w >> 4) & M) | E);
    o.z = bf2_sub136(((w >> 8) & M) | E);
    o.w = bf2_sub136(((w >> 12) & M) | E);
    return o;
}
__device__ __forceinline__ uint32_t i8pair_bf16(uint32_t u, uint32_t sel_lo, uint32_t sel_hi) {
    // bytes of u are q + 128; 0x4B000000 | byte = 2^23 + q + 128 exactly
    const float a = __uint_as_float(__byte_perm(u, 0x4Bu, sel_lo)) - 8388736.0f;
    const float b = __uint_as_float(__byte_perm(u, 0x4Bu, sel_hi)) - 8388736.0f;
    __nv_bfloat162 r = __floats2bfloat162_rn(a, b);  // |q| <= 127: exact
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint4 dq_int8(uint32_t w0, uint32_t w1) {
    const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u;
    uint4 o;
    o.x = i8pair_bf16(u0, 0x4550, 0x4551);
    o.y = i8pair_bf16(u0, 0x4552, 0x4553);
    o.z = i8pair_bf16(u1, 0x4550, 0x4551);
    o.w = i8pair_bf16(u1, 0x4552, 0x4553);
    return o;
}

template <int FMT, int BN, int S>
struct Layout {
    static constexpr int kX = BN * 128;                   // bytes per X stage
    static constexpr int kA = BM * 128;                   // bytes per dequantized W stage
    static constexpr int kP = BM * packed_bytes<FMT>();   // bytes per packed W stage
    static constexpr int offX = 0;
    static constexpr int offA = offX + S * kX;
    static constexpr int offP = offA + S * kA;
    static constexpr int offBar = offP + S * kP;          // full_tma[S], full_a[S], empty[S], acc_full
    static constexpr int offTmem = offBar + (3 * S + 1) * 8;
    static constexpr int offAbort = offTmem + 4;
    static constexpr int kBytes = offAbort + 4;
    static constexpr int kAlloc = kBytes + 1024;           // slack to align the base to 1024
    static_assert(kAlloc <= 227 * 1024, "shared memory per CTA exceeds 227 KB");
    static_assert(S >= 2, "need at least two stages");
};

template <int FMT, int BN, int S>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ GemmArgs a) {
    using L = Layout<FMT, BN, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Xs = smem + L::offX;
    uint8_t* As = smem + L::offA;
    uint8_t* Ps = smem + L::offP;
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(smem + L::offBar);
    uint64_t* full_a = full_tma + S;
    uint64_t* empty = full_a + S;
    uint64_t* acc_full = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::offTmem);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::offAbort);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM;   // first weight row
    const int m0 = blockIdx.y * BN;   // first token
    const int ksteps = a.k_steps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&full_a[s], 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            constexpr uint32_t kTx = L::kX + L::kP;
            int it = 0;
            for (; it < ksteps; ++it) {
                const int s = it % S;
                if (it >= S && !mbar_wait(&empty[s], ((it / S) & 1) ^ 1, abort_flag, a.err)) break;
                mbar_expect_tx(&full_tma[s], kTx);
                tma_load_2d(Xs + s * L::kX, &tmX, &full_tma[s], it * BK, m0);
                bulk_load(Ps + s * L::kP, a.q + ((int64_t)blockIdx.x * ksteps + it) * L::kP, L::kP, &full_tma[s]);
            }
            // drain: every issued copy has landed before the CTA can exit
            for (int j = (it > S ? it - S : 0); j < it; ++j)
                mbar_wait(&full_tma[j % S], (j / S) & 1, abort_flag, a.err);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16<BM, BN>();
            for (int it = 0; it < ksteps; ++it) {
                const int s = it % S;
                const uint32_t ph = (it / S) & 1;
                if (!mbar_wait(&full_a[s], ph, abort_flag, a.err)) break;
                if (!mbar_wait(&full_tma[s], ph, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t a_base = smem_u32(As + s * L::kA);
                const uint32_t b_base = smem_u32(Xs + s * L::kX);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    umma_bf16(tmem, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), idesc,
                              (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);  // fires when every MMA issued above has completed
        }
    } else {
        // ---------------- dequantize (threads 64..191 -> tile rows)
        const int q4 = warp & 3;                 // TMEM lane quarter this warp may access
        const int row = q4 * 32 + lane;          // row of the tile == TMEM lane
        for (int it = 0; it < ksteps; ++it) {
            const int s = it % S;
            if (!mbar_wait(&full_tma[s], (it / S) & 1, abort_flag, a.err)) break;
            const uint8_t* prow = Ps + s * L::kP + row * packed_bytes<FMT>();
            uint8_t* arow = As + s * L::kA + row * 128;
            if constexpr (FMT == BRAMHA_FMT_W8) {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    // int8 slices are stored 64-byte-swizzled (repack.cu)
                    const uint4 p = *reinterpret_cast<const uint4*>(prow + 16 * (h ^ ((row >> 1) & 3)));
                    const int c0 = 2 * h, c1 = 2 * h + 1;
                    *reinterpret_cast<uint4*>(arow + ((c0 ^ (row & 7)) << 4)) = dq_int8(p.x, p.y);
                    *reinterpret_cast<uint4*>(arow + ((c1 ^ (row & 7)) << 4)) = dq_int8(p.z, p.w);
                }
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 p = *reinterpret_cast<const uint4*>(prow + 16 * h);
                    const uint32_t wv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int c = 4 * h + i;
                        const uint4 o = (FMT == BRAMHA_FMT_LOG4) ? dq_log4(wv[i]) : dq_int4(wv[i]);
                        *reinterpret_cast<uint4*>(arow + ((c ^ (row & 7)) << 4)) = o;
                    }
                }
            }
            fence_async_smem();  // generic-proxy writes -> visible to the tensor core
            mbar_arrive(&full_a[s]);
        }
        // ---------------- epilogue (warp-uniform: tcgen05.ld is .sync.aligned)
        bool ok = true;
        if (lane == 0) ok = mbar_wait(acc_full, 0, abort_flag, a.err);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok) {
            tc_fence_after();
            const int grow = n0 + row;
            const float sc = grow < a.N ? __ldg(a.scales + grow) : 0.f;
            const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(taddr + c0, v);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int tok = m0 + c0 + j;
                    if (tok < a.M && grow < a.N) {
                        float acc = __uint_as_float(v[j]);
                        if constexpr (FMT == BRAMHA_FMT_LOG4) acc = fmaf(acc, 32768.0f, -__ldg(a.rowsum + tok));
                        float* dst = a.y + (int64_t)tok * a.ldy + grow;
                        *dst = a.accumulate ? fmaf(acc, sc, *dst) : acc * sc;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

// ---- activation preparation ------------------------------------------------
// bf16 copy with a TMA-friendly pitch and per-token sums of exactly the values
// the MMA sees.  From f32 the activation is split x = hi + lo (hi = bf16(x),
// lo = bf16(x - hi)), so two accumulating passes reproduce x to ~2^-16.
template <bool FROM_F32>
__global__ void prep_kernel(const void* __restrict__ x, int64_t ldx, int M, int K, int64_t ldb,
                            __nv_bfloat16* __restrict__ xhi, __nv_bfloat16* __restrict__ xlo,
                            float* __restrict__ rs_hi, float* __restrict__ rs_lo) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    float sh = 0.f, sl = 0.f;
    for (int k = lane; k < (int)ldb; k += 32) {
        float h = 0.f, l = 0.f;
        if (k < K) {
            if constexpr (FROM_F32) {
                const float v = static_cast<const float*>(x)[(int64_t)warp * ldx + k];
                const __nv_bfloat16 hb = __float2bfloat16_rn(v);
                h = __bfloat162float(hb);
                l = __bfloat162float(__float2bfloat16_rn(v - h));
            } else {
                h = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[(int64_t)warp * ldx + k]);
            }
        }
        if (xhi) xhi[(int64_t)warp * ldb + k] = __float2bfloat16_rn(h);
        if (xlo) xlo[(int64_t)warp * ldb + k] = __float2bfloat16_rn(l);
        sh += h;
        sl += l;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sh += __shfl_xor_sync(0xffffffffu, sh, o);
        sl += __shfl_xor_sync(0xffffffffu, sl, o);
    }
    if (lane == 0) {
        if (rs_hi) rs_hi[warp] = sh;
        if (rs_lo) rs_lo[warp] = sl;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int FMT, int BN, int S>
cudaError_t launch_tiles(const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    using L = Layout<FMT, BN, S>;
    auto kern = gemm_kernel<FMT, BN, S>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    dim3 grid((g.N + BM - 1) / BM, (g.M + BN - 1) / BN);
    kern<<<grid, kThreads, L::kAlloc, st>>>(tmX, g);
    return cudaGetLastError();
}

// Pipeline depth: as many stages as fit in the 227 KB of shared memory a CTA
// may use (at most 8).
template <int FMT, int BN>
constexpr int stages_for() {
    constexpr int per_stage = BN * 128 + BM * 128 + BM * packed_bytes<FMT>();
    constexpr int budget = 227 * 1024 - 1024 - 256;  // alignment slack, barriers
    constexpr int s = budget / per_stage;
    return s > 8 ? 8 : s;
}

template <int FMT>
cudaError_t launch_fmt(int bn, const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    switch (bn) {
        case 256: return launch_tiles<FMT, 256, stages_for<FMT, 256>()>(tmX, g, st);
        case 128: return launch_tiles<FMT, 128, stages_for<FMT, 128>()>(tmX, g, st);
        case 64: return launch_tiles<FMT, 64, stages_for<FMT, 64>()>(tmX, g, st);
        default: return launch_tiles<FMT, 32, stages_for<FMT, 32>()>(tmX, g, st);
    }
}

}  // namespace

// Tokens per tile for M tokens.
int gemm_tile_n(int64_t M) { return M >= 256 ? 256 : M > 64 ? 128 : M > 32 ? 64 : 32; }

namespace {
cudaError_t make_x_map(CUtensorMap* m, const void* xg, int64_t K, int64_t M, int64_t xld, int bn) {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(xld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(xg), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
cudaError_t run_pass(int fmt, int bn, const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    switch (fmt) {
        case BRAMHA_FMT_LOG4: return launch_fmt<BRAMHA_FMT_LOG4>(bn, tmX, g, st);
        case BRAMHA_FMT_W4ZP8: return launch_fmt<BRAMHA_FMT_W4ZP8>(bn, tmX, g, st);
        case BRAMHA_FMT_W8: return launch_fmt<BRAMHA_FMT_W8>(bn, tmX, g, st);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace

// y[M][ldy] = dequant(W)[N][K] applied to x[M][ldx] (bf16, or f32 split into
// two bf16 passes).  K is the number of columns the packed rows hold.
// Scratch (bf16 copies, per-token sums) comes from the stream-ordered pool.
cudaError_t launch_gemm_tcgen05(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N, int64_t K,
                                const void* x, int x_is_f32, int64_t ldx, int64_t M, float* y, int64_t ldy, int* err,
                                cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || K <= 0) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    const int64_t kp = (K + BK - 1) / BK * BK;  // bf16 copy pitch: whole K steps
    const bool need_copy = x_is_f32 || (ldx % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0;
    const bool log4 = fmt == BRAMHA_FMT_LOG4;
    const int npass = x_is_f32 ? 2 : 1;
    // scratch: [npass] bf16 copies, [npass] row sums
    size_t bytes = 0;
    if (need_copy) bytes += (size_t)npass * M * kp * sizeof(__nv_bfloat16);
    if (log4) bytes += (size_t)npass * M * sizeof(float);
    uint8_t* scratch = nullptr;
    cudaError_t e = bytes ? cudaMallocAsync(reinterpret_cast<void**>(&scratch), bytes, st) : cudaSuccess;
    if (e != cudaSuccess) return e;
    __nv_bfloat16* xb[2] = {nullptr, nullptr};
    float* rs[2] = {nullptr, nullptr};
    uint8_t* p = scratch;
    if (need_copy)
        for (int i = 0; i < npass; ++i, p += (size_t)M * kp * sizeof(__nv_bfloat16))
            xb[i] = reinterpret_cast<__nv_bfloat16*>(p);
    if (log4)
        for (int i = 0; i < npass; ++i, p += (size_t)M * sizeof(float)) rs[i] = reinterpret_cast<float*>(p);
    if (need_copy || log4) {
        const int wpb = 8;
        const unsigned blocks = (unsigned)((M + wpb - 1) / wpb);
        const int64_t ldb = need_copy ? kp : K;
        if (x_is_f32)
            prep_kernel<true><<<blocks, 32 * wpb, 0, st>>>(x, ldx, (int)M, (int)K, ldb, xb[0], xb[1], rs[0], rs[1]);
        else
            prep_kernel<false><<<blocks, 32 * wpb, 0, st>>>(x, ldx, (int)M, (int)K, ldb, xb[0], nullptr, rs[0],
                                                           nullptr);
        e = cudaGetLastError();
    }
    const int bn = gemm_tile_n(M);
    if ((reinterpret_cast<uintptr_t>(q) & 15) != 0) e = cudaErrorInvalidValue;
    for (int pass = 0; pass < npass && e == cudaSuccess; ++pass) {
        const void* xg = need_copy ? static_cast<const void*>(xb[pass]) : x;
        CUtensorMap tmX;
        e = make_x_map(&tmX, xg, K, M, need_copy ? kp : ldx, bn);
        if (e != cudaSuccess) break;
        GemmArgs g;
        g.q = q;
        g.scales = scales;
        g.rowsum = rs[pass];
        g.y = y;
        g.ldy = ldy;
        g.M = (int)M;
        g.N = (int)N;
        g.K = (int)K;
        g.k_steps = (int)((K + BK - 1) / BK);
        g.accumulate = pass;
        g.err = err;
        e = run_pass(fmt, bn, tmX, g, st);
    }
    if (scratch) {
        cudaError_t e2 = cudaFreeAsync(scratch, st);
        if (e == cudaSuccess) e = e2;
    }
    return e;
}

cudaError_t launch_gemm_tcgen05_bf16_noalloc(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N,
                                             int64_t K, const void* x, int64_t ldx, int64_t M, float* y,
                                             int64_t ldy, int* err, float* rowsum_scratch, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || K <= 0) return cudaErrorInvalidValue;
    if ((ldx % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaSuccess;
    float* rs = nullptr;
    if (fmt == BRAMHA_FMT_LOG4) {
        if (!rowsum_scratch) return cudaErrorInvalidValue;
        rs = rowsum_scratch;
        const int wpb = 8;
        const unsigned blocks = (unsigned)((M + wpb - 1) / wpb);
        // every one of the M sums is written here before the GEMM reads it
        prep_kernel<false><<<blocks, 32 * wpb, 0, st>>>(x, ldx, (int)M, (int)K, K, nullptr, nullptr, rs, nullptr);
        e = cudaGetLastError();
    }
    const int bn = gemm_tile_n(M);
    CUtensorMap tmX;
    if (e == cudaSuccess && (reinterpret_cast<uintptr_t>(q) & 15) != 0) e = cudaErrorInvalidValue;
    if (e == cudaSuccess) e = make_x_map(&tmX, x, K, M, ldx, bn);
    if (e != cudaSuccess) return e;
    GemmArgs g;
    g.q = q;
    g.scales = scales;
    g.rowsum = rs;
    g.y = y;
    g.ldy = ldy;
    g.M = (int)M;
    g.N = (int)N;
    g.K = (int)K;
    g.k_steps = (int)((K + BK - 1) / BK);
    g.accumulate = 0;
    g.err = err;
    return run_pass(fmt, bn, tmX, g, st);
}

}  // namespace bramha
