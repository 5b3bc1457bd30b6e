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
// Tiles are 128 weight rows x BN tokens: D = W_tile * X_tile^T ("weights as the
// M operand"), K in steps of 64.  The kernel is persistent (one CTA per SM walks
// tiles blockIdx.x, +gridDim.x, ...) and keeps two accumulators in TMEM, so the
// epilogue of one tile overlaps the main loop of the next.
//   warp 0      producer: per K step one TMA load of the X tile (bf16, 128-byte
//               swizzle) and one bulk copy of the packed weight block (tile-major
//               layout, repack.cu) into the load ring.
//   warp 1      allocates TMEM (2 x BN fp32 columns); one lane issues
//               tcgen05.mma (M=128, N=BN, K=16, both operands K-major SW128 in
//               shared memory) and tcgen05.commit releases the ring slots and
//               hands finished accumulators to the epilogue.
//   warps 2-5   dequantize: thread t owns weight row t, reads its packed bytes
//               from the load ring and writes 8 x 16-byte bf16 chunks into the
//               swizzled K-major layout of the operand ring.
//   warps 6-9   epilogue: tcgen05.ld of their TMEM lane quarter, scale (and the
//               log4 correction), fp32 stores; then release the accumulator.
// f32 activations are split x = hi + lo (both bf16) and laid side by side along
// K, so one pass over 2K accumulates both halves.
// Every mbarrier wait is bounded (~2 s of %globaltimer): on timeout the kernel
// records BRAMHA_ERR_TIMEOUT in an error word, drains, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <climits>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

constexpr int BM = 128;          // weight rows per tile (UMMA M)
constexpr int BK = 64;           // K per stage: 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 320;    // 10 warps

struct GemmArgs {
    const uint8_t* q;      // tile-major weight (repack.cu)
    const float* scales;   // [N]
    const float* rowsum;   // [M] sum of the activations the MMA sees (log4 only)
    float* y;              // [M][ldy]
    int64_t ldy;
    int M, N;
    int k_steps;           // 64-column weight blocks per tile row
    int x_steps;           // K steps per tile: k_steps, or 2 * k_steps for a hi|lo split
    int n_tiles, m_tiles;  // tiles along the weight rows and along the tokens
    int n_blocks;          // 128-row blocks of the repacked weight (ceil(N / 128))
    int* err;              // device error word (0 = ok)
    // Grouped GEMM (MoE experts; 1-SM kernel only): when `tiles` is set the
    // tile list comes from device memory -- *ntiles_dev entries of (128-row
    // block of the stacked weight, first token row, tokens in the tile,
    // first output column) -- and N is the row count of one group.
    const int4* tiles;
    const int* ntiles_dev;
    // Split in N (grouped mode): nonzero = the X copy holds the bf16 hi parts of
    // the M token rows at rows [0, M) and the lo parts at rows [lo_row,
    // lo_row + M); a tile carries BN/2 tokens, its hi rows in MMA columns
    // [0, BN/2) and its lo rows in [BN/2, BN), and the epilogue adds the two.
    // One pass over K: each weight block is loaded and dequantized once.  Also
    // used without a table (a tile then carries BN/2 tokens).
    int lo_row;
    // K split (single-CTA kernel, no tile table): each (weight block, token
    // block) is cut into ksplit ranges of ks_steps K steps; a range writes its
    // raw accumulators to `ws` and takes a ticket (one per TMEM lane quarter);
    // the last range to arrive adds them in range order, applies the scale
    // (and log4 correction) and stores y -- the result does not depend on
    // which range finishes first.
    int ksplit, ks_steps;
    float* ws;
    int* tickets;
};

// One output tile: 128-row block `wblk` of the (stacked) weight, token rows
// [tok0, tok0 + mcount) of X and y, output columns [col0, col0 + 128), K steps
// [kx0, kx1) (K split: range ks of the tile's nm-th (block, token block)).
struct TileInfo {
    int wblk, tok0, mcount, col0;
    int kx0, kx1, nm, ks;
};
template <int BN>
__device__ __forceinline__ TileInfo tile_info(const GemmArgs& a, int t) {
    if (a.tiles) {
        const int4 v = __ldg(a.tiles + t);
        return {v.x, v.y, v.z, v.w, 0, a.x_steps, t, 0};
    }
    const int tpt = a.lo_row ? BN / 2 : BN;  // tokens per tile
    const int ks = t % a.ksplit, nm = t / a.ksplit;
    const int nt = nm % a.n_tiles, mt = nm / a.n_tiles;
    const int kx0 = ks * a.ks_steps;
    return {nt, mt * tpt, min(tpt, a.M - mt * tpt), nt * BM, kx0, min(kx0 + a.ks_steps, a.x_steps), nm, ks};
}

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

// Shared memory: a load ring (X tile + packed weight block per slot, filled by
// the producer, freed by the MMA commit) and an operand ring (dequantized bf16
// weight tile per slot, filled by the dequant warps, freed by the MMA commit).
template <int FMT, int BN>
struct Layout {
    static constexpr int kX = BN * 128;                   // bytes per X slot
    static constexpr int kA = BM * 128;                   // bytes per dequantized W slot
    static constexpr int kP = BM * packed_bytes<FMT>();   // bytes per packed W slot
    static constexpr int kBudget = 227 * 1024 - 1024 - 512;  // alignment slack, barriers
    static constexpr int S2 = 4;                          // operand ring depth
    static constexpr int kS1 = (kBudget - S2 * kA) / (kX + kP);
    static constexpr int S1 = kS1 > 6 ? 6 : kS1;          // load ring depth
    static constexpr int offX = 0;
    static constexpr int offA = offX + S1 * kX;
    static constexpr int offP = offA + S2 * kA;
    // full_tma[S1], empty_x[S1], full_a[S2], empty_a[S2], acc_full[2], acc_empty[2], mma_done
    static constexpr int offBar = offP + S1 * kP;
    static constexpr int offTmem = offBar + (2 * S1 + 2 * S2 + 5) * 8;
    static constexpr int offAbort = offTmem + 4;
    static constexpr int kBytes = offAbort + 4;
    static constexpr int kAlloc = kBytes + 1024;          // slack to align the base to 1024
    static constexpr uint32_t kTmemCols = 2 * BN;         // two accumulators
    static_assert(kAlloc <= 227 * 1024, "shared memory per CTA exceeds 227 KB");
    static_assert(S1 >= 3, "load ring too shallow");
};

template <int FMT, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ GemmArgs a) {
    using L = Layout<FMT, BN>;
    constexpr int S1 = L::S1, S2 = L::S2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Xs = smem + L::offX;
    uint8_t* As = smem + L::offA;
    uint8_t* Ps = smem + L::offP;
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(smem + L::offBar);
    uint64_t* empty_x = full_tma + S1;
    uint64_t* full_a = empty_x + S1;
    uint64_t* empty_a = full_a + S2;
    uint64_t* acc_full = empty_a + S2;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::offTmem);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::offAbort);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = a.tiles ? __ldg(a.ntiles_dev) : a.n_tiles * a.m_tiles * a.ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S1; ++s) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&empty_x[s], 1);
        }
        for (int s = 0; s < S2; ++s) {
            mbar_init(&full_a[s], 128);
            mbar_init(&empty_a[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, L::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            constexpr uint32_t kTx = L::kX + L::kP;
            // test-only fault: CTA 0 withholds the copies of its second K step
            const int withheld = blockIdx.x == 0 && injected_fault(a.err) == kFaultGemmWithholdCopy ? 1 : -1;
            int g = 0;  // K steps issued by this CTA, over all its tiles
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const TileInfo ti = tile_info<BN>(a, t);
                const uint8_t* wsrc = a.q + (int64_t)ti.wblk * a.k_steps * L::kP;
                for (int kx = ti.kx0; kx < ti.kx1; ++kx, ++g) {
                    const int s = g % S1;
                    if (g >= S1 && !mbar_wait(&empty_x[s], ((g / S1) & 1) ^ 1, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    if (g == withheld) continue;
                    mbar_expect_tx(&full_tma[s], kTx);
                    if (a.lo_row) {  // hi and lo rows of the tile's tokens, one half slot each
                        tma_load_2d(Xs + s * L::kX, &tmX, &full_tma[s], kx * BK, ti.tok0);
                        tma_load_2d(Xs + s * L::kX + L::kX / 2, &tmX, &full_tma[s], kx * BK, a.lo_row + ti.tok0);
                    } else {
                        tma_load_2d(Xs + s * L::kX, &tmX, &full_tma[s], kx * BK, ti.tok0);
                    }
                    const int kw = kx < a.k_steps ? kx : kx - a.k_steps;
                    bulk_load(Ps + s * L::kP, wsrc + (int64_t)kw * L::kP, L::kP, &full_tma[s]);
                }
            }
            // every issued copy lands before the CTA can exit
            const uint64_t deadline = globaltimer() + wait_limit_ns(a.err);
            for (int j = (g > S1 ? g - S1 : 0); j < g; ++j)
                if (j != withheld) mbar_wait_until(&full_tma[j % S1], (j / S1) & 1, deadline);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16<BM, BN>();
            int g = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
                const int buf = lt & 1;
                if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * BN);
                const TileInfo ti = tile_info<BN>(a, t);
                for (int kx = ti.kx0; kx < ti.kx1; ++kx, ++g) {
                    const int s1 = g % S1, s2 = g % S2;
                    if (!mbar_wait(&full_a[s2], (g / S2) & 1, abort_flag, a.err) ||
                        !mbar_wait(&full_tma[s1], (g / S1) & 1, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(As + s2 * L::kA);
                    const uint32_t b_base = smem_u32(Xs + s1 * L::kX);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_bf16(d, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), idesc,
                                  (kx > ti.kx0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty_x[s1]);
                    umma_commit(&empty_a[s2]);
                }
                if (ok) umma_commit(&acc_full[buf]);
            }
            // every MMA issued above completes before TMEM is freed
            umma_commit(mma_done);
            mbar_wait_until(mma_done, 0, globaltimer() + wait_limit_ns(a.err));
        }
    } else if (warp < 6) {
        // ---------------- dequantize (threads 64..191 -> tile rows)
        const int row = (warp - 2) * 32 + lane;
        int g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const TileInfo ti = tile_info<BN>(a, t);
            for (int kx = ti.kx0; kx < ti.kx1; ++kx, ++g) {
                const int s1 = g % S1, s2 = g % S2;
                if (!mbar_wait(&full_tma[s1], (g / S1) & 1, abort_flag, a.err) ||
                    (g >= S2 && !mbar_wait(&empty_a[s2], ((g / S2) & 1) ^ 1, abort_flag, a.err))) {
                    ok = false;
                    break;
                }
                const uint8_t* prow = Ps + s1 * L::kP + row * packed_bytes<FMT>();
                uint8_t* arow = As + s2 * L::kA + row * 128;
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
                mbar_arrive(&full_a[s2]);
            }
        }
    } else {
        // ---------------- epilogue (warp-uniform: tcgen05.ld is .sync.aligned)
        const int q4 = warp & 3;  // TMEM lane quarter this warp may access
        const int row = q4 * 32 + lane;
        int lt = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
            const int buf = lt & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&acc_full[buf], (lt >> 1) & 1, abort_flag, a.err);
            if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
            tc_fence_after();
            const TileInfo ti = tile_info<BN>(a, t);
            const int grow = ti.col0 + row;
            const int m0 = ti.tok0, mc = ti.mcount;
            const bool row_ok = grow < a.N;
            // a tile inside the matrix stores without per-element bounds checks
            // (a conditional store per element costs ~4x in issue)
            const int ntok = a.lo_row ? BN / 2 : BN;  // tokens per tile
            const bool full = ti.col0 + BM <= a.N && mc == ntok;
            const float sc = row_ok ? __ldg(a.scales + (int64_t)ti.wblk * BM + row) : 0.f;
            float* ycol = a.y + grow;
            const uint32_t taddr = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q4 * 32) << 16);
            if (a.ksplit > 1) {
                // K split: this range's raw accumulators -> workspace (token-major,
                // a warp's 32 rows contiguous), then a ticket; the last range adds
                // the ranges in order and stores the scaled result
                float* part = a.ws + ((int64_t)ti.nm * a.ksplit + ti.ks) * (BM * ntok);
#pragma unroll 1
                for (int c0 = 0; c0 < ntok; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    float o[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = __uint_as_float(v[j]);
                    if (a.lo_row) {
                        tmem_ld32(taddr + (uint32_t)(BN / 2) + c0, v);
#pragma unroll
                        for (int j = 0; j < 32; ++j) o[j] += __uint_as_float(v[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) part[(int64_t)(c0 + j) * BM + row] = o[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);  // TMEM no longer read
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(&a.tickets[ti.nm * 4 + q4], 1) == a.ksplit - 1;
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    __threadfence();
                    const float* p0 = a.ws + (int64_t)ti.nm * a.ksplit * (BM * ntok);
#pragma unroll 1
                    for (int c0 = 0; c0 < ntok; c0 += 32) {
                        float rs = 0.f;
                        if constexpr (FMT == BRAMHA_FMT_LOG4) rs = c0 + lane < mc ? __ldg(a.rowsum + m0 + c0 + lane) : 0.f;
                        float o[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) o[j] = __ldcg(p0 + (int64_t)(c0 + j) * BM + row);
                        for (int r = 1; r < a.ksplit; ++r) {
                            const float* pr = p0 + (int64_t)r * (BM * ntok);
#pragma unroll
                            for (int j = 0; j < 32; ++j) o[j] += __ldcg(pr + (int64_t)(c0 + j) * BM + row);
                        }
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if constexpr (FMT == BRAMHA_FMT_LOG4)
                                o[j] = fmaf(o[j], 32768.0f, -__shfl_sync(0xffffffffu, rs, j));
                            o[j] *= sc;
                        }
                        float* yc = ycol + (int64_t)(m0 + c0) * a.ldy;
                        if (full) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) yc[(int64_t)j * a.ldy] = o[j];
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (row_ok && c0 + j < mc) yc[(int64_t)j * a.ldy] = o[j];
                        }
                    }
                    if (lane == 0) a.tickets[ti.nm * 4 + q4] = 0;  // ready for the next launch
                }
                continue;
            }
            // log4: per-token sums, one chunk of 32 ahead of its use
            float rs_next = 0.f;
            if constexpr (FMT == BRAMHA_FMT_LOG4) rs_next = lane < mc ? __ldg(a.rowsum + m0 + lane) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < ntok; c0 += 32) {
                const float rs = rs_next;
                if constexpr (FMT == BRAMHA_FMT_LOG4) {
                    const int tl = c0 + 32 + lane;
                    if (c0 + 32 < ntok) rs_next = tl < mc ? __ldg(a.rowsum + m0 + tl) : 0.f;
                }
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                float o[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __uint_as_float(v[j]);
                if (a.lo_row) {  // + the lo parts' accumulator (warp-uniform)
                    tmem_ld32(taddr + (uint32_t)(BN / 2) + c0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] += __uint_as_float(v[j]);
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if constexpr (FMT == BRAMHA_FMT_LOG4) o[j] = fmaf(o[j], 32768.0f, -__shfl_sync(0xffffffffu, rs, j));
                    o[j] *= sc;
                }
                float* yc = ycol + (int64_t)(m0 + c0) * a.ldy;
                if (full) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) yc[(int64_t)j * a.ldy] = o[j];
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (row_ok && c0 + j < mc) yc[(int64_t)j * a.ldy] = o[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, L::kTmemCols);
    }
}

// ---- SM-pair kernel ------------------------------------------------------------
// A tile of 256 weight rows x 256 tokens is computed by a cluster of two CTAs
// with tcgen05.mma.cta_group::2 (M=256, N=256, K=16), issued by one thread of
// CTA 0.  CTA r holds weight rows r*128.. of the tile (its own dequantized
// operand) and tokens r*128.. of the X tile (its half of B); each CTA's TMEM
// receives its 128 rows of D.  Per pair and K step the X tile crosses L2 once
// (each CTA loads half), so the L2 -> SM traffic per flop is ~1.8x lower than
// the single-CTA 128 x 256 tile, and each MMA instruction covers twice the work.
// Synchronisation across the pair: every copy completes on a barrier of its own
// CTA; each dequant warp, once its rows are written and this CTA's X half has
// landed, arrives on CTA 0's full_a barrier (through the cluster address for
// CTA 1), so full_a alone tells the MMA issuer that both CTAs' operands are in
// place; epilogue warps release an accumulator the same way (acc_empty); the
// MMA commits are multicast to the barrier at the same offset in both CTAs.
// Remote barrier traffic is one arrival per warp and step.  No TMA multicast.
constexpr int kPairTok = 256;  // tokens per pair tile (N of the MMA)
template <int FMT>
struct PairLayout {
    static constexpr int kX = (kPairTok / 2) * 128;       // this CTA's half of the X tile
    static constexpr int kA = BM * 128;                   // this CTA's dequantized weight rows
    static constexpr int kP = BM * packed_bytes<FMT>();   // this CTA's packed weight block
    static constexpr int kSlot = kX + kA + kP;
    static constexpr int kBudget = 227 * 1024 - 1024 - 512;
    static constexpr int S = kBudget / kSlot > 6 ? 6 : kBudget / kSlot;
    static constexpr int offX = 0;
    static constexpr int offA = offX + S * kX;
    static constexpr int offP = offA + S * kA;
    // full_x[S] (this CTA's X half), full_p[S] (this CTA's packed block), full_a[S] (CTA 0: 8 warps),
    // empty[S] (multicast commit), acc_full[2] (multicast commit), acc_empty[2] (CTA 0: 8 warps), mma_done
    static constexpr int offBar = offP + S * kP;
    static constexpr int offTmem = offBar + (4 * S + 5) * 8;
    static constexpr int offAbort = offTmem + 4;
    static constexpr int kBytes = offAbort + 4;
    static constexpr int kAlloc = kBytes + 1024;
    static constexpr int kThreads = 320;                  // producer, MMA, 4 dequant, 4 epilogue warps
    static constexpr uint32_t kTmemCols = 512;            // two 256-column accumulators
    static_assert(kAlloc <= 227 * 1024, "shared memory per CTA exceeds 227 KB");
    static_assert(S >= 4, "ring too shallow");
};

template <int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairLayout<FMT>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ GemmArgs a) {
    using L = PairLayout<FMT>;
    constexpr int S = L::S;
    constexpr int BNP = kPairTok;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Xs = smem + L::offX;
    uint8_t* As = smem + L::offA;
    uint8_t* Ps = smem + L::offP;
    uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + L::offBar);
    uint64_t* full_p = full_x + S;
    uint64_t* full_a = full_p + S;
    uint64_t* empty = full_a + S;
    uint64_t* acc_full = empty + S;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::offTmem);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::offAbort);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int ntiles = a.n_tiles * a.m_tiles;
    const int xs = a.x_steps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&full_p[s], 1);
            mbar_init(&full_a[s], 8);  // 4 dequant warps of each CTA
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);  // 4 epilogue warps of each CTA
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer (both CTAs): this CTA's X half and weight block
        if (lane == 0) {
            // test-only fault: CTA 0 of pair 0 withholds the copies of its second K step
            const int withheld = blockIdx.x == 0 && injected_fault(a.err) == kFaultGemmWithholdCopy ? 1 : -1;
            int g = 0;
            bool ok = true;
            for (int t = pair; t < ntiles && ok; t += npairs) {
                const int nt = t / a.m_tiles, mt = t % a.m_tiles;
                const int blk = nt * 2 + (int)rank;
                const bool has_w = blk < a.n_blocks;
                const uint8_t* wsrc = a.q + (int64_t)blk * a.k_steps * L::kP;
                for (int kx = 0; kx < xs; ++kx, ++g) {
                    const int s = g % S;
                    if (g >= S && !mbar_wait(&empty[s], ((g / S) & 1) ^ 1, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    if (g == withheld) continue;
                    mbar_expect_tx(&full_x[s], L::kX);
                    tma_load_2d(Xs + s * L::kX, &tmX, &full_x[s], kx * BK, mt * BNP + (int)rank * (BNP / 2));
                    mbar_expect_tx(&full_p[s], has_w ? L::kP : 0);
                    const int kw = kx < a.k_steps ? kx : kx - a.k_steps;
                    if (has_w) bulk_load(Ps + s * L::kP, wsrc + (int64_t)kw * L::kP, L::kP, &full_p[s]);
                }
            }
            // copies in flight land before the CTA can exit
            const uint64_t deadline = globaltimer() + wait_limit_ns(a.err);
            for (int j = (g > S ? g - S : 0); j < g; ++j) {
                if (j == withheld) continue;
                mbar_wait_until(&full_p[j % S], (j / S) & 1, deadline);
                mbar_wait_until(&full_x[j % S], (j / S) & 1, deadline);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (CTA 0)
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_bf16<256, BNP>();
            int g = 0, lt = 0;
            bool ok = true;
            for (int t = pair; t < ntiles && ok; t += npairs, ++lt) {
                const int buf = lt & 1;
                if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * BNP);
                for (int kx = 0; kx < xs; ++kx, ++g) {
                    const int s = g % S;
                    if (!mbar_wait(&full_a[s], (g / S) & 1, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(As + s * L::kA);
                    const uint32_t b_base = smem_u32(Xs + s * L::kX);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_bf16_pair(d, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), idesc,
                                       (kx > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_pair(&empty[s], 0x3);
                }
                if (ok) umma_commit_pair(&acc_full[buf], 0x3);
            }
            // every MMA issued above completes before the pair's TMEM and shared memory go away
            asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(mma_done))
                         : "memory");
            mbar_wait_until(mma_done, 0, globaltimer() + wait_limit_ns(a.err));
        }
    } else if (warp < 6) {
        // ---------------- dequantize (both CTAs, thread = weight row of this CTA's block)
        const int row = (warp - 2) * 32 + lane;
        int g = 0;
        bool ok = true;
        for (int t = pair; t < ntiles && ok; t += npairs) {
            for (int kx = 0; kx < xs; ++kx, ++g) {
                const int s = g % S;
                // outcomes are made warp-uniform: the step ends in a warp-collective arrival
                if (!__all_sync(0xffffffffu, mbar_wait(&full_p[s], (g / S) & 1, abort_flag, a.err))) {
                    ok = false;
                    break;
                }
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
                // the arrival below also certifies this CTA's X half of the step
                if (!__all_sync(0xffffffffu, mbar_wait(&full_x[s], (g / S) & 1, abort_flag, a.err))) {
                    ok = false;
                    break;
                }
                __syncwarp();  // orders every lane's writes before lane 0's arrival
                if (lane == 0) {
                    if (leader)
                        mbar_arrive(&full_a[s]);
                    else
                        mbar_arrive_cluster(mapa_shared(smem_u32(&full_a[s]), 0));
                }
            }
        }
    } else {
        // ---------------- epilogue (both CTAs: this CTA's 128 rows x 256 tokens)
        const int q4 = warp & 3;
        int lt = 0;
        for (int t = pair; t < ntiles; t += npairs, ++lt) {
            const int buf = lt & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&acc_full[buf], (lt >> 1) & 1, abort_flag, a.err);
            if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
            tc_fence_after();
            const int nt = t / a.m_tiles, mt = t % a.m_tiles;
            const int64_t row0 = (int64_t)nt * 256 + rank * 128;
            const int64_t grow = row0 + q4 * 32 + lane;
            const int m0 = mt * BNP;
            const bool row_ok = grow < a.N;
            // a tile inside the matrix stores without per-element bounds checks
            const bool full = row0 + 128 <= a.N && (int64_t)m0 + BNP <= a.M;
            const float sc = row_ok ? __ldg(a.scales + grow) : 0.f;
            float* ycol = a.y + grow;
            const uint32_t taddr = tmem + (uint32_t)(buf * BNP) + ((uint32_t)(q4 * 32) << 16);
            float rs_next = 0.f;
            if constexpr (FMT == BRAMHA_FMT_LOG4) rs_next = m0 + lane < a.M ? __ldg(a.rowsum + m0 + lane) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BNP; c0 += 32) {
                const float rs = rs_next;
                if constexpr (FMT == BRAMHA_FMT_LOG4) {
                    const int tl = m0 + c0 + 32 + lane;
                    if (c0 + 32 < BNP) rs_next = tl < a.M ? __ldg(a.rowsum + tl) : 0.f;
                }
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                float o[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    o[j] = __uint_as_float(v[j]);
                    if constexpr (FMT == BRAMHA_FMT_LOG4) o[j] = fmaf(o[j], 32768.0f, -__shfl_sync(0xffffffffu, rs, j));
                    o[j] *= sc;
                }
                float* yc = ycol + (int64_t)(m0 + c0) * a.ldy;
                if (full) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) yc[(int64_t)j * a.ldy] = o[j];
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (row_ok && m0 + c0 + j < a.M) yc[(int64_t)j * a.ldy] = o[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader)
                    mbar_arrive(&acc_empty[buf]);
                else
                    mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[buf]), 0));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the pair's remote arrivals and MMA reads of both CTAs are over
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, L::kTmemCols);
    }
}

// ---- activation preparation ------------------------------------------------
// bf16 copy with a TMA-friendly pitch kp (whole K steps) and per-token sums of
// exactly the values the MMA sees.  From f32 the activation is split
// x = hi + lo (hi = bf16(x), lo = bf16(x - hi)); hi fills columns [0, kp) and
// lo columns [kp, 2 kp) of the copy, so one pass over 2 kp reproduces x to ~2^-16.
// With ROWS (f32 only), lo goes to row M + r of a [2M][kp] copy instead.
// One block per token row, of prep_threads(M, K) threads: 1024 when a few long
// rows would leave the GPU idle (a batched GEMV), about 8 columns per thread when
// hundreds of rows fill it (a 2048 x 896 prefill lost ~5 us to 1024-thread
// blocks).  The row sum is reduced in a fixed order for a given block size, so
// results are reproducible for a given (M, K).
constexpr int kPrepThreads = 1024;
inline unsigned prep_threads(int64_t M, int64_t K) {
    if (M < 256) return kPrepThreads;
    const int64_t t = ((K + 7) / 8 + 31) / 32 * 32;
    return (unsigned)(t < 32 ? 32 : t > kPrepThreads ? kPrepThreads : t);
}
template <bool FROM_F32, bool ROWS = false>
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const void* __restrict__ x, int64_t ldx, int M, int K,
                                                            int64_t kp, __nv_bfloat16* __restrict__ xc,
                                                            float* __restrict__ rs) {
    __shared__ float part[kPrepThreads / 32][2];
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ldc = FROM_F32 && !ROWS ? 2 * kp : kp;
    const int64_t lo_off = ROWS ? (int64_t)M * kp : kp;
    float sh = 0.f, sl = 0.f;
#pragma unroll 4
    for (int k = threadIdx.x; k < (int)kp; k += blockDim.x) {
        float h = 0.f, l = 0.f;
        if (k < K) {
            if constexpr (FROM_F32) {
                const float v = static_cast<const float*>(x)[(int64_t)row * ldx + k];
                h = __bfloat162float(__float2bfloat16_rn(v));
                l = __bfloat162float(__float2bfloat16_rn(v - h));
            } else {
                h = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[(int64_t)row * ldx + k]);
            }
        }
        if (xc) {
            xc[(int64_t)row * ldc + k] = __float2bfloat16_rn(h);
            if constexpr (FROM_F32) xc[(int64_t)row * ldc + lo_off + k] = __float2bfloat16_rn(l);
        }
        sh += h;
        sl += l;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sh += __shfl_xor_sync(0xffffffffu, sh, o);
        sl += __shfl_xor_sync(0xffffffffu, sl, o);
    }
    if (lane == 0) {
        part[warp][0] = sh;
        part[warp][1] = sl;
    }
    __syncthreads();
    if (threadIdx.x == 0 && rs) {
        float a = 0.f, b = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
            a += part[w][0];
            b += part[w][1];
        }
        rs[row] = a + b;
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


// Per-device caches: SM count, and whether a kernel's shared-memory limit has
// been raised on that device (cudaFuncSetAttribute is per device).
int sm_count(int dev) {
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

template <int FMT, int BN>
cudaError_t launch_tiles(const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    using L = Layout<FMT, BN>;
    static std::atomic<uint64_t> attr_set{0};
    auto kern = gemm_kernel<FMT, BN>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit, std::memory_order_release);
    }
    const int64_t ntiles = (int64_t)g.n_tiles * g.m_tiles * g.ksplit;
    const int grid = (int)(ntiles < sm_count(dev) ? ntiles : sm_count(dev));
    kern<<<grid, kThreads, L::kAlloc, st>>>(tmX, g);
    return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_fmt(int bn, const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    switch (bn) {
        case 256: return launch_tiles<FMT, 256>(tmX, g, st);
        case 128: return launch_tiles<FMT, 128>(tmX, g, st);
        case 64: return launch_tiles<FMT, 64>(tmX, g, st);
        default: return launch_tiles<FMT, 32>(tmX, g, st);
    }
}

// Pairs of CTAs that can be resident at once (cached per device and format).
template <int FMT>
int max_pairs(int dev) {
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return sm_count(dev) / 2;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)sm_count(dev));
        cfg.blockDim = dim3(PairLayout<FMT>::kThreads);
        cfg.dynamicSmemBytes = PairLayout<FMT>::kAlloc;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<FMT>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sm_count(dev) / 2;
        }
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

template <int FMT>
cudaError_t launch_pair(const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    using L = PairLayout<FMT>;
    static std::atomic<uint64_t> attr_set{0};
    auto kern = gemm_pair_kernel<FMT>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit, std::memory_order_release);
    }
    const int64_t ntiles = (int64_t)g.n_tiles * g.m_tiles;
    const int pairs = (int)(ntiles < max_pairs<FMT>(dev) ? ntiles : max_pairs<FMT>(dev));
    kern<<<2 * pairs, L::kThreads, L::kAlloc, st>>>(tmX, g);
    return cudaGetLastError();
}

}  // namespace

// Tokens per tile for M tokens.
int gemm_tile_n(int64_t M) { return M >= 256 ? 256 : M > 64 ? 128 : M > 32 ? 64 : 32; }

namespace {
// X tensor map over a bf16 [M][cols] matrix with row pitch xld elements.
cudaError_t make_x_map(CUtensorMap* m, const void* xg, int64_t cols, int64_t M, int64_t xld, int bn) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(xld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(xg), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The SM-pair kernel takes GEMMs with at least four rounds of pair tiles on
// the GPU (lm_head-sized); with fewer, the single-CTA kernel's smaller tiles
// balance the SMs better.
bool use_pair(int64_t M, int64_t N, int sms) {
    const int64_t tiles = ((N + 2 * BM - 1) / (2 * BM)) * ((M + kPairTok - 1) / kPairTok);
    return M > 128 && N > BM && tiles >= 4 * (sms / 2);
}

cudaError_t run_gemm(int fmt, int bn, const CUtensorMap& tmX, const GemmArgs& g, cudaStream_t st) {
    if (bn == 0) {  // SM-pair kernel
        switch (fmt) {
            case BRAMHA_FMT_LOG4: return launch_pair<BRAMHA_FMT_LOG4>(tmX, g, st);
            case BRAMHA_FMT_W4ZP8: return launch_pair<BRAMHA_FMT_W4ZP8>(tmX, g, st);
            case BRAMHA_FMT_W8: return launch_pair<BRAMHA_FMT_W8>(tmX, g, st);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (fmt) {
        case BRAMHA_FMT_LOG4: return launch_fmt<BRAMHA_FMT_LOG4>(bn, tmX, g, st);
        case BRAMHA_FMT_W4ZP8: return launch_fmt<BRAMHA_FMT_W4ZP8>(bn, tmX, g, st);
        case BRAMHA_FMT_W8: return launch_fmt<BRAMHA_FMT_W8>(bn, tmX, g, st);
        default: return cudaErrorInvalidValue;
    }
}

// Fills the tile counts and steps of a GEMM over K packed columns.
cudaError_t gemm_args(GemmArgs* g, const uint8_t* q, const float* scales, const float* rowsum, float* y,
                      int64_t ldy, int64_t M, int64_t N, int64_t K, bool split, int bn, int* err) {
    // bn == 0 selects the SM-pair tiles: 256 weight rows x kPairTok tokens
    const int64_t k_steps = (K + BK - 1) / BK;
    const int64_t rows = bn == 0 ? 2 * BM : BM, toks = bn == 0 ? kPairTok : bn;
    const int64_t n_tiles = (N + rows - 1) / rows, m_tiles = (M + toks - 1) / toks;
    if (n_tiles * m_tiles > INT_MAX || 2 * k_steps > INT_MAX) return cudaErrorInvalidValue;
    g->q = q;
    g->scales = scales;
    g->rowsum = rowsum;
    g->y = y;
    g->ldy = ldy;
    g->M = (int)M;
    g->N = (int)N;
    g->k_steps = (int)k_steps;
    g->x_steps = (int)(split ? 2 * k_steps : k_steps);
    g->n_tiles = (int)n_tiles;
    g->n_blocks = (int)((N + BM - 1) / BM);
    g->m_tiles = (int)m_tiles;
    g->err = err;
    g->tiles = nullptr;
    g->ntiles_dev = nullptr;
    g->lo_row = 0;
    g->ksplit = 1;
    g->ks_steps = g->x_steps;
    g->ws = nullptr;
    g->tickets = nullptr;
    return cudaSuccess;
}

// K split of a single-CTA GEMM whose (weight block, token block) tiles do not
// fill the GPU: ranges of at least 4 K steps, as many as bring the tile count
// to about one per SM, within the workspace and ticket arrays.
void plan_ksplit(GemmArgs* g, int bn, int sms, float* ws, int64_t ws_floats, int* tickets, int64_t n_tickets) {
    const int64_t nm = (int64_t)g->n_tiles * g->m_tiles;
    if (!ws || !tickets || nm >= sms || 4 * nm > n_tickets) return;
    const int ntok = g->lo_row ? bn / 2 : bn;
    int ks = (int)(sms / nm);
    if (ks > g->x_steps / 4) ks = g->x_steps / 4;
    while (ks > 1 && (int64_t)ks * nm * BM * ntok > ws_floats) --ks;
    if (ks <= 1) return;
    const int steps = (g->x_steps + ks - 1) / ks;
    g->ksplit = (g->x_steps + steps - 1) / steps;  // no empty range
    g->ks_steps = steps;
    g->ws = ws;
    g->tickets = tickets;
}
}  // namespace

// y[M][ldy] = dequant(W)[N][K] applied to x[M][ldx] (bf16, or f32 split into
// bf16 hi + lo).  K is the number of columns the packed rows hold.
// f32 with M <= 128 tokens: the hi and lo parts are the two halves of the
// MMA's N (each weight block loaded and dequantized once); larger M: side by
// side along K.  GEMMs with fewer tiles than SMs are K-split through the
// caller's workspace (ws / tickets; NULL = no split).
// Scratch (bf16 copy, per-token sums) comes from the stream-ordered pool.
cudaError_t launch_gemm_tcgen05_multi(int fmt, int n, const GemmOut* outs, int64_t K, const void* x, int x_is_f32,
                                      int64_t ldx, int64_t M, int* err, float* ws, int64_t ws_floats, int* tickets,
                                      int64_t n_tickets, cudaStream_t st) {
    if (M <= 0 || n <= 0) return cudaSuccess;
    if (M > 0x7fffffff || K > 0x7fffffff || K <= 0) return cudaErrorInvalidValue;
    for (int i = 0; i < n; ++i)
        if (outs[i].N > 0x7fffffff || (reinterpret_cast<uintptr_t>(outs[i].q) & 15) != 0) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    const int64_t kp = (K + BK - 1) / BK * BK;  // copy pitch per half: whole K steps
    const bool nsplit = x_is_f32 && M <= 128;    // hi | lo as the halves of N
    const bool need_copy = x_is_f32 || (ldx % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0;
    const bool log4 = fmt == BRAMHA_FMT_LOG4;
    const int64_t cols = x_is_f32 && !nsplit ? 2 * kp : kp;  // columns of the bf16 copy
    const int64_t crow = nsplit ? 2 * M : M;                  // rows of the bf16 copy
    size_t copy_bytes = need_copy ? (size_t)crow * cols * sizeof(__nv_bfloat16) : 0;
    const size_t bytes = copy_bytes + (log4 ? (size_t)M * sizeof(float) : 0);
    uint8_t* scratch = nullptr;
    cudaError_t e = bytes ? cudaMallocAsync(reinterpret_cast<void**>(&scratch), bytes, st) : cudaSuccess;
    if (e != cudaSuccess) return e;
    __nv_bfloat16* xc = need_copy ? reinterpret_cast<__nv_bfloat16*>(scratch) : nullptr;
    float* rs = log4 ? reinterpret_cast<float*>(scratch + copy_bytes) : nullptr;
    if (need_copy || log4) {  // once for every weight that shares x
        const unsigned blocks = (unsigned)M;
        if (nsplit)
            prep_kernel<true, true><<<blocks, prep_threads(M, K), 0, st>>>(x, ldx, (int)M, (int)K, kp, xc, rs);
        else if (x_is_f32)
            prep_kernel<true><<<blocks, prep_threads(M, K), 0, st>>>(x, ldx, (int)M, (int)K, kp, xc, rs);
        else
            prep_kernel<false><<<blocks, prep_threads(M, K), 0, st>>>(x, ldx, (int)M, (int)K, need_copy ? kp : K, xc, rs);
        e = cudaGetLastError();
    }
    int dev = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
        const int64_t N = outs[i].N;
        if (N <= 0) continue;
        // N split: 2 x (32, 64 or 128) MMA columns (a 16-token half would not fill
        // the epilogue's 32-column chunks)
        const int bn =
            nsplit ? (M <= 32 ? 64 : M <= 64 ? 128 : 256) : use_pair(M, N, sm_count(dev)) ? 0 : gemm_tile_n(M);
        // X rows per TMA box: a pair's CTA loads half a tile; an N-split tile loads hi and lo halves
        const int box = bn == 0 ? kPairTok / 2 : nsplit ? bn / 2 : bn;
        GemmArgs g;
        CUtensorMap tmX;
        e = gemm_args(&g, outs[i].q, outs[i].scales, rs, outs[i].y, outs[i].ldy, M, N, K, x_is_f32 != 0 && !nsplit, bn,
                      err);
        if (e == cudaSuccess && nsplit) {
            g.lo_row = (int)M;
            g.m_tiles = 1;
        }
        // (bf16 prefill keeps one range per tile: its results stay those of the
        // allocation-free entry point, which has no workspace)
        if (e == cudaSuccess && bn != 0 && x_is_f32)
            plan_ksplit(&g, bn, sm_count(dev), ws, ws_floats, tickets, n_tickets);
        if (e == cudaSuccess)
            e = need_copy ? make_x_map(&tmX, xc, cols, crow, cols, box) : make_x_map(&tmX, x, K, M, ldx, box);
        if (e == cudaSuccess) e = run_gemm(fmt, bn, tmX, g, st);
    }
    if (scratch) {
        cudaError_t e2 = cudaFreeAsync(scratch, st);
        if (e == cudaSuccess) e = e2;
    }
    return e;
}

cudaError_t launch_gemm_tcgen05(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N, int64_t K,
                                const void* x, int x_is_f32, int64_t ldx, int64_t M, float* y, int64_t ldy, int* err,
                                float* ws, int64_t ws_floats, int* tickets, int64_t n_tickets, cudaStream_t st) {
    (void)ldq;
    if (N <= 0) return cudaSuccess;
    const GemmOut o = {q, scales, N, y, ldy};
    return launch_gemm_tcgen05_multi(fmt, 1, &o, K, x, x_is_f32, ldx, M, err, ws, ws_floats, tickets, n_tickets, st);
}

// Grouped GEMM for MoE experts: the tiles of a device-side table (built by the
// routing kernel, moe.cu), each a 128-row block of the group-stacked weight
// against up to kGemmGroupTok token rows of x.  x is f32 [M][ldx] (split into
// bf16 hi + lo, so results are within ~2^-16 of fp32), y [M][ldy]; N_group
// is the row count of one group (rows past it are not stored); max_tiles
// bounds the table (sizes the grid).  Scratch from the stream-ordered pool.
cudaError_t launch_gemm_tcgen05_grouped(int fmt, const uint8_t* q, const float* scales, int64_t N_group, int64_t K,
                                        const float* x, int64_t ldx, int64_t M, float* y, int64_t ldy,
                                        const int4* tiles, const int* ntiles_dev, int64_t max_tiles, int* err,
                                        cudaStream_t st) {
    if (M <= 0 || N_group <= 0 || max_tiles <= 0) return cudaSuccess;
    if (M > 0x7fffffff || N_group > 0x7fffffff || K > 0x7fffffff || K <= 0 || max_tiles > 0x7fffffff)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(q) & 15) != 0) return cudaErrorInvalidValue;
    if (fmt != BRAMHA_FMT_LOG4 && fmt != BRAMHA_FMT_W4ZP8 && fmt != BRAMHA_FMT_W8) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    const int64_t kp = (K + BK - 1) / BK * BK;
    const bool log4 = fmt == BRAMHA_FMT_LOG4;
    const size_t copy_bytes = (size_t)2 * M * kp * sizeof(__nv_bfloat16);  // hi rows, then lo rows
    const size_t bytes = copy_bytes + (log4 ? (size_t)M * sizeof(float) : 0);
    uint8_t* scratch = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), bytes, st);
    if (e != cudaSuccess) return e;
    __nv_bfloat16* xc = reinterpret_cast<__nv_bfloat16*>(scratch);
    float* rs = log4 ? reinterpret_cast<float*>(scratch + copy_bytes) : nullptr;
    prep_kernel<true, true><<<(unsigned)M, prep_threads(M, K), 0, st>>>(x, ldx, (int)M, (int)K, kp, xc, rs);
    e = cudaGetLastError();
    GemmArgs g;
    CUtensorMap tmX;
    constexpr int bn = 2 * kGemmGroupTok;  // MMA N: the tile's hi and lo rows
    if (e == cudaSuccess) e = gemm_args(&g, q, scales, rs, y, ldy, M, N_group, K, false, bn, err);
    if (e == cudaSuccess) {
        g.tiles = tiles;
        g.ntiles_dev = ntiles_dev;
        g.n_tiles = (int)max_tiles;  // with a table, only the grid size reads these
        g.m_tiles = 1;
        g.lo_row = (int)M;
        e = make_x_map(&tmX, xc, kp, 2 * M, kp, kGemmGroupTok);
    }
    if (e == cudaSuccess) e = run_gemm(fmt, bn, tmX, g, st);
    cudaError_t e2 = cudaFreeAsync(scratch, st);
    return e == cudaSuccess ? e2 : e;
}

cudaError_t launch_gemm_tcgen05_bf16_noalloc(int fmt, const uint8_t* q, int64_t ldq, const float* scales, int64_t N,
                                             int64_t K, const void* x, int64_t ldx, int64_t M, float* y,
                                             int64_t ldy, int* err, float* rowsum_scratch, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || K <= 0) return cudaErrorInvalidValue;
    if ((ldx % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(q) & 15) != 0) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaSuccess;
    float* rs = nullptr;
    if (fmt == BRAMHA_FMT_LOG4) {
        if (!rowsum_scratch) return cudaErrorInvalidValue;
        rs = rowsum_scratch;
        // every one of the M sums is written here before the GEMM reads it
        prep_kernel<false><<<(unsigned)M, prep_threads(M, K), 0, st>>>(x, ldx, (int)M, (int)K, K, nullptr, rs);
        e = cudaGetLastError();
    }
    int dev = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    const int bn = use_pair(M, N, sm_count(dev)) ? 0 : gemm_tile_n(M);
    GemmArgs g;
    CUtensorMap tmX;
    if (e == cudaSuccess) e = gemm_args(&g, q, scales, rs, y, ldy, M, N, K, false, bn, err);
    if (e == cudaSuccess) e = make_x_map(&tmX, x, K, M, ldx, bn == 0 ? kPairTok / 2 : bn);
    if (e == cudaSuccess) e = run_gemm(fmt, bn, tmX, g, st);
    return e;
}

}  // namespace bramha
