#pragma once
// gemv_tc.cuh -- pieces shared by the tensor-core GEMV kernels (gemv_tc.cu:
// one launch per GEMV; gemv_chain.cu: one persistent launch per chain of
// GEMVs): ring and TMEM geometry, 8-bit operand construction, UMMA
// descriptors, and the K-split plan.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

constexpr int TM = 128;                   // weight rows per tile (UMMA M, TMEM lanes)
constexpr int kSlotBytes = 8192;
constexpr int kSW = 16;                   // ring slots
constexpr int kPrologueSlots = 12;        // slots free during the prologue (the rest stage activations)
constexpr int kSD = kSW / 2;              // ring slot pairs (one barrier each)
constexpr int kNI = 4;                    // MMA issuers
constexpr int kGroups = 4;                // dequant groups (4 warps each)
constexpr int kIssWarp0 = 1;
constexpr int kNP = 2;                    // producers (warps 0 and 5)
constexpr int kProdWarp1 = 5;
constexpr int kDeqWarp0 = 8;
constexpr int kEpiWarp0 = kDeqWarp0 + 4 * kGroups;  // 24
constexpr int kThreads = (kEpiWarp0 + 4) * 32;      // 896
constexpr int kXBytes = 64 * 1024;        // B terms of one split
constexpr int kStageFloats = (kSW - kPrologueSlots) * kSlotBytes / 4;  // raw activations of one split
constexpr int kActThreads = 384;          // warps 0-7 and 24-27 stage the activations and build B
constexpr int kPerThread = 12;            // activation columns a thread loads per batch row
static_assert(kSW % kGroups == 0 && kSW % kNI == 0 && kSD % kNP == 0,
              "a ring slot must always have the same producer and consumer");
static_assert(kDeqWarp0 % 4 == 0 && kEpiWarp0 % 4 == 0, "TMEM lane quarters follow warp % 4");

// Per-format constants.
template <int FMT>
struct F {
    static constexpr bool kDeq = FMT != BRAMHA_FMT_W8;           // A through TMEM
    static constexpr int kStepsPerSlot = kDeq ? 2 : 1;           // 64-column blocks per slot
    static constexpr int kBlock = kTileRows * tile_slice_bytes(FMT);  // 4 KB / 8 KB
    static constexpr int kMmaPerSlot = kDeq ? 4 : 2;             // K = 32 each
    static constexpr int kTerms = FMT == BRAMHA_FMT_LOG4 ? 4 : 3;
};
template <int FMT, int B>
struct NB {
    static constexpr int N = (B * F<FMT>::kTerms <= 16) ? 16 : 32;  // MMA N (B columns)
    static constexpr int kXSlot = N * 128;                           // B bytes per 128 K
    static constexpr int kDCols = kNI * 2 * N;                       // accumulators: issuer x buffer
    static constexpr int kSA = (512 - kDCols) / 32 / 4 * 4;          // A stages (multiple of 4)
};
static_assert(NB<BRAMHA_FMT_LOG4, 1>::kSA == 12 && NB<BRAMHA_FMT_LOG4, 8>::kSA == 8, "TMEM plan");

// Every lane polls; the warp proceeds only if all lanes saw the phase (so the
// .sync.aligned TMEM instructions that follow stay warp-uniform on timeout).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
    const bool ok = mbar_wait(bar, parity, abort_flag, err);
    return __all_sync(0xffffffffu, ok);
}

// UMMA descriptor, K-major: 128-byte swizzle (B terms, 8-row groups 1 KB
// apart) or 64-byte swizzle (int8 weight blocks, 8-row groups 512 B apart).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46) |
           (4ull << 61);
}

// Instruction descriptors (M = 128): kind::i8 (D s32, A u8/s8, B s8) and
// kind::f8f6f4 (D f32, A e5m2, B e4m3).
template <int FMT, int N>
__device__ __forceinline__ constexpr uint32_t idesc8() {
    constexpr uint32_t mn = ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
    if constexpr (FMT == BRAMHA_FMT_LOG4) return (1u << 4) | (1u << 7) | (0u << 10) | mn;
    else if constexpr (FMT == BRAMHA_FMT_W4ZP8) return (2u << 4) | (0u << 7) | (1u << 10) | mn;
    else return (2u << 4) | (1u << 7) | (1u << 10) | mn;
}

template <int FMT>
__device__ __forceinline__ void mma8(uint32_t d, uint32_t a_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                     uint32_t acc) {
    if constexpr (FMT == BRAMHA_FMT_LOG4)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
            : "memory");
    else if constexpr (FMT == BRAMHA_FMT_W4ZP8)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
            : "memory");
}

// One device word (8 codes; repack.cu) -> two words of four 8-bit A values,
// K order (c0, c4, c1, c5) and (c2, c6, c3, c7).
template <int FMT>
__device__ __forceinline__ void dq_word8(uint32_t w, uint32_t& lo, uint32_t& hi) {
    constexpr uint32_t M = 0x0F0F0F0Fu;
    if constexpr (FMT == BRAMHA_FMT_LOG4) {  // e5m2 byte (c + 1) * 4 = 2^(c - 14)
        lo = (w & M) * 4u + 0x04040404u;
        hi = ((w >> 2) & 0x3C3C3C3Cu) + 0x04040404u;
    } else {                                 // u8 q
        lo = w & M;
        hi = (w >> 4) & M;
    }
}

// Position p of a 128-K B atom <-> column of the K range: 4-bit A words hold
// their codes in the order above, int8 A in natural order.
template <int FMT>
__device__ __forceinline__ int pos_to_col(int p) {
    if constexpr (FMT == BRAMHA_FMT_W8) return p;
    else {
        const int m = p & 7;
        return (p & ~7) + ((m >> 1) | ((m & 1) << 2));  // 0,4,1,5,2,6,3,7
    }
}

// Power-of-two activation scale of a batch row: max|x*s| < 128 (int8 terms)
// or < 256 (e4m3 terms).
template <int FMT>
__device__ __forceinline__ float act_scale(float amax) {
    if (!(amax > 0.f)) return 1.f;
    const int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127;  // amax in [2^e, 2^(e+1))
    float s = ldexpf(1.f, min((FMT == BRAMHA_FMT_LOG4 ? 7 : 6) - e, 126));
    if (FMT != BRAMHA_FMT_LOG4 && amax * s >= 127.5f) s *= 0.5f;
    return s;
}

// Four consecutive positions' scaled values -> T words of 8-bit terms.
template <int FMT, int T>
__device__ __forceinline__ void make_terms(float v0, float v1, float v2, float v3, uint32_t (&word)[T]) {
    if constexpr (FMT == BRAMHA_FMT_LOG4) {
        float2 a = make_float2(v0, v1), b = make_float2(v2, v3);
#pragma unroll
        for (int j = 0; j < T; ++j) {
            const __nv_fp8x2_storage_t ta = __nv_cvt_float2_to_fp8x2(a, __NV_SATFINITE, __NV_E4M3);
            const __nv_fp8x2_storage_t tb = __nv_cvt_float2_to_fp8x2(b, __NV_SATFINITE, __NV_E4M3);
            word[j] = (uint32_t)ta | ((uint32_t)tb << 16);
            if (j + 1 < T) {
                // residual * 16, exact: a - t is representable and the scaling is a power of two
                const float2 fa = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(ta, __NV_E4M3)));
                const float2 fb = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(tb, __NV_E4M3)));
                a = make_float2(fmaf(fa.x, -16.f, a.x * 16.f), fmaf(fa.y, -16.f, a.y * 16.f));
                b = make_float2(fmaf(fb.x, -16.f, b.x * 16.f), fmaf(fb.y, -16.f, b.y * 16.f));
            }
        }
    } else {
        float a[4] = {v0, v1, v2, v3};
#pragma unroll
        for (int j = 0; j < T; ++j) {
            uint32_t w = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = __float2int_rn(a[e]);
                w |= (uint32_t)(t & 0xFF) << (8 * e);
                a[e] = (a[e] - (float)t) * 128.f;
            }
            word[j] = w;
        }
    }
}

// Largest K range (64-column blocks) one CTA takes: its B terms fit the B
// area and its activation columns the threads' loads (rows that do not fit
// the staging area are read twice instead).
int max_split_steps(int fmt, int batch) {
    const int terms = fmt == BRAMHA_FMT_LOG4 ? 4 : 3;
    const int n = batch * terms <= 16 ? 16 : 32;
    int m = 2 * (kXBytes / (n * 128));
    const int by_threads = kPerThread * kActThreads / kTileK;
    if (by_threads < m) m = by_threads;
    return m;
}

// K split: the one that minimises the time of the busiest CTA (one CTA per
// SM), counted in 64-column blocks: its blocks, ~1 per tile for the
// epilogue, and for a split ~2 + ksplit/8 for the combine.  Splits start on
// even blocks so 4-bit slots stay whole.  False when no split fits.
bool plan_gemv_tc(int ntiles, int ksteps, int max_steps, int max_ksplit, int num_sms, int split_cost, int* ksplit_out,
                  int* steps_per_split_out, int* ctas_per_split_out) {
    int64_t best = INT64_MAX;
    int bk = 1, bspp = ksteps, bcps = 1;
    for (int ks = 1; ks <= ksteps && ks <= num_sms && ks <= max_ksplit; ++ks) {
        int spp = (ksteps + ks - 1) / ks;
        spp += spp & 1;
        if (spp > max_steps) continue;
        const int ks_eff = (ksteps + spp - 1) / spp;
        if (ks_eff != ks) continue;
        const int cps = ntiles < num_sms / ks ? ntiles : num_sms / ks;
        if (cps < 1) continue;
        const int64_t tpc = (ntiles + cps - 1) / cps;
        const int64_t cost = 8 * (tpc * (spp + 1)) + (ks > 1 ? split_cost + ks : 0);  // eighths of a block
        if (cost < best) {
            best = cost;
            bk = ks;
            bspp = spp;
            bcps = cps;
        }
    }
    *ksplit_out = bk;
    *steps_per_split_out = bspp;
    *ctas_per_split_out = bcps;
    return best != INT64_MAX;
}

}  // namespace
}  // namespace bramha
