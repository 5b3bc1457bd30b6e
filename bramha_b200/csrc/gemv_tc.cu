// gemv_tc.cu -- decode GEMV for the quantized formats (batch 1..8) on the
// tensor cores, with 8-bit operands.
//
// Same result as `matvec_mul_into` (src/inference/cpu_engine.rs:1307-1444) on
// int4 (quantize_to_int4, src/models/quantization.rs:41-83), int8
// (quantize_to_int8, :7-38) or log4 (dequantize_log4,
// spanda-engine/src/lib.rs:332-342) weights.
//
// A GEMV has N = batch, so its MMAs are tiny (M = 128, N = 16/32, K = 32):
// ~8 cycles of tensor work each, but one issuing thread waits ~55-68 cycles
// per tcgen05.mma (measured).  So four threads issue, each into its own
// accumulator (slot g goes to issuer g mod 4): ~17 cycles per MMA in
// aggregate (measured), several times what HBM can feed.  8-bit operands take
// K = 32 per MMA:
//   int8  (W8)    kind::i8: A = the int8 block exactly as stored (the repack
//                 writes it in the 64-byte-swizzle operand order), read by the
//                 MMA straight from the shared-memory ring: no dequantization.
//   int4  (W4ZP8) kind::i8: A = u8 q (0..15) in TMEM (one mask per 4 codes).
//   log4          kind::f8f6f4: A = e5m2 2^(c-14) in TMEM (exact; byte
//                 (c+1)*4: one mask + one multiply-add per 4 codes).
// The weights are exact in these types.  The activations become B columns of
// several 8-bit terms per batch row, scaled per row by a power of two s chosen
// from max|x| over the CTA's K range:
//   int8 terms: x*s = t1 + t2/128 + t3/16384 (abs. error <= 2^-22 max|x|),
//               integer accumulation, exact;
//   e4m3 terms: x*s = t1 + t2/16 + t3/256 + t4/4096 (rel. error ~2^-16),
//               fp32 accumulation.
// The epilogue adds the four issuers' accumulators (in issuer order), folds
// the terms, the zero points (int4 -8, log4 -1, with the row's sum(x)) and the
// row scale.
//
// Work: 128-row tiles of the tile-major weight (repack.cu) x a K range (a
// "split").  Persistent CTAs, one per SM, each walking the tiles of its split
// back to back.  With ksplit > 1 each split writes its partial tile result to
// a context-owned workspace and takes a ticket; the last split to arrive adds
// the partials in split order and writes y, so results do not depend on
// timing.  A ring slot is 8 KB: two 64-column blocks of a 4-bit tile (K = 128)
// or one int8 block (K = 64).
//   warps 0, 5   bulk copies into the 128 KB ring (16 slots of 8 KB, filled and
//                released in pairs: one barrier and, within a tile, one 16 KB
//                copy per pair; producer p takes pairs d = p, p+2, ...).  A
//                thread issuing 8 KB copies tops out near 4.9 TB/s, 16 KB
//                copies reach the HBM peak (measured).  Slots 0-11 are
//                requested during the prologue, right after the activation
//                loads; slots 12-15 hold the raw activations until the
//                prologue ends
//   warps 1-4    MMA issuers (lane 0)
//   warps 8-23   (4-bit) dequantize: four groups take slots g, g+4, ...; a
//                warp owns one TMEM lane quarter: 128 codes per row -> 32
//                words -> one tcgen05.st into an A stage
//   warps 24-27  epilogue (tcgen05.ld of the double-buffered accumulators)
//   prologue     warps 0-7 and 24-27 load the split's activations once
//                (staged raw), reduce max|x| and sum(x), and write the 8-bit
//                B terms (K-major, 128-byte swizzle, one 128-column atom per
//                128 K); meanwhile the dequant warps already decode the first
//                weights (they touch neither activations nor outputs).
// Launches are programmatically dependent (PDL): a CTA may start on an SM as
// soon as the previous launch's CTA there has exited, sets up its barriers,
// TMEM and first weight copies (weights are immutable), and waits for the
// previous launch to complete (griddepcontrol.wait) before it reads
// activations or writes outputs or the K-split workspace.
// Ring slots and A stages are multiples of 4 deep, so each one is always
// consumed by the same dequant group and the same issuer: a parity wait can
// never see a phase two generations old.  Every mbarrier wait is bounded
// (tc_common.cuh).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "gemv_tc.cuh"
#include "shard.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

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
    const float* x_up;     // non-null: the activation is silu(x) * x_up
    int* err;
    int nseg;
    int ntiles;
    int K;                 // columns held by the packed rows
    int ksteps;            // 64-column blocks per tile row
    int steps_per_split;
    int ctas_per_split;
    int ksplit;
    float* ws;             // [ntiles][ksplit][B][128] partials (ksplit > 1)
    int* tickets;          // [ntiles][4] arrivals per TMEM lane quarter, zero between launches
    int pf_ahead;          // slot pairs (even) prefetched into L2 ahead of the copies
    int pf_next_n;         // next launch's weight buffers (prefetched into L2 at our tail)
    const uint8_t* pf_next_ptr[kMaxSegments];
    int64_t pf_next_bytes[kMaxSegments];
    int64_t pf_next_total;
    int evict_first;       // weight copies marked first to be evicted from L2
    ShardArgs shard;       // column-shard group (shard.world > 1)
};

struct alignas(1024) TcSmem {
    uint8_t w[kSW][kSlotBytes];   // slots kPrologueSlots.. double as the activation staging area
    uint8_t x[kXBytes];
    uint64_t w_full[kSD], w_empty[kSD];  // per slot pair
    uint64_t a_full[12], a_empty[12];
    uint64_t acc_full[2], d_empty[2], mma_done;
    float amax[8], sx[8];
    float sx_part[kActThreads / 32][8];  // per-warp partial sums, added in warp order
    uint32_t tmem;
    int abort_flag;
};

__device__ __forceinline__ int seg_of(const TcGemvParams& p, int tile) {
    int si = 0;
    for (int i = 1; i < p.nseg; ++i)
        if (tile >= p.seg[i].tile_begin) si = i;
    return si;
}

template <int FMT, int B>
__global__ void __launch_bounds__(kThreads, 1) tc_gemv_kernel(const __grid_constant__ TcGemvParams p) {
    using Fm = F<FMT>;
    constexpr int N = NB<FMT, B>::N;
    constexpr int kXSlot = NB<FMT, B>::kXSlot;
    constexpr int kACol = NB<FMT, B>::kDCols;  // A stages after the accumulators
    constexpr int kSA = NB<FMT, B>::kSA;
    constexpr int T = Fm::kTerms;
    static_assert(kSA % kGroups == 0 && kSA % kNI == 0 && kSA <= 12, "an A stage must always have the same users");
    extern __shared__ uint8_t smem_raw[];
    TcSmem& S = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* abort_flag = &S.abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x / p.ctas_per_split;
    const int ci = blockIdx.x % p.ctas_per_split;
    const int step0 = split * p.steps_per_split;
    const int nsteps = min(p.steps_per_split, p.ksteps - step0);          // 64-column blocks per tile
    const int nslots = (nsteps + Fm::kStepsPerSlot - 1) / Fm::kStepsPerSlot;
    const int nkb = (nsteps + 1) >> 1;                                     // 128-K B atoms
    const int ntile_cta = (p.ntiles - 1 - ci) / p.ctas_per_split + 1;       // ci < ntiles (host)
    const int nunit_tiles = ntile_cta;
    const int total = ntile_cta * nslots;                                  // slots this CTA streams
    const int k0 = step0 * kTileK;                                         // first column of the split
    const int nk = nsteps * kTileK;                                        // columns of the split

    // source and size of this CTA's g-th slot
    // A producer walks its slots with a cursor (tile i, slot j in the tile,
    // the tile's first block of this split); the kernel-parameter segment
    // table is read only when the tile changes -- those reads are dependent
    // memory round trips, and per slot they capped a producer near 5 TB/s.
    struct Cursor {
        int i, j;
        const uint8_t* base;
    };
    auto tile_base = [&](int i) -> const uint8_t* {
        const int tile = ci + i * p.ctas_per_split;
        const TcSeg& sg = p.seg[seg_of(p, tile)];
        return sg.q + ((int64_t)(tile - sg.tile_begin) * p.ksteps + step0) * Fm::kBlock;
    };
    auto advance = [&](Cursor& c, int n) {
        c.j += n;
        if (c.j >= nslots) {
            do {
                c.j -= nslots;
                ++c.i;
            } while (c.j >= nslots);
            if (c.i < nunit_tiles) c.base = tile_base(c.i);
        }
    };
    // source ranges of slot pair d (slots 2d, 2d + 1; cursor c at slot 2d)
    auto pair_src = [&](int d, Cursor c, const uint8_t*& s0, uint32_t& b0, const uint8_t*& s1, uint32_t& b1) {
        const int g = 2 * d;
        b0 = (uint32_t)(min(Fm::kStepsPerSlot, nsteps - c.j * Fm::kStepsPerSlot) * Fm::kBlock);
        s0 = c.base + (int64_t)c.j * Fm::kStepsPerSlot * Fm::kBlock;
        b1 = 0;
        s1 = nullptr;
        if (g + 1 < total) {
            advance(c, 1);
            b1 = (uint32_t)(min(Fm::kStepsPerSlot, nsteps - c.j * Fm::kStepsPerSlot) * Fm::kBlock);
            s1 = c.base + (int64_t)c.j * Fm::kStepsPerSlot * Fm::kBlock;
        }
    };
    // copies of slot pair d into ring slots 2d % kSW, +1, completing on
    // w_full[d % kSD]; one copy when the pair is contiguous.  The weight lines
    // are read once: with p.evict_first they are marked first to be evicted
    // from L2, ahead of the lines prefetched for later copies.
    const uint64_t pol = policy_evict_first();
    auto issue_pair = [&](int d, Cursor c) {
        const int st = (2 * d) % kSW;
        const uint8_t *s0, *s1;
        uint32_t b0, b1;
        pair_src(d, c, s0, b0, s1, b1);
        uint64_t* bar = &S.w_full[d % kSD];
        mbar_expect_tx(bar, b0 + b1);
        auto copy = [&](void* dst, const uint8_t* src, uint32_t bytes) {
            if (p.evict_first)
                bulk_load_hint(dst, src, bytes, bar, pol);
            else
                bulk_load(dst, src, bytes, bar);
        };
        if (s1 && b0 == (uint32_t)kSlotBytes && s1 == s0 + kSlotBytes) {
            copy(&S.w[st][0], s0, b0 + b1);
        } else {
            copy(&S.w[st][0], s0, b0);
            if (s1) copy(&S.w[st + 1][0], s1, b1);
        }
    };
    // HBM -> L2 request of slot pair d, p.pf_ahead pairs before its copy
    auto prefetch_pair = [&](int d, Cursor c) {
        const uint8_t *s0, *s1;
        uint32_t b0, b1;
        pair_src(d, c, s0, b0, s1, b1);
        if (s1 == s0 + b0) {
            prefetch_l2(s0, b0 + b1);
        } else {
            prefetch_l2(s0, b0);
            if (s1) prefetch_l2(s1, b1);
        }
    };
    const int npairs = (total + 1) / 2;

    // the next launch may start its own set-up as our CTAs retire
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---------------- prologue: barriers, zeroed B area, the first weights requested
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSD; ++s) {
            mbar_init(&S.w_full[s], 1);
            mbar_init(&S.w_empty[s], Fm::kDeq ? 8 : 2);  // both slots' consumers
        }
        for (int s = 0; s < kSA; ++s) {
            mbar_init(&S.a_full[s], 4);
            mbar_init(&S.a_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.acc_full[i], kNI);
            mbar_init(&S.d_empty[i], 4);
        }
        mbar_init(&S.mma_done, kNI);
        for (int b = 0; b < 8; ++b) {
            S.amax[b] = 0.f;
            S.sx[b] = 0.f;
        }
        S.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&S.tmem, 512);
    {
        uint4* xz = reinterpret_cast<uint4*>(&S.x[0]);
        const int nz = nkb * kXSlot / 16;
        for (int i = threadIdx.x; i < nz; i += kThreads) xz[i] = make_uint4(0, 0, 0, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;
    const int first = min(kPrologueSlots / 2, npairs);  // slot pairs requested in the prologue
    float* stage = reinterpret_cast<float*>(&S.w[kPrologueSlots][0]);
    const bool producer = (warp == 0 || warp == kProdWarp1) && lane == 0;
    const int pid = warp == 0 ? 0 : 1;
    Cursor cur = {0, 0, nullptr};  // producer's cursor: slot 2 * (next pair of mine)
    Cursor pcur = {0, 0, nullptr};  // its L2 prefetch cursor, pair pd
    int pd = pid;
    // keeps the prefetch front p.pf_ahead pairs past pair d (pairs of this producer)
    auto prefetch_to = [&](int d) {
        for (; pd < npairs && pd <= d + p.pf_ahead; pd += kNP) {
            prefetch_pair(pd, pcur);
            advance(pcur, 2 * kNP);
        }
    };
    if (producer) {
        cur.base = tile_base(0);
        advance(cur, 2 * pid);
        pcur = cur;
        for (int d = pid; d < first; d += kNP) {
            issue_pair(d, cur);
            advance(cur, 2 * kNP);
        }
        // pairs issued above need no prefetch; start the front past them
        for (; pd < first; pd += kNP) advance(pcur, 2 * kNP);
        if (p.pf_ahead > 0) prefetch_to(first - kNP);
    }
    const bool act = warp < kDeqWarp0 || warp >= kEpiWarp0;       // activation warps
    const int ta = (warp < kDeqWarp0 ? warp : warp - kEpiWarp0 + kDeqWarp0) * 32 + lane;  // 0..383

    const bool sharded = p.shard.world > 1;
    if (act) {
        // activations, outputs and the K-split workspace belong to the stream order
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (sharded) {
            // every rank's rows of the previous sharded launch have landed here
            // (the activations may be that launch's output)
            if (ta == 0) shard_wait(p.shard, p.err);
            asm volatile("bar.sync 2, %0;" ::"n"(kActThreads) : "memory");
        }

        // ---------------- activations -> staging, max|x|, sum(x)
        // (a split whose rows do not fit the staging area reads them again from
        // global memory when it builds the terms, computing the same values)
        const int kv = min(nk, p.K - k0);
        // (at batch 1 and 2 every K range a plan gives fits: no second path)
        const bool staged = B <= 2 || B * nk <= kStageFloats;
        {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float* xr = p.x + (int64_t)b * p.ldx + k0;
                float v[kPerThread];
#pragma unroll
                for (int u = 0; u < kPerThread; ++u) {
                    const int k = ta + u * kActThreads;
                    // (written by other GPUs during this kernel when sharded: L2, not the read-only path)
                    v[u] = k < kv ? (sharded ? __ldcg(xr + k) : __ldg(xr + k)) : 0.f;
                }
                if (p.x_up) {  // SwiGLU: silu(g) * up, rounded as the separate silu_mul kernel rounds it
                    const float* ur = p.x_up + (int64_t)b * p.ldx + k0;
#pragma unroll
                    for (int u = 0; u < kPerThread; ++u) {
                        const int k = ta + u * kActThreads;
                        if (k < kv) {
                            const float g = v[u];
                            const float silu = __fmul_rn(g, 1.0f / __fadd_rn(1.0f, expf(-g)));
                            v[u] = __fmul_rn(silu, sharded ? __ldcg(ur + k) : __ldg(ur + k));
                        }
                    }
                }
                float am = 0.f, sm = 0.f;
#pragma unroll
                for (int u = 0; u < kPerThread; ++u) {
                    const int k = ta + u * kActThreads;
                    if (staged && k < nk) stage[b * nk + k] = v[u];
                    am = fmaxf(am, fabsf(v[u]));
                    sm += v[u];
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                    sm += __shfl_xor_sync(0xffffffffu, sm, o);
                }
                if (lane == 0) {
                    atomicMax(reinterpret_cast<int*>(&S.amax[b]), __float_as_int(am));  // am >= 0 (order-free)
                    S.sx_part[ta >> 5][b] = sm;
                }
            }
        }
        asm volatile("bar.sync 2, %0;" ::"n"(kActThreads) : "memory");
        if (ta < B) {  // sum(x) in a fixed order, so results do not depend on timing
            float s = 0.f;
            for (int w = 0; w < kActThreads / 32; ++w) s += S.sx_part[w][ta];
            S.sx[ta] = s;
        }

        // ---------------- B terms
        {
            const int bt = ta;
            float scl[B];
#pragma unroll
            for (int b = 0; b < B; ++b) scl[b] = act_scale<FMT>(S.amax[b]);
            const int npos4 = nkb * 32;  // 4-position groups per batch row
            for (int i = bt; i < B * npos4; i += kActThreads) {
                const int b = i / npos4, g4 = i - b * npos4;
                const int p0 = g4 * 4, kb = p0 >> 7, pin = p0 & 127;
                float s = scl[0];
#pragma unroll
                for (int bb = 1; bb < B; ++bb)
                    if (b == bb) s = scl[bb];
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int col = (kb << 7) + pos_to_col<FMT>(pin + e);
                    float a = 0.f;
                    if (staged) {
                        if (col < nk) a = stage[b * nk + col];
                    } else if (col < kv) {
                        const int64_t off = (int64_t)b * p.ldx + k0 + col;
                        a = sharded ? __ldcg(p.x + off) : __ldg(p.x + off);
                        if (p.x_up) {  // as in the first pass
                            const float silu = __fmul_rn(a, 1.0f / __fadd_rn(1.0f, expf(-a)));
                            a = __fmul_rn(silu, sharded ? __ldcg(p.x_up + off) : __ldg(p.x_up + off));
                        }
                    }
                    v[e] = a * s;
                }
                uint32_t word[T];
                make_terms<FMT, T>(v[0], v[1], v[2], v[3], word);
                uint8_t* atom = &S.x[kb * kXSlot];
#pragma unroll
                for (int j = 0; j < T; ++j) {
                    const int n = b * T + j;
                    *reinterpret_cast<uint32_t*>(atom + (n >> 3) * 1024 + (n & 7) * 128 + (((pin >> 4) ^ (n & 7)) << 4) +
                                                 (pin & 15)) = word[j];
                }
            }
        }
        // B terms: generic writes -> MMA reads; staging reads -> bulk copies into slots 12-15
        fence_async_smem();
        asm volatile("bar.sync 2, %0;" ::"n"(kActThreads) : "memory");
    }  // act

    if (warp == 0 || warp == kProdWarp1) {
        // ---------------- bulk-copy producer `pid`: slot pairs d = pid, pid + 2, ...
        if (lane == 0) {
            // test-only fault: producer 0 of CTA 0 withholds its first copy after the prologue
            const bool withhold = pid == 0 && blockIdx.x == 0 && injected_fault(p.err) == kFaultGemvWithholdCopy;
            int withheld = -1;
            bool ok = true;
            int d = first + ((pid - first % kNP + kNP) % kNP);  // first pair of mine not yet requested
            for (; d < npairs; d += kNP) {
                if (!mbar_wait(&S.w_empty[d % kSD], ((d / kSD) & 1) ^ 1, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
                if (withhold && withheld < 0)
                    withheld = d;
                else
                    issue_pair(d, cur);
                advance(cur, 2 * kNP);
                if (p.pf_ahead > 0) prefetch_to(d);
            }
            // the next launch of the chain: this producer's half of the CTA's
            // slice of its first pf_next_total bytes, HBM -> L2
            if (ok && p.pf_next_total > 0) {
                const int64_t per = (p.pf_next_total / gridDim.x + 4095) & ~(int64_t)4095;
                const int64_t half = (per / 2 + 4095) & ~(int64_t)4095;
                int64_t lo = (int64_t)blockIdx.x * per + pid * half;
                const int64_t hi = min(min((int64_t)blockIdx.x * per + per, lo + half), p.pf_next_total);
                int64_t base = 0;
                for (int r = 0; r < p.pf_next_n && lo < hi; ++r) {
                    const int64_t end = base + p.pf_next_bytes[r];
                    for (; lo < hi && lo < end;) {
                        const int64_t n = min(min(hi, end) - lo, (int64_t)65536);
                        prefetch_l2(p.pf_next_ptr[r] + (lo - base), (uint32_t)n);
                        lo += n;
                    }
                    base = end;
                }
            }
            // every copy this producer issued lands before the CTA exits
            const uint64_t deadline = globaltimer() + wait_limit_ns(p.err);
            for (int j = pid; j < d && j < npairs; j += kNP)
                if (j != withheld && j + kSD >= d && !mbar_wait_until(&S.w_full[j % kSD], (j / kSD) & 1, deadline))
                    break;
        }
    } else if (warp >= kIssWarp0 && warp < kIssWarp0 + kNI) {
        // ---------------- MMA issuer `me`: slots g with g % kNI == me, into accumulator `me`
        if (lane == 0) {
            const int me = warp - kIssWarp0;
            constexpr uint32_t idesc = idesc8<FMT, N>();
            const uint32_t xbase = smem_u32(&S.x[0]);
            bool ok = true;
            for (int i = 0; i < ntile_cta && ok; ++i) {
                const int buf = i & 1;
                if (i >= 2 && !mbar_wait(&S.d_empty[buf], ((i >> 1) - 1) & 1, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t dcol = tmem + (me * 2 + buf) * N;
                const int g0 = i * nslots;
                bool acc = false;
                for (int j = (me - g0 % kNI + kNI) % kNI; j < nslots; j += kNI) {
                    const int g = g0 + j;
                    if constexpr (Fm::kDeq) {
                        const int sa = g % kSA;
                        if (!mbar_wait(&S.a_full[sa], (g / kSA) & 1, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t xt = xbase + j * kXSlot;
#pragma unroll
                        for (int kk = 0; kk < Fm::kMmaPerSlot; ++kk)
                            mma8<FMT>(dcol, tmem + kACol + sa * 32 + kk * 8, 0, desc_sw128(xt + kk * 32), idesc,
                                      (acc || kk > 0) ? 1u : 0u);
                        umma_commit(&S.a_empty[sa]);
                    } else {
                        const int st = g % kSW, sd = (g >> 1) % kSD;
                        if (!mbar_wait(&S.w_full[sd], ((g >> 1) / kSD) & 1, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t xt = xbase + (j >> 1) * kXSlot + (j & 1) * 64;
                        const uint32_t wa = smem_u32(&S.w[st][0]);
#pragma unroll
                        for (int kk = 0; kk < Fm::kMmaPerSlot; ++kk)
                            mma8<FMT>(dcol, 0, desc_sw64(wa + kk * 32), desc_sw128(xt + kk * 32), idesc,
                                      (acc || kk > 0) ? 1u : 0u);
                        umma_commit(&S.w_empty[sd]);
                    }
                    acc = true;
                }
                if (ok) umma_commit(&S.acc_full[buf]);  // arrives at once when this issuer had no slot here
            }
            // all MMAs issued have completed before TMEM and the ring are released
            umma_commit(&S.mma_done);
            mbar_wait_until(&S.mma_done, 0, globaltimer() + wait_limit_ns(p.err));
        }
    } else if (warp >= kDeqWarp0 && warp < kEpiWarp0) {
        if constexpr (Fm::kDeq) {
            // ---------------- dequantize into TMEM
            // The wait for a slot's tcgen05.st is deferred until the group's
            // next slot is decoded (so the store latency overlaps work), unless
            // that slot has not landed yet.
            const int q4 = warp & 3;                         // TMEM lane quarter
            const int grp = (warp - kDeqWarp0) >> 2;
            const int row = q4 * 32 + lane;
            const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
            int pending = -1;
            auto publish = [&]() {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.a_full[pending]);
                pending = -1;
            };
            for (int g = grp; g < total; g += kGroups) {
                const int st = g % kSW, sd = (g >> 1) % kSD, sa = g % kSA;
                const uint32_t par = ((g >> 1) / kSD) & 1;
                if (pending >= 0 && !__all_sync(0xffffffffu, mbar_test(&S.w_full[sd], par))) publish();
                if (!warp_wait(&S.w_full[sd], par, abort_flag, p.err)) break;
                uint32_t v[32];
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // the slot's two 64-column blocks
                    // rows are 32 B apart: rows r and r+4 read their halves in
                    // opposite order, so each 8-lane phase of a 16-byte load hits
                    // 32 distinct banks
                    const uint8_t* sl = &S.w[st][h * Fm::kBlock + row * 32];
                    const int sw = (row >> 2) & 1;
                    const uint4 c0 = *reinterpret_cast<const uint4*>(sl + 16 * sw);
                    const uint4 c1 = *reinterpret_cast<const uint4*>(sl + 16 * (sw ^ 1));
                    const uint4 p0 = sw ? c1 : c0;
                    const uint4 p1 = sw ? c0 : c1;
                    const uint32_t wv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) dq_word8<FMT>(wv[i], v[16 * h + 2 * i], v[16 * h + 2 * i + 1]);
                }
                // the slot's bytes were read through the generic proxy; the next
                // bulk copy into it is an async-proxy write
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.w_empty[sd]);
                if (pending >= 0) publish();
                if (g >= kSA && !warp_wait(&S.a_empty[sa], ((g / kSA) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();  // the store follows the MMAs that read this stage
                tmem_st32(tmem + lane_base + kACol + sa * 32, v);
                pending = sa;
            }
            if (pending >= 0) publish();
        }
    } else if (warp >= kEpiWarp0) {
        // ---------------- epilogue, one warp per TMEM lane quarter
        const int q4 = warp & 3;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        constexpr int kCols = B * T;  // accumulator columns in use
        // output row `grow` of batch row b: this GPU's y, or (sharded) row
        // row0 + grow of every rank's copy of the full output
        auto store_y = [&](const TcSeg& sg, int si, int grow, int b, float v) {
            if (!sharded) {
                sg.y[(int64_t)b * sg.ldy + grow] = v;
                return;
            }
            const int64_t off = (int64_t)b * sg.ldy + p.shard.row0[si] + grow;
            for (int r = 0; r < p.shard.world; ++r) p.shard.peer_y[si][r][off] = v;
        };
        const int row = q4 * 32 + lane;
        // accumulator columns per TMEM load, issuers per wait (at most 32
        // registers of loads in flight)
        // (32 columns: two 16-column loads per issuer, a wait after each)
        constexpr int kNC = kCols <= 4 ? 4 : kCols <= 8 ? 8 : kCols <= 16 ? 16 : 32;
        constexpr int kLd = kNC == 32 ? 16 : kNC;  // columns per load
        constexpr int kPer = kNC <= 8 ? 4 : kNC == 16 ? 2 : 1;
        static_assert(kNC <= N && kNI % kPer == 0, "accumulator columns");
        bool ok = true;
        for (int i = 0; i < ntile_cta; ++i) {
            const int buf = i & 1;
            if (!warp_wait(&S.acc_full[buf], (i >> 1) & 1, abort_flag, p.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // add the accumulators of the issuers that had a slot in this tile, in
            // issuer order; the loads of kPer issuers are in flight before one wait
            const int g0 = i * nslots;
            uint32_t d[kNC];
#pragma unroll
            for (int c = 0; c < kNC; ++c) d[c] = 0;
#pragma unroll
            for (int m0 = 0; m0 < kNI; m0 += kPer) {
#pragma unroll
                for (int h = 0; h < kNC / kLd; ++h) {
                    uint32_t t[kPer][kLd];
#pragma unroll
                    for (int u = 0; u < kPer; ++u)
                        if ((m0 + u - g0 % kNI + kNI) % kNI < nslots)  // this issuer had a slot here
                            tmem_ld_nw<kLd>(tmem + lane_base + ((m0 + u) * 2 + buf) * N + h * kLd, t[u]);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < kPer; ++u) {
                        if ((m0 + u - g0 % kNI + kNI) % kNI >= nslots) continue;
#pragma unroll
                        for (int c = 0; c < kLd; ++c) {
                            if constexpr (FMT == BRAMHA_FMT_LOG4)
                                d[h * kLd + c] = __float_as_uint(__uint_as_float(d[h * kLd + c]) + __uint_as_float(t[u][c]));
                            else
                                d[h * kLd + c] += t[u][c];  // s32
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.d_empty[buf]);
            const int tile = ci + i * p.ctas_per_split;
            const int si = seg_of(p, tile);
            const TcSeg& sg = p.seg[si];
            const int grow = (tile - sg.tile_begin) * TM + row;
            float res[B];
            if (grow < sg.N) {
                const float sc = __ldg(sg.scales + grow);
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    float acc = 0.f;
                    if constexpr (FMT == BRAMHA_FMT_LOG4) {
#pragma unroll
                        for (int j = T - 1; j >= 0; --j) acc = acc * 0.0625f + __uint_as_float(d[b * T + j]);
                    } else {
#pragma unroll
                        for (int j = T - 1; j >= 0; --j) acc = acc * 0.0078125f + (float)(int)d[b * T + j];
                    }
                    // sum(a * x), a as held in A: acc / s with s = 2^k (normal, as is
                    // 1/s), so the product with 1/s (bits 254 - exponent) is exact
                    const float xq = acc * __int_as_float(0x7F000000 - __float_as_int(act_scale<FMT>(S.amax[b])));
                    const float sx = S.sx[b];
                    float dot;
                    if constexpr (FMT == BRAMHA_FMT_LOG4) dot = fmaf(xq, 16384.0f, -sx);  // sum((2^c - 1) x)
                    else if constexpr (FMT == BRAMHA_FMT_W4ZP8) dot = fmaf(-8.0f, sx, xq);  // sum((q - 8) x)
                    else dot = xq;
                    res[b] = dot * sc;
                }
            }
            if (p.ksplit == 1) {
                if (grow < sg.N)
#pragma unroll
                    for (int b = 0; b < B; ++b) store_y(sg, si, grow, b, res[b]);
                continue;
            }
            // K split: this split's partial of the tile; its ticket is taken
            // after the CTA's last tile (below), so the ticket round trips do not
            // hold up the accumulators of the next tiles
            float* part = p.ws + (int64_t)tile * p.ksplit * B * TM;
            if (grow < sg.N)
#pragma unroll
                for (int b = 0; b < B; ++b) part[((int64_t)split * B + b) * TM + row] = res[b];
        }
        if (ok && p.ksplit > 1) {
            // One fence for every partial of the CTA, then the tickets of all its
            // tiles at once (lane t takes tile c + t); the split that arrives last
            // at a tile adds all partials in split order.  Each warp (TMEM lane
            // quarter) has its own tickets, so no barrier across the epilogue
            // warps is needed (one that had given up a wait could not reach it).
            __threadfence();
            __syncwarp();
            for (int c = 0; c < ntile_cta; c += 32) {
                int last = 0;
                if (c + lane < ntile_cta) {
                    const int tile = ci + (c + lane) * p.ctas_per_split;
                    last = atomicAdd(&p.tickets[tile * 4 + q4], 1) == p.ksplit - 1;
                }
                unsigned mask = __ballot_sync(0xffffffffu, last);
                if (mask) __threadfence();
                while (mask) {
                    const int l = __ffs(mask) - 1;
                    mask &= mask - 1;
                    const int tile = ci + (c + l) * p.ctas_per_split;
                    const int si = seg_of(p, tile);
                    const TcSeg& sg = p.seg[si];
                    const int grow = (tile - sg.tile_begin) * TM + row;
                    const float* part = p.ws + (int64_t)tile * p.ksplit * B * TM;
                    if (grow < sg.N) {
                        // the partials are added in split order; up to 32 loads are in
                        // flight per lane (a load per split in turn would cost one L2
                        // round trip per split and batch row)
                        constexpr int U = B >= 8 ? 4 : B >= 4 ? 8 : 16;
                        float acc[B];
#pragma unroll
                        for (int b = 0; b < B; ++b) acc[b] = 0.f;
                        for (int s0 = 0; s0 < p.ksplit; s0 += U) {
                            float v[U][B];
#pragma unroll
                            for (int u = 0; u < U; ++u)
#pragma unroll
                                for (int b = 0; b < B; ++b)
                                    v[u][b] =
                                        s0 + u < p.ksplit ? __ldcg(part + ((int64_t)(s0 + u) * B + b) * TM + row) : 0.f;
#pragma unroll
                            for (int u = 0; u < U; ++u)
                                if (s0 + u < p.ksplit)
#pragma unroll
                                    for (int b = 0; b < B; ++b) acc[b] += v[u][b];
                        }
#pragma unroll
                        for (int b = 0; b < B; ++b) store_y(sg, si, grow, b, acc[b]);
                    }
                    if (lane == 0) p.tickets[tile * 4 + q4] = 0;  // ready for the next launch
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (sharded && threadIdx.x == 0) shard_arrive(p.shard, p.err);  // after the barrier: every store of the CTA is done
}

// A sharded launch in which this rank has no rows (publish = 1: one CTA that
// waits for the previous launch and arrives), or a wait for every rank's
// arrivals so far (publish = 0).
__global__ void shard_signal_kernel(const __grid_constant__ ShardArgs s, int* err, int publish) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x != 0) return;
    shard_wait(s, err);
    if (publish) shard_arrive(s, err);
}

template <int FMT, int B>
cudaError_t launch_b(TcGemvParams& p, int max_ksplit, int num_sms, int split_cost, cudaStream_t st) {
    auto kern = tc_gemv_kernel<FMT, B>;
    constexpr int smem = (int)sizeof(TcSmem) + 1024;
    static_assert(smem <= 227 * 1024, "shared memory per CTA exceeds 227 KB");
    if (!plan_gemv_tc(p.ntiles, p.ksteps, max_split_steps(FMT, B), max_ksplit, num_sms, split_cost, &p.ksplit,
                      &p.steps_per_split, &p.ctas_per_split))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)(p.ksplit * p.ctas_per_split));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, (const TcGemvParams)p);
}

}  // namespace

// Tensor-core GEMV over up to 8 fused quantized weights sharing x (batch 1..8).
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
    if (ntiles <= 0) return cudaErrorInvalidValue;
    p.x = a.x;
    p.ldx = a.ldx;
    p.x_up = a.x_up;
    p.err = a.err;
    p.nseg = a.nseg;
    p.ntiles = ntiles;
    p.K = a.K;
    p.ksteps = (int)k_steps(a.K);
    p.ws = a.split_ws;
    p.tickets = a.split_tickets;
    // splits need a workspace slot per (tile, split, batch row) and a ticket per tile
    int max_ksplit = 1;
    if (a.split_ws && a.split_tickets && 4 * (int64_t)ntiles <= a.split_tickets_n)
        max_ksplit = (int)(a.split_ws_floats / ((int64_t)ntiles * a.batch * TM));
    p.pf_ahead = a.pf_ahead < 0 ? 0 : (a.pf_ahead + 1) & ~1;
    p.pf_next_n = a.pf_next_n < 0 ? 0 : (a.pf_next_n > kMaxSegments ? kMaxSegments : a.pf_next_n);
    int64_t pf_avail = 0;
    for (int i = 0; i < p.pf_next_n; ++i) {
        if ((reinterpret_cast<uintptr_t>(a.pf_next_ptr[i]) & 15) != 0 || (a.pf_next_bytes[i] & 15) != 0)
            return cudaErrorInvalidValue;
        p.pf_next_ptr[i] = a.pf_next_ptr[i];
        p.pf_next_bytes[i] = a.pf_next_bytes[i];
        pf_avail += a.pf_next_bytes[i];
    }
    p.pf_next_total = (a.pf_next_total < pf_avail ? a.pf_next_total : pf_avail) & ~(int64_t)4095;
    p.shard = a.shard;
    p.evict_first = a.evict_first;
    if (p.shard.world > 1 && (p.shard.world > kMaxShardWorld || !p.shard.arrive || !p.shard.expected || !p.shard.done))
        return cudaErrorInvalidValue;
#define BRAMHA_TC_B(n)                                                                                   \
    case n:                                                                                              \
        return fmt == BRAMHA_FMT_LOG4    ? launch_b<BRAMHA_FMT_LOG4, n>(p, max_ksplit, num_sms, a.split_cost, st)      \
               : fmt == BRAMHA_FMT_W4ZP8 ? launch_b<BRAMHA_FMT_W4ZP8, n>(p, max_ksplit, num_sms, a.split_cost, st)     \
                                         : launch_b<BRAMHA_FMT_W8, n>(p, max_ksplit, num_sms, a.split_cost, st);
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

cudaError_t launch_shard_signal(const ShardArgs& s, int* err, int publish, cudaStream_t st) {
    if (s.world < 2 || s.world > kMaxShardWorld || !s.arrive || !s.expected || !s.done) return cudaErrorInvalidValue;
    shard_signal_kernel<<<1, 32, 0, st>>>(s, err, publish);
    return cudaGetLastError();
}

int gemv_tc_grid(int fmt, int batch, int ntiles, int K, int num_sms, int split_cost, int64_t split_ws_floats,
                 int split_tickets_n) {
    int max_ksplit = 1;
    if (split_ws_floats > 0 && 4 * (int64_t)ntiles <= split_tickets_n)
        max_ksplit = (int)(split_ws_floats / ((int64_t)ntiles * batch * TM));
    int ks = 1, spp = 1, cps = 1;
    if (!plan_gemv_tc(ntiles, (int)k_steps(K), max_split_steps(fmt, batch), max_ksplit, num_sms, split_cost, &ks, &spp,
                      &cps))
        return 0;
    return ks * cps;
}

}  // namespace bramha
