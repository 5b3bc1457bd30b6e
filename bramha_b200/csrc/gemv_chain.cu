// gemv_chain.cu -- a chain of dependent quantized GEMVs in ONE persistent,
// cooperative launch (bramha_cuda_gemv_program_*).
//
// The reference's decode loop calls `matvec_mul_into` (src/inference/
// cpu_engine.rs:1307-1444) back to back, each GEMV reading what the previous
// step wrote (fused_qkv_mul_into, o_proj, the MLP, lm_head; :2873-2976).  One
// launch per GEMV pays the launch, the prologue (barriers, TMEM, activation
// staging) and the drained pipeline at its end every time -- about 7 us per
// launch on B200, more than the weight stream of most of a 7B decode step's
// linears.  Here one CTA per SM runs the whole chain:
//   * the weight ring, the TMEM A stages and the double-buffered accumulators
//     keep their counters across ops, so the bulk-copy producers stream op
//     j+1's weights (and the dequant warps decode them) while op j finishes;
//   * op j+1 reads its activations only after every CTA has finished op j (a
//     per-op counter in global memory, bounded wait), so an op may read the
//     previous op's output, exactly as consecutive launches would;
//   * the epilogue warps (and two helpers) build op j+1's 8-bit activation
//     terms as soon as that counter completes; the MMA issuers wait for them.
// Each op has its own K-split plan (the one a single launch would use).
// Per-op work of a CTA: the tiles ci, ci + cps, ... of its split's K range.
// Results: the int formats equal the per-op launches bit for bit; log4 is
// within fp32 rounding of them (the four MMA accumulators group a tile's
// slots by their position in the whole chain, and sum(x) is reduced in
// another order).  Every wait is bounded (the context's wait limit).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "gemv_tc.cuh"
#include "tc_common.cuh"

namespace bramha {

// One op of a chain program (device memory, written by the host).
struct ChainOp {
    const uint8_t* q[kMaxSegments];  // tile-major weights
    const float* scales[kMaxSegments];
    float* y[kMaxSegments];          // [B][ldy]
    int64_t ldy[kMaxSegments];
    int N[kMaxSegments];
    int tile_begin[kMaxSegments];
    const float* x;                  // [B][ldx]
    const float* x_up;               // non-null: the activation is silu(x) * x_up
    int64_t ldx;
    int nseg, ntiles, K, ksteps;
    int ksplit, steps_per_split, ctas_per_split;
    int pad;
};

namespace {

// Trace stamps per op and CTA (epilogue warp 0): 0 op reached, 1 every CTA
// finished the previous op, 2 this CTA's MMAs of it are done (B area free),
// 3 activations loaded, 4 activation terms built, 5 last accumulator ready,
// 6 outputs stored, 7 completion published.
constexpr int kTraceStamps = 8;
constexpr int kActWarps = 6;                 // warps 6, 7 and the epilogue warps 24-27
constexpr int kActT = kActWarps * 32;        // 192 threads
constexpr int kMaxG = 3;                     // 8-column groups per act thread (<= 4608 columns)
static_assert(kMaxG * 8 * kActT >= 4608, "an act thread's groups cover the longest K range of a split");

struct ChainParams {
    const ChainOp* ops;
    int nops;
    const int* slots_total;  // [gridDim.x] weight slots each CTA streams over the chain
    unsigned* done;          // [nops] CTAs that finished op j; [nops] CTAs that finished the chain
    float* ws;               // K-split partials (ops run one after the other: shared)
    int* tickets;            // K-split tickets (4 per tile; back to zero after each op)
    int* err;
    // optional trace, [nops][gridDim.x][kTraceStamps] %globaltimer stamps per op
    // and CTA (kTraceStamps, below)
    unsigned long long* trace;
    // L2 lookahead: each producer requests its slot pairs this many of its own
    // pairs ahead of its copies (HBM -> L2), so the weight stream keeps going
    // while an op waits for the previous one (0 = off)
    int pf_ahead;
};

struct alignas(1024) ChSmem {
    uint8_t w[kSW][kSlotBytes];
    uint8_t x[kXBytes];
    uint64_t w_full[kSD], w_empty[kSD];
    uint64_t a_full[12], a_empty[12];
    uint64_t acc_full[2], d_empty[2], mma_done;
    uint64_t act_red, b_ready, b_free;
    float amax_part[kActWarps][8], sx_part[kActWarps][8];
    uint32_t tmem;
    int abort_flag;
    int epi_cnt;
};

// This CTA's part of an op.
struct Part {
    int ci, cps, step0, nsteps, nslots, ntile, ksteps;
};
template <int FMT>
__device__ __forceinline__ Part op_part(const ChainOp* o) {
    Part r;
    const int ksplit = o->ksplit, cps = o->ctas_per_split, spp = o->steps_per_split;
    r.cps = cps;
    r.ksteps = o->ksteps;
    const int b = blockIdx.x;
    if (b >= ksplit * cps) {
        r.ci = 0;
        r.step0 = 0;
        r.nsteps = 0;
        r.nslots = 0;
        r.ntile = 0;
        return r;
    }
    const int split = b / cps;
    r.ci = b - split * cps;
    r.step0 = split * spp;
    r.nsteps = min(spp, r.ksteps - r.step0);
    r.nslots = (r.nsteps + F<FMT>::kStepsPerSlot - 1) / F<FMT>::kStepsPerSlot;
    r.ntile = (o->ntiles - 1 - r.ci) / cps + 1;  // ci < ntiles (host)
    return r;
}

__device__ __forceinline__ int op_seg(const ChainOp* o, int tile) {
    int si = 0;
    for (int i = 1; i < o->nseg; ++i)
        if (tile >= o->tile_begin[i]) si = i;
    return si;
}

// The producers' walk over the CTA's weight slots of the whole chain.
struct Cur {
    int op, i, j;                // op, tile (of this CTA's tiles in the op), slot in the tile
    int nslots, ntile, nsteps;
    const uint8_t* base;         // the tile's first block of the CTA's K range
};

template <int FMT>
__device__ void cur_base(const ChainParams& p, Cur& c) {
    const ChainOp* o = p.ops + c.op;
    const Part pt = op_part<FMT>(o);
    const int tile = pt.ci + c.i * pt.cps;
    const int si = op_seg(o, tile);
    c.base = o->q[si] + ((int64_t)(tile - o->tile_begin[si]) * pt.ksteps + pt.step0) * F<FMT>::kBlock;
}
// Moves to the first op >= op in which this CTA has tiles (op = nops: done).
template <int FMT>
__device__ void cur_op(const ChainParams& p, Cur& c, int op) {
    for (; op < p.nops; ++op) {
        const Part pt = op_part<FMT>(p.ops + op);
        if (pt.ntile > 0) {
            c.nslots = pt.nslots;
            c.ntile = pt.ntile;
            c.nsteps = pt.nsteps;
            break;
        }
    }
    c.op = op;
    c.i = 0;
    if (op < p.nops) cur_base<FMT>(p, c);
}
template <int FMT>
__device__ void cur_advance(const ChainParams& p, Cur& c, int n) {
    c.j += n;
    while (c.op < p.nops && c.j >= c.nslots) {
        c.j -= c.nslots;
        if (++c.i >= c.ntile) {
            cur_op<FMT>(p, c, c.op + 1);
        } else {
            cur_base<FMT>(p, c);
        }
    }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* q) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
    return v;
}

// Lane 0 waits (bounded) until `count` CTAs have finished an op.
__device__ bool wait_count(const unsigned* c, unsigned count, volatile int* abort_flag, int* err) {
    if (ld_acquire_gpu(c) >= count) return true;
    const uint64_t t0 = globaltimer(), limit = wait_limit_ns(err);
    for (;;) {
        __nanosleep(64);
        if (ld_acquire_gpu(c) >= count) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > limit) {
            *abort_flag = 1;
            atomicCAS(err, 0, (int)BRAMHA_ERR_TIMEOUT);
            return false;
        }
    }
}


// An op's fields the act / epilogue warps use, held in registers (loaded
// before the wait for the previous op, so they are not on the critical path).
struct Meta {
    const float* x;
    const float* x_up;
    int64_t ldx;
    int K, ksplit, nseg;
    Part pt;
};
template <int FMT>
__device__ __forceinline__ void load_meta(const ChainOp* o, Meta& m) {
    m.x = o->x;
    m.x_up = o->x_up;
    m.ldx = o->ldx;
    m.K = o->K;
    m.ksplit = o->ksplit;
    m.nseg = o->nseg;
    m.pt = op_part<FMT>(o);
}

// The output side of one of the CTA's tiles of an op, for one epilogue lane:
// destination, row, scale.  Loaded a tile ahead (the first tile before the
// wait for the previous op), so its dependent global loads are never on the
// critical path.
struct TileMeta {
    float* y;
    int64_t ldy;
    int nrows, grow;
    float sc;
};
__device__ __forceinline__ void tile_meta(const ChainOp* o, const Part& pt, int nseg, int i, int row, TileMeta& t) {
    const int tile = pt.ci + i * pt.cps;
    int si = 0;
    for (int q = 1; q < nseg; ++q)
        if (tile >= o->tile_begin[q]) si = q;
    t.grow = (tile - o->tile_begin[si]) * TM + row;
    t.nrows = o->N[si];
    t.y = o->y[si];
    t.ldy = o->ldy[si];
    const float* scp = o->scales[si];
    t.sc = t.grow < t.nrows ? __ldg(scp + t.grow) : 0.f;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* a, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_release_gpu(unsigned* a, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

template <int FMT, int B>
__global__ void __launch_bounds__(kThreads, 1) chain_gemv_kernel(const __grid_constant__ ChainParams p) {
    using Fm = F<FMT>;
    constexpr int N = NB<FMT, B>::N;
    constexpr int kXSlot = NB<FMT, B>::kXSlot;
    constexpr int kACol = NB<FMT, B>::kDCols;  // A stages after the accumulators
    constexpr int kSA = NB<FMT, B>::kSA;
    constexpr int T = Fm::kTerms;
    constexpr bool kHold = B <= 2;  // act threads keep their activations in registers between passes
    static_assert(kSA % kGroups == 0 && kSA % kNI == 0 && kSA <= 12, "an A stage must always have the same users");
    extern __shared__ uint8_t smem_raw[];
    ChSmem& S = *reinterpret_cast<ChSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* abort_flag = &S.abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned G = gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSD; ++s) {
            mbar_init(&S.w_full[s], 1);
            mbar_init(&S.w_empty[s], Fm::kDeq ? 8 : 2);
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
        mbar_init(&S.act_red, kActWarps);
        mbar_init(&S.b_ready, kActWarps);
        mbar_init(&S.b_free, kNI);
        S.abort_flag = 0;
        S.epi_cnt = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&S.tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;

    if (warp == 0 || warp == kProdWarp1) {
        // ---------------- bulk-copy producer `pid`: slot pairs d = pid, pid + 2, ... of the whole chain
        if (lane == 0) {
            const int pid = warp == 0 ? 0 : 1;
            Cur cur;
            cur.j = 0;
            cur_op<FMT>(p, cur, 0);
            cur_advance<FMT>(p, cur, 2 * pid);
            // test-only fault: producer 0 of CTA 0 withholds its fourth pair's copy
            const int withheld =
                pid == 0 && blockIdx.x == 0 && injected_fault(p.err) == kFaultGemvWithholdCopy ? 6 : -1;
            int d = pid;
            // L2 prefetch front: pair pd of this producer, at cursor pc
            Cur pc = cur;
            int pd = d;
            auto prefetch_to = [&](int upto) {
                for (; pc.op < p.nops && pd <= upto; pd += kNP) {
                    const uint32_t b0 = (uint32_t)(min(Fm::kStepsPerSlot, pc.nsteps - pc.j * Fm::kStepsPerSlot) * Fm::kBlock);
                    const uint8_t* s0 = pc.base + (int64_t)pc.j * Fm::kStepsPerSlot * Fm::kBlock;
                    Cur c1 = pc;
                    cur_advance<FMT>(p, c1, 1);
                    if (c1.op < p.nops) {
                        const uint32_t b1 =
                            (uint32_t)(min(Fm::kStepsPerSlot, c1.nsteps - c1.j * Fm::kStepsPerSlot) * Fm::kBlock);
                        const uint8_t* s1 = c1.base + (int64_t)c1.j * Fm::kStepsPerSlot * Fm::kBlock;
                        if (s1 == s0 + b0) {
                            prefetch_l2(s0, b0 + b1);
                        } else {
                            prefetch_l2(s0, b0);
                            prefetch_l2(s1, b1);
                        }
                    } else {
                        prefetch_l2(s0, b0);
                    }
                    cur_advance<FMT>(p, pc, 2 * kNP);
                }
            };
            // the first kSD pairs go straight to shared memory; the front starts past them
            if (p.pf_ahead > 0) {
                for (int i = 0; i < kSD / kNP && pc.op < p.nops; ++i, pd += kNP) cur_advance<FMT>(p, pc, 2 * kNP);
                prefetch_to(pid + kSD + (p.pf_ahead - 1) * kNP);
            }
            for (; cur.op < p.nops; d += kNP) {
                if (p.pf_ahead > 0) prefetch_to(d + kSD + (p.pf_ahead - 1) * kNP);
                if (!mbar_wait(&S.w_empty[d % kSD], ((d / kSD) & 1) ^ 1, abort_flag, p.err)) break;
                if (d == withheld) {
                    cur_advance<FMT>(p, cur, 2 * kNP);
                    continue;
                }
                const int st = (2 * d) % kSW;
                const uint32_t b0 = (uint32_t)(min(Fm::kStepsPerSlot, cur.nsteps - cur.j * Fm::kStepsPerSlot) * Fm::kBlock);
                const uint8_t* s0 = cur.base + (int64_t)cur.j * Fm::kStepsPerSlot * Fm::kBlock;
                Cur c1 = cur;
                cur_advance<FMT>(p, c1, 1);
                uint32_t b1 = 0;
                const uint8_t* s1 = nullptr;
                if (c1.op < p.nops) {
                    b1 = (uint32_t)(min(Fm::kStepsPerSlot, c1.nsteps - c1.j * Fm::kStepsPerSlot) * Fm::kBlock);
                    s1 = c1.base + (int64_t)c1.j * Fm::kStepsPerSlot * Fm::kBlock;
                }
                uint64_t* bar = &S.w_full[d % kSD];
                mbar_expect_tx(bar, b0 + b1);
                if (s1 && b0 == (uint32_t)kSlotBytes && s1 == s0 + kSlotBytes) {
                    bulk_load(&S.w[st][0], s0, b0 + b1, bar);
                } else {
                    bulk_load(&S.w[st][0], s0, b0, bar);
                    if (s1) bulk_load(&S.w[st + 1][0], s1, b1, bar);
                }
                cur_advance<FMT>(p, cur, 2 * kNP);
            }
            // every copy this producer issued lands before the CTA exits
            const uint64_t deadline = globaltimer() + wait_limit_ns(p.err);
            for (int j = pid; j < d; j += kNP)
                if (j != withheld && j + kSD >= d && !mbar_wait_until(&S.w_full[j % kSD], (j / kSD) & 1, deadline))
                    break;
        }
    } else if (warp >= kIssWarp0 && warp < kIssWarp0 + kNI) {
        // ---------------- MMA issuer `me`: slots g with g % kNI == me, into accumulator `me`
        if (lane == 0) {
            const int me = warp - kIssWarp0;
            constexpr uint32_t idesc = idesc8<FMT, N>();
            const uint32_t xbase = smem_u32(&S.x[0]);
            int g = 0, lt = 0;
            bool ok = true;
            for (int j = 0; j < p.nops && ok; ++j) {
                if (!mbar_wait(&S.b_ready, j & 1, abort_flag, p.err)) break;  // this op's B terms are built
                tc_fence_after();
                const Part pt = op_part<FMT>(p.ops + j);
                for (int i = 0; i < pt.ntile && ok; ++i, ++lt) {
                    const int buf = lt & 1;
                    if (lt >= 2 && !mbar_wait(&S.d_empty[buf], ((lt >> 1) - 1) & 1, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dcol = tmem + (me * 2 + buf) * N;
                    const int g0 = g;
                    bool acc = false;
                    for (int r = (me - g0 % kNI + kNI) % kNI; r < pt.nslots; r += kNI) {
                        const int gg = g0 + r;
                        if constexpr (Fm::kDeq) {
                            const int sa = gg % kSA;
                            if (!mbar_wait(&S.a_full[sa], (gg / kSA) & 1, abort_flag, p.err)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t xt = xbase + r * kXSlot;
#pragma unroll
                            for (int kk = 0; kk < Fm::kMmaPerSlot; ++kk)
                                mma8<FMT>(dcol, tmem + kACol + sa * 32 + kk * 8, 0, desc_sw128(xt + kk * 32), idesc,
                                          (acc || kk > 0) ? 1u : 0u);
                            umma_commit(&S.a_empty[sa]);
                        } else {
                            const int st = gg % kSW, sd = (gg >> 1) % kSD;
                            if (!mbar_wait(&S.w_full[sd], ((gg >> 1) / kSD) & 1, abort_flag, p.err)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t xt = xbase + (r >> 1) * kXSlot + (r & 1) * 64;
                            const uint32_t wa = smem_u32(&S.w[st][0]);
#pragma unroll
                            for (int kk = 0; kk < Fm::kMmaPerSlot; ++kk)
                                mma8<FMT>(dcol, 0, desc_sw64(wa + kk * 32), desc_sw128(xt + kk * 32), idesc,
                                          (acc || kk > 0) ? 1u : 0u);
                            umma_commit(&S.w_empty[sd]);
                        }
                        acc = true;
                    }
                    if (ok) umma_commit(&S.acc_full[buf]);
                    g += pt.nslots;
                }
                if (ok) umma_commit(&S.b_free);  // arrives once this issuer's MMAs of op j are complete
            }
            umma_commit(&S.mma_done);
            mbar_wait_until(&S.mma_done, 0, globaltimer() + wait_limit_ns(p.err));
        }
    } else if (warp >= kDeqWarp0 && warp < kEpiWarp0) {
        if constexpr (Fm::kDeq) {
            // ---------------- dequantize into TMEM (the chain's slots in order, op-agnostic)
            const int total = p.slots_total[blockIdx.x];
            const int q4 = warp & 3;
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
                for (int h = 0; h < 2; ++h) {
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
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.w_empty[sd]);
                if (pending >= 0) publish();
                if (g >= kSA && !warp_wait(&S.a_empty[sa], ((g / kSA) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();
                tmem_st32(tmem + lane_base + kACol + sa * 32, v);
                pending = sa;
            }
            if (pending >= 0) publish();
        }
    } else {
        // ---------------- warps 6, 7 and 24-27: each op's activation terms; 24-27 also its epilogue
        const bool epi = warp >= kEpiWarp0;
        const int aw = epi ? warp - kEpiWarp0 + 2 : warp - 6;
        const int ta = aw * 32 + lane;
        const int q4 = warp & 3;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        int g = 0, lt = 0;
        bool ok = true;
        for (int j = 0; j < p.nops && ok; ++j) {
            const ChainOp* o = p.ops + j;
            Meta cm;
            load_meta<FMT>(o, cm);  // issued before the wait below, so it is not on the critical path
            TileMeta tm;
            if (epi && cm.pt.ntile > 0) tile_meta(o, cm.pt, cm.nseg, 0, q4 * 32 + lane, tm);
            unsigned long long* tr = p.trace ? p.trace + ((int64_t)j * gridDim.x + blockIdx.x) * kTraceStamps : nullptr;
            if (tr && warp == kEpiWarp0 && lane == 0) tr[0] = globaltimer();
            if (j > 0) {
                // every CTA has finished op j-1 (its output may be this op's input),
                // and this CTA's MMAs of op j-1 no longer read the B area
                int w = 1;
                if (lane == 0) w = wait_count(&p.done[j - 1], 4 * G, abort_flag, p.err);
                __syncwarp();
                if (!__shfl_sync(0xffffffffu, w, 0)) {
                    ok = false;
                    break;
                }
                if (tr && warp == kEpiWarp0 && lane == 0) tr[1] = globaltimer();
                if (!warp_wait(&S.b_free, (j - 1) & 1, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
            }
            const Part& pt = cm.pt;
            if (tr && warp == kEpiWarp0 && lane == 0) tr[2] = globaltimer();
            const int k0 = pt.step0 * kTileK, nk = pt.nsteps * kTileK;
            const int kv = max(0, min(nk, cm.K - k0));         // columns holding activations
            const int ngrp = ((pt.nsteps + 1) / 2) * 16;       // 8-column groups of whole 128-K atoms
            const float* xr0 = cm.x + k0;
            const float* ur0 = cm.x_up ? cm.x_up + k0 : nullptr;
            const int64_t ldx = cm.ldx;
            // pass 1: activations (SwiGLU formed as bramha_cuda_op_silu_mul rounds it), max|x|, sum(x)
            auto load8 = [&](int b, int c0, float (&v)[8]) {
                const float* xr = xr0 + (int64_t)b * ldx + c0;
                if (c0 + 8 <= kv) {
                    const float4 a = __ldcg(reinterpret_cast<const float4*>(xr));
                    const float4 c = __ldcg(reinterpret_cast<const float4*>(xr + 4));
                    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = c0 + e < kv ? __ldcg(xr + e) : 0.f;
                }
                if (ur0) {
                    const float* ur = ur0 + (int64_t)b * ldx + c0;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (c0 + e < kv) {
                            const float gv = v[e];
                            const float silu = __fmul_rn(gv, 1.0f / __fadd_rn(1.0f, expf(-gv)));
                            v[e] = __fmul_rn(silu, __ldcg(ur + e));
                        }
                }
            };
            float hv[kHold ? kMaxG : 1][kHold ? B : 1][8];
            float am[B], sm[B];
#pragma unroll
            for (int b = 0; b < B; ++b) {
                am[b] = 0.f;
                sm[b] = 0.f;
            }
            if (pt.ntile > 0) {
#pragma unroll
                for (int gi = 0; gi < kMaxG; ++gi) {
                    const int gidx = ta + gi * kActT;
                    if (gidx < ngrp) {
#pragma unroll
                        for (int b = 0; b < B; ++b) {
                            float v[8];
                            load8(b, gidx * 8, v);
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                am[b] = fmaxf(am[b], fabsf(v[e]));
                                sm[b] += v[e];
                                if constexpr (kHold) hv[gi][b][e] = v[e];
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < B; ++b) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    am[b] = fmaxf(am[b], __shfl_xor_sync(0xffffffffu, am[b], off));
                    sm[b] += __shfl_xor_sync(0xffffffffu, sm[b], off);
                }
            }
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    S.amax_part[aw][b] = am[b];
                    S.sx_part[aw][b] = sm[b];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.act_red);
            if (tr && warp == kEpiWarp0 && lane == 0) tr[3] = globaltimer();
            if (!warp_wait(&S.act_red, j & 1, abort_flag, p.err)) {
                ok = false;
                break;
            }
            float amax[B], sx[B], scl[B];
#pragma unroll
            for (int b = 0; b < B; ++b) {
                amax[b] = 0.f;
                sx[b] = 0.f;
                for (int w2 = 0; w2 < kActWarps; ++w2) {  // fixed order
                    amax[b] = fmaxf(amax[b], S.amax_part[w2][b]);
                    sx[b] += S.sx_part[w2][b];
                }
                scl[b] = act_scale<FMT>(amax[b]);
            }
            // pass 2: the 8-bit terms, K-major 128-byte-swizzled atoms (positions of
            // the 4-bit formats hold columns 0,4,1,5 | 2,6,3,7 of each 8)
            if (pt.ntile > 0) {
#pragma unroll
                for (int gi = 0; gi < kMaxG; ++gi) {
                    const int gidx = ta + gi * kActT;
                    if (gidx >= ngrp) continue;
                    const int c0 = gidx * 8, kb = c0 >> 7, pin = c0 & 127;
                    uint8_t* atom = &S.x[kb * kXSlot];
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        float v[8];
                        if constexpr (kHold) {
#pragma unroll
                            for (int e = 0; e < 8; ++e) v[e] = hv[gi][b][e];
                        } else {
                            load8(b, c0, v);
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) v[e] *= scl[b];
                        uint32_t w0[T], w1[T];
                        if constexpr (FMT == BRAMHA_FMT_W8) {
                            make_terms<FMT, T>(v[0], v[1], v[2], v[3], w0);
                            make_terms<FMT, T>(v[4], v[5], v[6], v[7], w1);
                        } else {
                            make_terms<FMT, T>(v[0], v[4], v[1], v[5], w0);
                            make_terms<FMT, T>(v[2], v[6], v[3], v[7], w1);
                        }
#pragma unroll
                        for (int t = 0; t < T; ++t) {
                            const int n = b * T + t;
                            uint8_t* rowp = atom + (n >> 3) * 1024 + (n & 7) * 128;
                            *reinterpret_cast<uint32_t*>(rowp + (((pin >> 4) ^ (n & 7)) << 4) + (pin & 15)) = w0[t];
                            const int p1 = pin + 4;
                            *reinterpret_cast<uint32_t*>(rowp + (((p1 >> 4) ^ (n & 7)) << 4) + (p1 & 15)) = w1[t];
                        }
                    }
                }
            }
            fence_async_smem();  // generic writes of the B terms -> the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.b_ready);
            if (tr && warp == kEpiWarp0 && lane == 0) tr[4] = globaltimer();
            if (!epi) continue;

            // ---------------- epilogue of op j's tiles, one warp per TMEM lane quarter
            constexpr int kCols = B * T;
            constexpr int kHalves = kCols > 16 ? 2 : 1;
            const int row = q4 * 32 + lane;
            const int split = pt.cps > 0 ? blockIdx.x / pt.cps : 0;
            for (int i = 0; i < pt.ntile; ++i, ++lt) {
                const int tile = pt.ci + i * pt.cps;
                const TileMeta cur = tm;
                if (i + 1 < pt.ntile) tile_meta(o, pt, cm.nseg, i + 1, row, tm);  // the next tile's, ahead
                const int grow = cur.grow, nrows = cur.nrows;
                float* y = cur.y;
                const int64_t ldy = cur.ldy;
                const float sc = cur.sc;
                const int buf = lt & 1;
                if (!warp_wait(&S.acc_full[buf], (lt >> 1) & 1, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (tr && warp == kEpiWarp0 && lane == 0 && i == pt.ntile - 1) tr[5] = globaltimer();
                const int g0 = g;
                g += pt.nslots;
                uint32_t d[16 * kHalves];
#pragma unroll
                for (int c = 0; c < 16 * kHalves; ++c) d[c] = 0;
#pragma unroll
                for (int me = 0; me < kNI; ++me) {
                    if ((me - g0 % kNI + kNI) % kNI >= pt.nslots) continue;
#pragma unroll
                    for (int h = 0; h < kHalves; ++h) {
                        uint32_t t[16];
                        tmem_ld16(tmem + lane_base + (me * 2 + buf) * N + h * 16, t);
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            if constexpr (FMT == BRAMHA_FMT_LOG4)
                                d[h * 16 + c] = __float_as_uint(__uint_as_float(d[h * 16 + c]) + __uint_as_float(t[c]));
                            else
                                d[h * 16 + c] += t[c];
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.d_empty[buf]);
                float res[B];
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    float acc = 0.f;
                    if constexpr (FMT == BRAMHA_FMT_LOG4) {
#pragma unroll
                        for (int t = T - 1; t >= 0; --t) acc = acc * 0.0625f + __uint_as_float(d[b * T + t]);
                    } else {
#pragma unroll
                        for (int t = T - 1; t >= 0; --t) acc = acc * 0.0078125f + (float)(int)d[b * T + t];
                    }
                    const float xq = acc / scl[b];
                    float dot;
                    if constexpr (FMT == BRAMHA_FMT_LOG4) dot = fmaf(xq, 16384.0f, -sx[b]);
                    else if constexpr (FMT == BRAMHA_FMT_W4ZP8) dot = fmaf(-8.0f, sx[b], xq);
                    else dot = xq;
                    res[b] = dot * sc;
                }
                const int ksplit = cm.ksplit;
                if (ksplit == 1) {
                    if (grow < nrows)
#pragma unroll
                        for (int b = 0; b < B; ++b) y[(int64_t)b * ldy + grow] = res[b];
                    continue;
                }
                // K split: this split's partial, then a ticket (acquire-release: the
                // last split sees every other split's partial)
                float* part = p.ws + (int64_t)tile * ksplit * B * TM;
                if (grow < nrows)
#pragma unroll
                    for (int b = 0; b < B; ++b) part[((int64_t)split * B + b) * TM + row] = res[b];
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atom_add_acq_rel_gpu(reinterpret_cast<unsigned*>(&p.tickets[tile * 4 + q4]), 1u) == (unsigned)(ksplit - 1);
                last = __shfl_sync(0xffffffffu, last, 0);
                __syncwarp();
                if (last) {
                    if (grow < nrows) {
                        constexpr int U = B >= 8 ? 4 : B >= 4 ? 8 : 16;
                        float acc[B];
#pragma unroll
                        for (int b = 0; b < B; ++b) acc[b] = 0.f;
                        for (int s0 = 0; s0 < ksplit; s0 += U) {
                            float v[U][B];
#pragma unroll
                            for (int u = 0; u < U; ++u)
#pragma unroll
                                for (int b = 0; b < B; ++b)
                                    v[u][b] = s0 + u < ksplit ? __ldcg(part + ((int64_t)(s0 + u) * B + b) * TM + row) : 0.f;
#pragma unroll
                            for (int u = 0; u < U; ++u)
                                if (s0 + u < ksplit)
#pragma unroll
                                    for (int b = 0; b < B; ++b) acc[b] += v[u][b];
                        }
#pragma unroll
                        for (int b = 0; b < B; ++b) y[(int64_t)b * ldy + grow] = acc[b];
                    }
                    if (lane == 0) p.tickets[tile * 4 + q4] = 0;  // ready for the next op
                }
            }
            if (!ok) break;
            // this warp is done with op j: its stores, then one release-add (the
            // op is done when all 4 epilogue warps of every CTA have added)
            __syncwarp();
            if (lane == 0) {
                if (tr && warp == kEpiWarp0) tr[6] = globaltimer();
                red_add_release_gpu(&p.done[j], 1u);
                if (tr && warp == kEpiWarp0) tr[7] = globaltimer();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0) {  // the last CTA out leaves every counter at zero for the next run
        __threadfence();
        if (atomicAdd(&p.done[p.nops], 1u) == G - 1) {
            for (int j = 0; j <= p.nops; ++j) p.done[j] = 0;
            __threadfence();
        }
    }
}


template <int FMT, int B>
cudaError_t launch_chain_fb(const ChainParams& p, int grid, cudaStream_t st) {
    auto kern = chain_gemv_kernel<FMT, B>;
    constexpr int smem = (int)sizeof(ChSmem) + 1024;
    static_assert(smem <= 227 * 1024, "shared memory per CTA exceeds 227 KB");
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (they wait on each other)
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int FMT, int B>
int chain_occupancy() {
    int n = 0;
    constexpr int smem = (int)sizeof(ChSmem) + 1024;
    if (cudaFuncSetAttribute(chain_gemv_kernel<FMT, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, chain_gemv_kernel<FMT, B>, kThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

template <int FMT>
cudaError_t launch_chain_f(int batch, const ChainParams& p, int grid, cudaStream_t st) {
    switch (batch) {
        case 1: return launch_chain_fb<FMT, 1>(p, grid, st);
        case 2: return launch_chain_fb<FMT, 2>(p, grid, st);
        case 3: return launch_chain_fb<FMT, 3>(p, grid, st);
        case 4: return launch_chain_fb<FMT, 4>(p, grid, st);
        case 5: return launch_chain_fb<FMT, 5>(p, grid, st);
        case 6: return launch_chain_fb<FMT, 6>(p, grid, st);
        case 7: return launch_chain_fb<FMT, 7>(p, grid, st);
        case 8: return launch_chain_fb<FMT, 8>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

struct ChainProgram {
    int fmt = 0, batch = 1, nops = 0, grid = 0;
    ChainOp* ops = nullptr;
    int* slots = nullptr;
    unsigned* done = nullptr;
    float* ws = nullptr;
    int* tickets = nullptr;
    unsigned long long* trace = nullptr;  // [nops][grid][kTraceStamps] when tracing is on
};

cudaError_t chain_program_create(int fmt, int batch, int nops, const GemvArgs* ops, int num_sms, int split_cost,
                                 float* ws, int64_t ws_floats, int* tickets, int n_tickets, ChainProgram** out) {
    *out = nullptr;
    if (!is_tiled(fmt) || batch < 1 || batch > kMaxGemvBatch || nops < 1 || num_sms < 1) return cudaErrorInvalidValue;
    const int occ = fmt == BRAMHA_FMT_LOG4 ? chain_occupancy<BRAMHA_FMT_LOG4, 1>()
                    : fmt == BRAMHA_FMT_W4ZP8 ? chain_occupancy<BRAMHA_FMT_W4ZP8, 1>()
                                              : chain_occupancy<BRAMHA_FMT_W8, 1>();
    if (occ < 1) return cudaErrorNotSupported;
    const int grid = num_sms;  // one CTA per SM
    std::vector<ChainOp> table((size_t)nops);
    std::vector<int> slots((size_t)grid, 0);
    const int steps_per_slot = fmt == BRAMHA_FMT_W8 ? 1 : 2;
    for (int j = 0; j < nops; ++j) {
        const GemvArgs& a = ops[j];
        ChainOp& o = table[(size_t)j];
        memset(&o, 0, sizeof o);
        int ntiles = 0;
        for (int i = 0; i < a.nseg; ++i) {
            const GemvSeg& sg = a.seg[i];
            if ((reinterpret_cast<uintptr_t>(sg.q) & 15) != 0 || sg.N <= 0) return cudaErrorInvalidValue;
            o.q[i] = sg.q;
            o.scales[i] = sg.scales;
            o.y[i] = sg.y;
            o.ldy[i] = sg.ldy;
            o.N[i] = sg.N;
            o.tile_begin[i] = ntiles;
            ntiles += (int)row_tiles(sg.N);
        }
        if (a.nseg < 1 || ntiles < 1 || a.K <= 0) return cudaErrorInvalidValue;
        o.x = a.x;
        o.x_up = a.x_up;
        o.ldx = a.ldx;
        o.nseg = a.nseg;
        o.ntiles = ntiles;
        o.K = a.K;
        o.ksteps = (int)k_steps(a.K);
        int max_ksplit = 1;
        if (ws && tickets && 4 * (int64_t)ntiles <= n_tickets)
            max_ksplit = (int)(ws_floats / ((int64_t)ntiles * batch * TM));
        if (!plan_gemv_tc(ntiles, o.ksteps, max_split_steps(fmt, batch), max_ksplit, grid, split_cost, &o.ksplit,
                          &o.steps_per_split, &o.ctas_per_split))
            return cudaErrorInvalidValue;
        for (int b = 0; b < o.ksplit * o.ctas_per_split && b < grid; ++b) {
            const int split = b / o.ctas_per_split, ci = b % o.ctas_per_split;
            const int nsteps = std::min(o.steps_per_split, o.ksteps - split * o.steps_per_split);
            const int ntile = (ntiles - 1 - ci) / o.ctas_per_split + 1;
            slots[(size_t)b] += ntile * ((nsteps + steps_per_slot - 1) / steps_per_slot);
        }
    }
    ChainProgram* prog = new (std::nothrow) ChainProgram();
    if (!prog) return cudaErrorMemoryAllocation;
    prog->fmt = fmt;
    prog->batch = batch;
    prog->nops = nops;
    prog->grid = grid;
    prog->ws = ws;
    prog->tickets = tickets;
    cudaError_t e = cudaMalloc(&prog->ops, sizeof(ChainOp) * (size_t)nops);
    if (e == cudaSuccess) e = cudaMalloc(&prog->slots, sizeof(int) * (size_t)grid);
    if (e == cudaSuccess) e = cudaMalloc(&prog->done, sizeof(unsigned) * (size_t)(nops + 1));
    if (e == cudaSuccess) e = cudaMemcpy(prog->ops, table.data(), sizeof(ChainOp) * (size_t)nops, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(prog->slots, slots.data(), sizeof(int) * (size_t)grid, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(prog->done, 0, sizeof(unsigned) * (size_t)(nops + 1));
    if (e != cudaSuccess) {
        chain_program_destroy(prog);
        return e;
    }
    *out = prog;
    return cudaSuccess;
}

cudaError_t chain_program_run(ChainProgram* prog, int* err, int64_t lookahead_bytes, cudaStream_t st) {
    ChainParams p;
    p.pf_ahead = (int)std::min<int64_t>(lookahead_bytes / (2 * kSlotBytes * kNP), 1 << 16);  // pairs per producer
    p.ops = prog->ops;
    p.nops = prog->nops;
    p.slots_total = prog->slots;
    p.done = prog->done;
    p.ws = prog->ws;
    p.tickets = prog->tickets;
    p.err = err;
    p.trace = prog->trace;
    switch (prog->fmt) {
        case BRAMHA_FMT_LOG4: return launch_chain_f<BRAMHA_FMT_LOG4>(prog->batch, p, prog->grid, st);
        case BRAMHA_FMT_W4ZP8: return launch_chain_f<BRAMHA_FMT_W4ZP8>(prog->batch, p, prog->grid, st);
        case BRAMHA_FMT_W8: return launch_chain_f<BRAMHA_FMT_W8>(prog->batch, p, prog->grid, st);
        default: return cudaErrorInvalidValue;
    }
}

void chain_program_destroy(ChainProgram* prog) {
    if (!prog) return;
    if (prog->ops) cudaFree(prog->ops);
    if (prog->slots) cudaFree(prog->slots);
    if (prog->done) cudaFree(prog->done);
    if (prog->trace) cudaFree(prog->trace);
    delete prog;
}

cudaError_t chain_program_trace(ChainProgram* prog, int on) {
    if (on && !prog->trace) {
        const size_t n = (size_t)prog->nops * prog->grid * kTraceStamps;
        cudaError_t e = cudaMalloc(&prog->trace, n * sizeof(unsigned long long));
        if (e == cudaSuccess) e = cudaMemset(prog->trace, 0, n * sizeof(unsigned long long));
        return e;
    }
    if (!on && prog->trace) {
        cudaDeviceSynchronize();
        cudaFree(prog->trace);
        prog->trace = nullptr;
    }
    return cudaSuccess;
}

cudaError_t chain_program_read_trace(ChainProgram* prog, unsigned long long* out, size_t n, int* grid) {
    *grid = prog->grid;
    if (!prog->trace) return cudaErrorInvalidValue;
    const size_t have = (size_t)prog->nops * prog->grid * kTraceStamps;
    return cudaMemcpy(out, prog->trace, (n < have ? n : have) * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
}

}  // namespace bramha
