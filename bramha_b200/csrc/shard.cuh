#pragma once
// shard.cuh -- device side of the column-shard group (ShardArgs, common.cuh):
// the bounded wait on the ranks' arrival counters and a CTA's arrival.  Plain
// loads, stores and reductions on peer memory (IPC mappings over NVLink); no
// multicast of any kind.
#include <cstdint>

#include "common.cuh"
#include "tc_common.cuh"

namespace bramha {
namespace {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_add_sys(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

// Waits until every rank's arrivals here have reached what this rank expects
// (all CTAs of every sharded launch before the running one); bounded by the
// context's wait limit: records BRAMHA_ERR_TIMEOUT and returns false when it
// runs out.
__device__ bool shard_wait(const ShardArgs& s, int* err) {
    const uint64_t t0 = globaltimer();
    const uint64_t limit = wait_limit_ns(err);
    for (int r = 0; r < s.world; ++r) {
        const unsigned want = *reinterpret_cast<volatile unsigned*>(s.expected + r);
        while ((int)(ld_acquire_sys(s.arrive + r) - want) < 0) {
            if (globaltimer() - t0 > limit) {
                atomicCAS(err, 0, (int)BRAMHA_ERR_TIMEOUT);
                return false;
            }
            __nanosleep(32);
        }
    }
    return true;
}

// Thread 0 of a CTA whose stores are done (every storing thread passed a CTA
// barrier after its stores): one system-scope fence makes them visible, then
// the CTA arrives in every rank's arena (unless a failure was recorded, so the
// other ranks' waits run out rather than read incomplete rows).  The launch's
// last CTA advances `expected` by every rank's grid for the next launch.
__device__ void shard_arrive(const ShardArgs& s, int* err) {
    fence_sc_sys();
    if (*reinterpret_cast<volatile int*>(err) == 0)
        for (int r = 0; r < s.world; ++r) red_add_sys(s.peer_arrive[r] + s.rank, 1u);
    const unsigned t = atomicAdd(s.done, 1u);
    if (t == gridDim.x - 1) {
        *s.done = 0;
        for (int r = 0; r < s.world; ++r) s.expected[r] += (unsigned)s.grid_of[r];
    }
}

}  // namespace
}  // namespace bramha
