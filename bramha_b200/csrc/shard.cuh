#pragma once
// shard.cuh -- device side of the column-shard group (ShardArgs, common.cuh):
// bounded waits on the epochs that ranks publish into each other's flag
// arrays, and the publication itself.  Plain loads and stores to peer memory
// (IPC mappings over NVLink); no multicast of any kind.
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
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until every rank has published at least epoch e here (bounded by the
// context's wait limit; records BRAMHA_ERR_TIMEOUT and returns false when it
// runs out).
__device__ bool shard_wait(const ShardArgs& s, unsigned e, int* err) {
    const uint64_t t0 = globaltimer();
    const uint64_t limit = wait_limit_ns(err);
    for (int r = 0; r < s.world; ++r) {
        while ((int)(ld_acquire_sys(s.flags + r) - e) < 0) {
            if (globaltimer() - t0 > limit) {
                atomicCAS(err, 0, (int)BRAMHA_ERR_TIMEOUT);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// Called by thread 0 of every CTA once the CTA's stores are done (after a
// system-scope fence by every storing thread and a CTA barrier): the last CTA
// of the launch advances this rank's epoch and, unless a failure was recorded,
// publishes it in every rank's flag array.
__device__ void shard_complete(const ShardArgs& s, int* err) {
    __threadfence_system();
    const unsigned t = atomicAdd(s.done, 1u);
    if (t == gridDim.x - 1) {
        __threadfence_system();
        *s.done = 0;
        volatile unsigned* ep = s.epoch;
        const unsigned e = *ep + 1;
        *ep = e;
        if (*reinterpret_cast<volatile int*>(err) == 0)
            for (int r = 0; r < s.world; ++r) st_release_sys(s.peer_flags[r] + s.rank, e);
    }
}

}  // namespace
}  // namespace bramha
