// p2p.cuh -- completion counts of the gathered (column-sharded) calls: publishing a call and the
// bounded wait for every rank's outputs.  Protocol: kernels.h (P2POut).
#pragma once

#include <stdint.h>

#include "kernels.h"

namespace b200q8 {

// One thread, once the stores to publish are ordered before it (the GEMV grid that made them has
// completed): one system-scope fence makes them (local and over NVLink) visible everywhere
// before the count moves, then a relaxed reduction adds `share` to counts[d][rank] on every
// rank d (this rank's own slot last).  One fence, not one per rank.
__device__ __forceinline__ void publish_share(unsigned long long* const* counts, int ndst, int rank,
                                              unsigned long long share)
{
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int i = 1; i <= ndst; i++) {
        const int d = (rank + i) % ndst;
        asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(counts[d] + rank), "l"(share) : "memory");
    }
}

// One thread: bounded wait (timeout_ns of %globaltimer) until every counts[j], j < n, holds as
// many whole calls as counts[self], this rank's own count, which is complete for every earlier
// call once the previous kernel in the stream has finished.  Relaxed system-scope polls, then
// one acquire fence: this thread's later reads -- and, across a barrier, its CTA's -- see every
// rank's outputs of those calls.  False when the limit ran out.
__device__ __forceinline__ bool wait_peers(const unsigned long long* counts, int n, int self,
                                           unsigned long long timeout_ns)
{
    unsigned long long own;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(own) : "l"(counts + self) : "memory");
    const unsigned long long target = own & ~((1ull << kCountShift) - 1ull);
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        bool all = true;
        for (int j = 0; j < n; j++) {
            unsigned long long v;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counts + j) : "memory");
            all = all && (long long)(v - target) >= 0;
        }
        if (all) break;
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > timeout_ns) return false;
        __nanosleep(32);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    return true;
}

}  // namespace b200q8
