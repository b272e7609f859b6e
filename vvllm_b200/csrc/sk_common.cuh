// sk_common.cuh -- persistent stream-K scheduling helpers shared by the tensor-core kernels.
//
// The (tile, K-stage) units of a problem are laid out tile-major and cut into
// gridDim.x equal contiguous ranges, one per CTA: CTA j owns units
// [j*U/G, (j+1)*U/G).  A tile whose units span several CTAs is reduced by the
// piece that arrives last (per-tile arrival counter); each piece writes its
// partial accumulator to workspace slot 2j (its range's first segment) or 2j+1
// (its last segment).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace b200q8 {
namespace sk {

// CTA owning unit u under the equal split of `units` over G CTAs.
__device__ __forceinline__ int cta_of_unit(long long u, long long units, int G)
{
    return (int)(((u + 1) * (long long)G - 1) / units);
}

__device__ __forceinline__ long long unit_begin(int j, long long units, int G)
{
    return (long long)j * units / G;
}

// Workspace slot holding CTA j's piece of the tile whose first unit is tb.
__device__ __forceinline__ int piece_slot(int j, long long tb, long long units, int G)
{
    return (unit_begin(j, units, G) >= tb) ? 2 * j : 2 * j + 1;
}

// Walks the segments (tile, k0, k1) of one CTA's unit range.
struct SegIter {
    long long u, end;
    int kbpt;
    __device__ SegIter(long long b, long long e, int k) : u(b), end(e), kbpt(k) {}
    __device__ bool next(int& t, int& k0, int& k1)
    {
        if (u >= end) return false;
        t = (int)(u / kbpt);
        k0 = (int)(u - (long long)t * kbpt);
        const long long left = end - u;
        k1 = (left < (long long)(kbpt - k0)) ? k0 + (int)left : kbpt;
        u += k1 - k0;
        return true;
    }
};

// Position in a ring of n stages: index and the parity of its current round.
struct Ring {
    int idx = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void next(int n)
    {
        if (++idx == n) {
            idx = 0;
            phase ^= 1u;
        }
    }
};

template <typename OT>
__device__ __forceinline__ void store_out(OT* p, float v);
template <>
__device__ __forceinline__ void store_out<float>(float* p, float v)
{
    *p = v;
}
template <>
__device__ __forceinline__ void store_out<__half>(__half* p, float v)
{
    *p = __float2half_rn(v);
}

}  // namespace sk
}  // namespace b200q8
