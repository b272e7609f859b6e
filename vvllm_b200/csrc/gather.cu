// gather.cu -- reorders an all-gathered, rank-major output [G][M][Ns] into [M][N].
//
// Rank r owns output channels [r*Ns, r*Ns + Ns) (the last ranks may own fewer);
// NCCL's all-gather leaves each rank's [M, Ns] slice contiguous.  One thread
// moves one element; columns at or beyond N (padding of short tail shards)
// are dropped.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace b200q8 {

namespace {

template <typename T>
__global__ void gather_permute_kernel(const T* __restrict__ src, T* __restrict__ dst, long long G,
                                      long long M, long long Ns, long long N)
{
    const long long total = M * N;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / N, n = i % N;
        const long long r = n / Ns, j = n % Ns;
        dst[i] = src[(r * M + m) * Ns + j];
    }
}

}  // namespace

cudaError_t launch_gather_permute(const void* src, void* dst, int elem_bytes, size_t G, size_t M,
                                  size_t Ns, size_t N, cudaStream_t stream)
{
    const long long total = (long long)(M * N);
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    if (elem_bytes == 2)
        gather_permute_kernel<uint16_t><<<(unsigned)blocks, 256, 0, stream>>>(
            (const uint16_t*)src, (uint16_t*)dst, (long long)G, (long long)M, (long long)Ns, (long long)N);
    else
        gather_permute_kernel<uint32_t><<<(unsigned)blocks, 256, 0, stream>>>(
            (const uint32_t*)src, (uint32_t*)dst, (long long)G, (long long)M, (long long)Ns, (long long)N);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace b200q8
