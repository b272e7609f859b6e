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

__device__ int g_kernel_error_p2p;  // bit 1: a peer's flag did not arrive in time

namespace {

// counts[j] grows by 2^kCountShift per call of rank j once all of that call's CTAs have
// stored their outputs here (system-scope release reductions); a peer can run at most one
// call ahead, so "arrived" is a wrapping compare.  The kernel is launched as a programmatic
// dependent of this rank's GEMV and lets its own dependents launch at once: they only pass
// griddepcontrol.wait once every rank's count, this rank's included, has been seen here.
__global__ void p2p_wait_kernel(const unsigned long long* counts, int nranks, int rank, unsigned int seq,
                                unsigned long long timeout_ns)
{
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    const unsigned long long target = (unsigned long long)seq << kCountShift;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (int i = 1; i <= nranks; i++) {
        const int j = (rank + i) % nranks;
        for (;;) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counts + j) : "memory");
            if ((long long)(v - target) >= 0) break;
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > timeout_ns) {
                atomicOr(&g_kernel_error_p2p, 2);
                return;
            }
            __nanosleep(64);
        }
    }
}

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

cudaError_t launch_p2p_wait(const unsigned long long* counts, int nranks, int rank, unsigned int seq,
                            unsigned long long timeout_ns, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, p2p_wait_kernel, counts, nranks, rank, seq, timeout_ns);
    if (e == cudaSuccess) note_launch();
    return e;
}

cudaError_t read_kernel_error_p2p(int* code, bool clear)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_kernel_error_p2p, sizeof(int));
    if (e != cudaSuccess) return e;
    *code = v;
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_kernel_error_p2p, &z, sizeof(int));
    }
    return e;
}

}  // namespace b200q8
