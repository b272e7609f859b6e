// prologue.cu -- standalone rms_norm / silu_mul over M tokens.
//
// The same arithmetic (prologue.cuh) as the SIMT GEMV applies while it stages x and the digit
// GEMV's prep kernel applies when it writes the activations,
// for the projections that run on the fp16 tensor-core GEMM (prefill: the activations are
// written once and the GEMM's TMA reads them) and for the b200q8_rms_norm / b200q8_silu_mul
// entry points (vvllm Backend::rms_norm per token, Backend::silu_mul over gate_up rows:
// include/vvllm/backend/backend.h:46-68, src/model/transformer.cc:40-50).
//
// 256-thread CTAs.  rms_norm: one CTA per token (the row is read twice, the second time from
// L2/L1; the sum is prologue.cuh's fixed-order one).  silu_mul: no reduction, so row_splits(K)
// CTAs share each row (one CTA per row left a 18944-wide decode row latency-bound on one SM).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "prologue.cuh"

namespace b200q8 {
namespace {

template <typename XT>
__global__ void __launch_bounds__(kSqThreads) prologue_kernel(const XT* __restrict__ x, XT* __restrict__ out,
                                                              int pro, const float* __restrict__ norm_w, float eps,
                                                              int K)
{
    pdl_launch_dependents();  // the projection may start streaming its weights
    pdl_wait();               // x is written by the previous kernel
    __shared__ double sq[kSqWarps];
    const int m = blockIdx.x;
    const XT* xrow = x + (size_t)m * (pro == kProSiluMul ? 2 * (size_t)K : (size_t)K);
    float rms = 1.0f;
    if (pro == kProRmsNorm) {
        const double w = sumsq_warp<XT>(xrow, K, threadIdx.x);
        if ((threadIdx.x & 31) == 0) sq[threadIdx.x >> 5] = w;
        __syncthreads();
        rms = rms_from(sq, K, eps);
    }
    // this CTA's share of the row's 4-element groups (the whole row for rms_norm)
    const int g4 = K >> 2;
    const int c0 = (int)((long long)g4 * blockIdx.y / gridDim.y);
    const int c1 = (int)((long long)g4 * (blockIdx.y + 1) / gridDim.y);
    XT* orow = out + (size_t)m * K;
    for (int i0 = c0 + threadIdx.x; i0 < c1; i0 += kRowBatch * kSqThreads) {
        float v[kRowBatch][4], aux[kRowBatch][4];
#pragma unroll
        for (int b = 0; b < kRowBatch; b++)  // every load of the batch first
            if (i0 + b * kSqThreads < c1) act4_load<XT>(pro, xrow, K, 4 * (i0 + b * kSqThreads), norm_w, v[b], aux[b]);
#pragma unroll
        for (int b = 0; b < kRowBatch; b++) {
            const int i = i0 + b * kSqThreads;
            if (i >= c1) break;
            act4_apply<XT>(pro, rms, v[b], aux[b]);
            store4<XT>(orow + 4 * i, v[b]);
        }
    }
}

}  // namespace

cudaError_t launch_prologue(int pro, const void* x, void* out, int dtype, const float* norm_w, float eps, size_t M,
                            size_t K, bool pdl, cudaStream_t stream)
{
    if ((pro != kProRmsNorm && pro != kProSiluMul) || K % 4 != 0 || K > (size_t)INT32_MAX ||
        M > (size_t)INT32_MAX)
        return cudaErrorInvalidValue;
    if (M == 0 || K == 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M, pro == kProSiluMul ? (unsigned)row_splits((long long)K) : 1u);
    cfg.blockDim = dim3(kSqThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e;
    if (dtype == kF16)
        e = cudaLaunchKernelEx(&cfg, prologue_kernel<__half>, reinterpret_cast<const __half*>(x),
                               reinterpret_cast<__half*>(out), pro, norm_w, eps, (int)K);
    else
        e = cudaLaunchKernelEx(&cfg, prologue_kernel<float>, reinterpret_cast<const float*>(x),
                               reinterpret_cast<float*>(out), pro, norm_w, eps, (int)K);
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace b200q8
