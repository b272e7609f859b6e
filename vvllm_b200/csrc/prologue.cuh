// prologue.cuh -- the elementwise step before a projection, computed where the
// projection reads its activations.
//
// vvllm runs two elementwise ops right before quantized linears in every layer:
//   rms_norm (src/backend/backend_naive.cc:67-75, CUDA src/backend/cuda_kernels.cu:69-104 and
//     :886-910): out[k] = x[k] / rms * w[k], rms = sqrt(sum_k x[k]^2 / K + eps), before the
//     q/k/v and gate_up projections (include/vvllm/model/transformer.h:135-144, :167-169);
//   silu_mul (backend_naive.cc:293-300, cuda_kernels.cu:55-63 and :876-884):
//     out[k] = (g / (1 + exp(-g))) * u on gate_up = [g | u] per token, before the down
//     projection (transformer.h:171-188).
// In fp16 mode the reference rounds the norm weight to fp16 when it caches it
// (backend_cuda.cc:135-145) and rounds the result to fp16; so does act4.
//
// The sum of squares is taken by kSqThreads = 256 threads in one fixed order (double partials
// over 4-element groups t, t+256, ...; an xor-shuffle tree per warp; the eight warps added in
// order), by every kernel that needs a token's rms: the SIMT GEMV's x staging, the digit GEMV's prep kernel
// and the standalone prologue kernel all get the same bits, so a fused projection equals
// the standalone prologue followed by the plain projection exactly.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200q8 {

enum Prologue : int { kProNone = 0, kProRmsNorm = 1, kProSiluMul = 2 };
constexpr int kSqThreads = 256;
constexpr int kSqWarps = kSqThreads / 32;

// Four consecutive activations as fp32 (fp16: one 8-byte load; fp32: one 16-byte load).
template <typename XT>
__device__ __forceinline__ void load4(const XT* p, float (&v)[4])
{
    if constexpr (sizeof(XT) == 2) {
        const uint2 raw = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
        const float4 raw = *reinterpret_cast<const float4*>(p);
        v[0] = raw.x; v[1] = raw.y; v[2] = raw.z; v[3] = raw.w;
    }
}

// Four consecutive activations stored as XT (fp16: round to nearest).
template <typename XT>
__device__ __forceinline__ void store4(XT* p, const float (&v)[4])
{
    if constexpr (sizeof(XT) == 2) {
        const __half2 a = __floats2half2_rn(v[0], v[1]);
        const __half2 b = __floats2half2_rn(v[2], v[3]);
        uint2 raw;
        raw.x = *reinterpret_cast<const uint32_t*>(&a);
        raw.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = raw;
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// The inputs of four activations at k .. k+3 of one token whose input row starts at xrow: x
// (kProSiluMul: the gate, xrow[k]) and the second operand (the norm weight, or the up half at
// xrow[K + k]).  Split from act4_apply so that callers can issue several groups' loads at once.
template <typename XT>
__device__ __forceinline__ void act4_load(int pro, const XT* xrow, int K, int k, const float* norm_w, float (&v)[4],
                                          float (&aux)[4])
{
    load4<XT>(xrow + k, v);
    if (pro == kProRmsNorm) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w + k));
        aux[0] = w.x; aux[1] = w.y; aux[2] = w.z; aux[3] = w.w;
    } else if (pro == kProSiluMul) {
        load4<XT>(xrow + K + k, aux);
    }
}

// The activations from act4_load's inputs (rms: the token's rms for kProRmsNorm).
template <typename XT>
__device__ __forceinline__ void act4_apply(int pro, float rms, float (&v)[4], const float (&aux)[4])
{
    if (pro == kProRmsNorm) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float w = aux[i];
            if constexpr (sizeof(XT) == 2) w = __half2float(__float2half_rn(w));
            v[i] = __fmul_rn(__fdiv_rn(v[i], rms), w);
        }
    } else if (pro == kProSiluMul) {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], __fadd_rn(1.0f, expf(-v[i]))), aux[i]);
    }
    if constexpr (sizeof(XT) == 2) {
        if (pro != kProNone) {
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = __half2float(__float2half_rn(v[i]));
        }
    }
}

// The activation the projection consumes at k .. k+3 of one token whose input row starts at
// xrow (kProSiluMul: gate at xrow[k], up at xrow[K + k]).  rms is the token's rms (kProRmsNorm).
template <typename XT>
__device__ __forceinline__ void act4(int pro, const XT* xrow, int K, int k, const float* norm_w, float rms,
                                     float (&v)[4])
{
    float aux[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    act4_load<XT>(pro, xrow, K, k, norm_w, v, aux);
    act4_apply<XT>(pro, rms, v, aux);
}

// Groups of a row handled per batch by one thread: all their loads are issued before any
// arithmetic, so a thread waits for memory once per batch rather than once per group.  Passes
// holding two operands per group in callers short of registers (the GEMV's warps, the prep
// kernel that must fit beside a GEMV CTA) use 2.
constexpr int kRowBatch = 4;

// Thread t (0..kSqThreads-1) of the token's sum of squares: its double partial over 4-element
// groups t, t+kSqThreads, ..., reduced over its warp (every lane gets the warp's sum).  K % 4 == 0.
// (The batch size B changes only when loads are issued, not the order of the sum.)
template <typename XT, int B = kRowBatch>
__device__ __forceinline__ double sumsq_warp(const XT* xrow, int K, int t)
{
    double s = 0.0;
    const int g4 = K >> 2;
    for (int i0 = t; i0 < g4; i0 += B * kSqThreads) {
        float v[B][4];
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int i = i0 + b * kSqThreads;
            if (i < g4) load4<XT>(xrow + 4 * i, v[b]);
            else v[b][0] = v[b][1] = v[b][2] = v[b][3] = 0.0f;
        }
#pragma unroll
        for (int b = 0; b < B; b++)  // groups in order t, t+256, ...: the fixed order
#pragma unroll
            for (int j = 0; j < 4; j++) s += (double)v[b][j] * (double)v[b][j];  // exact products
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// rms from the kSqWarps warps' partials (added in order): sqrt(sum / K + eps) in fp32, as the
// reference computes it.
__device__ __forceinline__ float rms_from(const double* warp_sums, int K, float eps)
{
    double s = warp_sums[0];
#pragma unroll
    for (int w = 1; w < kSqWarps; w++) s += warp_sums[w];
    return __fsqrt_rn(__fadd_rn(__fdiv_rn((float)s, (float)K), eps));
}

// How many CTAs share one token's row in the K-split elementwise kernels: about four 4-element
// groups per thread of a 256-thread CTA, at most 64 CTAs.
__host__ __device__ __forceinline__ int row_splits(long long K)
{
    const long long g = (K / 4 + 1023) / 1024;
    return g < 1 ? 1 : (g > 64 ? 64 : (int)g);
}

}  // namespace b200q8
