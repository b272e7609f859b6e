// q8_quantize.cu -- per-output-channel absmax int8 quantization on the GPU.
//
// Bit-identical to vvllm::quantize_per_channel (src/quantize/quantize.cc:9-48):
//   absmax = max_k |w|            std::max(a, |w|) == (a < |w|) ? |w| : a, so NaN is skipped
//   scale  = absmax / 127.0f      IEEE division (__fdiv_rn)
//   scale == 0 -> the row is all zeros
//   inv    = 1.0f / scale         IEEE division (overflows to +inf for tiny scales, as on x86)
//   q      = (int8) max(-128, min(127, roundf(w * inv)))   min/max as std::min/std::max
// The build keeps denormals (no -ftz, no fast-math), as the x86 reference does.
//
// One HBM pass: the row is held in registers (a warp per row for K <= 1024,
// a 256- or 512-thread CTA per row up to K = 20480), its absmax reduced with
// shuffles (and shared memory across warps), then quantized from registers.
// Other shapes (K % 4 != 0, misaligned, larger K) use a two-pass kernel that
// re-reads the row (from L2).
//
// The source is fp32 or bf16 (raw bfloat16 bits as stored in a safetensors file); bf16 is widened
// exactly (bits << 16), which is what vvllm's loader does before quantizing
// (SafeTensorsLoader::bf16_to_f32, src/safetensors/safetensors.cc:131-137), so a checkpoint can be
// quantized on the GPU straight from its stored bytes with the same result.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace b200q8 {

namespace {

__device__ __forceinline__ float ref_max(float a, float b) { return (a < b) ? b : a; }
__device__ __forceinline__ float ref_min(float a, float b) { return (b < a) ? b : a; }

__device__ __forceinline__ int8_t quant_one(float w, float inv)
{
    float v = __fmul_rn(w, inv);
    v = ref_max(-128.0f, ref_min(127.0f, roundf(v)));
    return (int8_t)(int)v;
}

// Four consecutive source elements as fp32: fp32 one 16-byte load, bf16 one 8-byte load
// (streaming: every weight is read once).
template <typename WT>
__device__ __forceinline__ float4 load4w(const WT* row, int i);
template <>
__device__ __forceinline__ float4 load4w<float>(const float* row, int i)
{
    return __ldcs(reinterpret_cast<const float4*>(row) + i);
}
template <>
__device__ __forceinline__ float4 load4w<uint16_t>(const uint16_t* row, int i)
{
    const uint2 r = __ldcs(reinterpret_cast<const uint2*>(row) + i);
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                       __uint_as_float(r.y & 0xFFFF0000u));
}
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

__device__ __forceinline__ float warp_absmax(float m)
{
    // Partial maxima are never NaN (they start at 0 and only take non-NaN |w|),
    // so any reduction order gives the sequential result.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

// Rows held in registers: T threads per row, E float4 per thread (K <= 4 * T * E).
template <typename WT, int T, int E>
__global__ void __launch_bounds__(T == 32 ? 256 : T) q8_quantize_reg_kernel(
    const WT* __restrict__ w, int8_t* __restrict__ q, float* __restrict__ scales, int N, int K)
{
    constexpr int kRowsPerBlock = (T == 32) ? 8 : 1;
    __shared__ float wmax[T == 32 ? 1 : T / 32];
    const int lane = threadIdx.x & 31;
    const int tid = (T == 32) ? lane : threadIdx.x;
    const int K4 = K >> 2;
    for (long long row = (long long)blockIdx.x * kRowsPerBlock + (T == 32 ? (threadIdx.x >> 5) : 0);
         row < N; row += (long long)gridDim.x * kRowsPerBlock) {
        const WT* src = w + row * K;
        float4 v[E];
        float m = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) {
            const int i = tid + e * T;
            if (i < K4) {
                v[e] = load4w<WT>(src, i);
                m = ref_max(m, fabsf(v[e].x));
                m = ref_max(m, fabsf(v[e].y));
                m = ref_max(m, fabsf(v[e].z));
                m = ref_max(m, fabsf(v[e].w));
            }
        }
        m = warp_absmax(m);
        if (T > 32) {
            if (lane == 0) wmax[threadIdx.x >> 5] = m;
            __syncthreads();
            float mm = 0.0f;
#pragma unroll
            for (int i = 0; i < T / 32; i++) mm = fmaxf(mm, wmax[i]);
            m = mm;
            __syncthreads();  // wmax is reused by the next row
        }
        const float scale = __fdiv_rn(m, 127.0f);
        if (tid == 0) scales[row] = scale;
        char4* dst = reinterpret_cast<char4*>(q + row * K);
        if (scale == 0.0f) {
#pragma unroll
            for (int e = 0; e < E; e++) {
                const int i = tid + e * T;
                if (i < K4) dst[i] = make_char4(0, 0, 0, 0);
            }
        } else {
            const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
            for (int e = 0; e < E; e++) {
                const int i = tid + e * T;
                if (i < K4)
                    dst[i] = make_char4(quant_one(v[e].x, inv), quant_one(v[e].y, inv),
                                        quant_one(v[e].z, inv), quant_one(v[e].w, inv));
            }
        }
    }
}

// Any K, any alignment: one CTA per row, absmax pass then quantize pass.
template <typename WT>
__global__ void __launch_bounds__(256) q8_quantize_generic_kernel(const WT* __restrict__ w,
                                                                  int8_t* __restrict__ q,
                                                                  float* __restrict__ scales, int N,
                                                                  long long K)
{
    __shared__ float wmax[8];
    for (long long row = blockIdx.x; row < N; row += gridDim.x) {
        const WT* src = w + row * K;
        float m = 0.0f;
        for (long long k = threadIdx.x; k < K; k += blockDim.x) m = ref_max(m, fabsf(to_f32(src[k])));
        m = warp_absmax(m);
        if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
        __syncthreads();
        float mm = 0.0f;
        for (int i = 0; i < 8; i++) mm = fmaxf(mm, wmax[i]);
        __syncthreads();
        const float scale = __fdiv_rn(mm, 127.0f);
        if (threadIdx.x == 0) scales[row] = scale;
        int8_t* dst = q + row * K;
        if (scale == 0.0f) {
            for (long long k = threadIdx.x; k < K; k += blockDim.x) dst[k] = 0;
        } else {
            const float inv = __fdiv_rn(1.0f, scale);
            for (long long k = threadIdx.x; k < K; k += blockDim.x) dst[k] = quant_one(to_f32(src[k]), inv);
        }
    }
}

template <typename WT, int T, int E>
cudaError_t launch_reg(const WT* w, size_t N, size_t K, int8_t* q, float* scales, int num_sms,
                       cudaStream_t stream)
{
    constexpr int kThreads = (T == 32) ? 256 : T;
    constexpr int kRowsPerBlock = (T == 32) ? 8 : 1;
    long long blocks = ((long long)N + kRowsPerBlock - 1) / kRowsPerBlock;
    const long long cap = (long long)num_sms * (2048 / kThreads);
    if (blocks > cap) blocks = cap;
    q8_quantize_reg_kernel<WT, T, E><<<(unsigned)blocks, kThreads, 0, stream>>>(w, q, scales, (int)N, (int)K);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

template <typename WT>
cudaError_t launch_typed(const WT* w, size_t N, size_t K, int8_t* q, float* scales, int num_sms, cudaStream_t stream)
{
    const bool vec = (K % 4 == 0) && ((uintptr_t)w % (4 * sizeof(WT)) == 0) && ((uintptr_t)q % 4 == 0) &&
                     K <= 20480 && N < (1u << 31);
    if (vec) {
        if (K <= 32 * 4 * 8) return launch_reg<WT, 32, 8>(w, N, K, q, scales, num_sms, stream);
        if (K <= 256 * 4 * 4) return launch_reg<WT, 256, 4>(w, N, K, q, scales, num_sms, stream);
        if (K <= 256 * 4 * 8) return launch_reg<WT, 256, 8>(w, N, K, q, scales, num_sms, stream);
        return launch_reg<WT, 512, 10>(w, N, K, q, scales, num_sms, stream);
    }
    long long blocks = (long long)N;
    if (blocks > (long long)num_sms * 8) blocks = (long long)num_sms * 8;
    if (blocks < 1) blocks = 1;
    q8_quantize_generic_kernel<WT><<<(unsigned)blocks, 256, 0, stream>>>(w, q, scales, (int)N, (long long)K);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace

cudaError_t launch_q8_quantize(const float* w, size_t N, size_t K, int8_t* q, float* scales,
                               int num_sms, cudaStream_t stream)
{
    return launch_typed<float>(w, N, K, q, scales, num_sms, stream);
}

cudaError_t launch_q8_quantize_bf16(const uint16_t* w, size_t N, size_t K, int8_t* q, float* scales, int num_sms,
                                    cudaStream_t stream)
{
    return launch_typed<uint16_t>(w, N, K, q, scales, num_sms, stream);
}

}  // namespace b200q8
