// common.cuh -- device helpers shared by the sm_100a kernels of b200q8.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200q8 {

// 16-byte streaming load of weight bytes: read once, so no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream16(const void* p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Exact int8 -> fp32 for the four bytes of `w`, without the I2F conversion
// pipe.  Flipping the sign bit turns int8 v into the unsigned byte v + 128;
// byte_perm drops that byte into the low mantissa bits of 2^23 (bit pattern
// 0x4B0000uu), so the float equals 2^23 + v + 128 exactly, and one packed
// subtraction of 2^23 + 128 leaves v.  (The exponent-bias conversion used by
// mixed-input GEMMs since the FasterTransformer kernels.)
__device__ __forceinline__ void i8x4_to_f32x4(uint32_t w, float2& lo, float2& hi)
{
    const uint32_t u = w ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    lo.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440));
    lo.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441));
    hi.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442));
    hi.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443));
    lo = __fadd2_rn(lo, bias);
    hi = __fadd2_rn(hi, bias);
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p)
{
    return *p;
}
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half* p)
{
    return __half2float(*p);
}

template <typename T>
__device__ __forceinline__ void store_from_f32(T* p, float v);
template <>
__device__ __forceinline__ void store_from_f32<float>(float* p, float v)
{
    *p = v;
}
template <>
__device__ __forceinline__ void store_from_f32<__half>(__half* p, float v)
{
    *p = __float2half_rn(v);
}

// Epilogue shared by every linear kernel, in the reference's order
// (src/backend/backend_naive.cc:283-288, then :333-334 for the residual):
// v = acc * scale; v = v + bias; v = v + residual.  Explicit _rn ops keep the
// compiler from contracting these into FMAs.
template <typename OT>
__device__ __forceinline__ void epilogue_store(OT* out, const OT* res, float acc, float scale,
                                               const float* bias, int row)
{
    float v = __fmul_rn(acc, scale);
    if (bias) v = __fadd_rn(v, bias[row]);
    if (res) v = __fadd_rn(v, load_as_f32<OT>(res));
    store_from_f32<OT>(out, v);
}

// Programmatic dependent launch: wait until the grid we depend on has
// finished its writes (no-op when the launch carries no PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

}  // namespace b200q8
