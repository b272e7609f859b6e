// tmap.cuh -- 2-D TMA tensor maps, encoded through the driver entry point and
// cached per host thread.
//
// A tensor map only describes an address range (base, extents, strides, box,
// swizzle), never the contents, so a map made for the same description is
// always valid again; caching it takes cuTensorMapEncodeTiled (several
// microseconds of host time) off every launch.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

namespace b200q8 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        cudaGetLastError();
    });
    return fn;
}

struct TmapDesc {
    const void* base;
    uint64_t inner, outer;    // extents in elements (inner = contiguous dimension)
    uint64_t row_bytes;       // stride of the outer dimension
    uint32_t box_inner, box_outer;
    int dtype;                // CUtensorMapDataType
    int swizzle;              // CUtensorMapSwizzle
    bool operator==(const TmapDesc& o) const { return memcmp(this, &o, sizeof(TmapDesc)) == 0; }
};

// Row-major 2-D map with zero fill out of range; false if the driver refuses it.
inline bool tmap_2d(CUtensorMap* out, const TmapDesc& d)
{
    constexpr int kEntries = 64;
    struct Cache {
        TmapDesc key[kEntries];
        CUtensorMap map[kEntries];
        int used = 0, next = 0;
    };
    static thread_local Cache c;
    for (int i = 0; i < c.used; i++)
        if (c.key[i] == d) {
            *out = c.map[i];
            return true;
        }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)d.inner, (cuuint64_t)d.outer};
    const cuuint64_t strides[1] = {(cuuint64_t)d.row_bytes};
    const cuuint32_t box[2] = {d.box_inner, d.box_outer};
    const cuuint32_t es[2] = {1, 1};
    CUtensorMap m;
    if (enc(&m, (CUtensorMapDataType)d.dtype, 2, const_cast<void*>(d.base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)d.swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const int slot = c.used < kEntries ? c.used++ : (c.next++ % kEntries);
    c.key[slot] = d;
    c.map[slot] = m;
    *out = m;
    return true;
}

}  // namespace b200q8
