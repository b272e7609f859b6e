// q8_gemm_tc.cu -- int8-weight x fp16-activation GEMM on the 5th-gen tensor cores.
//
// out[m, n] = (sum_k x[m, k] * float(W[n, k])) * scales[n] + bias[n] (+ res[m, n])
// (semantics of vvllm BackendCPU::linear_q8 / linear_q8_add,
//  src/backend/backend_naive.cc:155-291 and :322-335, with fp16 activations.)
//
// Tiling ("swap-AB"): a tile is 128 weight rows (UMMA M) x BN tokens (UMMA N,
// 16..128), so one kernel serves M = 1 decode through M = 512 prefill.  K
// runs in BK-wide pipeline stages (256 for decode tiles, 128 for wide token
// tiles); each stage carries BK/16 tcgen05.mma instructions, enough work to
// hide the per-stage control cost of the single issuing thread.
//
// Persistent stream-K schedule: the (tile, K-stage) units of the whole problem
// are laid out tile-major and cut into gridDim.x equal contiguous ranges, one
// per CTA (one CTA per SM).  A CTA works on a few whole tiles plus at most two
// partial tiles at the ends of its range; skinny shapes (few tiles, long K)
// still keep every SM busy, and no wave is left half-empty.  A tile split over
// several CTAs is finished deterministically: each piece stores its fp32
// partial accumulator to a workspace slot, bumps the tile's counter, and the
// piece that arrives last sums all pieces in K order, applies the epilogue and
// resets the counter.  No CTA ever waits on another.
//
// Warp roles (14 warps):
//   0      TMA producer: int8 weight tile [128 x BK] as 128-byte-swizzled
//          [128 x 128 B] boxes and fp16 activation tile [BN x BK] as
//          128-byte-swizzled [BN x 64] boxes into an S-stage shared-memory
//          ring, completing on mbarriers;
//   1      TMEM allocator; one thread issues tcgen05.mma.kind::f16
//          [D_tmem], [A_tmem], B_desc into one of two TMEM accumulators, and
//          tcgen05.commit frees the stages;
//   2..9   dequantizers in two groups taking alternate stages: a thread owns
//          one weight row (= TMEM lane), reads its BK int8 from shared memory
//          (conflict-free under the swizzle), converts them exactly to fp16
//          (exponent-bias trick) and tcgen05.st's them into an SA-stage TMEM
//          ring -- the MMA's A operand lives in tensor memory, so no fp16
//          weight copy ever touches shared memory or HBM;
//   10..13 epilogue: tcgen05.ld of the finished accumulator, then
//          v = acc * scale[n] (+ bias[n]) (+ res[m, n]) stored as fp16/fp32,
//          or the stream-K partial/fixup path.
// Every mbarrier wait is bounded (wall clock); a timeout sets a device error
// word, drains in-flight copies and MMAs, frees TMEM and returns.  No TMA
// multicast and no thread-block clusters are used.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_utils.cuh"

namespace b200q8 {

__device__ int g_kernel_error;  // bit 0: a bounded wait timed out in the tensor-core GEMM

namespace {

constexpr int kTileRows = 128;  // weight rows per tile (UMMA M)
constexpr int kWarps = 14;
constexpr int kThreads = kWarps * 32;
constexpr int kFirstConv = 2, kFirstEpi = 10;
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s: far above any legitimate wait

struct SkParams {
    const float* scales;
    const float* bias;
    const void* res;
    void* out;
    float* ws;          // [2 * gridDim.x][BN][128] fp32 partial accumulators
    int* counters;      // [tiles] arrival counters, zero between launches
    int M, N, K;
    int kbpt;           // K stages per tile
    int tiles_n;        // weight-row tiles
    long long units;    // tiles * kbpt
};

template <int BN, int BK, int S, int SA>
struct SkCfg {
    static constexpr int kWBoxes = BK / 128;            // [128 rows x 128 B] int8 boxes per stage
    static constexpr int kXBoxes = BK / 64;             // [BN rows x 64 fp16] boxes per stage
    static constexpr int kW8Bytes = kTileRows * BK;
    static constexpr int kXBoxBytes = BN * 128;
    static constexpr int kXBytes = kXBoxes * kXBoxBytes;
    static constexpr int kACols = BK / 2;               // TMEM columns of one A stage
    static constexpr int kDCols = (BN + 31) / 32 * 32;  // one accumulator, 32-column aligned
    static constexpr int kACol = 2 * kDCols;
    static constexpr int kColsNeeded = kACol + SA * kACols;
    static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                     : kColsNeeded <= 256 ? 256 : 512;
    static constexpr int kNumBars = 2 * S + 2 * SA + 4 + 1;  // + accfull[2], accempty[2], drain
    static constexpr int kSmemBytes = 1024 + S * (kW8Bytes + kXBytes) + kNumBars * 8 + 16;
    static_assert(kColsNeeded <= 512, "TMEM overflow");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 128, "UMMA N for M=128, two accumulators");
    static_assert(BK % 128 == 0, "stage K is whole 128-byte weight boxes");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kXBoxBytes % 1024 == 0, "activation boxes stay 1024-byte aligned");
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

__device__ __forceinline__ void raise_error(volatile int* abort)
{
    *abort = 1;
    atomicOr(&g_kernel_error, 1);
}

// CTA owning unit u under the equal split of `units` over G CTAs (CTA j owns [j*U/G, (j+1)*U/G)).
__device__ __forceinline__ int cta_of_unit(long long u, long long units, int G)
{
    return (int)(((u + 1) * (long long)G - 1) / units);
}

__device__ __forceinline__ long long unit_begin(int j, long long units, int G)
{
    return (long long)j * units / G;
}

// Walks the segments (tile, k0, k1) of this CTA's unit range.
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

// Position in a ring of N stages: index and the parity of its current round.
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

// Epilogue of up to 16 consecutive tokens of one output channel: element i goes to
// o[i * ld]; v = acc * scale (+ bias) (+ res), in the reference's order.
template <typename OT>
__device__ __forceinline__ void epi_chunk(OT* o, const OT* res, int ld, int cnt, const uint32_t (&d)[16], float scale,
                                          float bias, bool has_bias)
{
    if (cnt == 16) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            float v = __fmul_rn(__uint_as_float(d[i]), scale);
            if (has_bias) v = __fadd_rn(v, bias);
            if (res) v = __fadd_rn(v, load_as_f32<OT>(res + (size_t)i * ld));
            store_out<OT>(o + (size_t)i * ld, v);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (i < cnt) {
                float v = __fmul_rn(__uint_as_float(d[i]), scale);
                if (has_bias) v = __fadd_rn(v, bias);
                if (res) v = __fadd_rn(v, load_as_f32<OT>(res + (size_t)i * ld));
                store_out<OT>(o + (size_t)i * ld, v);
            }
        }
    }
}

template <int BN, int BK, int S, int SA, typename OT>
__global__ void __launch_bounds__(kThreads, 1)
    q8_gemm_sk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const SkParams p)
{
    using C = SkCfg<BN, BK, S, SA>;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* sW8 = smem;
    unsigned char* sX = smem + S * C::kW8Bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sX + S * C::kXBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_holder + 2);

    const uint32_t bar0 = tc::smem_u32(bars);
    const uint32_t full0 = bar0, empty0 = bar0 + 8u * S, afull0 = bar0 + 16u * S,
                   aempty0 = bar0 + 16u * S + 8u * SA, accfull0 = bar0 + 16u * S + 16u * SA,
                   accempty0 = accfull0 + 16u, drainbar = accfull0 + 32u;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int cta = blockIdx.x;
    const long long u_begin = unit_begin(cta, p.units, G), u_end = unit_begin(cta + 1, p.units, G);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            tc::mbar_init(full0 + 8u * s, 1);
            tc::mbar_init(empty0 + 8u * s, 1);
        }
        for (int s = 0; s < SA; s++) {
            tc::mbar_init(afull0 + 8u * s, 4);
            tc::mbar_init(aempty0 + 8u * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(accfull0 + 8u * b, 1);
            tc::mbar_init(accempty0 + 8u * b, 4);
        }
        tc::mbar_init(drainbar, 1);
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (threadIdx.x == 32) {
        tc::prefetch_tensormap(&tmW);
        tc::prefetch_tensormap(&tmX);
    }
    // Activations come from the previous kernel; hold no TMEM while waiting for it.
    pdl_wait();
    __syncwarp();
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_holder), C::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            Ring st;
            int issued = 0;
            int t, k0, k1;
            SegIter it(u_begin, u_end, p.kbpt);
            bool ok = true;
            const uint32_t sw_base = tc::smem_u32(sW8), sx_base = tc::smem_u32(sX);
            while (ok && it.next(t, k0, k1)) {
                const int row0 = (t % p.tiles_n) * kTileRows;
                const int m0 = (t / p.tiles_n) * BN;
                for (int kb = k0; kb < k1; kb++) {
                    if (issued >= S &&
                        !tc::mbar_wait(empty0 + 8u * st.idx, st.phase ^ 1u, abort, kWaitTimeoutNs)) {
                        raise_error(abort);
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8u * st.idx;
                    tc::mbar_arrive_expect_tx(fb, C::kW8Bytes + C::kXBytes);
                    const uint32_t wdst = sw_base + st.idx * C::kW8Bytes;
                    const uint32_t xdst = sx_base + st.idx * C::kXBytes;
#pragma unroll
                    for (int h = 0; h < C::kWBoxes; h++)
                        tc::tma_load_2d(wdst + h * (kTileRows * 128), &tmW, kb * BK + h * 128, row0, fb);
#pragma unroll
                    for (int h = 0; h < C::kXBoxes; h++)
                        tc::tma_load_2d(xdst + h * C::kXBoxBytes, &tmX, kb * BK + h * 64, m0, fb);
                    issued++;
                    st.next(S);
                }
            }
            if (*abort) {
                // drain: every copy this CTA issued lands before the CTA exits
                const int zero = 0;
                Ring d;
                for (int q = 0; q < issued; q++, d.next(S))
                    if (q + S >= issued) tc::mbar_wait(full0 + 8u * d.idx, d.phase, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::make_idesc_f16_f32(kTileRows, BN);
            Ring st, sa;
            int seg = 0, t, k0, k1;
            SegIter it(u_begin, u_end, p.kbpt);
            bool ok = true;
            const uint64_t bdesc0 = tc::make_sw128_kmajor_desc(tc::smem_u32(sX));
            while (ok && it.next(t, k0, k1)) {
                const int ab = seg & 1, use = seg >> 1;
                if (use > 0 &&
                    !tc::mbar_wait(accempty0 + 8u * ab, (uint32_t)((use - 1) & 1), abort, kWaitTimeoutNs)) {
                    raise_error(abort);
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem + ab * C::kDCols;
                for (int kb = k0; kb < k1; kb++) {
                    if (!tc::mbar_wait(full0 + 8u * st.idx, st.phase, abort, kWaitTimeoutNs) ||
                        !tc::mbar_wait(afull0 + 8u * sa.idx, sa.phase, abort, kWaitTimeoutNs)) {
                        raise_error(abort);
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t a_base = tmem + C::kACol + sa.idx * C::kACols;
                    // descriptor start address advances in 16-byte units
                    const uint64_t b_stage = bdesc0 + (uint64_t)((st.idx * C::kXBytes) >> 4);
#pragma unroll
                    for (int j = 0; j < BK / 16; j++)
                        tc::mma_f16_ts(d_tmem, a_base + j * 8,
                                       b_stage + (uint64_t)(((j >> 2) * C::kXBoxBytes + (j & 3) * 32) >> 4), idesc,
                                       (kb != k0 || j != 0) ? 1u : 0u);
                    tc::mma_commit(empty0 + 8u * st.idx);
                    tc::mma_commit(aempty0 + 8u * sa.idx);
                    st.next(S);
                    sa.next(SA);
                }
                if (!ok) break;
                tc::mma_commit(accfull0 + 8u * ab);
                seg++;
            }
            if (*abort) {
                const int zero = 0;
                tc::mma_commit(drainbar);  // MMAs in flight finish before TMEM is freed
                tc::mbar_wait(drainbar, 0, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp < kFirstEpi) {
        // ------------------------------------------------------------ dequantize into TMEM
        const int group = (warp - kFirstConv) >> 2;  // 0 or 1: alternate stages
        const int q = warp & 3;                       // TMEM lane quadrant this warp may access
        const int r = q * 32 + lane;
        const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
        const int sw = r & 7;  // 128-byte swizzle: 16-byte chunk j of row r sits at chunk j ^ (r & 7)
        Ring st, sa;
        int g = 0;
        int t, k0, k1;
        SegIter it(u_begin, u_end, p.kbpt);
        bool ok = true;
        while (ok && it.next(t, k0, k1)) {
            for (int kb = k0; kb < k1; kb++, g++, st.next(S), sa.next(SA)) {
                if ((g & 1) != group) continue;
                ok = __all_sync(0xffffffffu, tc::mbar_wait(full0 + 8u * st.idx, st.phase, abort, kWaitTimeoutNs));
                if (!ok) break;
                if (g >= SA) {
                    ok = __all_sync(0xffffffffu,
                                    tc::mbar_wait(aempty0 + 8u * sa.idx, sa.phase ^ 1u, abort, kWaitTimeoutNs));
                    if (!ok) break;
                }
                tc::tc_fence_after();
                const unsigned char* rowp = sW8 + st.idx * C::kW8Bytes + r * 128;
                const uint32_t a_col = tmem + t_lane + C::kACol + sa.idx * C::kACols;
#pragma unroll
                for (int h = 0; h < C::kWBoxes; h++) {
                    // 128 int8 of this row -> 64 packed half2 -> TMEM columns [64h, 64h + 64)
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        uint4 v[4];
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            v[j] = *reinterpret_cast<const uint4*>(rowp + h * (kTileRows * 128) +
                                                                   (((half * 4 + j) ^ sw) << 4));
                        uint32_t hh[32];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            tc::i8x4_to_h2x2(v[j].x, hh[8 * j + 0], hh[8 * j + 1]);
                            tc::i8x4_to_h2x2(v[j].y, hh[8 * j + 2], hh[8 * j + 3]);
                            tc::i8x4_to_h2x2(v[j].z, hh[8 * j + 4], hh[8 * j + 5]);
                            tc::i8x4_to_h2x2(v[j].w, hh[8 * j + 6], hh[8 * j + 7]);
                        }
                        tc::tmem_st_32x32b_x32(a_col + h * 64 + half * 32, hh);
                    }
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(afull0 + 8u * sa.idx);
            }
        }
        if (!ok) raise_error(abort);
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
        const int etid = threadIdx.x - kFirstEpi * 32;  // 0..127
        int seg = 0, t, k0, k1;
        SegIter it(u_begin, u_end, p.kbpt);
        bool ok = true;
        while (it.next(t, k0, k1)) {
            const int ab = seg & 1, use = seg >> 1;
            ok = __all_sync(0xffffffffu, tc::mbar_wait(accfull0 + 8u * ab, (uint32_t)(use & 1), abort, kWaitTimeoutNs));
            if (!ok) break;
            tc::tc_fence_after();
            const int row0 = (t % p.tiles_n) * kTileRows;
            const int m0 = (t / p.tiles_n) * BN;
            const int mvalid = min(BN, p.M - m0);
            const int n = row0 + r;
            const bool nv = n < p.N;
            const float scale = nv ? p.scales[n] : 0.0f;
            const float bias = (nv && p.bias) ? p.bias[n] : 0.0f;
            const uint32_t d_tmem = tmem + t_lane + ab * C::kDCols;
            const bool whole = (k0 == 0 && k1 == p.kbpt);
            const int slot = (seg == 0) ? 2 * cta : 2 * cta + 1;
            // workspace slot layout: [128 rows][BN tokens] fp32, so a row's partials are contiguous
            float* wrow = p.ws + ((size_t)slot * kTileRows + r) * BN;
            OT* orow = reinterpret_cast<OT*>(p.out) + (size_t)m0 * p.N + n;
            const OT* rrow = p.res ? reinterpret_cast<const OT*>(p.res) + (size_t)m0 * p.N + n : nullptr;
#pragma unroll 1
            for (int c0 = 0; c0 < mvalid; c0 += 16) {
                uint32_t d[16];
                __syncwarp();
                tc::tmem_ld_32x32b_x16(d_tmem + c0, d);
                tc::tmem_ld_wait();
                if (whole) {
                    if (nv) epi_chunk<OT>(orow + (size_t)c0 * p.N, rrow ? rrow + (size_t)c0 * p.N : nullptr, p.N,
                                          min(16, mvalid - c0), d, scale, bias, p.bias != nullptr);
                } else {
                    float4* w4 = reinterpret_cast<float4*>(wrow + c0);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        __stcg(w4 + i, make_float4(__uint_as_float(d[4 * i]), __uint_as_float(d[4 * i + 1]),
                                                   __uint_as_float(d[4 * i + 2]), __uint_as_float(d[4 * i + 3])));
                }
            }
            // accumulator drained: the MMA may reuse it
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(accempty0 + 8u * ab);
            if (!whole) {
                // stream-K fixup: the last of the tile's pieces to arrive reduces them in K order
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                const long long tb = (long long)t * p.kbpt;
                const int j0 = cta_of_unit(tb, p.units, G);
                const int j1 = cta_of_unit(tb + p.kbpt - 1, p.units, G);
                if (etid == 0) {
                    const int prev = atomicAdd(p.counters + t, 1);
                    *last_flag = (prev == j1 - j0) ? 1 : 0;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (*last_flag) {
                    __threadfence();
#pragma unroll 1
                    for (int c0 = 0; c0 < mvalid; c0 += 16) {
                        float acc[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) acc[i] = 0.0f;
#pragma unroll 1
                        for (int j = j0; j <= j1; j += 2) {
                            // two pieces in flight; summed in piece (= K) order
                            const int sa_ = (unit_begin(j, p.units, G) >= tb) ? 2 * j : 2 * j + 1;
                            const float4* pa = reinterpret_cast<const float4*>(
                                p.ws + ((size_t)sa_ * kTileRows + r) * BN + c0);
                            float4 va[4], vb[4];
#pragma unroll
                            for (int i = 0; i < 4; i++) va[i] = __ldcg(pa + i);
                            const bool two = j + 1 <= j1;
                            if (two) {
                                const int sb_ = (unit_begin(j + 1, p.units, G) >= tb) ? 2 * (j + 1) : 2 * (j + 1) + 1;
                                const float4* pb = reinterpret_cast<const float4*>(
                                    p.ws + ((size_t)sb_ * kTileRows + r) * BN + c0);
#pragma unroll
                                for (int i = 0; i < 4; i++) vb[i] = __ldcg(pb + i);
                            }
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                acc[4 * i] += va[i].x;
                                acc[4 * i + 1] += va[i].y;
                                acc[4 * i + 2] += va[i].z;
                                acc[4 * i + 3] += va[i].w;
                            }
                            if (two) {
#pragma unroll
                                for (int i = 0; i < 4; i++) {
                                    acc[4 * i] += vb[i].x;
                                    acc[4 * i + 1] += vb[i].y;
                                    acc[4 * i + 2] += vb[i].z;
                                    acc[4 * i + 3] += vb[i].w;
                                }
                            }
                        }
                        uint32_t d[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) d[i] = __float_as_uint(acc[i]);
                        if (nv)
                            epi_chunk<OT>(orow + (size_t)c0 * p.N, rrow ? rrow + (size_t)c0 * p.N : nullptr, p.N,
                                          min(16, mvalid - c0), d, scale, bias, p.bias != nullptr);
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (etid == 0) p.counters[t] = 0;  // ready for the next launch
                }
            }
            seg++;
        }
        if (!ok) raise_error(abort);
        pdl_launch_dependents();
    }

    // ---------------------------------------------------------------- teardown
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ----------------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
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

// Weight map: int8 [N, K] in [128 rows x 128 B] boxes; activation map: fp16 [M, K]
// in [BN rows x 64] boxes; both 128-byte swizzled, out-of-range rows/columns read 0.
bool make_maps(const LinearArgs& a, int BN, CUtensorMap* mw, CUtensorMap* mx)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint32_t es[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.N};
        const cuuint64_t strides[1] = {(cuuint64_t)a.K};
        const cuuint32_t box[2] = {128u, (cuuint32_t)kTileRows};
        if (enc(mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(a.w), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
        const cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
        const cuuint32_t box[2] = {64u, (cuuint32_t)BN};
        if (enc(mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

int pick_bn(size_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }
int pick_bk(int BN) { return BN <= 32 ? 256 : 128; }

template <int BN, int BK, int S, int SA, typename OT>
cudaError_t launch_cfg(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    using C = SkCfg<BN, BK, S, SA>;
    CUtensorMap mw, mx;
    if (!make_maps(a, BN, &mw, &mx)) return cudaErrorInvalidValue;
    auto kern = q8_gemm_sk_kernel<BN, BK, S, SA, OT>;
    static thread_local bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    SkParams p;
    p.scales = a.scales;
    p.bias = a.bias;
    p.res = a.res;
    p.out = a.out;
    p.M = (int)a.M;
    p.N = (int)a.N;
    p.K = (int)a.K;
    p.kbpt = (int)((a.K + BK - 1) / BK);
    p.tiles_n = (int)((a.N + kTileRows - 1) / kTileRows);
    const long long tiles = (long long)p.tiles_n * (long long)((a.M + BN - 1) / BN);
    p.units = tiles * p.kbpt;
    const int G = (int)((p.units < num_sms) ? p.units : num_sms);
    if ((long long)scratch.ws_floats < 2LL * G * BN * kTileRows || (long long)scratch.counters < tiles)
        return cudaErrorMemoryAllocation;
    p.ws = scratch.ws;
    p.counters = scratch.counter_ptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, mw, mx, p);
    if (e == cudaSuccess) note_launch();
    return e;
}

template <typename OT>
cudaError_t launch_typed(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    switch (pick_bn(a.M)) {
        case 16: return launch_cfg<16, 256, 5, 2, OT>(a, num_sms, scratch, stream);
        case 32: return launch_cfg<32, 256, 4, 2, OT>(a, num_sms, scratch, stream);
        case 64: return launch_cfg<64, 128, 6, 3, OT>(a, num_sms, scratch, stream);
        default: return launch_cfg<128, 128, 4, 3, OT>(a, num_sms, scratch, stream);
    }
}

}  // namespace

bool gemm_tc_supports(const LinearArgs& a)
{
    return a.in_dtype == kF16 && a.K % 16 == 0 && a.K >= 16 && ((uintptr_t)a.w % 16) == 0 &&
           ((uintptr_t)a.x % 16) == 0 && a.N >= 1 && a.M >= 1 && a.N <= (size_t)INT32_MAX &&
           a.M <= (size_t)INT32_MAX && encode_fn() != nullptr;
}

void gemm_tc_scratch_need(const LinearArgs& a, int num_sms, size_t* ws_floats, size_t* counters)
{
    const int BN = pick_bn(a.M);
    const int BK = pick_bk(BN);
    const long long tiles_n = (long long)((a.N + kTileRows - 1) / kTileRows);
    const long long tiles = tiles_n * (long long)((a.M + BN - 1) / BN);
    const long long units = tiles * (long long)((a.K + BK - 1) / BK);
    const long long G = units < num_sms ? units : num_sms;
    *ws_floats = (size_t)(2 * G * BN * kTileRows);
    *counters = (size_t)tiles;
}

cudaError_t launch_q8_gemm_tc(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    if (!gemm_tc_supports(a)) return cudaErrorNotSupported;
    return a.out_dtype == kF16 ? launch_typed<__half>(a, num_sms, scratch, stream)
                               : launch_typed<float>(a, num_sms, scratch, stream);
}

cudaError_t read_kernel_error(int* code, bool clear)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(int));
    if (e != cudaSuccess) return e;
    *code = v;
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(int));
    }
    return e;
}

}  // namespace b200q8
