// q8_gemm_tc.cu -- int8-weight x fp16-activation GEMM on the 5th-gen tensor cores.
//
// out[m, n] = (sum_k x[m, k] * float(W[n, k])) * scales[n] + bias[n] (+ res[m, n])
// (semantics of vvllm BackendCPU::linear_q8 / linear_q8_add,
//  src/backend/backend_naive.cc:155-291 and :322-335, with fp16 activations.)
//
// Tiling ("swap-AB"): a tile is 128 weight rows (UMMA M) x BN tokens (UMMA N,
// 16..256), so one kernel serves M = 1 decode through M >= 512 prefill.  K
// runs in BK-wide pipeline stages.  One tcgen05.mma takes a fixed ~45-70
// cycles to issue from the single issuing thread, so wide prefill tiles use
// UMMA N = 256 (128 cycles of tensor work per instruction) to keep the tensor
// pipe, not the issuing thread, the limit.
//
// Persistent stream-K schedule: the (tile, K-stage) units of the whole problem
// are laid out tile-major and cut into gridDim.x equal contiguous ranges, one
// per CTA (one CTA per SM).  A CTA works on a few whole tiles plus at most two
// partial tiles at the ends of its range; skinny shapes (few tiles, long K)
// still keep every SM busy, and no wave is left half-empty.  A tile split over
// several CTAs is finished deterministically by the piece that arrives last:
// a piece that finds every other piece already arrived keeps its accumulator in
// tensor memory and skips its workspace round trip; otherwise it stores its
// fp32 partial to a workspace slot (float4-interleaved by row, so a warp's
// stores and loads are contiguous) and bumps the tile's counter.  The last
// piece sums all pieces in K order (its own straight from TMEM), applies the
// epilogue and resets the counter.  No CTA ever waits on another.
//
// Warp roles (14 warps, 15 with a second MMA-issuing thread):
//   0      TMA producer: int8 weight tile [128 x BK] as swizzled boxes of
//          [128 rows x min(BK,128) B] (64- or 128-byte swizzle) and fp16
//          activation tile [BN x BK] as 128-byte-swizzled [BN x 64] boxes into
//          an S-stage shared-memory ring, completing on mbarriers.  The weight
//          boxes of the first stages are requested before the programmatic
//          dependency wait (weights do not depend on the previous kernel);
//   1      TMEM allocator; one thread issues tcgen05.mma.kind::f16
//          [D_tmem], [A_tmem], B_desc into one of kAcc TMEM accumulators, and
//          tcgen05.commit frees the stages;
//   2..9   dequantizers in two groups taking alternate stages: a thread owns
//          one weight row (= TMEM lane), reads its BK int8 from shared memory
//          (conflict-free under the swizzle), converts them exactly to fp16
//          (exponent-bias trick) and tcgen05.st's them into an SA-stage TMEM
//          ring -- the MMA's A operand lives in tensor memory, so no fp16
//          weight copy ever touches shared memory or HBM;
//   10..13 epilogue: tcgen05.ld of the finished accumulator, then
//          v = acc * scale[n] (+ bias[n]) (+ res[m, n]) stored as fp16/fp32,
//          or the stream-K partial/fixup path;
//   14     (two-issuer layouts) a second thread issuing the MMAs of every other
//          stage into its own accumulator; the epilogue adds the two.
// Every mbarrier wait is bounded (wall clock); a timeout sets a device error
// word, drains in-flight copies and MMAs, frees TMEM and returns.  No TMA
// multicast and no thread-block clusters are used.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_utils.cuh"
#include "tmap.cuh"

namespace b200q8 {

__device__ int g_kernel_error;  // bit 0: a bounded wait timed out in the tensor-core GEMM

// Per-CTA phase timestamps, compiled in only with -DB200Q8_TRACE (a profiling build; the
// product build has none): [cta][slot] = %globaltimer at slot 0, SM cycles since slot 0 after.
#ifdef B200Q8_TRACE
__device__ unsigned long long g_gemm_trace[1024][8];
#define GEMM_TRACE(slot, t0)                                                                     \
    do {                                                                                         \
        if (blockIdx.x < 1024)                                                                   \
            g_gemm_trace[blockIdx.x][slot] = (slot) == 0 ? tc::globaltimer_ns() : clock64() - (t0); \
    } while (0)
// Per-CTA role counters of the profiling build: [cta][slot] = SM cycles a role spent waiting on
// a barrier, or in its whole loop (slots listed with b200q8_trace_gemm_roles).
__device__ unsigned long long g_gemm_role[1024][16];
#define ROLE_TRACE(slot, v)                                                                        \
    do {                                                                                           \
        if (blockIdx.x < 1024) g_gemm_role[blockIdx.x][slot] = (unsigned long long)(v);           \
    } while (0)
#else
#define GEMM_TRACE(slot, t0) \
    do {                     \
    } while (0)
#define ROLE_TRACE(slot, v) \
    do {                    \
    } while (0)
#endif

namespace {

constexpr int kTileRows = 128;  // weight rows per tile (UMMA M)
constexpr int kFirstConv = 2, kFirstEpi = 10;
constexpr int kSecondIssuer = 14;  // warp of the second MMA-issuing thread (two-issuer layouts)
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s: far above any legitimate wait

// Bounded mbarrier wait; the profiling build adds the SM cycles it took to `acc`.
__device__ __forceinline__ bool timed_wait(uint32_t bar, uint32_t parity, const volatile int* abort, long long& acc)
{
#ifdef B200Q8_TRACE
    const long long t = clock64();
    const bool r = tc::mbar_wait(bar, parity, abort, kWaitTimeoutNs);
    acc += clock64() - t;
    return r;
#else
    (void)acc;
    return tc::mbar_wait(bar, parity, abort, kWaitTimeoutNs);
#endif
}

struct SkParams {
    const float* scales;
    const float* bias;
    const void* res;
    void* out;
    float* ws;          // [2 * gridDim.x] slots of [BN / 4][128][4] fp32 partial accumulators
    int* counters;      // [tiles] arrival counters, zero between launches
    int M, N, K;
    int kbpt;           // K stages per tile
    int tiles_n;        // weight-row tiles
    long long units;    // tiles * kbpt
    int tma_out;        // outputs leave by TMA store (16-byte aligned rows), else direct stores
    int w_evict_first;  // weight tiles are read by one token tile only: L2 evict-first
};

template <int BN, int BK, int S, int SA, int NI>
struct SkCfg {
    static constexpr int kWBoxW = BK < 128 ? BK : 128;  // bytes per weight-box row
    static constexpr int kWBoxes = BK / kWBoxW;
    static constexpr int kWBoxBytes = kTileRows * kWBoxW;
    static constexpr int kW8Bytes = kTileRows * BK;
    static constexpr int kXBoxes = BK / 64;             // [BN rows x 64 fp16] boxes per stage
    static constexpr int kXBoxBytes = BN * 128;
    static constexpr int kXBytes = kXBoxes * kXBoxBytes;
    static constexpr int kACols = BK / 2;               // TMEM columns of one A stage
    static constexpr int kDCols = (BN + 31) / 32 * 32;  // one accumulator, 32-column aligned
    // NI issuing threads, each with its own accumulator per buffer (they take alternate K-stages;
    // the epilogue adds the two)
    static constexpr int kAcc = (2 * NI * kDCols + SA * kACols <= 512) ? 2 : 1;
    static constexpr int kACol = kAcc * NI * kDCols;
    static constexpr int kColsNeeded = kACol + SA * kACols;
    static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                     : kColsNeeded <= 256 ? 256 : 512;
    static constexpr int kChunk = BN < 32 ? BN : 32;    // accumulator columns per tcgen05.ld in the epilogue
    // As many A stages in TMEM as shared-memory stages: they advance together, and one commit per
    // stage frees both (the dequantizers wait on the stage's empty barrier).  A commit costs the
    // issuing thread about as much as several MMAs.
    static constexpr bool kOneCommit = (S == SA);
    static constexpr int kNumBars = 2 * S + 2 * SA + 2 * kAcc + 3;  // + accfull/accempty[kAcc], drain x2, fixup
    static constexpr int kWarps = 14 + (NI - 1);
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kOutBufBytes = kChunk * kTileRows * 4;  // one staged chunk (fp32 or fp16 outputs, fp32 partials)
    static constexpr int kSmemBytes = 1024 + S * (kW8Bytes + kXBytes) + 2 * kOutBufBytes + kNumBars * 8 + 16;
    static_assert(kColsNeeded <= 512, "TMEM overflow");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M = 128");
    static_assert(BK == 64 || BK % 128 == 0, "stage K is one 64-byte box or whole 128-byte boxes");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kXBoxBytes % 1024 == 0 && kW8Bytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(BN % kChunk == 0, "epilogue chunks tile the accumulator");
    static_assert(NI == 1 || NI == 2, "one or two issuing threads");
};

// Byte offset of 16-byte chunk c of row r inside a weight box, under the box's
// TMA swizzle (128-byte rows: chunk ^= r & 7; 64-byte rows: chunk ^= (r >> 1) & 3).
template <int kBoxW>
__device__ __forceinline__ int wchunk(int r, int c)
{
    if constexpr (kBoxW == 128)
        return r * 128 + ((c ^ (r & 7)) << 4);
    else
        return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
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

// CH accumulator columns of this thread's TMEM lane, starting at column `col`.
template <int CH>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t col, float (&v)[CH]);

// The same columns summed over the issuers' accumulators: `col`, and `col + second` when second
// is non-zero (the second issuer's accumulator, its stages' partial sum).
template <int CH>
__device__ __forceinline__ void tmem_ld_acc(uint32_t col, int second, float (&v)[CH])
{
    tmem_ld_chunk<CH>(col, v);
    if (second) {
        float w[CH];
        tmem_ld_chunk<CH>(col + (uint32_t)second, w);
#pragma unroll
        for (int i = 0; i < CH; i++) v[i] += w[i];
    }
}

template <int CH>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t col, float (&v)[CH])
{
    if constexpr (CH == 32) {
        uint32_t d[32];
        tc::tmem_ld_32x32b_x32(col, d);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(d[i]);
    } else {
        static_assert(CH == 16, "chunk of 16 or 32 columns");
        uint32_t d[16];
        tc::tmem_ld_32x32b_x16(col, d);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = __uint_as_float(d[i]);
    }
}

template <int BN, int BK, int S, int SA, int NI, typename OT>
__global__ void __launch_bounds__(SkCfg<BN, BK, S, SA, NI>::kThreads, 1)
    q8_gemm_sk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const __grid_constant__ CUtensorMap tmO, const SkParams p)
{
    using C = SkCfg<BN, BK, S, SA, NI>;
    constexpr int CH = C::kChunk;
    constexpr int kRedSlotBytes = kTileRows * CH * 4;  // one piece's CH-column chunk
    constexpr int kRedSlots = S * (C::kW8Bytes + C::kXBytes) / kRedSlotBytes;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* sW8 = smem;
    unsigned char* sX = smem + S * C::kW8Bytes;
    unsigned char* sOut = sX + S * C::kXBytes;  // two output staging buffers
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + 2 * C::kOutBufBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_holder + 2);  // [2]: first / last segment

    const uint32_t bar0 = tc::smem_u32(bars);
    const uint32_t full0 = bar0, empty0 = bar0 + 8u * S, afull0 = bar0 + 16u * S,
                   aempty0 = bar0 + 16u * S + 8u * SA, accfull0 = bar0 + 16u * S + 16u * SA,
                   accempty0 = accfull0 + 8u * C::kAcc, drainbar = accempty0 + 8u * C::kAcc,
                   redbar = drainbar + 8u, drainbar2 = redbar + 8u;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int cta = blockIdx.x;
    const long long u_begin = unit_begin(cta, p.units, G), u_end = unit_begin(cta + 1, p.units, G);
    const uint32_t sw_base = tc::smem_u32(sW8), sx_base = tc::smem_u32(sX), sout_base = tc::smem_u32(sOut);

    int pre = 0;  // stages whose weight boxes were requested before the dependency wait
    const long long trace_t0 = clock64();
    (void)trace_t0;
    if (threadIdx.x == 0) {
        GEMM_TRACE(0, trace_t0);
        for (int s = 0; s < S; s++) {
            tc::mbar_init(full0 + 8u * s, 1);
            tc::mbar_init(empty0 + 8u * s, 1);
        }
        for (int s = 0; s < SA; s++) {
            tc::mbar_init(afull0 + 8u * s, 4);
            tc::mbar_init(aempty0 + 8u * s, 1);
        }
        for (int b = 0; b < C::kAcc; b++) {
            tc::mbar_init(accfull0 + 8u * b, NI);  // every issuer commits
            tc::mbar_init(accempty0 + 8u * b, 4);
        }
        tc::mbar_init(drainbar, 1);
        tc::mbar_init(redbar, 1);
        tc::mbar_init(drainbar2, 1);
        *abort = 0;
        tc::fence_mbar_init();
        // Weights do not depend on the previous kernel: start streaming them now.
        tc::prefetch_tensormap(&tmW);
        tc::prefetch_tensormap(&tmX);
        tc::prefetch_tensormap(&tmO);
        int t, k0, k1;
        SegIter it(u_begin, u_end, p.kbpt);
        while (pre < S && it.next(t, k0, k1)) {
            const int row0 = (t % p.tiles_n) * kTileRows;
            for (int kb = k0; kb < k1 && pre < S; kb++, pre++) {
                const uint32_t fb = full0 + 8u * pre;
                tc::mbar_arrive_expect_tx(fb, C::kW8Bytes + C::kXBytes);
#pragma unroll
                for (int h = 0; h < C::kWBoxes; h++)
                    tc::tma_load_2d(sw_base + pre * C::kW8Bytes + h * C::kWBoxBytes, &tmW, kb * BK + h * C::kWBoxW,
                                    row0, fb);
            }
        }
    }
    // Activations come from the previous kernel; hold no TMEM while waiting for it.
    pdl_wait();
    if (threadIdx.x == 0) GEMM_TRACE(1, trace_t0);
    __syncwarp();
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_holder), C::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (threadIdx.x == 0) GEMM_TRACE(2, trace_t0);
    // The next kernel may be scheduled now: its CTAs take SMs this grid leaves idle and run their
    // set-up and weight loads; everything they do with this grid's outputs waits in their
    // griddepcontrol.wait, which returns only once this grid has completed.
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            Ring st;
            int issued = 0;
            int t, k0, k1;
            SegIter it(u_begin, u_end, p.kbpt);
            bool ok = true;
            const uint64_t wpol = p.w_evict_first ? tc::l2_policy_evict_first() : tc::l2_policy_evict_normal();
            long long w_empty = 0;
            const long long t_role = clock64();
            while (ok && it.next(t, k0, k1)) {
                const int row0 = (t % p.tiles_n) * kTileRows;
                const int m0 = (t / p.tiles_n) * BN;
                for (int kb = k0; kb < k1; kb++) {
                    const uint32_t fb = full0 + 8u * st.idx;
                    if (issued >= pre) {
                        if (issued >= S && !timed_wait(empty0 + 8u * st.idx, st.phase ^ 1u, abort, w_empty)) {
                            raise_error(abort);
                            ok = false;
                            break;
                        }
                        tc::mbar_arrive_expect_tx(fb, C::kW8Bytes + C::kXBytes);
#pragma unroll
                        for (int h = 0; h < C::kWBoxes; h++)
                            tc::tma_load_2d_hint(sw_base + st.idx * C::kW8Bytes + h * C::kWBoxBytes, &tmW,
                                                 kb * BK + h * C::kWBoxW, row0, fb, wpol);
                    }
                    const uint32_t xdst = sx_base + st.idx * C::kXBytes;
#pragma unroll
                    for (int h = 0; h < C::kXBoxes; h++)
                        tc::tma_load_2d(xdst + h * C::kXBoxBytes, &tmX, kb * BK + h * 64, m0, fb);
                    issued++;
                    st.next(S);
                }
            }
            ROLE_TRACE(11, w_empty);
            ROLE_TRACE(12, clock64() - t_role);
            if (*abort) {
                // drain: every copy this CTA issued lands before the CTA exits
                const int zero = 0;
                Ring d;
                const int requested = issued > pre ? issued : pre;
                for (int q = 0; q < requested; q++, d.next(S))
                    if (q + S >= requested) tc::mbar_wait(full0 + 8u * d.idx, d.phase, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp == 1 || (NI == 2 && warp == kSecondIssuer)) {
        // ------------------------------------------------------------ MMA issuers
        // With two issuing threads, issuer i takes the stages kb - k0 = i, i + 2, ... of each
        // segment into its own accumulator (the epilogue adds them): one thread alone issues a
        // tcgen05.mma only every ~60-120 cycles whatever N, two keep the tensor pipe busier.
        const int issuer = warp == 1 ? 0 : 1;
        if (lane == 0) {
            constexpr uint32_t idesc = tc::make_idesc_f16_f32(kTileRows, BN);
            Ring st, sa;
            int seg = 0, t, k0, k1;
            SegIter it(u_begin, u_end, p.kbpt);
            bool ok = true;
            const uint64_t bdesc0 = tc::make_sw128_kmajor_desc(tc::smem_u32(sX));
            long long w_full = 0, w_afull = 0, w_acc = 0, nstages = 0;
            const long long t_role = clock64();
            while (ok && it.next(t, k0, k1)) {
                const int ab = seg % C::kAcc, use = seg / C::kAcc;
                if (use > 0 && !timed_wait(accempty0 + 8u * ab, (uint32_t)((use - 1) & 1), abort, w_acc)) {
                    raise_error(abort);
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem + (ab * NI + issuer) * C::kDCols;
                for (int kb = k0; kb < k1; kb++, st.next(S), sa.next(SA)) {
                    if ((kb - k0) % NI != issuer) continue;
                    nstages++;
                    if (!timed_wait(full0 + 8u * st.idx, st.phase, abort, w_full) ||
                        !timed_wait(afull0 + 8u * sa.idx, sa.phase, abort, w_afull)) {
                        raise_error(abort);
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    if (issuer == 0 && seg == 0 && kb == k0) GEMM_TRACE(3, trace_t0);
                    const uint32_t a_base = tmem + C::kACol + sa.idx * C::kACols;
                    // descriptor start address advances in 16-byte units
                    const uint64_t b_stage = bdesc0 + (uint64_t)((st.idx * C::kXBytes) >> 4);
#pragma unroll
                    for (int j = 0; j < BK / 16; j++)
                        tc::mma_f16_ts(d_tmem, a_base + j * 8,
                                       b_stage + (uint64_t)(((j >> 2) * C::kXBoxBytes + (j & 3) * 32) >> 4), idesc,
                                       (kb != k0 + issuer || j != 0) ? 1u : 0u);
                    tc::mma_commit(empty0 + 8u * st.idx);
                    if constexpr (!C::kOneCommit) tc::mma_commit(aempty0 + 8u * sa.idx);
                }
                if (!ok) break;
                // an issuer with no stage in this segment commits too (it arrives at once)
                tc::mma_commit(accfull0 + 8u * ab);
                if (issuer == 0) GEMM_TRACE(4, trace_t0);
                seg++;
            }
            if (issuer == 0) {
                ROLE_TRACE(0, w_full);
                ROLE_TRACE(1, w_afull);
                ROLE_TRACE(2, w_acc);
                ROLE_TRACE(3, clock64() - t_role);
                ROLE_TRACE(4, nstages);
            }
            if (*abort) {
                const int zero = 0;
                const uint32_t db = issuer == 0 ? drainbar : drainbar2;
                tc::mma_commit(db);  // this thread's MMAs in flight finish before TMEM is freed
                tc::mbar_wait(db, 0, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp >= kFirstConv && warp < kFirstEpi) {
        // ------------------------------------------------------------ dequantize into TMEM
        const int group = (warp - kFirstConv) >> 2;  // 0 or 1: alternate stages
        const int q = warp & 3;                       // TMEM lane quadrant this warp may access
        const int r = q * 32 + lane;
        const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
        Ring st, sa;
        int g = 0;
        int t, k0, k1;
        SegIter it(u_begin, u_end, p.kbpt);
        bool ok = true;
        long long w_full = 0, w_aempty = 0;
        const long long t_role = clock64();
        while (ok && it.next(t, k0, k1)) {
            for (int kb = k0; kb < k1; kb++, g++, st.next(S), sa.next(SA)) {
                if ((g & 1) != group) continue;
                ok = __all_sync(0xffffffffu, timed_wait(full0 + 8u * st.idx, st.phase, abort, w_full));
                if (!ok) break;
                if (g >= SA) {  // the MMAs that read this A stage last are done
                    const uint32_t free_bar = C::kOneCommit ? empty0 + 8u * st.idx : aempty0 + 8u * sa.idx;
                    ok = __all_sync(0xffffffffu, timed_wait(free_bar, sa.phase ^ 1u, abort, w_aempty));
                    if (!ok) break;
                }
                tc::tc_fence_after();
                const unsigned char* wst = sW8 + st.idx * C::kW8Bytes;
                const uint32_t a_col = tmem + t_lane + C::kACol + sa.idx * C::kACols;
#pragma unroll
                for (int h = 0; h < C::kWBoxes; h++) {
                    // 64 int8 of this row -> 32 packed half2 -> 32 TMEM columns
#pragma unroll
                    for (int half = 0; half < C::kWBoxW / 64; half++) {
                        uint4 v[4];
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            v[j] = *reinterpret_cast<const uint4*>(wst + h * C::kWBoxBytes +
                                                                   wchunk<C::kWBoxW>(r, half * 4 + j));
                        uint32_t hh[32];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            tc::i8x4_to_h2x2(v[j].x, hh[8 * j + 0], hh[8 * j + 1]);
                            tc::i8x4_to_h2x2(v[j].y, hh[8 * j + 2], hh[8 * j + 3]);
                            tc::i8x4_to_h2x2(v[j].z, hh[8 * j + 4], hh[8 * j + 5]);
                            tc::i8x4_to_h2x2(v[j].w, hh[8 * j + 6], hh[8 * j + 7]);
                        }
                        tc::tmem_st_32x32b_x32(a_col + h * (C::kWBoxW / 2) + half * 32, hh);
                    }
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(afull0 + 8u * sa.idx);
            }
        }
        if (lane == 0 && q == 2) {  // warps 2 and 6: one of each group
            ROLE_TRACE(5 + 3 * group, w_full);
            ROLE_TRACE(6 + 3 * group, w_aempty);
            ROLE_TRACE(7 + 3 * group, clock64() - t_role);
        }
        if (!ok) raise_error(abort);
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
        const int etid = threadIdx.x - kFirstEpi * 32;  // 0..127
        const bool has_bias = p.bias != nullptr;
        uint32_t redphase = 0;
        int nstore = 0;  // chunks staged so far (selects the staging buffer)
        int seg = 0, t, k0, k1;
        SegIter it(u_begin, u_end, p.kbpt);
        bool ok = true;
        long long w_accfull = 0;
        const long long t_role = clock64();
        // One chunk of outputs (tokens m .. m + CH - 1 of this thread's channel) goes
        // through a staging buffer in shared memory and leaves with one TMA store;
        // rows and columns beyond the output's extent are clipped by the store.
        // One chunk of outputs (tokens m .. m + cnt - 1 of this thread's channel): the epilogue
        // math runs branch-free over the whole chunk (warp-uniform choices are made once per
        // chunk; per-element conditions in an unrolled loop cost a reconvergence point each),
        // then the chunk goes through a staging buffer in shared memory and leaves with one
        // TMA store, which clips rows and columns beyond the output's extent.
        auto out_chunk = [&](const float (&v)[CH], int n0, int m, int cnt, float scale, float bias, const OT* rres) {
            float y[CH];
            if (has_bias) {
#pragma unroll
                for (int i = 0; i < CH; i++) y[i] = __fadd_rn(__fmul_rn(v[i], scale), bias);
            } else {
#pragma unroll
                for (int i = 0; i < CH; i++) y[i] = __fmul_rn(v[i], scale);
            }
            if (rres) {
                // rows past the output's end re-read its last row (in range) and are not stored
#pragma unroll
                for (int i = 0; i < CH; i++) {
                    const float rv = load_as_f32<OT>(rres + (size_t)min(i, cnt - 1) * p.N);
                    y[i] = i < cnt ? __fadd_rn(y[i], rv) : y[i];
                }
            }
            if (!p.tma_out) {  // output rows not 16-byte aligned: direct stores
                if (n0 + r < p.N) {
                    OT* o = reinterpret_cast<OT*>(p.out) + (size_t)m * p.N + n0 + r;
#pragma unroll
                    for (int i = 0; i < CH; i++)
                        if (i < cnt) store_from_f32<OT>(o + (size_t)i * p.N, y[i]);
                }
                return;
            }
            const int b = nstore & 1;
            if (etid == 0) tc::bulk_wait_read<1>();  // the store that used buffer b is done reading it
            asm volatile("bar.sync 1, 128;" ::: "memory");
            OT* buf = reinterpret_cast<OT*>(sOut + b * C::kOutBufBytes);
#pragma unroll
            for (int i = 0; i < CH; i++) store_from_f32<OT>(buf + i * kTileRows + r, y[i]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (etid == 0) {
                tc::tma_store_2d(&tmO, sout_base + b * C::kOutBufBytes, n0, m);
                tc::bulk_commit();
            }
            nstore++;
        };
        const float4* stage = reinterpret_cast<const float4*>(smem);  // staged pieces (mode 2)
        // Fixup piece j's slot: CTA j's first-segment slot (2j) if its range starts inside this
        // tile, else its last-segment slot (2j + 1).
        auto piece_slot = [&](int j, long long tb) -> const float* {
            const int sj = (unit_begin(j, p.units, G) >= tb) ? 2 * j : 2 * j + 1;
            return p.ws + (size_t)sj * kTileRows * BN;
        };
        while (ok && it.next(t, k0, k1)) {
            const int ab = seg % C::kAcc, use = seg / C::kAcc;
            const int row0 = (t % p.tiles_n) * kTileRows;
            const int m0 = (t / p.tiles_n) * BN;
            const int mvalid = min(BN, p.M - m0);
            const int nchunks = (mvalid + CH - 1) / CH;
            const int n = row0 + r;
            const bool nv = n < p.N;
            const float scale = nv ? p.scales[n] : 0.0f;
            const float bias = (nv && has_bias) ? p.bias[n] : 0.0f;
            const OT* rrow = (p.res && nv) ? reinterpret_cast<const OT*>(p.res) + (size_t)m0 * p.N + n : nullptr;
            // one verdict for all four epilogue warps: named barrier 1 follows
            ok = tc::bar_all<1, 128>(timed_wait(accfull0 + 8u * ab, (uint32_t)(use & 1), abort, w_accfull));
            if (!ok) break;
            if (etid == 0 && seg == 0) GEMM_TRACE(5, trace_t0);
            tc::tc_fence_after();
            const uint32_t d_tmem = tmem + t_lane + ab * NI * C::kDCols;
            // the second issuer's accumulator holds stages only if the segment has two or more
            const bool two = NI == 2 && k1 - k0 >= 2;
            const long long tb = (long long)t * p.kbpt;
            const bool whole = (k0 == 0 && k1 == p.kbpt);
            const int j0 = whole ? cta : cta_of_unit(tb, p.units, G);
            const int j1 = whole ? cta : cta_of_unit(tb + p.kbpt - 1, p.units, G);
            const int others = j1 - j0;  // pieces of other CTAs
            const int before = cta - j0;  // of them, those that precede this CTA's piece in K
            volatile int* lf = last_flag + (seg == 0 ? 0 : 1);
            // mode: 0 = write the output, 1 = store this piece's partial, 2 = reduce staged
            // pieces (bulk copies into the idle pipeline smem), 3 = reduce pieces read from
            // the workspace (pipeline still busy).  One loop serves all four, so the store
            // and reduction code is shared and stays warm in the instruction cache.
            int mode = 0;
            if (!whole) {
                if (etid == 0) {
                    int seen;
                    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(p.counters + t) : "memory");
                    *lf = (seen == others) ? 1 : 0;  // every other piece is in already
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                mode = *lf ? 2 : 1;
            }
            for (int pass = 0; pass < 2 && ok; pass++) {
                if (mode == 2) {
                    __threadfence();  // acquire: the other pieces' partials
                    if (!(it.u >= it.end && others <= kRedSlots)) mode = 3;
                }
                const int per_batch = mode == 2 ? kRedSlots / others : nchunks;
                float* my_slot = p.ws + (size_t)(seg == 0 ? 2 * cta : 2 * cta + 1) * kTileRows * BN;
#pragma unroll 1
                for (int cb = 0; cb < nchunks; cb += per_batch) {
                    const int ce = min(nchunks, cb + per_batch);
                    if (mode == 2) {
                        if (etid == 0) {
                            // the batch before was read by every thread (barrier below); order
                            // those reads and the partials' acquire before the copies
                            asm volatile("fence.proxy.async;" ::: "memory");
                            tc::mbar_arrive_expect_tx(redbar, (uint32_t)((ce - cb) * others * kRedSlotBytes));
                            int slot = 0;
                            for (int c = cb; c < ce; c++)
                                for (int j = j0; j <= j1; j++) {
                                    if (j == cta) continue;
                                    tc::bulk_load(sw_base + slot * kRedSlotBytes, piece_slot(j, tb) + (size_t)c * kTileRows * CH,
                                                  kRedSlotBytes, redbar);
                                    slot++;
                                }
                        }
                        ok = tc::bar_all<1, 128>(tc::mbar_wait(redbar, redphase, abort, kWaitTimeoutNs));
                        redphase ^= 1u;
                        if (!ok) {  // let the copies in flight land before the CTA can exit
                            const int zero = 0;
                            tc::mbar_wait(redbar, redphase ^ 1u, &zero, kWaitTimeoutNs);
                            break;
                        }
                    }
#pragma unroll 1
                    for (int c = cb; c < ce; c++) {
                        const int c0 = c * CH;
                        float acc[CH];
                        if (mode < 2) {
                            __syncwarp();
                            tmem_ld_acc<CH>(d_tmem + c0, two ? C::kDCols : 0, acc);
                        } else {
                            // pieces in K order: those before this CTA's, its own (from TMEM), the rest
                            const float4* sp = mode == 2 ? stage + (size_t)((c - cb) * others) * (kRedSlotBytes / 16) + r
                                                         : nullptr;
#pragma unroll
                            for (int i = 0; i < CH; i++) acc[i] = 0.0f;
#pragma unroll 1
                            for (int k = 0; k <= others; k++) {
                                if (k == before) {
                                    float own[CH];
                                    __syncwarp();
                                    tmem_ld_acc<CH>(d_tmem + c0, two ? C::kDCols : 0, own);
#pragma unroll
                                    for (int i = 0; i < CH; i++) acc[i] = before > 0 ? acc[i] + own[i] : own[i];
                                }
                                if (k == others) break;
                                const float4* src = mode == 2 ? sp + (size_t)k * (kRedSlotBytes / 16)
                                                              : reinterpret_cast<const float4*>(piece_slot(j0 + k + (k >= before ? 1 : 0), tb)) +
                                                                    (size_t)(c0 >> 2) * kTileRows + r;
#pragma unroll
                                for (int i = 0; i < CH / 4; i++) {
                                    const float4 q4 = mode == 2 ? src[i * kTileRows] : __ldcg(src + i * kTileRows);
                                    acc[4 * i] += q4.x;
                                    acc[4 * i + 1] += q4.y;
                                    acc[4 * i + 2] += q4.z;
                                    acc[4 * i + 3] += q4.w;
                                }
                            }
                        }
                        if (mode == 1) {
                            // partial -> this CTA's workspace slot through a staging buffer
                            const int b = nstore & 1;
                            if (etid == 0) tc::bulk_wait_read<1>();
                            asm volatile("bar.sync 1, 128;" ::: "memory");
                            float4* buf = reinterpret_cast<float4*>(sOut + b * C::kOutBufBytes);
#pragma unroll
                            for (int i = 0; i < CH / 4; i++)
                                buf[i * kTileRows + r] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                            asm volatile("bar.sync 1, 128;" ::: "memory");
                            if (etid == 0) {
                                tc::bulk_store(my_slot + (size_t)c0 * kTileRows, sout_base + b * C::kOutBufBytes,
                                               (uint32_t)(CH * kTileRows * 4));
                                tc::bulk_commit();
                            }
                            nstore++;
                        } else {
                            out_chunk(acc, row0, m0 + c0, min(CH, mvalid - c0), scale, bias,
                                      rrow ? rrow + (size_t)c0 * p.N : nullptr);
                        }
                    }
                    if (mode == 2) asm volatile("bar.sync 1, 128;" ::: "memory");  // the batch is consumed
                }
                if (mode == 1) {
                    if (etid == 0) {
                        tc::bulk_wait_all();  // the partial is in global memory ...
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        __threadfence();      // ... before the counter says so
                        const int prev = atomicAdd(p.counters + t, 1);
                        *lf = (prev == others) ? 1 : 0;
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (!*lf) break;
                    mode = 2;  // arrived last after all: reduce (own piece still in TMEM)
                } else {
                    if (mode >= 2) {
                        asm volatile("bar.sync 1, 128;" ::: "memory");
                        if (etid == 0) p.counters[t] = 0;  // ready for the next launch
                    }
                    break;
                }
            }
            // accumulator drained: the MMA may reuse it
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(accempty0 + 8u * ab);
            seg++;
        }
        if (!ok) raise_error(abort);
        if (etid == 0) tc::bulk_wait_all();  // outputs written before the grid completes
        if (etid == 0) GEMM_TRACE(6, trace_t0);
        if (etid == 0) {
            ROLE_TRACE(13, w_accfull);
            ROLE_TRACE(14, clock64() - t_role);
        }
    }

    // ---------------------------------------------------------------- teardown
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, C::kTmemCols);
    }
    if (threadIdx.x == 0) GEMM_TRACE(7, trace_t0);
}

// ----------------------------------------------------------------------------- host
// Weight map: int8 [N, K] in [128 rows x min(BK, 128) B] boxes (128- or 64-byte
// swizzle); activation map: fp16 [M, K] in [BN rows x 64] boxes, 128-byte
// swizzled; out-of-range rows/columns read 0.
bool make_maps(const LinearArgs& a, int BN, int BK, CUtensorMap* mw, CUtensorMap* mx)
{
    TmapDesc w{};
    w.base = a.w;
    w.inner = a.K;
    w.outer = a.N;
    w.row_bytes = a.K;
    w.box_inner = BK < 128 ? (uint32_t)BK : 128u;
    w.box_outer = kTileRows;
    w.dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    w.swizzle = w.box_inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    TmapDesc x{};
    x.base = a.x;
    x.inner = a.K;
    x.outer = a.M;
    x.row_bytes = a.K * 2;
    x.box_inner = 64;
    x.box_outer = (uint32_t)BN;
    x.dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    x.swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
    return tmap_2d(mw, w) && tmap_2d(mx, x);
}

// Output map: [M, N] fp16 or fp32, row-major, stored in [CH tokens x 128 channels]
// boxes from an unswizzled staging buffer; out-of-range rows/columns are not written.
bool make_out_map(const LinearArgs& a, int CH, CUtensorMap* mo)
{
    TmapDesc o{};
    o.base = a.out;
    o.inner = a.N;
    o.outer = a.M;
    o.row_bytes = a.N * (a.out_dtype == kF16 ? 2 : 4);
    o.box_inner = kTileRows;
    o.box_outer = (uint32_t)CH;
    o.dtype = a.out_dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    o.swizzle = CU_TENSOR_MAP_SWIZZLE_NONE;
    return tmap_2d(mo, o);
}

// Token-tile width: the smallest UMMA N that covers M up to 128 tokens; above
// that, 256-token tiles (issue-bound 128-token MMAs run at ~half rate) unless
// that leaves fewer than a quarter as many tiles as SMs, where the stream-K
// fixup of the many pieces per tile would cost more than it saves.
int pick_bn(size_t M, size_t N, int num_sms)
{
#ifdef B200Q8_TRACE
    if (const char* f = getenv("B200Q8_TRACE_BN")) return atoi(f);  // profiling build: forced tile width
#endif
    if (M <= 16) return 16;
    if (M <= 32) return 32;
    if (M <= 64) return 64;
    if (M <= 128) return 128;
    const long long tiles_n = (long long)((N + kTileRows - 1) / kTileRows);
    // Small problems whose 32-token tiles all fit on the SMs run fastest as many narrow whole
    // tiles (measured on B200 at M = 512: 896x896 16.0 -> 14.2 us, 4864x896 32.7 -> 28.2 us).
    if (tiles_n * (long long)((M + 31) / 32) <= num_sms) return 32;
    const long long tiles256 = tiles_n * (long long)((M + 255) / 256);
    return 4 * tiles256 >= num_sms ? 256 : 128;
}
int pick_bk(int BN) { return BN <= 32 ? 256 : BN <= 128 ? 128 : 64; }

// Grid size: one CTA per SM with stream-K over all units, unless the tiles fit on
// the SMs whole and finishing each tile in one CTA is quicker than splitting them:
// a split tile costs its pieces a workspace round trip and a serial fixup (about
// 12 us plus 1 us per piece, measured), which small problems cannot amortize.
long long pick_grid(long long tiles, long long kbpt, int BN, int BK, int num_sms)
{
    const long long units = tiles * kbpt;
#ifdef B200Q8_TRACE
    if (const char* f = getenv("B200Q8_TRACE_GRID")) {  // profiling build: 1 = whole tiles, 2 = stream-K,
        if (atoi(f) == 1) return tiles;                  // larger: that many CTAs (at most the SMs)
        if (atoi(f) == 2) return units < num_sms ? units : num_sms;
        if (atoi(f) > 2) return std::min<long long>(std::min<long long>(units, num_sms), atoi(f));
    }
#endif
    const long long sk = units < num_sms ? units : num_sms;
    if (tiles > num_sms || units % sk == 0 && (units / sk) % kbpt == 0) return sk;  // no split anyway
    // per-unit time: BK/16 MMAs of max(issue ~70, BN/2) cycles, at ~1.9 GHz, x1.3 for data movement
    const double unit_us = (BK / 16) * (BN / 2 > 70 ? BN / 2 : 70) / 1900.0 * 1.3;
    const double dp_us = (double)kbpt * unit_us;
    const double pieces = (double)sk / (double)tiles + 1.0;
    const double sk_us = (double)units / (double)sk * unit_us + 12.0 + pieces;
    if (dp_us <= sk_us) return tiles;
    // Splitting: as many pieces per tile for every tile when that keeps >= 90 % of the SMs (each
    // tile's pieces then end together).  Measured on B200, 7B down projection (28 tiles): 140 CTAs
    // vs 148 -- M = 64 26.2 vs 28.5 us, M = 8 23.1 vs 23.4 us.
    const long long aligned = tiles * (sk / tiles);
    return (aligned > tiles && 10 * aligned >= 9 * sk) ? aligned : sk;
}

template <int BN, int BK, int S, int SA, int NI, typename OT>
cudaError_t launch_cfg(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    using C = SkCfg<BN, BK, S, SA, NI>;
    CUtensorMap mw, mx, mo;
    if (!make_maps(a, BN, BK, &mw, &mx)) return cudaErrorInvalidValue;
    const size_t ob = a.out_dtype == kF16 ? 2 : 4;
    const bool tma_out = ((uintptr_t)a.out % 16) == 0 && (a.N * ob) % 16 == 0;
    if (tma_out) {
        if (!make_out_map(a, C::kChunk, &mo)) return cudaErrorInvalidValue;
    } else {
        mo = mx;  // unused by the kernel
    }
    auto kern = q8_gemm_sk_kernel<BN, BK, S, SA, NI, OT>;
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
    p.tma_out = tma_out ? 1 : 0;
    // Weight tiles read by one token tile only (M <= BN) are streamed through L2 once.  (Keeping
    // weight stages requested into L2 ahead of the ring measured slower at M = 64: 7B lm_head
    // 146 -> 150-156 us for 8-32 stages ahead.)
    p.w_evict_first = a.M <= (size_t)BN ? 1 : 0;
    const int G = (int)pick_grid(tiles, p.kbpt, BN, BK, num_sms);
    if ((long long)scratch.ws_floats < 2LL * G * BN * kTileRows || (long long)scratch.counters < tiles)
        return cudaErrorMemoryAllocation;
    p.ws = scratch.ws;
    p.counters = scratch.counter_ptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, mw, mx, mo, p);
    if (e == cudaSuccess) note_launch();
    return e;
}

template <typename OT>
cudaError_t launch_typed(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    // One A stage in TMEM per shared-memory stage (one commit per stage).  Measured on B200 against
    // the earlier layouts with fewer A stages (16: 5/2, 32: 4/2, 64: 6/3, 128: 4/3 stages), 7B
    // projections back to back: M = 64 lm_head 153.4 -> 142.7 us, M = 8-16 1-4 % faster, M = 32 equal.
    // 64-token tiles take two MMA-issuing threads (alternate stages, single-buffered accumulators):
    // M = 64 lm_head 142.9 -> 126.9 us, gate/up 39.5 -> 33.5, down 31.0 -> 28.9 (with double-buffered
    // accumulators and 4 stages: 135.2, 38.4, 32.7; with 256-wide K-stages, three of them: 128.7,
    // 36.3, 28.8).  For 16- and 32-token tiles a second issuer
    // measured within +-4 %, mostly slower, on the 7B projections and on the config-4 GEMMs at
    // M = 512 (set of four 54.5 vs 54.7 us).
    switch (pick_bn(a.M, a.N, num_sms)) {
        case 16: return launch_cfg<16, 256, 3, 3, 1, OT>(a, num_sms, scratch, stream);
        case 32: return launch_cfg<32, 256, 3, 3, 1, OT>(a, num_sms, scratch, stream);
        case 64: return launch_cfg<64, 128, 6, 6, 2, OT>(a, num_sms, scratch, stream);
        case 128: return launch_cfg<128, 128, 4, 4, 1, OT>(a, num_sms, scratch, stream);
        default: return launch_cfg<256, 64, 4, 4, 1, OT>(a, num_sms, scratch, stream);
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
    const int BN = pick_bn(a.M, a.N, num_sms);
    const int BK = pick_bk(BN);
    const long long tiles_n = (long long)((a.N + kTileRows - 1) / kTileRows);
    const long long tiles = tiles_n * (long long)((a.M + BN - 1) / BN);
    const long long G = pick_grid(tiles, (long long)((a.K + BK - 1) / BK), BN, BK, num_sms);
    *ws_floats = (size_t)(2 * G * BN * kTileRows);
    *counters = (size_t)tiles;
}

cudaError_t launch_q8_gemm_tc(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream)
{
    if (!gemm_tc_supports(a)) return cudaErrorNotSupported;
    return a.out_dtype == kF16 ? launch_typed<__half>(a, num_sms, scratch, stream)
                               : launch_typed<float>(a, num_sms, scratch, stream);
}

#ifdef B200Q8_TRACE
// Profiling build only: copies the per-CTA phase timestamps of the last GEMM launches.
// dst null: clear them.
extern "C" __attribute__((visibility("default"))) int b200q8_trace_gemm(void* dst, size_t bytes)
{
    if (!dst) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemm_trace) != cudaSuccess) return -2;
        return cudaMemset(p, 0, sizeof(g_gemm_trace)) == cudaSuccess ? 0 : -2;
    }
    if (bytes > sizeof(g_gemm_trace)) bytes = sizeof(g_gemm_trace);
    return cudaMemcpyFromSymbol(dst, g_gemm_trace, bytes) == cudaSuccess ? 0 : -2;
}

// Profiling build only: copies the per-CTA role counters of the last GEMM launches, [1024][16]
// SM cycles: 0-2 the MMA thread's waits (stage loaded, A stage dequantized, accumulator free),
// 3 its whole loop, 4 its stage count; 5-7 and 8-10 one warp of each dequantizer group (waits
// for the stage, for the A stage to be free, whole loop); 11-12 the producer (wait for a free
// stage, whole loop); 13-14 the epilogue (wait for an accumulator, whole loop).
// dst null: clear them.
extern "C" __attribute__((visibility("default"))) int b200q8_trace_gemm_roles(void* dst, size_t bytes)
{
    if (!dst) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemm_role) != cudaSuccess) return -2;
        return cudaMemset(p, 0, sizeof(g_gemm_role)) == cudaSuccess ? 0 : -2;
    }
    if (bytes > sizeof(g_gemm_role)) bytes = sizeof(g_gemm_role);
    return cudaMemcpyFromSymbol(dst, g_gemm_role, bytes) == cudaSuccess ? 0 : -2;
}
#endif

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
