// q8_gemv_tc.cu -- int8-weight GEMV / skinny GEMM on the tensor cores with exact
// multi-digit activations (kind::i8), for M = 1..42 tokens per launch group.
//
// out[m, n] = (sum_k x[m, k] * float(W[n, k])) * scales[n] + bias[n] (+ res[m, n])
// (semantics of vvllm BackendCPU::linear_q8 / linear_q8_add,
//  src/backend/backend_naive.cc:155-291 and :322-335.)
//
// Decode streams every weight byte once, so the kernel must turn HBM bytes
// into MACs with as little per-byte work as possible.  The int8 weights are
// never converted: the TMA-loaded weight tile IS the MMA's A operand.  The
// activations are made exact integers instead: x_q = x * 2^e with
//   fp16 x: e = 24, which makes every finite fp16 value an integer below 2^40
//           (exact, no data-dependent scale);
//   fp32 x: e = 39 - floor(log2(max_k |x_m,k|)) per token (rounded to an
//           integer, 2^-40 relative to the row maximum).
// x_q is split into six base-128 digits (five unsigned 7-bit digits and a
// signed top digit, all int8), which become 6*M rows of the MMA's B operand
// (N = 6M padded to a multiple of 16; M = 1 decode pads to 16 anyway, so the
// digits cost nothing).  tcgen05.mma.kind::i8 (K = 32 per instruction)
// accumulates exact int32 digit sums in TMEM; the epilogue recombines them in
// double (sum_d D_d * 2^(7d) * 2^-e), rounds once to fp32 and applies the
// per-row scale, bias and residual in the reference's order.
//
// Pipeline (one CTA per SM, persistent stream-K over (128-row tile, K-stage)
// units, exact int64 fixup of split tiles):
//   warp 0     TMA producer: weight boxes [128 rows x 128 B], 128-byte swizzled,
//              into an S-stage ring (starts at launch: weights never wait for
//              the previous kernel);
//   warp 1     TMEM allocator + one thread issuing BK/32 kind::i8 MMAs per stage;
//   warps 2-5  epilogue: tcgen05.ld, digit recombination, stores / fixup;
//   warps 6-9  digitizers: read x for the stage (fp32: after the per-token
//              exponents are ready; fp16 uses the fixed exponent), write the six
//              digit rows per token straight into the stage's swizzled B tile in
//              shared memory.
// A prep kernel (one CTA per token) computes the exponents and flags rows with
// Inf/NaN (their outputs are NaN).  Every mbarrier wait is bounded; a timeout
// sets a device error word, drains in-flight copies and MMAs, frees TMEM and
// returns.  No TMA multicast and no clusters.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "p2p.cuh"
#include "prologue.cuh"
#include "sk_common.cuh"
#include "tc_utils.cuh"
#include "tmap.cuh"

namespace b200q8 {

__device__ int g_kernel_error_i8;  // bit 0: a bounded wait timed out in the digit GEMV

namespace {

constexpr int kTileRows = 128;
constexpr int kWarps = 10;
constexpr int kThreads = kWarps * 32;
constexpr int kFirstEpi = 2, kFirstDig = 6;
constexpr int kDigits = 6;
constexpr int kF16Exp = 24;  // 2^24 * fp16 is an integer for every finite fp16
constexpr int kQBits = 40;   // |x_q| < 2^40
constexpr int kMaxTokens = 42;  // 6 * 42 = 252 <= 256 digit rows
// Up to this many tokens of at most this length, every CTA scans x for the exponents itself
// (saves the prep kernel's launch); longer rows would delay the first digits more than that.
constexpr int kFusedExpTokens = 4;
constexpr size_t kFusedExpMaxK = 4096;
// Longer rows are scanned in-kernel too when the weights are small (the next constant): there
// the prep kernel's launch is a large share of the call.  Measured on B200, one fp16 token: Qwen2.5-0.5B
// down (896 x 4864) 10.9 -> 9.9 us in-kernel; Qwen2-7B down (3584 x 18944) 20.0 -> 20.4 us.
constexpr size_t kFusedExpMaxKSmall = 20480;
// ... for weights up to this size.
constexpr size_t kInKernelScanMaxBytes = (size_t)32 << 20;
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;
constexpr uint64_t kPeerTimeoutNs = 2000000000ull;  // a peer's flag of the previous gathered call
// Weight bytes (all CTAs together) requested into L2 beyond the shared-memory rings at the start.
constexpr long long kPrefetchBytes = 32ll << 20;

struct DigParams {
    const void* x;    // [M, K] fp16 or fp32
    const float* scales;
    const float* bias;
    const void* res;
    void* out;
    const int* prep_part;  // [M][prep_splits] the prep kernel's words (without in-kernel exponents)
    int prep_splits;
    int* ws;          // [2 * gridDim.x][128][NC] int32 partial digit sums
    int* counters;    // [tiles] arrival counters, zero between launches
    int M, N, K;
    int kbpt;
    long long units;
    P2POut po;        // output placement: local only (ndst = 1) or every rank's copy
    int fused_exps;   // exponents computed in-kernel (few tokens) instead of by the prep kernel
    // Stages past the ring whose weight boxes the producer asks L2 for at the start (0: none):
    // HBM keeps streaming while the digitizers wait for the previous kernel (or the previous
    // gathered call), and CTAs that start on SMs the previous kernel left idle fetch early.
    int prefetch_stages;
    // Digit tiles of every K-stage, made once per launch by the prep kernel ([kbpt][kDBytes], each
    // the exact shared-memory image of the stage's B tile) and copied in by the producer beside
    // the weights; null: the digitizer warps make each stage's tile themselves.
    const unsigned char* dig_img;
    int early_trigger;  // dependents may launch right after set-up (else at the epilogue's end)
    int w_evict_first;  // weight tiles are loaded with an L2 evict-first policy
    // Greedy argmax over each token's outputs (null: none): packed (value, index) keys, zero
    // between launches; the launch's last CTA turns them into indices and re-zeroes them.
    unsigned long long* amax_keys;  // [M]
    unsigned int* amax_done;        // CTAs finished, zero between launches
    int* amax_out;                  // [M] result
};

template <int NC, int BK, int S>
struct DigCfg {
    static constexpr int kBoxes = BK / 128;  // 128-byte K boxes per stage
    static constexpr int kWBytes = kTileRows * BK;
    static constexpr int kDBoxBytes = NC * 128;
    static constexpr int kDBytes = kBoxes * kDBoxBytes;
    static constexpr int kDCols = (NC + 31) / 32 * 32;
    static constexpr int kColsNeeded = 2 * kDCols;
    static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                     : kColsNeeded <= 256 ? 256 : 512;
    static constexpr int kNumBars = 3 * S + 4 + 1;  // full, dfull, empty per stage; acc x4; drain
    static constexpr int kSmemBytes =
        1024 + S * (kWBytes + kDBytes) + kNumBars * 8 + 16 + 4 * kMaxTokens + 64 + 8 * kMaxTokens + 8;
    static_assert(NC % 16 == 0 && NC >= 16 && NC <= 256, "kind::i8 N for M=128");
    static_assert(BK % 128 == 0, "whole 128-byte boxes");
    static_assert(kColsNeeded <= 512, "TMEM overflow");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kDBoxBytes % 1024 == 0, "digit boxes stay 1024-byte aligned");
};

__device__ __forceinline__ void raise_error(volatile int* abort)
{
    *abort = 1;
    atomicOr(&g_kernel_error_i8, 1);
}

// Bounded wait until a split tile's arrival counter reaches `target` (read with gpu-scope
// acquire); false after timeout_ns or once the CTA aborts.
__device__ bool wait_tile_pieces(const int* ctr, int target, volatile int* abort, uint64_t timeout_ns)
{
    const uint64_t t0 = tc::globaltimer_ns();
    for (;;) {
        int seen;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(ctr) : "memory");
        if (seen >= target) return true;
        if (*abort || tc::globaltimer_ns() - t0 > timeout_ns) return false;
        __nanosleep(32);
    }
}

// ----------------------------------------------------------------------------- prep
// max |a| over the 4-element groups [c0, c1) of one token's row taken by thread t of nt, and
// whether any a is Inf/NaN; a is x or, with a prologue, the activations it makes from x, which
// are also stored to act_row when it is given.
template <typename XT, int B>
__device__ __forceinline__ void scan_groups(int pro, const XT* xrow, int K, const float* norm_w, float rms, int c0,
                                            int c1, int t, int nt, float& mx, int& bad, XT* act_row = nullptr)
{
    if (pro != kProNone) {
        for (int i0 = c0 + t; i0 < c1; i0 += B * nt) {
            float v[B][4], aux[B][4];
#pragma unroll
            for (int b = 0; b < B; b++)  // every load of the batch first
                if (i0 + b * nt < c1) act4_load<XT>(pro, xrow, K, 4 * (i0 + b * nt), norm_w, v[b], aux[b]);
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int i = i0 + b * nt;
                if (i >= c1) break;
                act4_apply<XT>(pro, rms, v[b], aux[b]);
                if (act_row) store4<XT>(act_row + 4 * i, v[b]);
#pragma unroll
                for (int j = 0; j < 4; j++) {  // NaN and Inf fail a <= FLT_MAX
                    const float a = fabsf(v[b][j]);
                    bad |= (a <= FLT_MAX) ? 0 : 1;
                    mx = (a <= FLT_MAX) ? fmaxf(mx, a) : mx;
                }
            }
        }
    } else if (sizeof(XT) == 2) {
        // 8-byte loads: fp16 activations are only required to be 8-byte aligned; the exponent
        // is fixed, only Inf/NaN (exponent field all ones) matter
        const uint2* xr = reinterpret_cast<const uint2*>(xrow);
        for (int i0 = c0 + t; i0 < c1; i0 += 4 * B * nt) {
            uint2 v[4 * B];
#pragma unroll
            for (int b = 0; b < 4 * B; b++)  // every load of the batch first
                v[b] = (i0 + b * nt < c1) ? xr[i0 + b * nt] : make_uint2(0u, 0u);
#pragma unroll
            for (int b = 0; b < 4 * B; b++) {
                const uint32_t w[2] = {v[b].x, v[b].y};
#pragma unroll
                for (int j = 0; j < 2; j++)
                    bad |= (((w[j] & 0x7C00u) == 0x7C00u) || ((w[j] & 0x7C000000u) == 0x7C000000u)) ? 1 : 0;
            }
        }
    } else {
        const float4* xr = reinterpret_cast<const float4*>(xrow);
        for (int i0 = c0 + t; i0 < c1; i0 += 2 * B * nt) {
            float4 v[2 * B];
#pragma unroll
            for (int b = 0; b < 2 * B; b++)  // every load of the batch first
                v[b] = (i0 + b * nt < c1) ? xr[i0 + b * nt] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < 2 * B; b++) {
                const float a[4] = {fabsf(v[b].x), fabsf(v[b].y), fabsf(v[b].z), fabsf(v[b].w)};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    bad |= (a[j] <= FLT_MAX) ? 0 : 1;
                    mx = (a[j] <= FLT_MAX) ? fmaxf(mx, a[j]) : mx;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
}

// The token's exponent: fp16 e = 24; fp32 e = 39 - floor(log2 max|a|); INT_MIN if any Inf/NaN.
template <typename XT>
__device__ __forceinline__ int token_exp(float m_all, int bad)
{
    if (bad) return INT_MIN;
    if (sizeof(XT) == 2) return kF16Exp;
    return (m_all > 0.0f) ? (kQBits - 1) - ilogbf(m_all) : 0;
}

// Grid (M tokens, ns = row_splits(K) CTAs per token), 256 threads: CTA (m, sp) scans its share
// of token m's row and stores one word, part[m * ns + sp] = the bits of its max |a| (a finite
// float >= 0, so integer order is float order) or -1 if it met an Inf/NaN; the GEMV folds the
// words into the exponents.  With a prologue, act_out [M, K] receives the activations and the
// GEMV reads them as its x.  No atomics: nothing sits between the last load and the GEMV's
// start.  A 256-thread CTA capped at 40 registers fits beside a GEMV CTA (320 threads at <= 168
// registers) on one SM, so the GEMV launched behind this kernel keeps all its CTAs resident.
template <typename XT>
__global__ void __launch_bounds__(kSqThreads, 6) exps_kernel(const XT* __restrict__ x, int K,
                                                          const unsigned long long* wait_counts, int wait_n,
                                                          int wait_self, unsigned long long wait_ns,
                                                          int pro, const float* norm_w,
                                                          float eps, int* __restrict__ part, XT* __restrict__ act_out)
{
    pdl_launch_dependents();  // the GEMV may start streaming weights right away
    pdl_wait();               // x is written by the previous kernel
    __shared__ float red[kSqWarps];
    __shared__ int bad_w[kSqWarps];
    __shared__ double sq[kSqWarps];
    const int m = blockIdx.x;
    const int sp = blockIdx.y, ns = gridDim.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // x is the gathered output of a deferred call: every rank's part must have landed
    if (tid == 0 && wait_counts && !wait_peers(wait_counts, wait_n, wait_self, wait_ns))
        atomicOr(&g_kernel_error_i8, 2);
    __syncthreads();
    const XT* xrow = x + (size_t)m * (pro == kProSiluMul ? 2 * (size_t)K : (size_t)K);
    float rms = 1.0f;
    if (pro == kProRmsNorm) {  // every CTA of the token takes the whole (fixed-order) sum
        const double w = sumsq_warp<XT>(xrow, K, tid);
        if (lane == 0) sq[warp] = w;
        __syncthreads();
        rms = rms_from(sq, K, eps);
    }
    const int g4 = K >> 2;
    const int c0 = (int)((long long)g4 * sp / ns), c1 = (int)((long long)g4 * (sp + 1) / ns);
    float mx = 0.0f;
    int bad = 0;
    scan_groups<XT, 2>(pro, xrow, K, norm_w, rms, c0, c1, tid, kSqThreads, mx, bad,
                       act_out ? act_out + (size_t)m * K : nullptr);
    if (lane == 0) {
        red[warp] = mx;
        bad_w[warp] = bad;
    }
    __syncthreads();
    if (tid != 0) return;
    float m_all = 0.0f;
    int b_all = 0;
    for (int w = 0; w < kSqWarps; w++) {
        m_all = fmaxf(m_all, red[w]);
        b_all |= bad_w[w];
    }
    part[(size_t)m * ns + sp] = b_all ? -1 : __float_as_int(m_all);
}

// The prep kernel's words folded into the tokens' exponents in shared memory by NT threads
// (sid 0..NT-1) that meet at named barrier BAR: warp w takes tokens w, w + NT/32, ...
// fp32: the epilogue and digitizer warps together (256, barrier 3); fp16, whose digits use the
// fixed exponent: the epilogue warps alone (128, barrier 2).
template <typename XT, int NT, int BAR>
__device__ __forceinline__ void fold_prep(const DigParams& p, int sid, int* s_exps)
{
    const int sw = sid >> 5, lane = sid & 31;
    for (int m = sw; m < p.M; m += NT / 32) {
        int hi = 0, lo = 0;
        for (int j = lane; j < p.prep_splits; j += 32) {
            const int v = p.prep_part[(size_t)m * p.prep_splits + j];
            hi = max(hi, v);
            lo = min(lo, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        }
        if (lane == 0) s_exps[m] = token_exp<XT>(__int_as_float(hi), lo < 0 ? 1 : 0);
    }
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
}

// The exponents of a few tokens, computed inside the GEMV with the prep kernel's rules by NT
// threads (sid 0..NT-1) that meet at named barrier BAR, as for fold_prep.
template <typename XT, int NT, int BAR>
__device__ __forceinline__ void fused_scan(const DigParams& p, int sid, int* s_exps, float* s_red)
{
    constexpr int NW = NT / 32;
    static_assert(NW <= kSqWarps, "s_red holds 2 * kSqWarps words");
    const int sw = sid >> 5, lane = sid & 31;
#pragma unroll 1
    for (int m = 0; m < p.M; m++) {
        const XT* xrow = reinterpret_cast<const XT*>(p.x) + (size_t)m * p.K;
        float mx = 0.0f;
        int bad = 0;
        scan_groups<XT, NT == 128 ? 4 : 2>(kProNone, xrow, p.K, nullptr, 1.0f, 0, p.K >> 2, sid, NT, mx, bad);
        if (lane == 0) {
            s_red[sw] = mx;
            s_red[kSqWarps + sw] = __int_as_float(bad);
        }
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
        if (sid == 0) {
            float m_all = 0.0f;
            int b_all = 0;
            for (int i = 0; i < NW; i++) {
                m_all = fmaxf(m_all, s_red[i]);
                b_all |= __float_as_int(s_red[kSqWarps + i]);
            }
            s_exps[m] = token_exp<XT>(m_all, b_all);
        }
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    }
}

// Six base-128 digits of q (|q| < 2^40): d0..d4 unsigned 7-bit, d5 signed.
__device__ __forceinline__ void digits6(long long q, uint32_t (&d)[kDigits], int byte)
{
#pragma unroll
    for (int i = 0; i < kDigits - 1; i++) d[i] |= (uint32_t)((q >> (7 * i)) & 127) << (8 * byte);
    d[kDigits - 1] |= (uint32_t)((int)(q >> 35) & 0xFF) << (8 * byte);
}

// The six digit words of 4 consecutive activations (one byte per activation) at exponent e.
__device__ __forceinline__ void digit_words(const float (&v)[4], int e, uint32_t (&d)[kDigits])
{
#pragma unroll
    for (int i = 0; i < kDigits; i++) d[i] = 0;
    if (e != INT_MIN) {  // beyond K the values are 0: zero digits
#pragma unroll
        for (int i = 0; i < 4; i++) digits6(__float2ll_rn(ldexpf(v[i], e)), d, i);
    }
}

// Stores token m's digit words for K offset kk (a multiple of 4, within the stage) into a stage's
// B tile: digit i of token m is row 6m + i; boxes of [rows x 128 B], 128-byte swizzle.
template <int kDBoxBytes>
__device__ __forceinline__ void put_digit_words(unsigned char* tile, int m, int kk, const uint32_t (&d)[kDigits])
{
    const int h = kk >> 7, c = (kk & 127) >> 4, byte = kk & 15;
#pragma unroll
    for (int i = 0; i < kDigits; i++) {
        const int r = m * kDigits + i;
        *reinterpret_cast<uint32_t*>(tile + h * kDBoxBytes + r * 128 + ((c ^ (r & 7)) << 4) + byte) = d[i];
    }
}

// Prep kernel of a launch whose GEMV copies its digit tiles in (fp16 activations, no prologue, no
// gather; gemv_i8_images): grid = the kbpt K-stages, 256 threads.  CTA kb writes the exact
// shared-memory image of stage kb's B tile -- every token's six digit rows at the fixed fp16
// exponent, the same bytes the digitizer warps would write, and zero rows up to NC -- and
// part[m * kbpt + kb] = -1 if token m's values in the stage hold an Inf/NaN, else 0 (folded by
// the GEMV's epilogue warps like the scan words).  The digits are made once per launch instead of
// once per tile and stage: with several tokens the digitizer warps were the GEMV's limit.
template <int NC, int BK>
__global__ void __launch_bounds__(kSqThreads) digit_tiles_kernel(const __half* __restrict__ x, int M, int K,
                                                               int* __restrict__ part,
                                                               unsigned char* __restrict__ img)
{
    pdl_launch_dependents();  // the GEMV may start streaming weights right away
    pdl_wait();               // x is written by the previous kernel
    constexpr int kIpt = BK / 4;  // items (4 consecutive k of one token) per token and stage
    constexpr int kDBoxBytes = NC * 128;
    __shared__ int bad[kMaxTokens];
    const int kb = blockIdx.x, tid = threadIdx.x;
    unsigned char* tile = img + (size_t)kb * (NC * BK);
    for (int m = tid; m < M; m += kSqThreads) bad[m] = 0;
    __syncthreads();
    for (int item = tid; item < M * kIpt; item += kSqThreads) {
        const int m = item / kIpt, kk = (item - m * kIpt) * 4, k = kb * BK + kk;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (k < K) load4<__half>(x + (size_t)m * K + k, v);
        int nf = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) nf |= (fabsf(v[i]) <= FLT_MAX) ? 0 : 1;  // NaN and Inf fail
        if (nf) atomicOr(&bad[m], 1);
        uint32_t d[kDigits];
        digit_words(v, kF16Exp, d);
        put_digit_words<kDBoxBytes>(tile, m, kk, d);
    }
    // digit rows 6M .. NC-1: zero (16-byte chunks; all-zero rows need no swizzle)
    constexpr int kChunks = BK / 16;  // per row
    const int zr = kDigits * M;
    for (int i = tid; i < (NC - zr) * kChunks; i += kSqThreads) {
        const int r = zr + i / kChunks, c16 = i % kChunks;
        *reinterpret_cast<uint4*>(tile + (c16 >> 3) * kDBoxBytes + r * 128 + (c16 & 7) * 16) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    for (int m = tid; m < M; m += kSqThreads) part[(size_t)m * gridDim.x + kb] = bad[m] ? -1 : 0;
}

__device__ __forceinline__ float recombine(const long long (&dsum)[kDigits], int e)
{
    if (e == INT_MIN) return __int_as_float(0x7fc00000);  // the token row holds Inf/NaN
    double acc = 0.0;
#pragma unroll
    for (int i = kDigits - 1; i >= 0; i--) acc = acc * 128.0 + (double)dsum[i];
    return __double2float_rn(ldexp(acc, -e));
}

// v = acc * scale (+ bias) (+ res[m, n]) stored at column ocol0 + n of row m in every
// output copy (one local copy, or each rank's copy over NVLink for the sharded gather).
// Returns the output as stored (rounded to OT).
template <typename OT>
__device__ __forceinline__ float epi_out(const DigParams& p, int m, int n, float acc, float scale, float bias,
                                         bool has_bias)
{
    float v = __fmul_rn(acc, scale);
    if (has_bias) v = __fadd_rn(v, bias);
    if (p.res) v = __fadd_rn(v, load_as_f32<OT>(reinterpret_cast<const OT*>(p.res) + (size_t)m * p.N + n));
    const size_t o = (size_t)m * p.po.ldo + p.po.ocol0 + n;
    for (int d = 0; d < p.po.ndst; d++) sk::store_out<OT>(reinterpret_cast<OT*>(p.po.dst[d]) + o, v);
    if (sizeof(OT) == 2) v = __half2float(__float2half_rn(v));
    return v;
}

// Greedy-argmax key of output n with stored value v: larger key = larger value, then smaller
// index.  The order is std::max_element's over the row (src/sampler/sampler.cc:20-24): the first
// maximum wins, NaNs are never greater than anything -- except a NaN at index 0, which
// std::max_element keeps, so it gets the largest key.  -0 compares equal to +0.
__device__ __forceinline__ unsigned long long argmax_key(float v, int n)
{
    uint32_t ord;
    if (v != v) {
        ord = n == 0 ? 0xFFFFFFFFu : 0u;
    } else {
        const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
        ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

// ----------------------------------------------------------------------------- GEMV
template <int NC, int BK, int S, typename XT, typename OT>
__global__ void __launch_bounds__(kThreads, 1)
    q8_gemv_dig_kernel(const __grid_constant__ CUtensorMap tmW, const DigParams p)
{
    using C = DigCfg<NC, BK, S>;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* sW = smem;
    unsigned char* sD = smem + S * C::kWBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sD + S * C::kDBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    // tmem_holder[2..3]: spare
    int* s_exps = reinterpret_cast<int*>(tmem_holder + 4);                          // [kMaxTokens]
    float* s_red = reinterpret_cast<float*>(s_exps + kMaxTokens);                   // [16] exponent reduction
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(                 // [kMaxTokens] argmax keys
        (reinterpret_cast<uintptr_t>(s_red + 2 * kSqWarps) + 7) & ~static_cast<uintptr_t>(7));

    const uint32_t bar0 = tc::smem_u32(bars);
    const uint32_t full0 = bar0, dfull0 = bar0 + 8u * S, empty0 = bar0 + 16u * S, accfull0 = bar0 + 24u * S,
                   accempty0 = accfull0 + 16u, drainbar = accfull0 + 32u;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int cta = blockIdx.x;
    const long long u_begin = sk::unit_begin(cta, p.units, G), u_end = sk::unit_begin(cta + 1, p.units, G);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            tc::mbar_init(full0 + 8u * s, 1);
            tc::mbar_init(dfull0 + 8u * s, 4);
            tc::mbar_init(empty0 + 8u * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(accfull0 + 8u * b, 1);
            tc::mbar_init(accempty0 + 8u * b, 4);
        }
        tc::mbar_init(drainbar, 1);
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (threadIdx.x == 32) tc::prefetch_tensormap(&tmW);
    // Digit rows past 6M stay zero for the whole kernel: clear every stage's B tile once (the
    // prep kernel's digit tiles carry their zero rows).
    if (!p.dig_img)
        for (int i = threadIdx.x; i < S * C::kDBytes / 16; i += kThreads)
            reinterpret_cast<uint4*>(sD)[i] = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
    __syncwarp();
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_holder), C::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // Every CTA of the grid is resident (G <= SMs) and none waits on another, so the next kernel
    // may take the SMs this grid leaves idle now: its set-up and first weight requests overlap
    // this grid's streaming.  Its griddepcontrol.wait still waits for this grid's completion.
    if (p.early_trigger) pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (weights)
        if (lane == 0) {
            const uint64_t wpol = p.w_evict_first ? tc::l2_policy_evict_first() : tc::l2_policy_evict_normal();
            sk::Ring st;
            int issued = 0;
            bool ok = true;
            int t, k0, k1;
            sk::SegIter it(u_begin, u_end, p.kbpt);
            const uint32_t sw_base = tc::smem_u32(sW), sd_base = tc::smem_u32(sD);
            // With the prep kernel's digit tiles, each stage's full barrier also counts its digit
            // tile's bytes.  The first S stages' weights are requested at once; their digit tiles
            // (written by the prep kernel) only after griddepcontrol.wait, and every later stage
            // requests both together.
            const uint32_t stage_tx = C::kWBytes + (p.dig_img ? C::kDBytes : 0);
            bool img_ready = false;
            auto load_digits = [&](int q, int slot) {  // unit u_begin + q into ring slot `slot`
                const long long u = u_begin + q;
                const int kb = (int)(u - (u / p.kbpt) * p.kbpt);
                tc::bulk_load(sd_base + slot * C::kDBytes, p.dig_img + (size_t)kb * C::kDBytes, C::kDBytes,
                              full0 + 8u * slot);
            };
            auto catch_up = [&]() {  // digit tiles of the stages issued before the wait
                pdl_wait();
                for (int q = 0; q < issued; q++) load_digits(q, q);
                img_ready = true;
            };
            while (ok && it.next(t, k0, k1)) {
                const int row0 = t * kTileRows;
                for (int kb = k0; kb < k1; kb++) {
                    if (issued == S && p.prefetch_stages > 0) {
                        // The ring is full: the boxes of the next prefetch_stages stages into L2
                        // before the first wait for a free slot.  (Keeping a rolling window of
                        // stages requested ahead all along measured slower: 7B decode step
                        // 119 -> 134 us.)
                        for (int j = S; j < S + p.prefetch_stages && u_begin + j < u_end; j++) {
                            const long long u = u_begin + j;
                            const int pt = (int)(u / p.kbpt), pk = (int)(u - (long long)pt * p.kbpt);
#pragma unroll
                            for (int h = 0; h < C::kBoxes; h++)
                                tc::tma_prefetch_l2_2d(&tmW, pk * BK + h * 128, pt * kTileRows);
                        }
                    }
                    if (p.dig_img && issued == S) catch_up();
                    if (issued >= S &&
                        !tc::mbar_wait(empty0 + 8u * st.idx, st.phase ^ 1u, abort, kWaitTimeoutNs)) {
                        raise_error(abort);
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8u * st.idx;
                    tc::mbar_arrive_expect_tx(fb, stage_tx);
#pragma unroll
                    for (int h = 0; h < C::kBoxes; h++)
                        tc::tma_load_2d_hint(sw_base + st.idx * C::kWBytes + h * (kTileRows * 128), &tmW,
                                             kb * BK + h * 128, row0, fb, wpol);
                    if (img_ready) load_digits(issued, st.idx);
                    issued++;
                    st.next(S);
                }
            }
            if (p.dig_img && !img_ready) catch_up();  // fewer stages than the ring holds
            if (*abort) {
                const int zero = 0;
                sk::Ring d;
                for (int q = 0; q < issued; q++, d.next(S))
                    if (q + S >= issued) tc::mbar_wait(full0 + 8u * d.idx, d.phase, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::make_idesc_s8_s32(kTileRows, NC);
            sk::Ring st;
            int seg = 0, t, k0, k1;
            sk::SegIter it(u_begin, u_end, p.kbpt);
            bool ok = true;
            const uint64_t adesc0 = tc::make_sw128_kmajor_desc(tc::smem_u32(sW));
            const uint64_t bdesc0 = tc::make_sw128_kmajor_desc(tc::smem_u32(sD));
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
                        (!p.dig_img && !tc::mbar_wait(dfull0 + 8u * st.idx, st.phase, abort, kWaitTimeoutNs))) {
                        raise_error(abort);
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint64_t a_stage = adesc0 + (uint64_t)((st.idx * C::kWBytes) >> 4);
                    const uint64_t b_stage = bdesc0 + (uint64_t)((st.idx * C::kDBytes) >> 4);
#pragma unroll
                    for (int j = 0; j < BK / 32; j++)
                        tc::mma_s8_ss(d_tmem, a_stage + (uint64_t)(((j >> 2) * (kTileRows * 128) + (j & 3) * 32) >> 4),
                                      b_stage + (uint64_t)(((j >> 2) * C::kDBoxBytes + (j & 3) * 32) >> 4), idesc,
                                      (kb != k0 || j != 0) ? 1u : 0u);
                    tc::mma_commit(empty0 + 8u * st.idx);
                    st.next(S);
                }
                if (!ok) break;
                tc::mma_commit(accfull0 + 8u * ab);
                seg++;
            }
            if (*abort) {
                const int zero = 0;
                tc::mma_commit(drainbar);
                tc::mbar_wait(drainbar, 0, &zero, kWaitTimeoutNs);
            }
        }
    } else if (warp >= kFirstDig) {
        // ------------------------------------------------------------ digitizers
        const int dtid = threadIdx.x - kFirstDig * 32;  // 0..127
        pdl_wait();  // x (and the prep kernel's exponents) are ready
        // x is the gathered output of the previous call: wait until every rank's part landed
        if (p.po.wait_counts && dtid == 0 &&
            !wait_peers(p.po.wait_counts, p.po.wait_n, p.po.rank,
                        p.po.wait_timeout_ns ? p.po.wait_timeout_ns : kPeerTimeoutNs)) {
            atomicOr(&g_kernel_error_i8, 2);
            raise_error(abort);
        }
        if (p.po.wait_counts)
            asm volatile("bar.sync 3, 256;" ::: "memory");  // peers' outputs landed (the epilogue reads them too)
        // fp32: the per-token exponents into shared memory, by the epilogue and digitizer warps
        // together (found here for few tokens, else folded from the prep kernel's words).  fp16
        // digits use the fixed exponent, so the digitizers start at once; the epilogue warps find
        // the tokens holding Inf/NaN (their outputs are NaN; their digits are never used).
        if constexpr (sizeof(XT) != 2) {
            if (p.fused_exps) fused_scan<XT, 256, 3>(p, 128 + dtid, s_exps, s_red);
            else fold_prep<XT, 256, 3>(p, 128 + dtid, s_exps);
        }
        const int* exps = s_exps;
        sk::Ring st;
        int g = 0, t, k0, k1;
        // with the prep kernel's digit tiles the producer copies them in: nothing to do here
        sk::SegIter it(u_begin, p.dig_img ? u_begin : u_end, p.kbpt);
        bool ok = true;
        const XT* xg = reinterpret_cast<const XT*>(p.x);
        // Thread -> items of 4 consecutive k of one token (BK/4 items per token per stage), at most
        // kItems per thread.  Every load of a stage is issued first, before the wait for the ring
        // slot: one L2 round trip per stage, overlapping the wait, instead of one per item.
        constexpr int kItems = ((NC / kDigits) * (BK / 4) + 127) / 128;
        const int nitems = p.M * (BK / 4);
        while (ok && it.next(t, k0, k1)) {
            for (int kb = k0; kb < k1; kb++, g++, st.next(S)) {
                float v[kItems][4];
#pragma unroll
                for (int j = 0; j < kItems; j++) {
                    const int item = dtid + j * 128;
                    const int m = item / (BK / 4);
                    const int k = kb * BK + (item - m * (BK / 4)) * 4;
                    if (item < nitems && k < p.K) {
                        load4<XT>(xg + (size_t)m * p.K + k, v[j]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; i++) v[j][i] = 0.0f;
                    }
                }
                if (g >= S) {
                    ok = __all_sync(0xffffffffu,
                                    tc::mbar_wait(empty0 + 8u * st.idx, st.phase ^ 1u, abort, kWaitTimeoutNs));
                    if (!ok) break;
                }
                unsigned char* bst = sD + st.idx * C::kDBytes;
#pragma unroll
                for (int j = 0; j < kItems; j++) {
                    const int item = dtid + j * 128;
                    if (item >= nitems) break;
                    const int m = item / (BK / 4);
                    const int kk = (item - m * (BK / 4)) * 4;  // 0..BK-4
                    uint32_t d[kDigits];
                    digit_words(v[j], sizeof(XT) == 2 ? kF16Exp : exps[m], d);
                    put_digit_words<C::kDBoxBytes>(bst, m, kk, d);
                }
                // generic-proxy writes -> visible to the tensor core's async-proxy reads
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(dfull0 + 8u * st.idx);
            }
        }
        if (!ok) raise_error(abort);
    } else {
        // ------------------------------------------------------------ epilogue
        pdl_wait();  // the prep kernel's words are complete
        if (p.amax_keys) {
            if (threadIdx.x - kFirstEpi * 32 < p.M) s_best[threadIdx.x - kFirstEpi * 32] = 0ull;
            asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        if (p.po.wait_counts)
            asm volatile("bar.sync 3, 256;" ::: "memory");  // peers' outputs landed
        // the per-token exponents, once per CTA (read for every output): fp32 with the digitizer
        // warps; fp16 (only the Inf/NaN flags) by these warps alone while the digits stream
        if constexpr (sizeof(XT) == 2) {
            if (p.fused_exps) fused_scan<XT, 128, 2>(p, threadIdx.x - kFirstEpi * 32, s_exps, s_red);
            else fold_prep<XT, 128, 2>(p, threadIdx.x - kFirstEpi * 32, s_exps);
        } else {
            if (p.fused_exps) fused_scan<XT, 256, 3>(p, threadIdx.x - kFirstEpi * 32, s_exps, s_red);
            else fold_prep<XT, 256, 3>(p, threadIdx.x - kFirstEpi * 32, s_exps);
        }
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
        const int etid = threadIdx.x - kFirstEpi * 32;
        const bool has_bias = p.bias != nullptr;
        int seg = 0, t, k0, k1;
        sk::SegIter it(u_begin, u_end, p.kbpt);
        bool ok = true;
        const int ncols = kDigits * p.M;
        while (it.next(t, k0, k1)) {
            const int ab = seg & 1, use = seg >> 1;
            // the row's scale and bias load while the accumulator fills
            const int n = t * kTileRows + r;
            const bool nv = n < p.N;
            const float scale = nv ? p.scales[n] : 0.0f;
            const float bias = (nv && has_bias) ? p.bias[n] : 0.0f;
            // one verdict for all four epilogue warps: named barrier 1 follows
            ok = tc::bar_all<1, 128>(tc::mbar_wait(accfull0 + 8u * ab, (uint32_t)(use & 1), abort, kWaitTimeoutNs));
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t d_tmem = tmem + t_lane + ab * C::kDCols;
            const bool whole = (k0 == 0 && k1 == p.kbpt);
            const long long tb = (long long)t * p.kbpt;
            const int j0 = whole ? cta : sk::cta_of_unit(tb, p.units, G);
            const int j1 = whole ? cta : sk::cta_of_unit(tb + p.kbpt - 1, p.units, G);
            bool last = whole;
            if (!whole && cta == j0) {
                // The piece holding the tile's first k-blocks reduces.  CTA j0 reaches them at the
                // end of its range, after the other pieces' CTAs have done theirs at the start of
                // theirs, so it rarely waits; it adds the other pieces' stored sums to its own taken
                // straight from TMEM.  Bounded wait: the pieces come from co-resident CTAs of
                // higher index whose waits, if any, are in later segments.
                if (etid == 0 && !wait_tile_pieces(p.counters + t, j1 - j0, abort, kWaitTimeoutNs))
                    raise_error(abort);
                asm volatile("bar.sync 1, 128;" ::: "memory");
                last = true;
            }
            const int slot = (seg == 0) ? 2 * cta : 2 * cta + 1;
            int* wrow = p.ws + ((size_t)slot * kTileRows + r) * NC;
            // Each token's six digit sums sit in consecutive TMEM columns; take kGT tokens (kGC
            // columns, 16-column loads) at a time.  A non-reducing piece stores them to its
            // workspace slot; the reducing piece adds every other piece's sums (all loads in flight)
            // and writes the outputs.
            constexpr int kGT = NC >= 48 ? 8 : NC / kDigits;     // tokens per group
            constexpr int kGC = (kGT * kDigits + 15) / 16 * 16;  // TMEM columns per group
#pragma unroll 1
            for (int pass = 0; pass < 2; pass++) {
#pragma unroll 1
                for (int mg = 0; mg < p.M; mg += kGT) {
                    const int base = mg * kDigits;
                    int dreg[kGC];
#pragma unroll
                    for (int c = 0; c < kGC; c += 16) {
                        if (base + c < ncols) {
                            uint32_t d[16];
                            __syncwarp();
                            tc::tmem_ld_32x32b_x16(d_tmem + base + c, d);
                            tc::tmem_ld_wait();
#pragma unroll
                            for (int i = 0; i < 16; i++) dreg[c + i] = (int)d[i];
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; i++) dreg[c + i] = 0;
                        }
                    }
                    if (!last) {
#pragma unroll
                        for (int c = 0; c < kGC; c += 4)
                            if (base + c < ncols)
                                __stcg(reinterpret_cast<int4*>(wrow + base + c),
                                       make_int4(dreg[c], dreg[c + 1], dreg[c + 2], dreg[c + 3]));
                        continue;
                    }
                    const int mend = min(kGT, p.M - mg);
#pragma unroll 1
                    for (int tt = 0; tt < mend; tt++) {
                        const int m = mg + tt;
                        long long ds[kDigits];
#pragma unroll
                        for (int i = 0; i < kDigits; i++) ds[i] = 0;
                        // this CTA's own sums (dreg is indexed with a run-time token: select by tt)
#pragma unroll
                        for (int u = 0; u < kGT; u++)
                            if (u == tt) {
#pragma unroll
                                for (int i = 0; i < kDigits; i++) ds[i] = dreg[u * kDigits + i];
                            }
                        // the other pieces, kPB at a time with all their loads in flight (more
                        // would spill registers)
                        constexpr int kPB = 4;
#pragma unroll 1
                        for (int j = j0; j <= j1; j += kPB) {
                            int vv[kPB][kDigits];
#pragma unroll
                            for (int u = 0; u < kPB; u++) {
                                const int jj = j + u;
                                if (jj <= j1 && jj != cta) {
                                    const int2* pj = reinterpret_cast<const int2*>(
                                        p.ws + ((size_t)sk::piece_slot(jj, tb, p.units, G) * kTileRows + r) * NC + m * kDigits);
#pragma unroll
                                    for (int i = 0; i < kDigits / 2; i++) {
                                        const int2 w = __ldcg(pj + i);
                                        vv[u][2 * i] = w.x;
                                        vv[u][2 * i + 1] = w.y;
                                    }
                                } else {
#pragma unroll
                                    for (int i = 0; i < kDigits; i++) vv[u][i] = 0;
                                }
                            }
#pragma unroll
                            for (int u = 0; u < kPB; u++)
#pragma unroll
                                for (int i = 0; i < kDigits; i++) ds[i] += vv[u][i];
                        }
                        const float vout = nv ? epi_out<OT>(p, m, n, recombine(ds, s_exps[m]), scale, bias, has_bias)
                                              : 0.0f;
                        if (p.amax_keys) {  // this warp's best output of token m, then the CTA's
                            unsigned long long key = nv ? argmax_key(vout, n) : 0ull;
                            for (int o = 16; o > 0; o >>= 1) {
                                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                                key = other > key ? other : key;
                            }
                            if (lane == 0) atomicMax(s_best + m, key);
                        }
                    }
                }
                if (last) {
                    if (!whole) {
                        asm volatile("bar.sync 1, 128;" ::: "memory");
                        if (etid == 0) p.counters[t] = 0;  // ready for the next launch
                    }
                    break;
                }
                // this piece's sums are out: count it in for the reducing piece
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (etid == 0) atomicAdd(p.counters + t, 1);
                break;
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(accempty0 + 8u * ab);  // accumulator drained
            seg++;
        }
        if (!ok) raise_error(abort);
        if (p.amax_keys) {  // this CTA's best per token into the launch's keys
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (etid < p.M && s_best[etid]) atomicMax(p.amax_keys + etid, s_best[etid]);
        }
        if (!p.early_trigger) pdl_launch_dependents();
    }

    // ---------------------------------------------------------------- teardown
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, C::kTmemCols);
    }
    if (p.amax_keys && threadIdx.x == 0) {
        // the launch's last CTA turns the keys into indices and leaves them zero again
        __threadfence();
        const unsigned int prev = atomicAdd(p.amax_done, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            for (int m = 0; m < p.M; m++) {
                const unsigned long long k = atomicExch(p.amax_keys + m, 0ull);
                p.amax_out[m] = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
            }
            *p.amax_done = 0;
        }
    }
}

// Completion of a gathered call (kernels.h, P2POut), launched behind its GEMV.  One thread:
// after the GEMV grid has completed (griddepcontrol.wait: its stores are performed), publish
// this call -- unless a bounded wait gave up somewhere in the digit GEMV, whose outputs are then
// invalid -- and/or wait for every rank's outputs of the calls so far.
__global__ void p2p_sync_kernel(const P2POut po, int publish, int wait)
{
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x != 0) return;
    if (publish) {
        int err;
        asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(err) : "l"(&g_kernel_error_i8) : "memory");
        if (err == 0) publish_share(po.counts, po.ndst, po.rank, 1ull << kCountShift);
    }
    if (wait && !wait_peers(po.wait_counts, po.wait_n, po.rank,
                            po.wait_timeout_ns ? po.wait_timeout_ns : kPeerTimeoutNs))
        atomicOr(&g_kernel_error_i8, 2);
}

// ----------------------------------------------------------------------------- host
// int8 [rows, K] row-major in [box_rows x 128 B] boxes, 128-byte swizzle, out-of-range reads 0.
bool make_i8_map(CUtensorMap* m, const void* base, size_t K, size_t rows, int box_rows)
{
    TmapDesc d{};
    d.base = base;
    d.inner = K;
    d.outer = rows;
    d.row_bytes = K;
    d.box_inner = 128;
    d.box_outer = (uint32_t)box_rows;
    d.dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    d.swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
    return tmap_2d(m, d);
}

// Grid size.  All SMs share HBM, so the stream needs enough of them (one SM pulls ~75 GB/s with
// its 3-stage ring), but every extra CTA on a tile is one more stream-K piece whose partial the
// reducing piece must fetch (four pieces per round trip of ~1 us).  Few-tile long-K shapes (a 7B
// down projection sharded 8 ways: 4 tiles of 37 K-stages) would otherwise split each tile into
// dozens of pieces; this takes the grid (all SMs, or a whole number of CTAs per tile) with the
// lowest estimated stream + fixup time, preferring more CTAs on ties.
long long pick_grid_i8(long long tiles, long long kbpt, long long weight_bytes, int num_sms)
{
    const long long units = tiles * kbpt;
    const long long all = units < num_sms ? units : num_sms;
    auto est = [&](long long G) {
        // B/s: ~60 GB/s per CTA in the decode step (with the L2 burst and the next projection's
        // CTAs on the idle SMs), up to HBM.  Measured on B200, the 7B down projection (28 row
        // tiles) inside the decode step: 84 CTAs 119.7-120.0 us per step, 112 CTAs 117.7-117.8,
        // 148 CTAs 118.7-119.0, 56 CTAs 123.5-123.6.
        const double bw = std::min(6.5e12, (double)G * 6.0e10);
        const long long pieces = (G + tiles - 1) / tiles;
        const double fix = pieces > 1 ? 1.0e-6 * (1.0 + (double)((pieces - 1 + 3) / 4)) : 0.0;
        return (double)weight_bytes / bw + fix;
    };
    long long best = all;
    double best_t = est(all);
    for (long long p = 1; tiles * p < all; p++) {
        const long long G = tiles * p;
        const double t = est(G);
        if (t < best_t * 0.97) {  // clearly better only: prefer the larger grid on near ties
            best = G;
            best_t = t;
        }
    }
    return best;
}

int pick_nc(size_t M)
{
    const int need = (int)(kDigits * M);
    return need <= 16 ? 16 : need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : 256;
}
int pick_bk_i8(int NC) { return NC <= 16 ? 512 : NC <= 64 ? 256 : 128; }

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (e == cudaSuccess) note_launch();
    return e;
}

template <int NC, int BK, int S, typename XT, typename OT>
cudaError_t launch_cfg(const LinearArgs& a, int num_sms, const TcScratch& sc, cudaStream_t stream)
{
    using C = DigCfg<NC, BK, S>;
    CUtensorMap mw;
    if (!make_i8_map(&mw, a.w, a.K, a.N, kTileRows)) return cudaErrorInvalidValue;
    auto kern = q8_gemv_dig_kernel<NC, BK, S, XT, OT>;
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
    DigParams p;
    p.x = a.x;
    p.scales = a.scales;
    p.bias = a.bias;
    p.res = a.res;
    p.out = a.out;
    // exps scratch: the prep kernel's words [M][ns]
    const int ns = row_splits((long long)a.K);
    p.prep_part = sc.exps;
    p.prep_splits = ns;
    p.dig_img = nullptr;
    p.fused_exps = gemv_i8_fused_exps(a) ? 1 : 0;
    p.amax_keys = a.amax_keys;
    p.amax_done = a.amax_done;
    p.amax_out = a.amax_out;
    p.ws = reinterpret_cast<int*>(sc.ws);
    p.counters = sc.counter_ptr;
    p.M = (int)a.M;
    p.N = (int)a.N;
    p.K = (int)a.K;
    p.kbpt = (int)((a.K + BK - 1) / BK);
    const long long tiles = (long long)((a.N + kTileRows - 1) / kTileRows);
    p.units = tiles * p.kbpt;
    if (a.p2p) {
        p.po = *a.p2p;
    } else {  // one local [M, N] output
        p.po = P2POut();
        p.po.ndst = a.out ? 1 : 0;  // no output copy: argmax only
        p.po.dst[0] = a.out;
        p.po.ldo = (long long)a.N;
        p.po.ocol0 = 0;
    }
    // Without in-kernel exponents the prep kernel reads x first: it pays the deferred wait.
    const unsigned long long* prep_wait = p.fused_exps ? nullptr : p.po.wait_counts;
    if (!p.fused_exps) p.po.wait_counts = nullptr;
    const int G = (int)pick_grid_i8(tiles, p.kbpt, (long long)a.N * (long long)a.K, num_sms);
    // Weight stages past the ring that each CTA asks L2 for when it starts.  With the early
    // trigger, CTAs that land on SMs the previous kernel leaves idle stream before that kernel
    // ends; a gathered call whose input is the previous call's gathered output keeps HBM busy
    // while it waits for the peers (up to 96 MB in all there, well inside L2).
    long long pf_bytes = (a.p2p && a.p2p->wait_counts) ? (96ll << 20) : kPrefetchBytes;
    p.early_trigger = 1;
    p.w_evict_first = 1;
#ifdef B200Q8_TRACE
    if (const char* v = getenv("B200Q8_TRACE_PF_MB")) pf_bytes = atoll(v) << 20;
    if (const char* v = getenv("B200Q8_TRACE_EARLY")) p.early_trigger = atoi(v);
    if (const char* v = getenv("B200Q8_TRACE_EVICT")) p.w_evict_first = atoi(v);
#endif
    p.prefetch_stages = 0;
    if (pf_bytes > 0) {
        const long long per_cta = (p.units + G - 1) / G;
        const long long budget = pf_bytes / ((long long)G * C::kWBytes);
        p.prefetch_stages = (int)std::max(0ll, std::min(per_cta - S, budget));
    }
    // A prologue: the prep kernel writes the activations once, the GEMV reads them as plain x.
    const bool materialize = a.prologue != kProNone;
    if ((long long)sc.ws_floats < 2LL * G * NC * kTileRows || (long long)sc.counters < tiles ||
        sc.exps_count < a.M * (size_t)ns || (materialize && sc.act_bytes < a.M * a.K * sizeof(XT)))
        return cudaErrorMemoryAllocation;
    if (materialize) p.x = sc.act;
    if constexpr (sizeof(XT) == 2) {
        if (gemv_i8_images(a)) {  // the prep kernel makes every stage's digit tile once
            if (sc.act_bytes < (size_t)p.kbpt * C::kDBytes || sc.exps_count < a.M * (size_t)p.kbpt)
                return cudaErrorMemoryAllocation;
            p.dig_img = sc.act;
            p.prep_splits = p.kbpt;
            e = launch_ex(digit_tiles_kernel<NC, BK>, dim3((unsigned)p.kbpt), dim3(kSqThreads), 0, stream, a.pdl,
                          reinterpret_cast<const __half*>(a.x), (int)a.M, (int)a.K, sc.exps, sc.act);
            if (e != cudaSuccess) return e;
            return launch_ex(kern, dim3((unsigned)G), dim3(kThreads), (size_t)C::kSmemBytes, stream, true, mw, p);
        }
    }
    if (p.fused_exps)  // one launch: the GEMV finds the exponents itself
        return launch_ex(kern, dim3((unsigned)G), dim3(kThreads), (size_t)C::kSmemBytes, stream, a.pdl, mw, p);
    e = launch_ex(exps_kernel<XT>, dim3((unsigned)a.M, (unsigned)ns), dim3(kSqThreads), 0, stream, a.pdl,
                  reinterpret_cast<const XT*>(a.x), (int)a.K, prep_wait, p.po.wait_n, p.po.rank,
                  p.po.wait_timeout_ns ? p.po.wait_timeout_ns : (unsigned long long)kPeerTimeoutNs, a.prologue,
                  a.norm_w, a.eps, sc.exps, materialize ? reinterpret_cast<XT*>(sc.act) : nullptr);
    if (e != cudaSuccess) return e;
    return launch_ex(kern, dim3((unsigned)G), dim3(kThreads), (size_t)C::kSmemBytes, stream, true, mw, p);
}

template <typename XT, typename OT>
cudaError_t launch_typed(const LinearArgs& a, int num_sms, const TcScratch& sc, cudaStream_t stream)
{
    switch (pick_nc(a.M)) {
        case 16: return launch_cfg<16, 512, 3, XT, OT>(a, num_sms, sc, stream);
        case 32: return launch_cfg<32, 256, 5, XT, OT>(a, num_sms, sc, stream);
        case 64: return launch_cfg<64, 256, 4, XT, OT>(a, num_sms, sc, stream);
        case 128: return launch_cfg<128, 128, 6, XT, OT>(a, num_sms, sc, stream);
        default: return launch_cfg<256, 128, 4, XT, OT>(a, num_sms, sc, stream);
    }
}

}  // namespace

int gemv_i8_max_tokens() { return kMaxTokens; }

bool gemv_i8_fused_exps(const LinearArgs& a)
{
    // A prologue is applied by the prep kernel, which writes the activations once.
    if (a.M > (size_t)kFusedExpTokens || a.prologue != kProNone || a.force_prep) return false;
    // fp16: the scan (Inf/NaN flags only) is the epilogue warps' alone, off the digits' path
    if (a.in_dtype == kF16 && a.M == 1 && a.K <= kFusedExpMaxKSmall) return true;
    return a.K <= kFusedExpMaxK || (a.N * a.K <= kInKernelScanMaxBytes && a.K <= kFusedExpMaxKSmall);
}

bool gemv_i8_images(const LinearArgs& a)
{
    // Several fp16 tokens (the prep kernel runs anyway): digit tiles made once per launch.  Not
    // for fp32 (the digits need the scanned exponents first), a prologue (its prep kernel
    // writes the activations), a gathered call, or the allocation-free entry.
    return a.in_dtype == kF16 && a.prologue == kProNone && !a.p2p && !a.force_prep && !a.no_digit_images &&
           !gemv_i8_fused_exps(a);
}

bool gemv_i8_supports(const LinearArgs& a)
{
    const size_t xa = a.in_dtype == kF16 ? 8 : 16;  // 4-element vector loads of x
    return a.M >= 1 && a.M <= (size_t)kMaxTokens && a.K % 16 == 0 && a.K >= 16 && a.K <= 131072 &&
           ((uintptr_t)a.w % 16) == 0 && ((uintptr_t)a.x % xa) == 0 && a.N >= 1 && a.N <= (size_t)INT32_MAX &&
           encode_fn() != nullptr;
}

void gemv_i8_scratch_need(const LinearArgs& a, int num_sms, size_t* ws_floats, size_t* counters, size_t* act_bytes,
                          size_t* exps)
{
    const int NC = pick_nc(a.M);
    const int BK = pick_bk_i8(NC);
    const long long tiles = (long long)((a.N + kTileRows - 1) / kTileRows);
    const long long G = pick_grid_i8(tiles, (long long)((a.K + BK - 1) / BK), (long long)a.N * (long long)a.K, num_sms);
    *ws_floats = (size_t)(2 * G * NC * kTileRows);
    *counters = (size_t)tiles;
    // the prologue's activations, when the prep kernel writes them for the GEMV
    const size_t kbpt = (a.K + BK - 1) / BK;
    if (gemv_i8_images(a)) {  // the digit tiles [kbpt][NC x BK bytes] and one word per token and stage
        *act_bytes = kbpt * (size_t)NC * (size_t)BK;
        *exps = a.M * kbpt;
        return;
    }
    *act_bytes = (a.prologue != kProNone && !gemv_i8_fused_exps(a)) ? a.M * a.K * (a.in_dtype == kF16 ? 2 : 4) : 0;
    *exps = a.M * (size_t)row_splits((long long)a.K);  // the prep kernel's words
}

cudaError_t launch_q8_gemv_i8(const LinearArgs& a, int num_sms, const TcScratch& sc, cudaStream_t stream)
{
    if (!gemv_i8_supports(a)) return cudaErrorNotSupported;
    if (a.in_dtype == kF16)
        return a.out_dtype == kF16 ? launch_typed<__half, __half>(a, num_sms, sc, stream)
                                   : launch_typed<__half, float>(a, num_sms, sc, stream);
    return a.out_dtype == kF16 ? launch_typed<float, __half>(a, num_sms, sc, stream)
                               : launch_typed<float, float>(a, num_sms, sc, stream);
}

int* p2p_error_word()
{
    static std::mutex mu;
    static int* word[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!word[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_kernel_error_i8) != cudaSuccess) return nullptr;
        word[dev] = static_cast<int*>(ptr);
    }
    return word[dev];
}

cudaError_t launch_p2p_sync(const P2POut& po, bool publish, bool wait, cudaStream_t stream)
{
    if (wait && !po.wait_counts) return cudaErrorInvalidValue;
    return launch_ex(p2p_sync_kernel, dim3(1), dim3(32), 0, stream, true, po, publish ? 1 : 0, wait ? 1 : 0);
}

cudaError_t read_kernel_error_i8(int* code, bool clear)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_kernel_error_i8, sizeof(int));
    if (e != cudaSuccess) return e;
    *code = v;
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_kernel_error_i8, &z, sizeof(int));
    }
    return e;
}

// ============================================================================
// Allocation-free variant of the int8 digit GEMV (b200q8_linear_q8_noalloc).
//
// Some callers may not call cudaMalloc: hosts whose device memory belongs to a
// pool or budget that nothing may bypass (vvllm's own tensors come from a
// caching pool, src/tensor/tensor.cc:35-68), and latency-critical decode loops
// that cannot take the device-wide synchronisation cudaMalloc and cudaFree may
// cause.  The regular entry points allocate their stream-K scratch lazily;
// this one uses a fixed file-scope device array instead, so it allocates
// nothing.  Every GPU that loads the library holds the array (kNoAllocBytes,
// about 2.6 MB) until the process exits.  All calls share it and it keeps the
// last call's contents; the tile counters, which must start at zero, are
// cleared by every call.  Calls that overlap on one GPU (for example on two
// streams) race on the array and must be serialised by the caller; each GPU
// has its own copy.
// ============================================================================
namespace {

constexpr int kNoAllocMaxTokens = 2;      // 6 digit rows per token: NC = 16
constexpr int kNoAllocMaxCtas = 160;      // stream-K CTAs (a B200 has 148 SMs)
constexpr int kNoAllocMaxTiles = 4096;    // 128-row tiles: N <= 524288
constexpr size_t kNoAllocPartialInts = (size_t)2 * kNoAllocMaxCtas * kTileRows * 16;
constexpr size_t kNoAllocExps = 256;  // the prep kernel's words: 2 tokens x up to 64 splits
constexpr size_t kNoAllocBytes = (kNoAllocPartialInts + kNoAllocMaxTiles + kNoAllocExps) * sizeof(int);

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_base[64];

// Device address of the array on the current device, looked up once per device
// (the first call on a device does this set-up).
cudaError_t noalloc_base(int dev, void** out)
{
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_base[dev] = p;
    }
    *out = g_noalloc_base[dev];
    return cudaSuccess;
}

}  // namespace

// Returns 0 and launches, or a reason the shape exceeds the array's limits
// (1: tokens, 2: rows, 3: SM count, 4: K / alignment, 5: scratch beyond the array),
// or -1 with *err set.
int launch_q8_gemv_i8_noalloc(const LinearArgs& a, int num_sms, cudaStream_t stream, cudaError_t* err)
{
    *err = cudaSuccess;
    if (a.M > (size_t)kNoAllocMaxTokens) return 1;
    const size_t tiles = (a.N + kTileRows - 1) / kTileRows;
    if (tiles > (size_t)kNoAllocMaxTiles) return 2;
    if (num_sms > kNoAllocMaxCtas) return 3;
    if (!gemv_i8_supports(a)) return 4;
    int dev = 0;
    if ((*err = cudaGetDevice(&dev)) != cudaSuccess) return -1;
    if (dev < 0 || dev >= 64) {
        *err = cudaErrorInvalidDevice;
        return -1;
    }
    // The limits above keep every grid the launch can pick inside the array; check it anyway,
    // so a shape outside it is refused as such rather than reported as a failed allocation.
    LinearArgs b = a;
    b.no_digit_images = true;  // no scratch for digit tiles here
    size_t need_ws = 0, need_ctr = 0, need_act = 0, need_exps = 0;
    gemv_i8_scratch_need(b, num_sms, &need_ws, &need_ctr, &need_act, &need_exps);
    if (need_ws > kNoAllocPartialInts || need_ctr > (size_t)kNoAllocMaxTiles || need_exps > kNoAllocExps ||
        need_act > 0)
        return 5;
    void* base = nullptr;
    if ((*err = noalloc_base(dev, &base)) != cudaSuccess) return -1;
    TcScratch sc;
    sc.ws = reinterpret_cast<float*>(base);
    sc.ws_floats = kNoAllocPartialInts;
    sc.counter_ptr = reinterpret_cast<int*>(base) + kNoAllocPartialInts;
    sc.counters = kNoAllocMaxTiles;
    sc.exps = sc.counter_ptr + kNoAllocMaxTiles;
    sc.exps_count = kNoAllocExps;
    // the counters must start at zero: clear the ones this call uses (no allocation)
    if ((*err = cudaMemsetAsync(sc.counter_ptr, 0, tiles * sizeof(int), stream)) != cudaSuccess) return -1;
    *err = launch_q8_gemv_i8(b, num_sms, sc, stream);
    return *err == cudaSuccess ? 0 : -1;
}

}  // namespace b200q8
