// q8_gemv.cu -- HBM-streaming int8-weight GEMV for small token counts (M = 1..4).
//
// out[m, n] = (sum_k x[m, k] * float(W[n, k])) * scales[n] + bias[n] (+ res[m, n])
//
// Semantics follow vvllm's BackendCPU::linear_q8 / linear_q8_add
// (src/backend/backend_naive.cc:155-291, :322-335); the reference's own GPU
// path instead dequantizes W to an fp16 copy and calls cuBLAS
// (src/backend/backend_cuda.cc:188-213), reading 2 bytes per weight.  This
// kernel reads each int8 weight byte exactly once from HBM.
//
// Design (sm_100a):
//  * A CTA is 8 warps = RW row slots x KW K-slices (RW * KW = 8).  A warp owns
//    R consecutive weight rows and one contiguous K-slice of them; lanes take
//    16-byte chunks of that slice round-robin, so every warp load instruction
//    covers 512 contiguous bytes of one row.  U chunks per row are issued
//    before any is consumed (R * U * 16 bytes in flight per lane).
//  * The activation rows (M x K) are staged once per CTA in shared memory as
//    fp32, in a chunk-transposed layout (float4 index (t*4 + q) * C + c for
//    chunk c, quarter q) so the per-lane float4 reads are bank-conflict free.
//    fp16 activations are widened exactly while staging.
//  * int8 -> fp32 uses the exponent-bias trick (PRMT + packed FADD2) and the
//    dot product uses sm_100 packed FFMA2, two fp32 FMAs per instruction.
//  * Partial sums: warp shuffle reduction, then (KW > 1) a fixed-order sum of
//    the KW slices through shared memory, double-buffered so one named
//    barrier per row group suffices.  Results are deterministic.
//  * The grid is persistent: blocks loop over row groups with a grid stride.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "p2p.cuh"
#include "prologue.cuh"

namespace b200q8 {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct GemvParams {
    const void* x;       // [M, ldx] fp32 or fp16
    const int8_t* w;     // [N, K]
    const float* scales; // [N]
    const float* bias;   // [N] or null
    const void* res;     // [M, ldo] (OT) or null
    void* out;           // [M, ldo] (OT)
    long long ldx, ldo;
    int N, K, M;         // M <= MT
    int KW;              // K slices per CTA (1, 2, 4, 8)
    int pro;             // prologue applied while x is staged (prologue.cuh); x rows are ldx apart
    const float* norm_w;
    float eps;
    // The streaming kernel reads its matrices from these arrays: nmat projections of the same x
    // (1 for a single one, where [0] repeats w / scales / bias / out / N above), matrix i with
    // Nm[i] rows, its own weights, scales, bias and [M, Nm[i]] output, and row groups
    // gofs[i] .. gofs[i+1] (gofs set at launch).
    int nmat;
    const int8_t* wm[kMaxGroup];
    const float* sm[kMaxGroup];
    const float* bm[kMaxGroup];
    void* om[kMaxGroup];
    int Nm[kMaxGroup];
    int gofs[kMaxGroup + 1];
    // Column-sharded gather (b200q8_linear_q8_sharded_p2p, one matrix): with ndst > 0 the output
    // of row `row` for token t goes to dsts[d][t * ldo + ocol0 + row] on each of the ndst ranks
    // instead of om[0]; with wait_counts set, every rank's part of the previous gathered call (x)
    // must have landed before x is read (p2p.cuh), else bit 1 of *err.
    int ndst, ocol0;
    void* dsts[kMaxRanks];
    const unsigned long long* wait_counts;
    int wait_n, wait_rank;
    unsigned long long wait_ns;
    int* err;
};

// out = acc * scale (+ bias) (+ res), into the projection's own output, or -- gathered -- into
// every rank's copy of the full output.
template <typename OT>
__device__ __forceinline__ void store_result(const GemvParams& p, int mi, int t, int row, const OT* res, float acc)
{
    if (p.ndst == 0) {
        const long long o = (long long)t * p.Nm[mi] + row;
        epilogue_store<OT>(reinterpret_cast<OT*>(p.om[mi]) + o, res ? res + o : nullptr, acc, p.sm[mi][row], p.bm[mi],
                           row);
        return;
    }
    float v = __fmul_rn(acc, p.sm[mi][row]);
    if (p.bm[mi]) v = __fadd_rn(v, p.bm[mi][row]);
    const long long o = (long long)t * p.ldo + p.ocol0 + row;
    for (int d = 0; d < p.ndst; d++) store_from_f32<OT>(reinterpret_cast<OT*>(p.dsts[d]) + o, v);
}

// The matrix row group g belongs to.  Only this index and the group's offset stay in registers
// across the streaming loop; the matrix's pointers are read from the parameters where used.
__device__ __forceinline__ int group_matrix(const GemvParams& p, int g)
{
    int i = 0;
#pragma unroll
    for (int j = 1; j < kMaxGroup; j++)
        if (j < p.nmat && g >= p.gofs[j]) i = j;
    return i;
}
static_assert(kThreads == kSqThreads, "the prologue's fixed-order sum is taken by one 256-thread CTA");

template <typename XT>
__device__ __forceinline__ void stage_x(float4* xs4, const XT* x, long long ldx, int M, int K);

// fp32: one float4 per thread-step; chunk c = idx / 4, quarter q = idx % 4.
template <>
__device__ __forceinline__ void stage_x<float>(float4* xs4, const float* x, long long ldx, int M,
                                               int K)
{
    const int C = K >> 4;
    const int n4 = K >> 2;
    for (int t = 0; t < M; t++) {
        const float4* src = reinterpret_cast<const float4*>(x + (long long)t * ldx);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const int c = i >> 2, q = i & 3;
            xs4[(t * 4 + q) * C + c] = src[i];
        }
    }
}

// fp16: eight halves per thread-step (quarters 2h and 2h+1 of chunk c).
template <>
__device__ __forceinline__ void stage_x<__half>(float4* xs4, const __half* x, long long ldx,
                                                int M, int K)
{
    const int C = K >> 4;
    const int n8 = K >> 3;
    for (int t = 0; t < M; t++) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
        for (int i = threadIdx.x; i < n8; i += blockDim.x) {
            const uint4 v = src[i];
            const int c = i >> 1, h = i & 1;
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
            const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
            xs4[(t * 4 + 2 * h) * C + c] = make_float4(a.x, a.y, b.x, b.y);
            xs4[(t * 4 + 2 * h + 1) * C + c] = make_float4(d.x, d.y, e.x, e.y);
        }
    }
}

// The prologue's activations staged like stage_x<float> stages x: the same act4 values the fused
// digit GEMV and the standalone prologue kernel compute (the token's rms from the shared
// fixed-order sum of this 256-thread CTA), so the projection equals the standalone op followed
// by the plain GEMV bit for bit.
// (Out of line: it runs once per CTA and must not take registers from the streaming loop.)
template <typename XT>
__device__ __noinline__ void stage_x_pro(float4* xs4, const XT* x, long long ldx, int M, int K, int pro,
                                         const float* norm_w, float eps)
{
    __shared__ double sq[kSqWarps];
    const int C = K >> 4;
    const int g4 = K >> 2;
    for (int t = 0; t < M; t++) {
        const XT* xrow = x + (long long)t * ldx;
        float rms = 1.0f;
        if (pro == kProRmsNorm) {
            const double w = sumsq_warp<XT>(xrow, K, threadIdx.x);
            if ((threadIdx.x & 31) == 0) sq[threadIdx.x >> 5] = w;
            __syncthreads();
            rms = rms_from(sq, K, eps);
            __syncthreads();  // sq is reused by the next token
        }
        for (int i0 = threadIdx.x; i0 < g4; i0 += 2 * kThreads) {
            float v[2][4], aux[2][4];
#pragma unroll
            for (int b = 0; b < 2; b++)  // both groups' loads first
                if (i0 + b * kThreads < g4) act4_load<XT>(pro, xrow, K, 4 * (i0 + b * kThreads), norm_w, v[b], aux[b]);
#pragma unroll
            for (int b = 0; b < 2; b++) {
                const int i = i0 + b * kThreads;
                if (i < g4) {
                    act4_apply<XT>(pro, rms, v[b], aux[b]);
                    xs4[(t * 4 + (i & 3)) * C + (i >> 2)] = make_float4(v[b][0], v[b][1], v[b][2], v[b][3]);
                }
            }
        }
    }
}

// acc += dot(16 int8 weights in `wv`, 16 fp32 activations x0..x3)
__device__ __forceinline__ void fma_chunk(float2& acc0, float2& acc1, const uint4& wv,
                                          const float4& x0, const float4& x1, const float4& x2,
                                          const float4& x3)
{
    float2 w0, w1;
    i8x4_to_f32x4(wv.x, w0, w1);
    acc0 = __ffma2_rn(w0, make_float2(x0.x, x0.y), acc0);
    acc1 = __ffma2_rn(w1, make_float2(x0.z, x0.w), acc1);
    i8x4_to_f32x4(wv.y, w0, w1);
    acc0 = __ffma2_rn(w0, make_float2(x1.x, x1.y), acc0);
    acc1 = __ffma2_rn(w1, make_float2(x1.z, x1.w), acc1);
    i8x4_to_f32x4(wv.z, w0, w1);
    acc0 = __ffma2_rn(w0, make_float2(x2.x, x2.y), acc0);
    acc1 = __ffma2_rn(w1, make_float2(x2.z, x2.w), acc1);
    i8x4_to_f32x4(wv.w, w0, w1);
    acc0 = __ffma2_rn(w0, make_float2(x3.x, x3.y), acc0);
    acc1 = __ffma2_rn(w1, make_float2(x3.z, x3.w), acc1);
}

template <int MT, int R, int U, typename XT, typename OT>
__global__ void __launch_bounds__(kThreads) q8_gemv_kernel(const GemvParams p)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float4* xs4 = reinterpret_cast<float4*>(smem_raw);
    // partial-sum exchange: [2 buffers][kWarps][MT * R]
    float* red = reinterpret_cast<float*>(smem_raw + (size_t)MT * p.K * sizeof(float));

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int KW = p.KW;
    const int RW = kWarps / KW;
    const int kw = warp % KW;
    const int rw = warp / KW;
    const int C = p.K >> 4;
    const int c_begin = (int)((long long)kw * C / KW);
    const int c_end = (int)((long long)(kw + 1) * C / KW);
    const int rows_per_cta = RW * R;
    // a group of projections numbers its row groups matrix by matrix (offsets set at launch)
    const int num_groups = p.gofs[p.nmat];

    // The weights do not depend on the previous kernel in the stream, x does: pull this CTA's
    // row groups (each one contiguous range of rows_per_cta rows, 16-byte aligned on this path;
    // at most 48 MiB in all, inside L2) into L2 while that kernel -- or, for a gathered call,
    // the peers -- finish, then wait.
    if (threadIdx.x == 0) {
        for (int g = blockIdx.x; g < num_groups; g += gridDim.x) {
            const int mi = group_matrix(p, g);
            const int r0 = (g - p.gofs[mi]) * rows_per_cta;
            const int nr = min(rows_per_cta, p.Nm[mi] - r0);
            const unsigned bytes = (unsigned)((long long)nr * p.K);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.wm[mi] + (long long)r0 * p.K),
                         "r"(bytes)
                         : "memory");
        }
    }
    pdl_wait();
    if (p.wait_counts) {  // x is the gathered output of the previous call: every rank's part landed
        if (threadIdx.x == 0 && !wait_peers(p.wait_counts, p.wait_n, p.wait_rank, p.wait_ns)) atomicOr(p.err, 2);
        __syncthreads();
    }
    if (p.pro != kProNone)
        stage_x_pro<XT>(xs4, reinterpret_cast<const XT*>(p.x), p.ldx, p.M, p.K, p.pro, p.norm_w, p.eps);
    else
        stage_x<XT>(xs4, reinterpret_cast<const XT*>(p.x), p.ldx, p.M, p.K);
    __syncthreads();
    pdl_launch_dependents();

    const OT* res = reinterpret_cast<const OT*>(p.res);  // single projections only (ldo = N)

    int iter = 0;
    for (int g = blockIdx.x; g < num_groups; g += gridDim.x, iter++) {
        const int mi = group_matrix(p, g);
        const int row0 = (g - p.gofs[mi]) * rows_per_cta + rw * R;
        const int8_t* wrow[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int row = min(row0 + r, p.Nm[mi] - 1);  // tail rows re-read a valid row; never stored
            wrow[r] = p.wm[mi] + (long long)row * p.K;
        }

        float2 acc[MT][R][2];
#pragma unroll
        for (int t = 0; t < MT; t++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[t][r][0] = acc[t][r][1] = make_float2(0.f, 0.f);

        for (int c0 = c_begin + lane; c0 < c_end; c0 += 32 * U) {
            uint4 wv[U][R];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = c0 + 32 * u;
#pragma unroll
                for (int r = 0; r < R; r++)
                    wv[u][r] = (c < c_end) ? ldg_stream16(wrow[r] + (long long)c * 16)
                                           : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = c0 + 32 * u;
                if (c < c_end) {
#pragma unroll
                    for (int t = 0; t < MT; t++) {
                        if (t < p.M) {
                            const float4 x0 = xs4[(t * 4 + 0) * C + c];
                            const float4 x1 = xs4[(t * 4 + 1) * C + c];
                            const float4 x2 = xs4[(t * 4 + 2) * C + c];
                            const float4 x3 = xs4[(t * 4 + 3) * C + c];
#pragma unroll
                            for (int r = 0; r < R; r++)
                                fma_chunk(acc[t][r][0], acc[t][r][1], wv[u][r], x0, x1, x2, x3);
                        }
                    }
                }
            }
        }

        // Reduce: lanes -> warp, then K-slices -> row slot.
        float v[MT][R];
#pragma unroll
        for (int t = 0; t < MT; t++)
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float s = (acc[t][r][0].x + acc[t][r][0].y) + (acc[t][r][1].x + acc[t][r][1].y);
                v[t][r] = warp_sum(s);
            }

        if (KW == 1) {
#pragma unroll
            for (int t = 0; t < MT; t++)
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int row = row0 + r;
                    if (lane == t * R + r && t < p.M && row < p.Nm[mi]) store_result<OT>(p, mi, t, row, res, v[t][r]);
                }
        } else {
            float* buf = red + ((iter & 1) * kWarps + warp) * (MT * R);
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < MT; t++)
#pragma unroll
                    for (int r = 0; r < R; r++) buf[t * R + r] = v[t][r];
            }
            // named barrier over the KW warps of this row slot
            asm volatile("bar.sync %0, %1;" ::"r"(1 + rw), "r"(KW * 32) : "memory");
            if (kw == 0 && lane < MT * R) {
                const int t = lane / R, r = lane % R;
                const int row = row0 + r;
                if (t < p.M && row < p.Nm[mi]) {
                    const float* base = red + ((iter & 1) * kWarps + rw * KW) * (MT * R);
                    float s = 0.f;
                    for (int k = 0; k < KW; k++) s += base[k * (MT * R) + lane];
                    store_result<OT>(p, mi, t, row, res, s);
                }
            }
        }
    }
}

// Generic path for shapes the streaming kernel does not take (K % 16 != 0 or
// misaligned pointers): one warp per (token, row), scalar loads, the same
// epilogue.  Correct for any K; used only off the configured shapes.
template <typename XT, typename OT>
__global__ void __launch_bounds__(256) q8_gemv_generic_kernel(const GemvParams p)
{
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const long long total = (long long)p.M * p.N;
    const XT* x = reinterpret_cast<const XT*>(p.x);
    const OT* res = reinterpret_cast<const OT*>(p.res);
    OT* out = reinterpret_cast<OT*>(p.out);
    for (long long e = gw; e < total; e += (long long)gridDim.x * 8) {
        const int t = (int)(e / p.N), row = (int)(e % p.N);
        const int8_t* wr = p.w + (long long)row * p.K;
        const XT* xr = x + (long long)t * p.ldx;
        float s = 0.f;
        for (int k = lane; k < p.K; k += 32) s = fmaf(load_as_f32<XT>(xr + k), (float)wr[k], s);
        s = warp_sum(s);
        if (lane == 0) {
            const long long o = (long long)t * p.ldo + row;
            epilogue_store<OT>(out + o, res ? res + o : nullptr, s, p.scales[row], p.bias, row);
        }
    }
}

template <typename Kern>
cudaError_t launch(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   const GemvParams& p, bool pdl)
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e == cudaSuccess) note_launch();
    return e;
}

template <int MT, int R, int U, typename XT, typename OT>
cudaError_t launch_stream_kernel(const GemvParams& p, int num_sms, cudaStream_t stream, bool pdl)
{
    auto kern = q8_gemv_kernel<MT, R, U, XT, OT>;
    const size_t smem = (size_t)MT * p.K * sizeof(float) + 2 * kWarps * MT * R * sizeof(float);
    // Per (template instance, thread, device): the largest dynamic smem opted into so far, and
    // the occupancy computed for the last smem size.
    struct Cfg {
        int configured_smem = 0, occ_smem = -1, per_sm = 0;
    };
    static thread_local Cfg cfgs[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    Cfg& c = cfgs[dev];
    if ((int)smem > c.configured_smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        c.configured_smem = (int)smem;
    }
    if (c.occ_smem != (int)smem) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c.per_sm, kern, kThreads, smem);
        if (e != cudaSuccess) return e;
        c.occ_smem = (int)smem;
    }
    const int per_sm = c.per_sm;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int rows_per_cta = (kWarps / p.KW) * R;
    GemvParams pg = p;  // row groups numbered matrix by matrix
    pg.gofs[0] = 0;
    for (int i = 0; i < p.nmat; i++) pg.gofs[i + 1] = pg.gofs[i] + (p.Nm[i] + rows_per_cta - 1) / rows_per_cta;
    const long long groups = pg.gofs[p.nmat];
    long long grid = (long long)per_sm * num_sms;
    if (groups < grid) grid = groups;
    return launch(kern, dim3((unsigned)grid), dim3(kThreads), smem, stream, pg, pdl);
}

template <typename XT, typename OT>
cudaError_t dispatch_typed(const GemvParams& p0, int num_sms, cudaStream_t stream, bool pdl)
{
    GemvParams p = p0;
    const int C = p.K >> 4;
    // K split: aim for >= 2 chunks per lane per slice, up to 8 slices.
    int KW = 1;
    while (KW < 8 && C / (KW * 2) >= 64) KW *= 2;
    // Few rows: split K harder so enough warps stream concurrently -- but not past 4 slices on
    // rows of 4096 and longer (Qwen2.5-0.5B down, 896 x 4864: 8 slices 4.66 us, 4 slices 4.19 us).
    while (KW < 8 && (long long)p.N * KW < 64LL * num_sms && C / (KW * 2) >= 16 && !(KW >= 4 && p.K >= 4096))
        KW *= 2;
    bool small_n = (long long)p.N < 4LL * num_sms * (8 / KW);
    // Few rows on a long K (the 7B down projection's shard at 8 GPUs, 448 x 18944): one row per
    // CTA would stage all of x in every CTA; four rows per CTA (K split 4, two rows per warp)
    // measured 8.07 -> 6.32 us on B200.
    if (p.M == 1 && KW == 8 && small_n && p.K >= 8192) {
        KW = 4;
        small_n = false;
    }
    p.KW = KW;
    const int chunks_per_lane = (C / KW + 31) / 32;
    if (p.M == 1) {
        if (small_n)
            return chunks_per_lane <= 2 ? launch_stream_kernel<1, 1, 2, XT, OT>(p, num_sms, stream, pdl)
                                        : launch_stream_kernel<1, 1, 4, XT, OT>(p, num_sms, stream, pdl);
        return chunks_per_lane <= 2 ? launch_stream_kernel<1, 2, 2, XT, OT>(p, num_sms, stream, pdl)
                                    : launch_stream_kernel<1, 2, 4, XT, OT>(p, num_sms, stream, pdl);
    }
    if (p.M == 2) return launch_stream_kernel<2, 2, 2, XT, OT>(p, num_sms, stream, pdl);
    return launch_stream_kernel<4, 1, 2, XT, OT>(p, num_sms, stream, pdl);
}

template <typename XT, typename OT>
cudaError_t dispatch_generic(const GemvParams& p, cudaStream_t stream, bool pdl)
{
    const long long warps = (long long)p.M * p.N;
    long long blocks = (warps + 7) / 8;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    return launch(q8_gemv_generic_kernel<XT, OT>, dim3((unsigned)blocks), dim3(256), 0, stream, p,
                  pdl);
}

}  // namespace

int gemv_max_tokens() { return 4; }

size_t gemv_smem_bytes(int M, int K) { return (size_t)M * K * sizeof(float) + 2 * kWarps * 8 * sizeof(float); }

bool gemv_stream_supports(const LinearArgs& a, size_t max_smem)
{
    const size_t xbytes = a.in_dtype == kF16 ? 2 : 4;
    const bool aligned = (a.K % 16 == 0) && ((uintptr_t)a.w % 16 == 0) && ((uintptr_t)a.x % 16 == 0) &&
                         ((a.K * xbytes) % 16 == 0) && (a.prologue != kProRmsNorm || (uintptr_t)a.norm_w % 16 == 0);
    const int mt = a.M <= 1 ? 1 : (a.M == 2 ? 2 : 4);
    return aligned && a.M <= 4 && a.K <= (size_t)INT32_MAX && gemv_smem_bytes(mt, (int)a.K) <= max_smem;
}

cudaError_t launch_q8_gemv(const LinearArgs& a, int num_sms, size_t max_smem, cudaStream_t stream)
{
    GemvParams p{};
    p.x = a.x;
    p.w = a.w;
    p.scales = a.scales;
    p.bias = a.bias;
    p.res = a.res;
    p.out = a.out;
    p.ldx = a.prologue == kProSiluMul ? 2 * (long long)a.K : (long long)a.K;
    p.ldo = a.N;
    p.N = (int)a.N;
    p.K = (int)a.K;
    p.M = (int)a.M;
    p.KW = 1;
    p.pro = a.prologue;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.nmat = 1;
    p.wm[0] = p.w;
    p.sm[0] = p.scales;
    p.bm[0] = p.bias;
    p.om[0] = p.out;
    p.Nm[0] = p.N;
    if (a.p2p) {  // the gathered call: the streaming kernel only
        if (!gemv_stream_supports(a, max_smem) || a.M > 4 || a.res) return cudaErrorNotSupported;
        p.ndst = a.p2p->ndst;
        for (int d = 0; d < a.p2p->ndst; d++) p.dsts[d] = a.p2p->dst[d];
        p.ldo = a.p2p->ldo;
        p.ocol0 = a.p2p->ocol0;
        p.wait_counts = a.p2p->wait_counts;
        p.wait_n = a.p2p->wait_n;
        p.wait_rank = a.p2p->rank;
        p.wait_ns = a.p2p->wait_timeout_ns ? a.p2p->wait_timeout_ns : 2000000000ull;
        if (!(p.err = p2p_error_word())) return cudaErrorInvalidSymbol;
    }
    const bool x16 = (a.in_dtype == kF16);
    const bool o16 = (a.out_dtype == kF16);
    if (gemv_stream_supports(a, max_smem)) {
        if (x16) return o16 ? dispatch_typed<__half, __half>(p, num_sms, stream, a.pdl)
                            : dispatch_typed<__half, float>(p, num_sms, stream, a.pdl);
        return o16 ? dispatch_typed<float, __half>(p, num_sms, stream, a.pdl)
                   : dispatch_typed<float, float>(p, num_sms, stream, a.pdl);
    }
    if (a.prologue != kProNone) return cudaErrorNotSupported;  // the generic kernel reads plain x
    if (x16) return o16 ? dispatch_generic<__half, __half>(p, stream, a.pdl)
                        : dispatch_generic<__half, float>(p, stream, a.pdl);
    return o16 ? dispatch_generic<float, __half>(p, stream, a.pdl)
               : dispatch_generic<float, float>(p, stream, a.pdl);
}

cudaError_t launch_q8_gemv_group(const LinearArgs& a, int n, const int8_t* const* w, const float* const* scales,
                                 const float* const* bias, void* const* outs, const size_t* Ns, int num_sms,
                                 size_t max_smem, cudaStream_t stream)
{
    if (n < 1 || n > kMaxGroup) return cudaErrorInvalidValue;
    LinearArgs b = a;
    size_t total = 0;
    for (int i = 0; i < n; i++) {
        b.w = w[i];
        if (!gemv_stream_supports(b, max_smem) || Ns[i] == 0 || Ns[i] > (size_t)INT32_MAX) return cudaErrorNotSupported;
        total += Ns[i];
    }
    if (total > (size_t)INT32_MAX) return cudaErrorNotSupported;
    GemvParams p{};
    p.x = a.x;
    p.w = w[0];
    p.scales = scales[0];
    p.bias = bias[0];
    p.res = nullptr;
    p.out = outs[0];
    p.ldx = a.prologue == kProSiluMul ? 2 * (long long)a.K : (long long)a.K;
    p.ldo = (long long)Ns[0];
    p.N = (int)total;  // the dispatch heuristics see the group's rows
    p.K = (int)a.K;
    p.M = (int)a.M;
    p.KW = 1;
    p.pro = a.prologue;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.nmat = n;
    for (int i = 0; i < n; i++) {
        p.wm[i] = w[i];
        p.sm[i] = scales[i];
        p.bm[i] = bias[i];
        p.om[i] = outs[i];
        p.Nm[i] = (int)Ns[i];
    }
    const bool x16 = (a.in_dtype == kF16);
    const bool o16 = (a.out_dtype == kF16);
    if (x16) return o16 ? dispatch_typed<__half, __half>(p, num_sms, stream, a.pdl)
                        : dispatch_typed<__half, float>(p, num_sms, stream, a.pdl);
    return o16 ? dispatch_typed<float, __half>(p, num_sms, stream, a.pdl)
               : dispatch_typed<float, float>(p, num_sms, stream, a.pdl);
}

}  // namespace b200q8
