// b200q8_api.cu -- the extern "C" boundary (include/b200q8.h) over the sm_100a kernels.
//
// Host C++20.  No entry point exits the process or falls back to the CPU:
// every failure becomes a negative status plus a thread-local message.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "b200q8.h"
#include "kernels.h"
#include "prologue.cuh"

namespace b200q8 {

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

thread_local std::string t_last_error;

// Records the message for b200q8_last_error() and returns status.
int fail(int status, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char* what)
{
    return fail(B200Q8_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {

struct DeviceInfo {
    int num_sms = 0;
    size_t max_smem = 0;  // opt-in dynamic shared memory per block
    int cc_major = 0, cc_minor = 0;
    bool valid = false;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo* out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(B200Q8_ERR_UNSUPPORTED, "device %d out of range", dev);
    if (!g_dev[dev].valid) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (!g_dev[dev].valid) {
            DeviceInfo d;
            int v = 0;
            if ((e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
                return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
            if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
                return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
            d.max_smem = (size_t)v;
            cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
            cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
            d.valid = true;
            g_dev[dev] = d;
        }
    }
    *out = g_dev[dev];
    if (out->cc_major != 10)
        return fail(B200Q8_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only",
                    dev, out->cc_major, out->cc_minor);
    return B200Q8_OK;
}

bool valid_dtype(int d) { return d == B200Q8_F32 || d == B200Q8_F16; }

// Stream-K scratch of the tensor-core GEMM, one per (device, stream): launches
// on one stream are ordered, so they may share it; different streams may run
// concurrently, so they do not.  Allocated on first use (outside any graph
// capture) and grown when a larger shape needs more; never shrunk.
struct ScratchKey {
    int dev;
    cudaStream_t stream;
    bool operator==(const ScratchKey& o) const { return dev == o.dev && stream == o.stream; }
};
struct ScratchKeyHash {
    size_t operator()(const ScratchKey& k) const
    {
        return std::hash<uintptr_t>()((uintptr_t)k.stream) * 31u + (size_t)k.dev;
    }
};
std::mutex g_scratch_mu;
std::unordered_map<ScratchKey, TcScratch, ScratchKeyHash> g_scratch;

struct ScratchNeed {
    size_t ws = 0, counters = 0, exps = 0, act = 0;
    bool amax = false;
};

// Grows one device buffer of `s` to at least `need` elements (never shrinks).
template <typename T>
int grow(T** buf, size_t* have, size_t need, size_t dflt, cudaStream_t stream, bool zero, const char* what)
{
    if (*have >= need) return B200Q8_OK;
    const size_t n = need > dflt ? need : dflt;
    T* nb = nullptr;
    cudaError_t e = cudaMalloc(&nb, n * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(B200Q8_ERR_ALLOC, "scratch %s: cudaMalloc(%zu): %s", what, n * sizeof(T), cudaGetErrorString(e));
    }
    if (zero && (e = cudaMemsetAsync(nb, 0, n * sizeof(T), stream)) != cudaSuccess) {
        cudaFree(nb);
        return cuda_fail(e, "scratch memset");
    }
    if (*buf) {  // the old buffer may still be in use by queued work on this stream
        cudaStreamSynchronize(stream);
        cudaFree(*buf);
    }
    *buf = nb;
    *have = n;
    return B200Q8_OK;
}

int get_scratch(const ScratchNeed& need, int num_sms, cudaStream_t stream, TcScratch* out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    TcScratch& s = g_scratch[ScratchKey{dev, stream}];
    // Default capacities: 128-column partials on every SM, 64K tiles.
    int st;
    if ((st = grow(&s.ws, &s.ws_floats, need.ws, (size_t)2 * num_sms * 128 * 128, stream, false, "partials")) ||
        (st = grow(&s.counter_ptr, &s.counters, need.counters, (size_t)1 << 16, stream, true, "counters")) ||
        (st = grow(&s.exps, &s.exps_count, need.exps, (size_t)320, stream, false, "exponent words")) ||
        (st = grow(&s.act, &s.act_bytes, need.act, 0, stream, false, "prologue activations")))
        return st;
    if (need.amax && !s.amax) {  // argmax keys + done counter, zero at rest
        size_t have = 0;
        if ((st = grow(&s.amax, &have, (size_t)kMaxArgmaxTokens + 1, 0, stream, true, "argmax")))
            return st;
    }
    *out = s;
    return B200Q8_OK;
}

// After a bounded wait gave up, tile counters may be left non-zero: reset them.
int reset_scratch_counters(int dev)
{
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (auto& kv : g_scratch) {
        if (kv.first.dev != dev) continue;
        cudaError_t e = cudaSuccess;
        if (kv.second.counter_ptr) e = cudaMemset(kv.second.counter_ptr, 0, kv.second.counters * sizeof(int));
        if (e == cudaSuccess && kv.second.amax)
            e = cudaMemset(kv.second.amax, 0, (kMaxArgmaxTokens + 1) * sizeof(unsigned long long));
        if (e != cudaSuccess) return cuda_fail(e, "reset scratch counters");
    }
    return B200Q8_OK;
}

// Weights up to this size with few tokens go to the SIMT GEMV under ALGO_AUTO.
constexpr size_t kSimtMaxWeightBytes = (size_t)48 << 20;

// pro / norm_w / eps: an elementwise prologue (prologue.cuh) that turns inp into the activations
// -- fused into the int8 digit GEMV, or run first into scratch when the GEMM takes the shape.
int linear_impl(void* out, int out_dtype, const void* inp, int in_dtype, const int8_t* weight,
                const float* scales, const float* bias, const void* residual, size_t M, size_t N,
                size_t K, cudaStream_t stream, int algo = B200Q8_ALGO_AUTO, int pro = kProNone,
                const float* norm_w = nullptr, float eps = 0.0f)
{
    if (algo != B200Q8_ALGO_AUTO && algo != B200Q8_ALGO_SIMT && algo != B200Q8_ALGO_TC &&
        algo != B200Q8_ALGO_TC_I8)
        return fail(B200Q8_ERR_INVALID, "linear_q8: unknown algo %d", algo);
    if (!valid_dtype(out_dtype) || !valid_dtype(in_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8: dtype must be B200Q8_F32 or B200Q8_F16");
    if (M == 0 || N == 0) return B200Q8_OK;
    if (!out || !inp || !weight || !scales)
        return fail(B200Q8_ERR_INVALID, "linear_q8: null out/inp/weight/scales");
    if (K == 0) return fail(B200Q8_ERR_INVALID, "linear_q8: K == 0");
    if (N > (size_t)INT32_MAX || K > (size_t)INT32_MAX || M > (size_t)INT32_MAX ||
        N * K / K != N)
        return fail(B200Q8_ERR_INVALID, "linear_q8: sizes overflow (M=%zu N=%zu K=%zu)", M, N, K);
    const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4, ib = in_dtype == B200Q8_F16 ? 2 : 4;
    const size_t ldx = pro == kProSiluMul ? 2 * K : K;  // input row length
    {   // inp must not overlap out
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t i0 = (uintptr_t)inp, i1 = i0 + M * ldx * ib;
        if (o0 < i1 && i0 < o1) return fail(B200Q8_ERR_INVALID, "linear_q8: inp overlaps out");
    }
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;

    LinearArgs a;
    a.x = inp;
    a.w = weight;
    a.scales = scales;
    a.bias = bias;
    a.res = residual;
    a.out = out;
    a.M = M;
    a.N = N;
    a.K = K;
    a.in_dtype = in_dtype;
    a.out_dtype = out_dtype;
    a.pdl = true;
    cudaError_t e;
    // Kernel choice (AUTO): up to 4 tokens on at most 48 MiB of weights -> the SIMT streaming GEMV
    // (the tensor-core kernels' fixed costs -- barrier and TMEM set-up, pipeline fill, stream-K
    // fixup, ~6 us -- exceed a few-MB projection's whole streaming time: measured on B200, one
    // token, 896x896 2.5 vs 6.0 us, 896x4864 4.6 vs 9.6 us, 49152x576 12.2 vs 12.5 us, a 7B down
    // shard 1792x18944 (34 MB) 14.3 vs 16.4 us, and a Qwen2.5-0.5B decode step 555 vs 1070 us; the
    // 7B down projection itself, 68 MB, is 23.3 vs 20.2 us); up to 16 tokens -> int8 tensor-core GEMV with
    // exact activation digits; more tokens with fp16 activations -> fp16 tensor-core GEMM
    // (weights dequantized into TMEM); more tokens with fp32 activations -> the digit kernel in
    // groups of up to 42 tokens.  Shapes the tensor-core kernels cannot take (K % 16 != 0,
    // misaligned) use the SIMT GEMV.
    const bool tc_ok = gemm_tc_supports(a);
    LinearArgs a1 = a;
    a1.M = M < (size_t)gemv_i8_max_tokens() ? M : (size_t)gemv_i8_max_tokens();
    const bool i8_ok = gemv_i8_supports(a1);
    if (algo == B200Q8_ALGO_TC && !tc_ok)
        return fail(B200Q8_ERR_UNSUPPORTED,
                    "linear_q8: fp16 tensor-core path needs fp16 activations, K %% 16 == 0 and 16-byte aligned "
                    "weight/activation pointers (in_dtype=%d K=%zu)", in_dtype, K);
    if (algo == B200Q8_ALGO_TC_I8 && !i8_ok)
        return fail(B200Q8_ERR_UNSUPPORTED,
                    "linear_q8: int8 tensor-core path needs K %% 16 == 0, K <= 131072 and a 16-byte aligned "
                    "weight pointer (K=%zu)", K);
    const bool small = M <= (size_t)gemv_max_tokens() && N * K <= kSimtMaxWeightBytes;
    // Few fp16 tokens: the int8 digit GEMV, which streams the raw weights, up to 4 tokens, and up
    // to 8 on wide projections; beyond that the digit tiles (6 rows per token) cost more than the
    // fp16 GEMM's dequantization.  Measured on B200, 7B projections at M = 8 (digit GEMV vs GEMM):
    // lm_head 96 vs 111 us, gate/up 32 vs 31 us, down 33 vs 24 us; at M = 12 the GEMM wins on all.
    const bool i8_first = M <= 4 || (M <= 8 && N >= 16384);
    const bool use_i8 = algo == B200Q8_ALGO_TC_I8 ||
                        (algo == B200Q8_ALGO_AUTO && i8_ok && !small && (i8_first || !tc_ok));
    const bool use_tc =
        !use_i8 && (algo == B200Q8_ALGO_TC || (algo == B200Q8_ALGO_AUTO && tc_ok && !small));
    // The SIMT streaming kernel applies a prologue while it stages x (one launch); so does the
    // digit GEMV.  For the GEMM, or SIMT shapes only its generic kernel takes, write the
    // activations once into scratch first.
    bool simt_pro = false;
    if (pro != kProNone && !use_i8 && !use_tc) {
        LinearArgs s1 = a;
        s1.M = M < (size_t)gemv_max_tokens() ? M : (size_t)gemv_max_tokens();
        s1.prologue = pro;
        s1.norm_w = norm_w;
        simt_pro = gemv_stream_supports(s1, d.max_smem);
    }
    if (pro != kProNone && !use_i8 && !simt_pro) {
        ScratchNeed need;
        need.act = M * K * ib;
        TcScratch scratch;
        if ((st = get_scratch(need, d.num_sms, stream, &scratch))) return st;
        e = launch_prologue(pro, inp, scratch.act, in_dtype, norm_w, eps, M, K, true, stream);
        if (e != cudaSuccess) return cuda_fail(e, "prologue launch");
        a.x = inp = scratch.act;
        pro = kProNone;
    }
    if (pro != kProNone) {
        a.prologue = pro;
        a.norm_w = norm_w;
        a.eps = eps;
    }
    if (use_tc) {
        ScratchNeed need;
        gemm_tc_scratch_need(a, d.num_sms, &need.ws, &need.counters);
        TcScratch scratch;
        if ((st = get_scratch(need, d.num_sms, stream, &scratch))) return st;
        e = launch_q8_gemm_tc(a, d.num_sms, scratch, stream);
        if (e != cudaSuccess) return cuda_fail(e, "q8_gemm_tc launch");
        return B200Q8_OK;
    }
    if (use_i8) {
        const size_t mt = (size_t)gemv_i8_max_tokens();
        for (size_t m0 = 0; m0 < M; m0 += mt) {
            LinearArgs b = a;
            b.M = (M - m0 < mt) ? (M - m0) : mt;
            b.x = (const char*)inp + m0 * ldx * ib;
            b.out = (char*)out + m0 * N * ob;
            b.res = residual ? (const char*)residual + m0 * N * ob : nullptr;
            ScratchNeed need;
            gemv_i8_scratch_need(b, d.num_sms, &need.ws, &need.counters, &need.act, &need.exps);
            TcScratch scratch;
            if ((st = get_scratch(need, d.num_sms, stream, &scratch))) return st;
            e = launch_q8_gemv_i8(b, d.num_sms, scratch, stream);
            if (e != cudaSuccess) return cuda_fail(e, "q8_gemv_i8 launch");
        }
        return B200Q8_OK;
    }
    if ((int)M <= gemv_max_tokens()) {
        e = launch_q8_gemv(a, d.num_sms, d.max_smem, stream);
        if (e != cudaSuccess) return cuda_fail(e, "q8_gemv launch");
        return B200Q8_OK;
    }
    // M beyond the GEMV's token count and not taken by the tensor-core GEMM:
    // stream the weights once per group of up to 4 tokens.
    const int mt = gemv_max_tokens();
    const size_t xstride = pro == kProSiluMul ? 2 * K : K;  // input row length (prologue not materialized)
    for (size_t m0 = 0; m0 < M; m0 += (size_t)mt) {
        LinearArgs b = a;
        b.M = (M - m0 < (size_t)mt) ? (M - m0) : (size_t)mt;
        b.x = (const char*)inp + m0 * xstride * ib;
        b.out = (char*)out + m0 * N * ob;
        b.res = residual ? (const char*)residual + m0 * N * ob : nullptr;
        e = launch_q8_gemv(b, d.num_sms, d.max_smem, stream);
        if (e != cudaSuccess) return cuda_fail(e, "q8_gemv launch");
    }
    return B200Q8_OK;
}

}  // namespace
}  // namespace b200q8

using namespace b200q8;

extern "C" {

int b200q8_abi_version(void) { return B200Q8_ABI_VERSION; }

const char* b200q8_last_error(void) { return t_last_error.c_str(); }

uint64_t b200q8_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int b200q8_quantize_per_channel(const float* w, size_t N, size_t K, int8_t* q, float* scales,
                                b200q8_stream_t stream)
{
    if (N == 0) return B200Q8_OK;
    if (!w || !q || !scales) return fail(B200Q8_ERR_INVALID, "quantize: null pointer");
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(scales, 0, N * sizeof(float), stream);
        return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    if (N > (size_t)INT32_MAX || K > ((size_t)1 << 40))
        return fail(B200Q8_ERR_INVALID, "quantize: sizes overflow (N=%zu K=%zu)", N, K);
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;
    cudaError_t e = launch_q8_quantize(w, N, K, q, scales, d.num_sms, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "q8_quantize launch");
    return B200Q8_OK;
}

int b200q8_quantize_per_channel_bf16(const uint16_t* w, size_t N, size_t K, int8_t* q, float* scales,
                                     b200q8_stream_t stream)
{
    if (N == 0) return B200Q8_OK;
    if (!w || !q || !scales) return fail(B200Q8_ERR_INVALID, "quantize_bf16: null pointer");
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(scales, 0, N * sizeof(float), stream);
        return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    if (N > (size_t)INT32_MAX || K > ((size_t)1 << 40))
        return fail(B200Q8_ERR_INVALID, "quantize_bf16: sizes overflow (N=%zu K=%zu)", N, K);
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;
    cudaError_t e = launch_q8_quantize_bf16(w, N, K, q, scales, d.num_sms, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "q8_quantize_bf16 launch");
    return B200Q8_OK;
}

int b200q8_linear_q8(void* out, int out_dtype, const void* inp, int in_dtype, const int8_t* weight,
                     const float* scales, const float* bias, size_t M, size_t N, size_t K,
                     b200q8_stream_t stream)
{
    return linear_impl(out, out_dtype, inp, in_dtype, weight, scales, bias, nullptr, M, N, K,
                       (cudaStream_t)stream);
}

int b200q8_linear_q8_ex(void* out, int out_dtype, const void* inp, int in_dtype, const int8_t* weight,
                        const float* scales, const float* bias, const void* residual, size_t M, size_t N,
                        size_t K, int algo, b200q8_stream_t stream)
{
    if (residual && residual != out && M && N) {
        const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4;
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t r0 = (uintptr_t)residual, r1 = r0 + M * N * ob;
        if (o0 < r1 && r0 < o1)
            return fail(B200Q8_ERR_INVALID, "linear_q8_ex: residual partially overlaps out");
    }
    return linear_impl(out, out_dtype, inp, in_dtype, weight, scales, bias, residual, M, N, K,
                       (cudaStream_t)stream, algo);
}

int b200q8_kernel_error(int* code, int clear)
{
    if (!code) return fail(B200Q8_ERR_INVALID, "kernel_error: null code");
    int c1 = 0, c2 = 0;
    cudaError_t e = read_kernel_error(&c1, clear != 0);
    if (e == cudaSuccess) e = read_kernel_error_i8(&c2, clear != 0);
    if (e != cudaSuccess) return cuda_fail(e, "kernel_error: read device word");
    *code = c1 | c2;
    if (clear && *code) {
        int dev = 0;
        if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
        return reset_scratch_counters(dev);
    }
    return B200Q8_OK;
}

// Allocation-free linear_q8 / linear_q8_add for callers that may not call
// cudaMalloc (a device-memory pool or budget they must not bypass, or a decode
// loop that cannot take cudaMalloc's device-wide synchronisation).  Runs the
// int8 digit GEMV on the fixed device array of q8_gemv_tc.cu.
int b200q8_linear_q8_noalloc(void* out, int out_dtype, const void* inp, int in_dtype, const int8_t* weight,
                             const float* scales, const float* bias, const void* residual, size_t M, size_t N,
                             size_t K, b200q8_stream_t stream)
{
    if (!valid_dtype(out_dtype) || !valid_dtype(in_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8_noalloc: dtype must be B200Q8_F32 or B200Q8_F16");
    if (M == 0 || N == 0) return B200Q8_OK;
    if (!out || !inp || !weight || !scales)
        return fail(B200Q8_ERR_INVALID, "linear_q8_noalloc: null out/inp/weight/scales");
    if (K == 0 || N > (size_t)INT32_MAX || K > (size_t)INT32_MAX || N * K / K != N)
        return fail(B200Q8_ERR_INVALID, "linear_q8_noalloc: bad sizes (N=%zu K=%zu)", N, K);
    const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4, ib = in_dtype == B200Q8_F16 ? 2 : 4;
    {
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t i0 = (uintptr_t)inp, i1 = i0 + M * K * ib;
        if (o0 < i1 && i0 < o1) return fail(B200Q8_ERR_INVALID, "linear_q8_noalloc: inp overlaps out");
        if (residual && residual != out) {
            const uintptr_t r0 = (uintptr_t)residual, r1 = r0 + M * N * ob;
            if (o0 < r1 && r0 < o1)
                return fail(B200Q8_ERR_INVALID, "linear_q8_noalloc: residual partially overlaps out");
        }
    }
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;
    LinearArgs a;
    a.x = inp;
    a.w = weight;
    a.scales = scales;
    a.bias = bias;
    a.res = residual;
    a.out = out;
    a.M = M;
    a.N = N;
    a.K = K;
    a.in_dtype = in_dtype;
    a.out_dtype = out_dtype;
    a.pdl = true;
    cudaError_t e = cudaSuccess;
    switch (launch_q8_gemv_i8_noalloc(a, d.num_sms, (cudaStream_t)stream, &e)) {
        case 0: return B200Q8_OK;
        case 1: return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_noalloc: M=%zu exceeds the fixed scratch (at most 2 tokens)", M);
        case 2: return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_noalloc: N=%zu exceeds the fixed scratch (at most 524288 rows)", N);
        case 3: return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_noalloc: %d SMs exceed the fixed scratch (at most 160)", d.num_sms);
        case 4: return fail(B200Q8_ERR_UNSUPPORTED,
                            "linear_q8_noalloc: needs K %% 16 == 0, 16 <= K <= 131072, a 16-byte aligned weight and an "
                            "8-byte (fp16) / 16-byte (fp32) aligned input (K=%zu)", K);
        case 5: return fail(B200Q8_ERR_UNSUPPORTED,
                            "linear_q8_noalloc: M=%zu N=%zu K=%zu needs more scratch than the fixed array holds", M, N, K);
        default: return cuda_fail(e, "linear_q8_noalloc");
    }
}

// The bounded wait of the gathered calls, run on caller memory so that a test can make it run
// out on one GPU (a count nothing advances) and see the status the host reads afterwards.
int b200q8_diag_peer_wait(const uint64_t* counts, int n, int self, double timeout_s, int where, void* out,
                          const void* x, const int8_t* weight, const float* scales, size_t N, size_t K,
                          b200q8_stream_t stream)
{
    if (!counts || n < 1 || n > kMaxRanks || self < 0 || self >= n)
        return fail(B200Q8_ERR_INVALID, "diag_peer_wait: counts, 1 <= n <= %d and 0 <= self < n required", kMaxRanks);
    if (!(timeout_s >= 1e-3 && timeout_s <= 10.0))
        return fail(B200Q8_ERR_INVALID, "diag_peer_wait: timeout_s must lie in [0.001, 10]");
    if (where < 0 || where > 2) return fail(B200Q8_ERR_INVALID, "diag_peer_wait: where must be 0, 1 or 2");
    const unsigned long long ns = (unsigned long long)(timeout_s * 1e9);
    const unsigned long long* cts = reinterpret_cast<const unsigned long long*>(counts);
    cudaError_t e;
    if (where == 0) {
        P2POut wo;
        wo.rank = self;
        wo.wait_counts = cts;
        wo.wait_n = n;
        wo.wait_timeout_ns = ns;
        e = launch_p2p_sync(wo, false, true, (cudaStream_t)stream);
        return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "diag_peer_wait: wait launch");
    }
    if (!out || !x || !weight || !scales || N == 0 || K == 0 || N > (size_t)INT32_MAX || K > (size_t)INT32_MAX)
        return fail(B200Q8_ERR_INVALID, "diag_peer_wait: the GEMV needs out, x, weight, scales, N and K");
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;
    P2POut po;
    po.ndst = 1;
    po.dst[0] = out;
    po.ldo = (long long)N;
    po.rank = self;
    po.wait_counts = cts;
    po.wait_n = n;
    po.wait_timeout_ns = ns;
    LinearArgs a;
    a.x = x;
    a.w = weight;
    a.scales = scales;
    a.out = out;
    a.M = 1;
    a.N = N;
    a.K = K;
    a.in_dtype = B200Q8_F16;
    a.out_dtype = B200Q8_F16;
    a.pdl = true;
    a.p2p = &po;
    a.force_prep = where == 2;
    if (!gemv_i8_supports(a))
        return fail(B200Q8_ERR_UNSUPPORTED, "diag_peer_wait: the digit GEMV does not take K=%zu or these pointers", K);
    if (where == 1 && !gemv_i8_fused_exps(a))
        return fail(B200Q8_ERR_UNSUPPORTED, "diag_peer_wait: K=%zu is scanned by the prep kernel (use where=2)", K);
    ScratchNeed need;
    gemv_i8_scratch_need(a, d.num_sms, &need.ws, &need.counters, &need.act, &need.exps);
    TcScratch scratch;
    if ((st = get_scratch(need, d.num_sms, (cudaStream_t)stream, &scratch))) return st;
    e = launch_q8_gemv_i8(a, d.num_sms, scratch, (cudaStream_t)stream);
    return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "diag_peer_wait: GEMV launch");
}

int b200q8_linear_q8_argmax(void* out, int out_dtype, const void* inp, int in_dtype, const int8_t* weight,
                            const float* scales, const float* bias, size_t M, size_t N, size_t K, int* argmax,
                            b200q8_stream_t stream)
{
    if (!valid_dtype(out_dtype) || !valid_dtype(in_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8_argmax: dtype must be B200Q8_F32 or B200Q8_F16");
    if (M == 0) return B200Q8_OK;
    if (N == 0) return fail(B200Q8_ERR_INVALID, "linear_q8_argmax: N = 0 has no argmax");
    if (!inp || !weight || !scales || !argmax)
        return fail(B200Q8_ERR_INVALID, "linear_q8_argmax: null inp/weight/scales/argmax");
    if (K == 0 || N > (size_t)INT32_MAX || K > (size_t)INT32_MAX || N * K / K != N)
        return fail(B200Q8_ERR_INVALID, "linear_q8_argmax: bad sizes (N=%zu K=%zu)", N, K);
    if (M > (size_t)gemv_i8_max_tokens() || M > (size_t)kMaxArgmaxTokens)
        return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_argmax: at most %d tokens (M=%zu)", gemv_i8_max_tokens(), M);
    if (out) {
        const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4, ib = in_dtype == B200Q8_F16 ? 2 : 4;
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t i0 = (uintptr_t)inp, i1 = i0 + M * K * ib;
        if (o0 < i1 && i0 < o1) return fail(B200Q8_ERR_INVALID, "linear_q8_argmax: inp overlaps out");
    }
    DeviceInfo d;
    int st = device_info(&d);
    if (st) return st;
    LinearArgs a;
    a.x = inp;
    a.w = weight;
    a.scales = scales;
    a.bias = bias;
    a.out = out;
    a.M = M;
    a.N = N;
    a.K = K;
    a.in_dtype = in_dtype;
    a.out_dtype = out_dtype;
    a.pdl = true;
    if (!gemv_i8_supports(a))
        return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_argmax: needs K %% 16 == 0, 16 <= K <= 131072, a 16-byte "
                                            "aligned weight and an 8-byte (fp16) / 16-byte (fp32) aligned input");
    ScratchNeed need;
    gemv_i8_scratch_need(a, d.num_sms, &need.ws, &need.counters, &need.act, &need.exps);
    need.amax = true;
    TcScratch scratch;
    if ((st = get_scratch(need, d.num_sms, (cudaStream_t)stream, &scratch))) return st;
    a.amax_keys = scratch.amax;
    a.amax_done = reinterpret_cast<unsigned int*>(scratch.amax + kMaxArgmaxTokens);
    a.amax_out = argmax;
    const cudaError_t e = launch_q8_gemv_i8(a, d.num_sms, scratch, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "linear_q8_argmax: launch");
    return B200Q8_OK;
}

int b200q8_linear_q8_add(void* out, int out_dtype, const void* inp, int in_dtype,
                         const int8_t* weight, const float* scales, const float* bias,
                         const void* residual, size_t M, size_t N, size_t K, b200q8_stream_t stream)
{
    if (!residual && M && N) return fail(B200Q8_ERR_INVALID, "linear_q8_add: null residual");
    if (residual && residual != out && M && N) {
        // residual must either be out itself or not overlap it
        const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4;
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t r0 = (uintptr_t)residual, r1 = r0 + M * N * ob;
        if (o0 < r1 && r0 < o1)
            return fail(B200Q8_ERR_INVALID, "linear_q8_add: residual partially overlaps out");
    }
    return linear_impl(out, out_dtype, inp, in_dtype, weight, scales, bias, residual, M, N, K,
                       (cudaStream_t)stream);
}

}  // extern "C"

namespace b200q8 {
namespace {

// Shape / alignment rules shared by the prologue entry points: rows of 4-element groups,
// fp16 rows 8-byte and fp32 rows 16-byte aligned (the prologue's vector loads).
int check_prologue_io(const char* what, const void* x, const void* out, int dtype, size_t M, size_t K, size_t ldx)
{
    if (!valid_dtype(dtype)) return fail(B200Q8_ERR_INVALID, "%s: dtype must be B200Q8_F32 or B200Q8_F16", what);
    if (!x || !out) return fail(B200Q8_ERR_INVALID, "%s: null input/output", what);
    const size_t eb = dtype == B200Q8_F16 ? 2 : 4, al = dtype == B200Q8_F16 ? 8 : 16;
    if (K % 4 != 0 || K > (size_t)INT32_MAX || M > (size_t)INT32_MAX)
        return fail(B200Q8_ERR_UNSUPPORTED, "%s: needs K %% 4 == 0 (K=%zu)", what, K);
    if ((uintptr_t)x % al || (uintptr_t)out % al)
        return fail(B200Q8_ERR_UNSUPPORTED, "%s: input/output must be %zu-byte aligned", what, al);
    const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * K * eb, i0 = (uintptr_t)x, i1 = i0 + M * ldx * eb;
    if (o0 < i1 && i0 < o1) return fail(B200Q8_ERR_INVALID, "%s: input overlaps output", what);
    return B200Q8_OK;
}

}  // namespace
}  // namespace b200q8

extern "C" {

int b200q8_rms_norm(void* out, const void* x, int dtype, const float* norm_weight, float eps, size_t M, size_t K,
                    b200q8_stream_t stream)
{
    if (M == 0 || K == 0) return B200Q8_OK;
    int st = check_prologue_io("rms_norm", x, out, dtype, M, K, K);
    if (st) return st;
    if (!norm_weight) return fail(B200Q8_ERR_INVALID, "rms_norm: null norm_weight");
    if ((uintptr_t)norm_weight % 16) return fail(B200Q8_ERR_UNSUPPORTED, "rms_norm: norm_weight must be 16-byte aligned");
    const cudaError_t e = launch_prologue(kProRmsNorm, x, out, dtype, norm_weight, eps, M, K, true, (cudaStream_t)stream);
    return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "rms_norm launch");
}

int b200q8_silu_mul(void* out, const void* gate_up, int dtype, size_t M, size_t K, b200q8_stream_t stream)
{
    if (M == 0 || K == 0) return B200Q8_OK;
    int st = check_prologue_io("silu_mul", gate_up, out, dtype, M, K, 2 * K);
    if (st) return st;
    const cudaError_t e = launch_prologue(kProSiluMul, gate_up, out, dtype, nullptr, 0.0f, M, K, true,
                                          (cudaStream_t)stream);
    return e == cudaSuccess ? B200Q8_OK : cuda_fail(e, "silu_mul launch");
}

int b200q8_rms_norm_linear_q8(void* out, int out_dtype, const void* x, int in_dtype, const float* norm_weight,
                              float eps, const int8_t* weight, const float* scales, const float* bias, size_t M,
                              size_t N, size_t K, b200q8_stream_t stream)
{
    if (M == 0 || N == 0) return B200Q8_OK;
    if (!valid_dtype(in_dtype)) return fail(B200Q8_ERR_INVALID, "rms_norm_linear_q8: bad in_dtype");
    if (!norm_weight) return fail(B200Q8_ERR_INVALID, "rms_norm_linear_q8: null norm_weight");
    if ((uintptr_t)norm_weight % 16)
        return fail(B200Q8_ERR_UNSUPPORTED, "rms_norm_linear_q8: norm_weight must be 16-byte aligned");
    if (!x) return fail(B200Q8_ERR_INVALID, "rms_norm_linear_q8: null x");
    const size_t al = in_dtype == B200Q8_F16 ? 8 : 16;
    if (K % 4 != 0 || (uintptr_t)x % al)
        return fail(B200Q8_ERR_UNSUPPORTED, "rms_norm_linear_q8: needs K %% 4 == 0 and a %zu-byte aligned x (K=%zu)",
                    al, K);
    return linear_impl(out, out_dtype, x, in_dtype, weight, scales, bias, nullptr, M, N, K, (cudaStream_t)stream,
                       B200Q8_ALGO_AUTO, kProRmsNorm, norm_weight, eps);
}

int b200q8_silu_mul_linear_q8_add(void* out, int out_dtype, const void* gate_up, int in_dtype,
                                  const int8_t* weight, const float* scales, const float* bias, const void* residual,
                                  size_t M, size_t N, size_t K, b200q8_stream_t stream)
{
    if (M == 0 || N == 0) return B200Q8_OK;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype))
        return fail(B200Q8_ERR_INVALID, "silu_mul_linear_q8_add: dtype must be B200Q8_F32 or B200Q8_F16");
    if (!gate_up) return fail(B200Q8_ERR_INVALID, "silu_mul_linear_q8_add: null gate_up");
    const size_t al = in_dtype == B200Q8_F16 ? 8 : 16;
    if (K % 4 != 0 || (uintptr_t)gate_up % al)
        return fail(B200Q8_ERR_UNSUPPORTED,
                    "silu_mul_linear_q8_add: needs K %% 4 == 0 and a %zu-byte aligned gate_up (K=%zu)", al, K);
    if (residual && residual != out) {  // residual must either be out itself or not overlap it
        const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4;
        const uintptr_t o0 = (uintptr_t)out, o1 = o0 + M * N * ob;
        const uintptr_t r0 = (uintptr_t)residual, r1 = r0 + M * N * ob;
        if (o0 < r1 && r0 < o1)
            return fail(B200Q8_ERR_INVALID, "silu_mul_linear_q8_add: residual partially overlaps out");
    }
    return linear_impl(out, out_dtype, gate_up, in_dtype, weight, scales, bias, residual, M, N, K,
                       (cudaStream_t)stream, B200Q8_ALGO_AUTO, kProSiluMul);
}

int b200q8_linear_q8_group(int n, void* const* outs, int out_dtype, const void* x, int in_dtype,
                           const float* norm_weight, float eps, const int8_t* const* weights,
                           const float* const* scales, const float* const* biases, const size_t* Ns, size_t M,
                           size_t K, b200q8_stream_t stream)
{
    if (n < 1 || n > B200Q8_MAX_GROUP)
        return fail(B200Q8_ERR_INVALID, "linear_q8_group: n must be 1..%d (n=%d)", B200Q8_MAX_GROUP, n);
    if (!outs || !weights || !scales || !Ns) return fail(B200Q8_ERR_INVALID, "linear_q8_group: null array");
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8_group: dtype must be B200Q8_F32 or B200Q8_F16");
    if (M == 0) return B200Q8_OK;
    if (!x) return fail(B200Q8_ERR_INVALID, "linear_q8_group: null x");
    if (K == 0 || K > (size_t)INT32_MAX || M > (size_t)INT32_MAX)
        return fail(B200Q8_ERR_INVALID, "linear_q8_group: bad sizes (M=%zu K=%zu)", M, K);
    const int pro = norm_weight ? kProRmsNorm : kProNone;
    if (pro != kProNone) {
        const size_t al = in_dtype == B200Q8_F16 ? 8 : 16;
        if ((uintptr_t)norm_weight % 16)
            return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_group: norm_weight must be 16-byte aligned");
        if (K % 4 != 0 || (uintptr_t)x % al)
            return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_group: the norm needs K %% 4 == 0 and a %zu-byte aligned x",
                        al);
    }
    const size_t ob = out_dtype == B200Q8_F16 ? 2 : 4, ib = in_dtype == B200Q8_F16 ? 2 : 4;
    const int8_t* w[kMaxGroup];
    const float* s[kMaxGroup];
    const float* b[kMaxGroup];
    void* o[kMaxGroup];
    size_t nn[kMaxGroup];
    int live = 0;
    size_t wbytes = 0;
    for (int i = 0; i < n; i++) {
        if (Ns[i] == 0) continue;
        if (!outs[i] || !weights[i] || !scales[i])
            return fail(B200Q8_ERR_INVALID, "linear_q8_group: null out/weight/scales of projection %d", i);
        if (Ns[i] > (size_t)INT32_MAX || Ns[i] * K / K != Ns[i])
            return fail(B200Q8_ERR_INVALID, "linear_q8_group: sizes overflow (N[%d]=%zu K=%zu)", i, Ns[i], K);
        const uintptr_t o0 = (uintptr_t)outs[i], o1 = o0 + M * Ns[i] * ob;
        const uintptr_t i0 = (uintptr_t)x, i1 = i0 + M * K * ib;
        if (o0 < i1 && i0 < o1) return fail(B200Q8_ERR_INVALID, "linear_q8_group: x overlaps out %d", i);
        for (int j = 0; j < live; j++) {
            const uintptr_t p0 = (uintptr_t)o[j], p1 = p0 + M * nn[j] * ob;
            if (o0 < p1 && p0 < o1) return fail(B200Q8_ERR_INVALID, "linear_q8_group: outputs overlap");
        }
        w[live] = weights[i];
        s[live] = scales[i];
        b[live] = biases ? biases[i] : nullptr;
        o[live] = outs[i];
        nn[live] = Ns[i];
        wbytes += Ns[i] * K;
        live++;
    }
    if (live == 0) return B200Q8_OK;
    // Few tokens on a few MB of weights: one streaming launch that stages x (and normalizes it)
    // once for every projection.  Otherwise, or for shapes that kernel does not take, one
    // projection at a time through the ordinary dispatch.
    if (live > 1 && M <= (size_t)gemv_max_tokens() && wbytes <= kSimtMaxWeightBytes) {
        DeviceInfo d;
        int st = device_info(&d);
        if (st) return st;
        LinearArgs a;
        a.x = x;
        a.M = M;
        a.K = K;
        a.in_dtype = in_dtype;
        a.out_dtype = out_dtype;
        a.pdl = true;
        a.prologue = pro;
        a.norm_w = norm_weight;
        a.eps = eps;
        const cudaError_t e = launch_q8_gemv_group(a, live, w, s, b, o, nn, d.num_sms, d.max_smem,
                                                   (cudaStream_t)stream);
        if (e == cudaSuccess) return B200Q8_OK;
        if (e != cudaErrorNotSupported) return cuda_fail(e, "q8_gemv group launch");
    }
    for (int i = 0; i < live; i++) {
        const int st = linear_impl(o[i], out_dtype, x, in_dtype, w[i], s[i], b[i], nullptr, M, nn[i], K,
                                   (cudaStream_t)stream, B200Q8_ALGO_AUTO, pro, norm_weight, eps);
        if (st) return st;
    }
    return B200Q8_OK;
}

}  // extern "C"

// ===========================================================================
// Backend layer: host weight pointers cached on the device by host address.
// Mirrors BackendCUDA::cache_weight (src/backend/backend_cuda.cc:51-59) --
// first use uploads, later uses look up; entries live as long as the backend.
// ===========================================================================
struct b200q8_backend {
    int device = 0;
    bool fp16 = false;
    cudaStream_t stream = nullptr;
    struct Buf {
        void* ptr;
        size_t bytes;
    };
    std::unordered_map<const void*, Buf> cache;
    size_t cached_bytes = 0;
};

namespace {

int set_device(int dev)
{
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != dev && (e = cudaSetDevice(dev)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    return B200Q8_OK;
}

int cache_upload(b200q8_backend* be, const void* host, size_t bytes, void** dptr)
{
    auto it = be->cache.find(host);
    if (it != be->cache.end()) {
        if (it->second.bytes < bytes)
            return fail(B200Q8_ERR_INVALID,
                        "weight cache: host pointer %p was first seen with %zu bytes, now %zu", host,
                        it->second.bytes, bytes);
        *dptr = it->second.ptr;
        return B200Q8_OK;
    }
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(B200Q8_ERR_ALLOC, "weight cache: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    // The host buffer is pageable model memory: a synchronous copy, once per weight.
    e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "weight cache: cudaMemcpy H2D");
    }
    be->cache.emplace(host, b200q8_backend::Buf{d, bytes});
    be->cached_bytes += bytes;
    *dptr = d;
    return B200Q8_OK;
}

int backend_linear(b200q8_backend* be, float* out, const float* inp, const int8_t* weight,
                   const float* scales, const float* bias, const float* residual, size_t M, size_t N,
                   size_t K)
{
    if (!be) return fail(B200Q8_ERR_INVALID, "backend: null handle");
    if (M == 0 || N == 0) return B200Q8_OK;
    if (!weight || !scales) return fail(B200Q8_ERR_INVALID, "backend: null weight/scales");
    int st = set_device(be->device);
    if (st) return st;
    void *dw = nullptr, *ds = nullptr, *db = nullptr;
    if ((st = cache_upload(be, weight, N * K, &dw))) return st;
    if ((st = cache_upload(be, scales, N * sizeof(float), &ds))) return st;
    if (bias && (st = cache_upload(be, bias, N * sizeof(float), &db))) return st;
    const int dt = be->fp16 ? B200Q8_F16 : B200Q8_F32;
    return linear_impl(out, dt, inp, dt, (const int8_t*)dw, (const float*)ds, (const float*)db,
                       residual, M, N, K, be->stream);
}

}  // namespace

extern "C" {

int b200q8_backend_create(int device, int fp16, b200q8_backend** out)
{
    if (!out) return fail(B200Q8_ERR_INVALID, "backend_create: null out");
    *out = nullptr;
    int st = set_device(device);
    if (st) return st;
    DeviceInfo d;
    if ((st = device_info(&d))) return st;
    auto* be = new (std::nothrow) b200q8_backend();
    if (!be) return fail(B200Q8_ERR_ALLOC, "backend_create: out of host memory");
    be->device = device;
    be->fp16 = fp16 != 0;
    *out = be;
    return B200Q8_OK;
}

int b200q8_backend_destroy(b200q8_backend* be)
{
    if (!be) return B200Q8_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(be->device);
    for (auto& kv : be->cache) cudaFree(kv.second.ptr);
    if (cur >= 0) cudaSetDevice(cur);
    delete be;
    return B200Q8_OK;
}

int b200q8_backend_set_stream(b200q8_backend* be, b200q8_stream_t stream)
{
    if (!be) return fail(B200Q8_ERR_INVALID, "backend: null handle");
    be->stream = (cudaStream_t)stream;
    return B200Q8_OK;
}

int b200q8_backend_cached_bytes(const b200q8_backend* be, size_t* bytes)
{
    if (!be || !bytes) return fail(B200Q8_ERR_INVALID, "backend: null argument");
    *bytes = be->cached_bytes;
    return B200Q8_OK;
}

int b200q8_backend_linear_q8(b200q8_backend* be, float* out, const float* inp, const int8_t* weight,
                             const float* scales, const float* bias, size_t M, size_t N, size_t K)
{
    return backend_linear(be, out, inp, weight, scales, bias, nullptr, M, N, K);
}

int b200q8_backend_linear_q8_add(b200q8_backend* be, float* out, const float* inp,
                                 const int8_t* weight, const float* scales, const float* bias,
                                 const float* residual, size_t M, size_t N, size_t K)
{
    if (!residual && M && N) return fail(B200Q8_ERR_INVALID, "linear_q8_add: null residual");
    return backend_linear(be, out, inp, weight, scales, bias, residual, M, N, K);
}

int b200q8_backend_quantize_per_channel(b200q8_backend* be, const float* weight, size_t N, size_t K,
                                        int8_t* q, float* scales)
{
    if (!be) return fail(B200Q8_ERR_INVALID, "backend: null handle");
    if (N == 0) return B200Q8_OK;
    if (!weight || !q || !scales) return fail(B200Q8_ERR_INVALID, "quantize: null pointer");
    int st = set_device(be->device);
    if (st) return st;
    float* dw = nullptr;
    int8_t* dq = nullptr;
    float* ds = nullptr;
    cudaError_t e;
    const size_t nk = N * K;
    if ((e = cudaMalloc(&dw, nk * sizeof(float) + 16)) != cudaSuccess ||
        (e = cudaMalloc(&dq, nk + 16)) != cudaSuccess ||
        (e = cudaMalloc(&ds, N * sizeof(float))) != cudaSuccess) {
        cudaFree(dw);
        cudaFree(dq);
        cudaFree(ds);
        cudaGetLastError();
        return fail(B200Q8_ERR_ALLOC, "quantize: cudaMalloc: %s", cudaGetErrorString(e));
    }
    int rc = B200Q8_OK;
    if ((e = cudaMemcpyAsync(dw, weight, nk * sizeof(float), cudaMemcpyHostToDevice, be->stream)) != cudaSuccess)
        rc = cuda_fail(e, "quantize: H2D");
    if (!rc) rc = b200q8_quantize_per_channel(dw, N, K, dq, ds, be->stream);
    if (!rc && (e = cudaMemcpyAsync(q, dq, nk, cudaMemcpyDeviceToHost, be->stream)) != cudaSuccess)
        rc = cuda_fail(e, "quantize: D2H q");
    if (!rc && (e = cudaMemcpyAsync(scales, ds, N * sizeof(float), cudaMemcpyDeviceToHost, be->stream)) != cudaSuccess)
        rc = cuda_fail(e, "quantize: D2H scales");
    if (!rc && (e = cudaStreamSynchronize(be->stream)) != cudaSuccess) rc = cuda_fail(e, "quantize: sync");
    cudaFree(dw);
    cudaFree(dq);
    cudaFree(ds);
    return rc;
}

}  // extern "C"

// ===========================================================================
// Sharded layer.  NCCL is resolved at run time (dlopen of libnccl.so.2): in a
// process that already loaded NCCL (e.g. through torch.distributed) the same
// library instance is reused; this library has no link-time NCCL dependency.
// ===========================================================================
namespace {

struct NcclApi {
    bool loaded = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

template <typename F>
bool sym(void* h, const char* name, F* out)
{
    *out = reinterpret_cast<F>(dlsym(h, name));
    return *out != nullptr;
}

const NcclApi& nccl()
{
    std::call_once(g_nccl_once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            g_nccl.why = std::string("dlopen(libnccl.so.2) failed: ") + dlerror();
            return;
        }
        bool ok = sym(h, "ncclGetUniqueId", &g_nccl.GetUniqueId) &&
                  sym(h, "ncclCommInitRankConfig", &g_nccl.CommInitRankConfig) &&
                  sym(h, "ncclCommGetAsyncError", &g_nccl.CommGetAsyncError) &&
                  sym(h, "ncclCommAbort", &g_nccl.CommAbort) &&
                  sym(h, "ncclCommFinalize", &g_nccl.CommFinalize) &&
                  sym(h, "ncclCommDestroy", &g_nccl.CommDestroy) &&
                  sym(h, "ncclAllGather", &g_nccl.AllGather) &&
                  sym(h, "ncclGetErrorString", &g_nccl.GetErrorString);
        if (!ok) {
            g_nccl.why = "libnccl.so.2 lacks a required symbol";
            return;
        }
        g_nccl.loaded = true;
    });
    return g_nccl;
}

}  // namespace

// Device memory allocated on every rank and mapped into every other rank's
// address space (CUDA IPC over NVLink): peer[j] is rank j's copy.
struct SymAlloc {
    void* local = nullptr;
    size_t bytes = 0;
    void* peer[b200q8::kMaxRanks] = {};
};

struct b200q8_comm {
    ncclComm_t comm = nullptr;
    int device = 0, nranks = 1, rank = 0;
    double timeout_s = 60.0;
    cudaStream_t xstream = nullptr;  // internal stream for handle exchanges
    std::vector<SymAlloc> syms;
    SymAlloc flags;                  // u64 counts[nranks] per rank, advanced by the peers' GEMVs
    bool pending = false;            // a deferred gathered call's wait is still owed
};

namespace {

int nccl_fail(ncclResult_t r, const char* what)
{
    const char* s = nccl().GetErrorString ? nccl().GetErrorString(r) : "?";
    return fail(B200Q8_ERR_NCCL, "%s: NCCL error %d (%s)", what, (int)r, s);
}

// Non-blocking communicators may answer ncclInProgress; poll until done or the deadline.
int nccl_settle(b200q8_comm* c, ncclResult_t r, const char* what)
{
    if (r == ncclSuccess) return B200Q8_OK;
    if (r != ncclInProgress) return nccl_fail(r, what);
    // Enqueueing a collective finishes in microseconds: poll without sleeping (a sleep here
    // would leave the GPU idle), checking the deadline now and then.
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t i = 0;; i++) {
        ncclResult_t a = ncclInProgress;
        ncclResult_t q = nccl().CommGetAsyncError(c->comm, &a);
        if (q != ncclSuccess) return nccl_fail(q, "ncclCommGetAsyncError");
        if (a == ncclSuccess) return B200Q8_OK;
        if (a != ncclInProgress) return nccl_fail(a, what);
        if ((i & 1023) == 1023) {
            const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            if (el > c->timeout_s) return fail(B200Q8_ERR_TIMEOUT, "%s: still in progress after %.1f s", what, el);
            std::this_thread::yield();
        }
    }
}

// All ranks' 64-byte IPC handles, gathered through the library's own NCCL communicator.
int exchange_handles(b200q8_comm* c, const cudaIpcMemHandle_t& mine, std::vector<cudaIpcMemHandle_t>* all)
{
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    cudaError_t e;
    if (!c->xstream && (e = cudaStreamCreateWithFlags(&c->xstream, cudaStreamNonBlocking)) != cudaSuccess)
        return cuda_fail(e, "sym: stream");
    const size_t G = (size_t)c->nranks;
    void* d = nullptr;
    if ((e = cudaMalloc(&d, 64 * G)) != cudaSuccess) return cuda_fail(e, "sym: exchange buffer");
    int st = B200Q8_OK;
    if ((e = cudaMemcpy((char*)d + 64 * c->rank, &mine, 64, cudaMemcpyHostToDevice)) != cudaSuccess)
        st = cuda_fail(e, "sym: H2D handle");
    if (!st) st = nccl_settle(c, nccl().AllGather((char*)d + 64 * c->rank, d, 64, ncclUint8, c->comm, c->xstream),
                              "ncclAllGather(handles)");
    if (!st && (e = cudaStreamSynchronize(c->xstream)) != cudaSuccess) st = cuda_fail(e, "sym: sync");
    all->resize(G);
    if (!st && (e = cudaMemcpy(all->data(), d, 64 * G, cudaMemcpyDeviceToHost)) != cudaSuccess)
        st = cuda_fail(e, "sym: D2H handles");
    cudaFree(d);
    return st;
}

void sym_close(b200q8_comm* c, SymAlloc* s)
{
    for (int j = 0; j < c->nranks; j++)
        if (j != c->rank && s->peer[j]) cudaIpcCloseMemHandle(s->peer[j]);
    if (s->local) cudaFree(s->local);
    *s = SymAlloc();
}

// Collective: `bytes` of zeroed device memory on every rank, every copy mapped here.
int sym_open(b200q8_comm* c, size_t bytes, SymAlloc* out)
{
    SymAlloc s;
    s.bytes = bytes;
    cudaError_t e;
    if ((e = cudaMalloc(&s.local, bytes)) != cudaSuccess) {
        cudaGetLastError();
        return fail(B200Q8_ERR_ALLOC, "sym: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    if ((e = cudaMemset(s.local, 0, bytes)) != cudaSuccess) {
        cudaFree(s.local);
        return cuda_fail(e, "sym: memset");
    }
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, s.local)) != cudaSuccess) {
        cudaFree(s.local);
        return cuda_fail(e, "sym: cudaIpcGetMemHandle");
    }
    std::vector<cudaIpcMemHandle_t> all;
    int st = exchange_handles(c, h, &all);
    if (st) {
        cudaFree(s.local);
        return st;
    }
    s.peer[c->rank] = s.local;
    for (int j = 0; j < c->nranks; j++) {
        if (j == c->rank) continue;
        if ((e = cudaIpcOpenMemHandle(&s.peer[j], all[j], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
            s.peer[j] = nullptr;
            sym_close(c, &s);
            return cuda_fail(e, "sym: cudaIpcOpenMemHandle");
        }
    }
    *out = s;
    return B200Q8_OK;
}

void comm_release(b200q8_comm* c)
{
    for (auto& s : c->syms) sym_close(c, &s);
    c->syms.clear();
    if (c->flags.local) sym_close(c, &c->flags);
    if (c->xstream) cudaStreamDestroy(c->xstream);
    c->xstream = nullptr;
}

}  // namespace

extern "C" {

int b200q8_comm_sym_alloc(b200q8_comm* c, size_t bytes, void** local)
{
    if (!c || !local || bytes == 0) return fail(B200Q8_ERR_INVALID, "comm_sym_alloc: bad arguments");
    if (c->nranks > kMaxRanks) return fail(B200Q8_ERR_UNSUPPORTED, "comm_sym_alloc: at most %d ranks", kMaxRanks);
    int st = set_device(c->device);
    if (st) return st;
    SymAlloc s;
    if ((st = sym_open(c, bytes, &s))) return st;
    c->syms.push_back(s);
    *local = s.local;
    return B200Q8_OK;
}

int b200q8_comm_sym_free(b200q8_comm* c, void* local)
{
    if (!c || !local) return fail(B200Q8_ERR_INVALID, "comm_sym_free: bad arguments");
    for (size_t i = 0; i < c->syms.size(); i++) {
        if (c->syms[i].local == local) {
            sym_close(c, &c->syms[i]);
            c->syms.erase(c->syms.begin() + (long)i);
            return B200Q8_OK;
        }
    }
    return fail(B200Q8_ERR_INVALID, "comm_sym_free: %p is not a symmetric allocation of this communicator", local);
}

int b200q8_shard_range(size_t N, int nranks, int rank, size_t* row0, size_t* rows)
{
    if (nranks < 1 || rank < 0 || rank >= nranks || !row0 || !rows)
        return fail(B200Q8_ERR_INVALID, "shard_range: bad rank %d of %d", rank, nranks);
    const size_t per = (N + (size_t)nranks - 1) / (size_t)nranks;
    const size_t a = per * (size_t)rank;
    *row0 = a < N ? a : N;
    *rows = a < N ? ((N - a) < per ? (N - a) : per) : 0;
    return B200Q8_OK;
}

int b200q8_comm_unique_id(uint8_t id[128])
{
    if (!id) return fail(B200Q8_ERR_INVALID, "comm_unique_id: null id");
    if (!nccl().loaded) return fail(B200Q8_ERR_NCCL, "%s", nccl().why.c_str());
    ncclUniqueId u;
    ncclResult_t r = nccl().GetUniqueId(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    memcpy(id, &u, 128);
    return B200Q8_OK;
}

int b200q8_comm_init(int device, int nranks, int rank, const uint8_t id[128], double timeout_s,
                     b200q8_comm** out)
{
    if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks)
        return fail(B200Q8_ERR_INVALID, "comm_init: bad arguments");
    *out = nullptr;
    if (!nccl().loaded) return fail(B200Q8_ERR_NCCL, "%s", nccl().why.c_str());
    int st = set_device(device);
    if (st) return st;
    auto* c = new (std::nothrow) b200q8_comm();
    if (!c) return fail(B200Q8_ERR_ALLOC, "comm_init: out of host memory");
    c->device = device;
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_s = timeout_s > 0 ? timeout_s : 60.0;
    ncclUniqueId u;
    memcpy(&u, id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        int rc = nccl_fail(r, "ncclCommInitRankConfig");
        delete c;
        return rc;
    }
    st = nccl_settle(c, r, "ncclCommInitRankConfig");
    if (st) {
        std::string msg = t_last_error;
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        t_last_error = msg;
        return st;
    }
    *out = c;
    return B200Q8_OK;
}

int b200q8_comm_abort(b200q8_comm* c)
{
    if (!c) return B200Q8_OK;
    if (c->comm && nccl().loaded) nccl().CommAbort(c->comm);
    comm_release(c);
    delete c;
    return B200Q8_OK;
}

int b200q8_comm_destroy(b200q8_comm* c)
{
    if (!c) return B200Q8_OK;
    cudaDeviceSynchronize();  // this rank's stores into peers' memory are done
    if (c->xstream) {
        // Barrier before unmapping: a peer may still be storing into this rank's memory.
        // Every rank has xstream iff it made the same collective symmetric allocations.
        cudaIpcMemHandle_t none;
        memset(&none, 0, sizeof(none));
        std::vector<cudaIpcMemHandle_t> all;
        exchange_handles(c, none, &all);
    }
    comm_release(c);
    int rc = B200Q8_OK;
    if (c->comm && nccl().loaded) {
        ncclResult_t r = nccl().CommFinalize(c->comm);
        rc = nccl_settle(c, r, "ncclCommFinalize");
        if (rc) {
            nccl().CommAbort(c->comm);
        } else {
            r = nccl().CommDestroy(c->comm);
            if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommDestroy");
        }
    }
    delete c;
    return rc;
}

int b200q8_linear_q8_sharded_p2p_ex(b200q8_comm* c, void* out, int out_dtype, const void* inp, int in_dtype,
                                    const int8_t* w_shard, const float* scales_shard, const float* bias_shard,
                                    size_t M, size_t N, size_t K, unsigned int flags, b200q8_stream_t stream)
{
    if (!c) return fail(B200Q8_ERR_INVALID, "linear_q8_sharded_p2p: null comm");
    if (!valid_dtype(out_dtype) || !valid_dtype(in_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8_sharded_p2p: bad dtype");
    if (flags & ~(unsigned)B200Q8_P2P_DEFER_WAIT) return fail(B200Q8_ERR_INVALID, "linear_q8_sharded_p2p: bad flags");
    if (M == 0 || N == 0) return b200q8_comm_wait(c, stream);
    if (!out || !inp || !w_shard || !scales_shard)
        return fail(B200Q8_ERR_INVALID, "linear_q8_sharded_p2p: null pointer");
    const int G = c->nranks;
    if (G > kMaxRanks) return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_sharded_p2p: at most %d ranks", kMaxRanks);
    if (M > (size_t)gemv_i8_max_tokens())
        return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_sharded_p2p: at most %d tokens (M=%zu)", gemv_i8_max_tokens(), M);
    size_t row0 = 0, rows = 0, l0 = 0, lrows = 0;
    int st = b200q8_shard_range(N, G, c->rank, &row0, &rows);
    if (!st) st = b200q8_shard_range(N, G, G - 1, &l0, &lrows);
    if (st) return st;
    if (lrows == 0)  // every rank reaches the same verdict
        return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_sharded_p2p: N=%zu leaves rank %d without rows", N, G - 1);
    const size_t eb = out_dtype == B200Q8_F16 ? 2 : 4;
    const SymAlloc* sym = nullptr;
    for (const auto& s : c->syms)
        if ((uintptr_t)out >= (uintptr_t)s.local && (uintptr_t)out + M * N * eb <= (uintptr_t)s.local + s.bytes) sym = &s;
    if (!sym)
        return fail(B200Q8_ERR_INVALID,
                    "linear_q8_sharded_p2p: out must lie in a buffer from b200q8_comm_sym_alloc on this communicator");
    if ((st = set_device(c->device))) return st;
    cudaError_t e;
    if (!c->flags.local) {  // first call: the completion counts every peer adds to (collective)
        if ((st = sym_open(c, 256, &c->flags))) return st;
    }
    const size_t off = (uintptr_t)out - (uintptr_t)sym->local;
    P2POut po;
    po.ndst = G;
    for (int j = 0; j < G; j++) {
        po.dst[j] = (char*)sym->peer[j] + off;
        po.counts[j] = reinterpret_cast<unsigned long long*>(c->flags.peer[j]);
    }
    po.ldo = (long long)N;
    po.ocol0 = (int)row0;
    po.rank = c->rank;
    DeviceInfo d;
    if ((st = device_info(&d))) return st;
    LinearArgs a;
    a.x = inp;
    a.w = w_shard;
    a.scales = scales_shard;
    a.bias = bias_shard;
    a.out = out;
    a.M = M;
    a.N = rows;
    a.K = K;
    a.in_dtype = in_dtype;
    a.out_dtype = out_dtype;
    a.pdl = true;
    a.p2p = &po;
    if (!gemv_i8_supports(a))
        return fail(B200Q8_ERR_UNSUPPORTED, "linear_q8_sharded_p2p: needs K %% 16 == 0, 16 <= K <= 131072 and "
                                            "aligned pointers (K=%zu)", K);
    ScratchNeed need;
    gemv_i8_scratch_need(a, d.num_sms, &need.ws, &need.counters, &need.act, &need.exps);
    TcScratch scratch;
    if ((st = get_scratch(need, d.num_sms, (cudaStream_t)stream, &scratch))) return st;
    // A deferred wait of the previous call is owed before this call reads its input: it is paid
    // inside whichever of this call's kernels reads x first (the GEMV, or its prep kernel).
    if (c->pending) {
        po.wait_counts = reinterpret_cast<const unsigned long long*>(c->flags.local);
        po.wait_n = G;
    }
    // The shard runs on the streaming GEMV for a few tokens on a few MB of weights (as the local
    // dispatch would), else on the int8 tensor-core GEMV (the local dispatch's choice up to 4
    // tokens; beyond, it may pick the fp16 GEMM, which has no gathering epilogue).
    const bool simt = M <= (size_t)gemv_max_tokens() && rows * K <= kSimtMaxWeightBytes &&
                      gemv_stream_supports(a, d.max_smem);
    if (simt)
        e = launch_q8_gemv(a, d.num_sms, d.max_smem, (cudaStream_t)stream);
    else
        e = launch_q8_gemv_i8(a, d.num_sms, scratch, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "linear_q8_sharded_p2p: GEMV launch");
    // Behind the GEMV: publish this call once its grid has completed, and -- unless the wait is
    // deferred to the next gathered call or b200q8_comm_wait -- wait for every rank's part.
    // (Publishing from the GEMV's last CTA instead, after a system-scope fence in every CTA, measured
    // slower on two GPUs: 101.5 vs 94.7 us per 7B decode step; each CTA then waits for its NVLink
    // stores to be acknowledged before it retires.)
    const bool defer = (flags & B200Q8_P2P_DEFER_WAIT) != 0;
    po.wait_counts = reinterpret_cast<const unsigned long long*>(c->flags.local);
    po.wait_n = G;
    if ((e = launch_p2p_sync(po, true, !defer, (cudaStream_t)stream)) != cudaSuccess)
        return cuda_fail(e, "linear_q8_sharded_p2p: completion launch");
    c->pending = defer;  // the next gathered call (or b200q8_comm_wait) waits for it
    return B200Q8_OK;
}

int b200q8_linear_q8_sharded_p2p(b200q8_comm* c, void* out, int out_dtype, const void* inp, int in_dtype,
                                 const int8_t* w_shard, const float* scales_shard, const float* bias_shard,
                                 size_t M, size_t N, size_t K, b200q8_stream_t stream)
{
    return b200q8_linear_q8_sharded_p2p_ex(c, out, out_dtype, inp, in_dtype, w_shard, scales_shard, bias_shard,
                                           M, N, K, 0u, stream);
}

int b200q8_comm_wait(b200q8_comm* c, b200q8_stream_t stream)
{
    if (!c) return fail(B200Q8_ERR_INVALID, "comm_wait: null comm");
    if (!c->pending) return B200Q8_OK;
    int st = set_device(c->device);
    if (st) return st;
    P2POut po;
    po.rank = c->rank;
    po.wait_counts = reinterpret_cast<const unsigned long long*>(c->flags.local);
    po.wait_n = c->nranks;
    cudaError_t e = launch_p2p_sync(po, false, true, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "comm_wait: wait launch");
    c->pending = false;
    return B200Q8_OK;
}



int b200q8_comm_allgather(b200q8_comm* c, void* buf, size_t count, int dtype, b200q8_stream_t stream)
{
    if (!c || !buf) return fail(B200Q8_ERR_INVALID, "comm_allgather: null argument");
    if (!valid_dtype(dtype)) return fail(B200Q8_ERR_INVALID, "comm_allgather: bad dtype");
    if (!nccl().loaded) return fail(B200Q8_ERR_NCCL, "%s", nccl().why.c_str());
    const size_t eb = dtype == B200Q8_F16 ? 2 : 4;
    ncclResult_t r = nccl().AllGather((char*)buf + (size_t)c->rank * count * eb, buf, count,
                                      dtype == B200Q8_F16 ? ncclFloat16 : ncclFloat32, c->comm,
                                      (cudaStream_t)stream);
    return nccl_settle(c, r, "ncclAllGather");
}

int b200q8_linear_q8_sharded(b200q8_comm* c, void* out, int out_dtype, const void* inp, int in_dtype,
                             const int8_t* w_shard, const float* scales_shard, const float* bias_shard,
                             size_t M, size_t N, size_t K, void* gather, b200q8_stream_t stream)
{
    if (!c) return fail(B200Q8_ERR_INVALID, "linear_q8_sharded: null comm");
    if (!valid_dtype(out_dtype) || !valid_dtype(in_dtype))
        return fail(B200Q8_ERR_INVALID, "linear_q8_sharded: bad dtype");
    if (M == 0 || N == 0) return B200Q8_OK;
    const size_t G = (size_t)c->nranks;
    size_t row0 = 0, rows = 0;
    int st = b200q8_shard_range(N, c->nranks, c->rank, &row0, &rows);
    if (st) return st;
    const size_t per = (N + G - 1) / G;  // padded shard width
    const size_t eb = out_dtype == B200Q8_F16 ? 2 : 4;
    const ncclDataType_t nt = out_dtype == B200Q8_F16 ? ncclFloat16 : ncclFloat32;
    cudaStream_t s = (cudaStream_t)stream;
    const bool direct = (M == 1) && (N % G == 0);
    if (!direct && !gather)
        return fail(B200Q8_ERR_INVALID, "linear_q8_sharded: gather scratch required (M=%zu, N %% G = %zu)",
                    M, N % G);
    // local slice: [M, rows] with row stride `per` inside the rank's gather slot
    char* slot = direct ? (char*)out + (size_t)c->rank * per * eb
                        : (char*)gather + (size_t)c->rank * M * per * eb;
    if (rows > 0) {
        if (M == 1 || rows == per) {
            st = linear_impl(slot, out_dtype, inp, in_dtype, w_shard, scales_shard, bias_shard, nullptr,
                             M, rows, K, s);
        } else {
            // tail rank with fewer rows: compute each token row separately into the padded slot
            for (size_t m = 0; m < M && !st; m++)
                st = linear_impl(slot + m * per * eb, out_dtype, (const char*)inp + m * K * (in_dtype == B200Q8_F16 ? 2 : 4),
                                 in_dtype, w_shard, scales_shard, bias_shard, nullptr, 1, rows, K, s);
        }
        if (st) return st;
    }
    if (!nccl().loaded) return fail(B200Q8_ERR_NCCL, "%s", nccl().why.c_str());
    void* recv = direct ? out : gather;
    ncclResult_t r = nccl().AllGather(slot, recv, M * per, nt, c->comm, s);
    st = nccl_settle(c, r, "ncclAllGather");
    if (st) return st;
    if (!direct) {
        cudaError_t e = launch_gather_permute(gather, out, (int)eb, G, M, per, N, s);
        if (e != cudaSuccess) return cuda_fail(e, "gather permute launch");
    }
    return B200Q8_OK;
}

}  // extern "C"
