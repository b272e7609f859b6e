// kernels.h -- internal launch interface between the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200q8 {

enum DType : int { kF32 = 0, kF16 = 1 };

// Output placement for the column-sharded path with an in-kernel gather: every
// output element is stored into `ndst` copies of the full [M, ldo] output
// (the local one and each peer's, mapped over NVLink), at column ocol0 + row.
//
// Completion: the GEMV's CTAs store and retire; they do not wait for the NVLink
// acknowledgements of their stores.  The small kernel launched behind the GEMV
// (launch_p2p_sync) passes griddepcontrol.wait once the GEMV grid has completed,
// then one thread makes its stores visible system-wide (one fence) and adds 2^20
// to counts[rank] on every rank.  So counts[j] on a rank holds 2^20 per call of
// rank j whose outputs have landed there.  Nothing is published after a launch
// that set the device error word (a bounded wait gave up): its peers' waits run
// out too, instead of reading invalid outputs.
//
// Waits are relative, so nothing about them is fixed at launch time and the calls
// can be captured in a CUDA graph and replayed: after the previous kernel in the
// stream (the previous call's sync kernel) has completed, a rank's own count holds
// all of its earlier calls; the wait holds until every counts[j] holds as many.
constexpr int kMaxRanks = 8;
constexpr int kCountShift = 20;  // each call adds 2^20 to every rank's count slot
struct P2POut {
    int ndst = 1;
    void* dst[kMaxRanks] = {};
    long long ldo = 0;
    int ocol0 = 0;
    unsigned long long* counts[kMaxRanks] = {};  // count array base on every rank
    int rank = 0;
    // Deferred wait of the previous gathered call: before x (or a residual) is read, every
    // rank's count in wait_counts[0..wait_n) must hold as many whole calls as
    // wait_counts[rank] (this rank's own count).  wait_counts null: nothing to wait for.
    const unsigned long long* wait_counts = nullptr;
    int wait_n = 0;
    unsigned long long wait_timeout_ns = 0;  // limit of that wait (0: the default, 2 s)
};

struct LinearArgs {
    const void* x = nullptr;        // [M, K] activations (in_dtype)
    const int8_t* w = nullptr;      // [N, K] int8, row-major
    const float* scales = nullptr;  // [N]
    const float* bias = nullptr;    // [N] or null
    const void* res = nullptr;      // [M, N] residual (out_dtype) or null
    void* out = nullptr;            // [M, N] (out_dtype)
    size_t M = 0, N = 0, K = 0;
    int in_dtype = kF32, out_dtype = kF32;
    bool pdl = false;               // launch with programmatic stream serialization
    const P2POut* p2p = nullptr;    // int8 digit GEMV and streaming GEMV (M <= 4): gather into peers' outputs
    // int8 digit GEMV only: greedy argmax of each token's outputs into amax_out[M] (keys and
    // counter are scratch that starts at zero and is left at zero).  out may then be null.
    unsigned long long* amax_keys = nullptr;
    unsigned int* amax_done = nullptr;
    int* amax_out = nullptr;
    // SIMT streaming GEMV and int8 digit GEMV: an elementwise prologue computed from x (the SIMT
    // kernel while it stages x, the digit GEMV's prep kernel into scratch; prologue.cuh;
    // kProNone: x is the activation).  x is then the prologue's
    // input: [M, K] for kProRmsNorm (norm_w [K], eps), [M, 2K] gate | up for kProSiluMul.
    int prologue = 0;
    const float* norm_w = nullptr;
    float eps = 0.0f;
    // int8 digit GEMV only: find the per-token exponents in the prep kernel even where the GEMV
    // would scan x itself (lets a deferred peer wait be paid in the prep kernel on any shape).
    bool force_prep = false;
    // int8 digit GEMV only: never have the prep kernel write the activations' digit tiles to
    // scratch (the GEMV then digitizes every stage itself); the allocation-free entry sets it.
    bool no_digit_images = false;
};

// The kernel behind a gathered call's GEMV (one thread does the work; it lets its own dependents
// launch at once, and they pass griddepcontrol.wait only when it is done).  After the previous
// kernel in the stream has completed: with `publish`, unless the device error word of the digit
// GEMV is set, one system-scope fence and 2^20 added to counts[d][rank] on each of the ndst
// ranks; with `wait`, a bounded wait (timeout_ns) until every wait_counts[j], j < n, holds as
// many whole calls as wait_counts[rank] (bit 1 of the error word on expiry).
cudaError_t launch_p2p_sync(const P2POut& po, bool publish, bool wait, cudaStream_t stream);
// Device address of that error word on the current device (looked up once per device), for the
// other kernels a gathered call may run (the streaming GEMV); null if the lookup failed.
int* p2p_error_word();

// Streaming SIMT GEMV, M <= gemv_max_tokens().  Also takes any M/K through a
// generic (slow, correct) kernel when the fast one cannot (alignment, K % 16).
cudaError_t launch_q8_gemv(const LinearArgs& a, int num_sms, size_t max_smem, cudaStream_t stream);
// The streaming SIMT kernel takes the shape (aligned, K % 16 == 0, M <= 4, x fits in shared
// memory); only then may a.prologue be set (it is applied while x is staged).
bool gemv_stream_supports(const LinearArgs& a, size_t max_smem);

// A group of up to kMaxGroup projections of the same x in one SIMT launch (x staged, and its
// prologue applied, once per CTA): matrix i is w[i] [Ns[i], a.K] with scales[i] and bias[i] (or
// null) into outs[i] [a.M, Ns[i]] in a.out_dtype (a.w, a.out, a.res and a.N are not used).
// cudaErrorNotSupported when the stream kernel cannot take the shapes or pointers.
constexpr int kMaxGroup = 4;  // B200Q8_MAX_GROUP
cudaError_t launch_q8_gemv_group(const LinearArgs& a, int n, const int8_t* const* w, const float* const* scales,
                                 const float* const* bias, void* const* outs, const size_t* Ns, int num_sms,
                                 size_t max_smem, cudaStream_t stream);
int gemv_max_tokens();
size_t gemv_smem_bytes(int M, int K);

// Per-row absmax quantization (bit-exact with vvllm::quantize_per_channel).
cudaError_t launch_q8_quantize(const float* w, size_t N, size_t K, int8_t* q, float* scales,
                               int num_sms, cudaStream_t stream);
// The same from bf16 bits (widened exactly, bits << 16).
cudaError_t launch_q8_quantize_bf16(const uint16_t* w, size_t N, size_t K, int8_t* q, float* scales, int num_sms,
                                    cudaStream_t stream);

// Scratch of the stream-K tensor-core GEMM: fp32 partial accumulators of split
// tiles and per-tile arrival counters (zero between launches; every launch
// leaves them zero unless a bounded wait gave up).
struct TcScratch {
    float* ws = nullptr;         // partial accumulators (fp32 or int32 words)
    size_t ws_floats = 0;
    int* counter_ptr = nullptr;  // per-tile arrival counters
    size_t counters = 0;
    int* exps = nullptr;         // the digit GEMV's prep kernel words [M][row splits]
    size_t exps_count = 0;
    unsigned char* act = nullptr;  // activations a prologue wrote for the following GEMV / GEMM
    size_t act_bytes = 0;
    unsigned long long* amax = nullptr;  // argmax keys [kMaxArgmaxTokens] + a counter word, zero at rest
};
constexpr int kMaxArgmaxTokens = 64;

// Tensor-core GEMV for M <= gemv_i8_max_tokens() with exact 6-digit int8
// activations (fp16 or fp32 inputs) and kind::i8 MMAs on the raw int8 weights.
cudaError_t launch_q8_gemv_i8(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream);
bool gemv_i8_supports(const LinearArgs& a);
// True when the GEMV computes the per-token exponents itself (one launch, x read only in-kernel,
// so a deferred peer wait can happen inside it).
bool gemv_i8_fused_exps(const LinearArgs& a);
// True when the GEMV's prep kernel writes every K-stage's digit tile to scratch once per launch.
bool gemv_i8_images(const LinearArgs& a);
int gemv_i8_max_tokens();
void gemv_i8_scratch_need(const LinearArgs& a, int num_sms, size_t* ws_floats, size_t* counters, size_t* act_bytes,
                          size_t* exps);
cudaError_t read_kernel_error_i8(int* code, bool clear);

// The int8 digit GEMV on a fixed file-scope device array instead of allocated
// scratch (see q8_gemv_tc.cu).  0: launched; 1..4: the shape exceeds the
// array's limits (tokens, rows, SM count, K/alignment, scratch size); -1: CUDA error in *err.
int launch_q8_gemv_i8_noalloc(const LinearArgs& a, int num_sms, cudaStream_t stream, cudaError_t* err);

// tcgen05 / TMEM GEMM for fp16 activations, M >= 1 (decode, skinny and prefill).
// Returns cudaErrorNotSupported when the shape is outside what it takes and
// cudaErrorMemoryAllocation when `scratch` is smaller than gemm_tc_scratch_need says.
cudaError_t launch_q8_gemm_tc(const LinearArgs& a, int num_sms, const TcScratch& scratch, cudaStream_t stream);
bool gemm_tc_supports(const LinearArgs& a);
void gemm_tc_scratch_need(const LinearArgs& a, int num_sms, size_t* ws_floats, size_t* counters);

// Reads (and optionally clears) the device error word the tensor-core kernel
// sets when a bounded wait gives up (bit 0).
cudaError_t read_kernel_error(int* code, bool clear);

// [G][M][Ns] (rank-major gather result) -> [M][N] (N = true width, Ns = padded shard width)
cudaError_t launch_gather_permute(const void* src, void* dst, int elem_bytes, size_t G, size_t M,
                                  size_t Ns, size_t N, cudaStream_t stream);

// Standalone prologue (prologue.cuh) over M tokens: out[M, K] in `dtype` from x ([M, K] for
// kProRmsNorm, [M, 2K] for kProSiluMul).  K % 4 == 0; x and out 8-byte (fp16) / 16-byte (fp32)
// aligned.  Same arithmetic as the prologue fused into the SIMT GEMV and the digit GEMV's prep.
cudaError_t launch_prologue(int pro, const void* x, void* out, int dtype, const float* norm_w, float eps, size_t M,
                            size_t K, bool pdl, cudaStream_t stream);

// Error reporting of the C ABI: record the message b200q8_last_error() returns, return status.
int fail(int status, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

// Counts every kernel launch made by this library (for the bench's launch count).
void note_launch();

}  // namespace b200q8
