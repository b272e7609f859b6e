/*
 * b200q8.h -- C ABI of the B200 (sm_100a) quantized-linear library.
 *
 * This is the drop-in boundary for vvllm's quantized linear hot path
 * (hoobean1996/vvllm).  Every entry point returns an int status (0 = ok,
 * negative = error, see B200Q8_ERR_*) and never exits the process; the
 * message for the last failure on the calling thread is b200q8_last_error().
 * No entry point has a CPU fallback: if the GPU path cannot run, it fails.
 *
 * Three layers:
 *   1. kernel layer  -- device pointers, caller's stream, no allocation;
 *   2. backend layer -- the exact argument conventions of vvllm::Backend
 *      (device activations, host weight pointers cached on first use);
 *   3. sharded layer -- output-channel column sharding over NCCL.
 *
 * Types: int8 weights are row-major [N, K] with one fp32 scale per output row
 * (per-channel absmax).  Activations are fp32 or fp16 ("half", IEEE binary16);
 * all accumulation is fp32.
 */
#ifndef B200Q8_H
#define B200Q8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B200Q8_API __attribute__((visibility("default")))
#else
#define B200Q8_API
#endif

/* Same object as cudaStream_t (NULL = the legacy default stream). */
typedef struct CUstream_st* b200q8_stream_t;

#define B200Q8_ABI_VERSION 1

/* Status codes. */
#define B200Q8_OK 0
#define B200Q8_ERR_INVALID (-1)     /* bad argument (null pointer, bad dtype, size overflow) */
#define B200Q8_ERR_CUDA (-2)        /* a CUDA runtime / driver call failed */
#define B200Q8_ERR_UNSUPPORTED (-3) /* shape or device the kernels do not handle */
#define B200Q8_ERR_NCCL (-4)        /* an NCCL call failed or NCCL is unavailable */
#define B200Q8_ERR_TIMEOUT (-5)     /* a bounded wait (NCCL init, peer flag) ran out */
#define B200Q8_ERR_ALLOC (-6)       /* device allocation failed */
#define B200Q8_ERR_IO (-7)          /* a file could not be opened, mapped or written */
#define B200Q8_ERR_NOT_FOUND (-8)   /* no tensor of that name in the file */

/* Element types of activations / outputs. */
#define B200Q8_F32 0
#define B200Q8_F16 1

B200Q8_API int b200q8_abi_version(void);
/* Message of the last failing call made on this thread ("" if none). */
B200Q8_API const char* b200q8_last_error(void);
/* Number of kernel launches this library has issued in this process. */
B200Q8_API uint64_t b200q8_launch_count(void);

/* ------------------------------------------------------------------------
 * 1. Kernel layer.  All pointers are device pointers; work is enqueued on
 *    `stream` and the call returns without synchronising.
 * ------------------------------------------------------------------------ */

/* q[N,K], scales[N] = per-row absmax int8 quantization of w[N,K] (fp32).
 * Bit-identical to vvllm::quantize_per_channel
 * (replaces include/vvllm/quantize/quantize.h:18, src/quantize/quantize.cc:9-48). */
B200Q8_API int b200q8_quantize_per_channel(const float* w, size_t N, size_t K, int8_t* q, float* scales,
                                b200q8_stream_t stream);

/* The same from bfloat16 bits ([N,K] uint16, as a safetensors "BF16" tensor stores them): each
 * value is widened exactly (bits << 16) as vvllm's loader does (SafeTensorsLoader::bf16_to_f32,
 * src/safetensors/safetensors.cc:131-137, then quantize_per_channel in
 * src/model/qwen2/model.cc:27-38), so a checkpoint quantizes on the GPU from its stored bytes. */
B200Q8_API int b200q8_quantize_per_channel_bf16(const uint16_t* w, size_t N, size_t K, int8_t* q, float* scales,
                                                b200q8_stream_t stream);

/* out[M,N] = (inp[M,K] . float(weight[N,K])^T) * scales[N] + bias[N]
 * bias may be NULL.  inp is fp32 or fp16 (in_dtype); out is fp32 or fp16
 * (out_dtype).  inp must not overlap out.
 * Replaces vvllm::Backend::linear_q8 (include/vvllm/backend/backend.h:62-65)
 * as implemented by BackendCPU (src/backend/backend_naive.cc:155-291) and
 * BackendCUDA (src/backend/backend_cuda.cc:188-213). */
B200Q8_API int b200q8_linear_q8(void* out, int out_dtype, const void* inp, int in_dtype,
                     const int8_t* weight, const float* scales, const float* bias, size_t M,
                     size_t N, size_t K, b200q8_stream_t stream);

/* As b200q8_linear_q8, plus residual[M,N] (same dtype as out) added last.
 * out may be the same pointer as residual (in-place residual connection).
 * Replaces vvllm::Backend::linear_q8_add (include/vvllm/backend/backend.h:75-78;
 * src/backend/backend_naive.cc:322-335, src/backend/backend_cuda.cc:246-275). */
B200Q8_API int b200q8_linear_q8_add(void* out, int out_dtype, const void* inp, int in_dtype,
                         const int8_t* weight, const float* scales, const float* bias,
                         const void* residual, size_t M, size_t N, size_t K,
                         b200q8_stream_t stream);

/* Kernel choice for b200q8_linear_q8_ex. */
#define B200Q8_ALGO_AUTO 0  /* M <= 4 on <= 48 MiB of weights: SIMT; else M <= 4, or M <= 8 with
                               N >= 16384: TC_I8; larger M: TC for fp16, TC_I8 (42-token groups) for fp32 */
#define B200Q8_ALGO_SIMT 1  /* streaming SIMT GEMV (any dtype, any K; groups of <= 4 tokens) */
#define B200Q8_ALGO_TC 2    /* tcgen05 kind::f16 GEMM, weights dequantized into TMEM (fp16 activations) */
#define B200Q8_ALGO_TC_I8 3 /* tcgen05 kind::i8 GEMV on raw int8 weights, activations as exact 6-digit int8
                               (fp16 or fp32 activations, groups of <= 42 tokens, K <= 131072) */

/* Both of the above in one call (residual may be NULL) with an explicit
 * kernel choice; B200Q8_ERR_UNSUPPORTED if the chosen kernel cannot take the
 * shape.  Same semantics as b200q8_linear_q8 / b200q8_linear_q8_add. */
B200Q8_API int b200q8_linear_q8_ex(void* out, int out_dtype, const void* inp, int in_dtype,
                                   const int8_t* weight, const float* scales, const float* bias,
                                   const void* residual, size_t M, size_t N, size_t K, int algo,
                                   b200q8_stream_t stream);

/* Allocation-free linear_q8 / linear_q8_add (residual may be NULL), for
 * callers that may not call cudaMalloc: a device-memory pool or budget they
 * must not bypass, or a decode loop that cannot take the device-wide
 * synchronisation cudaMalloc and cudaFree may cause.  No counterpart in the
 * reference (vvllm has no allocation-free path).  It runs the int8 tensor-core
 * GEMV with its scratch in a fixed device array of about 2.6 MB that every GPU
 * loading this library holds until exit, and allocates nothing.  Limits: M <= 2
 * tokens, N <= 524288 rows, K % 16 == 0 with 16 <= K <= 131072, at most 160 SMs;
 * larger shapes return B200Q8_ERR_UNSUPPORTED.  The first call on a device looks
 * up the array's device address; make that first call before any stream
 * capture.  All calls share the array, which keeps the last call's contents
 * (each call clears the counters it needs); calls that overlap on one GPU race
 * on it and must be serialised by the caller. */
B200Q8_API int b200q8_linear_q8_noalloc(void* out, int out_dtype, const void* inp, int in_dtype,
                                        const int8_t* weight, const float* scales, const float* bias,
                                        const void* residual, size_t M, size_t N, size_t K,
                                        b200q8_stream_t stream);

/* Quantized lm_head with greedy decoding fused in: argmax[m] = the index of the largest of
 * out[m, 0..N) where out = b200q8_linear_q8(...), computed in the same kernel.  The order is the
 * reference CPU sampler's (SamplerCPU::sample, temperature 0: std::max_element over the logits,
 * src/sampler/sampler.cc:20-24): the first maximum wins, NaNs are skipped unless the first
 * logit is NaN (then 0); values are compared as stored in out_dtype.  out may be NULL (the logits
 * are then not written).  argmax is an int[M] device array.  M <= 42, K % 16 == 0,
 * 16 <= K <= 131072.  Stream-ordered; calls on one stream share a small scratch. */
B200Q8_API int b200q8_linear_q8_argmax(void* out, int out_dtype, const void* inp, int in_dtype,
                                       const int8_t* weight, const float* scales, const float* bias,
                                       size_t M, size_t N, size_t K, int* argmax, b200q8_stream_t stream);

/* ------------------------------------------------------------------------
 * Safetensors files on either side of the quantize step (host code).
 *
 * vvllm mmaps a safetensors checkpoint (src/safetensors/safetensors.cc:43-83), widens BF16 to
 * fp32 on the host (:101-117) and quantizes every projection on the host at load
 * (src/model/qwen2/model.cc:27-38).  b200q8_st_quantize does that quantization once, on the
 * GPU, and writes a quantized safetensors file; b200q8_st_open reads either kind with the same
 * layout rules (header parsed once, tensor data returned as pointers into the read-only map).
 * ------------------------------------------------------------------------ */
typedef struct b200q8_st b200q8_st;

/* Tensor element types as reported by b200q8_st_info (the file's dtype string otherwise). */
#define B200Q8_ST_F32 0
#define B200Q8_ST_F16 1
#define B200Q8_ST_BF16 2
#define B200Q8_ST_I8 3
#define B200Q8_ST_OTHER 4 /* U8, BOOL, I16..U64, F64, F8: carried through unchanged */

/* b200q8_st_quantize flags: also quantize the output head -- "lm_head.weight" (replaced), or
 * when the model ties it to the embedding, "model.embed_tokens.weight" (kept for the lookup,
 * quantized copy added). */
#define B200Q8_ST_LM_HEAD 1u

/* Opens and maps `path`, validates the header (offsets inside the data, sizes matching shapes,
 * no overlaps, no duplicate names).  Close with b200q8_st_close. */
B200Q8_API int b200q8_st_open(const char* path, b200q8_st** out);
B200Q8_API int b200q8_st_close(b200q8_st* f);
/* Tensors in file-data order: count, then per index its name, type, shape and data (pointers
 * stay valid until close). */
B200Q8_API int b200q8_st_count(const b200q8_st* f, size_t* n);
B200Q8_API int b200q8_st_info(const b200q8_st* f, size_t i, const char** name, int* dtype, size_t* ndim,
                              const size_t** shape, const void** data, size_t* nbytes);
/* Index of tensor `name`; B200Q8_ERR_NOT_FOUND if absent. */
B200Q8_API int b200q8_st_find(const b200q8_st* f, const char* name, size_t* index);
/* The quantized pair of projection `name` ("<name>.q8" I8 [N, K], "<name>.q8_scales" F32 [N]):
 * exactly what quantize_per_channel returns for the source weight (QuantizedWeight::data /
 * scales, include/vvllm/quantize/quantize.h); B200Q8_ERR_NOT_FOUND if the file has none. */
B200Q8_API int b200q8_st_quantized(const b200q8_st* f, const char* name, size_t* N, size_t* K, const int8_t** q,
                                   const float** scales);
/* Writes dst_path: src_path with every 2-D F32/BF16 tensor named "*_proj.weight" (the
 * projections vvllm quantizes: q/k/v/o, gate/up/down) replaced by its quantized pair, computed
 * on GPU `device` with the bit-exact quantize kernels; all other tensors are copied byte for
 * byte and the source metadata is kept (plus a "b200q8" entry).  gate_proj and up_proj stay
 * separate: quantization is per row, so quantizing their row concatenation (model.cc:66-76)
 * equals concatenating their quantized rows and scales. */
B200Q8_API int b200q8_st_quantize(const char* src_path, const char* dst_path, int device, unsigned int flags);

/* Projections with the elementwise op before them fused in.  vvllm runs, per layer,
 *   norm = rms_norm(x) then q/k/v (or gate_up) = linear_q8(norm)
 *     (include/vvllm/model/transformer.h:135-144, :167-169; rms_norm per token,
 *      src/model/transformer.cc:40-50, src/backend/backend_naive.cc:67-75), and
 *   h = silu_mul(gate_up[:, :K], gate_up[:, K:]) then x = linear_q8_add(h, x)
 *     (transformer.h:171-188; backend_naive.cc:293-300).
 * These compute the same results with the elementwise op done where the projection reads its
 * activations: for few tokens on small weights the streaming GEMV applies it while it stages
 * x (one launch, nothing written); for the int8 tensor-core GEMV its per-token prep kernel
 * applies it and writes the activations once; for the fp16 prefill GEMM it runs first as its
 * own kernel into scratch.
 * Arithmetic: rms = sqrt(sum_k x^2 / K + eps) (sum taken in double, one fixed order), then
 * x / rms * w; silu_mul = (g / (1 + exp(-g))) * u.  With fp16 activations the norm weight is
 * rounded to fp16 and the result to fp16, as vvllm's fp16 backend does
 * (src/backend/backend_cuda.cc:135-145, cuda_kernels.cu:876-910).  Results are bit-identical to
 * b200q8_rms_norm / b200q8_silu_mul followed by b200q8_linear_q8 / b200q8_linear_q8_add.
 *   rms_norm_linear_q8:    x [M, K] (in_dtype), norm_weight [K] fp32, out [M, N].
 *   silu_mul_linear_q8_add: gate_up [M, 2K] (in_dtype; gate = columns 0..K-1, up = K..2K-1),
 *                           residual [M, N] (out_dtype) or NULL, may equal out.
 * K % 4 == 0; x / gate_up 8-byte (fp16) or 16-byte (fp32) aligned; norm_weight 16-byte aligned. */
B200Q8_API int b200q8_rms_norm_linear_q8(void* out, int out_dtype, const void* x, int in_dtype,
                                         const float* norm_weight, float eps, const int8_t* weight,
                                         const float* scales, const float* bias, size_t M, size_t N, size_t K,
                                         b200q8_stream_t stream);
B200Q8_API int b200q8_silu_mul_linear_q8_add(void* out, int out_dtype, const void* gate_up, int in_dtype,
                                             const int8_t* weight, const float* scales, const float* bias,
                                             const void* residual, size_t M, size_t N, size_t K,
                                             b200q8_stream_t stream);

/* Up to B200Q8_MAX_GROUP projections of the same activations: the rms_norm + q / k / v
 * sequence of vvllm's attention block (include/vvllm/model/transformer.h:134-144, which calls
 * rms_norm_seq and then linear three times on norm_out).  Projection i:
 *   outs[i] [M, Ns[i]] = linear_q8(rms_norm(x), weights[i] [Ns[i], K], scales[i], biases[i])
 * with biases null (no bias anywhere) or biases[i] null for a projection without one, and
 * norm_weight null for no norm (then x is used as is).  Ns[i] == 0 skips projection i.
 * With M <= 4 and at most 48 MiB of weights in all, one SIMT launch stages (and normalizes) x
 * once for every projection; otherwise the projections run one after another through the
 * b200q8_linear_q8 dispatch (norm fused or materialized as for b200q8_rms_norm_linear_q8).
 * Each output equals the one of the single-projection call on the same inputs to 1e-5
 * normwise (fp32) / 2e-3 (fp16).  No vvllm counterpart as one call. */
#define B200Q8_MAX_GROUP 4
B200Q8_API int b200q8_linear_q8_group(int n, void* const* outs, int out_dtype, const void* x, int in_dtype,
                                      const float* norm_weight, float eps, const int8_t* const* weights,
                                      const float* const* scales, const float* const* biases, const size_t* Ns,
                                      size_t M, size_t K, b200q8_stream_t stream);

/* The elementwise ops alone, same arithmetic (vvllm Backend::rms_norm applied per token, as
 * rms_norm_seq does, src/model/transformer.cc:40-50; Backend::silu_mul over each gate_up row,
 * transformer.h:175-180): out [M, K] in dtype from x [M, K] / gate_up [M, 2K] in dtype. */
B200Q8_API int b200q8_rms_norm(void* out, const void* x, int dtype, const float* norm_weight, float eps, size_t M,
                               size_t K, b200q8_stream_t stream);
B200Q8_API int b200q8_silu_mul(void* out, const void* gate_up, int dtype, size_t M, size_t K,
                               b200q8_stream_t stream);

/* Device error word of the current device: bit 0 is set when a bounded wait
 * inside a tensor-core kernel gave up; bit 1 when a sharded call's wait for
 * the peers' outputs ran out (2 s).  Either way the outputs are invalid.
 * clear != 0 resets it.  Synchronises with the device. */
B200Q8_API int b200q8_kernel_error(int* code, int clear);

/* Diagnostics (no vvllm counterpart): the bounded wait a gathered call makes for its peers'
 * outputs (b200q8_linear_q8_sharded_p2p), run on caller memory so that a failure test can make
 * it run out on one GPU -- a count that nothing advances stands for a rank that never finished.
 * counts [n] (device uint64, 1 <= n <= 8) are completion counts as the gathered calls keep them
 * (2^20 per finished call); the wait holds until every counts[j] holds as many whole calls as
 * counts[self], within timeout_s (0.001 .. 10 s); otherwise bit 1 of b200q8_kernel_error is set
 * and the kernel returns.  where: 0 = the standalone wait kernel (what b200q8_comm_wait
 * enqueues); 1 = inside the int8 digit GEMV before it reads x (how a deferred wait is paid; a
 * give-up also sets bit 0 and the GEMV's outputs are invalid); 2 = inside that GEMV's per-token
 * prep kernel.  For 1 and 2 the GEMV out[1, N] = linear_q8(x[1, K], weight[N, K], scales) runs
 * with fp16 x and out, exactly as b200q8_linear_q8_ex(..., B200Q8_ALGO_TC_I8) would. */
B200Q8_API int b200q8_diag_peer_wait(const uint64_t* counts, int n, int self, double timeout_s, int where,
                                     void* out, const void* x, const int8_t* weight, const float* scales, size_t N,
                                     size_t K, b200q8_stream_t stream);

/* ------------------------------------------------------------------------
 * 2. Backend layer.  Mirrors vvllm::BackendCUDA's hot-path conventions:
 *    activations (out, inp, residual) are device pointers, fp32 or -- when the
 *    backend was created with fp16=1 -- fp16 data behind float* pointers
 *    (include/vvllm/model/transformer.h:82,93); weight, scales and bias are
 *    HOST pointers, uploaded on first use and cached by host address for the
 *    backend's lifetime (src/backend/backend_cuda.cc:51-77).  The int8 weight
 *    stays int8 on the device: no fp16 copy is ever built.
 * ------------------------------------------------------------------------ */
typedef struct b200q8_backend b200q8_backend;

/* Replaces BackendCUDA::BackendCUDA(bool fp16) (src/backend/backend_cuda.cc:13-26). */
B200Q8_API int b200q8_backend_create(int device, int fp16, b200q8_backend** out);
B200Q8_API int b200q8_backend_destroy(b200q8_backend* be);
/* Stream used by the backend calls (default: the legacy default stream). */
B200Q8_API int b200q8_backend_set_stream(b200q8_backend* be, b200q8_stream_t stream);
/* Bytes of device memory held by the weight cache. */
B200Q8_API int b200q8_backend_cached_bytes(const b200q8_backend* be, size_t* bytes);

/* Backend::linear_q8 (include/vvllm/backend/backend.h:64-65). */
B200Q8_API int b200q8_backend_linear_q8(b200q8_backend* be, float* out, const float* inp,
                             const int8_t* weight, const float* scales, const float* bias,
                             size_t M, size_t N, size_t K);
/* Backend::linear_q8_add (include/vvllm/backend/backend.h:76-78); out may equal residual. */
B200Q8_API int b200q8_backend_linear_q8_add(b200q8_backend* be, float* out, const float* inp,
                                 const int8_t* weight, const float* scales, const float* bias,
                                 const float* residual, size_t M, size_t N, size_t K);
/* quantize_per_channel with host input and host outputs, run on the GPU
 * (include/vvllm/quantize/quantize.h:18): q[N*K], scales[N]. */
B200Q8_API int b200q8_backend_quantize_per_channel(b200q8_backend* be, const float* weight, size_t N,
                                        size_t K, int8_t* q, float* scales);

/* ------------------------------------------------------------------------
 * 3. Sharded layer: output-channel (column) sharding of one projection over
 *    G GPUs of one node, outputs all-gathered over NVLink with NCCL.  The
 *    reference has no multi-GPU path; there is no counterpart to cite.
 * ------------------------------------------------------------------------ */
typedef struct b200q8_comm b200q8_comm;

/* Rows [row0, row0 + rows) of an N-row weight belong to `rank` of `nranks`:
 * every rank owns ceil(N / nranks) rows except the tail ranks. */
B200Q8_API int b200q8_shard_range(size_t N, int nranks, int rank, size_t* row0, size_t* rows);

/* 128-byte NCCL unique id, made on one rank and sent to the others by the caller. */
B200Q8_API int b200q8_comm_unique_id(uint8_t id[128]);
/* Non-blocking NCCL communicator init, polled until `timeout_s` runs out
 * (then the communicator is aborted and B200Q8_ERR_TIMEOUT returned). */
B200Q8_API int b200q8_comm_init(int device, int nranks, int rank, const uint8_t id[128], double timeout_s,
                     b200q8_comm** out);
B200Q8_API int b200q8_comm_destroy(b200q8_comm* comm);
/* Aborts outstanding NCCL work and frees the communicator. */
B200Q8_API int b200q8_comm_abort(b200q8_comm* comm);

/* In-place all-gather of equal slices: rank r's `count` elements sit at
 * buf + r * count (elements of `dtype`) and every rank ends with all of them. */
B200Q8_API int b200q8_comm_allgather(b200q8_comm* comm, void* buf, size_t count, int dtype,
                                     b200q8_stream_t stream);

/* Each rank computes its shard out_local[M, rows] = linear_q8 over its weight
 * rows (w_shard [rows, K], scales_shard, bias_shard), then all ranks gather
 * out[M, N].  out_dtype F16 or F32.  `gather` is caller scratch of
 * nranks * M * ceil(N/nranks) elements of out_dtype; it may be NULL when
 * M == 1 and nranks divides N (the gather then lands in `out` directly).
 * Stream-ordered on `stream`. */
B200Q8_API int b200q8_linear_q8_sharded(b200q8_comm* comm, void* out, int out_dtype, const void* inp,
                             int in_dtype, const int8_t* w_shard, const float* scales_shard,
                             const float* bias_shard, size_t M, size_t N, size_t K, void* gather,
                             b200q8_stream_t stream);

/* Symmetric device memory (collective: every rank calls it with the same
 * `bytes`, in the same order): `bytes` of zeroed memory on this GPU, mapped
 * into every other rank's address space (CUDA IPC over NVLink).  Freed by
 * b200q8_comm_sym_free (collective) or with the communicator. */
B200Q8_API int b200q8_comm_sym_alloc(b200q8_comm* comm, size_t bytes, void** local);
B200Q8_API int b200q8_comm_sym_free(b200q8_comm* comm, void* local);

/* Sharded layer with the gather fused into the GEMV -- the streaming GEMV for up to 4 tokens
 * on up to 48 MiB of weights (as b200q8_linear_q8 would pick), else the int8 tensor-core
 * GEMV: each rank's kernel stores
 * its [M, rows] slice straight into columns [row0, row0 + rows) of `out` on
 * EVERY rank (peer stores over NVLink).  A one-thread kernel behind it, once the
 * GEMV has completed, makes those stores visible system-wide and adds the call
 * to its completion count on each rank, then acquires every rank's count
 * (bounded: 2 s, then bit 1 of b200q8_kernel_error).  After a bounded wait gave
 * up in the int8 GEMV (the error word is set) nothing more is published until
 * b200q8_kernel_error clears it, so the peers' waits run out as well instead of
 * reading invalid outputs.  `out` [M, N] of out_dtype must
 * lie inside one b200q8_comm_sym_alloc buffer at the same offset on every
 * rank.  M <= 42; K % 16 == 0 and 16 <= K <= 131072; every rank must own rows.
 * A peer may run one call ahead of this rank, so consecutive calls must use
 * different `out` buffers (double-buffer) unless the caller has finished
 * reading the previous result before the peers can start the next call.
 * Every wait is relative -- each rank waits until every rank has completed as
 * many gathered calls as itself -- so nothing in a call is tied to the host's
 * count of calls: a sequence of these calls (with b200q8_comm_wait) may be
 * captured in a CUDA graph and replayed, the same sequence on every rank.
 * The first call allocates the completion counts (collective: all ranks make it,
 * outside any stream capture). */
B200Q8_API int b200q8_linear_q8_sharded_p2p(b200q8_comm* comm, void* out, int out_dtype, const void* inp,
                                            int in_dtype, const int8_t* w_shard, const float* scales_shard,
                                            const float* bias_shard, size_t M, size_t N, size_t K,
                                            b200q8_stream_t stream);

/* As b200q8_linear_q8_sharded_p2p, with B200Q8_P2P_DEFER_WAIT in `flags`: the call publishes
 * but enqueues no wait, so `out` is NOT yet complete in stream order.  The wait is owed by the
 * communicator and paid by its next gathered call (inside the first of that call's kernels that
 * reads its input) or by b200q8_comm_wait.  Any other consumer of `out` must come after
 * b200q8_comm_wait on the same stream.  Chains of deferred calls must stay on one stream, with
 * no kernel of their own between them that lets its dependents start before it completes. */
#define B200Q8_P2P_DEFER_WAIT 1u
B200Q8_API int b200q8_linear_q8_sharded_p2p_ex(b200q8_comm* comm, void* out, int out_dtype, const void* inp,
                                               int in_dtype, const int8_t* w_shard, const float* scales_shard,
                                               const float* bias_shard, size_t M, size_t N, size_t K,
                                               unsigned int flags, b200q8_stream_t stream);
/* Enqueues the wait a deferred gathered call still owes (no-op when none is owed). */
B200Q8_API int b200q8_comm_wait(b200q8_comm* comm, b200q8_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200Q8_H */
