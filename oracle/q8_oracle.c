/*
 * q8_oracle.c -- CPU restatement of vvllm's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the sm_100a
 * kernels in vvllm_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it.  The product path
 * never calls into it and has no CPU fallback.
 *
 * Every function restates one reference function, cited as path:line inside
 * hoobean1996/vvllm:
 *
 *   q8o_quantize_per_channel  src/quantize/quantize.cc:9-48
 *   q8o_linear_q8             src/backend/backend_naive.cc:155-291 (x86 AVX2+FMA
 *                             branch :216-274, epilogue :283-288)
 *   q8o_linear_q8_add         src/backend/backend_naive.cc:322-335 (+ add :43-49)
 *   q8o_rms_norm              src/backend/backend_naive.cc:67-75, applied per token as
 *                             rms_norm_seq does (src/model/transformer.cc:40-50)
 *   q8o_silu_mul              src/backend/backend_naive.cc:293-300, applied to each
 *                             [gate | up] row (include/vvllm/model/transformer.h:175-180)
 *
 * The AVX2 branch keeps 4 accumulators of 8 lanes over 32-wide K blocks,
 * combines them pairwise, folds 8 lanes to 4, then does two horizontal adds,
 * and finishes with a scalar tail.  The restatement below performs the same
 * roundings in the same order with scalar code (fmaf for each vfmadd lane), so
 * its outputs are bit-identical to the reference compiled with
 * -O2 -std=c++20 -mavx2 -mfma.  Build with -ffp-contract=off (no implicit
 * fusion: the reference's ISO C++ mode does not contract either) and without
 * -ffast-math.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* quantize.cc:21 uses std::max(absmax, std::abs(w)), i.e. (a < b) ? b : a.
 * A NaN |w| therefore never replaces the running maximum. */
static inline float ref_max(float a, float b) { return (a < b) ? b : a; }
/* std::min(127, r) is (r < 127) ? r : 127, so NaN maps to 127. */
static inline float ref_min(float a, float b) { return (b < a) ? b : a; }

/* src/quantize/quantize.cc:9-48, one row. */
static void quantize_row(const float* w, size_t K, int8_t* q, float* scale_out)
{
    float absmax = 0.0f; /* :18 */
    for (size_t k = 0; k < K; k++) absmax = ref_max(absmax, fabsf(w[k])); /* :19-22 */
    float scale = absmax / 127.0f; /* :24 */
    *scale_out = scale;            /* :25 */
    if (scale == 0.0f) {           /* :27-34 */
        memset(q, 0, K);
        return;
    }
    float inv_scale = 1.0f / scale; /* :37 */
    for (size_t k = 0; k < K; k++) {
        float val = w[k] * inv_scale;                          /* :40 */
        val = ref_max(-128.0f, ref_min(127.0f, roundf(val))); /* :41 */
        q[k] = (int8_t)val;                                    /* :42 */
    }
}

void q8o_quantize_per_channel(const float* w, size_t N, size_t K, int8_t* q, float* scales)
{
    for (size_t j = 0; j < N; j++) quantize_row(w + j * K, K, q + j * K, scales + j);
}

/* One output element of src/backend/backend_naive.cc:160-288 (AVX2+FMA order). */
static float dot_row_avx2_order(const float* in_row, const int8_t* w_row, size_t K)
{
    float acc[4][8];
    memset(acc, 0, sizeof(acc)); /* :219-222 */
    size_t k = 0;
    for (; k + 32 <= K; k += 32) { /* :225 */
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 8; l++) {
                /* wf_g lane l is byte 8g+l (:231-243); in_g lane l is in_row[k+8g+l] (:246-249) */
                float wf = (float)w_row[k + 8 * g + l];
                acc[g][l] = fmaf(wf, in_row[k + 8 * g + l], acc[g][l]); /* :252-255 */
            }
    }
    float a0[8], a2[8];
    for (int l = 0; l < 8; l++) {
        a0[l] = acc[0][l] + acc[1][l]; /* :259 */
        a2[l] = acc[2][l] + acc[3][l]; /* :260 */
    }
    for (int l = 0; l < 8; l++) a0[l] = a0[l] + a2[l]; /* :261 */
    float r[4];
    for (int l = 0; l < 4; l++) r[l] = a0[l] + a0[l + 4]; /* :263-265 */
    /* _mm_hadd_ps(r, r) = {r0+r1, r2+r3, r0+r1, r2+r3}; twice -> (r0+r1)+(r2+r3) (:266-268) */
    float h0 = r[0] + r[1];
    float h1 = r[2] + r[3];
    float sum = h0 + h1;
    for (; k < K; k++) { /* :271-274, no contraction */
        float p = in_row[k] * (float)w_row[k];
        sum = sum + p;
    }
    return sum;
}

/* src/backend/backend_naive.cc:155-291 */
void q8o_linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales,
                   const float* bias, size_t M, size_t N, size_t K)
{
    for (size_t i = 0; i < M; i++) {
        const float* in_row = inp + i * K;
        for (size_t j = 0; j < N; j++) {
            float sum = dot_row_avx2_order(in_row, weight + j * K, K);
            sum = sum * scales[j];        /* :283 */
            if (bias) sum = sum + bias[j]; /* :284-287 */
            out[i * N + j] = sum;          /* :288 */
        }
    }
}

/* Rows [j0, j1) only, written to out[i*ldo + (j - j0)] -- lets callers check a
 * sample of output channels of a large matrix without computing all of it. */
void q8o_linear_q8_rows(float* out, size_t ldo, const float* inp, const int8_t* weight,
                        const float* scales, const float* bias, size_t M, size_t K, size_t j0,
                        size_t j1)
{
    for (size_t i = 0; i < M; i++) {
        for (size_t j = j0; j < j1; j++) {
            float sum = dot_row_avx2_order(inp + i * K, weight + j * K, K);
            sum = sum * scales[j];
            if (bias) sum = sum + bias[j];
            out[i * ldo + (j - j0)] = sum;
        }
    }
}

/* Selected rows (index list) -- same arithmetic as q8o_linear_q8. out is [M, n_idx]. */
void q8o_linear_q8_gather(float* out, const float* inp, const int8_t* weight, const float* scales,
                          const float* bias, size_t M, size_t K, const int64_t* rows, size_t n_idx)
{
    for (size_t i = 0; i < M; i++) {
        for (size_t t = 0; t < n_idx; t++) {
            size_t j = (size_t)rows[t];
            float sum = dot_row_avx2_order(inp + i * K, weight + j * K, K);
            sum = sum * scales[j];
            if (bias) sum = sum + bias[j];
            out[i * n_idx + t] = sum;
        }
    }
}

/* src/backend/backend_naive.cc:322-335: residual is saved first when it aliases
 * out, then out = linear_q8(...) and out = out + residual (add, :43-49). */
void q8o_linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales,
                       const float* bias, const float* residual, size_t M, size_t N, size_t K)
{
    float* saved = NULL;
    if (out == residual) {
        saved = (float*)malloc(M * N * sizeof(float));
        memcpy(saved, residual, M * N * sizeof(float));
        residual = saved;
    }
    q8o_linear_q8(out, inp, weight, scales, bias, M, N, K);
    for (size_t t = 0; t < M * N; t++) out[t] = out[t] + residual[t];
    free(saved);
}

/* ---- multi-threaded driver for the CPU baseline (disjoint output-channel slices) ---- */
typedef struct {
    float* out;
    const float* inp;
    const int8_t* w;
    const float* s;
    const float* b;
    size_t M, N, K, j0, j1;
} slice_job;

static void* slice_worker(void* arg)
{
    slice_job* jb = (slice_job*)arg;
    q8o_linear_q8_rows(jb->out + jb->j0, jb->N, jb->inp, jb->w, jb->s, jb->b, jb->M, jb->K, jb->j0,
                       jb->j1);
    return NULL;
}

/* Same result as q8o_linear_q8 (each output element is computed identically);
 * output channels are split into nthreads contiguous slices. */
int q8o_linear_q8_mt(float* out, const float* inp, const int8_t* weight, const float* scales,
                     const float* bias, size_t M, size_t N, size_t K, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    if ((size_t)nthreads > N) nthreads = (int)(N ? N : 1);
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    slice_job* jobs = (slice_job*)calloc((size_t)nthreads, sizeof(slice_job));
    if (!th || !jobs) {
        free(th);
        free(jobs);
        return -1;
    }
    for (int t = 0; t < nthreads; t++) {
        size_t j0 = N * (size_t)t / (size_t)nthreads, j1 = N * (size_t)(t + 1) / (size_t)nthreads;
        jobs[t] = (slice_job){out, inp, weight, scales, bias, M, N, K, j0, j1};
        pthread_create(&th[t], NULL, slice_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return 0;
}

/* src/backend/backend_naive.cc:67-75 for each of M tokens: the sum of squares is a left fold in
 * float (std::accumulate with acc + x * x, no contraction), rms = sqrt(sum / n + eps) (the float
 * sum divided by n converted to float; sqrt in double and narrowed, which equals the correctly
 * rounded float sqrt), then out = x / rms * w. */
void q8o_rms_norm(float* out, const float* x, const float* w, size_t M, size_t K, float eps)
{
    for (size_t m = 0; m < M; m++) {
        const float* xr = x + m * K;
        float* o = out + m * K;
        float sum = 0.0f;
        for (size_t k = 0; k < K; k++) {
            const float sq = xr[k] * xr[k];
            sum = sum + sq;
        }
        const float rms = (float)sqrt((double)(sum / (float)K + eps));
        for (size_t k = 0; k < K; k++) o[k] = xr[k] / rms * w[k];
    }
}

/* src/backend/backend_naive.cc:293-300 for each of M rows of gate_up = [gate (K) | up (K)]:
 * out = (g / (1 + exp(-g))) * u with the float exp. */
void q8o_silu_mul(float* out, const float* gate_up, size_t M, size_t K)
{
    for (size_t m = 0; m < M; m++) {
        const float* g = gate_up + m * 2 * K;
        const float* u = g + K;
        float* o = out + m * K;
        for (size_t k = 0; k < K; k++) {
            const float v = g[k];
            o[k] = (v / (1.0f + expf(-v))) * u[k];
        }
    }
}
