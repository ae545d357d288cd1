/*
 * ORACLE -- test infrastructure, not product code.
 *
 * CPU restatement of image-forger's quantized-linear CPU path, used only by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg to check
 * and time the CUDA library.  Nothing in the qwen_imager_b200 package calls it.
 *
 * Parity pin: oracle_dequantize_bf16 reproduces MLX 0.32.3's own
 * `dequantized` tensors of the reference fixture (tests/golden/) bit for bit,
 * and oracle_linear_bf16 reproduces its `y` within the reference test's bound
 * (tests/test_oracle.py).
 *
 * Reference algorithm followed (paths relative to the reference repository):
 *   src/quant.rs:555-569  dequantize: per row, per column
 *                         word = packed[row*words + col/per_word]
 *                         q    = (word >> (bits*(col % per_word))) & mask
 *                         g    = row*groups + col/group
 *                         w    = scales_f[g] * (f32)q + offsets_f[g]   (f32)
 *   src/quant.rs:570-575  bf16 output: half::bf16::from_f32 (round to nearest even)
 *   src/quant.rs:105-113  forward_f32: W (f32, NOT rounded to bf16), x -> f32,
 *                         bias -> f32, candle_nn::Linear::forward = x.W^T then
 *                         broadcast_add(bias), all in f32
 *   src/quant.rs:119      .to_dtype(BF16) of the f32 result
 * The f32 GEMM itself lives in the third-party `gemm` crate behind candle-core
 * 0.9 (unpinned beyond "0.9": no Cargo.lock ships).  Its summation order is
 * not restated; the oracle accumulates each dot product in f64 and rounds it
 * to f32 once, i.e. it is at least as accurate as any f32 ordering.
 *
 * Build: oracle/Makefile (gcc -O2 -pthread -ffp-contract=off).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "qmm_oracle.h"

/* Row-parallel for, the stand-in for rayon's par_chunks_mut (src/quant.rs:559-569).
 * The image has no OpenMP runtime, so this is plain pthreads. */
typedef void (*row_fn)(void *ctx, int64_t row);
typedef struct {
    row_fn fn;
    void *ctx;
    int64_t begin, end;
} row_job;

static void *row_worker(void *arg) {
    row_job *j = (row_job *)arg;
    for (int64_t r = j->begin; r < j->end; r++) j->fn(j->ctx, r);
    return NULL;
}

static int g_threads = 0;

void oracle_set_threads(int32_t n) { g_threads = n; }

int32_t oracle_get_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int32_t)n : 1;
}

static void parallel_rows(int64_t rows, row_fn fn, void *ctx) {
    int nt = oracle_get_threads();
    if (nt > 256) nt = 256;
    if (rows < nt) nt = rows > 0 ? (int)rows : 1;
    if (nt <= 1) {
        for (int64_t r = 0; r < rows; r++) fn(ctx, r);
        return;
    }
    pthread_t tid[256];
    row_job jobs[256];
    int64_t chunk = (rows + nt - 1) / nt;
    int started = 0;
    for (int t = 0; t < nt; t++) {
        int64_t b = t * chunk, e = b + chunk < rows ? b + chunk : rows;
        if (b >= e) break;
        jobs[t] = (row_job){fn, ctx, b, e};
        if (pthread_create(&tid[t], NULL, row_worker, &jobs[t]) != 0) {
            row_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}

float oracle_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* half::bf16::from_f32: NaN keeps its sign and payload top bits with the quiet
 * bit set; everything else rounds to nearest, ties to even. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    uint32_t round_bit = 0x00008000u;
    if ((u & round_bit) && (u & (3u * round_bit - 1u))) return (uint16_t)((u >> 16) + 1u);
    return (uint16_t)(u >> 16);
}

void oracle_bf16_from_f32_array(const float *src, uint16_t *dst, int64_t count) {
    for (int64_t i = 0; i < count; i++) dst[i] = oracle_f32_to_bf16(src[i]);
}

void oracle_f32_from_bf16_array(const uint16_t *src, float *dst, int64_t count) {
    for (int64_t i = 0; i < count; i++) dst[i] = oracle_bf16_to_f32(src[i]);
}

/* src/quant.rs:555-569 */
typedef struct {
    const uint32_t *packed;
    const uint16_t *scales, *offsets;
    int64_t input;
    int32_t bits, group;
    float *dst_f32;
    uint16_t *dst_bf16;
} dq_ctx;

static void dq_row(void *p, int64_t row) {
    const dq_ctx *c = (const dq_ctx *)p;
    const int64_t groups = c->input / c->group;
    const int64_t per_word = 32 / c->bits;
    const int64_t words = c->input / per_word;
    const uint32_t mask = (1u << c->bits) - 1u;
    for (int64_t col = 0; col < c->input; col++) {
        uint32_t word = c->packed[row * words + col / per_word];
        uint32_t q = (word >> (c->bits * (col % per_word))) & mask;
        int64_t g = row * groups + col / c->group;
        float s = oracle_bf16_to_f32(c->scales[g]);
        float o = oracle_bf16_to_f32(c->offsets[g]);
        float prod = s * (float)q; /* exact: 8-bit x 8-bit significands */
        float w = prod + o;
        if (c->dst_f32) c->dst_f32[row * c->input + col] = w;
        else c->dst_bf16[row * c->input + col] = oracle_f32_to_bf16(w);
    }
}

void oracle_dequantize_f32(const uint32_t *packed, const uint16_t *scales,
                           const uint16_t *offsets, int64_t output, int64_t input,
                           int32_t bits, int32_t group, float *dst) {
    dq_ctx c = {packed, scales, offsets, input, bits, group, dst, NULL};
    parallel_rows(output, dq_row, &c);
}

/* src/quant.rs:570-573 (bf16 scales => bf16 output) */
void oracle_dequantize_bf16(const uint32_t *packed, const uint16_t *scales,
                            const uint16_t *offsets, int64_t output, int64_t input,
                            int32_t bits, int32_t group, uint16_t *dst) {
    dq_ctx c = {packed, scales, offsets, input, bits, group, NULL, dst};
    parallel_rows(output, dq_row, &c);
}

/* y_f32 [m, n] = x . W^T (+ bias), src/quant.rs:105-113, with W already f32. */
typedef struct {
    const float *x, *w;
    const uint16_t *bias;
    int64_t n, k;
    float *y;
} mm_ctx;

/* One output row; rows of W are visited in blocks so that a block stays in cache. */
static void mm_row(void *p, int64_t i) {
    const mm_ctx *c = (const mm_ctx *)p;
    const float *xr = c->x + i * c->k;
    for (int64_t j = 0; j < c->n; j++) {
        const float *wr = c->w + j * c->k;
        double acc = 0.0;
        for (int64_t t = 0; t < c->k; t++) acc += (double)xr[t] * (double)wr[t];
        float v = (float)acc;
        if (c->bias) v = v + oracle_bf16_to_f32(c->bias[j]);
        c->y[i * c->n + j] = v;
    }
}

void oracle_matmul_f32(const float *x, const float *w, const uint16_t *bias,
                       int64_t m, int64_t n, int64_t k, float *y) {
    mm_ctx c = {x, w, bias, n, k, y};
    parallel_rows(m, mm_row, &c);
}

/* forward_f32 followed by .to_dtype(BF16): src/quant.rs:105-113, 119. */
void oracle_linear_f32(const uint16_t *x, int64_t m, const uint32_t *packed,
                       const uint16_t *scales, const uint16_t *offsets,
                       const uint16_t *bias, int64_t n, int64_t k, int32_t bits,
                       int32_t group, float *w_scratch, float *x_scratch, float *y) {
    oracle_dequantize_f32(packed, scales, offsets, n, k, bits, group, w_scratch);
    oracle_f32_from_bf16_array(x, x_scratch, m * k);
    oracle_matmul_f32(x_scratch, w_scratch, bias, m, n, k, y);
}

static float act_apply(float t, int32_t act) {
    if (act == 1) {
        const float c = 0.7978845608028654f; /* sqrt(2/pi) */
        return 0.5f * t * (1.0f + tanhf(c * (t + 0.044715f * t * t * t)));
    }
    if (act == 2) return t / (1.0f + expf(-t));
    return t;
}

/*
 * Fused-epilogue reference: out = residual + gate * act(y_f32), evaluated in
 * f32 and rounded to bf16 once.  `y_f32` already includes the layer bias.
 * gate [n] and residual [m, n] may be NULL.
 */
void oracle_epilogue_bf16(const float *y_f32, const uint16_t *gate,
                          const uint16_t *residual, int32_t activation, int64_t m,
                          int64_t n, uint16_t *out) {
    for (int64_t i = 0; i < m; i++) {
        for (int64_t j = 0; j < n; j++) {
            float t = act_apply(y_f32[i * n + j], activation);
            if (gate) t = t * oracle_bf16_to_f32(gate[j]);
            if (residual) t = oracle_bf16_to_f32(residual[i * n + j]) + t;
            out[i * n + j] = oracle_f32_to_bf16(t);
        }
    }
}
