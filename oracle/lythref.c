/*
 * lythref.c -- CPU restatement of the LYTH host IR evaluator. TEST INFRASTRUCTURE ONLY:
 * the checker for the CUDA back end, never a product path. See lythref.h for the map from
 * each function to the reference file it restates.
 *
 * Every arithmetic step is the IEEE single-precision operation the reference evaluator
 * performs: `a + b`, `a * b` each round once (this file is compiled with
 * -ffp-contract=off so the compiler cannot fuse them), and `f32::mul_add` is `fmaf`.
 */
#include "lythref.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>
#include <pthread.h>
#include <unistd.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- a static range split over pthreads: element order never matters where it is used,
 * and where it does (a reduction's blocks) each range owns whole blocks. */
static int g_threads = 0;

int lr_threads(void) {
    if (g_threads <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        g_threads = c > 0 ? (int)c : 1;
    }
    return g_threads;
}
void lr_set_threads(int n) { g_threads = n; }

typedef void (*range_fn)(void *ctx, int64_t begin, int64_t end);
struct range_job { range_fn fn; void *ctx; int64_t begin, end; };

static void *range_thread(void *p) {
    struct range_job *j = (struct range_job *)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static void par_range(int64_t n, range_fn fn, void *ctx) {
    int t = lr_threads();
    if (t > 256) t = 256;
    if (n < 4096 || t <= 1) { fn(ctx, 0, n); return; }
    if ((int64_t)t > n) t = (int)n;
    pthread_t th[256];
    struct range_job jobs[256];
    int started[256];
    for (int i = 0; i < t; i++) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].begin = n * i / t; jobs[i].end = n * (i + 1) / t;
        started[i] = pthread_create(&th[i], NULL, range_thread, &jobs[i]) == 0;
        if (!started[i]) fn(ctx, jobs[i].begin, jobs[i].end);
    }
    for (int i = 0; i < t; i++) if (started[i]) pthread_join(th[i], NULL);
}

/* The arguments of every parallel loop below; each loop reads the fields it needs. */
struct args {
    uint64_t n, w, wc, wt, seed;
    uint32_t rows, cols, k, group, grid, block;
    int op, fmt;
    float a, b, c0, c1, c2, c3, s;
    double mu, sigma;
    const float *m, *x, *y, *re, *im, *cb;
    float *out, *qr, *qi;
    uint16_t *out16;
    const uint8_t *wq;
    const uint16_t *scales, *xh;
    double *y64;
};

#define RANGE(name) static void name(void *ctx_, int64_t lo, int64_t hi)
#define ARGS struct args *A = (struct args *)ctx_

/* ===================================================================== half.rs:28-151 */

/* f32 -> binary16 bits, round-half-to-even, as integer bit manipulation (half.rs:28-90). */
uint16_t lr_f32_to_f16_bits(float x) {
    uint32_t b = f2u(x);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    int32_t exp = (int32_t)((b >> 23) & 0xffu);
    uint32_t mant = b & 0x007fffffu;
    if (exp == 0xff) return mant != 0 ? (uint16_t)(sign | 0x7e00u) : (uint16_t)(sign | 0x7c00u);
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = mant | 0x00800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = 1u << (shift - 1);
        uint32_t low = m & ((1u << shift) - 1);
        uint32_t out = m >> shift;
        if (low > half || (low == half && (out & 1u) == 1u)) out += 1;
        return (uint16_t)(sign | out);
    }
    uint32_t half = 0x1000u;
    uint32_t low = mant & 0x1fffu;
    uint32_t out = ((uint32_t)e << 10) | (mant >> 13);
    if (low > half || (low == half && (out & 1u) == 1u)) out += 1;
    return (uint16_t)(sign | out);
}

/* binary16 bits -> f32, exact; subnormals renormalised (half.rs:93-122). */
float lr_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x03ffu;
    if (exp == 0) {
        if (mant == 0) return u2f(sign);
        uint32_t k = 31u - (uint32_t)__builtin_clz(mant);
        uint32_t e = k + 103u;
        uint32_t m = (mant << (23 - k)) & 0x007fffffu;
        return u2f(sign | (e << 23) | m);
    }
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (mant << 13));
    return u2f(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

float lr_round_f16(float x) { return lr_f16_bits_to_f32(lr_f32_to_f16_bits(x)); }

/* f32 -> bfloat16 bits: a rounding shift, NaN quieted explicitly (half.rs:128-141). */
uint16_t lr_f32_to_bf16_bits(float x) {
    uint32_t b = f2u(x);
    if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu) != 0)
        return (uint16_t)((b >> 16) | 0x0040u);
    uint32_t low = b & 0xffffu;
    uint32_t out = b >> 16;
    if (low > 0x8000u || (low == 0x8000u && (out & 1u) == 1u)) out += 1;
    return (uint16_t)out;
}

float lr_bf16_bits_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }
float lr_round_bf16(float x) { return lr_bf16_bits_to_f32(lr_f32_to_bf16_bits(x)); }

RANGE(rng_round_bf16) { ARGS; for (int64_t i = lo; i < hi; i++) A->out[i] = lr_round_bf16(A->x[i]); }
RANGE(rng_to_f16) { ARGS; for (int64_t i = lo; i < hi; i++) A->out16[i] = lr_f32_to_f16_bits(A->x[i]); }
RANGE(rng_to_bf16) { ARGS; for (int64_t i = lo; i < hi; i++) A->out16[i] = lr_f32_to_bf16_bits(A->x[i]); }

void lr_round_bf16_array(uint64_t n, const float *in, float *out) {
    struct args a = {0}; a.x = in; a.out = out;
    par_range((int64_t)n, rng_round_bf16, &a);
}
void lr_f32_to_f16_array(uint64_t n, const float *in, uint16_t *out) {
    struct args a = {0}; a.x = in; a.out16 = out;
    par_range((int64_t)n, rng_to_f16, &a);
}
void lr_f32_to_bf16_array(uint64_t n, const float *in, uint16_t *out) {
    struct args a = {0}; a.x = in; a.out16 = out;
    par_range((int64_t)n, rng_to_bf16, &a);
}

/* =================================================================== inputs.rs:18-57 */

uint32_t lr_seed_of(const char *name) {
    uint32_t a = 1;
    for (const unsigned char *p = (const unsigned char *)name; *p; ++p) a = a * 31u + *p;
    return a;
}

/* Knuth's multiplicative hash of the index, xor the mixed seed, >> 8, mod 2003, onto
 * [-4, 4) in steps of 1/251; rounded to the buffer's width at the source (inputs.rs:33-52). */
float lr_element(const char *name, int ty, uint32_t i) {
    uint32_t h = ((i * 2654435761u) ^ (lr_seed_of(name) * 0x85EBCA6Bu)) >> 8;
    float v = (float)(h % 2003u) / 251.0f - 4.0f;
    if (ty == 1) return lr_round_f16(v);
    if (ty == 2) return lr_round_bf16(v);
    return v;
}

void lr_buffer(const char *name, int ty, uint32_t len, float *out) {
    for (uint32_t i = 0; i < len; i++) out[i] = lr_element(name, ty, i);
}

/* ============================================ lyth-circuit/src/lib.rs:418-433 (Rng) */

static inline uint64_t splitmix_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t lr_splitmix_next(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ull;
    return splitmix_mix(*state);
}

/* The state after i+1 calls is seed + (i+1)*gamma, so output i needs no loop. */
uint64_t lr_splitmix_at(uint64_t seed, uint64_t i) {
    return splitmix_mix(seed + (i + 1) * 0x9E3779B97F4A7C15ull);
}

static inline float uniform_of(uint64_t r) {
    return (float)(r >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f;
}

RANGE(rng_uniform) { ARGS; for (int64_t i = lo; i < hi; i++) A->out[i] = uniform_of(lr_splitmix_at(A->seed, (uint64_t)i)); }

void lr_uniform(uint64_t seed, uint64_t n, float *out) {
    struct args a = {0}; a.seed = seed; a.out = out;
    par_range((int64_t)n, rng_uniform, &a);
}

RANGE(rng_normal) {
    ARGS;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = lo; i < hi; i++) {
        /* u1 in (0, 1]: 53-bit uniforms, shifted off zero so the log is finite. */
        double u1 = ((double)(lr_splitmix_at(A->seed, 2 * (uint64_t)i) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(lr_splitmix_at(A->seed, 2 * (uint64_t)i + 1) >> 11) * (1.0 / 9007199254740992.0);
        double z = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
        A->out[i] = (float)(A->mu + A->sigma * z);
    }
}

void lr_normal(uint64_t seed, uint64_t n, double mu, double sigma, float *out) {
    struct args a = {0}; a.seed = seed; a.mu = mu; a.sigma = sigma; a.out = out;
    par_range((int64_t)n, rng_normal, &a);
}

/* ====================================================== ast.rs:178-249 and :559-568 */

float lr_identity(int op) {
    if (op == 1) return -INFINITY;
    if (op == 2) return INFINITY;
    return 0.0f;
}

/* f32::max / f32::min: the non-NaN operand when exactly one is NaN. */
static inline float rust_max(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}
static inline float rust_min(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a < b ? a : b;
}

/* ReduceOp::combine: sum adds; max/min take the positive (max) or negative (min) zero when
 * both operands are zeros, and otherwise defer to f32::max / f32::min. */
float lr_combine(int op, float a, float b) {
    if (op == 1) {
        if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
        return rust_max(a, b);
    }
    if (op == 2) {
        if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
        return rust_min(a, b);
    }
    float s = a + b;
    return s;
}

/* ============================================ elementwise bodies (eval.rs:262-308) */

/* saxpy.lyth `y = a * x + y`: Add(Mul(a, x), y) -> fma(a, x, y). */
RANGE(rng_saxpy) { ARGS; for (int64_t i = lo; i < hi; i++) A->out[i] = fmaf(A->a, A->x[i], A->out[i]); }
void lr_saxpy(uint64_t n, float a, const float *x, float *y) {
    struct args g = {0}; g.a = a; g.x = x; g.out = y;
    par_range((int64_t)n, rng_saxpy, &g);
}

/* axpby.lyth `y = a * x + b * y`: the lhs is the Mul -> fma(a, x, mul(b, y)). */
RANGE(rng_axpby) {
    ARGS;
    for (int64_t i = lo; i < hi; i++) {
        float by = A->b * A->out[i];
        A->out[i] = fmaf(A->a, A->x[i], by);
    }
}
void lr_axpby(uint64_t n, float a, float b, const float *x, float *y) {
    struct args g = {0}; g.a = a; g.b = b; g.x = x; g.out = y;
    par_range((int64_t)n, rng_axpby, &g);
}

/* lerp.lyth `z = x + t * (y - x)`: the rhs is the Mul -> fma(t, sub(y, x), x). */
RANGE(rng_lerp) {
    ARGS;
    for (int64_t i = lo; i < hi; i++) {
        float d = A->y[i] - A->x[i];
        A->out[i] = fmaf(A->a, d, A->x[i]);
    }
}
void lr_lerp(uint64_t n, float t, const float *x, const float *y, float *z) {
    struct args g = {0}; g.a = t; g.x = x; g.y = y; g.out = z;
    par_range((int64_t)n, rng_lerp, &g);
}

/* horner.lyth `y = ((c3*x + c2)*x + c1)*x + c0` -> fma(fma(fma(c3, x, c2), x, c1), x, c0). */
RANGE(rng_horner) {
    ARGS;
    for (int64_t i = lo; i < hi; i++) {
        float v = A->x[i];
        A->out[i] = fmaf(fmaf(fmaf(A->c3, v, A->c2), v, A->c1), v, A->c0);
    }
}
void lr_horner(uint64_t n, float c0, float c1, float c2, float c3, const float *x, float *y) {
    struct args g = {0}; g.c0 = c0; g.c1 = c1; g.c2 = c2; g.c3 = c3; g.x = x; g.out = y;
    par_range((int64_t)n, rng_horner, &g);
}

/* copy2d.lyth `b[i, j] = a[i, j]` over `space i, j : rows, cols` (eval.rs:247-257). */
RANGE(rng_copy) { ARGS; for (int64_t k = lo; k < hi; k++) A->out[k] = A->x[k]; }
void lr_copy2d(uint32_t rows, uint32_t cols, const float *a, float *b) {
    struct args g = {0}; g.x = a; g.out = b;
    par_range((int64_t)rows * cols, rng_copy, &g);
}

/* transpose.lyth `b[j, i] = a[i, j]`: linear k -> (i, j) = (k / cols, k % cols); `a` is
 * row-major with rows of `cols`, `b` with rows of `rows`, its indices swapped. */
RANGE(rng_transpose) {
    ARGS;
    for (int64_t k = lo; k < hi; k++) {
        uint64_t i = (uint64_t)k / A->cols, j = (uint64_t)k % A->cols;
        A->out[j * A->rows + i] = A->x[i * A->cols + j];
    }
}
void lr_transpose(uint32_t rows, uint32_t cols, const float *a, float *b) {
    struct args g = {0}; g.rows = rows; g.cols = cols; g.x = a; g.out = b;
    par_range((int64_t)rows * cols, rng_transpose, &g);
}

/* ================================================ reductions (eval.rs:314-345, 537-546) */

/* tree_reduce: halve the stride, combine slots[t] with slots[t + stride], repeat. */
static float tree_reduce(float *slots, uint32_t len, int op) {
    uint32_t stride = len / 2;
    while (stride > 0) {
        for (uint32_t t = 0; t < stride; t++) slots[t] = lr_combine(op, slots[t], slots[t + stride]);
        stride /= 2;
    }
    return len ? slots[0] : lr_identity(op);
}

/* Per block b: each thread t folds elements b*block + t, + grid*block, ... in sequence,
 * starting from the identity; then the block's slots go through the tree. */
RANGE(rng_reduce) {
    ARGS;
    float *slots = (float *)malloc(sizeof(float) * A->block);
    if (!slots) return;
    uint64_t stride = (uint64_t)A->grid * A->block;
    for (int64_t b = lo; b < hi; b++) {
        for (uint32_t t = 0; t < A->block; t++) {
            float acc = lr_identity(A->op);
            for (uint64_t i = (uint64_t)b * A->block + t; i < A->n; i += stride) {
                float v;
                if (A->y) { v = A->x[i] * A->y[i]; } else { v = A->x[i]; }
                acc = lr_combine(A->op, acc, v);
            }
            slots[t] = acc;
        }
        A->out[b] = tree_reduce(slots, A->block, A->op);
    }
    free(slots);
}

int lr_reduce(int op, uint64_t n, const float *x, const float *y, uint32_t grid, uint32_t block,
              float *partial) {
    if (grid == 0 || block == 0) return -1;
    struct args g = {0};
    g.op = op; g.n = n; g.x = x; g.y = y; g.grid = grid; g.block = block; g.out = partial;
    par_range((int64_t)grid, rng_reduce, &g);
    return 0;
}

double lr_sum_f64(uint64_t n, const float *x, const float *y) {
    double s = 0.0;
    for (uint64_t i = 0; i < n; i++) s += y ? (double)x[i] * (double)y[i] : (double)x[i];
    return s;
}

/* ======================================================= eval_contraction, eval.rs:374-526 */

RANGE(rng_matmul) {
    ARGS;
    /* Columns in blocks so the inner p loop streams rows of b; each c[i, j] is still its own
     * accumulator, walked p = 0, 1, ..., k-1 from the sum identity 0.0. */
    enum { JB = 256 };
    float acc[JB];
    uint32_t n = A->cols, k = A->k;
    for (int64_t i = lo; i < hi; i++) {
        for (uint32_t j0 = 0; j0 < n; j0 += JB) {
            uint32_t jn = (n - j0) < JB ? (n - j0) : JB;
            for (uint32_t j = 0; j < jn; j++) acc[j] = 0.0f;
            for (uint32_t p = 0; p < k; p++) {
                float av = A->x[(uint64_t)i * k + p];
                const float *brow = A->y + (uint64_t)p * n + j0;
                for (uint32_t j = 0; j < jn; j++) {
                    float prod = av * brow[j];
                    acc[j] = acc[j] + prod;
                }
            }
            for (uint32_t j = 0; j < jn; j++) A->out[(uint64_t)i * n + j0 + j] = acc[j];
        }
    }
}

void lr_matmul(uint32_t m, uint32_t n, uint32_t k, const float *a, const float *b, float *c,
               uint32_t row_begin, uint32_t row_end) {
    if (row_end > m) row_end = m;
    if (row_begin >= row_end) return;
    struct args g = {0};
    g.cols = n; g.k = k; g.x = a; g.y = b;
    /* The range function indexes rows from 0; shift the pointers to the first row. */
    g.x = a + (uint64_t)row_begin * k;
    g.out = c + (uint64_t)row_begin * n;
    int64_t rowsn = (int64_t)(row_end - row_begin);
    /* par_range runs small ranges inline; rows are heavy, so split them even when few. */
    int t = lr_threads();
    if (t > 1 && rowsn > 1) {
        if (t > 256) t = 256;
        if ((int64_t)t > rowsn) t = (int)rowsn;
        pthread_t th[256];
        struct range_job jobs[256];
        int started[256];
        for (int i = 0; i < t; i++) {
            jobs[i].fn = rng_matmul; jobs[i].ctx = &g;
            jobs[i].begin = rowsn * i / t; jobs[i].end = rowsn * (i + 1) / t;
            started[i] = pthread_create(&th[i], NULL, range_thread, &jobs[i]) == 0;
            if (!started[i]) rng_matmul(&g, jobs[i].begin, jobs[i].end);
        }
        for (int i = 0; i < t; i++) if (started[i]) pthread_join(th[i], NULL);
    } else {
        rng_matmul(&g, 0, rowsn);
    }
}

/* ================================================= split views (ir.rs:78-81, :340-351) */

uint64_t lr_view_index(uint64_t w, uint32_t part, uint64_t k) {
    return (k / w) * 2 * w + (uint64_t)part * w + (k % w);
}

void lr_widths_ct(uint32_t c, uint32_t t, uint64_t *wc, uint64_t *wt) {
    *wc = 1ull << c;
    *wt = t < c ? (1ull << t) : (1ull << (t - 1));
}

/* split_pairs (ir.rs:202-261): a level of length len splits by w exactly when w >= 1 and
 * 2w divides len. */
int lr_check_split(uint64_t len, uint64_t w, int depth) {
    (void)depth;
    if (w == 0) return -1;
    if (len % (2 * w) != 0) return -1;
    return 0;
}

/* ================================ state-vector gates: the bodies of the _q examples, lowered */

/* hadamard_q.lyth: q0 = s * (p0 + p1), q1 = s * (p0 - p1); Mul of a Bin, so no fma. */
RANGE(rng_hadamard) {
    ARGS;
    for (int64_t k = lo; k < hi; k++) {
        uint64_t i0 = lr_view_index(A->w, 0, (uint64_t)k), i1 = lr_view_index(A->w, 1, (uint64_t)k);
        float p0r = A->re[i0], p0i = A->im[i0], p1r = A->re[i1], p1i = A->im[i1];
        float ar = p0r + p1r, ai = p0i + p1i, sr = p0r - p1r, si = p0i - p1i;
        A->qr[i0] = A->s * ar;
        A->qi[i0] = A->s * ai;
        A->qr[i1] = A->s * sr;
        A->qi[i1] = A->s * si;
    }
}

int lr_hadamard_q(uint64_t n, uint64_t w, float s, const float *re, const float *im,
                  float *qr, float *qi) {
    if (lr_check_split(n, w, 0)) return -1;
    struct args g = {0}; g.w = w; g.s = s; g.re = re; g.im = im; g.qr = qr; g.qi = qi;
    par_range((int64_t)(n / 2), rng_hadamard, &g);
    return 0;
}

/* gate_q.lyth, lowered by the fma rule:
 *   q0r = fma(ar, p0r, fma(-ai, p0i, fma(br, p1r, mul(-bi, p1i))))
 *   q0i = fma(ar, p0i, fma( ai, p0r, fma(br, p1i, mul( bi, p1r))))
 *   q1r = fma(cr, p0r, fma(-ci, p0i, fma(dr, p1r, mul(-di, p1i))))
 *   q1i = fma(cr, p0i, fma( ci, p0r, fma(dr, p1i, mul( di, p1r)))) */
static inline void u_chains(const float *m, float p0r, float p0i, float p1r, float p1i,
                            float *q0r, float *q0i, float *q1r, float *q1i) {
    float ar = m[0], ai = m[1], br = m[2], bi = m[3], cr = m[4], ci = m[5], dr = m[6], di = m[7];
    float t;
    t = (-bi) * p1i; *q0r = fmaf(ar, p0r, fmaf(-ai, p0i, fmaf(br, p1r, t)));
    t = bi * p1r;    *q0i = fmaf(ar, p0i, fmaf(ai, p0r, fmaf(br, p1i, t)));
    t = (-di) * p1i; *q1r = fmaf(cr, p0r, fmaf(-ci, p0i, fmaf(dr, p1r, t)));
    t = di * p1r;    *q1i = fmaf(cr, p0i, fmaf(ci, p0r, fmaf(dr, p1i, t)));
}

RANGE(rng_gate) {
    ARGS;
    for (int64_t k = lo; k < hi; k++) {
        uint64_t i0 = lr_view_index(A->w, 0, (uint64_t)k), i1 = lr_view_index(A->w, 1, (uint64_t)k);
        float a, b, c, d;
        u_chains(A->m, A->re[i0], A->im[i0], A->re[i1], A->im[i1], &a, &b, &c, &d);
        A->qr[i0] = a; A->qi[i0] = b; A->qr[i1] = c; A->qi[i1] = d;
    }
}

int lr_gate_q(uint64_t n, uint64_t w, const float *m, const float *re, const float *im,
              float *qr, float *qi) {
    if (lr_check_split(n, w, 0)) return -1;
    struct args g = {0}; g.w = w; g.m = m; g.re = re; g.im = im; g.qr = qr; g.qi = qi;
    par_range((int64_t)(n / 2), rng_gate, &g);
    return 0;
}

/* Leaf pXY of a depth-2 split: view (wt, part Y) of view (wc, part X) of the buffer,
 * resolved leaf first as base_index does. */
static inline uint64_t leaf2(uint64_t wc, uint64_t wt, uint32_t x, uint32_t y, uint64_t k) {
    return lr_view_index(wc, x, lr_view_index(wt, y, k));
}

/* cu_q.lyth: U on the control=1 leaves (p10, p11); the control=0 leaves are copied. */
RANGE(rng_cu) {
    ARGS;
    for (int64_t k = lo; k < hi; k++) {
        uint64_t i00 = leaf2(A->wc, A->wt, 0, 0, (uint64_t)k), i01 = leaf2(A->wc, A->wt, 0, 1, (uint64_t)k);
        uint64_t i10 = leaf2(A->wc, A->wt, 1, 0, (uint64_t)k), i11 = leaf2(A->wc, A->wt, 1, 1, (uint64_t)k);
        float p00r = A->re[i00], p00i = A->im[i00], p01r = A->re[i01], p01i = A->im[i01];
        float a, b, c, d;
        u_chains(A->m, A->re[i10], A->im[i10], A->re[i11], A->im[i11], &a, &b, &c, &d);
        A->qr[i10] = a; A->qi[i10] = b; A->qr[i11] = c; A->qi[i11] = d;
        A->qr[i00] = p00r; A->qi[i00] = p00i; A->qr[i01] = p01r; A->qi[i01] = p01i;
    }
}

int lr_cu_q(uint64_t n, uint64_t wc, uint64_t wt, const float *m, const float *re,
            const float *im, float *qr, float *qi) {
    if (lr_check_split(n, wc, 0) || lr_check_split(n / 2, wt, 1)) return -1;
    struct args g = {0}; g.wc = wc; g.wt = wt; g.m = m; g.re = re; g.im = im; g.qr = qr; g.qi = qi;
    par_range((int64_t)(n / 4), rng_cu, &g);
    return 0;
}

/* swap_q.lyth: |01> <-> |10>; |00> and |11> are copied. */
RANGE(rng_swap) {
    ARGS;
    for (int64_t k = lo; k < hi; k++) {
        uint64_t i00 = leaf2(A->wc, A->wt, 0, 0, (uint64_t)k), i01 = leaf2(A->wc, A->wt, 0, 1, (uint64_t)k);
        uint64_t i10 = leaf2(A->wc, A->wt, 1, 0, (uint64_t)k), i11 = leaf2(A->wc, A->wt, 1, 1, (uint64_t)k);
        float r00 = A->re[i00], m00 = A->im[i00], r01 = A->re[i01], m01 = A->im[i01];
        float r10 = A->re[i10], m10 = A->im[i10], r11 = A->re[i11], m11 = A->im[i11];
        A->qr[i00] = r00; A->qi[i00] = m00;
        A->qr[i01] = r10; A->qi[i01] = m10;
        A->qr[i10] = r01; A->qi[i10] = m01;
        A->qr[i11] = r11; A->qi[i11] = m11;
    }
}

int lr_swap_q(uint64_t n, uint64_t wc, uint64_t wt, const float *re, const float *im,
              float *qr, float *qi) {
    if (lr_check_split(n, wc, 0) || lr_check_split(n / 2, wt, 1)) return -1;
    struct args g = {0}; g.wc = wc; g.wt = wt; g.re = re; g.im = im; g.qr = qr; g.qi = qi;
    par_range((int64_t)(n / 4), rng_swap, &g);
    return 0;
}

/* ============================================================ gate_proj GEMV (unpinned) */

/* Inverse standard-normal CDF: Acklam's rational approximation (P. J. Acklam, 2003),
 * refined by two Halley steps on erfc, which brings it to double precision. */
static double norm_ppf(double p) {
    static const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                                1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
    static const double b[5] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                                6.680131188771972e+01, -1.328068155288572e+01};
    static const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                                -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
    static const double d[4] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                                3.754408661907416e+00};
    const double plow = 0.02425, phigh = 1 - plow;
    double x;
    if (p < plow) {
        double q = sqrt(-2 * log(p));
        x = (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
            ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    } else if (p <= phigh) {
        double q = p - 0.5, r = q * q;
        x = (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
            (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1);
    } else {
        double q = sqrt(-2 * log(1 - p));
        x = -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
            ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    }
    for (int it = 0; it < 2; it++) {
        double e = 0.5 * erfc(-x / sqrt(2.0)) - p;
        double u = e * sqrt(2 * 3.14159265358979323846) * exp(x * x / 2);
        x = x - u / (1 + x * u / 2);
    }
    return x;
}

/* NF4: 8 positive normal quantiles on linspace(offset, 0.5, 9)[:-1], 7 negative ones on
 * linspace(offset, 0.5, 8)[:-1], and an exact zero, sorted and normalised by the largest
 * magnitude. offset = 0.9677083 as published (the mean of 1 - 1/(2*15) and 1 - 1/(2*16)). */
void lr_nf4_codebook(float out[16]) {
    const double offset = 0.9677083;
    double v[16];
    int k = 0;
    for (int i = 0; i < 8; i++) v[k++] = norm_ppf(offset + (0.5 - offset) * i / 8.0);
    v[k++] = 0.0;
    for (int i = 0; i < 7; i++) v[k++] = -norm_ppf(offset + (0.5 - offset) * i / 7.0);
    for (int i = 1; i < 16; i++) {
        double t = v[i];
        int j = i - 1;
        while (j >= 0 && v[j] > t) { v[j + 1] = v[j]; j--; }
        v[j + 1] = t;
    }
    double mx = 0;
    for (int i = 0; i < 16; i++) if (fabs(v[i]) > mx) mx = fabs(v[i]);
    for (int i = 0; i < 16; i++) out[i] = (float)(v[i] / mx);
}

static inline float dequant_one(int fmt, const float *cb, uint8_t byte, int hi, float scale) {
    uint32_t nib = hi ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 0xfu);
    if (fmt == 0) {
        int q = (int)nib - ((nib & 8u) ? 16 : 0);
        float qf = (float)q;
        return qf * scale; /* exact: a 4-bit integer times an 11-bit significand */
    }
    return cb[nib] * scale; /* one rounding, mul.rn */
}

RANGE(rng_dequant) {
    ARGS;
    uint32_t groups = A->k / A->group;
    for (int64_t r = lo; r < hi; r++) {
        for (uint32_t c = 0; c < A->k; c++) {
            uint64_t e = (uint64_t)r * A->k + c;
            float s = lr_f16_bits_to_f32(A->scales[(uint64_t)r * groups + c / A->group]);
            A->out[e] = dequant_one(A->fmt, A->cb, A->wq[e >> 1], (int)(e & 1), s);
        }
    }
}

void lr_gemv_dequant(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                     const uint16_t *scales, float *out) {
    float cb[16];
    lr_nf4_codebook(cb);
    struct args g = {0};
    g.fmt = fmt; g.k = k; g.group = group; g.wq = w; g.scales = scales; g.out = out; g.cb = cb;
    par_range((int64_t)rows, rng_dequant, &g);
}

RANGE(rng_gemv) {
    ARGS;
    uint32_t groups = A->k / A->group;
    for (int64_t r = lo; r < hi; r++) {
        double acc = 0.0;
        for (uint32_t c = 0; c < A->k; c++) {
            uint64_t e = (uint64_t)r * A->k + c;
            float s = lr_f16_bits_to_f32(A->scales[(uint64_t)r * groups + c / A->group]);
            float wv = dequant_one(A->fmt, A->cb, A->wq[e >> 1], (int)(e & 1), s);
            acc += (double)wv * (double)lr_f16_bits_to_f32(A->xh[c]);
        }
        A->y64[r] = acc;
    }
}

void lr_gemv_f64(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                 const uint16_t *scales, const uint16_t *x, double *y64) {
    float cb[16];
    lr_nf4_codebook(cb);
    struct args g = {0};
    g.fmt = fmt; g.k = k; g.group = group; g.wq = w; g.scales = scales; g.xh = x; g.y64 = y64; g.cb = cb;
    par_range((int64_t)rows, rng_gemv, &g);
}
