/*
 * lythref -- CPU restatement of the LYTH host IR evaluator, for TEST USE ONLY.
 *
 * This library is the checker, never the product: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it. It restates, function by function, the Rust
 * reference (QuantumDrizzy/LYTH) that cannot be compiled in this image (no cargo/rustc):
 *
 *   crates/lyth-lang/src/half.rs      f32 <-> binary16 / bfloat16, round-half-to-even
 *   crates/lyth-lang/src/inputs.rs    seed_of / element: the deterministic `lyth run` inputs
 *   crates/lyth-lang/src/ast.rs       ReduceOp::{identity, combine}, BinOp::apply
 *   crates/lyth-lang/src/ir.rs        view_index, base_index, the fma-formation rule
 *   crates/lyth-lang/src/eval.rs      eval_with_launch (elementwise, rank-2 walk, reduction
 *                                     two-stage order, tree_reduce), eval_contraction
 *   crates/lyth-circuit/src/lib.rs    f32s, widths_ct, circuits::Rng (SplitMix64)
 *   examples/{saxpy,axpby,lerp,horner,copy2d,transpose,sum,dot,max,min,
 *             hadamard_q,gate_q,cu_q,swap_q,matmul}.lyth   the bodies, lowered by hand with
 *                                     the fma rule of ir.rs:2388-2429
 *
 * The INT4/NF4 gate_proj GEMV has no executable reference (only cost fixtures); its routines
 * here define this project's format and are "parity unpinned".
 *
 * Build: oracle/Makefile (gcc, -ffp-contract=off so that every a*b+c the reference leaves
 * unfused stays unfused; fused steps call fmaf explicitly).
 */
#ifndef LYTHREF_H
#define LYTHREF_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- half.rs ---------------------------------------------------------------------- */
uint16_t lr_f32_to_f16_bits(float x);
float lr_f16_bits_to_f32(uint16_t h);
uint16_t lr_f32_to_bf16_bits(float x);
float lr_bf16_bits_to_f32(uint16_t h);
float lr_round_f16(float x);
float lr_round_bf16(float x);
void lr_round_bf16_array(uint64_t n, const float *in, float *out);
void lr_f32_to_f16_array(uint64_t n, const float *in, uint16_t *out);
void lr_f32_to_bf16_array(uint64_t n, const float *in, uint16_t *out);

/* ---- inputs.rs --------------------------------------------------------------------- */
/* ty: 0 = f32, 1 = f16, 2 = bf16 */
uint32_t lr_seed_of(const char *name);
float lr_element(const char *name, int ty, uint32_t i);
void lr_buffer(const char *name, int ty, uint32_t len, float *out);

/* ---- circuits::Rng (SplitMix64) and the seeded synthetic inputs ------------------------ */
uint64_t lr_splitmix_next(uint64_t *state);
/* Output i of the SplitMix64 stream started at `seed`, computed without the i calls before it. */
uint64_t lr_splitmix_at(uint64_t seed, uint64_t i);
/* out[i] = ((stream_i >> 40) as f32) * 2^-24 * 2 - 1, uniform in [-1, 1). */
void lr_uniform(uint64_t seed, uint64_t n, float *out);
/* Box-Muller on stream outputs 2i, 2i+1 in f64, rounded once to f32. */
void lr_normal(uint64_t seed, uint64_t n, double mu, double sigma, float *out);

/* ---- ast.rs ---------------------------------------------------------------------------- */
/* op: 0 = sum, 1 = max, 2 = min */
float lr_identity(int op);
float lr_combine(int op, float a, float b);

/* ---- the elementwise bodies, lowered (ir.rs:2388-2429 decides which a*b+c is one fma) -- */
void lr_saxpy(uint64_t n, float a, const float *x, float *y);
void lr_axpby(uint64_t n, float a, float b, const float *x, float *y);
void lr_lerp(uint64_t n, float t, const float *x, const float *y, float *z);
void lr_horner(uint64_t n, float c0, float c1, float c2, float c3, const float *x, float *y);
/* rank-2 walk, eval.rs:202-257 */
void lr_copy2d(uint32_t rows, uint32_t cols, const float *a, float *b);
void lr_transpose(uint32_t rows, uint32_t cols, const float *a, float *b);

/* ---- reductions: eval.rs:314-345 and tree_reduce eval.rs:537-546 ------------------------ */
/* y may be NULL (sum/max/min of x); with y the per-element value is x*y (dot). block must
 * be a power of two for the tree to cover every slot, as the reference's emitter requires.
 * Returns 0, or -1 on a zero grid/block. */
int lr_reduce(int op, uint64_t n, const float *x, const float *y, uint32_t grid, uint32_t block,
              float *partial);
/* f64 sum of x (or x*y), for the tolerance of a combined total. */
double lr_sum_f64(uint64_t n, const float *x, const float *y);

/* ---- contraction: eval_contraction, eval.rs:374-526 ------------------------------------- */
/* C[i,j] = sum_p A[i,p]*B[p,j], p ascending, mul.rn then add.rn, acc from 0.0.
 * Rows [row_begin, row_end) only, so a large problem can be sampled. */
void lr_matmul(uint32_t m, uint32_t n, uint32_t k, const float *a, const float *b, float *c,
               uint32_t row_begin, uint32_t row_end);

/* ---- split views: ir.rs:78-81 and base_index ir.rs:340-351 ------------------------------ */
uint64_t lr_view_index(uint64_t w, uint32_t part, uint64_t k);
/* lyth-circuit widths_ct: the inner width counts elements of the parent view (lost bit c). */
void lr_widths_ct(uint32_t c, uint32_t t, uint64_t *wc, uint64_t *wt);
/* The launch check of split_pairs (ir.rs:202-261): 0 when every level divides, else -1. */
int lr_check_split(uint64_t n, uint64_t w, int depth);

/* ---- state-vector gates: examples/{hadamard_q,gate_q,cu_q,swap_q}.lyth ------------------ */
/* m = ar ai br bi cr ci dr di. n amplitudes; qr/qi may alias re/im. Return 0 or -1 (refused). */
int lr_hadamard_q(uint64_t n, uint64_t w, float s, const float *re, const float *im,
                  float *qr, float *qi);
int lr_gate_q(uint64_t n, uint64_t w, const float *m, const float *re, const float *im,
              float *qr, float *qi);
int lr_cu_q(uint64_t n, uint64_t wc, uint64_t wt, const float *m, const float *re,
            const float *im, float *qr, float *qi);
int lr_swap_q(uint64_t n, uint64_t wc, uint64_t wt, const float *re, const float *im,
              float *qr, float *qi);

/* ---- gate_proj GEMV (format defined by this project; parity unpinned) ------------------- */
/* The 16 NF4 levels from the QLoRA construction (Dettmers et al., 2023). */
void lr_nf4_codebook(float out[16]);
/* Packed weights: row r (output) contiguous along k, byte (r*K + k)/2, low nibble = even k.
 * fmt 0 = INT4 (two's-complement nibble, -8..7), 1 = NF4 (nibble indexes the codebook).
 * scales: fp16 bits, [rows][K/group]. x: fp16 bits [K]. */
void lr_gemv_dequant(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                     const uint16_t *scales, float *out /* rows*k */);
/* y64[r] = sum_k f64(dequant(w)[r,k]) * f64(x[k]) (dequant is exact in f32). */
void lr_gemv_f64(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                 const uint16_t *scales, const uint16_t *x, double *y64);

/* Threads the OpenMP loops use (for the CPU-baseline report). */
int lr_threads(void);
void lr_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
