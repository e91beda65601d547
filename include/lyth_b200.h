/*
 * lyth_b200.h -- the C ABI of liblyth_b200.so, a B200 (sm_100a) execution back end for the
 * kernel classes LYTH's `.lyth` compiler lowers to.
 *
 * Two surfaces:
 *
 *  1. The ADR-0016 callable surface, per kernel, with the exact names, signatures and
 *     contract macros LYTH's C binding generator emits (reference:
 *     crates/lyth/src/bind_c.rs:39-395; worked example crates/lyth/tests/generated/saxpy.h:17-38).
 *     `lyth_<k>_load` hands out the precompiled sm_100a kernel instead of JIT-loading PTX;
 *     `lyth_<k>_launch` / `_launch_with` launch it with cuLaunchKernel on stream 0, as the
 *     generated bodies do (bind_c.rs:345-395). LYTH never owns memory (ADR-0016 rule 1):
 *     every buffer is the caller's device pointer.
 *
 *  2. The B200 surface `lyth_b200_*` / `lyth_sv_*`: the same kernels with 64-bit sizes and an
 *     explicit stream, the kernel classes the reference only costs (INT4/NF4 GEMV, bf16
 *     tensor-core contraction), and the sharded state vector (no reference counterpart: the
 *     reference has no multi-GPU code). Status: 0 = ok, > 0 = a cudaError_t passed through,
 *     < 0 = a LYTH refusal (below).
 *
 * Nothing here allocates except lyth_sv_create (the state vector it owns) and the one-time
 * module set-up inside the CUDA runtime. There is no CPU fallback: without a device every
 * launch returns the CUDA error.
 */
#ifndef LYTH_B200_H
#define LYTH_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------ */
/* Status codes of the B200 surface. CUDA errors pass through as their positive value.   */
#define LYTH_OK 0
/* A split launch refused: a width of 0, or 2*width not dividing the level's length
 * (crates/lyth-lang/src/ir.rs:164-184, split_pairs ir.rs:202-261). Nothing ran. */
#define LYTH_E_SPLIT (-1)
/* A shape or parameter the kernel class does not take (mirrors EmitError, lyth-ptx/src/lib.rs:48-62). */
#define LYTH_E_UNSUPPORTED (-2)
/* A null pointer, an extent of zero where one is needed, or a size past a 32-bit index. */
#define LYTH_E_INVALID (-3)
/* A bounded device-side wait ran out; the kernel returned without finishing. */
#define LYTH_E_TIMEOUT (-4)
/* NCCL reported an error (or a peer failed) during a state-vector exchange. */
#define LYTH_E_NCCL (-5)
/* The NCCL library could not be loaded for a multi-rank state vector. */
#define LYTH_E_NO_NCCL (-6)
/* A state-vector allocation failed. */
#define LYTH_E_OOM (-7)

/* A human-readable name for any status above (LYTH or CUDA). Never NULL. */
const char *lyth_b200_error_string(int status);
/* ABI version of this header: major * 10000 + minor * 100 + patch. */
int lyth_b200_version(void);

/* ==================================================================================== */
/* 1. ADR-0016 surface (bind_c.rs). `MACHINE` names the image this library carries.        */
/* ==================================================================================== */

/* ---- saxpy: examples/saxpy.lyth, y = a*x + y -> fma(a, x, y) ------------------------- */
#define LYTH_SAXPY_KERNEL "saxpy"
#define LYTH_SAXPY_MACHINE "sm_100a"
#define LYTH_SAXPY_BLOCK 256u
#define LYTH_SAXPY_SHARED_BYTES 0u
#define LYTH_SAXPY_MAX_GRID 1048576u
#define LYTH_SAXPY_DERIVED_INTENSITY 0.16666666666666666
#define LYTH_SAXPY_FLOPS_PER_ELEMENT 2.0
#define LYTH_SAXPY_BYTES_PER_ELEMENT 12.0
#define LYTH_SAXPY_COALESCENCE 1.0
unsigned int lyth_saxpy_elements(unsigned int n);
unsigned int lyth_saxpy_grid(unsigned int n);
/* The kernel writes: y. */
CUresult lyth_saxpy_load(CUmodule *module, CUfunction *fn);
CUresult lyth_saxpy_launch(CUfunction fn, unsigned int n, float a, CUdeviceptr x, CUdeviceptr y);
CUresult lyth_saxpy_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float a, CUdeviceptr x, CUdeviceptr y);

/* ---- axpby: examples/axpby.lyth, y = a*x + b*y -> fma(a, x, mul(b, y)) --------------- */
#define LYTH_AXPBY_KERNEL "axpby"
#define LYTH_AXPBY_MACHINE "sm_100a"
#define LYTH_AXPBY_BLOCK 256u
#define LYTH_AXPBY_SHARED_BYTES 0u
#define LYTH_AXPBY_MAX_GRID 1048576u
#define LYTH_AXPBY_DERIVED_INTENSITY 0.25
#define LYTH_AXPBY_FLOPS_PER_ELEMENT 3.0
#define LYTH_AXPBY_BYTES_PER_ELEMENT 12.0
#define LYTH_AXPBY_COALESCENCE 1.0
unsigned int lyth_axpby_elements(unsigned int n);
unsigned int lyth_axpby_grid(unsigned int n);
/* The kernel writes: y. */
CUresult lyth_axpby_load(CUmodule *module, CUfunction *fn);
CUresult lyth_axpby_launch(CUfunction fn, unsigned int n, float a, float b, CUdeviceptr x, CUdeviceptr y);
CUresult lyth_axpby_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float a, float b, CUdeviceptr x, CUdeviceptr y);

/* ---- lerp: examples/lerp.lyth, z = x + t*(y - x) -> fma(t, sub(y, x), x) ------------- */
#define LYTH_LERP_KERNEL "lerp"
#define LYTH_LERP_MACHINE "sm_100a"
#define LYTH_LERP_BLOCK 256u
#define LYTH_LERP_SHARED_BYTES 0u
#define LYTH_LERP_MAX_GRID 1048576u
#define LYTH_LERP_DERIVED_INTENSITY 0.25
#define LYTH_LERP_FLOPS_PER_ELEMENT 3.0
#define LYTH_LERP_BYTES_PER_ELEMENT 12.0
#define LYTH_LERP_COALESCENCE 1.0
unsigned int lyth_lerp_elements(unsigned int n);
unsigned int lyth_lerp_grid(unsigned int n);
/* The kernel writes: z. */
CUresult lyth_lerp_load(CUmodule *module, CUfunction *fn);
CUresult lyth_lerp_launch(CUfunction fn, unsigned int n, float t, CUdeviceptr x, CUdeviceptr y, CUdeviceptr z);
CUresult lyth_lerp_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float t, CUdeviceptr x, CUdeviceptr y, CUdeviceptr z);

/* ---- horner: examples/horner.lyth, y = fma(fma(fma(c3, x, c2), x, c1), x, c0) -------- */
#define LYTH_HORNER_KERNEL "horner"
#define LYTH_HORNER_MACHINE "sm_100a"
#define LYTH_HORNER_BLOCK 256u
#define LYTH_HORNER_SHARED_BYTES 0u
#define LYTH_HORNER_MAX_GRID 1048576u
#define LYTH_HORNER_DERIVED_INTENSITY 0.75
#define LYTH_HORNER_FLOPS_PER_ELEMENT 6.0
#define LYTH_HORNER_BYTES_PER_ELEMENT 8.0
#define LYTH_HORNER_COALESCENCE 1.0
unsigned int lyth_horner_elements(unsigned int n);
unsigned int lyth_horner_grid(unsigned int n);
/* The kernel writes: y. */
CUresult lyth_horner_load(CUmodule *module, CUfunction *fn);
CUresult lyth_horner_launch(CUfunction fn, unsigned int n, float c0, float c1, float c2, float c3, CUdeviceptr x, CUdeviceptr y);
CUresult lyth_horner_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float c0, float c1, float c2, float c3, CUdeviceptr x, CUdeviceptr y);

/* ---- copy2d: examples/copy2d.lyth, b[i, j] = a[i, j] (the coalesced control) --------- */
#define LYTH_COPY2D_KERNEL "copy2d"
#define LYTH_COPY2D_MACHINE "sm_100a"
#define LYTH_COPY2D_BLOCK 256u
#define LYTH_COPY2D_SHARED_BYTES 0u
#define LYTH_COPY2D_MAX_GRID 1048576u
#define LYTH_COPY2D_DERIVED_INTENSITY 0.0
#define LYTH_COPY2D_FLOPS_PER_ELEMENT 0.0
#define LYTH_COPY2D_BYTES_PER_ELEMENT 8.0
#define LYTH_COPY2D_COALESCENCE 1.0
unsigned int lyth_copy2d_elements(unsigned int rows, unsigned int cols);
unsigned int lyth_copy2d_grid(unsigned int rows, unsigned int cols);
/* The kernel writes: b. */
CUresult lyth_copy2d_load(CUmodule *module, CUfunction *fn);
CUresult lyth_copy2d_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);
CUresult lyth_copy2d_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);

/* ---- transpose: examples/transpose.lyth, b[j, i] = a[i, j], untiled (the strided control) */
#define LYTH_TRANSPOSE_KERNEL "transpose"
#define LYTH_TRANSPOSE_MACHINE "sm_100a"
#define LYTH_TRANSPOSE_BLOCK 256u
#define LYTH_TRANSPOSE_SHARED_BYTES 0u
#define LYTH_TRANSPOSE_MAX_GRID 1048576u
#define LYTH_TRANSPOSE_DERIVED_INTENSITY 0.0
#define LYTH_TRANSPOSE_FLOPS_PER_ELEMENT 0.0
#define LYTH_TRANSPOSE_BYTES_PER_ELEMENT 8.0
#define LYTH_TRANSPOSE_COALESCENCE 0.2222222222222222
unsigned int lyth_transpose_elements(unsigned int rows, unsigned int cols);
unsigned int lyth_transpose_grid(unsigned int rows, unsigned int cols);
/* The kernel writes: b. */
CUresult lyth_transpose_load(CUmodule *module, CUfunction *fn);
CUresult lyth_transpose_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);
CUresult lyth_transpose_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);

/* ---- transpose_tiled: examples/transpose-tiled.lyth, the same body staged through a
 * bank-skewed shared tile. The reference's tile is 32x32 with stride 33 (ir.rs:2056-2062,
 * block 1024, 4224 B); this image keeps the derived rule (stride = the tile width padded to be
 * coprime with 32 banks) at a 64x64 tile, stride 65, 256 threads, 16640 B. One block per
 * tile, as the Tiled grid rule says (manifest.rs:176-181). */
#define LYTH_TRANSPOSE_TILED_KERNEL "transpose_tiled"
#define LYTH_TRANSPOSE_TILED_MACHINE "sm_100a"
#define LYTH_TRANSPOSE_TILED_TILE 64u
#define LYTH_TRANSPOSE_TILED_SKEWED_STRIDE 65u
#define LYTH_TRANSPOSE_TILED_BLOCK 256u
#define LYTH_TRANSPOSE_TILED_SHARED_BYTES 16640u
#define LYTH_TRANSPOSE_TILED_MAX_GRID 2147483647u
#define LYTH_TRANSPOSE_TILED_DERIVED_INTENSITY 0.0
#define LYTH_TRANSPOSE_TILED_FLOPS_PER_ELEMENT 0.0
#define LYTH_TRANSPOSE_TILED_BYTES_PER_ELEMENT 8.0
#define LYTH_TRANSPOSE_TILED_COALESCENCE 1.0
unsigned int lyth_transpose_tiled_elements(unsigned int rows, unsigned int cols);
unsigned int lyth_transpose_tiled_grid(unsigned int rows, unsigned int cols);
/* The kernel writes: b. */
CUresult lyth_transpose_tiled_load(CUmodule *module, CUfunction *fn);
CUresult lyth_transpose_tiled_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);
CUresult lyth_transpose_tiled_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b);

/* ---- reductions: examples/{sum,dot,max,min}.lyth. One partial per block, bit for bit the
 * reference's two-stage order (eval.rs:326-345): thread t of block b folds elements
 * b*256+t, +grid*256, ... in sequence, then the block's 256 slots go through the
 * stride-halving tree (tree_reduce, eval.rs:537-546). Grid = ceil(n / (256*8)), capped
 * (manifest.rs:186-192). The caller combines the partials. */
#define LYTH_SUM_KERNEL "sum"
#define LYTH_SUM_MACHINE "sm_100a"
#define LYTH_SUM_BLOCK 256u
#define LYTH_SUM_SHARED_BYTES 1024u
#define LYTH_SUM_MAX_GRID 1048576u
#define LYTH_SUM_DERIVED_INTENSITY 0.25
#define LYTH_SUM_FLOPS_PER_ELEMENT 1.0
#define LYTH_SUM_BYTES_PER_ELEMENT 4.0
#define LYTH_SUM_COALESCENCE 1.0
unsigned int lyth_sum_elements(unsigned int n);
unsigned int lyth_sum_grid(unsigned int n);
/* Elements `partial` must hold: one per block, NOT one per element. */
unsigned int lyth_sum_partial_len(unsigned int n);
/* The kernel writes: partial. */
CUresult lyth_sum_load(CUmodule *module, CUfunction *fn);
CUresult lyth_sum_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial);
CUresult lyth_sum_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial);

#define LYTH_DOT_KERNEL "dot"
#define LYTH_DOT_MACHINE "sm_100a"
#define LYTH_DOT_BLOCK 256u
#define LYTH_DOT_SHARED_BYTES 1024u
#define LYTH_DOT_MAX_GRID 1048576u
#define LYTH_DOT_DERIVED_INTENSITY 0.25
#define LYTH_DOT_FLOPS_PER_ELEMENT 2.0
#define LYTH_DOT_BYTES_PER_ELEMENT 8.0
#define LYTH_DOT_COALESCENCE 1.0
unsigned int lyth_dot_elements(unsigned int n);
unsigned int lyth_dot_grid(unsigned int n);
unsigned int lyth_dot_partial_len(unsigned int n);
/* The kernel writes: partial. */
CUresult lyth_dot_load(CUmodule *module, CUfunction *fn);
CUresult lyth_dot_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr y, CUdeviceptr partial);
CUresult lyth_dot_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr y, CUdeviceptr partial);

#define LYTH_MAX_OF_KERNEL "max_of"
#define LYTH_MAX_OF_MACHINE "sm_100a"
#define LYTH_MAX_OF_BLOCK 256u
#define LYTH_MAX_OF_SHARED_BYTES 1024u
#define LYTH_MAX_OF_MAX_GRID 1048576u
#define LYTH_MAX_OF_DERIVED_INTENSITY 0.0
#define LYTH_MAX_OF_FLOPS_PER_ELEMENT 0.0
#define LYTH_MAX_OF_BYTES_PER_ELEMENT 4.0
#define LYTH_MAX_OF_COALESCENCE 1.0
unsigned int lyth_max_of_elements(unsigned int n);
unsigned int lyth_max_of_grid(unsigned int n);
unsigned int lyth_max_of_partial_len(unsigned int n);
/* The kernel writes: partial. */
CUresult lyth_max_of_load(CUmodule *module, CUfunction *fn);
CUresult lyth_max_of_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial);
CUresult lyth_max_of_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial);

#define LYTH_MIN_OF_KERNEL "min_of"
#define LYTH_MIN_OF_MACHINE "sm_100a"
#define LYTH_MIN_OF_BLOCK 256u
#define LYTH_MIN_OF_SHARED_BYTES 1024u
#define LYTH_MIN_OF_MAX_GRID 1048576u
#define LYTH_MIN_OF_DERIVED_INTENSITY 0.0
#define LYTH_MIN_OF_FLOPS_PER_ELEMENT 0.0
#define LYTH_MIN_OF_BYTES_PER_ELEMENT 4.0
#define LYTH_MIN_OF_COALESCENCE 1.0
unsigned int lyth_min_of_elements(unsigned int n);
unsigned int lyth_min_of_grid(unsigned int n);
unsigned int lyth_min_of_partial_len(unsigned int n);
/* The kernel writes: partial. */
CUresult lyth_min_of_load(CUmodule *module, CUfunction *fn);
CUresult lyth_min_of_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial);
CUresult lyth_min_of_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial);

/* ---- matmul: examples/matmul.lyth, C[i, j] = sum_p A[i, p] * B[p, j]. The ADR-0016 entry
 * keeps the reference's contract bit for bit: p ascending, mul.rn then add.rn, accumulator
 * from 0.0 (contracted.rs:23-26, eval.rs:459-508). Traffic is an expression in k (the
 * symbolic cost, bind_c.rs:150-185), here at the 128x128 tile this image stages. */
#define LYTH_MATMUL_KERNEL "matmul"
#define LYTH_MATMUL_MACHINE "sm_100a"
#define LYTH_MATMUL_TILE 128u
#define LYTH_MATMUL_BLOCK 256u
#define LYTH_MATMUL_SHARED_BYTES 32768u
#define LYTH_MATMUL_MAX_GRID 2147483647u
#define LYTH_MATMUL_COALESCENCE 1.0
static inline double lyth_matmul_derived_bytes_per_element(unsigned int k)
{
    return 0.0625 * (double)k + 4.0;
}
static inline double lyth_matmul_derived_flops_per_element(unsigned int k)
{
    return 2.0 * (double)k + 0.0;
}
static inline double lyth_matmul_derived_intensity(unsigned int k)
{
    return lyth_matmul_derived_flops_per_element(k) / lyth_matmul_derived_bytes_per_element(k);
}
unsigned int lyth_matmul_elements(unsigned int m, unsigned int n);
unsigned int lyth_matmul_grid(unsigned int m, unsigned int n);
/* The kernel writes: c. */
CUresult lyth_matmul_load(CUmodule *module, CUfunction *fn);
CUresult lyth_matmul_launch(CUfunction fn, unsigned int m, unsigned int n, unsigned int k, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c);
CUresult lyth_matmul_launch_with(CUfunction fn, unsigned int grid, unsigned int m, unsigned int n, unsigned int k, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c);

/* ---- state-vector gates. The reference's C generator refuses split kernels
 * (crates/lyth/src/main.rs:897-905); the Rust binding carries check_splits
 * (bind_rust.rs:298-360). This ABI gives C the same: `_check_splits` returns LYTH_OK or
 * LYTH_E_SPLIT, and `_launch` / `_launch_with` refuse (CUDA_ERROR_INVALID_VALUE) before
 * anything runs. n is the amplitude count; the walk is n/2 pairs (depth 1) or n/4 quads
 * (depth 2). Output buffers may alias the inputs (an in-place pass). */

/* hadamard_q: examples/hadamard_q.lyth, q0 = s*(p0 + p1), q1 = s*(p0 - p1). */
#define LYTH_HADAMARD_Q_KERNEL "hadamard_q"
#define LYTH_HADAMARD_Q_MACHINE "sm_100a"
#define LYTH_HADAMARD_Q_BLOCK 256u
#define LYTH_HADAMARD_Q_SHARED_BYTES 0u
#define LYTH_HADAMARD_Q_MAX_GRID 1048576u
#define LYTH_HADAMARD_Q_DERIVED_INTENSITY 0.25
#define LYTH_HADAMARD_Q_FLOPS_PER_ELEMENT 8.0
#define LYTH_HADAMARD_Q_BYTES_PER_ELEMENT 32.0
#define LYTH_HADAMARD_Q_COALESCENCE 1.0
unsigned int lyth_hadamard_q_elements(unsigned int n);
unsigned int lyth_hadamard_q_grid(unsigned int n);
int lyth_hadamard_q_check_splits(unsigned int n, unsigned int w);
/* The kernel writes: qr, qi. */
CUresult lyth_hadamard_q_load(CUmodule *module, CUfunction *fn);
CUresult lyth_hadamard_q_launch(CUfunction fn, unsigned int n, unsigned int w, float s, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);
CUresult lyth_hadamard_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int w, float s, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);

/* gate_q: examples/gate_q.lyth, any 1-qubit U = [[a, b], [c, d]] in four fixed fma chains. */
#define LYTH_GATE_Q_KERNEL "gate_q"
#define LYTH_GATE_Q_MACHINE "sm_100a"
#define LYTH_GATE_Q_BLOCK 256u
#define LYTH_GATE_Q_SHARED_BYTES 0u
#define LYTH_GATE_Q_MAX_GRID 1048576u
#define LYTH_GATE_Q_DERIVED_INTENSITY 0.875
#define LYTH_GATE_Q_FLOPS_PER_ELEMENT 28.0
#define LYTH_GATE_Q_BYTES_PER_ELEMENT 32.0
#define LYTH_GATE_Q_COALESCENCE 1.0
unsigned int lyth_gate_q_elements(unsigned int n);
unsigned int lyth_gate_q_grid(unsigned int n);
int lyth_gate_q_check_splits(unsigned int n, unsigned int w);
/* The kernel writes: qr, qi. */
CUresult lyth_gate_q_load(CUmodule *module, CUfunction *fn);
CUresult lyth_gate_q_launch(CUfunction fn, unsigned int n, unsigned int w, float ar, float ai, float br, float bi, float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);
CUresult lyth_gate_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int w, float ar, float ai, float br, float bi, float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);

/* cu_q: examples/cu_q.lyth, controlled U on (c, t) with widths (wc, wt) as
 * lyth-circuit widths_ct gives them (lib.rs:387-389); the control=0 half is copied.
 * cu_q_grouped (examples/cu_q_grouped.lyth) is the same kernel: its only difference in the
 * reference is the order of the stores, which this image chooses itself. */
#define LYTH_CU_Q_KERNEL "cu_q"
#define LYTH_CU_Q_MACHINE "sm_100a"
#define LYTH_CU_Q_BLOCK 256u
#define LYTH_CU_Q_SHARED_BYTES 0u
#define LYTH_CU_Q_MAX_GRID 1048576u
#define LYTH_CU_Q_DERIVED_INTENSITY 0.4375
#define LYTH_CU_Q_FLOPS_PER_ELEMENT 28.0
#define LYTH_CU_Q_BYTES_PER_ELEMENT 64.0
#define LYTH_CU_Q_COALESCENCE 1.0
unsigned int lyth_cu_q_elements(unsigned int n);
unsigned int lyth_cu_q_grid(unsigned int n);
int lyth_cu_q_check_splits(unsigned int n, unsigned int wc, unsigned int wt);
/* The kernel writes: qr, qi. */
CUresult lyth_cu_q_load(CUmodule *module, CUfunction *fn);
CUresult lyth_cu_q_launch(CUfunction fn, unsigned int n, unsigned int wc, unsigned int wt, float ar, float ai, float br, float bi, float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);
CUresult lyth_cu_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int wc, unsigned int wt, float ar, float ai, float br, float bi, float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);

/* swap_q: examples/swap_q.lyth, |01> <-> |10>, |00> and |11> copied; no arithmetic. */
#define LYTH_SWAP_Q_KERNEL "swap_q"
#define LYTH_SWAP_Q_MACHINE "sm_100a"
#define LYTH_SWAP_Q_BLOCK 256u
#define LYTH_SWAP_Q_SHARED_BYTES 0u
#define LYTH_SWAP_Q_MAX_GRID 1048576u
#define LYTH_SWAP_Q_DERIVED_INTENSITY 0.0
#define LYTH_SWAP_Q_FLOPS_PER_ELEMENT 0.0
#define LYTH_SWAP_Q_BYTES_PER_ELEMENT 64.0
#define LYTH_SWAP_Q_COALESCENCE 1.0
unsigned int lyth_swap_q_elements(unsigned int n);
unsigned int lyth_swap_q_grid(unsigned int n);
int lyth_swap_q_check_splits(unsigned int n, unsigned int wc, unsigned int wt);
/* The kernel writes: qr, qi. */
CUresult lyth_swap_q_load(CUmodule *module, CUfunction *fn);
CUresult lyth_swap_q_launch(CUfunction fn, unsigned int n, unsigned int wc, unsigned int wt, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);
CUresult lyth_swap_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int wc, unsigned int wt, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi);

/* ==================================================================================== */
/* 2. B200 surface: 64-bit sizes, explicit streams.                                        */
/* ==================================================================================== */

/* Streams (replaces the launch of lyth run, crates/lyth/src/main.rs:1320-1499, for these
 * bodies). x/y/z may be any alignment; 16-byte aligned buffers take the 128-bit path. */
int lyth_b200_saxpy(uint64_t n, float a, const float *x, float *y, cudaStream_t stream);
int lyth_b200_axpby(uint64_t n, float a, float b, const float *x, float *y, cudaStream_t stream);
int lyth_b200_lerp(uint64_t n, float t, const float *x, const float *y, float *z, cudaStream_t stream);
int lyth_b200_horner(uint64_t n, float c0, float c1, float c2, float c3, const float *x, float *y,
                     cudaStream_t stream);

/* Rank-2 walks of examples/{copy2d,transpose,transpose-tiled}.lyth. a is rows x cols row-major;
 * b is rows x cols (copy2d) or cols x rows (transposes). */
int lyth_b200_copy2d(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t stream);
int lyth_b200_transpose_naive(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t stream);
int lyth_b200_transpose_tiled(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t stream);

/* Reductions. op: 0 = sum, 1 = max, 2 = min (ast.rs ReduceOp); y != NULL makes it dot (sum
 * of x*y, mul.rn then add.rn). */
#define LYTH_REDUCE_SUM 0
#define LYTH_REDUCE_MAX 1
#define LYTH_REDUCE_MIN 2
/* The reference's default grid for a reduction over n: ceil(n / 2048), in [1, 2^20]. */
uint32_t lyth_b200_reduce_grid(uint64_t n);
/* One partial per block, bit-exact to the reference's order for this (grid, 256). */
int lyth_b200_reduce_partials(int op, uint64_t n, const float *x, const float *y, uint32_t grid,
                              float *partial, cudaStream_t stream);
/* The whole reduction to one f32 in `out` (device memory): the same per-block partials
 * (grid = lyth_b200_reduce_grid(n)), combined across each thread-block cluster through
 * distributed shared memory, then across clusters. `workspace` is caller-owned device
 * memory of lyth_b200_reduce_workspace_bytes(n) bytes (ADR-0016: LYTH never owns memory). */
size_t lyth_b200_reduce_workspace_bytes(uint64_t n);
int lyth_b200_reduce(int op, uint64_t n, const float *x, const float *y, float *out, void *workspace,
                     size_t workspace_bytes, cudaStream_t stream);
/* The same whole reduction for callers that cannot provide device memory -- a host whose device
 * memory all belongs to its own arena, a runtime that embeds these kernels and does not let them
 * allocate, a loop that cannot take the synchronisation of cudaMalloc. It has no counterpart in
 * the reference. It allocates nothing: the cluster results go to a fixed 64 KiB array in the
 * library's own device memory, which every GPU that loads the library keeps until the process
 * exits, so n is limited to LYTH_REDUCE_NOALLOC_MAX_N elements (larger n: LYTH_E_UNSUPPORTED,
 * nothing runs). The first call on a device looks the array's address up; make it before any
 * stream capture. All calls share the array: each writes every slot it reads, so no clearing is
 * needed, but calls that overlap on the GPU race. Result: bit for bit lyth_b200_reduce's. */
#define LYTH_REDUCE_NOALLOC_MAX_N 268435456ull
int lyth_b200_reduce_noalloc(int op, uint64_t n, const float *x, const float *y, float *out,
                             cudaStream_t stream);

/* Contraction C = A * B, row-major, A m x k, B k x n, C m x n (examples/matmul.lyth).
 * exact = 1: the reference's order bit for bit (p ascending, mul.rn then add.rn).
 * exact = 0: FFMA register-tiled (p ascending, fused), within 1e-5 relative of the reference. */
int lyth_b200_matmul_f32(uint32_t m, uint32_t n, uint32_t k, const float *a, const float *b, float *c,
                         int exact, cudaStream_t stream);
/* bf16 inputs (raw bfloat16 bits), f32 accumulate and output, on the tcgen05 tensor cores with
 * TMEM accumulators. m a multiple of 128, n of 256 and k of 64 (16-byte aligned buffers) take the
 * tensor-core path; other shapes return LYTH_E_UNSUPPORTED. m a multiple of 256 runs on CTA pairs
 * (tcgen05.mma.cta_group::2, 256 x 256 tiles, each SM staging half of each operand), other m on
 * single SMs (128 x 256 tiles). No reference kernel: the reference never uses tensor cores.
 * Compared with eval_contraction on the bf16-rounded inputs within 1e-2 relative. */
int lyth_b200_matmul_bf16(uint32_t m, uint32_t n, uint32_t k, const uint16_t *a, const uint16_t *b,
                          float *c, cudaStream_t stream);
/* The same with the form chosen: pair = 1 the CTA-pair kernel (m a multiple of 256, else
 * LYTH_E_UNSUPPORTED), pair = 0 the single-SM kernel. For tests and measurements of both. */
int lyth_b200_matmul_bf16_form(int pair, uint32_t m, uint32_t n, uint32_t k, const uint16_t *a,
                               const uint16_t *b, float *c, cudaStream_t stream);
/* CTA pairs the pair form runs on the current device (clusters of 2 resident at once), or a
 * negative status. */
int lyth_b200_matmul_bf16_pairs(void);
/* LYTH_E_TIMEOUT when a bounded device-side wait of any kernel in this library ran out since the
 * last call (the flag is then cleared), else LYTH_OK. Synchronises with the current device. */
int lyth_b200_device_error(void);
/* Bounded-wait self-test (no counterpart in the reference, which has no device-side waits): one
 * thread waits on something that never completes -- which = 0: an mbarrier phase, the wait of the
 * TMA-fed kernels; which = 1: a device flag, the wait of the multi-GPU transport -- through the
 * same wait functions, with a limit of limit_us microseconds (1 .. 2,000,000) instead of 2 s. The
 * wait gives up and the kernel returns; lyth_b200_device_error then reports LYTH_E_TIMEOUT once.
 * LYTH_E_INVALID for another `which` or limit. */
int lyth_b200_wait_selftest(int which, uint32_t limit_us, cudaStream_t stream);

/* gate_proj GEMV (fixtures/kernel/gate_proj_int4.json, fixtures/poly/gate-proj-int4-nf4.json:
 * cost contracts only; the reference has no kernel). y[r] = sum_k dequant(W)[r, k] * x[k].
 * W: rows x k 4-bit, row r contiguous along k, byte (r*k + c)/2, low nibble = even c.
 * fmt 0 = INT4 (two's-complement nibble, -8..7, w = q * scale, exact in f32);
 * fmt 1 = NF4 (nibble indexes lyth_b200_nf4_codebook, w = code * scale, one rounding).
 * scales: fp16 bits [rows][k / group]; x: fp16 bits [k]; y: fp16 bits [rows] (f32 accumulate,
 * rounded once, RNE). k a multiple of 64; group a multiple of 32 dividing k. */
#define LYTH_GEMV_INT4 0
#define LYTH_GEMV_NF4 1
int lyth_b200_gemv_q4(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                      const uint16_t *scales, const uint16_t *x, uint16_t *y, cudaStream_t stream);
/* The dequantised matrix (rows x k f32, 16-byte aligned; k and group multiples of 8), decoded
 * by the same device function the GEMV's kernels decode W with (decode_word, k_gemv.cu): INT4
 * q * scale, exact; NF4 code * scale, one rounding. Bit-exact against the format's definition. */
int lyth_b200_gemv_dequant(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                           const uint16_t *scales, float *out, cudaStream_t stream);
/* The 16 NF4 levels (QLoRA's normal-float construction, computed on the host at load). */
void lyth_b200_nf4_codebook(float out[16]);

/* State-vector gates on the caller's buffers (examples/{hadamard_q,gate_q,cu_q,swap_q}.lyth),
 * 64-bit: n amplitudes, split re/im f32. m = ar ai br bi cr ci dr di (lyth-circuit f32s,
 * lib.rs:49-56) as a host array. qr/qi may alias re/im. Power-of-two widths take the fast
 * kernels; any other width that divides takes the general view_index path. */
int lyth_b200_hadamard(uint64_t n, uint64_t w, float s, const float *re, const float *im, float *qr,
                       float *qi, cudaStream_t stream);
int lyth_b200_gate(uint64_t n, uint64_t w, const float *m, const float *re, const float *im, float *qr,
                   float *qi, cudaStream_t stream);
int lyth_b200_cu(uint64_t n, uint64_t wc, uint64_t wt, const float *m, const float *re, const float *im,
                 float *qr, float *qi, cudaStream_t stream);
int lyth_b200_swap(uint64_t n, uint64_t wc, uint64_t wt, const float *re, const float *im, float *qr,
                   float *qi, cudaStream_t stream);

/* ---- narrow storage (f16 / bf16 buffers, f32 arithmetic: crates/lyth-ptx/src/lib.rs:607-732,
 * docs/ADR-0024-half-the-element.md). Each element is widened exactly on load, the body is the f32
 * kernel's chain, and each drained value is rounded once, to nearest even, at the store
 * (eval.rs:557-570 round_narrow_outputs). Buffers hold the 16-bit patterns. */
#define LYTH_NARROW_F16 1
#define LYTH_NARROW_BF16 2
#define LYTH_STREAM_SAXPY 0   /* out = fma(a, x, y); scalars {a}; out may be y */
#define LYTH_STREAM_AXPBY 1   /* out = fma(a, x, b * y); scalars {a, b} */
#define LYTH_STREAM_LERP 2    /* out = fma(t, y - x, x); scalars {t} */
#define LYTH_STREAM_HORNER 3  /* out = ((c3 x + c2) x + c1) x + c0 as three fmas; scalars {c0, c1, c2, c3} */
#define LYTH_STREAM_COPY 4    /* out = x (examples/copy2d.lyth at 2 bytes an element) */
int lyth_b200_stream_narrow(int op, int ty, uint64_t n, const float *scalars, const uint16_t *x, const uint16_t *y,
                            uint16_t *out, cudaStream_t stream);
/* b[j, i] = a[i, j] for 2-byte elements (examples/transpose-tiled.lyth at f16 / bf16 storage). */
int lyth_b200_transpose_narrow(int ty, uint32_t rows, uint32_t cols, const uint16_t *a, uint16_t *b,
                               cudaStream_t stream);
/* One f32 partial per block from f16 / bf16 inputs, in lyth_b200_reduce_partials's order. */
int lyth_b200_reduce_partials_narrow(int op, int ty, uint64_t n, const uint16_t *x, const uint16_t *y, uint32_t grid,
                                     float *partial, cudaStream_t stream);

/* ---- the back-end entry: a lowered kernel in, a kernel of this library (or a refusal) out.
 * Replaces lyth_ptx::emit(&KernelIr, arch) -> Module (crates/lyth-ptx/src/lib.rs:65-253; refusals
 * EmitError, :48-62) and Function::launch_shared with Arg slots in declaration order
 * (crates/lyth-cuda/src/lib.rs:483-549). The descriptor is the part of lyth-lang's KernelIr
 * (crates/lyth-lang/src/ir.rs:24-56) a back end reads: parameters in declaration order, the rank-2
 * space, tile, coarsen, contraction, reduction, split views (ir.rs:58-81) and the lowered body
 * (Op, ir.rs:463-503) with the registers each drained buffer takes. Registers are indices into
 * `ops` (op i defines register i). */
#define LYTH_TY_U32 0
#define LYTH_TY_F32 1
#define LYTH_TY_BUF_F32 2
#define LYTH_TY_BUF_F16 3
#define LYTH_TY_BUF_BF16 4
#define LYTH_IR_LOAD 0   /* name = buffer or view; transposed = rank-2 access [j, i] */
#define LYTH_IR_PARAM 1  /* name = scalar parameter */
#define LYTH_IR_CONST 2  /* value */
#define LYTH_IR_BIN 3    /* bin = LYTH_BIN_*, a, b */
#define LYTH_IR_FMA 4    /* a * b + c, one rounding */
#define LYTH_IR_NEG 5    /* a */
#define LYTH_BIN_ADD 0
#define LYTH_BIN_SUB 1
#define LYTH_BIN_MUL 2
#define LYTH_BIN_DIV 3
#define LYTH_BIN_MAX 4
#define LYTH_BIN_MIN 5
typedef struct lyth_ir_param {
    const char *name;
    int32_t ty;                 /* LYTH_TY_* */
} lyth_ir_param;
typedef struct lyth_ir_view {   /* element k of `name` is view_index(width, part, k) of `base` */
    const char *name, *base, *width;
    uint32_t part;
} lyth_ir_view;
typedef struct lyth_ir_op {
    int32_t kind, bin;
    int32_t a, b, c;            /* operand registers */
    double value;
    const char *name;
    uint32_t transposed;
} lyth_ir_op;
typedef struct lyth_ir_drain {
    const char *buffer;         /* a buffer parameter or a view */
    int32_t reg;
    uint32_t transposed;
} lyth_ir_drain;
typedef struct lyth_ir {
    const char *name, *machine;
    uint32_t nparams;
    const lyth_ir_param *params;
    uint32_t rank;              /* 1, or 2 (a `space i, j`) */
    uint32_t tile[2];           /* {0, 0}: no tile */
    uint32_t coarsen[2];        /* {0, 0}: none */
    uint32_t contract;          /* 1: `contract sum p` (a[i, p] * b[p, j] in the body) */
    int32_t reduce_op;          /* -1: none; LYTH_SUM / LYTH_MAX / LYTH_MIN (0, 1, 2) */
    int32_t reduce_reg;
    const char *reduce_into;
    uint32_t reduce_via_smem;   /* the declared path is reg -> smem -> dram */
    uint32_t nviews;
    const lyth_ir_view *views;
    uint32_t nops;
    const lyth_ir_op *ops;
    uint32_t ndrains;
    const lyth_ir_drain *drains;
} lyth_ir;
#define LYTH_CLASS_SAXPY 1
#define LYTH_CLASS_AXPBY 2
#define LYTH_CLASS_LERP 3
#define LYTH_CLASS_HORNER 4
#define LYTH_CLASS_COPY2D 5
#define LYTH_CLASS_TRANSPOSE 6
#define LYTH_CLASS_TRANSPOSE_TILED 7
#define LYTH_CLASS_SUM 8
#define LYTH_CLASS_DOT 9
#define LYTH_CLASS_MAX 10
#define LYTH_CLASS_MIN 11
#define LYTH_CLASS_MATMUL_F32 12
#define LYTH_CLASS_MATMUL_BF16 13
#define LYTH_CLASS_HADAMARD_Q 14
#define LYTH_CLASS_GATE_Q 15
#define LYTH_CLASS_CU_Q 16
#define LYTH_CLASS_SWAP_Q 17
typedef struct lyth_kernel {
    int32_t cls;                /* LYTH_CLASS_*, 0 when refused */
    char entry[48];             /* the class's name */
    uint32_t nparams;           /* the kernel's parameters, declaration order */
    int32_t param_ty[32];
    int32_t slot[16];           /* class argument j <- declaration slot slot[j] */
    uint32_t retargeted;        /* 1: written for another machine the sm_100a file accepts */
    int32_t storage;            /* 0: f32 buffers; LYTH_NARROW_F16 / _BF16: every data buffer 16-bit */
    char message[320];          /* why it was refused (EmitError's text), or a note */
} lyth_kernel;
typedef struct lyth_launch {    /* optional: NULL takes the kernel's own launch shape */
    uint32_t grid;              /* reductions: the number of partials (default lyth_b200_reduce_grid(n)) */
} lyth_launch;
/* 0 and a kernel, or LYTH_E_UNSUPPORTED / LYTH_E_INVALID with out->message: no bound (EmitError
 * NoBound), no drain (NoDrain), an unknown machine (UnknownTarget: sm_100a, sm_100 and the
 * machines fixtures/machine/sm_100a.json accepts, sm_120), a reduction not staged through shared
 * memory, a coarsened tile that does not contract, or a body no kernel of this library computes.
 * Never a fallback: a refusal runs nothing. */
int lyth_b200_select(const lyth_ir *ir, lyth_kernel *out);
/* Launch a selected kernel. args[i] points to declaration slot i's value, as cuLaunchKernel's
 * kernelParams: a uint32_t, a float, or a device pointer (CUdeviceptr) for a buffer. Returns 0,
 * a CUDA error, or a LYTH refusal (split widths, shapes) before anything runs. */
int lyth_b200_launch(const lyth_kernel *k, void *const *args, const lyth_launch *launch, cudaStream_t stream);
/* Device scratch a launch of this kernel with these arguments needs: 0 for every class this
 * library has (reductions write their partials to the caller's `into` buffer). */
size_t lyth_b200_workspace_bytes(const lyth_kernel *k, void *const *args);

/* Host-only self-test of the fused pass's tile layouts (no counterpart in the reference; no device
 * is touched): plans `groups` random gate groups over 14..33 local qubits and checks that the
 * copies into shared memory and the warps' reads agree on every amplitude, that tensor-map boxes
 * tile the index space with aligned origins, that no warp read has a bank conflict, and that each
 * gate lands on its group's bits. LYTH_OK, or a negative code naming the first failed check;
 * `planned` / `boxes` (may be NULL) count the plans and those that copy by tensor-map boxes. */
int lyth_b200_fused_layout_selftest(uint64_t seed, uint32_t groups, uint32_t *planned, uint32_t *boxes);

/* ---- the state vector (lyth-circuit, crates/lyth-circuit/src/lib.rs:327-371, re-designed:
 * in place, a qubit map that makes SWAP a relabel, and sharded over ranks on its high qubits
 * with pairwise NCCL exchange for gates on those qubits). One handle per rank/GPU. ---------- */
typedef struct lyth_sv lyth_sv;

/* A gate as lyth-circuit's Gate enum (lib.rs:29-46): kind 0 = U on q0, 1 = CU control q0 /
 * target q1, 2 = Swap(q0, q1). m = ar ai br bi cr ci dr di (unused for Swap). */
#define LYTH_GATE_U 0
#define LYTH_GATE_CU 1
#define LYTH_GATE_SWAP 2
typedef struct lyth_gate {
    uint32_t kind;
    uint32_t q0;
    uint32_t q1;
    float m[8];
} lyth_gate;

/* Bytes of an NCCL unique id (ncclUniqueId). */
#define LYTH_SV_ID_BYTES 128
/* Fill `id` on one rank (usually 0) and hand it to every rank's lyth_sv_create. */
int lyth_sv_unique_id(unsigned char id[LYTH_SV_ID_BYTES]);
/* A state of 2^qubits amplitudes over `nranks` ranks (a power of two); this rank's shard of
 * 2^(qubits - log2 nranks) amplitudes lives on `device`. nranks = 1 needs no id (NULL). */
int lyth_sv_create(lyth_sv **out, uint32_t qubits, int device, int rank, int nranks,
                   const unsigned char *id);
int lyth_sv_destroy(lyth_sv *sv);
/* This rank's shard length, and the stream every operation of the handle is ordered on. */
uint64_t lyth_sv_local_len(const lyth_sv *sv);
cudaStream_t lyth_sv_stream(const lyth_sv *sv);
/* |index> (lyth-circuit's initial |0...0> is index 0). */
int lyth_sv_init_basis(lyth_sv *sv, uint64_t index);
/* re, im ~ U[-1, 1) from SplitMix64 keyed by the global amplitude index (re: stream output 2i,
 * im: 2i+1), then scaled by 1/sqrt(sum |a|^2) (the sum in f64, applied in f32). */
int lyth_sv_init_random(lyth_sv *sv, uint64_t seed);
/* Copy this rank's shard in/out, in logical qubit order (the qubit map is undone first by
 * real permutation passes). Pointers may be host (pageable or pinned) or device memory. */
int lyth_sv_set_local(lyth_sv *sv, const float *re, const float *im);
int lyth_sv_get_local(lyth_sv *sv, float *re, float *im);
/* Apply `count` gates in order. Returns when the work is queued on lyth_sv_stream. */
int lyth_sv_apply(lyth_sv *sv, const lyth_gate *gates, uint64_t count);
/* Wait for the handle's streams; LYTH_E_TIMEOUT if a pass gave up one of its bounded waits. With
 * an NCCL communicator the wait polls the streams and ncclCommGetAsyncError and gives up at the
 * handle's deadline (lyth_sv_set_deadline): an async error aborts the communicator
 * (ncclCommAbort) and returns LYTH_E_NCCL; the deadline aborts it and returns LYTH_E_TIMEOUT. An
 * aborted handle refuses further collective work with LYTH_E_NCCL; destroy it. */
int lyth_sv_sync(lyth_sv *sv);
/* The host-side deadline of the handle's NCCL waits, in milliseconds (>= 1; default 300000). No
 * counterpart in the reference (no multi-GPU code). */
int lyth_sv_set_deadline(lyth_sv *sv, double ms);
/* Copy-engine queues one swap-in pull is spread over (1..8): each component's slice from each
 * partner is cut into this many pieces, issued round-robin. 0 (the default): every partner's re
 * and im slices get a queue each, up to 8 -- 2 queues for a pairwise swap-in, 6 for a batched one
 * among 4 ranks -- so the pulls from several partners run at once. Collective: every rank, same
 * value. No counterpart in the reference. */
int lyth_sv_set_pull_queues(lyth_sv *sv, int queues);
/* Host-only check of the deadline logic with fake hooks, no device or NCCL (scenario 0: done after
 * 3 polls -> LYTH_OK; 1: async error -> LYTH_E_NCCL, one abort; 2: never done -> LYTH_E_TIMEOUT at
 * the deadline, one abort; 3: a CUDA error from the stream -> that status, no abort). */
int lyth_sv_deadline_selftest(int scenario, double deadline_ms, int *aborts, uint64_t *polls);
/* Counters since creation: data passes run, exchange steps run, bytes sent over NCCL. */
int lyth_sv_stats(const lyth_sv *sv, uint64_t *passes, uint64_t *exchanges, uint64_t *bytes_sent);
/* Kernel launches since creation (every pass, exchange chunk and permutation kernel). */
uint64_t lyth_sv_launches(const lyth_sv *sv);
/* Per-class device timing: when on, every data pass is bracketed by CUDA events on the stream it
 * runs on. Classes: 0 = 1-qubit local pass, 1 = 2-qubit local pass, 2 = exchange gate (first
 * chunk's send to last chunk's compute, on the compute stream). lyth_sv_timing synchronises,
 * folds the recorded pairs into (count, total ms) per class, and keeps the totals. */
#define LYTH_SV_T_U 0
#define LYTH_SV_T_CU 1
#define LYTH_SV_T_EXCHANGE 2
#define LYTH_SV_T_FUSED 3
/* 4 = a rank-bit qubit swapped into a local bit (pack, transfer and unpack of half the shard). */
#define LYTH_SV_T_SWAP 4
/* Fusion (lyth-circuit fuse, lib.rs:72-100; docs/ADR-0030): consecutive local gates touching at
 * most `max_qubits` (1..13) bits run as one pass with the same chains in circuit order, bit-exact
 * with the unfused passes. A group must also fit one pass at the shard's size: states of 2^14
 * amplitudes and more take the tile pass (at most 8 of a group's bits above bit 4), smaller ones
 * the register pass (at most 6 bits). 1 = one pass per gate. The default is 13. */
int lyth_sv_set_fusion(lyth_sv *sv, int max_qubits);
/* A gate on a qubit that currently lives on a rank bit: on = 1 (default) first swaps it with the
 * local qubit used furthest ahead in the gate list (half the shard crosses NVLink each way) and
 * then runs the gate as a local (fusable) pass; on = 0 exchanges the whole shard with the partner
 * rank and computes this rank's row of the gate. Both are bit-exact. */
int lyth_sv_set_remap(lyth_sv *sv, int on);
/* A diagonal gate (off-diagonal entries zero: phases, Z, S, T, controlled phases) whose target
 * lives on a rank bit: on = 1 (default) moves no data -- on a shard whose rank bit is v the gate
 * is the scalar u_vv, applied (under the gate's control where it has one) as the local gate
 * diag(u_vv, u_vv) in the open fused group, and skipped where u_vv = 1. Every amplitude gets the
 * value the full gate gives it; the chains differ only by products with the zero entries, so the
 * sign of an amplitude that is exactly zero may differ from the evaluator's (a non-finite partner
 * would also not turn it into NaN). on = 0 treats it like any other gate (swap-in or exchange)
 * and is bit-identical with the evaluator in every case. Collective: every rank, same value. */
int lyth_sv_set_diagonal(lyth_sv *sv, int on);
/* With remap on: the most rank-bit qubits one swap-in brings in together (1..6, default 6; 1 = one
 * at a time). Extra ones join only while each is needed before the local bit it displaces; k of
 * them cost one exchange of (2^k - 1) / 2^k of the shard among 2^k ranks instead of k half-shard
 * swaps (fewer bytes and fewer passes, though a pull from several partners runs slower per byte
 * than a pairwise one). Bit-exact either way. Collective: every rank, same value. */
int lyth_sv_set_swap_batch(lyth_sv *sv, int max_qubits);
/* Transport of swap-ins on a multi-rank handle: 1 = copy engines (each rank pulls its partners'
 * packed chunks over NVLink with cudaMemcpyAsync through CUDA IPC mappings, ordered by sequence
 * flags), 2 = peer loads (the same mappings and
 * flags; the SMs read the partners' packed chunks and store them straight into the shard, the
 * unpack fused into the pull), 3 = mixed (copy engines for a pairwise swap-in, peer loads for a
 * batched one with several partners; the default when every rank could map every peer),
 * 4 = peer stores (the SMs store this rank's packed chunks straight into the partners' shards,
 * once each partner has packed the positions they go to), 0 = NCCL send / recv. 1-4 need the IPC
 * mappings (LYTH_E_UNSUPPORTED without them); other values LYTH_E_INVALID. Collective: every rank
 * sets the same value at the same point. lyth_sv_transport reports the one in use (0-4). */
int lyth_sv_set_transport(lyth_sv *sv, int kind);
/* The exchanges' pipeline chunk in amplitudes per component (a power of two from 1024 up to the
 * allocated 2^28, or the shard if smaller; the default is the largest). Collective. Smaller
 * chunks cut every exchange into more pipelined pieces (used by the tests to drive many). */
int lyth_sv_set_chunk(lyth_sv *sv, uint64_t elements);
int lyth_sv_transport(const lyth_sv *sv);
int lyth_sv_set_timing(lyth_sv *sv, int on);
int lyth_sv_timing(lyth_sv *sv, int cls, uint64_t *count, double *ms);
int lyth_sv_reset_timing(lyth_sv *sv);

/* ---- plan recording (no counterpart in the reference; the host-side check of the sharded
 * engine). A plan handle runs the same planner as lyth_sv_create's handle -- fusion, qubit map,
 * swap-in victims, exchanges -- but holds no device memory, makes no CUDA or NCCL call, and
 * appends each step it would run to a list instead. lyth_sv_apply, lyth_sv_set_fusion,
 * lyth_sv_set_remap and lyth_sv_stats work on it; set_local / init_* only reset the qubit map;
 * lyth_sv_get_local records the permutation steps that undo the map and copies nothing (re and
 * im may be NULL). Replaying the steps on every rank's shard gives the engine's result. */
#define LYTH_SV_FUSE_MAX_QUBITS 13
#define LYTH_SV_FUSE_MAX_GATES 48
#define LYTH_SV_OP_U 0           /* U on local bit a */
#define LYTH_SV_OP_CU 1          /* CU, control local bit a, target local bit b */
#define LYTH_SV_OP_FUSED 2       /* gates[0..ngates) in order on levels of bits[0..k) */
#define LYTH_SV_OP_EXCHANGE 3    /* gate on rank bit a with the partner rank ^ (1 << a); control
                                    local bit c (or -1); this rank keeps its row */
#define LYTH_SV_OP_SWAP_LOCAL 4  /* swap local bits a, b */
#define LYTH_SV_OP_SWAP_LR 5     /* swap local bit a with rank bit b (half the shard each way) */
#define LYTH_SV_OP_SWAP_RR 6     /* swap rank bits a, b (whole shards, where the bits differ) */
#define LYTH_SV_OP_SWAP_MULTI 7  /* swap local bits bits[j] with rank bits rbits[j], j < k (k >= 2):
                                    one exchange among the 2^k ranks differing in those bits */
#define LYTH_SV_OP_PERMUTE 8     /* one pass moving local bit bits[j] to local bit rbits[j], j < k
                                    (the read-out's undoing of the qubit map) */
typedef struct lyth_sv_op {
    int32_t kind;
    int32_t a, b, c;
    float m[8];                                /* U, CU, EXCHANGE */
    int32_t k;                                 /* FUSED: levels */
    uint32_t bits[LYTH_SV_FUSE_MAX_QUBITS];    /* FUSED: level -> local bit; SWAP_MULTI: local bits */
    uint32_t rbits[LYTH_SV_FUSE_MAX_QUBITS];   /* SWAP_MULTI: rank bits; PERMUTE: destination bits */
    uint32_t ngates;                           /* FUSED */
    int8_t gt[LYTH_SV_FUSE_MAX_GATES];         /* FUSED: target level of gate i */
    int8_t gc[LYTH_SV_FUSE_MAX_GATES];         /* FUSED: control level of gate i, or -1 */
    float gm[LYTH_SV_FUSE_MAX_GATES][8];       /* FUSED: matrix of gate i */
} lyth_sv_op;
int lyth_sv_plan_create(lyth_sv **out, uint32_t qubits, int rank, int nranks);
uint64_t lyth_sv_plan_count(const lyth_sv *sv);
int lyth_sv_plan_op(const lyth_sv *sv, uint64_t index, lyth_sv_op *out);
int lyth_sv_plan_clear(lyth_sv *sv);

#ifdef __cplusplus
}
#endif
#endif
