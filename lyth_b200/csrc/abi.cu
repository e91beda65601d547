// The ADR-0016 callable surface (crates/lyth/src/bind_c.rs:39-395): per kernel, `_elements`,
// `_grid`, `_load`, `_launch`, `_launch_with`, with the signatures LYTH's C generator emits.
//
// `_load` hands out the precompiled sm_100a kernel of this library (cudaGetFuncBySymbol; the
// CUfunction is the driver's handle to it) in place of cuModuleLoadData on embedded PTX. The
// module it reports belongs to the CUDA runtime of this library and lives until the process
// ends; the caller must not unload it. `_launch_with` builds the argument array in declaration
// order and calls cuLaunchKernel(fn, grid, BLOCK, SHARED_BYTES, stream 0) as the generated
// bodies do (bind_c.rs:345-395). The driver entry points are fetched through the runtime, so the
// library links no libcuda and loads on a machine without a GPU.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace lyth {
// Kernels defined in the other translation units.
template <typename I> __global__ void saxpy_kernel(I, float, const float *, float *);
template <typename I> __global__ void axpby_kernel(I, float, float, const float *, float *);
template <typename I> __global__ void lerp_kernel(I, float, const float *, const float *, float *);
template <typename I> __global__ void horner_kernel(I, float, float, float, float, const float *, float *);
template <typename I> __global__ void copy2d_kernel(I, I, const float *, float *);
template <typename I> __global__ void transpose_kernel(I, I, const float *, float *);
template <typename I> __global__ void transpose_tiled_kernel(I, I, const float *, float *);
template <typename I> __global__ void sum_kernel(I, const float *, float *);
template <typename I> __global__ void dot_kernel(I, const float *, const float *, float *);
template <typename I> __global__ void max_of_kernel(I, const float *, float *);
template <typename I> __global__ void min_of_kernel(I, const float *, float *);
__global__ void matmul_kernel(uint32_t, uint32_t, uint32_t, const float *, const float *, float *);
template <typename I> __global__ void hadamard_q_kernel(I, I, float, const float *, const float *, float *, float *);
template <typename I>
__global__ void gate_q_kernel(I, I, float, float, float, float, float, float, float, float, const float *,
                              const float *, float *, float *);
template <typename I>
__global__ void cu_q_kernel(I, I, I, float, float, float, float, float, float, float, float, const float *,
                            const float *, float *, float *);
template <typename I> __global__ void swap_q_kernel(I, I, I, const float *, const float *, float *, float *);
}  // namespace lyth

using namespace lyth;

namespace {

typedef CUresult (*PFN_launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                               CUstream, void **, void **);
typedef CUresult (*PFN_func_module)(CUmodule *, CUfunction);

PFN_launch g_launch = nullptr;
PFN_func_module g_func_module = nullptr;
bool g_entry_done = false;

void fetch_entry_points() {
    if (g_entry_done) return;
    g_entry_done = true;
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuLaunchKernel", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_launch = reinterpret_cast<PFN_launch>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuFuncGetModule", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_func_module = reinterpret_cast<PFN_func_module>(p);
}

CUresult cu_of(cudaError_t e) {
    switch (e) {
        case cudaSuccess: return CUDA_SUCCESS;
        case cudaErrorInvalidValue: return CUDA_ERROR_INVALID_VALUE;
        case cudaErrorNoDevice: return CUDA_ERROR_NO_DEVICE;
        case cudaErrorInsufficientDriver: return CUDA_ERROR_NOT_INITIALIZED;
        case cudaErrorMemoryAllocation: return CUDA_ERROR_OUT_OF_MEMORY;
        default: return CUDA_ERROR_UNKNOWN;
    }
}

CUresult load_symbol(const void *sym, CUmodule *module, CUfunction *fn) {
    if (!fn) return CUDA_ERROR_INVALID_VALUE;
    cudaFunction_t f = nullptr;
    cudaError_t e = cudaGetFuncBySymbol(&f, sym);
    if (e != cudaSuccess) return cu_of(e);
    *fn = reinterpret_cast<CUfunction>(f);
    if (module) {
        *module = nullptr;
        fetch_entry_points();
        if (g_func_module) g_func_module(module, *fn);
    }
    return CUDA_SUCCESS;
}

CUresult launch(CUfunction fn, unsigned grid, unsigned block, unsigned shared, void **args) {
    if (!fn) return CUDA_ERROR_INVALID_HANDLE;
    if (grid == 0) return CUDA_ERROR_INVALID_VALUE;
    fetch_entry_points();
    if (!g_launch) return CUDA_ERROR_NOT_INITIALIZED;
    return g_launch(fn, grid, 1, 1, block, 1, 1, shared, nullptr, args, nullptr);
}

// manifest.rs:161-183: one element (min_elements_per_thread of them) per thread, ceiling, >= 1,
// capped; 0 when the element count is 0.
unsigned elementwise_grid(uint64_t total, unsigned block, unsigned per_thread, unsigned max_grid) {
    if (total == 0) return 0;
    uint64_t per_block = (uint64_t)block * per_thread;
    uint64_t g = (total + per_block - 1) / per_block;
    if (g == 0) g = 1;
    if (g > max_grid) g = max_grid;
    return (unsigned)g;
}

unsigned elements2(unsigned a, unsigned b) {
    unsigned long long t = (unsigned long long)a * b;
    return t > 0xFFFFFFFFull ? 0u : (unsigned)t;
}

bool split_ok(uint64_t len, uint64_t w) { return w != 0 && len % (2 * w) == 0; }

}  // namespace

extern "C" {

int lyth_b200_version(void) { return 100; }

const char *lyth_b200_error_string(int status) {
    switch (status) {
        case LYTH_OK: return "ok";
        case LYTH_E_SPLIT: return "split refused: a width is 0 or 2*width does not divide the level's length";
        case LYTH_E_UNSUPPORTED: return "unsupported shape or parameter for this kernel class";
        case LYTH_E_INVALID: return "invalid argument: null pointer, zero extent, or size past the index range";
        case LYTH_E_TIMEOUT: return "a bounded device wait ran out";
        case LYTH_E_NCCL: return "NCCL error during a state-vector exchange";
        case LYTH_E_NO_NCCL: return "the NCCL library could not be loaded";
        case LYTH_E_OOM: return "state-vector allocation failed";
        default: break;
    }
    if (status > 0) return cudaGetErrorString((cudaError_t)status);
    return "unknown LYTH status";
}

// ---------------------------------------------------------------------- saxpy
unsigned int lyth_saxpy_elements(unsigned int n) { return n; }
unsigned int lyth_saxpy_grid(unsigned int n) { return elementwise_grid(n, LYTH_SAXPY_BLOCK, 1, LYTH_SAXPY_MAX_GRID); }
CUresult lyth_saxpy_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)saxpy_kernel<uint32_t>, module, fn); }
CUresult lyth_saxpy_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float a, CUdeviceptr x, CUdeviceptr y) {
    void *args[] = {&n, &a, &x, &y};
    return launch(fn, grid, LYTH_SAXPY_BLOCK, LYTH_SAXPY_SHARED_BYTES, args);
}
CUresult lyth_saxpy_launch(CUfunction fn, unsigned int n, float a, CUdeviceptr x, CUdeviceptr y) {
    unsigned grid = lyth_saxpy_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_saxpy_launch_with(fn, grid, n, a, x, y);
}

// ---------------------------------------------------------------------- axpby
unsigned int lyth_axpby_elements(unsigned int n) { return n; }
unsigned int lyth_axpby_grid(unsigned int n) { return elementwise_grid(n, LYTH_AXPBY_BLOCK, 1, LYTH_AXPBY_MAX_GRID); }
CUresult lyth_axpby_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)axpby_kernel<uint32_t>, module, fn); }
CUresult lyth_axpby_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float a, float b, CUdeviceptr x, CUdeviceptr y) {
    void *args[] = {&n, &a, &b, &x, &y};
    return launch(fn, grid, LYTH_AXPBY_BLOCK, LYTH_AXPBY_SHARED_BYTES, args);
}
CUresult lyth_axpby_launch(CUfunction fn, unsigned int n, float a, float b, CUdeviceptr x, CUdeviceptr y) {
    unsigned grid = lyth_axpby_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_axpby_launch_with(fn, grid, n, a, b, x, y);
}

// ---------------------------------------------------------------------- lerp
unsigned int lyth_lerp_elements(unsigned int n) { return n; }
unsigned int lyth_lerp_grid(unsigned int n) { return elementwise_grid(n, LYTH_LERP_BLOCK, 1, LYTH_LERP_MAX_GRID); }
CUresult lyth_lerp_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)lerp_kernel<uint32_t>, module, fn); }
CUresult lyth_lerp_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float t, CUdeviceptr x, CUdeviceptr y, CUdeviceptr z) {
    void *args[] = {&n, &t, &x, &y, &z};
    return launch(fn, grid, LYTH_LERP_BLOCK, LYTH_LERP_SHARED_BYTES, args);
}
CUresult lyth_lerp_launch(CUfunction fn, unsigned int n, float t, CUdeviceptr x, CUdeviceptr y, CUdeviceptr z) {
    unsigned grid = lyth_lerp_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_lerp_launch_with(fn, grid, n, t, x, y, z);
}

// ---------------------------------------------------------------------- horner
unsigned int lyth_horner_elements(unsigned int n) { return n; }
unsigned int lyth_horner_grid(unsigned int n) { return elementwise_grid(n, LYTH_HORNER_BLOCK, 1, LYTH_HORNER_MAX_GRID); }
CUresult lyth_horner_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)horner_kernel<uint32_t>, module, fn); }
CUresult lyth_horner_launch_with(CUfunction fn, unsigned int grid, unsigned int n, float c0, float c1, float c2, float c3,
                                 CUdeviceptr x, CUdeviceptr y) {
    void *args[] = {&n, &c0, &c1, &c2, &c3, &x, &y};
    return launch(fn, grid, LYTH_HORNER_BLOCK, LYTH_HORNER_SHARED_BYTES, args);
}
CUresult lyth_horner_launch(CUfunction fn, unsigned int n, float c0, float c1, float c2, float c3, CUdeviceptr x, CUdeviceptr y) {
    unsigned grid = lyth_horner_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_horner_launch_with(fn, grid, n, c0, c1, c2, c3, x, y);
}

// ---------------------------------------------------------------------- copy2d / transposes
unsigned int lyth_copy2d_elements(unsigned int rows, unsigned int cols) { return elements2(rows, cols); }
unsigned int lyth_copy2d_grid(unsigned int rows, unsigned int cols) {
    return elementwise_grid(lyth_copy2d_elements(rows, cols), LYTH_COPY2D_BLOCK, 1, LYTH_COPY2D_MAX_GRID);
}
CUresult lyth_copy2d_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)copy2d_kernel<uint32_t>, module, fn); }
CUresult lyth_copy2d_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b) {
    void *args[] = {&rows, &cols, &a, &b};
    return launch(fn, grid, LYTH_COPY2D_BLOCK, LYTH_COPY2D_SHARED_BYTES, args);
}
CUresult lyth_copy2d_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b) {
    unsigned grid = lyth_copy2d_grid(rows, cols);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_copy2d_launch_with(fn, grid, rows, cols, a, b);
}

unsigned int lyth_transpose_elements(unsigned int rows, unsigned int cols) { return elements2(rows, cols); }
unsigned int lyth_transpose_grid(unsigned int rows, unsigned int cols) {
    return elementwise_grid(lyth_transpose_elements(rows, cols), LYTH_TRANSPOSE_BLOCK, 1, LYTH_TRANSPOSE_MAX_GRID);
}
CUresult lyth_transpose_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)transpose_kernel<uint32_t>, module, fn); }
CUresult lyth_transpose_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b) {
    void *args[] = {&rows, &cols, &a, &b};
    return launch(fn, grid, LYTH_TRANSPOSE_BLOCK, LYTH_TRANSPOSE_SHARED_BYTES, args);
}
CUresult lyth_transpose_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b) {
    unsigned grid = lyth_transpose_grid(rows, cols);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_transpose_launch_with(fn, grid, rows, cols, a, b);
}

unsigned int lyth_transpose_tiled_elements(unsigned int rows, unsigned int cols) { return elements2(rows, cols); }
unsigned int lyth_transpose_tiled_grid(unsigned int rows, unsigned int cols) {
    // One block per tile (manifest.rs:176-181); 0 when the count passes the cap.
    unsigned long long blocks = 1ull;
    blocks *= (rows + LYTH_TRANSPOSE_TILED_TILE - 1u) / LYTH_TRANSPOSE_TILED_TILE;
    blocks *= (cols + LYTH_TRANSPOSE_TILED_TILE - 1u) / LYTH_TRANSPOSE_TILED_TILE;
    if (blocks == 0ull) blocks = 1ull;
    if (blocks > LYTH_TRANSPOSE_TILED_MAX_GRID) return 0u;
    return (unsigned)blocks;
}
CUresult lyth_transpose_tiled_load(CUmodule *module, CUfunction *fn) {
    return load_symbol((const void *)transpose_tiled_kernel<uint32_t>, module, fn);
}
CUresult lyth_transpose_tiled_launch_with(CUfunction fn, unsigned int grid, unsigned int rows, unsigned int cols, CUdeviceptr a,
                                          CUdeviceptr b) {
    void *args[] = {&rows, &cols, &a, &b};
    // The tile lives in static shared memory; SHARED_BYTES documents it, the launch adds none.
    return launch(fn, grid, LYTH_TRANSPOSE_TILED_BLOCK, 0, args);
}
CUresult lyth_transpose_tiled_launch(CUfunction fn, unsigned int rows, unsigned int cols, CUdeviceptr a, CUdeviceptr b) {
    unsigned grid = lyth_transpose_tiled_grid(rows, cols);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_transpose_tiled_launch_with(fn, grid, rows, cols, a, b);
}

// ---------------------------------------------------------------------- reductions
#define LYTH_REDUCTION_COMMON(k, K)                                                                         \
    unsigned int lyth_##k##_elements(unsigned int n) { return n; }                                          \
    unsigned int lyth_##k##_grid(unsigned int n) {                                                          \
        return elementwise_grid(n, LYTH_##K##_BLOCK, 8, LYTH_##K##_MAX_GRID);                               \
    }                                                                                                       \
    unsigned int lyth_##k##_partial_len(unsigned int n) { return lyth_##k##_grid(n); }

LYTH_REDUCTION_COMMON(sum, SUM)
LYTH_REDUCTION_COMMON(dot, DOT)
LYTH_REDUCTION_COMMON(max_of, MAX_OF)
LYTH_REDUCTION_COMMON(min_of, MIN_OF)

// The partial buffer lives in static shared memory in these kernels; the launch adds none.
CUresult lyth_sum_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)sum_kernel<uint32_t>, module, fn); }
CUresult lyth_sum_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    void *args[] = {&n, &x, &partial};
    return launch(fn, grid, LYTH_SUM_BLOCK, 0, args);
}
CUresult lyth_sum_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    unsigned grid = lyth_sum_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_sum_launch_with(fn, grid, n, x, partial);
}
CUresult lyth_dot_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)dot_kernel<uint32_t>, module, fn); }
CUresult lyth_dot_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr y, CUdeviceptr partial) {
    void *args[] = {&n, &x, &y, &partial};
    return launch(fn, grid, LYTH_DOT_BLOCK, 0, args);
}
CUresult lyth_dot_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr y, CUdeviceptr partial) {
    unsigned grid = lyth_dot_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_dot_launch_with(fn, grid, n, x, y, partial);
}
CUresult lyth_max_of_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)max_of_kernel<uint32_t>, module, fn); }
CUresult lyth_max_of_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    void *args[] = {&n, &x, &partial};
    return launch(fn, grid, LYTH_MAX_OF_BLOCK, 0, args);
}
CUresult lyth_max_of_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    unsigned grid = lyth_max_of_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_max_of_launch_with(fn, grid, n, x, partial);
}
CUresult lyth_min_of_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)min_of_kernel<uint32_t>, module, fn); }
CUresult lyth_min_of_launch_with(CUfunction fn, unsigned int grid, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    void *args[] = {&n, &x, &partial};
    return launch(fn, grid, LYTH_MIN_OF_BLOCK, 0, args);
}
CUresult lyth_min_of_launch(CUfunction fn, unsigned int n, CUdeviceptr x, CUdeviceptr partial) {
    unsigned grid = lyth_min_of_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_min_of_launch_with(fn, grid, n, x, partial);
}

// ---------------------------------------------------------------------- matmul
unsigned int lyth_matmul_elements(unsigned int m, unsigned int n) { return elements2(m, n); }
unsigned int lyth_matmul_grid(unsigned int m, unsigned int n) {
    unsigned long long blocks = (unsigned long long)((m + LYTH_MATMUL_TILE - 1u) / LYTH_MATMUL_TILE) *
                                ((n + LYTH_MATMUL_TILE - 1u) / LYTH_MATMUL_TILE);
    if (blocks == 0ull) blocks = 1ull;
    if (blocks > LYTH_MATMUL_MAX_GRID) return 0u;
    return (unsigned)blocks;
}
CUresult lyth_matmul_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)matmul_kernel, module, fn); }
CUresult lyth_matmul_launch_with(CUfunction fn, unsigned int grid, unsigned int m, unsigned int n, unsigned int k, CUdeviceptr a,
                                 CUdeviceptr b, CUdeviceptr c) {
    void *args[] = {&m, &n, &k, &a, &b, &c};
    return launch(fn, grid, LYTH_MATMUL_BLOCK, 0, args);
}
CUresult lyth_matmul_launch(CUfunction fn, unsigned int m, unsigned int n, unsigned int k, CUdeviceptr a, CUdeviceptr b,
                            CUdeviceptr c) {
    unsigned grid = lyth_matmul_grid(m, n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_matmul_launch_with(fn, grid, m, n, k, a, b, c);
}

// ---------------------------------------------------------------------- state-vector gates
// The walk is n >> depth pairs / quads (GridRule::blocks with split_depth, manifest.rs:161-172).
unsigned int lyth_hadamard_q_elements(unsigned int n) { return n; }
unsigned int lyth_hadamard_q_grid(unsigned int n) {
    return elementwise_grid(n >> 1, LYTH_HADAMARD_Q_BLOCK, 1, LYTH_HADAMARD_Q_MAX_GRID);
}
int lyth_hadamard_q_check_splits(unsigned int n, unsigned int w) { return split_ok(n, w) ? LYTH_OK : LYTH_E_SPLIT; }
CUresult lyth_hadamard_q_load(CUmodule *module, CUfunction *fn) {
    return load_symbol((const void *)hadamard_q_kernel<uint32_t>, module, fn);
}
CUresult lyth_hadamard_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int w, float s, CUdeviceptr re,
                                     CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi) {
    if (lyth_hadamard_q_check_splits(n, w) != LYTH_OK) return CUDA_ERROR_INVALID_VALUE;
    void *args[] = {&n, &w, &s, &re, &im, &qr, &qi};
    return launch(fn, grid, LYTH_HADAMARD_Q_BLOCK, LYTH_HADAMARD_Q_SHARED_BYTES, args);
}
CUresult lyth_hadamard_q_launch(CUfunction fn, unsigned int n, unsigned int w, float s, CUdeviceptr re, CUdeviceptr im,
                                CUdeviceptr qr, CUdeviceptr qi) {
    unsigned grid = lyth_hadamard_q_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_hadamard_q_launch_with(fn, grid, n, w, s, re, im, qr, qi);
}

unsigned int lyth_gate_q_elements(unsigned int n) { return n; }
unsigned int lyth_gate_q_grid(unsigned int n) { return elementwise_grid(n >> 1, LYTH_GATE_Q_BLOCK, 1, LYTH_GATE_Q_MAX_GRID); }
int lyth_gate_q_check_splits(unsigned int n, unsigned int w) { return split_ok(n, w) ? LYTH_OK : LYTH_E_SPLIT; }
CUresult lyth_gate_q_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)gate_q_kernel<uint32_t>, module, fn); }
CUresult lyth_gate_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int w, float ar, float ai, float br,
                                 float bi, float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr,
                                 CUdeviceptr qi) {
    if (lyth_gate_q_check_splits(n, w) != LYTH_OK) return CUDA_ERROR_INVALID_VALUE;
    void *args[] = {&n, &w, &ar, &ai, &br, &bi, &cr, &ci, &dr, &di, &re, &im, &qr, &qi};
    return launch(fn, grid, LYTH_GATE_Q_BLOCK, LYTH_GATE_Q_SHARED_BYTES, args);
}
CUresult lyth_gate_q_launch(CUfunction fn, unsigned int n, unsigned int w, float ar, float ai, float br, float bi, float cr,
                            float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi) {
    unsigned grid = lyth_gate_q_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_gate_q_launch_with(fn, grid, n, w, ar, ai, br, bi, cr, ci, dr, di, re, im, qr, qi);
}

unsigned int lyth_cu_q_elements(unsigned int n) { return n; }
unsigned int lyth_cu_q_grid(unsigned int n) { return elementwise_grid(n >> 2, LYTH_CU_Q_BLOCK, 1, LYTH_CU_Q_MAX_GRID); }
int lyth_cu_q_check_splits(unsigned int n, unsigned int wc, unsigned int wt) {
    return (split_ok(n, wc) && split_ok(n / 2, wt)) ? LYTH_OK : LYTH_E_SPLIT;
}
CUresult lyth_cu_q_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)cu_q_kernel<uint32_t>, module, fn); }
CUresult lyth_cu_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int wc, unsigned int wt, float ar,
                               float ai, float br, float bi, float cr, float ci, float dr, float di, CUdeviceptr re,
                               CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi) {
    if (lyth_cu_q_check_splits(n, wc, wt) != LYTH_OK) return CUDA_ERROR_INVALID_VALUE;
    void *args[] = {&n, &wc, &wt, &ar, &ai, &br, &bi, &cr, &ci, &dr, &di, &re, &im, &qr, &qi};
    return launch(fn, grid, LYTH_CU_Q_BLOCK, LYTH_CU_Q_SHARED_BYTES, args);
}
CUresult lyth_cu_q_launch(CUfunction fn, unsigned int n, unsigned int wc, unsigned int wt, float ar, float ai, float br, float bi,
                          float cr, float ci, float dr, float di, CUdeviceptr re, CUdeviceptr im, CUdeviceptr qr,
                          CUdeviceptr qi) {
    unsigned grid = lyth_cu_q_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_cu_q_launch_with(fn, grid, n, wc, wt, ar, ai, br, bi, cr, ci, dr, di, re, im, qr, qi);
}

unsigned int lyth_swap_q_elements(unsigned int n) { return n; }
unsigned int lyth_swap_q_grid(unsigned int n) { return elementwise_grid(n >> 2, LYTH_SWAP_Q_BLOCK, 1, LYTH_SWAP_Q_MAX_GRID); }
int lyth_swap_q_check_splits(unsigned int n, unsigned int wc, unsigned int wt) {
    return (split_ok(n, wc) && split_ok(n / 2, wt)) ? LYTH_OK : LYTH_E_SPLIT;
}
CUresult lyth_swap_q_load(CUmodule *module, CUfunction *fn) { return load_symbol((const void *)swap_q_kernel<uint32_t>, module, fn); }
CUresult lyth_swap_q_launch_with(CUfunction fn, unsigned int grid, unsigned int n, unsigned int wc, unsigned int wt, CUdeviceptr re,
                                 CUdeviceptr im, CUdeviceptr qr, CUdeviceptr qi) {
    if (lyth_swap_q_check_splits(n, wc, wt) != LYTH_OK) return CUDA_ERROR_INVALID_VALUE;
    void *args[] = {&n, &wc, &wt, &re, &im, &qr, &qi};
    return launch(fn, grid, LYTH_SWAP_Q_BLOCK, LYTH_SWAP_Q_SHARED_BYTES, args);
}
CUresult lyth_swap_q_launch(CUfunction fn, unsigned int n, unsigned int wc, unsigned int wt, CUdeviceptr re, CUdeviceptr im,
                            CUdeviceptr qr, CUdeviceptr qi) {
    unsigned grid = lyth_swap_q_grid(n);
    if (grid == 0u) return CUDA_ERROR_INVALID_VALUE;
    return lyth_swap_q_launch_with(fn, grid, n, wc, wt, re, im, qr, qi);
}

}  // extern "C"
