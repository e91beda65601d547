// Streamed elementwise bodies (examples/{saxpy,axpby,lerp,horner}.lyth) and the rank-2 walks
// (examples/{copy2d,transpose,transpose-tiled}.lyth) for sm_100a.
//
// The reference emits one scalar ld/st per element per thread (crates/lyth-ptx/src/lib.rs:
// 299-763). Here every stream moves in 128-bit vectors, grid-stride over a grid sized to fill
// the 148 SMs, two vectors per stream in flight per thread; a scalar path serves unaligned
// buffers and the n % 4 tail. The arithmetic is the lowered body, op for op: fma only where
// ir.rs:2388-2429 forms one, every other op one rounding (built with -fmad=false).
#include "common.cuh"

namespace lyth {

// ------------------------------------------------------------------ elementwise bodies
struct SaxpyBody {
    float a;
    LYTH_D float operator()(float x, float y) const { return __fmaf_rn(a, x, y); }
};
struct AxpbyBody {
    float a, b;
    LYTH_D float operator()(float x, float y) const { return __fmaf_rn(a, x, __fmul_rn(b, y)); }
};
struct LerpBody {
    float t;
    LYTH_D float operator()(float x, float y) const { return __fmaf_rn(t, __fsub_rn(y, x), x); }
};
struct HornerBody {
    float c0, c1, c2, c3;
    LYTH_D float operator()(float x, float) const {
        return __fmaf_rn(__fmaf_rn(__fmaf_rn(c3, x, c2), x, c1), x, c0);
    }
};
struct CopyBody {
    LYTH_D float operator()(float x, float) const { return x; }
};

template <typename F>
LYTH_D float4 apply4(const F &f, float4 x, float4 y) {
    return make_float4(f(x.x, y.x), f(x.y, y.y), f(x.z, y.z), f(x.w, y.w));
}

// out[i] = f(x[i], y[i]) over i < n. TWO_IN: whether y is read (saxpy/axpby/lerp read it;
// horner/copy do not). `out` may equal `y` (the in-place drains of saxpy and axpby): each
// element is read before it is written by the same thread, and no other thread touches it.
template <bool TWO_IN, typename F, typename I>
LYTH_D void stream_body(I n, const F &f, const float *x, const float *y, float *out) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nn = (uint64_t)n;
    const bool vec = ((((uintptr_t)x) | ((uintptr_t)out) | (TWO_IN ? (uintptr_t)y : 0)) & 15u) == 0;
    if (vec) {
        const uint64_t nv = nn >> 2;  // float4 count
        uint64_t v = tid;
        // Two vectors per stream in flight per thread: v and v + nthreads.
        for (; v + nthreads < nv; v += 2 * nthreads) {
            const uint64_t v2 = v + nthreads;
            float4 x0 = ld_stream4(x + 4 * v), x1 = ld_stream4(x + 4 * v2);
            float4 y0 = make_float4(0.f, 0.f, 0.f, 0.f), y1 = y0;
            if (TWO_IN) { y0 = ld4(y + 4 * v); y1 = ld4(y + 4 * v2); }
            st4(out + 4 * v, apply4(f, x0, y0));
            st4(out + 4 * v2, apply4(f, x1, y1));
        }
        if (v < nv) {
            float4 x0 = ld_stream4(x + 4 * v);
            float4 y0 = TWO_IN ? ld4(y + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
            st4(out + 4 * v, apply4(f, x0, y0));
        }
        // The ragged tail: at most three elements.
        const uint64_t t = (nv << 2) + tid;
        if (t < nn) out[t] = f(x[t], TWO_IN ? y[t] : 0.f);
    } else {
        for (uint64_t i = tid; i < nn; i += nthreads) out[i] = f(x[i], TWO_IN ? y[i] : 0.f);
    }
}

// The kernels carry the reference's parameter lists in declaration order, so the ADR-0016
// launchers can hand cuLaunchKernel the same argument array the generated C bodies build.
template <typename I>
__global__ void __launch_bounds__(256) saxpy_kernel(I n, float a, const float *x, float *y) {
    stream_body<true>(n, SaxpyBody{a}, x, y, y);
}
template <typename I>
__global__ void __launch_bounds__(256) axpby_kernel(I n, float a, float b, const float *x, float *y) {
    stream_body<true>(n, AxpbyBody{a, b}, x, y, y);
}
template <typename I>
__global__ void __launch_bounds__(256) lerp_kernel(I n, float t, const float *x, const float *y, float *z) {
    stream_body<true>(n, LerpBody{t}, x, y, z);
}
template <typename I>
__global__ void __launch_bounds__(256) horner_kernel(I n, float c0, float c1, float c2, float c3, const float *x,
                                                     float *y) {
    stream_body<false>(n, HornerBody{c0, c1, c2, c3}, x, nullptr, y);
}
// copy2d: rank 2, but both buffers walk the same row-major order, so it is a linear copy.
template <typename I>
__global__ void __launch_bounds__(256) copy2d_kernel(I rows, I cols, const float *a, float *b) {
    stream_body<false>((uint64_t)rows * cols, CopyBody{}, a, nullptr, b);
}

// The untiled transpose, kept as the strided control (examples/transpose.lyth): linear k
// walks `a` row-major, k -> (i, j) = (k / cols, k % cols), and writes b[j][i].
template <typename I>
__global__ void __launch_bounds__(256) transpose_kernel(I rows, I cols, const float *a, float *b) {
    const uint64_t n = (uint64_t)rows * cols;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += nthreads) {
        const uint64_t i = k / cols, j = k % cols;
        b[j * rows + i] = a[k];
    }
}

// ------------------------------------------------------------------ the tiled transpose
// One 64 x 64 tile per block-iteration through shared memory whose row stride is the
// derived skew: the tile width padded until it is coprime with the 32 banks (ir.rs:2056-2062
// gives 33 for the reference's 32-wide tile; 65 here). With that stride and eight lanes per
// 32-float row segment, both the staging writes and the transposed reads of a warp hit 32
// distinct banks: lane l touches row (l / 8) and column 4*(l % 8) + e, and with stride = 1
// (mod 32) its bank is l/8 + 4*(l % 8) + e, distinct over the warp for each e.
constexpr int kTile = 64;
constexpr int kTileStride = 65;  // skewed_stride(64)

template <typename I>
__global__ void __launch_bounds__(256) transpose_tiled_kernel(I rows_, I cols_, const float *a, float *b) {
    __shared__ float tile[kTile * kTileStride];
    const uint32_t rows = (uint32_t)rows_, cols = (uint32_t)cols_;
    const uint32_t tiles_x = (cols + kTile - 1) / kTile, tiles_y = (rows + kTile - 1) / kTile;
    const uint64_t tiles = (uint64_t)tiles_x * tiles_y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lr = lane >> 3;        // row within a 4-row patch
    const int lc = (lane & 7) << 2;  // first of four columns within a 32-column half
    // 128-bit paths need every row start 16-byte aligned on both sides.
    const bool vec = ((cols & 3u) == 0) && ((rows & 3u) == 0) && ((((uintptr_t)a) | ((uintptr_t)b)) & 15u) == 0;

    for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const uint32_t r0 = (uint32_t)(t / tiles_x) * kTile, c0 = (uint32_t)(t % tiles_x) * kTile;
        // Stage: 32 patches of 4 rows x 32 columns; warp w takes patches w, w+8, w+16, w+24.
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int patch = warp + 8 * p;
            const int tr = (patch >> 1) * 4 + lr, tc = (patch & 1) * 32 + lc;
            const uint32_t r = r0 + tr, c = c0 + tc;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < rows) {
                const float *src = a + (uint64_t)r * cols + c;
                if (vec) {
                    if (c < cols) v = ld_stream4(src);
                } else {
                    if (c < cols) v.x = src[0];
                    if (c + 1 < cols) v.y = src[1];
                    if (c + 2 < cols) v.z = src[2];
                    if (c + 3 < cols) v.w = src[3];
                }
            }
            float *d = tile + tr * kTileStride + tc;
            d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
        }
        __syncthreads();
        // Drain: output row c0 + oc of b (an input column), elements r0 + orr .. + 3.
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int patch = warp + 8 * p;
            const int oc = (patch >> 1) * 4 + lr, orr = (patch & 1) * 32 + lc;
            const uint32_t c = c0 + oc, r = r0 + orr;
            if (c < cols) {
                float4 v;
                v.x = tile[(orr + 0) * kTileStride + oc];
                v.y = tile[(orr + 1) * kTileStride + oc];
                v.z = tile[(orr + 2) * kTileStride + oc];
                v.w = tile[(orr + 3) * kTileStride + oc];
                float *dst = b + (uint64_t)c * rows + r;
                if (vec) {
                    if (r < rows) st_stream4(dst, v);
                } else {
                    if (r < rows) dst[0] = v.x;
                    if (r + 1 < rows) dst[1] = v.y;
                    if (r + 2 < rows) dst[2] = v.z;
                    if (r + 3 < rows) dst[3] = v.w;
                }
            }
        }
        __syncthreads();
    }
}

// Explicit instantiations: u32 for the ADR-0016 launchers, u64 for the B200 surface.
template __global__ void saxpy_kernel<uint32_t>(uint32_t, float, const float *, float *);
template __global__ void axpby_kernel<uint32_t>(uint32_t, float, float, const float *, float *);
template __global__ void lerp_kernel<uint32_t>(uint32_t, float, const float *, const float *, float *);
template __global__ void horner_kernel<uint32_t>(uint32_t, float, float, float, float, const float *, float *);
template __global__ void copy2d_kernel<uint32_t>(uint32_t, uint32_t, const float *, float *);
template __global__ void transpose_kernel<uint32_t>(uint32_t, uint32_t, const float *, float *);
template __global__ void transpose_tiled_kernel<uint32_t>(uint32_t, uint32_t, const float *, float *);

}  // namespace lyth

using namespace lyth;

// ------------------------------------------------------------------ B200 surface
namespace {
inline unsigned elem_grid(uint64_t n) { return stream_grid((n + 3) / 4, 2ull * kStreamBlock); }
}  // namespace

extern "C" int lyth_b200_saxpy(uint64_t n, float a, const float *x, float *y, cudaStream_t s) {
    if (n == 0) return LYTH_OK;
    if (!x || !y) return LYTH_E_INVALID;
    saxpy_kernel<uint64_t><<<elem_grid(n), kStreamBlock, 0, s>>>(n, a, x, y);
    return last_launch_status();
}
extern "C" int lyth_b200_axpby(uint64_t n, float a, float b, const float *x, float *y, cudaStream_t s) {
    if (n == 0) return LYTH_OK;
    if (!x || !y) return LYTH_E_INVALID;
    axpby_kernel<uint64_t><<<elem_grid(n), kStreamBlock, 0, s>>>(n, a, b, x, y);
    return last_launch_status();
}
extern "C" int lyth_b200_lerp(uint64_t n, float t, const float *x, const float *y, float *z, cudaStream_t s) {
    if (n == 0) return LYTH_OK;
    if (!x || !y || !z) return LYTH_E_INVALID;
    lerp_kernel<uint64_t><<<elem_grid(n), kStreamBlock, 0, s>>>(n, t, x, y, z);
    return last_launch_status();
}
extern "C" int lyth_b200_horner(uint64_t n, float c0, float c1, float c2, float c3, const float *x, float *y,
                                cudaStream_t s) {
    if (n == 0) return LYTH_OK;
    if (!x || !y) return LYTH_E_INVALID;
    horner_kernel<uint64_t><<<elem_grid(n), kStreamBlock, 0, s>>>(n, c0, c1, c2, c3, x, y);
    return last_launch_status();
}
extern "C" int lyth_b200_copy2d(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * cols;
    if (n == 0) return LYTH_OK;
    if (!a || !b) return LYTH_E_INVALID;
    copy2d_kernel<uint32_t><<<elem_grid(n), kStreamBlock, 0, s>>>(rows, cols, a, b);
    return last_launch_status();
}
extern "C" int lyth_b200_transpose_naive(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * cols;
    if (n == 0) return LYTH_OK;
    if (!a || !b) return LYTH_E_INVALID;
    transpose_kernel<uint32_t><<<stream_grid(n, kStreamBlock), kStreamBlock, 0, s>>>(rows, cols, a, b);
    return last_launch_status();
}
extern "C" int lyth_b200_transpose_tiled(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t s) {
    if ((uint64_t)rows * cols == 0) return LYTH_OK;
    if (!a || !b) return LYTH_E_INVALID;
    const uint64_t tiles = (uint64_t)((rows + kTile - 1) / kTile) * ((cols + kTile - 1) / kTile);
    const unsigned grid = (unsigned)(tiles < 0x7fffffffull ? tiles : 0x7fffffffull);
    transpose_tiled_kernel<uint32_t><<<grid, 256, 0, s>>>(rows, cols, a, b);
    return last_launch_status();
}
