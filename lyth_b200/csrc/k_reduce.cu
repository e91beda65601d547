// Reductions for sm_100a: examples/{sum,dot,max,min}.lyth.
//
// The partials are the reference's, bit for bit (eval.rs:326-345): block b, thread t folds
// x[b*256 + t], x[b*256 + t + grid*256], ... in that order from the identity, then the 256
// slots of the block go through the stride-halving tree (tree_reduce, eval.rs:537-546):
// slots[t] = slots[t] (+) slots[t + s] for s = 128, 64, ..., 1. Here the three widest levels
// run in shared memory and the last five are warp shuffles: __shfl_down_sync(v, s) hands lane
// t exactly slots[t + s], so the tree, and every rounding in it, is unchanged.
//
// The whole reduction (lyth_b200_reduce) launches the same blocks in clusters of 8: after the
// partials, each cluster's leader reads its seven neighbours' partials from their shared
// memory (DSMEM) and folds the eight in block order; a last single-block pass folds the
// cluster results in cluster order. The combine order is therefore fixed and documented, and
// the host oracle reproduces it exactly.
#include <cuda.h>

#include <cooperative_groups.h>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lyth {

constexpr int kRedBlock = 256;
constexpr int kRedPerThread = 8;  // manifest.rs:186-192: a reduction walks 8 elements per thread
constexpr int kCluster = 8;

template <int OP>
LYTH_D float identity_of() {
    return OP == 1 ? -__int_as_float(0x7f800000) : (OP == 2 ? __int_as_float(0x7f800000) : 0.0f);
}

// ReduceOp::combine (ast.rs:222-249). sum: add.rn. max / min: the hardware max.f32 / min.f32
// already order -0 below +0 whichever operand comes first and return the non-NaN operand, which
// is exactly the reference's rule (the signed-zero branch exists in the host evaluator because
// f32::max leaves that case unspecified); the GPU tests pin it on both operand orders.
template <int OP>
LYTH_D float combine(float a, float b) {
    if (OP == 0) return __fadd_rn(a, b);
    return OP == 1 ? fmaxf(a, b) : fminf(a, b);
}

// Element j of a buffer of storage type TY (0 f32, 1 f16, 2 bf16) as f32: the widening of a narrow
// element is exact (ADR-0024: storage, not arithmetic, is narrow).
template <int TY>
LYTH_D float load_el(const void *p, uint64_t j) {
    if (TY == 0) return static_cast<const float *>(p)[j];
    const uint16_t h = static_cast<const uint16_t *>(p)[j];
    return TY == 1 ? __half2float(__ushort_as_half(h)) : __uint_as_float((uint32_t)h << 16);
}

// One block's partial, in the reference's order. `grid` is the grid of the reference's launch
// (the stride is grid * 256); blocks at or past it contribute the identity.
template <int OP, bool DOT, int TY = 0>
LYTH_D float block_partial(uint64_t n, const void *x, const void *y, uint64_t grid, float *slots) {
    const unsigned t = threadIdx.x;
    const uint64_t stride = grid * kRedBlock;
    float acc = identity_of<OP>();
    if (blockIdx.x < grid) {
        uint64_t i = (uint64_t)blockIdx.x * kRedBlock + t;
        // Issue up to eight independent loads, then fold them strictly in order.
        while (i < n) {
            float v[kRedPerThread];
#pragma unroll
            for (int u = 0; u < kRedPerThread; u++) {
                const uint64_t j = i + (uint64_t)u * stride;
                if (j < n) v[u] = DOT ? __fmul_rn(load_el<TY>(x, j), load_el<TY>(y, j)) : load_el<TY>(x, j);
            }
#pragma unroll
            for (int u = 0; u < kRedPerThread; u++) {
                const uint64_t j = i + (uint64_t)u * stride;
                if (j < n) acc = combine<OP>(acc, v[u]);
            }
            i += (uint64_t)kRedPerThread * stride;
        }
    }
    // The tree. Levels 128, 64, 32 through shared memory ...
    slots[t] = acc;
    __syncthreads();
    if (t < 128) slots[t] = combine<OP>(slots[t], slots[t + 128]);
    __syncthreads();
    if (t < 64) slots[t] = combine<OP>(slots[t], slots[t + 64]);
    __syncthreads();
    float v = 0.0f;
    if (t < 32) {
        v = combine<OP>(slots[t], slots[t + 32]);
        // ... and 16, 8, 4, 2, 1 in registers.
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) v = combine<OP>(v, __shfl_down_sync(0xffffffffu, v, s));
    }
    return v;  // valid in thread 0
}

// The B200 surface's partials: the same reference blocks, each still folded and tree-reduced by
// 256 threads in the reference's order, but a CUDA block takes D of them at a time: its threads
// issue the loads of all D (8 x D per thread) before folding any, and the D trees share their
// barriers (three per D reference blocks instead of three per block). One CUDA block per
// reference block keeps too few bytes in flight per SM when a reference block is small (2048
// elements: 8 KiB of f32, 4 KiB of bf16) and pays its barriers and its launch per block.
template <int OP, bool DOT, int TY>
__host__ __device__ constexpr int partials_batch() {
    return DOT ? 2 : 4;
}
template <int OP, bool DOT, int TY>
__global__ void __launch_bounds__(kRedBlock) partials_batched_kernel(uint64_t n, const void *x, const void *y,
                                                                     uint64_t grid, float *partial) {
    constexpr int D = partials_batch<OP, DOT, TY>();
    __shared__ float slots[D][kRedBlock];
    const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint64_t stride = grid * kRedBlock;
    const uint64_t span = (uint64_t)kRedPerThread * stride;
    const uint64_t batches = (grid + D - 1) / D;
    for (uint64_t bt = blockIdx.x; bt < batches; bt += gridDim.x) {
        float vx[D][kRedPerThread], vy[D][kRedPerThread];
        const uint64_t i0 = bt * D * kRedBlock + t;
        if ((bt + 1) * D <= grid && i0 + (D - 1) * kRedBlock + (kRedPerThread - 1) * stride < n) {
            // the whole batch is inside: element (d, u) sits d * 256 after (0, u)
            using E = typename std::conditional<TY == 0, float, uint16_t>::type;
            const E *px = static_cast<const E *>(x) + i0;
            const E *py = static_cast<const E *>(y) + i0;
#pragma unroll
            for (int u = 0; u < kRedPerThread; u++) {
#pragma unroll
                for (int d = 0; d < D; d++) {
                    vx[d][u] = load_el<TY>(px, d * kRedBlock);
                    if (DOT) vy[d][u] = load_el<TY>(py, d * kRedBlock);
                }
                px += stride;
                if (DOT) py += stride;
            }
        } else {
#pragma unroll
            for (int d = 0; d < D; d++) {
                const uint64_t i = i0 + d * kRedBlock;  // reference blocks past `grid` load nothing
#pragma unroll
                for (int u = 0; u < kRedPerThread; u++) {
                    const uint64_t j = i + (uint64_t)u * stride;
                    const bool in = bt * D + d < grid && j < n;
                    vx[d][u] = in ? load_el<TY>(x, j) : 0.0f;
                    if (DOT) vy[d][u] = in ? load_el<TY>(y, j) : 0.0f;
                }
            }
        }
#pragma unroll
        for (int d = 0; d < D; d++) {
            float acc = identity_of<OP>();
            uint64_t i = (bt * D + d) * kRedBlock + t;
            if (bt * D + d < grid) {
#pragma unroll
                for (int u = 0; u < kRedPerThread; u++)
                    if (i + (uint64_t)u * stride < n)
                        acc = combine<OP>(acc, DOT ? __fmul_rn(vx[d][u], vy[d][u]) : vx[d][u]);
                for (i += span; i < n; i += span) {  // inputs longer than 8 * 256 * grid (grid capped at 2^20)
                    float v[kRedPerThread];
#pragma unroll
                    for (int u = 0; u < kRedPerThread; u++) {
                        const uint64_t j = i + (uint64_t)u * stride;
                        if (j < n) v[u] = DOT ? __fmul_rn(load_el<TY>(x, j), load_el<TY>(y, j)) : load_el<TY>(x, j);
                    }
#pragma unroll
                    for (int u = 0; u < kRedPerThread; u++)
                        if (i + (uint64_t)u * stride < n) acc = combine<OP>(acc, v[u]);
                }
            }
            slots[d][t] = acc;
        }
        // The D trees, level by level: 128, 64 in shared memory, then warp d finishes tree d
        // (32 through the last shuffles).
        __syncthreads();
        if (t < 128)
#pragma unroll
            for (int d = 0; d < D; d++) slots[d][t] = combine<OP>(slots[d][t], slots[d][t + 128]);
        __syncthreads();
        if (t < 64)
#pragma unroll
            for (int d = 0; d < D; d++) slots[d][t] = combine<OP>(slots[d][t], slots[d][t + 64]);
        __syncthreads();
        if (warp < (unsigned)D && bt * D + warp < grid) {
            float v = combine<OP>(slots[warp][lane], slots[warp][lane + 32]);
#pragma unroll
            for (int s2 = 16; s2 > 0; s2 >>= 1) v = combine<OP>(v, __shfl_down_sync(0xffffffffu, v, s2));
            if (lane == 0) partial[bt * D + warp] = v;
        }
        __syncthreads();  // the slots are rewritten by the next batch
    }
}

// 16-bit elements: a thread takes two neighbouring reference threads (elements 2j and 2j + 1 of
// a reference block) with one 32-bit load each step and keeps their two folds apart, so a CUDA
// block of 256 threads covers two reference blocks per slot; D reference blocks (S slots) per
// iteration. Every fold and every tree is still the reference's.
template <int OP, bool DOT, int TY>
__host__ __device__ constexpr int pair_slots() {
    return DOT ? 2 : 4;
}
template <int TY>
LYTH_D float widen16(uint32_t h) {
    return TY == 1 ? __half2float(__ushort_as_half((uint16_t)h)) : __uint_as_float(h << 16);
}
template <int OP, bool DOT, int TY>
__global__ void __launch_bounds__(kRedBlock) partials_pair_kernel(uint64_t n, const uint16_t *x, const uint16_t *y,
                                                                  uint64_t grid, float *partial) {
    constexpr int S = pair_slots<OP, DOT, TY>(), D = 2 * S;
    __shared__ float slots[D][kRedBlock];
    const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31, h = t >> 7, tt = t & 127;
    const uint64_t stride = grid * kRedBlock;
    const uint64_t span = (uint64_t)kRedPerThread * stride;
    const uint64_t batches = (grid + D - 1) / D;
    for (uint64_t bt = blockIdx.x; bt < batches; bt += gridDim.x) {
        const uint64_t rb0 = bt * D;
        float lo[S], hi[S];
        if ((bt + 1) * D <= grid && span >= n && (rb0 + D) * kRedBlock + (kRedPerThread - 1) * stride <= n) {
            uint32_t wx[S][kRedPerThread], wy[S][kRedPerThread];
#pragma unroll
            for (int q = 0; q < S; q++) {
                const uint32_t *px = reinterpret_cast<const uint32_t *>(x + (rb0 + 2 * q + h) * kRedBlock + 2 * tt);
                const uint32_t *py = reinterpret_cast<const uint32_t *>(y + (rb0 + 2 * q + h) * kRedBlock + 2 * tt);
#pragma unroll
                for (int u = 0; u < kRedPerThread; u++) {
                    wx[q][u] = px[(uint64_t)u * (stride >> 1)];
                    if (DOT) wy[q][u] = py[(uint64_t)u * (stride >> 1)];
                }
            }
#pragma unroll
            for (int q = 0; q < S; q++) {
                float a0 = identity_of<OP>(), a1 = identity_of<OP>();
#pragma unroll
                for (int u = 0; u < kRedPerThread; u++) {
                    const float x0 = widen16<TY>(wx[q][u] & 0xFFFFu), x1 = widen16<TY>(wx[q][u] >> 16);
                    if (DOT) {
                        const float y0 = widen16<TY>(wy[q][u] & 0xFFFFu), y1 = widen16<TY>(wy[q][u] >> 16);
                        a0 = combine<OP>(a0, __fmul_rn(x0, y0));
                        a1 = combine<OP>(a1, __fmul_rn(x1, y1));
                    } else {
                        a0 = combine<OP>(a0, x0);
                        a1 = combine<OP>(a1, x1);
                    }
                }
                lo[q] = a0;
                hi[q] = a1;
            }
        } else {
#pragma unroll
            for (int q = 0; q < S; q++) {
                const uint64_t rb = rb0 + 2 * q + h;
                float a[2] = {identity_of<OP>(), identity_of<OP>()};
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    if (rb >= grid) continue;  // reference blocks past `grid` load nothing
                    for (uint64_t i = rb * kRedBlock + 2 * tt + e; i < n; i += span) {
                        float v[kRedPerThread];
#pragma unroll
                        for (int u = 0; u < kRedPerThread; u++) {
                            const uint64_t j = i + (uint64_t)u * stride;
                            if (j < n) v[u] = DOT ? __fmul_rn(load_el<TY>(x, j), load_el<TY>(y, j)) : load_el<TY>(x, j);
                        }
#pragma unroll
                        for (int u = 0; u < kRedPerThread; u++)
                            if (i + (uint64_t)u * stride < n) a[e] = combine<OP>(a[e], v[u]);
                    }
                }
                lo[q] = a[0];
                hi[q] = a[1];
            }
        }
#pragma unroll
        for (int q = 0; q < S; q++) {
            slots[2 * q + h][2 * tt] = lo[q];
            slots[2 * q + h][2 * tt + 1] = hi[q];
        }
        // The D trees level by level (128, 64 in shared memory), then warp d finishes tree d.
        __syncthreads();
#pragma unroll
        for (unsigned k = t; k < (unsigned)D * 128; k += kRedBlock)
            slots[k >> 7][k & 127] = combine<OP>(slots[k >> 7][k & 127], slots[k >> 7][(k & 127) + 128]);
        __syncthreads();
#pragma unroll
        for (unsigned k = t; k < (unsigned)D * 64; k += kRedBlock)
            slots[k >> 6][k & 63] = combine<OP>(slots[k >> 6][k & 63], slots[k >> 6][(k & 63) + 64]);
        __syncthreads();
        if (warp < (unsigned)D && rb0 + warp < grid) {
            float v = combine<OP>(slots[warp][lane], slots[warp][lane + 32]);
#pragma unroll
            for (int s2 = 16; s2 > 0; s2 >>= 1) v = combine<OP>(v, __shfl_down_sync(0xffffffffu, v, s2));
            if (lane == 0) partial[rb0 + warp] = v;
        }
        __syncthreads();  // the slots are rewritten by the next batch
    }
}

template <int OP, bool DOT, int TY>
int launch_pair(uint64_t n, const uint16_t *x, const uint16_t *y, uint32_t grid, float *partial, cudaStream_t s) {
    static int per_sm = 0;
    if (per_sm == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, partials_pair_kernel<OP, DOT, TY>, kRedBlock, 0) !=
                cudaSuccess ||
            b < 1)
            b = 1;
        per_sm = b;
    }
    constexpr int D = 2 * pair_slots<OP, DOT, TY>();
    const uint64_t cap = (uint64_t)device_sms() * per_sm;
    const uint64_t batches = (grid + D - 1) / D;
    const unsigned blocks = (unsigned)(batches < cap ? batches : cap);
    partials_pair_kernel<OP, DOT, TY><<<blocks, kRedBlock, 0, s>>>(n, x, y, grid, partial);
    return last_launch_status();
}

// Blocks of the grid: as many as fit on the device at once, at most one per batch of reference
// blocks.
template <int OP, bool DOT, int TY>
int launch_batched(uint64_t n, const void *x, const void *y, uint32_t grid, float *partial, cudaStream_t s) {
    static int per_sm = 0;
    if (per_sm == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, partials_batched_kernel<OP, DOT, TY>, kRedBlock, 0) !=
                cudaSuccess ||
            b < 1)
            b = 1;
        per_sm = b;
    }
    const uint64_t cap = (uint64_t)device_sms() * per_sm;
    const uint64_t batches = (grid + partials_batch<OP, DOT, TY>() - 1) / partials_batch<OP, DOT, TY>();
    const unsigned blocks = (unsigned)(batches < cap ? batches : cap);
    partials_batched_kernel<OP, DOT, TY><<<blocks, kRedBlock, 0, s>>>(n, x, y, grid, partial);
    return last_launch_status();
}

// The ADR-0016 kernels, in the reference's parameter order.
template <typename I>
__global__ void __launch_bounds__(kRedBlock) sum_kernel(I n, const float *x, float *partial) {
    __shared__ float slots[kRedBlock];
    const float v = block_partial<0, false>((uint64_t)n, x, nullptr, gridDim.x, slots);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
}
template <typename I>
__global__ void __launch_bounds__(kRedBlock) dot_kernel(I n, const float *x, const float *y, float *partial) {
    __shared__ float slots[kRedBlock];
    const float v = block_partial<0, true>((uint64_t)n, x, y, gridDim.x, slots);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
}
template <typename I>
__global__ void __launch_bounds__(kRedBlock) max_of_kernel(I n, const float *x, float *partial) {
    __shared__ float slots[kRedBlock];
    const float v = block_partial<1, false>((uint64_t)n, x, nullptr, gridDim.x, slots);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
}
template <typename I>
__global__ void __launch_bounds__(kRedBlock) min_of_kernel(I n, const float *x, float *partial) {
    __shared__ float slots[kRedBlock];
    const float v = block_partial<2, false>((uint64_t)n, x, nullptr, gridDim.x, slots);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
}

template __global__ void sum_kernel<uint32_t>(uint32_t, const float *, float *);
template __global__ void dot_kernel<uint32_t>(uint32_t, const float *, const float *, float *);
template __global__ void max_of_kernel<uint32_t>(uint32_t, const float *, float *);
template __global__ void min_of_kernel<uint32_t>(uint32_t, const float *, float *);

// Clusters of 8 blocks: the partial of every block, then the leader folds the cluster's
// eight partials (blocks 8q .. 8q+7, in order) reading its neighbours' shared memory.
template <int OP, bool DOT>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kRedBlock)
    reduce_cluster_kernel(uint64_t n, const float *x, const float *y, uint64_t grid, float *cluster_out) {
    __shared__ float slots[kRedBlock];
    __shared__ float mine;
    cg::cluster_group cluster = cg::this_cluster();
    const float v = block_partial<OP, DOT>(n, x, y, grid, slots);
    if (threadIdx.x == 0) mine = v;
    cluster.sync();
    if (cluster.block_rank() == 0 && threadIdx.x == 0) {
        float acc = mine;
        for (unsigned r = 1; r < kCluster; r++) {
            const float *peer = cluster.map_shared_rank(&mine, r);
            acc = combine<OP>(acc, *peer);
        }
        cluster_out[blockIdx.x / kCluster] = acc;
    }
    // No block may leave while the leader may still read its shared memory.
    cluster.sync();
}

// Fold `count` values in index order, one thread: the last step is tiny (grid / 8 values).
template <int OP>
__global__ void fold_kernel(uint64_t count, const float *in, float *out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        float acc = in[0];
        for (uint64_t i = 1; i < count; i++) acc = combine<OP>(acc, in[i]);
        *out = acc;
    }
}

template <int OP, bool DOT>
int reduce_full(uint64_t n, const float *x, const float *y, float *out, float *ws, cudaStream_t s) {
    const uint64_t grid = lyth_b200_reduce_grid(n);
    const uint64_t clusters = (grid + kCluster - 1) / kCluster;
    reduce_cluster_kernel<OP, DOT><<<(unsigned)(clusters * kCluster), kRedBlock, 0, s>>>(n, x, y, grid, ws);
    int st = last_launch_status();
    if (st) return st;
    fold_kernel<OP><<<1, 32, 0, s>>>(clusters, ws, out);
    return last_launch_status();
}

}  // namespace lyth

using namespace lyth;

extern "C" uint32_t lyth_b200_reduce_grid(uint64_t n) {
    uint64_t per = (uint64_t)kRedBlock * kRedPerThread;
    uint64_t g = (n + per - 1) / per;
    if (g == 0) g = 1;
    if (g > (1u << 20)) g = 1u << 20;
    return (uint32_t)g;
}

template <int TY>
static int launch_partials(int op, uint64_t n, const void *x, const void *y, uint32_t grid, float *partial,
                           cudaStream_t s) {
    if (op == 0 && y) return launch_batched<0, true, TY>(n, x, y, grid, partial, s);
    if (op == 0) return launch_batched<0, false, TY>(n, x, y, grid, partial, s);
    if (op == 1 && !y) return launch_batched<1, false, TY>(n, x, y, grid, partial, s);
    if (op == 2 && !y) return launch_batched<2, false, TY>(n, x, y, grid, partial, s);
    return LYTH_E_UNSUPPORTED;
}

template <int TY>
static int launch_partials_pair(int op, uint64_t n, const uint16_t *x, const uint16_t *y, uint32_t grid,
                                float *partial, cudaStream_t s) {
    if (op == 0 && y) return launch_pair<0, true, TY>(n, x, y, grid, partial, s);
    if (op == 0) return launch_pair<0, false, TY>(n, x, y, grid, partial, s);
    if (op == 1 && !y) return launch_pair<1, false, TY>(n, x, y, grid, partial, s);
    if (op == 2 && !y) return launch_pair<2, false, TY>(n, x, y, grid, partial, s);
    return LYTH_E_UNSUPPORTED;
}

extern "C" int lyth_b200_reduce_partials_narrow(int op, int ty, uint64_t n, const uint16_t *x, const uint16_t *y,
                                                uint32_t grid, float *partial, cudaStream_t s) {
    if (!x || !partial || grid == 0) return LYTH_E_INVALID;
    // buffers on 4-byte boundaries take the paired 32-bit loads
    if (!((((uintptr_t)x) | ((uintptr_t)y)) & 3u)) {
        if (ty == LYTH_NARROW_F16) return launch_partials_pair<1>(op, n, x, y, grid, partial, s);
        if (ty == LYTH_NARROW_BF16) return launch_partials_pair<2>(op, n, x, y, grid, partial, s);
    }
    if (ty == LYTH_NARROW_F16) return launch_partials<1>(op, n, x, y, grid, partial, s);
    if (ty == LYTH_NARROW_BF16) return launch_partials<2>(op, n, x, y, grid, partial, s);
    return LYTH_E_UNSUPPORTED;
}

extern "C" int lyth_b200_reduce_partials(int op, uint64_t n, const float *x, const float *y, uint32_t grid,
                                         float *partial, cudaStream_t s) {
    if (!x || !partial || grid == 0) return LYTH_E_INVALID;
    return launch_partials<0>(op, n, x, y, grid, partial, s);
}

extern "C" size_t lyth_b200_reduce_workspace_bytes(uint64_t n) {
    const uint64_t grid = lyth_b200_reduce_grid(n);
    return (size_t)((grid + kCluster - 1) / kCluster) * sizeof(float);
}

extern "C" int lyth_b200_reduce(int op, uint64_t n, const float *x, const float *y, float *out, void *workspace,
                                size_t workspace_bytes, cudaStream_t s) {
    if (!x || !out || !workspace) return LYTH_E_INVALID;
    if (workspace_bytes < lyth_b200_reduce_workspace_bytes(n)) return LYTH_E_INVALID;
    float *ws = static_cast<float *>(workspace);
    if (op == 0 && y) return reduce_full<0, true>(n, x, y, out, ws, s);
    if (op == 0) return reduce_full<0, false>(n, x, nullptr, out, ws, s);
    if (op == 1 && !y) return reduce_full<1, false>(n, x, nullptr, out, ws, s);
    if (op == 2 && !y) return reduce_full<2, false>(n, x, nullptr, out, ws, s);
    return LYTH_E_UNSUPPORTED;
}

// ---------------------------------------------------------------------------------------------
// The whole reduction without any allocation by anyone: lyth_b200_reduce_noalloc.
//
// Some callers cannot hand this library a device workspace: a host that has given all device
// memory to its own arena and forbids further allocation, a runtime that embeds LYTH kernels as
// plug-ins and does not let them allocate, or a latency-bound loop that cannot afford the device
// synchronisation cudaMalloc brings. For them the cluster results of the reduction go to a
// fixed array in the library's own device memory instead of a caller workspace. The kernels and
// the combine order are those of lyth_b200_reduce, so the result is the same, bit for bit.
//
// The array holds 16384 cluster results (64 KiB), enough for n up to LYTH_REDUCE_NOALLOC_MAX_N =
// 2^28 elements (16384 clusters x 8 blocks x 2048 elements); every GPU that loads the library
// keeps it until the process exits. The first call on a device looks the array's address up
// (cudaGetSymbolAddress); make that first call before any stream capture. Each call writes every slot it
// later reads, so nothing has to start at zero, but all calls share the array: two calls that
// overlap on the GPU (different streams, or devices sharing nothing but this process) race.
namespace lyth {

constexpr uint32_t kNoAllocClusters = 16384;
static __device__ __align__(256) float g_noalloc_clusters[kNoAllocClusters];

// The array's device address, looked up with the device current (a host-side use of the
// symbol's name is not a device address) on the first call in each CUDA context: it is cached per
// device together with the context it was found in, and looked up again when the device's current
// context is another one (after a cudaDeviceReset, say). A mutex guards the cache, so host threads
// may call concurrently.
typedef CUresult (*PFN_ctx_get_current)(CUcontext *);

static CUcontext current_context() {
    static PFN_ctx_get_current fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_ctx_get_current>(p);
    });
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

static float *noalloc_scratch(int *status) {
    static std::mutex mu;
    static float *ptr_of[64] = {nullptr};
    static CUcontext ctx_of[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = status_of(e);
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        *status = LYTH_E_UNSUPPORTED;
        return nullptr;
    }
    // No context current on this thread yet (null) also means "look it up": the lookup makes
    // the device's primary context current.
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(mu);
    if (!ptr_of[dev] || !ctx || ctx_of[dev] != ctx) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_clusters);
        if (e != cudaSuccess) {
            *status = status_of(e);
            return nullptr;
        }
        ptr_of[dev] = static_cast<float *>(p);
        ctx_of[dev] = current_context();
    }
    *status = LYTH_OK;
    return ptr_of[dev];
}

}  // namespace lyth

extern "C" int lyth_b200_reduce_noalloc(int op, uint64_t n, const float *x, const float *y, float *out,
                                        cudaStream_t s) {
    if (!x || !out) return LYTH_E_INVALID;
    if (n > LYTH_REDUCE_NOALLOC_MAX_N) return LYTH_E_UNSUPPORTED;  // more clusters than the array holds
    if (!((op == 0) || ((op == 1 || op == 2) && !y))) return LYTH_E_UNSUPPORTED;
    int st = LYTH_OK;
    float *ws = noalloc_scratch(&st);
    if (!ws) return st;
    if (op == 0 && y) return reduce_full<0, true>(n, x, y, out, ws, s);
    if (op == 0) return reduce_full<0, false>(n, x, nullptr, out, ws, s);
    if (op == 1) return reduce_full<1, false>(n, x, nullptr, out, ws, s);
    return reduce_full<2, false>(n, x, nullptr, out, ws, s);
}
