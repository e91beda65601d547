// Streamed elementwise bodies (examples/{saxpy,axpby,lerp,horner}.lyth) and the rank-2 walks
// (examples/{copy2d,transpose,transpose-tiled}.lyth) for sm_100a.
//
// The reference emits one scalar ld/st per element per thread (crates/lyth-ptx/src/lib.rs:
// 299-763). Here every stream moves in 128-bit vectors, grid-stride over a grid sized to fill
// the 148 SMs, two vectors per stream in flight per thread; a scalar path serves unaligned
// buffers and the n % 4 tail. The arithmetic is the lowered body, op for op: fma only where
// ir.rs:2388-2429 forms one, every other op one rounding (built with -fmad=false).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <string.h>

#include "common.cuh"
#include "mbar.cuh"

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

// ------------------------------------------------------------------ the TMA-staged transpose
// The tiled transpose for shapes whose rows and columns are multiples of 4 (16-byte row pitches,
// what a tensor map needs): 32 x 32 tiles move global -> shared and shared -> global as tensor-map
// boxes (cp.async.bulk.tensor.2d, no multicast), never through the SM's load/store units.
//
// The reference skews its shared tile to a 33-word row (ir.rs:2056-2062): a column walk then hits
// 32 distinct banks. A TMA box lands densely, 128 bytes a row, so the skew becomes the tensor
// map's 128-byte swizzle: the 16-byte chunk c of row r is stored at chunk c ^ (r & 7). A thread
// moves a 4 x 4 block -- four 128-bit loads of rows 4tr..4tr+3 at chunk tc, a transpose in
// registers, four 128-bit stores into the output tile's rows 4tc..4tc+3 at chunk tr -- and the
// 64 threads of a tile take (tr, tc) = (p ^ q, p) for lane p = t % 8 of group q = t / 8, so the 8
// lanes of every quarter-warp reach 8 distinct chunks on both the loads (tc ^ (4tr + i) & 7) and
// the stores (tr ^ (4tc + j) & 7): no bank conflicts, which is what the skew was for.
//
// A CTA is four teams of 64 threads; a team double-buffers its input tiles (the tile two ahead is
// loaded while this one is transposed), writes the transposed tile to its output buffer, and its
// leader stores it with one box (edges clip: coordinates past the extents are not written) and
// waits for the store to have read the buffer before the team writes it again. Every wait is
// bounded; the team decides together (bar.red.and) whether a tile arrived.
constexpr int kTxTeams = 4, kTxTeamThreads = 64;
constexpr uint32_t kTxTileBytes = 32 * 32 * sizeof(float);
constexpr size_t kTxSmem = 1024 + (size_t)kTxTeams * 3 * kTxTileBytes + kTxTeams * 2 * sizeof(uint64_t);
__device__ int g_tx_error;

LYTH_D void tensor_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
LYTH_D void tensor_store_2d(const CUtensorMap *map, int c0, int c1, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"((uint64_t)map),
                 "r"(c0), "r"(c1), "r"(src)
                 : "memory");
}
LYTH_D float4 tx_lds(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a) : "memory");
    return v;
}
LYTH_D void tx_sts(uint32_t a, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
LYTH_D void team_sync(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(kTxTeamThreads) : "memory"); }
LYTH_D bool team_all(int id, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\t"
        "setp.ne.u32 a, %1, 0;\n\t"
        "bar.red.and.pred b, %2, %3, a;\n\t"
        "selp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "n"(kTxTeamThreads)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kTxTeams * kTxTeamThreads)
    transpose_tma_kernel(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout,
                         uint32_t rows, uint32_t cols) {
    extern __shared__ uint8_t tx_raw[];
    const uint32_t raw = smem_u32(tx_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // the 128-byte swizzle repeats every 1 KiB
    const int team = threadIdx.x / kTxTeamThreads, t = threadIdx.x % kTxTeamThreads;
    const int bar_id = 1 + team;
    const uint32_t in0 = base + (uint32_t)team * 3 * kTxTileBytes, out = in0 + 2 * kTxTileBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(tx_raw + (base - raw) + (size_t)kTxTeams * 3 * kTxTileBytes) + team * 2;
    const uint32_t tiles_x = (cols + 31) / 32, tiles_y = (rows + 31) / 32;
    const uint64_t tiles = (uint64_t)tiles_x * tiles_y;
    const uint64_t stride = (uint64_t)gridDim.x * kTxTeams;
    const uint64_t first = (uint64_t)blockIdx.x * kTxTeams + team;
    const uint64_t mine = tiles > first ? (tiles - first + stride - 1) / stride : 0;
    auto tile_of = [&](uint64_t k) { return first + k * stride; };
    auto load = [&](uint64_t k) {
        const uint64_t tl = tile_of(k);
        const uint32_t b = smem_u32(bars + (k & 1));
        mbar_expect_tx(b, kTxTileBytes);
        tensor_load_2d(in0 + (uint32_t)(k & 1) * kTxTileBytes, &tin, (int)((tl % tiles_x) * 32), (int)((tl / tiles_x) * 32),
                       b);
    };
    if (t == 0) {
        mbar_init(smem_u32(bars), 1);
        mbar_init(smem_u32(bars + 1), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (uint64_t k = 0; k < 2 && k < mine; k++) load(k);
    }
    team_sync(bar_id);
    const int p = t & 7, q = t >> 3;
    const int tc = p, tr = p ^ q;
    uint64_t armed = mine < 2 ? mine : 2, used = 0;
    for (uint64_t k = 0; k < mine; k++) {
        const bool ok = mbar_wait(smem_u32(bars + (k & 1)), (uint32_t)(k >> 1) & 1u, &g_tx_error);
        if (!team_all(bar_id, ok)) break;
        used++;
        const uint32_t in = in0 + (uint32_t)(k & 1) * kTxTileBytes;
        float4 v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t r = 4 * tr + i;
            v[i] = tx_lds(in + r * 128u + (uint32_t)((tc ^ (r & 7)) << 4));
        }
        if (t == 0) bulk_wait_read0();  // the previous tile's store has read the output buffer
        team_sync(bar_id);
        // every thread has read this stage: the leader may refill it with the tile two ahead
        if (t == 0 && k + 2 < mine) {
            load(k + 2);
            armed++;
        }
        const float4 o[4] = {make_float4(v[0].x, v[1].x, v[2].x, v[3].x), make_float4(v[0].y, v[1].y, v[2].y, v[3].y),
                             make_float4(v[0].z, v[1].z, v[2].z, v[3].z), make_float4(v[0].w, v[1].w, v[2].w, v[3].w)};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t r = 4 * tc + j;
            tx_sts(out + r * 128u + (uint32_t)((tr ^ (r & 7)) << 4), o[j]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        team_sync(bar_id);
        if (t == 0) {
            const uint64_t tl = tile_of(k);
            tensor_store_2d(&tout, (int)((tl / tiles_x) * 32), (int)((tl % tiles_x) * 32), out);
            bulk_commit();
        }
    }
    if (t == 0) {
        bulk_wait0();
        // after a timed-out wait, a load may still be in flight: wait for it (bounded)
        for (uint64_t k = used; k < armed; k++) mbar_wait(smem_u32(bars + (k & 1)), (uint32_t)(k >> 1) & 1u, &g_tx_error);
    }
}

// The same for 16-bit elements (the narrow transpose): a 128-byte box row holds 64 elements, so
// a tile is 64 x 64 (8 KiB) and a thread moves an 8 x 8 block -- eight 128-bit loads of rows
// 8tr..8tr+7 at chunk tc, a transpose in registers (one PRMT per output word: word w of output
// row j takes element j of input rows 2w and 2w+1), eight 128-bit stores into output rows
// 8tc..8tc+7 at chunk tr. The swizzled chunk of row r is c ^ (r & 7) and r & 7 is the block's own
// row index, so with (tr, tc) = (p ^ q, p) every quarter-warp again reaches 8 distinct chunks.
constexpr uint32_t kTx16TileBytes = 64 * 64 * 2;
constexpr size_t kTx16Smem = 1024 + (size_t)kTxTeams * 3 * kTx16TileBytes + kTxTeams * 2 * sizeof(uint64_t);

__global__ void __launch_bounds__(kTxTeams * kTxTeamThreads)
    transpose_tma16_kernel(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout,
                           uint32_t rows, uint32_t cols) {
    extern __shared__ uint8_t tx_raw[];
    const uint32_t raw = smem_u32(tx_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // the 128-byte swizzle repeats every 1 KiB
    const int team = threadIdx.x / kTxTeamThreads, t = threadIdx.x % kTxTeamThreads;
    const int bar_id = 1 + team;
    const uint32_t in0 = base + (uint32_t)team * 3 * kTx16TileBytes, out = in0 + 2 * kTx16TileBytes;
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(tx_raw + (base - raw) + (size_t)kTxTeams * 3 * kTx16TileBytes) + team * 2;
    const uint32_t tiles_x = (cols + 63) / 64, tiles_y = (rows + 63) / 64;
    const uint64_t tiles = (uint64_t)tiles_x * tiles_y;
    const uint64_t stride = (uint64_t)gridDim.x * kTxTeams;
    const uint64_t first = (uint64_t)blockIdx.x * kTxTeams + team;
    const uint64_t mine = tiles > first ? (tiles - first + stride - 1) / stride : 0;
    auto tile_of = [&](uint64_t k) { return first + k * stride; };
    auto load = [&](uint64_t k) {
        const uint64_t tl = tile_of(k);
        const uint32_t b = smem_u32(bars + (k & 1));
        mbar_expect_tx(b, kTx16TileBytes);
        tensor_load_2d(in0 + (uint32_t)(k & 1) * kTx16TileBytes, &tin, (int)((tl % tiles_x) * 64),
                       (int)((tl / tiles_x) * 64), b);
    };
    if (t == 0) {
        mbar_init(smem_u32(bars), 1);
        mbar_init(smem_u32(bars + 1), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (uint64_t k = 0; k < 2 && k < mine; k++) load(k);
    }
    team_sync(bar_id);
    const int p = t & 7, q = t >> 3;
    const int tc = p, tr = p ^ q;
    uint64_t armed = mine < 2 ? mine : 2, used = 0;
    for (uint64_t k = 0; k < mine; k++) {
        const bool ok = mbar_wait(smem_u32(bars + (k & 1)), (uint32_t)(k >> 1) & 1u, &g_tx_error);
        if (!team_all(bar_id, ok)) break;
        used++;
        const uint32_t in = in0 + (uint32_t)(k & 1) * kTx16TileBytes;
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t r = 8 * tr + i;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v[i].x), "=r"(v[i].y), "=r"(v[i].z), "=r"(v[i].w)
                         : "r"(in + r * 128u + (uint32_t)((tc ^ i) << 4))
                         : "memory");
        }
        if (t == 0) bulk_wait_read0();  // the previous tile's store has read the output buffer
        team_sync(bar_id);
        // every thread has read this stage: the leader may refill it with the tile two ahead
        if (t == 0 && k + 2 < mine) {
            load(k + 2);
            armed++;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const uint32_t *a = reinterpret_cast<const uint32_t *>(&v[2 * h]);
                const uint32_t *b = reinterpret_cast<const uint32_t *>(&v[2 * h + 1]);
                uint32_t d;
                asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a[j >> 1]), "r"(b[j >> 1]), "r"((j & 1) ? 0x7632u : 0x5410u));
                w[h] = d;
            }
            const uint32_t r = 8 * tc + j;
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(out + r * 128u + (uint32_t)((tr ^ j) << 4)),
                         "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                         : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        team_sync(bar_id);
        if (t == 0) {
            const uint64_t tl = tile_of(k);
            tensor_store_2d(&tout, (int)((tl / tiles_x) * 64), (int)((tl % tiles_x) * 64), out);
            bulk_commit();
        }
    }
    if (t == 0) {
        bulk_wait0();
        // after a timed-out wait, a load may still be in flight: wait for it (bounded)
        for (uint64_t k = used; k < armed; k++) mbar_wait(smem_u32(bars + (k & 1)), (uint32_t)(k >> 1) & 1u, &g_tx_error);
    }
}

// ------------------------------------------------------------------ narrow storage (ADR-0024)
// f16 / bf16 buffers, f32 arithmetic: each element is widened exactly on load, the body runs the
// same f32 chain as the f32 kernel, and each drained value is rounded once, to nearest even, at
// the store (cvt.rn: eval.rs:557-570's round_narrow_outputs). 128-bit vectors carry 8 elements.
template <int TY>
LYTH_D float widen(uint16_t h) {
    return TY == 1 ? __half2float(__ushort_as_half(h)) : __uint_as_float((uint32_t)h << 16);
}
template <int TY>
LYTH_D uint16_t narrow(float f) {
    return TY == 1 ? __half_as_ushort(__float2half_rn(f)) : __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
template <int TY, typename F>
LYTH_D uint32_t pair(const F &f, uint32_t x, uint32_t y) {
    const uint16_t lo = narrow<TY>(f(widen<TY>((uint16_t)(x & 0xffffu)), widen<TY>((uint16_t)(y & 0xffffu))));
    const uint16_t hi = narrow<TY>(f(widen<TY>((uint16_t)(x >> 16)), widen<TY>((uint16_t)(y >> 16))));
    return (uint32_t)lo | ((uint32_t)hi << 16);
}

template <int TY, bool TWO_IN, typename F>
__global__ void __launch_bounds__(256) stream_narrow_kernel(uint64_t n, F f, const uint16_t *x, const uint16_t *y,
                                                            uint16_t *out) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const bool vec = ((((uintptr_t)x) | ((uintptr_t)out) | (TWO_IN ? (uintptr_t)y : 0)) & 15u) == 0;
    if (vec) {
        const uint64_t nv = n >> 3;  // 8 elements per 16-byte vector
        for (uint64_t v = tid; v < nv; v += nthreads) {
            const uint4 xv = *reinterpret_cast<const uint4 *>(x + 8 * v);
            const uint4 yv = TWO_IN ? *reinterpret_cast<const uint4 *>(y + 8 * v) : make_uint4(0, 0, 0, 0);
            uint4 o;
            o.x = pair<TY>(f, xv.x, yv.x);
            o.y = pair<TY>(f, xv.y, yv.y);
            o.z = pair<TY>(f, xv.z, yv.z);
            o.w = pair<TY>(f, xv.w, yv.w);
            *reinterpret_cast<uint4 *>(out + 8 * v) = o;
        }
        for (uint64_t i = (nv << 3) + tid; i < n; i += nthreads)
            out[i] = narrow<TY>(f(widen<TY>(x[i]), TWO_IN ? widen<TY>(y[i]) : 0.f));
    } else {
        for (uint64_t i = tid; i < n; i += nthreads)
            out[i] = narrow<TY>(f(widen<TY>(x[i]), TWO_IN ? widen<TY>(y[i]) : 0.f));
    }
}

// The transpose of 2-byte elements (either narrow type: a transpose moves bits): 32 x 32 tiles in
// shared memory with a 34-element row (17 words, coprime with the 32 banks: the derived skew for
// 2-byte elements), 8 rows per warp pass.
__global__ void __launch_bounds__(256) transpose_u16_kernel(uint32_t rows, uint32_t cols, const uint16_t *a,
                                                            uint16_t *b) {
    __shared__ uint16_t tile[32 * 34];
    const uint32_t tiles_x = (cols + 31) / 32, tiles_y = (rows + 31) / 32;
    const uint64_t tiles = (uint64_t)tiles_x * tiles_y;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const uint32_t r0 = (uint32_t)(t / tiles_x) * 32, c0 = (uint32_t)(t % tiles_x) * 32;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t r = r0 + ty + 8 * k, c = c0 + tx;
            tile[(ty + 8 * k) * 34 + tx] = (r < rows && c < cols) ? a[(uint64_t)r * cols + c] : (uint16_t)0;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t oc = ty + 8 * k;  // output row c0 + oc, output column r0 + tx
            const uint32_t c = c0 + oc, r = r0 + tx;
            if (c < cols && r < rows) b[(uint64_t)c * rows + r] = tile[tx * 34 + oc];
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
namespace {
// The tensor maps of the TMA transpose: a (rows x cols, row-major) and b (cols x rows), 32 x 32
// boxes, 128-byte swizzle. False when the shape or the buffers do not allow one.
bool transpose_maps(uint32_t rows, uint32_t cols, const float *a, float *b, CUtensorMap &ta, CUtensorMap &tb) {
    if ((rows & 3u) || (cols & 3u) || !aligned16(a) || !aligned16(b)) return false;
    PFN_encode_tiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint32_t box[2] = {32, 32}, estr[2] = {1, 1};
    const cuuint64_t da[2] = {cols, rows}, sa[1] = {(cuuint64_t)cols * sizeof(float)};
    const cuuint64_t db[2] = {rows, cols}, sb[1] = {(cuuint64_t)rows * sizeof(float)};
    memset(&ta, 0, sizeof ta);
    memset(&tb, 0, sizeof tb);
    return enc(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(a), da, sa, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
           enc(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, b, db, sb, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
               CUDA_SUCCESS;
}
}  // namespace

namespace lyth {
int transpose_take_device_error() {
    int v = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&v, g_tx_error, sizeof(int));
    if (e != cudaSuccess) return status_of(e);
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_tx_error, &zero, sizeof(int));
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}
}  // namespace lyth

extern "C" int lyth_b200_transpose_tiled(uint32_t rows, uint32_t cols, const float *a, float *b, cudaStream_t s) {
    if ((uint64_t)rows * cols == 0) return LYTH_OK;
    if (!a || !b) return LYTH_E_INVALID;
    CUtensorMap ta, tb;
    if (transpose_maps(rows, cols, a, b, ta, tb)) {
        static bool attr_done[64] = {false};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return LYTH_E_INVALID;
        if (dev >= 0 && dev < 64 && !attr_done[dev]) {
            const cudaError_t e =
                cudaFuncSetAttribute(transpose_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTxSmem);
            if (e != cudaSuccess) return status_of(e);
            attr_done[dev] = true;
        }
        const uint64_t tiles = (uint64_t)((rows + 31) / 32) * ((cols + 31) / 32);
        uint64_t grid = (tiles + kTxTeams - 1) / kTxTeams;
        const uint64_t cap = (uint64_t)device_sms() * 4;  // four CTAs (16 teams) per SM
        if (grid > cap) grid = cap;
        transpose_tma_kernel<<<(unsigned)grid, kTxTeams * kTxTeamThreads, kTxSmem, s>>>(ta, tb, rows, cols);
        return last_launch_status();
    }
    const uint64_t tiles = (uint64_t)((rows + kTile - 1) / kTile) * ((cols + kTile - 1) / kTile);
    const unsigned grid = (unsigned)(tiles < 0x7fffffffull ? tiles : 0x7fffffffull);
    transpose_tiled_kernel<uint32_t><<<grid, 256, 0, s>>>(rows, cols, a, b);
    return last_launch_status();
}

// ------------------------------------------------------------------ narrow storage surface
namespace {
template <int TY>
int launch_stream_narrow(int op, uint64_t n, const float *c, const uint16_t *x, const uint16_t *y, uint16_t *out,
                         cudaStream_t s) {
    const unsigned grid = stream_grid((n + 7) / 8, kStreamBlock);
    switch (op) {
        case LYTH_STREAM_SAXPY: stream_narrow_kernel<TY, true><<<grid, kStreamBlock, 0, s>>>(n, SaxpyBody{c[0]}, x, y, out); break;
        case LYTH_STREAM_AXPBY: stream_narrow_kernel<TY, true><<<grid, kStreamBlock, 0, s>>>(n, AxpbyBody{c[0], c[1]}, x, y, out); break;
        case LYTH_STREAM_LERP: stream_narrow_kernel<TY, true><<<grid, kStreamBlock, 0, s>>>(n, LerpBody{c[0]}, x, y, out); break;
        case LYTH_STREAM_HORNER:
            stream_narrow_kernel<TY, false><<<grid, kStreamBlock, 0, s>>>(n, HornerBody{c[0], c[1], c[2], c[3]}, x, y, out);
            break;
        case LYTH_STREAM_COPY: stream_narrow_kernel<TY, false><<<grid, kStreamBlock, 0, s>>>(n, CopyBody{}, x, y, out); break;
        default: return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}
}  // namespace

extern "C" int lyth_b200_stream_narrow(int op, int ty, uint64_t n, const float *scalars, const uint16_t *x,
                                       const uint16_t *y, uint16_t *out, cudaStream_t s) {
    if (n == 0) return LYTH_OK;
    const bool two_in = op == LYTH_STREAM_SAXPY || op == LYTH_STREAM_AXPBY || op == LYTH_STREAM_LERP;
    if (!x || !out || (two_in && !y) || (op != LYTH_STREAM_COPY && !scalars)) return LYTH_E_INVALID;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    const int nc = op == LYTH_STREAM_HORNER ? 4 : (op == LYTH_STREAM_AXPBY ? 2 : (op == LYTH_STREAM_COPY ? 0 : 1));
    for (int i = 0; i < nc; i++) c[i] = scalars[i];
    if (ty == LYTH_NARROW_F16) return launch_stream_narrow<1>(op, n, c, x, y, out, s);
    if (ty == LYTH_NARROW_BF16) return launch_stream_narrow<2>(op, n, c, x, y, out, s);
    return LYTH_E_UNSUPPORTED;
}

extern "C" int lyth_b200_transpose_narrow(int ty, uint32_t rows, uint32_t cols, const uint16_t *a, uint16_t *b,
                                          cudaStream_t s) {
    if (ty != LYTH_NARROW_F16 && ty != LYTH_NARROW_BF16) return LYTH_E_UNSUPPORTED;
    if ((uint64_t)rows * cols == 0) return LYTH_OK;
    if (!a || !b) return LYTH_E_INVALID;
    // 16-byte row pitches (rows and cols multiples of 8) and aligned buffers: the TMA tiles
    PFN_encode_tiled enc = tensor_map_encoder();
    if (!(rows & 7u) && !(cols & 7u) && aligned16(a) && aligned16(b) && enc) {
        const cuuint32_t box[2] = {64, 64}, estr[2] = {1, 1};
        const cuuint64_t da[2] = {cols, rows}, sa[1] = {(cuuint64_t)cols * 2};
        const cuuint64_t db[2] = {rows, cols}, sb[1] = {(cuuint64_t)rows * 2};
        CUtensorMap ta, tb;
        memset(&ta, 0, sizeof ta);
        memset(&tb, 0, sizeof tb);
        if (enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t *>(a), da, sa, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
            enc(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, b, db, sb, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            static bool attr_done[64] = {false};
            int dev = 0;
            if (cudaGetDevice(&dev) != cudaSuccess) return LYTH_E_INVALID;
            if (dev >= 0 && dev < 64 && !attr_done[dev]) {
                const cudaError_t e = cudaFuncSetAttribute(transpose_tma16_kernel,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTx16Smem);
                if (e != cudaSuccess) return status_of(e);
                attr_done[dev] = true;
            }
            const uint64_t tiles = (uint64_t)((rows + 63) / 64) * ((cols + 63) / 64);
            uint64_t grid = (tiles + kTxTeams - 1) / kTxTeams;
            const uint64_t cap = (uint64_t)device_sms() * 2;  // two CTAs (8 teams) per SM
            if (grid > cap) grid = cap;
            transpose_tma16_kernel<<<(unsigned)grid, kTxTeams * kTxTeamThreads, kTx16Smem, s>>>(ta, tb, rows, cols);
            return last_launch_status();
        }
    }
    const uint64_t tiles = (uint64_t)((rows + 31) / 32) * ((cols + 31) / 32);
    uint64_t grid = tiles;
    const uint64_t cap = (uint64_t)device_sms() * 8;
    if (grid > cap) grid = cap;
    transpose_u16_kernel<<<(unsigned)grid, 256, 0, s>>>(rows, cols, a, b);
    return last_launch_status();
}
