// The f32 contraction C = A * B (examples/matmul.lyth, matmul-coarse.lyth) for sm_100a, on
// the FP32 pipe.
//
// The reference stages square tiles in skewed shared memory and gives each thread ci x cj
// accumulators (crates/lyth-ptx/src/contracted.rs:177-663), walking p in ascending order with
// an unfused mul.rn + add.rn (contracted.rs:23-26). Here a 256-thread block owns a 128 x 128
// tile of C and each thread an 8 x 8 register tile (two 4-row by two 4-column quarters, so the
// shared-memory reads of a warp are broadcasts and 128-bit vectors), K moves in steps of 16
// with the next step's operands prefetched into registers while this step's are used. A is
// stored transposed (and XOR-swizzled, see sgemm_tile) in shared memory so both operands are read
// as vectors along the tile.
//
// EXACT = true keeps the reference's contract bit for bit: every output is its own
// accumulator, p strictly ascending, product rounded, then sum rounded. EXACT = false uses
// the fused multiply-add (one rounding per step; within 1e-5 relative of the reference).
#include "common.cuh"

namespace lyth {

constexpr int kBM = 128, kBN = 128, kBK = 16;

template <bool EXACT>
LYTH_D float mac(float acc, float a, float b) {
    if (EXACT) return __fadd_rn(acc, __fmul_rn(a, b));
    return __fmaf_rn(a, b, acc);
}

// One 128 x 128 tile of C at (bm, bn). Needs m % 128 == 0, n % 128 == 0, k % 16 == 0 and
// 16-byte aligned rows.
template <bool EXACT>
LYTH_D void sgemm_tile(uint32_t n, uint32_t k, const float *a, const float *b, float *c, uint32_t bm, uint32_t bn,
                       float (*As)[kBK][kBM], float (*Bs)[kBK][kBN]) {
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;

    // Global -> register staging: A tile 128 x 16 (two float4 per thread along k),
    // B tile 16 x 128 (two float4 per thread along n).
    const int a_row = tid >> 2, a_col = (tid & 3) * 4;          // rows 0..63 (+64), k 0..15
    const int b_row = tid >> 5, b_col = (tid & 31) * 4;         // k rows 0..7 (+8), n 0..127
    const float *ap0 = a + (uint64_t)(bm + a_row) * k + a_col;
    const float *ap1 = ap0 + (uint64_t)64 * k;
    const float *bp0 = b + (uint64_t)b_row * n + bn + b_col;
    const float *bp1 = bp0 + (uint64_t)8 * n;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    float4 ra0 = ld4(ap0), ra1 = ld4(ap1), rb0 = ld4(bp0), rb1 = ld4(bp1);
    // A is stored transposed with its rows XOR'ed by sw(p) = 8 * ((p >> 2) & 3): the 8 rows and
    // 4 k-groups a warp stores then land in 32 distinct banks (unswizzled, the 4 k-groups of a
    // row share a bank), and a 4-row group stays contiguous for the 128-bit reads below.
    const int sw = 8 * ((a_col >> 2) & 3);
    auto stage = [&](int buf) {
        As[buf][a_col + 0][a_row ^ sw] = ra0.x; As[buf][a_col + 1][a_row ^ sw] = ra0.y;
        As[buf][a_col + 2][a_row ^ sw] = ra0.z; As[buf][a_col + 3][a_row ^ sw] = ra0.w;
        As[buf][a_col + 0][(a_row + 64) ^ sw] = ra1.x; As[buf][a_col + 1][(a_row + 64) ^ sw] = ra1.y;
        As[buf][a_col + 2][(a_row + 64) ^ sw] = ra1.z; As[buf][a_col + 3][(a_row + 64) ^ sw] = ra1.w;
        *reinterpret_cast<float4 *>(&Bs[buf][b_row][b_col]) = rb0;
        *reinterpret_cast<float4 *>(&Bs[buf][b_row + 8][b_col]) = rb1;
    };
    stage(0);
    __syncthreads();

    const uint32_t ktiles = k / kBK;
    for (uint32_t kt = 0; kt < ktiles; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) {
            const uint64_t off = (uint64_t)(kt + 1) * kBK;
            ra0 = ld4(ap0 + off); ra1 = ld4(ap1 + off);
            rb0 = ld4(bp0 + off * n); rb1 = ld4(bp1 + off * n);
        }
#pragma unroll
        for (int p = 0; p < kBK; p++) {
            const int swp = 8 * ((p >> 2) & 3);
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][p][(ty * 4) ^ swp]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][p][(64 + ty * 4) ^ swp]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][p][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][p][64 + tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = mac<EXACT>(acc[i][j], av[i], bv[j]);
        }
        if (kt + 1 < ktiles) {
            stage(buf ^ 1);
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t row = bm + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        float *crow = c + (uint64_t)row * n + bn;
        *reinterpret_cast<float4 *>(crow + tx * 4) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        *reinterpret_cast<float4 *>(crow + 64 + tx * 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
    }
}

LYTH_D bool tiles_fit(uint32_t m, uint32_t n, uint32_t k, const float *a, const float *b, const float *c) {
    return (m % kBM == 0) && (n % kBN == 0) && (k % kBK == 0) && k > 0 &&
           ((((uintptr_t)a) | ((uintptr_t)b) | ((uintptr_t)c)) & 15u) == 0;
}

// One block per tile of C, grid-stride over tiles (row-major tile order). Two blocks per SM (128
// registers a thread: a few bytes of the next step's prefetch spill once per K step), so one
// block's shared-memory waits overlap the other's FMAs.
template <bool EXACT>
__global__ void __launch_bounds__(256, 2) sgemm_tiled_kernel(uint32_t m, uint32_t n, uint32_t k, const float *a,
                                                          const float *b, float *c) {
    __shared__ __align__(16) float As[2][kBK][kBM];
    __shared__ __align__(16) float Bs[2][kBK][kBN];
    const uint32_t tiles_n = n / kBN, tiles = tiles_n * (m / kBM);
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        sgemm_tile<EXACT>(n, k, a, b, c, (t / tiles_n) * kBM, (t % tiles_n) * kBN, As, Bs);
        __syncthreads();
    }
}

// Any shape: one output per thread, p ascending. Used for ragged sizes and as the ADR-0016
// kernel's fallback inside the same launch shape.
template <bool EXACT>
__global__ void __launch_bounds__(256) sgemm_general_kernel(uint32_t m, uint32_t n, uint32_t k, const float *a,
                                                            const float *b, float *c) {
    const uint64_t total = (uint64_t)m * n;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = e / n, j = e % n;
        float acc = 0.0f;
        for (uint32_t p = 0; p < k; p++) acc = mac<EXACT>(acc, a[i * k + p], b[(uint64_t)p * n + j]);
        c[e] = acc;
    }
}

// The ADR-0016 kernel (reference parameter order m, n, k, a, b, c), exact, any shape, one
// block per 128 x 128 tile of C (the Tiled grid rule). Aligned shapes run the tiled body;
// any other shape computes each output of the tile with the general walk.
__global__ void __launch_bounds__(256) matmul_kernel(uint32_t m, uint32_t n, uint32_t k, const float *a,
                                                     const float *b, float *c) {
    __shared__ __align__(16) float As[2][kBK][kBM];
    __shared__ __align__(16) float Bs[2][kBK][kBN];
    const uint32_t tiles_n = (n + kBN - 1) / kBN;
    const uint32_t tiles = tiles_n * ((m + kBM - 1) / kBM);
    const bool fit = tiles_fit(m, n, k, a, b, c);
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const uint32_t tm = t / tiles_n, tn = t % tiles_n;
        if (fit) {
            sgemm_tile<true>(n, k, a, b, c, tm * kBM, tn * kBN, As, Bs);
            __syncthreads();
            continue;
        }
        for (uint32_t e = threadIdx.x; e < (uint32_t)(kBM * kBN); e += blockDim.x) {
            const uint32_t i = tm * kBM + e / kBN, j = tn * kBN + e % kBN;
            if (i >= m || j >= n) continue;
            float acc = 0.0f;
            for (uint32_t p = 0; p < k; p++) acc = mac<true>(acc, a[(uint64_t)i * k + p], b[(uint64_t)p * n + j]);
            c[(uint64_t)i * n + j] = acc;
        }
    }
}

}  // namespace lyth

using namespace lyth;

extern "C" int lyth_b200_matmul_f32(uint32_t m, uint32_t n, uint32_t k, const float *a, const float *b, float *c,
                                    int exact, cudaStream_t s) {
    if (!a || !b || !c) return LYTH_E_INVALID;
    if ((uint64_t)m * n == 0) return LYTH_OK;
    const bool tiled = (m % kBM == 0) && (n % kBN == 0) && (k % kBK == 0) && k > 0 &&
                       ((((uintptr_t)a) | ((uintptr_t)b) | ((uintptr_t)c)) & 15u) == 0;
    if (tiled) {
        const unsigned grid = (n / kBN) * (m / kBM);
        if (exact) sgemm_tiled_kernel<true><<<grid, 256, 0, s>>>(m, n, k, a, b, c);
        else sgemm_tiled_kernel<false><<<grid, 256, 0, s>>>(m, n, k, a, b, c);
    } else {
        const unsigned grid = stream_grid((uint64_t)m * n, 256);
        if (exact) sgemm_general_kernel<true><<<grid, 256, 0, s>>>(m, n, k, a, b, c);
        else sgemm_general_kernel<false><<<grid, 256, 0, s>>>(m, n, k, a, b, c);
    }
    return last_launch_status();
}
