// gate_proj GEMV for sm_100a: y = W x with W in 4-bit INT4 or NF4, fp16 per-group scales,
// fp16 activations, f32 accumulation, fp16 output.
//
// The reference has no kernel for this class: only cost contracts
// (fixtures/kernel/gate_proj_int4.json, fixtures/poly/gate-proj-int4-nf4.json: 0.5 B of
// weight per element, a scale per group, 2 flops per weight). The format is this project's:
// row r of W is contiguous along k, byte (r*k + c) / 2, low nibble = even c; INT4 nibbles are
// two's complement (-8..7); NF4 nibbles index the 16-level normal-float codebook of QLoRA.
//
// Decode (one function, `decode_word`, used by the GEMV and by the dequantisation entry point, so
// the dequantised matrix the tests compare bit for bit is what the GEMV multiplies): a 32-bit word
// holds 8 weights; its even and odd nibbles are split into bytes, and one PRMT per weight builds
// INT4: the float whose bits are 0x3F00_0000 | v << 16 with v = q + 8 (the word xor 0x88888888),
// i.e. f = 0.5 + v/256 = 17/32 + q/256 exactly; NF4: the nibble as an index into a 16-entry
// shared table of the codebook. The INT4 GEMV accumulates f x and corrects each 32-weight chunk
// once: sum q x = 256 (sum f x - 17/32 sum x), with sum x per chunk precomputed per block (x is
// shared by every row; the cancellation costs ~5 of f32's 24 bits, far inside the 1e-3 output
// tolerance). The dequantisation reads q back as (f - 17/32) * 256 (both steps exact) and
// multiplies by the scale: q * scale, the format's definition, bit for bit.
//
// Kernel (the ring kernel, `gemv_ring_kernel`): one persistent block per SM owns a contiguous range
// of rows, so its weights and scales are one contiguous range of memory each. A producer warp
// streams them through a ring of shared-memory stages with 1-D bulk copies (cp.async.bulk, 8 rows
// of W and their scales per stage, completion on an mbarrier, no multicast), issuing the first
// stages before anything else so the weights are in flight while the 16 consumer warps stage x.
// Consumers take alternate stages in two groups of 8 warps, a warp per row: a lane owns 32-weight
// chunks (16 bytes, conflict-free 128-bit shared loads), multiplies pairs of weights at once with
// fma.rn.f32x2 (two independent IEEE fmas: the scalar chain's rounding), and the row's partials
// combine with shuffles; the row is rounded once to fp16. x is staged once per block in shared
// memory as f32, one 32-value chunk per row of 36 floats (the pad keeps 128-bit reads
// conflict-free). Every wait is bounded (mbar.cuh); a wait that runs out sets the device error
// flag read by lyth_b200_device_error and the block winds down. Shapes the ring does not take
// (scales not 16-byte aligned per stage) run the row kernel: the same decode, one warp per row,
// weights loaded straight from global memory.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "mbar.cuh"

namespace lyth {

__constant__ float c_nf4[16];
__device__ int g_gemv_error;

LYTH_D float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

LYTH_D uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// The 8 weights of one 32-bit word of W, in element order (f[j] from nibble j). INT4:
// f = 0.5 + (q + 8)/256; NF4: the codebook level (lut = the 16-entry table).
template <int FMT>
LYTH_D void decode_word(uint32_t w, const float *lut, float (&f)[8]) {
    if (FMT == 0) w ^= 0x88888888u;                  // v = q + 8 in every nibble
    const uint32_t lo = w & 0x0F0F0F0Fu;             // nibbles 0, 2, 4, 6 as bytes
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;      // nibbles 1, 3, 5, 7 as bytes
#pragma unroll
    for (int b = 0; b < 4; b++) {
        if (FMT == 0) {
            // bytes [0, 0, v, 0x3F] -> bits 0x3F00_0000 | v << 16 -> 0.5 + v / 256
            f[2 * b] = __uint_as_float(prmt(lo, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
            f[2 * b + 1] = __uint_as_float(prmt(hi, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
        } else {
            f[2 * b] = lut[prmt(lo, 0u, 0x4440u | (uint32_t)b)];
            f[2 * b + 1] = lut[prmt(hi, 0u, 0x4440u | (uint32_t)b)];
        }
    }
}

LYTH_D uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
LYTH_D uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// One 16-byte chunk (32 weights) against its 32 staged x values: INT4 returns sum f x (the caller
// corrects), NF4 sum code[v] x. Four partial sums -- even and odd weights (the two lanes of one
// packed fma) of words 0, 2 and of words 1, 3 (two independent fma chains) -- added at the end.
template <int FMT>
LYTH_D float chunk_dot(uint4 v, const float *xr, const float *lut) {
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
    uint64_t acc[2] = {0, 0};  // words 0, 2 and 1, 3: (even, odd) weights each, from (+0, +0)
#pragma unroll
    for (int q = 0; q < 4; q++) {
        float f[8];
        decode_word<FMT>(words[q], lut, f);
        const float4 xa = *reinterpret_cast<const float4 *>(xr + 8 * q);
        const float4 xb = *reinterpret_cast<const float4 *>(xr + 8 * q + 4);
        uint64_t &a = acc[q & 1];
        a = fma2(pk2(f[0], f[1]), pk2(xa.x, xa.y), a);
        a = fma2(pk2(f[2], f[3]), pk2(xa.z, xa.w), a);
        a = fma2(pk2(f[4], f[5]), pk2(xb.x, xb.y), a);
        a = fma2(pk2(f[6], f[7]), pk2(xb.z, xb.w), a);
    }
    float e0, o0, e1, o1;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(e0), "=f"(o0) : "l"(acc[0]));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(e1), "=f"(o1) : "l"(acc[1]));
    return __fadd_rn(__fadd_rn(e0, o0), __fadd_rn(e1, o1));
}

constexpr int kGemvRowStride = 36;  // floats per staged 32-value chunk (pad 4: conflict-free LDS.128)

// Stage x (fp16, k values) as f32 chunks of 36 floats and, for INT4, each chunk's sum (the
// correction term): each thread moves 8 values (one 16-byte load) per step; four consecutive
// threads cover one chunk and combine their sums with two shuffles. nthr threads take part,
// in whole warps.
template <int FMT>
LYTH_D void stage_x(uint32_t k, const uint16_t *x, float *xs, float *xsum, uint32_t tid, uint32_t nthr) {
    const uint4 *x16 = reinterpret_cast<const uint4 *>(x);
    const uint32_t nvec = k >> 3;
    for (uint32_t v0 = 0; v0 < nvec; v0 += 4 * nthr) {
        uint4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t v = v0 + u * nthr + tid;
            if (v < nvec) raw[u] = x16[v];
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t v = v0 + u * nthr + tid;
            float part = 0.0f;
            if (v < nvec) {
                const uint32_t hw[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
                float *dst = xs + (v >> 2) * kGemvRowStride + (v & 3) * 8;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hw[e]));
                    dst[2 * e] = f.x;
                    dst[2 * e + 1] = f.y;
                    part = __fadd_rn(part, __fadd_rn(f.x, f.y));
                }
            }
            // Whole warps take part in the shuffles; v < nvec is uniform per 4-lane group.
            part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 1));
            part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 2));
            if (FMT == 0 && v < nvec && (v & 3) == 0) xsum[v >> 2] = part;
        }
    }
}

// A warp's row: lane owns chunks lane + 32 s; w16 = the row's 16-byte weight words (shared or
// global memory), srow = its fp16 scales. Returns the row's sum in every lane.
template <int FMT, bool SHARED_W>
LYTH_D float row_dot(uint32_t k, uint32_t group, const uint4 *w16, const uint16_t *srow, const float *xs,
                     const float *xsum, const float *lut, int lane) {
    // the chunk's scale: chunk * 32 / group, a shift when the group is a power of two (a division
    // by a run-time divisor costs a reciprocal and conversions per chunk otherwise)
    const bool pow2 = (group & (group - 1)) == 0;
    const uint32_t gshift = pow2 ? (uint32_t)__ffs(group >> 5) - 1u : 0u;
    const uint32_t steps = k >> 10;  // 32 chunks (one per lane) per warp-step
    float acc = 0.0f;
    for (uint32_t s0 = 0; s0 < steps; s0 += 4) {
        uint4 v[4];
        float sc[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (s0 + u < steps) {
                const uint32_t chunk = lane + 32 * (s0 + u);
                if (SHARED_W) {
                    v[u] = w16[chunk];
                } else {
                    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                                 : "l"(w16 + chunk));
                }
                sc[u] = half_bits_to_float(srow[pow2 ? (chunk >> gshift) : (chunk * 32) / group]);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (s0 + u < steps) {
                const uint32_t chunk = lane + 32 * (s0 + u);
                float part = chunk_dot<FMT>(v[u], xs + chunk * kGemvRowStride, lut);
                if (FMT == 0) part = __fmul_rn(256.0f, __fmaf_rn(-0.53125f, xsum[chunk], part));
                acc = __fmaf_rn(sc[u], part, acc);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    return acc;
}

// ---- the ring kernel
constexpr int kGvRowsPerStage = 8;                 // rows per stage = warps per consumer group
constexpr int kGvGroups = 2;                       // consumer groups, alternate stages
constexpr int kGvConsumers = kGvGroups * kGvRowsPerStage;
constexpr int kGvThreads = (kGvConsumers + 1) * 32;  // + one producer warp
constexpr int kGvMaxStages = 16;

struct GvArgs {
    uint32_t rows, k, group, stages;   // stages: ring depth (even)
    uint32_t w_stage_bytes, s_stage_bytes;
    const uint8_t *w;
    const uint16_t *scales;
    const uint16_t *x;
    uint16_t *y;
};

template <int FMT>
__global__ void __launch_bounds__(kGvThreads, 1) gemv_ring_kernel(const __grid_constant__ GvArgs a) {
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const uint32_t S = a.stages;
    const uint32_t groups = a.k / a.group;
    uint8_t *ring = gv_smem;                                            // S x (W stage, scale stage)
    const uint32_t stage_bytes = a.w_stage_bytes + a.s_stage_bytes;
    float *xs = reinterpret_cast<float *>(ring + (size_t)S * stage_bytes);
    float *xsum = xs + (a.k >> 5) * kGemvRowStride;
    float *lut = xsum + (a.k >> 5);
    uint64_t *full = reinterpret_cast<uint64_t *>(lut + 16);           // 8-byte aligned: see host
    uint64_t *empty = full + kGvMaxStages;
    uint32_t *n_armed = reinterpret_cast<uint32_t *>(empty + kGvMaxStages);
    uint32_t *n_used = n_armed + kGvMaxStages;

    const uint32_t r0 = (uint32_t)(((uint64_t)a.rows * blockIdx.x) / gridDim.x);
    const uint32_t r1 = (uint32_t)(((uint64_t)a.rows * (blockIdx.x + 1)) / gridDim.x);
    const uint32_t nst = (r1 - r0 + kGvRowsPerStage - 1) / kGvRowsPerStage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row_w = a.k >> 1;        // bytes of W per row
    const uint32_t row_s = groups * 2u;     // bytes of scales per row

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; s++) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), kGvRowsPerStage);
            n_armed[s] = 0;
            n_used[s] = 0;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kGvConsumers) {
        // producer: stage j (rows r0 + 8j ..) into slot j % S once its previous use is released
        if (lane == 0) {
            for (uint32_t j = 0; j < nst; j++) {
                const uint32_t slot = j % S, use = j / S;
                if (use > 0 && !mbar_wait(smem_u32(empty + slot), (use - 1) & 1u, &g_gemv_error)) break;
                const uint32_t rs = r0 + j * kGvRowsPerStage;
                const uint32_t nr = min((uint32_t)kGvRowsPerStage, r1 - rs);
                uint8_t *dst = ring + (size_t)slot * stage_bytes;
                const uint32_t wb = nr * row_w, sb = nr * row_s;
                mbar_expect_tx(smem_u32(full + slot), wb + sb);
                bulk_load(smem_u32(dst), a.w + (size_t)rs * row_w, wb, smem_u32(full + slot));
                bulk_load(smem_u32(dst + a.w_stage_bytes), a.scales + (size_t)rs * groups, sb, smem_u32(full + slot));
                n_armed[slot]++;
            }
        }
    } else {
        if (FMT == 1 && threadIdx.x < 16) lut[threadIdx.x] = c_nf4[threadIdx.x];
        stage_x<FMT>(a.k, a.x, xs, xsum, threadIdx.x, kGvConsumers * 32);
        asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");  // consumers only
        const int grp = warp / kGvRowsPerStage, wid = warp % kGvRowsPerStage;
        for (uint32_t j = grp; j < nst; j += kGvGroups) {
            const uint32_t slot = j % S;
            const bool ok = mbar_wait(smem_u32(full + slot), (j / S) & 1u, &g_gemv_error);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (wid == 0 && lane == 0) n_used[slot]++;
            const uint32_t r = r0 + j * kGvRowsPerStage + wid;
            if (r < r1) {
                const uint8_t *st = ring + (size_t)slot * stage_bytes;
                const float acc = row_dot<FMT, true>(
                    a.k, a.group, reinterpret_cast<const uint4 *>(st + (size_t)wid * row_w),
                    reinterpret_cast<const uint16_t *>(st + a.w_stage_bytes) + (size_t)wid * groups, xs, xsum, lut,
                    lane);
                if (lane == 0) a.y[r] = __half_as_ushort(__float2half_rn(acc));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(empty + slot));
        }
    }
    // Every armed stage has landed before the block may leave: after a timed-out wait one use
    // per slot may still be in flight (bounded wait for it).
    __syncthreads();
    if (threadIdx.x == 0)
        for (uint32_t s = 0; s < S; s++)
            if (n_armed[s] != n_used[s]) mbar_wait(smem_u32(full + s), (n_armed[s] - 1u) & 1u, &g_gemv_error);
}

// ---- the row kernel (shapes the ring does not take): one warp per row, weights from global.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_row_kernel(uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                                       const uint16_t *scales, const uint16_t *x, uint16_t *y) {
    extern __shared__ __align__(16) float smem[];
    const uint32_t chunks = k >> 5;
    float *xs = smem;
    float *xsum = smem + chunks * kGemvRowStride;
    float *lut = xsum + chunks;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    stage_x<FMT>(k, x, xs, xsum, threadIdx.x, blockDim.x);
    if (FMT == 1 && threadIdx.x < 16) lut[threadIdx.x] = c_nf4[threadIdx.x];
    __syncthreads();
    const uint32_t groups = k / group;
    for (uint32_t r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
        const float acc = row_dot<FMT, false>(k, group, reinterpret_cast<const uint4 *>(w + (uint64_t)r * (k >> 1)),
                                              scales + (uint64_t)r * groups, xs, xsum, lut, lane);
        if (lane == 0) y[r] = __half_as_ushort(__float2half_rn(acc));
    }
}

// The dequantised matrix through decode_word, one 32-bit word (8 weights) per thread-step:
// INT4 q = (f - 17/32) * 256 (exact), w = q * scale (exact); NF4 w = code * scale (one rounding).
template <int FMT>
__global__ void __launch_bounds__(256) gemv_dequant_kernel(uint32_t rows, uint32_t k, uint32_t group,
                                                           const uint8_t *w, const uint16_t *scales, float *out) {
    __shared__ float lut[16];
    if (FMT == 1 && threadIdx.x < 16) lut[threadIdx.x] = c_nf4[threadIdx.x];
    __syncthreads();
    const uint64_t nwords = (uint64_t)rows * k / 8;
    const uint32_t groups = k / group;
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(w);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t e = i * 8, r = e / k, c = e % k;  // 8 weights of one row (k % 8 == 0)
        const float s = half_bits_to_float(scales[r * groups + c / group]);  // group % 8 == 0
        float f[8];
        decode_word<FMT>(w32[i], lut, f);
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            o[j] = FMT == 0 ? __fmul_rn(__fmul_rn(__fsub_rn(f[j], 0.53125f), 256.0f), s) : __fmul_rn(f[j], s);
        float4 *dst = reinterpret_cast<float4 *>(out + e);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
}

// ---- the NF4 codebook, computed on the host (QLoRA, Dettmers et al. 2023): 8 positive
// normal quantiles on linspace(offset, 1/2, 9)[:-1], 7 negative ones on
// linspace(offset, 1/2, 8)[:-1], and an exact zero, normalised by the largest magnitude;
// offset = 0.9677083 as published. The inverse normal CDF is Acklam's rational approximation
// refined by two Halley steps on erfc.
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
    double xq;
    if (p < plow) {
        const double q = sqrt(-2 * log(p));
        xq = (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
             ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    } else if (p <= phigh) {
        const double q = p - 0.5, r = q * q;
        xq = (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
             (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1);
    } else {
        const double q = sqrt(-2 * log(1 - p));
        xq = -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
             ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    }
    for (int it = 0; it < 2; it++) {
        const double e = 0.5 * erfc(-xq / sqrt(2.0)) - p;
        const double u = e * sqrt(2 * 3.14159265358979323846) * exp(xq * xq / 2);
        xq = xq - u / (1 + xq * u / 2);
    }
    return xq;
}

static void nf4_levels(float out[16]) {
    const double offset = 0.9677083;
    double v[16];
    int n = 0;
    for (int i = 0; i < 8; i++) v[n++] = norm_ppf(offset + (0.5 - offset) * i / 8.0);
    v[n++] = 0.0;
    for (int i = 0; i < 7; i++) v[n++] = -norm_ppf(offset + (0.5 - offset) * i / 7.0);
    for (int i = 1; i < 16; i++) {
        const double t = v[i];
        int j = i - 1;
        while (j >= 0 && v[j] > t) { v[j + 1] = v[j]; j--; }
        v[j + 1] = t;
    }
    double mx = 0;
    for (int i = 0; i < 16; i++) mx = fabs(v[i]) > mx ? fabs(v[i]) : mx;
    for (int i = 0; i < 16; i++) out[i] = (float)(v[i] / mx);
}

// Uploads the codebook to the current device once per device.
static int ensure_nf4_on_device() {
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return status_of(e);
    if (dev >= 0 && dev < 64 && done[dev]) return LYTH_OK;
    float cb[16];
    nf4_levels(cb);
    e = cudaMemcpyToSymbol(c_nf4, cb, sizeof(cb));
    if (e != cudaSuccess) return status_of(e);
    if (dev >= 0 && dev < 64) done[dev] = true;
    return LYTH_OK;
}

}  // namespace lyth

using namespace lyth;

extern "C" void lyth_b200_nf4_codebook(float out[16]) { nf4_levels(out); }

// The ring's layout for this shape, or false when it does not take it.
static bool ring_layout(uint32_t k, uint32_t group, const uint16_t *scales, GvArgs &a, size_t &smem) {
    const uint32_t groups = k / group;
    const uint32_t row_s = groups * 2u;
    if ((row_s & 15u) || (((uintptr_t)scales) & 15u)) return false;  // 16-byte bulk-copy rule
    a.w_stage_bytes = kGvRowsPerStage * (k >> 1);
    a.s_stage_bytes = kGvRowsPerStage * row_s;
    const size_t fixed = ((size_t)(k >> 5) * (kGemvRowStride + 1) + 16) * sizeof(float) +
                         2 * kGvMaxStages * sizeof(uint64_t) + 2 * kGvMaxStages * sizeof(uint32_t);
    const size_t stage = (size_t)a.w_stage_bytes + a.s_stage_bytes;
    const size_t budget = 220 * 1024;
    if (fixed + 2 * stage > budget) return false;
    uint32_t S = (uint32_t)((budget - fixed) / stage);
    if (S > kGvMaxStages) S = kGvMaxStages;
    S &= ~1u;  // even: every use of a slot belongs to one consumer group
    a.stages = S;
    smem = (size_t)S * stage + fixed;
    return true;
}

template <int FMT>
static int launch_gemv(uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w, const uint16_t *scales,
                       const uint16_t *x, uint16_t *y, cudaStream_t s) {
    GvArgs a{};
    size_t smem = 0;
    if (ring_layout(k, group, scales, a, smem)) {
        a.rows = rows; a.k = k; a.group = group; a.w = w; a.scales = scales; a.x = x; a.y = y;
        const cudaError_t e = cudaFuncSetAttribute(gemv_ring_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return status_of(e);
        unsigned grid = (unsigned)device_sms();
        const unsigned need = (rows + kGvRowsPerStage - 1) / kGvRowsPerStage;
        if (grid > need) grid = need;
        gemv_ring_kernel<FMT><<<grid, kGvThreads, smem, s>>>(a);
        return last_launch_status();
    }
    const size_t rsmem = ((size_t)(k >> 5) * (kGemvRowStride + 1) + 16) * sizeof(float);
    if (rsmem > 200 * 1024) return LYTH_E_UNSUPPORTED;
    unsigned grid = (rows + 7) / 8;
    const unsigned cap = (unsigned)device_sms() * 4u;
    if (grid > cap) grid = cap;
    if (rsmem > 48 * 1024) cudaFuncSetAttribute(gemv_row_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem);
    gemv_row_kernel<FMT><<<grid, 256, rsmem, s>>>(rows, k, group, w, scales, x, y);
    return last_launch_status();
}

extern "C" int lyth_b200_gemv_q4(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                 const uint16_t *scales, const uint16_t *x, uint16_t *y, cudaStream_t s) {
    if (!w || !scales || !x || !y) return LYTH_E_INVALID;
    if (rows == 0) return LYTH_OK;
    if (k == 0 || k % 1024 != 0 || group == 0 || group % 32 != 0 || k % group != 0) return LYTH_E_UNSUPPORTED;
    if ((((uintptr_t)w) & 15u) != 0 || (((uintptr_t)x) & 15u) != 0) return LYTH_E_UNSUPPORTED;
    if (fmt == LYTH_GEMV_INT4) return launch_gemv<0>(rows, k, group, w, scales, x, y, s);
    if (fmt == LYTH_GEMV_NF4) {
        const int st = ensure_nf4_on_device();
        if (st) return st;
        return launch_gemv<1>(rows, k, group, w, scales, x, y, s);
    }
    return LYTH_E_UNSUPPORTED;
}

extern "C" int lyth_b200_gemv_dequant(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                      const uint16_t *scales, float *out, cudaStream_t s) {
    if (!w || !scales || !out) return LYTH_E_INVALID;
    if (rows == 0 || k == 0) return LYTH_OK;
    if ((k & 7u) || group == 0 || (group & 7u) || k % group != 0) return LYTH_E_UNSUPPORTED;
    if ((((uintptr_t)w) & 3u) || (((uintptr_t)out) & 15u)) return LYTH_E_UNSUPPORTED;
    const unsigned grid = stream_grid((uint64_t)rows * k / 8, 256);
    if (fmt == LYTH_GEMV_INT4) {
        gemv_dequant_kernel<0><<<grid, 256, 0, s>>>(rows, k, group, w, scales, out);
    } else if (fmt == LYTH_GEMV_NF4) {
        int st = ensure_nf4_on_device();
        if (st) return st;
        gemv_dequant_kernel<1><<<grid, 256, 0, s>>>(rows, k, group, w, scales, out);
    } else {
        return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}

namespace lyth {
int gemv_take_device_error() {
    int v = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int));
    if (e != cudaSuccess) return status_of(e);
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(int));
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}
}  // namespace lyth
