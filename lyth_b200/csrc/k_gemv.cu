// gate_proj GEMV for sm_100a: y = W x with W in 4-bit INT4 or NF4, fp16 per-group scales,
// fp16 activations, f32 accumulation, fp16 output.
//
// The reference has no kernel for this class: only cost contracts
// (fixtures/kernel/gate_proj_int4.json, fixtures/poly/gate-proj-int4-nf4.json: 0.5 B of
// weight per element, a scale per group, 2 flops per weight). The format is this project's:
// row r of W is contiguous along k, byte (r*k + c) / 2, low nibble = even c; INT4 nibbles are
// two's complement (-8..7); NF4 nibbles index the 16-level normal-float codebook of QLoRA.
//
// Kernel: one warp per output row at a time. A lane owns 32-weight chunks (16 bytes of W):
// chunk = lane + 32 * s, so each step of a warp is one coalesced 512-byte load, and every step
// of a row is issued before any is used. x is staged once per block in shared memory, widened
// to f32, one 32-value chunk per row of 36 floats (the pad makes a lane's 128-bit reads
// conflict-free: 8 lanes of a phase hit 8 different 4-bank groups). A chunk lies inside one
// scale group (the group is a multiple of 32), so the scale multiplies a chunk's partial once.
//
// The arithmetic is the instruction budget: 58.7 M weights in ~5 us leaves ~3 instructions per
// weight on 148 SMs. INT4: the word is xor'ed with 0x88888888 (nibble v = q + 8, 0..15), split
// into its even and odd nibbles as bytes, and one PRMT per weight builds the float whose bits
// are 0x3F00_0000 | v << 16, i.e. 0.5 + v/256; one FFMA accumulates it against x. Per chunk,
// sum q x = 256 * (sum f x - (17/32) * sum x), with sum x over the chunk precomputed once per
// block (x is shared by every row); the cancellation costs ~5 of f32's 24 bits, far inside the
// 1e-3 output tolerance. NF4: the same byte split, a PRMT to an index, and a 16-entry shared
// table. The warp's chunk partials combine with shuffles; the row is rounded once to fp16.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"

namespace lyth {

__constant__ float c_nf4[16];

LYTH_D float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

LYTH_D uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// One 16-byte chunk (32 weights) against its 32 staged x values. INT4 returns sum f x with
// f = 0.5 + (q + 8)/256 (the caller corrects); NF4 returns sum code[v] x.
template <int FMT>
LYTH_D float chunk_dot(uint4 v, const float *xr, const float *lut) {
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t w = words[q];
        if (FMT == 0) w ^= 0x88888888u;            // v = q + 8 in every nibble
        const uint32_t lo = w & 0x0F0F0F0Fu;        // nibbles 0, 2, 4, 6 as bytes
        const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu; // nibbles 1, 3, 5, 7 as bytes
        const float4 xa = *reinterpret_cast<const float4 *>(xr + 8 * q);
        const float4 xb = *reinterpret_cast<const float4 *>(xr + 8 * q + 4);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int b = 0; b < 4; b++) {
            float f0, f1;
            if (FMT == 0) {
                // bytes [0, 0, v, 0x3F] -> bits 0x3F00_0000 | v << 16 -> 0.5 + v / 256
                f0 = __uint_as_float(prmt(lo, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
                f1 = __uint_as_float(prmt(hi, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
            } else {
                f0 = lut[prmt(lo, 0u, 0x4440u | (uint32_t)b)];
                f1 = lut[prmt(hi, 0u, 0x4440u | (uint32_t)b)];
            }
            acc0 = __fmaf_rn(f0, xv[2 * b], acc0);
            acc1 = __fmaf_rn(f1, xv[2 * b + 1], acc1);
        }
    }
    return __fadd_rn(acc0, acc1);
}

constexpr int kGemvRowStride = 36;  // floats per staged 32-value chunk (pad 4: conflict-free LDS.128)

template <int FMT>
__global__ void __launch_bounds__(256) gemv_q4_kernel(uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                                      const uint16_t *scales, const uint16_t *x, uint16_t *y) {
    extern __shared__ __align__(16) float smem[];
    const uint32_t chunks = k >> 5;
    float *xs = smem;                                 // chunks x 36
    float *xsum = smem + chunks * kGemvRowStride;     // chunks
    float *lut = xsum + chunks;                       // 16
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // Stage x: each thread moves 8 fp16 values (one 16-byte load) per step, all loads issued
    // before any conversion; four consecutive threads cover one 32-value chunk, and their four
    // 8-value sums combine with two shuffles into that chunk's sum (INT4's correction term).
    {
        const uint4 *x16 = reinterpret_cast<const uint4 *>(x);
        const uint32_t nvec = k >> 3;  // 16-byte groups of x
        for (uint32_t v0 = 0; v0 < nvec; v0 += 4 * blockDim.x) {
            uint4 raw[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t v = v0 + u * blockDim.x + threadIdx.x;
                if (v < nvec) raw[u] = x16[v];
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t v = v0 + u * blockDim.x + threadIdx.x;
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
    if (FMT == 1 && threadIdx.x < 16) lut[threadIdx.x] = c_nf4[threadIdx.x];
    __syncthreads();

    const uint32_t groups = k / group;
    const uint32_t steps = chunks >> 5;  // 32 chunks (one per lane) per warp-step
    for (uint32_t r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
        const uint4 *wrow = reinterpret_cast<const uint4 *>(w + (uint64_t)r * (k >> 1));
        const uint16_t *srow = scales + (uint64_t)r * groups;
        float acc = 0.0f;
        for (uint32_t s0 = 0; s0 < steps; s0 += 4) {
            uint4 v[4];
            float sc[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (s0 + u < steps) {
                    const uint32_t chunk = lane + 32 * (s0 + u);
                    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                                 : "l"(wrow + chunk));
                    sc[u] = half_bits_to_float(srow[(chunk * 32) / group]);
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
        if (lane == 0) y[r] = __half_as_ushort(__float2half_rn(acc));
    }
}

// The dequantised matrix, one weight per thread: q * scale (INT4, exact) or code * scale
// (NF4, one rounding) -- the same values the GEMV's weights take before the scale is factored.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_dequant_kernel(uint32_t rows, uint32_t k, uint32_t group,
                                                           const uint8_t *w, const uint16_t *scales, float *out) {
    const uint64_t n = (uint64_t)rows * k;
    const uint32_t groups = k / group;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = e / k, c = e % k;
        const uint32_t byte = w[e >> 1];
        const uint32_t nib = (e & 1) ? (byte >> 4) : (byte & 0xfu);
        const float s = half_bits_to_float(scales[r * groups + c / group]);
        float v;
        if (FMT == 0) v = __fmul_rn(__fsub_rn(__uint_as_float((nib ^ 8u) | 0x4b000000u), 8388616.0f), s);
        else v = __fmul_rn(c_nf4[nib], s);
        out[e] = v;
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

extern "C" int lyth_b200_gemv_q4(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                 const uint16_t *scales, const uint16_t *x, uint16_t *y, cudaStream_t s) {
    if (!w || !scales || !x || !y) return LYTH_E_INVALID;
    if (rows == 0) return LYTH_OK;
    if (k == 0 || k % 1024 != 0 || group == 0 || group % 32 != 0 || k % group != 0) return LYTH_E_UNSUPPORTED;
    if ((((uintptr_t)w) & 15u) != 0) return LYTH_E_UNSUPPORTED;
    const size_t smem = ((size_t)(k >> 5) * (kGemvRowStride + 1) + 16) * sizeof(float);
    if (smem > 200 * 1024) return LYTH_E_UNSUPPORTED;
    // Persistent: at most 4 blocks per SM (the register budget), each walking rows, so x is
    // staged once per block rather than once per 8 rows.
    unsigned grid = (rows + 7) / 8;
    const unsigned cap = (unsigned)device_sms() * 4u;
    if (grid > cap) grid = cap;
    if (fmt == LYTH_GEMV_INT4) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_q4_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        gemv_q4_kernel<0><<<grid, 256, smem, s>>>(rows, k, group, w, scales, x, y);
    } else if (fmt == LYTH_GEMV_NF4) {
        int st = ensure_nf4_on_device();
        if (st) return st;
        if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_q4_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        gemv_q4_kernel<1><<<grid, 256, smem, s>>>(rows, k, group, w, scales, x, y);
    } else {
        return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}

extern "C" int lyth_b200_gemv_dequant(int fmt, uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                      const uint16_t *scales, float *out, cudaStream_t s) {
    if (!w || !scales || !out) return LYTH_E_INVALID;
    if (rows == 0 || k == 0) return LYTH_OK;
    if ((k & 1u) || group == 0 || k % group != 0) return LYTH_E_UNSUPPORTED;
    const unsigned grid = stream_grid((uint64_t)rows * k, 256);
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
