// gate_proj GEMV for sm_100a: y = W x with W in 4-bit INT4 or NF4, fp16 per-group scales,
// fp16 activations, f32 accumulation, fp16 output.
//
// The reference has no kernel for this class: only cost contracts
// (fixtures/kernel/gate_proj_int4.json, fixtures/poly/gate-proj-int4-nf4.json: 0.5 B of
// weight per element, a scale per group, 2 flops per weight). The format is this project's:
// row r of W is contiguous along k, byte (r*k + c) / 2, low nibble = even c; INT4 nibbles are
// two's complement (-8..7); NF4 nibbles index the 16-level normal-float codebook of QLoRA.
//
// Kernel: one warp per output row. A lane loads 16 bytes (32 weights) per step, 512 bytes a
// warp, so a 4096-wide row is four coalesced 128-bit loads per lane, all issued before any is
// used. x is staged once per block in shared memory, widened to f32 and permuted so that lane
// l's 32 values at step s sit in 32 different words of 32 different banks. A lane's 32
// weights lie in one scale group (the group is a multiple of 32), so the scale multiplies the
// lane's partial once per step instead of once per weight. The warp's partials combine with
// shuffles; the row result is rounded once to fp16 (RNE).
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"

namespace lyth {

__constant__ float c_nf4[16];

// INT4: (nibble ^ 8) is q + 8 in 0..15; OR-ing it into the mantissa of 2^23 gives the float
// 8388608 + q + 8 exactly, and one subtraction leaves q. One LOP3 and one FADD per weight.
LYTH_D float int4_of(uint32_t word, int j) {
    const uint32_t bits = ((word >> (4 * j)) & 0xfu) ^ 0x4b000008u;
    return __fsub_rn(__uint_as_float(bits), 8388616.0f);
}

template <int FMT>
LYTH_D float weight_of(uint32_t word, int j, const float *lut) {
    if (FMT == 0) return int4_of(word, j);
    return lut[(word >> (4 * j)) & 0xfu];
}

LYTH_D float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

template <int FMT>
__global__ void __launch_bounds__(256) gemv_q4_kernel(uint32_t rows, uint32_t k, uint32_t group, const uint8_t *w,
                                                      const uint16_t *scales, const uint16_t *x, uint16_t *y) {
    extern __shared__ float smem[];
    float *xs = smem;        // k floats, permuted: [step][j][lane]
    float *lut = smem + k;   // 16 floats
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t steps = k / 1024;  // 1024 weights per warp-step (32 lanes x 32)
    // Stage x: element c = 32*(lane + 32*s) + j goes to xs[(s*32 + j)*32 + lane].
    for (uint32_t c = threadIdx.x; c < k; c += blockDim.x) {
        const uint32_t chunk = c >> 5, j = c & 31;
        const uint32_t s = chunk >> 5, l = chunk & 31;
        xs[(s * 32 + j) * 32 + l] = half_bits_to_float(x[c]);
    }
    if (FMT == 1 && threadIdx.x < 16) lut[threadIdx.x] = c_nf4[threadIdx.x];
    __syncthreads();

    const uint32_t groups = k / group;
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
                    const float *xv = xs + (uint64_t)(s0 + u) * 1024 + lane;
                    const uint32_t words[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                    float part = 0.0f;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            part = __fmaf_rn(weight_of<FMT>(words[q], j, lut), xv[(q * 8 + j) * 32], part);
                        }
                    }
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
    const size_t smem = (size_t)k * sizeof(float) + 16 * sizeof(float);
    if (smem > 200 * 1024) return LYTH_E_UNSUPPORTED;
    const unsigned grid = (rows + 7) / 8;
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
