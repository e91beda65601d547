// State-vector gate passes for sm_100a: examples/{hadamard_q,gate_q,cu_q,swap_q}.lyth.
//
// Addressing. A split view's element k is (k / w) * 2w + part * w + (k % w) of its base
// (ir.rs:78-81); for a power-of-two width w = 2^p that is k with a bit of value `part`
// inserted at position p, and a depth-2 leaf (cu_q, swap_q) is two insertions
// (base_index, ir.rs:340-351). The power-of-two kernels use the insertions; any other width
// that divides takes the literal view_index path.
//
// Vectors. When every inserted bit is at position >= 2, four consecutive k map to four
// consecutive amplitudes in every leaf, so each leaf moves as one 128-bit vector. A gate on
// bit 0 or 1 instead finds both members of its pairs inside one aligned float4.
//
// Arithmetic. The lowered body, op for op (gates.cuh), so every pass is bit-exact with the
// host evaluator.
#include "gates.cuh"

namespace lyth {

// ------------------------------------------------------------------ 1-qubit passes
template <typename Op>
LYTH_D void pair_apply4(const Op &op, float4 r0, float4 i0, float4 r1, float4 i1, float4 &qr0, float4 &qi0,
                        float4 &qr1, float4 &qi1) {
    op(r0.x, i0.x, r1.x, i1.x, qr0.x, qi0.x, qr1.x, qi1.x);
    op(r0.y, i0.y, r1.y, i1.y, qr0.y, qi0.y, qr1.y, qi1.y);
    op(r0.z, i0.z, r1.z, i1.z, qr0.z, qi0.z, qr1.z, qi1.z);
    op(r0.w, i0.w, r1.w, i1.w, qr0.w, qi0.w, qr1.w, qi1.w);
}

// One pass over all n/2 pairs of bit p (w = 2^p) or, when pow2 is false, of width w.
template <typename Op>
LYTH_D void pairs_body(uint64_t n, uint64_t w, const Op &op, const float *re, const float *im, float *qr,
                       float *qi) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t pairs = n >> 1;
    const bool pow2 = w != 0 && (w & (w - 1)) == 0;
    const bool vec = ((((uintptr_t)re) | ((uintptr_t)im) | ((uintptr_t)qr) | ((uintptr_t)qi)) & 15u) == 0 &&
                     (n & 3u) == 0;
    if (pow2 && vec && w >= 4) {
        const unsigned p = __ffsll((long long)w) - 1;
        const uint64_t groups = pairs >> 2;  // 4 pairs per group
        for (uint64_t g = tid; g < groups; g += nthreads) {
            const uint64_t i0 = insert_bit(g << 2, p, 0), i1 = i0 + w;
            float4 r0 = ld_stream4(re + i0), m0 = ld_stream4(im + i0);
            float4 r1 = ld_stream4(re + i1), m1 = ld_stream4(im + i1);
            float4 a, b, c, d;
            pair_apply4(op, r0, m0, r1, m1, a, b, c, d);
            st4(qr + i0, a); st4(qi + i0, b); st4(qr + i1, c); st4(qi + i1, d);
        }
    } else if (pow2 && vec && w == 2) {
        // float4 at 4g = (p0, p0, p1, p1): pairs (x, z) and (y, w).
        const uint64_t groups = n >> 2;
        for (uint64_t g = tid; g < groups; g += nthreads) {
            float4 r = ld_stream4(re + 4 * g), m = ld_stream4(im + 4 * g), qrv, qiv;
            op(r.x, m.x, r.z, m.z, qrv.x, qiv.x, qrv.z, qiv.z);
            op(r.y, m.y, r.w, m.w, qrv.y, qiv.y, qrv.w, qiv.w);
            st4(qr + 4 * g, qrv); st4(qi + 4 * g, qiv);
        }
    } else if (pow2 && vec && w == 1) {
        // float4 at 4g = (p0, p1, p0, p1): pairs (x, y) and (z, w).
        const uint64_t groups = n >> 2;
        for (uint64_t g = tid; g < groups; g += nthreads) {
            float4 r = ld_stream4(re + 4 * g), m = ld_stream4(im + 4 * g), qrv, qiv;
            op(r.x, m.x, r.y, m.y, qrv.x, qiv.x, qrv.y, qiv.y);
            op(r.z, m.z, r.w, m.w, qrv.z, qiv.z, qrv.w, qiv.w);
            st4(qr + 4 * g, qrv); st4(qi + 4 * g, qiv);
        }
    } else {
        for (uint64_t k = tid; k < pairs; k += nthreads) {
            const uint64_t i0 = view_index(w, 0, k), i1 = view_index(w, 1, k);
            float a, b, c, d;
            op(re[i0], im[i0], re[i1], im[i1], a, b, c, d);
            qr[i0] = a; qi[i0] = b; qr[i1] = c; qi[i1] = d;
        }
    }
}

// The ADR-0016 kernels: the reference's parameter lists, in declaration order.
template <typename I>
__global__ void __launch_bounds__(256) hadamard_q_kernel(I n, I w, float s, const float *re, const float *im,
                                                         float *qr, float *qi) {
    pairs_body((uint64_t)n, (uint64_t)w, HadamardOp{s}, re, im, qr, qi);
}
template <typename I>
__global__ void __launch_bounds__(256) gate_q_kernel(I n, I w, float ar, float ai, float br, float bi, float cr,
                                                     float ci, float dr, float di, const float *re,
                                                     const float *im, float *qr, float *qi) {
    pairs_body((uint64_t)n, (uint64_t)w, UOp{U8{ar, ai, br, bi, cr, ci, dr, di}}, re, im, qr, qi);
}

// ------------------------------------------------------------------ 2-qubit passes
// Leaf XY of quad k: bit c = X, bit t = Y. Power-of-two: two insertions at (lo, hi). Else the
// reference's composed view_index with widths (wc, wt).
struct Quad {
    uint64_t i00, i01, i10, i11;
};
LYTH_D Quad quad_pow2(uint64_t k, unsigned c, unsigned t) {
    const unsigned lo = c < t ? c : t, hi = c < t ? t : c;
    const uint64_t b = insert_bit(insert_bit(k, lo, 0), hi, 0);
    const uint64_t mc = 1ull << c, mt = 1ull << t;
    return Quad{b, b | mt, b | mc, b | mc | mt};
}
LYTH_D Quad quad_general(uint64_t k, uint64_t wc, uint64_t wt) {
    return Quad{view_index(wc, 0, view_index(wt, 0, k)), view_index(wc, 0, view_index(wt, 1, k)),
                view_index(wc, 1, view_index(wt, 0, k)), view_index(wc, 1, view_index(wt, 1, k))};
}

// kind 0: controlled U on (c, t); kind 1: swap. `copy_all`: also move the leaves a gate
// leaves unchanged (needed out of place; in place they are skipped: half the traffic).
template <int KIND>
LYTH_D void quad_apply_scalar(const U8 &m, const Quad &q, const float *re, const float *im, float *qr, float *qi,
                              bool copy_all) {
    if (KIND == 0) {
        const float p0r = re[q.i10], p0i = im[q.i10], p1r = re[q.i11], p1i = im[q.i11];
        float a, b, c, d;
        row0(m, p0r, p0i, p1r, p1i, a, b);
        row1(m, p0r, p0i, p1r, p1i, c, d);
        if (copy_all) {
            const float r00 = re[q.i00], m00 = im[q.i00], r01 = re[q.i01], m01 = im[q.i01];
            qr[q.i00] = r00; qi[q.i00] = m00; qr[q.i01] = r01; qi[q.i01] = m01;
        }
        qr[q.i10] = a; qi[q.i10] = b; qr[q.i11] = c; qi[q.i11] = d;
    } else {
        const float r01 = re[q.i01], m01 = im[q.i01], r10 = re[q.i10], m10 = im[q.i10];
        if (copy_all) {
            const float r00 = re[q.i00], m00 = im[q.i00], r11 = re[q.i11], m11 = im[q.i11];
            qr[q.i00] = r00; qi[q.i00] = m00; qr[q.i11] = r11; qi[q.i11] = m11;
        }
        qr[q.i01] = r10; qi[q.i01] = m10; qr[q.i10] = r01; qi[q.i10] = m01;
    }
}

template <int KIND>
LYTH_D void quads_body(uint64_t n, bool pow2, unsigned c, unsigned t, uint64_t wc, uint64_t wt, const U8 &m,
                       const float *re, const float *im, float *qr, float *qi) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t quads = n >> 2;
    const bool inplace = (re == qr) && (im == qi);
    const bool vec = pow2 && (c >= 2 && t >= 2) && (n & 15u) == 0 &&
                     ((((uintptr_t)re) | ((uintptr_t)im) | ((uintptr_t)qr) | ((uintptr_t)qi)) & 15u) == 0;
    const bool copy_all = !inplace;
    if (vec) {
        const uint64_t groups = quads >> 2;
        for (uint64_t g = tid; g < groups; g += nthreads) {
            const Quad q = quad_pow2(g << 2, c, t);
            if (KIND == 0) {
                float4 r0 = ld_stream4(re + q.i10), m0 = ld_stream4(im + q.i10);
                float4 r1 = ld_stream4(re + q.i11), m1 = ld_stream4(im + q.i11);
                float4 a, b, cc, d;
                pair_apply4(UOp{m}, r0, m0, r1, m1, a, b, cc, d);
                if (copy_all) {
                    float4 x0 = ld_stream4(re + q.i00), y0 = ld_stream4(im + q.i00);
                    float4 x1 = ld_stream4(re + q.i01), y1 = ld_stream4(im + q.i01);
                    st4(qr + q.i00, x0); st4(qi + q.i00, y0); st4(qr + q.i01, x1); st4(qi + q.i01, y1);
                }
                st4(qr + q.i10, a); st4(qi + q.i10, b); st4(qr + q.i11, cc); st4(qi + q.i11, d);
            } else {
                float4 r01 = ld_stream4(re + q.i01), m01 = ld_stream4(im + q.i01);
                float4 r10 = ld_stream4(re + q.i10), m10 = ld_stream4(im + q.i10);
                if (copy_all) {
                    float4 x0 = ld_stream4(re + q.i00), y0 = ld_stream4(im + q.i00);
                    float4 x1 = ld_stream4(re + q.i11), y1 = ld_stream4(im + q.i11);
                    st4(qr + q.i00, x0); st4(qi + q.i00, y0); st4(qr + q.i11, x1); st4(qi + q.i11, y1);
                }
                st4(qr + q.i01, r10); st4(qi + q.i01, m10); st4(qr + q.i10, r01); st4(qi + q.i10, m01);
            }
        }
    } else {
        for (uint64_t k = tid; k < quads; k += nthreads) {
            const Quad q = pow2 ? quad_pow2(k, c, t) : quad_general(k, wc, wt);
            quad_apply_scalar<KIND>(m, q, re, im, qr, qi, copy_all);
        }
    }
}

// (wc, wt) as the reference's launch gives them -> physical bits, when both are powers of
// two: c = log2 wc; the inner width counts elements of the view that lost bit c, so
// t = log2 wt, plus one when that position is at or above c (widths_ct, lyth-circuit lib.rs:387).
LYTH_D bool ct_of(uint64_t wc, uint64_t wt, unsigned &c, unsigned &t) {
    if (wc == 0 || wt == 0 || (wc & (wc - 1)) || (wt & (wt - 1))) return false;
    c = __ffsll((long long)wc) - 1;
    const unsigned lt = __ffsll((long long)wt) - 1;
    t = lt < c ? lt : lt + 1;
    return true;
}

template <typename I>
__global__ void __launch_bounds__(256) cu_q_kernel(I n, I wc, I wt, float ar, float ai, float br, float bi,
                                                   float cr, float ci, float dr, float di, const float *re,
                                                   const float *im, float *qr, float *qi) {
    unsigned c = 0, t = 0;
    const bool pow2 = ct_of((uint64_t)wc, (uint64_t)wt, c, t);
    quads_body<0>((uint64_t)n, pow2, c, t, (uint64_t)wc, (uint64_t)wt, U8{ar, ai, br, bi, cr, ci, dr, di}, re, im,
                  qr, qi);
}
template <typename I>
__global__ void __launch_bounds__(256) swap_q_kernel(I n, I wc, I wt, const float *re, const float *im, float *qr,
                                                     float *qi) {
    unsigned c = 0, t = 0;
    const bool pow2 = ct_of((uint64_t)wc, (uint64_t)wt, c, t);
    quads_body<1>((uint64_t)n, pow2, c, t, (uint64_t)wc, (uint64_t)wt, U8{}, re, im, qr, qi);
}

// The engine's physical-bit variants (no width decoding).
__global__ void __launch_bounds__(256) cu_bits_kernel(uint64_t n, unsigned c, unsigned t, U8 m, const float *re,
                                                      const float *im, float *qr, float *qi) {
    quads_body<0>(n, true, c, t, 0, 0, m, re, im, qr, qi);
}
__global__ void __launch_bounds__(256) swap_bits_kernel(uint64_t n, unsigned a, unsigned b, const float *re,
                                                        const float *im, float *qr, float *qi) {
    quads_body<1>(n, true, a, b, 0, 0, U8{}, re, im, qr, qi);
}

// ------------------------------------------------------------------ exchange compute half
__global__ void __launch_bounds__(256) exchange_u_kernel(uint64_t len, uint64_t base, int side, int ctrl_bit, U8 m,
                                                         float *ore, float *oim, const float *rre,
                                                         const float *rim) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const bool vec = ((len & 3u) == 0) && ((base & 3u) == 0) && (ctrl_bit < 0 || ctrl_bit >= 2) &&
                     ((((uintptr_t)ore) | ((uintptr_t)oim) | ((uintptr_t)rre) | ((uintptr_t)rim)) & 15u) == 0;
    if (vec) {
        for (uint64_t g = tid; g < (len >> 2); g += nthreads) {
            const uint64_t i = g << 2;
            if (ctrl_bit >= 0 && !(((base + i) >> ctrl_bit) & 1ull)) continue;
            float4 orv = ld4(ore + i), oiv = ld4(oim + i);
            float4 rrv = ld_stream4(rre + i), riv = ld_stream4(rim + i);
            float4 xr, xi;
            if (side == 0) {
                row0(m, orv.x, oiv.x, rrv.x, riv.x, xr.x, xi.x);
                row0(m, orv.y, oiv.y, rrv.y, riv.y, xr.y, xi.y);
                row0(m, orv.z, oiv.z, rrv.z, riv.z, xr.z, xi.z);
                row0(m, orv.w, oiv.w, rrv.w, riv.w, xr.w, xi.w);
            } else {
                row1(m, rrv.x, riv.x, orv.x, oiv.x, xr.x, xi.x);
                row1(m, rrv.y, riv.y, orv.y, oiv.y, xr.y, xi.y);
                row1(m, rrv.z, riv.z, orv.z, oiv.z, xr.z, xi.z);
                row1(m, rrv.w, riv.w, orv.w, oiv.w, xr.w, xi.w);
            }
            st4(ore + i, xr); st4(oim + i, xi);
        }
    } else {
        for (uint64_t i = tid; i < len; i += nthreads) {
            if (ctrl_bit >= 0 && !(((base + i) >> ctrl_bit) & 1ull)) continue;
            float xr, xi;
            if (side == 0) row0(m, ore[i], oim[i], rre[i], rim[i], xr, xi);
            else row1(m, rre[i], rim[i], ore[i], oim[i], xr, xi);
            ore[i] = xr; oim[i] = xi;
        }
    }
}

template __global__ void hadamard_q_kernel<uint32_t>(uint32_t, uint32_t, float, const float *, const float *, float *, float *);
template __global__ void gate_q_kernel<uint32_t>(uint32_t, uint32_t, float, float, float, float, float, float, float,
                                                 float, const float *, const float *, float *, float *);
template __global__ void cu_q_kernel<uint32_t>(uint32_t, uint32_t, uint32_t, float, float, float, float, float, float,
                                               float, float, const float *, const float *, float *, float *);
template __global__ void swap_q_kernel<uint32_t>(uint32_t, uint32_t, uint32_t, const float *, const float *, float *,
                                                 float *);

// ------------------------------------------------------------------ host launchers
static inline unsigned pass_grid(uint64_t units) { return stream_grid(units, kStreamBlock); }

int launch_u(uint64_t n, unsigned p, const U8 &m, const float *re, const float *im, float *qr, float *qi,
             cudaStream_t s) {
    const U8 mm = m;
    gate_q_kernel<uint64_t><<<pass_grid(n / 8 + 1), kStreamBlock, 0, s>>>(
        n, 1ull << p, mm.ar, mm.ai, mm.br, mm.bi, mm.cr, mm.ci, mm.dr, mm.di, re, im, qr, qi);
    return last_launch_status();
}
int launch_h(uint64_t n, unsigned p, float sc, const float *re, const float *im, float *qr, float *qi,
             cudaStream_t s) {
    hadamard_q_kernel<uint64_t><<<pass_grid(n / 8 + 1), kStreamBlock, 0, s>>>(n, 1ull << p, sc, re, im, qr, qi);
    return last_launch_status();
}
int launch_cu(uint64_t n, unsigned c, unsigned t, const U8 &m, const float *re, const float *im, float *qr,
              float *qi, cudaStream_t s) {
    cu_bits_kernel<<<pass_grid(n / 16 + 1), kStreamBlock, 0, s>>>(n, c, t, m, re, im, qr, qi);
    return last_launch_status();
}
int launch_swap(uint64_t n, unsigned a, unsigned b, const float *re, const float *im, float *qr, float *qi,
                cudaStream_t s) {
    swap_bits_kernel<<<pass_grid(n / 16 + 1), kStreamBlock, 0, s>>>(n, a, b, re, im, qr, qi);
    return last_launch_status();
}
int launch_exchange_u(uint64_t len, uint64_t base_index, int side, int ctrl_bit, const U8 &m, float *ore,
                      float *oim, const float *rre, const float *rim, cudaStream_t s) {
    exchange_u_kernel<<<pass_grid(len / 4 + 1), kStreamBlock, 0, s>>>(len, base_index, side, ctrl_bit, m, ore, oim,
                                                                     rre, rim);
    return last_launch_status();
}

}  // namespace lyth

using namespace lyth;

// ------------------------------------------------------------------ B200 surface
namespace {
bool split_ok(uint64_t len, uint64_t w) { return w != 0 && len % (2 * w) == 0; }
}  // namespace

extern "C" int lyth_b200_hadamard(uint64_t n, uint64_t w, float s, const float *re, const float *im, float *qr,
                                  float *qi, cudaStream_t st) {
    if (!split_ok(n, w)) return LYTH_E_SPLIT;
    if (!re || !im || !qr || !qi) return LYTH_E_INVALID;
    hadamard_q_kernel<uint64_t><<<pass_grid(n / 8 + 1), kStreamBlock, 0, st>>>(n, w, s, re, im, qr, qi);
    return last_launch_status();
}
extern "C" int lyth_b200_gate(uint64_t n, uint64_t w, const float *m, const float *re, const float *im, float *qr,
                              float *qi, cudaStream_t st) {
    if (!split_ok(n, w)) return LYTH_E_SPLIT;
    if (!m || !re || !im || !qr || !qi) return LYTH_E_INVALID;
    gate_q_kernel<uint64_t><<<pass_grid(n / 8 + 1), kStreamBlock, 0, st>>>(n, w, m[0], m[1], m[2], m[3], m[4], m[5],
                                                                          m[6], m[7], re, im, qr, qi);
    return last_launch_status();
}
extern "C" int lyth_b200_cu(uint64_t n, uint64_t wc, uint64_t wt, const float *m, const float *re, const float *im,
                            float *qr, float *qi, cudaStream_t st) {
    if (!split_ok(n, wc) || !split_ok(n / 2, wt)) return LYTH_E_SPLIT;
    if (!m || !re || !im || !qr || !qi) return LYTH_E_INVALID;
    cu_q_kernel<uint64_t><<<pass_grid(n / 16 + 1), kStreamBlock, 0, st>>>(n, wc, wt, m[0], m[1], m[2], m[3], m[4],
                                                                         m[5], m[6], m[7], re, im, qr, qi);
    return last_launch_status();
}
extern "C" int lyth_b200_swap(uint64_t n, uint64_t wc, uint64_t wt, const float *re, const float *im, float *qr,
                              float *qi, cudaStream_t st) {
    if (!split_ok(n, wc) || !split_ok(n / 2, wt)) return LYTH_E_SPLIT;
    if (!re || !im || !qr || !qi) return LYTH_E_INVALID;
    swap_q_kernel<uint64_t><<<pass_grid(n / 16 + 1), kStreamBlock, 0, st>>>(n, wc, wt, re, im, qr, qi);
    return last_launch_status();
}
