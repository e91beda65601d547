// State-vector gate passes shared by the gate entry points and the state-vector engine.
#pragma once

#include "common.cuh"

namespace lyth {

// A 2x2 complex matrix as lyth-circuit's f32s gives it: ar ai br bi cr ci dr di.
struct U8 {
    float ar, ai, br, bi, cr, ci, dr, di;
};

inline U8 u8_of(const float *m) { return U8{m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7]}; }

// The four fma chains of examples/gate_q.lyth, lowered by ir.rs:2388-2429:
//   q0r = fma(ar, p0r, fma(-ai, p0i, fma(br, p1r, mul(-bi, p1i))))
//   q0i = fma(ar, p0i, fma( ai, p0r, fma(br, p1i, mul( bi, p1r))))
//   q1r = fma(cr, p0r, fma(-ci, p0i, fma(dr, p1r, mul(-di, p1i))))
//   q1i = fma(cr, p0i, fma( ci, p0r, fma(dr, p1i, mul( di, p1r))))
LYTH_D void row0(const U8 &m, float p0r, float p0i, float p1r, float p1i, float &q0r, float &q0i) {
    q0r = __fmaf_rn(m.ar, p0r, __fmaf_rn(-m.ai, p0i, __fmaf_rn(m.br, p1r, __fmul_rn(-m.bi, p1i))));
    q0i = __fmaf_rn(m.ar, p0i, __fmaf_rn(m.ai, p0r, __fmaf_rn(m.br, p1i, __fmul_rn(m.bi, p1r))));
}
LYTH_D void row1(const U8 &m, float p0r, float p0i, float p1r, float p1i, float &q1r, float &q1i) {
    q1r = __fmaf_rn(m.cr, p0r, __fmaf_rn(-m.ci, p0i, __fmaf_rn(m.dr, p1r, __fmul_rn(-m.di, p1i))));
    q1i = __fmaf_rn(m.cr, p0i, __fmaf_rn(m.ci, p0r, __fmaf_rn(m.dr, p1i, __fmul_rn(m.di, p1r))));
}

// examples/hadamard_q.lyth: q0 = s * (p0 + p1), q1 = s * (p0 - p1). No fma: a Mul of a Bin.
struct HadamardOp {
    float s;
    LYTH_D void operator()(float p0r, float p0i, float p1r, float p1i, float &q0r, float &q0i, float &q1r,
                           float &q1i) const {
        q0r = __fmul_rn(s, __fadd_rn(p0r, p1r));
        q0i = __fmul_rn(s, __fadd_rn(p0i, p1i));
        q1r = __fmul_rn(s, __fsub_rn(p0r, p1r));
        q1i = __fmul_rn(s, __fsub_rn(p0i, p1i));
    }
};
struct UOp {
    U8 m;
    LYTH_D void operator()(float p0r, float p0i, float p1r, float p1i, float &q0r, float &q0i, float &q1r,
                           float &q1i) const {
        row0(m, p0r, p0i, p1r, p1i, q0r, q0i);
        row1(m, p0r, p0i, p1r, p1i, q1r, q1i);
    }
};

// ---- host-side launchers (k_gates.cu). All take amplitude counts in 64 bits, power-of-two
// physical bit positions, and allow qr == re, qi == im (in place).

// A 1-qubit pass on bit p. op: U (m) or Hadamard (s).
int launch_u(uint64_t n, unsigned p, const U8 &m, const float *re, const float *im, float *qr, float *qi,
             cudaStream_t s);
int launch_h(uint64_t n, unsigned p, float sc, const float *re, const float *im, float *qr, float *qi,
             cudaStream_t s);
// Controlled U, control bit c, target bit t (physical positions). With qr == re and qi == im
// the control=0 half is left alone (it is a copy); otherwise it is copied.
int launch_cu(uint64_t n, unsigned c, unsigned t, const U8 &m, const float *re, const float *im, float *qr,
              float *qi, cudaStream_t s);
// Swap bits a and b.
int launch_swap(uint64_t n, unsigned a, unsigned b, const float *re, const float *im, float *qr, float *qi,
                cudaStream_t s);

// The compute half of a gate whose target lives across ranks: this rank owns one side of
// every pair (side 0: it holds p0, 1: it holds p1) and has received the partner's side in
// (rre, rim). own[i] becomes row `side` of the gate at local index i. ctrl_bit >= 0 limits
// the update to local indices with that bit set (a CU whose control is local); the rest are
// a copy and are not touched. base_index is the chunk's first local index.
int launch_exchange_u(uint64_t len, uint64_t base_index, int side, int ctrl_bit, const U8 &m, float *ore,
                      float *oim, const float *rre, const float *rim, cudaStream_t s);

}  // namespace lyth
