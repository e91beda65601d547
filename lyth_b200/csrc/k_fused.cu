// Fused state-vector passes (lyth-circuit Group, crates/lyth-circuit/src/lib.rs:72-208 and
// docs/ADR-0030): one pass over the state applies a run of consecutive gates that together
// touch at most K <= 6 qubits.
//
// A tuple is the 2^K amplitudes that differ only in the group's K bits. It is loaded once
// (consecutive threads take consecutive values of the other bits, so every load of a warp is
// contiguous), the group's gates are applied in circuit order with the same fma chains as the
// unfused passes, and it is stored back in place. The values between two gates are exactly the
// values the unfused passes would write and read back, so fused equals unfused bit for bit
// (the reference's claim, ADR-0030 Q1).
//
// Registers, not memory: a gate's target / control is a run-time level of the group, but every
// case is its own fully unrolled code path behind a uniform branch, so the amplitudes are only
// ever indexed by compile-time constants.
//
// Packed arithmetic: the tuple is held as float2 pairs along level 0 (X[i] = re of tuple
// elements 2i and 2i+1, Y[i] the same for im). A gate on any other level then pairs X[i] with
// X[i | bit] and runs each chain on both halves at once with fma.rn.f32x2 / mul.rn.f32x2 --
// two independent IEEE operations with the same rounding as the scalar ones, half the
// instructions. Gates on level 0 (and CUs controlled by it) use the scalar halves. The host puts
// the group bit with the fewest gates at level 0.
//
// Lane pairs (K = 5, 6): a tuple is split over lanes l and l ^ 16 of a warp on the last level
// ("split"): lane half h holds the amplitudes whose split bit is h. A gate targeting the split
// level swaps the partner's values in with shuffles and each lane computes its own row (row 0
// with p0 = own, p1 = partner; row 1 with p0 = partner, p1 = own): the same chains on the same
// values. A CU controlled by the split level runs only on the h = 1 lanes.
#include "fused.cuh"

namespace lyth {

// ------------------------------------------------------------------ packed f32x2 helpers
LYTH_D uint64_t pk(float2 a) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
LYTH_D float2 upk(uint64_t r) {
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(r));
    return d;
}
LYTH_D float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
    return upk(d);
}
LYTH_D float2 mul2(float2 a, float2 b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
    return upk(d);
}
LYTH_D float2 bc(float v) { return make_float2(v, v); }

// gate_q's chains on packed operands (each half is the scalar chain of gates.cuh row0/row1).
LYTH_D void row0_2(const U8 &m, float2 p0r, float2 p0i, float2 p1r, float2 p1i, float2 &q0r, float2 &q0i) {
    q0r = fma2(bc(m.ar), p0r, fma2(bc(-m.ai), p0i, fma2(bc(m.br), p1r, mul2(bc(-m.bi), p1i))));
    q0i = fma2(bc(m.ar), p0i, fma2(bc(m.ai), p0r, fma2(bc(m.br), p1i, mul2(bc(m.bi), p1r))));
}
LYTH_D void row1_2(const U8 &m, float2 p0r, float2 p0i, float2 p1r, float2 p1i, float2 &q1r, float2 &q1i) {
    q1r = fma2(bc(m.cr), p0r, fma2(bc(-m.ci), p0i, fma2(bc(m.dr), p1r, mul2(bc(-m.di), p1i))));
    q1i = fma2(bc(m.cr), p0i, fma2(bc(m.ci), p0r, fma2(bc(m.dr), p1i, mul2(bc(m.di), p1r))));
}

// ------------------------------------------------------------------ gates on a lane's pairs
// KL levels in the lane, P = 2^(KL-1) float2 pairs. Level 0 is inside a pair; level T >= 1 is
// bit T-1 of the pair index. CM: a control mask on tuple element index j (0 = no control).

// U (or CU with control level C >= 1) on level T >= 1: packed.
template <int KL, int T, int C>
LYTH_D void gate_hi(const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        if (i & (1 << (T - 1))) continue;
        if (C >= 1 && !(i & (1 << (C - 1)))) continue;
        const int i1 = i | (1 << (T - 1));
        float2 a, b, c, d;
        row0_2(m, X[i], Y[i], X[i1], Y[i1], a, b);
        row1_2(m, X[i], Y[i], X[i1], Y[i1], c, d);
        X[i] = a; Y[i] = b; X[i1] = c; Y[i1] = d;
    }
}
// CU controlled by level 0, target level T >= 1: only the .y halves (element bit 0 = 1).
template <int KL, int T>
LYTH_D void gate_hi_c0(const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        if (i & (1 << (T - 1))) continue;
        const int i1 = i | (1 << (T - 1));
        float a, b, c, d;
        row0(m, X[i].y, Y[i].y, X[i1].y, Y[i1].y, a, b);
        row1(m, X[i].y, Y[i].y, X[i1].y, Y[i1].y, c, d);
        X[i].y = a; Y[i].y = b; X[i1].y = c; Y[i1].y = d;
    }
}
// U (or CU with control level C >= 1) on level 0: scalar, inside each pair.
template <int KL, int C>
LYTH_D void gate_lo(const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        if (C >= 1 && !(i & (1 << (C - 1)))) continue;
        float a, b, c, d;
        row0(m, X[i].x, Y[i].x, X[i].y, Y[i].y, a, b);
        row1(m, X[i].x, Y[i].x, X[i].y, Y[i].y, c, d);
        X[i].x = a; Y[i].x = b; X[i].y = c; Y[i].y = d;
    }
}

// Run-time (t, c) -> compile-time case. c < 0: no control.
template <int KL, int T, int C>
LYTH_D void gate_case(const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
    if constexpr (T == 0) gate_lo<KL, C>(m, X, Y);
    else if constexpr (C == 0) gate_hi_c0<KL, T>(m, X, Y);
    else gate_hi<KL, T, (C < 0 ? 0 : C)>(m, X, Y);
}
template <int KL, int T, int C = -1>
LYTH_D void dispatch_c(int c, const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
    if constexpr (C < KL) {
        if constexpr (C != T) {
            if (c == C) {
                gate_case<KL, T, C>(m, X, Y);
                return;
            }
        }
        dispatch_c<KL, T, C + 1>(c, m, X, Y);
    }
}
template <int KL, int T = 0>
LYTH_D void dispatch_gate(int t, int c, const U8 &m, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
    if constexpr (T < KL) {
        if (t == T) dispatch_c<KL, T>(c, m, X, Y);
        else dispatch_gate<KL, T + 1>(t, c, m, X, Y);
    }
}

// A gate on the split level (lane pairs): partner values by shuffle, own row computed.
// CMASK: -1 no control; 0 control on level 0 (only .y); c >= 1 control on pair-index bit c-1.
template <int KL, int CL>
LYTH_D void split_gate(const U8 &m, int h, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        float2 oX, oY;
        oX.x = __shfl_xor_sync(0xffffffffu, X[i].x, 16);
        oX.y = __shfl_xor_sync(0xffffffffu, X[i].y, 16);
        oY.x = __shfl_xor_sync(0xffffffffu, Y[i].x, 16);
        oY.y = __shfl_xor_sync(0xffffffffu, Y[i].y, 16);
        if (CL >= 1 && !(i & (1 << (CL - 1)))) continue;
        if (CL == 0) {
            float a, b;
            if (h == 0) row0(m, X[i].y, Y[i].y, oX.y, oY.y, a, b);
            else row1(m, oX.y, oY.y, X[i].y, Y[i].y, a, b);
            X[i].y = a; Y[i].y = b;
        } else {
            float2 a, b;
            if (h == 0) row0_2(m, X[i], Y[i], oX, oY, a, b);
            else row1_2(m, oX, oY, X[i], Y[i], a, b);
            X[i] = a; Y[i] = b;
        }
    }
}
template <int KL, int CL = -1>
LYTH_D void dispatch_split(int c, const U8 &m, int h, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
    if constexpr (CL < KL) {
        if (c == CL) split_gate<KL, CL>(m, h, X, Y);
        else dispatch_split<KL, CL + 1>(c, m, h, X, Y);
    }
}

// ------------------------------------------------------------------ the kernel
// SPLIT = false: a thread owns a whole tuple of K levels. SPLIT = true: lanes l, l ^ 16 share
// it; level K-1 is the split level and each lane owns K-1 levels.
template <int K, bool SPLIT>
constexpr int fused_min_blocks() {
    return SPLIT ? (K >= 6 ? 2 : 3) : (K >= 4 ? 2 : 3);
}

template <int K, bool SPLIT>
__global__ void __launch_bounds__(256, fused_min_blocks<K, SPLIT>())
    fused_pass_kernel(uint64_t len, const __grid_constant__ FusedGroup G, float *re, float *im) {
    constexpr int KL = SPLIT ? K - 1 : K;  // levels inside a lane
    constexpr int P = 1 << (KL - 1);       // float2 pairs per lane
    const int lane = threadIdx.x & 31;
    const int h = SPLIT ? (lane >> 4) : 0;
    const uint64_t gtid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t rest = len >> K;
    // Tuples per step: SPLIT: a warp takes 16 (lanes l, l+16 share one); else one per thread.
    const uint64_t first = SPLIT ? (gtid >> 5) * 16 + (lane & 15) : gtid;
    const uint64_t step = SPLIT ? (((uint64_t)gridDim.x * blockDim.x) >> 5) * 16 : (uint64_t)gridDim.x * blockDim.x;
    const uint64_t end = SPLIT ? ((rest + 15) & ~15ull) : rest;  // every lane of a warp runs each step
    for (uint64_t r = first; r < end; r += step) {
        const bool live = r < rest;
        uint64_t base = live ? r : 0;
#pragma unroll
        for (int l = 0; l < K; l++) base = insert_bit(base, G.sorted[l], 0);
        // The strides are re-read per iteration (the empty asm keeps the compiler from hoisting
        // 2^K 64-bit offsets into registers).
        uint64_t stride[K];
#pragma unroll
        for (int l = 0; l < K; l++) {
            stride[l] = 1ull << G.bits[l];
            asm volatile("" : "+l"(stride[l]));
        }
        if (SPLIT && h) base += stride[K - 1];
        float2 X[P], Y[P];
#pragma unroll
        for (int i = 0; i < P; i++) {
            uint64_t off = 0;
#pragma unroll
            for (int l = 1; l < KL; l++)
                if (i & (1 << (l - 1))) off += stride[l];
            const uint64_t a0 = base + off, a1 = a0 + stride[0];
            X[i] = live ? make_float2(re[a0], re[a1]) : make_float2(0.f, 0.f);
            Y[i] = live ? make_float2(im[a0], im[a1]) : make_float2(0.f, 0.f);
        }
        for (uint32_t g = 0; g < G.ngates; g++) {
            const FusedGate &fg = G.gates[g];
            const U8 m{fg.m[0], fg.m[1], fg.m[2], fg.m[3], fg.m[4], fg.m[5], fg.m[6], fg.m[7]};
            if (SPLIT && fg.t == K - 1) {
                dispatch_split<KL>(fg.c, m, h, X, Y);
            } else if (SPLIT && fg.c == K - 1) {
                if (h) dispatch_gate<KL>(fg.t, -1, m, X, Y);
            } else {
                dispatch_gate<KL>(fg.t, fg.c, m, X, Y);
            }
        }
        if (live) {
#pragma unroll
            for (int i = 0; i < P; i++) {
                uint64_t off = 0;
#pragma unroll
                for (int l = 1; l < KL; l++)
                    if (i & (1 << (l - 1))) off += stride[l];
                const uint64_t a0 = base + off, a1 = a0 + stride[0];
                re[a0] = X[i].x; re[a1] = X[i].y;
                im[a0] = Y[i].x; im[a1] = Y[i].y;
            }
        }
    }
}

// Level order for the kernel: level 0 = the bit with the fewest gates on it (target or
// control), and with lane pairs the last level = the bit with the fewest gates targeting it
// among the rest (every such gate costs a round of shuffles).
static FusedGroup arrange_levels(const FusedGroup &g, bool split) {
    const int k = g.k;
    int use[kFuseMaxQubits] = {0}, tgt[kFuseMaxQubits] = {0};
    for (uint32_t i = 0; i < g.ngates; i++) {
        use[g.gates[i].t]++;
        tgt[g.gates[i].t]++;
        if (g.gates[i].c >= 0) use[g.gates[i].c]++;
    }
    int order[kFuseMaxQubits];
    for (int l = 0; l < k; l++) order[l] = l;
    // position 0: fewest uses
    int best = 0;
    for (int l = 1; l < k; l++)
        if (use[l] < use[best]) best = l;
    int t0 = order[0]; order[0] = order[best]; order[best] = t0;
    if (split && k >= 2) {
        int bl = 1;
        for (int p = 2; p < k; p++)
            if (tgt[order[p]] < tgt[order[bl]]) bl = p;
        int t1 = order[k - 1]; order[k - 1] = order[bl]; order[bl] = t1;
    }
    int new_of_old[kFuseMaxQubits];
    for (int p = 0; p < k; p++) new_of_old[order[p]] = p;
    FusedGroup o = g;
    for (int p = 0; p < k; p++) o.bits[p] = g.bits[order[p]];
    for (uint32_t i = 0; i < o.ngates; i++) {
        o.gates[i].t = (int8_t)new_of_old[g.gates[i].t];
        o.gates[i].c = g.gates[i].c >= 0 ? (int8_t)new_of_old[g.gates[i].c] : (int8_t)-1;
    }
    return o;
}

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s) {
    const bool split = g.k >= 5;
    const FusedGroup o = arrange_levels(g, split);
    const uint64_t threads = split ? (len >> g.k) * 2 : (len >> g.k);
    const unsigned grid = stream_grid(threads, kStreamBlock);
    switch (g.k) {
        case 1: fused_pass_kernel<1, false><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        case 2: fused_pass_kernel<2, false><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        case 3: fused_pass_kernel<3, false><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        case 4: fused_pass_kernel<4, false><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        case 5: fused_pass_kernel<5, true><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        case 6: fused_pass_kernel<6, true><<<grid, kStreamBlock, 0, s>>>(len, o, re, im); break;
        default: return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}

}  // namespace lyth
