// Fused state-vector passes (lyth-circuit Group, crates/lyth-circuit/src/lib.rs:72-208 and
// docs/ADR-0030): one pass over the state applies a run of consecutive gates that together
// touch at most K qubits -- K <= 13 in the tile pass (states of 2^14 amplitudes and more, below),
// K <= 6 in the register pass described first, which small states take.
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
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "fused.cuh"
#include "mbar.cuh"

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

// A gate on a lane level (lanes l and l ^ lm hold the two values of the target): partner
// values by shuffle, own row computed. h = this lane's target bit: h = 0 computes row 0 of
// (p0 = own, p1 = partner), h = 1 row 1 of (p0 = partner, p1 = own). Both are the row-0 chain
// with the row's coefficients and operands selected per lane, so there is no divergent branch.
// CL: -1 no control; 0 control on level 0 (only .y); c >= 1 control on pair-index bit c-1.
// `on` = false keeps this lane's values (a control on another lane bit that is 0 here); every
// lane still shuffles.
template <int KL, int CL>
LYTH_D void split_gate(const U8 &m, int h, int lm, bool on, float2 (&X)[1 << (KL - 1)],
                       float2 (&Y)[1 << (KL - 1)]) {
    const U8 r{h ? m.cr : m.ar, h ? m.ci : m.ai, h ? m.dr : m.br, h ? m.di : m.bi, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        float2 oX, oY;
        oX.x = __shfl_xor_sync(0xffffffffu, X[i].x, lm);
        oX.y = __shfl_xor_sync(0xffffffffu, X[i].y, lm);
        oY.x = __shfl_xor_sync(0xffffffffu, Y[i].x, lm);
        oY.y = __shfl_xor_sync(0xffffffffu, Y[i].y, lm);
        if (CL >= 1 && !(i & (1 << (CL - 1)))) continue;
        if (CL == 0) {
            float a, b;
            row0(r, h ? oX.y : X[i].y, h ? oY.y : Y[i].y, h ? X[i].y : oX.y, h ? Y[i].y : oY.y, a, b);
            if (on) { X[i].y = a; Y[i].y = b; }
        } else {
            float2 a, b;
            row0_2(r, h ? oX : X[i], h ? oY : Y[i], h ? X[i] : oX, h ? Y[i] : oY, a, b);
            if (on) { X[i] = a; Y[i] = b; }
        }
    }
}
template <int KL, int CL = -1>
LYTH_D void dispatch_split(int c, const U8 &m, int h, int lm, bool on, float2 (&X)[1 << (KL - 1)],
                           float2 (&Y)[1 << (KL - 1)]) {
    if constexpr (CL < KL) {
        if (c == CL) split_gate<KL, CL>(m, h, lm, on, X, Y);
        else dispatch_split<KL, CL + 1>(c, m, h, lm, on, X, Y);
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
                dispatch_split<KL>(fg.c, m, h, 16, true, X, Y);
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

// ------------------------------------------------------------------ the tile pass
// For states of 2^14 amplitudes and more. The register pass above loads a whole tuple, computes
// and stores, so at most its resident warps' loads are in flight, and it holds at most 6 qubits.
// The tile pass moves the state through shared memory in tiles and applies a group of up to 13
// qubits per pass:
//
//  * a tile is 2^13 amplitudes whose indices differ in 13 "tile bits": address bits 0..4 (128
//    contiguous bytes of each component) and eight more -- the group's bits above bit 4 (at most
//    eight) filled up with the lowest free bits. A group's whole gate list therefore runs on data
//    in shared memory: one HBM pass per group, whatever its size.
//  * one persistent CTA per SM, 16 warps in two groups of 8 that take alternate tiles from a
//    3-stage ring (64 KiB a stage: re and im). A tile arrives as one to sixteen rank-5 tensor-map
//    boxes per component (cp.async.bulk.tensor.5d, completion on an mbarrier; dimension 0 = address
//    bits 0..4, one further dimension per range of consecutive tile bits, iterated boxes beyond
//    four ranges; no multicast), stored with the 128-byte swizzle: in every 1 KiB of shared memory
//    the 16-byte chunk index of a word is XOR'ed with its 128-byte row index.
//  * the group's gates run in segments: a segment's gates target at most five "register levels" --
//    address bits 0 and 1 (the four words of one 16-byte chunk) and up to three more tile bits.
//    Per segment a thread reads its 32 amplitudes with eight 128-bit shared loads per component,
//    applies the segment's gates in registers (the packed chains of the register pass: pairs
//    along address bit 0, fma.rn.f32x2 on every other level), writes them back in place, and the
//    group synchronises before the next segment reads with its own layout. The eight tile bits
//    that are not register levels are the thread's lane and warp bits; lanes 0..2 take bits whose
//    swizzled chunks differ, so every quarter-warp's 128-bit access covers all 32 banks. A control
//    on a lane or warp bit is a predicate: all of a thread's amplitudes share its value.
//  * after the last segment every thread fences its shared-memory writes for the async proxy, the
//    group synchronises, and warp 0 of the group stores the tile back with the same boxes
//    (cp.async.bulk.tensor store, bulk group), waits until the store has read the stage, and
//    issues the tile three ahead into it.
//  * with no gates and each tile bit written at its image under a permutation of tile bits, the
//    same kernel permutes the state in place (every tile maps onto itself): the read-out's
//    permutation passes.
//  * every wait is bounded (mbar.cuh); a group decides together (bar.red.and) whether its tile
//    arrived, so no warp is left at a group barrier; before the block leaves, its stores have
//    completed and every armed load has landed (bounded).
//
// The arithmetic per amplitude is the unfused passes' chain in circuit order, so the result is
// bit-identical to them whatever the segments.
constexpr int kTpTileBits = 13;
constexpr int kTpTile = 1 << kTpTileBits;            // amplitudes per tile
constexpr int kTpRegs = 5;                           // register levels: 32 amplitudes per thread
constexpr int kTpLaneBits = 5;
constexpr int kTpWarpBits = kTpTileBits - kTpLaneBits - kTpRegs;  // 3
constexpr int kTpGroupWarps = 1 << kTpWarpBits;      // 8 warps per tile
constexpr int kTpGroups = 2;                         // consumer groups, alternate tiles
constexpr int kTpStages = 3;
constexpr int kTpThreads = kTpGroups * kTpGroupWarps * 32;
constexpr int kTpHighBits = kTpTileBits - 5;         // group bits above bit 4 a tile holds
constexpr int kTpMaxBoxes = 16;
constexpr uint32_t kTpMinBits = 14;                  // local bits from which the tile pass runs
constexpr uint32_t kTpCompBytes = kTpTile * (uint32_t)sizeof(float);
constexpr uint32_t kTpStageBytes = 2 * kTpCompBytes;
constexpr int kTpBars = kTpStages * kTpGroups;
constexpr size_t kTpSmem = 1024 + (size_t)kTpStages * kTpStageBytes + kTpBars * sizeof(uint64_t) +
                           2 * kTpBars * sizeof(uint32_t);

// A segment: shared-memory word images (swizzled word offsets) of the thread's lane bits, warp
// bits and register levels 2..4 (levels 0 and 1 are address bits 0 and 1: words +1, +2), and its
// gates [g0, g1).
struct TpSeg {
    uint32_t lane_img[kTpLaneBits], warp_img[kTpWarpBits], reg_img[3];
    uint16_t g0, g1;
};
// A gate of the tile pass: case_ = T * 8 + C + 1 (target register level T, control register level
// C or -1); cl = a control on lane bit cl (0..4) or warp bit cl - 5 (5..7), else -1.
struct TpGate {
    int16_t case_;
    int8_t cl, pad;
    float m[8];
};
struct TpPlan {
    uint32_t tile_bits[kTpTileBits];  // ascending
    uint32_t dim_lo[5], dim_len[5], dim_box[5];
    uint32_t nbox, box_words;
    uint64_t box_off[kTpMaxBoxes];
    uint64_t ntiles;
    uint32_t nseg, ngates;
    uint32_t permute;                                                   // a permutation pass
    uint32_t wlane_img[kTpLaneBits], wwarp_img[kTpWarpBits], wreg_img[kTpRegs];  // its write images
    TpSeg segs[kFuseMaxGates];
    TpGate gates[kFuseMaxGates];
};

__device__ int g_fused_error;

LYTH_D uint64_t tp_tile_base(const TpPlan &P, uint64_t tile) {
    uint64_t b = tile;
#pragma unroll
    for (int k = 0; k < kTpTileBits; k++) b = insert_bit(b, P.tile_bits[k], 0);
    return b;
}
LYTH_D float4 lds128(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a) : "memory");
    return v;
}
LYTH_D void sts128(uint32_t a, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
LYTH_D void sts32(uint32_t a, float v) { asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory"); }
LYTH_D void group_sync(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(kTpGroupWarps * 32) : "memory"); }
// Every thread of the group passes `p`; all get the AND (a barrier: all of them must arrive).
LYTH_D bool group_all(int id, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\t"
        "setp.ne.u32 a, %1, 0;\n\t"
        "bar.red.and.pred b, %2, %3, a;\n\t"
        "selp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "n"(kTpGroupWarps * 32)
        : "memory");
    return r != 0;
}

// Box coordinates of box b of the tile whose first amplitude is `base`.
LYTH_D void tp_coords(const TpPlan &P, uint64_t base, uint32_t b, int (&c)[5]) {
    const uint64_t a = base + P.box_off[b];
#pragma unroll
    for (int k = 0; k < 5; k++) c[k] = (int)((a >> P.dim_lo[k]) & ((1ull << P.dim_len[k]) - 1));
}
// Warp-wide: load tile t into the stage at (sre, sre + kTpCompBytes), completing on `bar`.
LYTH_D void tp_load(const TpPlan &P, const CUtensorMap *tre, const CUtensorMap *tim, uint64_t t, uint32_t sre,
                    uint32_t bar, int lane) {
    if (lane == 0) mbar_expect_tx(bar, kTpStageBytes);
    __syncwarp();
    if ((uint32_t)lane < P.nbox) {
        int c[5];
        tp_coords(P, tp_tile_base(P, t), (uint32_t)lane, c);
        const uint32_t w = (uint32_t)lane * P.box_words * (uint32_t)sizeof(float);
        tensor_load_5d(sre + w, tre, c[0], c[1], c[2], c[3], c[4], bar);
        tensor_load_5d(sre + kTpCompBytes + w, tim, c[0], c[1], c[2], c[3], c[4], bar);
    }
}
// Warp-wide: store the stage back to tile t (one bulk group per lane, committed).
LYTH_D void tp_store(const TpPlan &P, const CUtensorMap *tre, const CUtensorMap *tim, uint64_t t, uint32_t sre,
                     int lane) {
    if ((uint32_t)lane < P.nbox) {
        int c[5];
        tp_coords(P, tp_tile_base(P, t), (uint32_t)lane, c);
        const uint32_t w = (uint32_t)lane * P.box_words * (uint32_t)sizeof(float);
        tensor_store_5d(tre, c[0], c[1], c[2], c[3], c[4], sre + w);
        tensor_store_5d(tim, c[0], c[1], c[2], c[3], c[4], sre + kTpCompBytes + w);
    }
    bulk_commit();
}

#define LYTH_TP_REG(T, C) \
    case (T) * 8 + (C) + 1: gate_case<kTpRegs, T, C>(m, X, Y); break;
#define LYTH_TP_REG_T(T) \
    LYTH_TP_REG(T, -1) LYTH_TP_IF(T, 0) LYTH_TP_IF(T, 1) LYTH_TP_IF(T, 2) LYTH_TP_IF(T, 3) LYTH_TP_IF(T, 4)
// (T, C) with C == T never occurs; its label maps to no work
#define LYTH_TP_IF(T, C) \
    case (T) * 8 + (C) + 1: if constexpr ((T) != (C)) gate_case<kTpRegs, T, ((T) != (C) ? (C) : -1)>(m, X, Y); break;

template <bool PERMUTE>
__global__ void __launch_bounds__(kTpThreads, 1)
    tile_pass_kernel(const __grid_constant__ TpPlan P, const __grid_constant__ CUtensorMap tre,
                     const __grid_constant__ CUtensorMap tim) {
    constexpr int NP = 1 << (kTpRegs - 1);  // float2 pairs per thread
    extern __shared__ uint8_t tp_raw[];
    const uint32_t raw = smem_u32(tp_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;  // 1 KiB aligned: the 128-byte swizzle's period
    uint64_t *bars = reinterpret_cast<uint64_t *>(tp_raw + (ring - raw) + (size_t)kTpStages * kTpStageBytes);
    uint32_t *n_armed = reinterpret_cast<uint32_t *>(bars + kTpBars);
    uint32_t *n_used = n_armed + kTpBars;
    // Tiles of this CTA: t_j = blockIdx.x + j * gridDim.x, in stage j % 3, taken by group j % 2.
    // A tile's arrival is signalled on the barrier of its (stage, group): a group consumes the
    // uses of its barriers in order, so it never waits more than one phase ahead.
    auto bar_of = [&](uint64_t j) { return (uint32_t)((j % kTpStages) * kTpGroups + (j % kTpGroups)); };
    auto full = [&](uint64_t j) { return smem_u32(bars + bar_of(j)); };
    auto full_parity = [&](uint64_t j) { return (uint32_t)(j / kTpBars) & 1u; };
    auto stage = [&](uint64_t j) { return ring + (uint32_t)(j % kTpStages) * kTpStageBytes; };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / kTpGroupWarps, wid = warp % kTpGroupWarps;
    const int bar_id = 1 + grp;
    const uint64_t ntiles = P.ntiles > blockIdx.x ? (P.ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    if (warp == 0) {
        if (lane == 0) {
            for (int b = 0; b < kTpBars; b++) {
                mbar_init(smem_u32(bars + b), 1);
                n_armed[b] = 0;
                n_used[b] = 0;
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        for (uint32_t j = 0; j < (uint32_t)kTpStages && j < ntiles; j++) {
            tp_load(P, &tre, &tim, blockIdx.x + (uint64_t)j * gridDim.x, stage(j), full(j), lane);
            if (lane == 0) n_armed[bar_of(j)]++;
        }
    }
    __syncthreads();

    for (uint64_t j = grp; j < ntiles; j += kTpGroups) {
        const uint64_t t = blockIdx.x + j * gridDim.x;
        const bool ok = mbar_wait(full(j), full_parity(j), &g_fused_error);
        if (!group_all(bar_id, ok)) break;  // the whole group leaves together
        if (wid == 0 && lane == 0) n_used[bar_of(j)]++;
        const uint32_t sre = stage(j), sim = sre + kTpCompBytes;
        for (uint32_t s = 0; s < P.nseg; s++) {
            const TpSeg &sg = P.segs[s];
            uint32_t base = 0;
#pragma unroll
            for (int b = 0; b < kTpLaneBits; b++)
                if ((lane >> b) & 1) base ^= sg.lane_img[b];
#pragma unroll
            for (int b = 0; b < kTpWarpBits; b++)
                if ((wid >> b) & 1) base ^= sg.warp_img[b];
            uint32_t ri[3];
#pragma unroll
            for (int l = 0; l < 3; l++) {
                ri[l] = sg.reg_img[l];
                asm volatile("" : "+r"(ri[l]));
            }
            // word of chunk q (register levels 2..4 = the bits of q), as a byte offset
            auto addr = [&](int q) {
                uint32_t a = base;
#pragma unroll
                for (int l = 0; l < 3; l++)
                    if ((q >> l) & 1) a ^= ri[l];
                return a * (uint32_t)sizeof(float);
            };
            float2 X[NP], Y[NP];
#pragma unroll
            for (int q = 0; q < NP / 2; q++) {
                const uint32_t a = addr(q);
                const float4 vr = lds128(sre + a), vi = lds128(sim + a);
                X[2 * q] = make_float2(vr.x, vr.y);
                X[2 * q + 1] = make_float2(vr.z, vr.w);
                Y[2 * q] = make_float2(vi.x, vi.y);
                Y[2 * q + 1] = make_float2(vi.z, vi.w);
            }
            if constexpr (PERMUTE) {
                // every thread has read before any writes: the images are other threads' words
                group_sync(bar_id);
                uint32_t wbase = 0;
#pragma unroll
                for (int b = 0; b < kTpLaneBits; b++)
                    if ((lane >> b) & 1) wbase ^= P.wlane_img[b];
#pragma unroll
                for (int b = 0; b < kTpWarpBits; b++)
                    if ((wid >> b) & 1) wbase ^= P.wwarp_img[b];
#pragma unroll
                for (int q = 0; q < NP / 2; q++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        uint32_t a = wbase;
                        if (e & 1) a ^= P.wreg_img[0];
                        if (e & 2) a ^= P.wreg_img[1];
#pragma unroll
                        for (int l = 0; l < 3; l++)
                            if ((q >> l) & 1) a ^= P.wreg_img[2 + l];
                        const float2 x = X[2 * q + (e >> 1)], y = Y[2 * q + (e >> 1)];
                        sts32(sre + a * (uint32_t)sizeof(float), (e & 1) ? x.y : x.x);
                        sts32(sim + a * (uint32_t)sizeof(float), (e & 1) ? y.y : y.x);
                    }
            } else {
                for (uint32_t g = sg.g0; g < sg.g1; g++) {
                    const TpGate &tg = P.gates[g];
                    const bool on = tg.cl < 0 || (tg.cl < kTpLaneBits ? ((lane >> tg.cl) & 1)
                                                                      : ((wid >> (tg.cl - kTpLaneBits)) & 1));
                    if (!on) continue;
                    const U8 m{tg.m[0], tg.m[1], tg.m[2], tg.m[3], tg.m[4], tg.m[5], tg.m[6], tg.m[7]};
                    switch (tg.case_) {
                        LYTH_TP_REG_T(0) LYTH_TP_REG_T(1) LYTH_TP_REG_T(2) LYTH_TP_REG_T(3) LYTH_TP_REG_T(4)
                        default: break;
                    }
                }
#pragma unroll
                for (int q = 0; q < NP / 2; q++) {
                    const uint32_t a = addr(q);
                    sts128(sre + a, make_float4(X[2 * q].x, X[2 * q].y, X[2 * q + 1].x, X[2 * q + 1].y));
                    sts128(sim + a, make_float4(Y[2 * q].x, Y[2 * q].y, Y[2 * q + 1].x, Y[2 * q + 1].y));
                }
            }
            if (s + 1 < P.nseg) group_sync(bar_id);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> the store
        group_sync(bar_id);
        if (wid == 0) {
            tp_store(P, &tre, &tim, t, sre, lane);
            bulk_wait_read0();  // the store has read the stage: it may be refilled
            __syncwarp();
            if (j + kTpStages < ntiles) {
                tp_load(P, &tre, &tim, t + (uint64_t)kTpStages * gridDim.x, sre, full(j + kTpStages), lane);
                if (lane == 0) n_armed[bar_of(j + kTpStages)]++;
            }
        }
    }
    if (wid == 0) bulk_wait0();  // this warp's stores have completed
    // Every armed tile has landed before the block may leave. Normally each was consumed; after
    // a timed-out wait, one use per barrier may be outstanding (bounded wait for it).
    __syncthreads();
    if (threadIdx.x == 0)
        for (int b = 0; b < kTpBars; b++)
            if (n_armed[b] != n_used[b]) mbar_wait(smem_u32(bars + b), (n_armed[b] - 1u) & 1u, &g_fused_error);
}
#undef LYTH_TP_REG
#undef LYTH_TP_REG_T
#undef LYTH_TP_IF

// ---- host planning
// The swizzled word of a logical word bit w: the 128-byte swizzle XORs word bits 2..4 (the 16-byte
// chunk) with bits 5..7 (the row within 1 KiB). XOR-ing images of disjoint bits gives the word.
static uint32_t tp_img(uint32_t w) { return (1u << w) ^ ((w >= 5 && w < 8) ? (1u << (w - 3)) : 0u); }

// The tile of a group (its bits `gbits`) over L local bits: tile bits, tensor-map dimensions and
// boxes, and each tile bit's logical word position wpos[] (bits 0..4 = address bits 0..4, then the
// boxes' dimensions, then the iterated bits). False when the group does not fit a tile.
static bool tp_layout(const uint32_t *gbits, int k, uint32_t L, TpPlan &P, int *wpos) {
    if (L < kTpMinBits || L > 48) return false;
    bool tile[64] = {false};
    int cnt = 5, nhigh = 0;
    for (int b = 0; b < 5; b++) tile[b] = true;
    for (int l = 0; l < k; l++) {
        const uint32_t b = gbits[l];
        if (b >= L) return false;
        if (!tile[b]) { tile[b] = true; cnt++; nhigh++; }
    }
    if (nhigh > kTpHighBits) return false;
    for (uint32_t b = 5; b < L && cnt < kTpTileBits; b++)
        if (!tile[b]) { tile[b] = true; cnt++; }
    if (cnt != kTpTileBits) return false;
    struct Range { uint32_t lo, len; };
    Range rg[kTpHighBits];
    int nr = 0;
    for (uint32_t b = 5; b < L;) {
        if (!tile[b]) { b++; continue; }
        uint32_t e = b;
        while (e < L && tile[e]) e++;
        rg[nr++] = {b, e - b};
        b = e;
    }
    bool iter[kTpHighBits] = {false};
    for (int kept = nr; kept > 4; kept--) {  // iterate the smallest range (ties: the highest)
        int pick = -1;
        for (int i = 0; i < nr; i++)
            if (!iter[i] && (pick < 0 || rg[i].len < rg[pick].len || (rg[i].len == rg[pick].len && rg[i].lo > rg[pick].lo)))
                pick = i;
        iter[pick] = true;
    }
    memset(P.dim_lo, 0, sizeof P.dim_lo);
    memset(P.dim_len, 0, sizeof P.dim_len);
    memset(P.dim_box, 0, sizeof P.dim_box);
    int nd = 1;
    P.dim_box[0] = 5;
    for (int i = 0; i < nr; i++)
        if (!iter[i]) { P.dim_lo[nd] = rg[i].lo; P.dim_box[nd] = rg[i].len; nd++; }
    for (int d = 0; d < nd; d++) {
        uint32_t next = L;
        for (int q = 0; q < nd; q++)
            if (P.dim_lo[q] > P.dim_lo[d] && P.dim_lo[q] < next) next = P.dim_lo[q];
        P.dim_len[d] = next - P.dim_lo[d];
        if (P.dim_len[d] > 31 || P.dim_len[d] < P.dim_box[d]) return false;
    }
    int w = 0;
    for (uint32_t b = 0; b < 5; b++) wpos[b] = w++;
    for (int d = 1; d < nd; d++)
        for (uint32_t i = 0; i < P.dim_box[d]; i++) wpos[P.dim_lo[d] + i] = w++;
    P.box_words = 1u << w;
    uint32_t it[kTpHighBits];
    int nit = 0;
    for (int i = 0; i < nr; i++)
        if (iter[i])
            for (uint32_t x = 0; x < rg[i].len; x++) { it[nit] = rg[i].lo + x; wpos[it[nit]] = w++; nit++; }
    if (w != kTpTileBits || P.box_words < 256 || (1 << nit) > kTpMaxBoxes) return false;
    P.nbox = 1u << nit;
    for (uint32_t bx = 0; bx < P.nbox; bx++) {
        uint64_t off = 0;
        for (int i = 0; i < nit; i++)
            if ((bx >> i) & 1) off += 1ull << it[i];
        P.box_off[bx] = off;
    }
    int n = 0;
    for (uint32_t b = 0; b < L && n < kTpTileBits; b++)
        if (tile[b]) P.tile_bits[n++] = b;
    P.ntiles = 1ull << (L - kTpTileBits);
    return true;
}

// Whether register levels (address bits, by their word positions) leave every quarter-warp's
// 128-bit access conflict-free: for each chunk bit i, word bit 2+i or 5+i must be left to a lane.
static bool tp_regs_ok(const uint32_t *regs, int n, const int *wpos) {
    bool has[kTpTileBits] = {false};
    for (int i = 0; i < n; i++) has[wpos[regs[i]]] = true;
    for (int i = 0; i < 3; i++)
        if (has[2 + i] && has[5 + i]) return false;
    return true;
}

// Thread mapping of a segment whose extra register levels are R (tile address bits, not 0 or 1):
// levels = [0, 1, R..., pads], lanes 0..2 = one of word bits 2+i / 5+i each, then the rest.
struct TpMap {
    uint32_t reg[kTpRegs], lane[kTpLaneBits], warp[kTpWarpBits];
};
static bool tp_map(const TpPlan &P, const int *wpos, const uint32_t *R, int nR, TpMap &M) {
    uint32_t regs[kTpRegs] = {0, 1};
    int n = 2;
    for (int i = 0; i < nR; i++) regs[n++] = R[i];
    auto in = [&](uint32_t b, const uint32_t *v, int m) {
        for (int i = 0; i < m; i++)
            if (v[i] == b) return true;
        return false;
    };
    // pads: tile bits at word positions 8..12 (they bear on no chunk bit), lowest first
    for (int wp = 8; wp < kTpTileBits && n < kTpRegs; wp++)
        for (int t = 0; t < kTpTileBits; t++) {
            const uint32_t b = P.tile_bits[t];
            if (wpos[b] == wp && !in(b, regs, n)) { regs[n++] = b; break; }
        }
    if (n != kTpRegs || !tp_regs_ok(regs + 2, kTpRegs - 2, wpos)) return false;
    uint32_t by_w[kTpTileBits];
    for (int t = 0; t < kTpTileBits; t++) by_w[wpos[P.tile_bits[t]]] = P.tile_bits[t];
    uint32_t used[kTpTileBits];
    int nu = 0;
    for (int i = 0; i < kTpRegs; i++) used[nu++] = regs[i];
    for (int i = 0; i < 3; i++) {
        uint32_t b = by_w[2 + i];
        if (in(b, regs, kTpRegs)) b = by_w[5 + i];
        if (in(b, used, nu)) return false;
        M.lane[i] = b;
        used[nu++] = b;
    }
    int li = 3, wi = 0;
    for (int wp = 0; wp < kTpTileBits; wp++) {
        const uint32_t b = by_w[wp];
        if (in(b, used, nu)) continue;
        if (li < kTpLaneBits) M.lane[li++] = b;
        else M.warp[wi++] = b;
        used[nu++] = b;
    }
    if (li != kTpLaneBits || wi != kTpWarpBits) return false;
    for (int i = 0; i < kTpRegs; i++) M.reg[i] = regs[i];
    return true;
}

static void tp_fill_seg(const TpMap &M, const int *wpos, TpSeg &S) {
    for (int b = 0; b < kTpLaneBits; b++) S.lane_img[b] = tp_img((uint32_t)wpos[M.lane[b]]);
    for (int b = 0; b < kTpWarpBits; b++) S.warp_img[b] = tp_img((uint32_t)wpos[M.warp[b]]);
    for (int l = 0; l < 3; l++) S.reg_img[l] = tp_img((uint32_t)wpos[M.reg[2 + l]]);
}

// The tile-pass plan of a fused group over L local bits: layout, then segments (greedy in gate
// order: a gate whose target is not yet a register level adds it while there is room and the
// levels stay conflict-free; else the segment closes).
static bool plan_tile(const FusedGroup &g, uint32_t L, TpPlan &P) {
    if (g.k < 1 || g.k > kFuseMaxQubits || g.ngates > (uint32_t)kFuseMaxGates) return false;
    memset(&P, 0, sizeof P);
    int wpos[64];
    for (int i = 0; i < 64; i++) wpos[i] = -1;
    if (!tp_layout(g.bits, g.k, L, P, wpos)) return false;
    uint32_t R[3];
    int nR = 0;
    uint32_t g0 = 0;
    auto close = [&](uint32_t g1) -> bool {
        TpMap M;
        if (!tp_map(P, wpos, R, nR, M)) return false;
        TpSeg &S = P.segs[P.nseg++];
        tp_fill_seg(M, wpos, S);
        S.g0 = (uint16_t)g0;
        S.g1 = (uint16_t)g1;
        for (uint32_t i = g0; i < g1; i++) {
            const FusedGate &fg = g.gates[i];
            TpGate &tg = P.gates[i];
            const uint32_t tb = g.bits[fg.t];
            int T = -1, C = -1;
            tg.cl = -1;
            for (int l = 0; l < kTpRegs; l++) if (M.reg[l] == tb) T = l;
            if (T < 0) return false;
            if (fg.c >= 0) {
                const uint32_t cb = g.bits[fg.c];
                for (int l = 0; l < kTpRegs; l++) if (M.reg[l] == cb) C = l;
                if (C < 0) {
                    for (int b = 0; b < kTpLaneBits; b++) if (M.lane[b] == cb) tg.cl = (int8_t)b;
                    for (int b = 0; b < kTpWarpBits; b++) if (M.warp[b] == cb) tg.cl = (int8_t)(kTpLaneBits + b);
                    if (tg.cl < 0) return false;
                }
            }
            tg.case_ = (int16_t)(T * 8 + C + 1);
            tg.pad = 0;
            memcpy(tg.m, fg.m, sizeof tg.m);
        }
        return true;
    };
    for (uint32_t i = 0; i < g.ngates; i++) {
        const uint32_t t = g.bits[g.gates[i].t];
        bool have = t < 2;
        for (int r = 0; r < nR; r++) have = have || R[r] == t;
        if (have) continue;
        if (nR < 3) {
            R[nR] = t;
            if (tp_regs_ok(R, nR + 1, wpos)) { nR++; continue; }
        }
        if (!close(i)) return false;
        g0 = i;
        R[0] = t;
        nR = 1;
    }
    if (!close(g.ngates)) return false;
    P.ngates = g.ngates;
    return true;
}

// A permutation pass over the tile holding `src`: one segment with no gates, each tile bit written
// at its image (src[j] -> dst[j], the other tile bits in place).
static bool plan_tile_permute(const uint32_t *src, const uint32_t *dst, int k, uint32_t L, TpPlan &P) {
    memset(&P, 0, sizeof P);
    int wpos[64];
    for (int i = 0; i < 64; i++) wpos[i] = -1;
    if (k < 1 || k > kTpTileBits || !tp_layout(src, k, L, P, wpos)) return false;
    TpMap M;
    if (!tp_map(P, wpos, nullptr, 0, M)) return false;
    auto image = [&](uint32_t a) {
        for (int j = 0; j < k; j++)
            if (src[j] == a) return dst[j];
        return a;
    };
    for (int j = 0; j < k; j++)
        if (wpos[dst[j]] < 0) return false;  // an image outside the tile
    TpSeg &S = P.segs[P.nseg++];
    tp_fill_seg(M, wpos, S);
    S.g0 = S.g1 = 0;
    for (int b = 0; b < kTpLaneBits; b++) P.wlane_img[b] = tp_img((uint32_t)wpos[image(M.lane[b])]);
    for (int b = 0; b < kTpWarpBits; b++) P.wwarp_img[b] = tp_img((uint32_t)wpos[image(M.warp[b])]);
    for (int l = 0; l < kTpRegs; l++) P.wreg_img[l] = tp_img((uint32_t)wpos[image(M.reg[l])]);
    P.permute = 1;
    return true;
}

// The two tensor maps of a tile plan (re and im over 2^L f32 amplitudes), 128-byte swizzle.
// Unused dimensions have extent 1.
static bool encode_tile_maps(const TpPlan &P, uint32_t L, float *re, float *im, CUtensorMap &tre, CUtensorMap &tim) {
    PFN_encode_tiled enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[5], strides[4];
    cuuint32_t box[5], estr[5] = {1, 1, 1, 1, 1};
    for (int k = 0; k < 5; k++) {
        const bool used = P.dim_len[k] > 0;
        dims[k] = used ? (1ull << P.dim_len[k]) : 1;
        box[k] = used ? (1u << P.dim_box[k]) : 1;
        if (k > 0) strides[k - 1] = used ? (1ull << P.dim_lo[k]) * sizeof(float) : (1ull << L) * sizeof(float);
    }
    auto one = [&](CUtensorMap &map, float *base) {
        return enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    return one(tre, re) && one(tim, im);
}

static int launch_tile(const TpPlan &P, uint32_t L, float *re, float *im, cudaStream_t s) {
    CUtensorMap tre, tim;
    memset(&tre, 0, sizeof tre);
    memset(&tim, 0, sizeof tim);
    if (!encode_tile_maps(P, L, re, im, tre, tim)) return LYTH_E_UNSUPPORTED;
    static bool attr_done[2][64] = {{false}};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LYTH_E_INVALID;
    const int pm = P.permute ? 1 : 0;
    if (dev >= 0 && dev < 64 && !attr_done[pm][dev]) {
        const cudaError_t e = pm ? cudaFuncSetAttribute(tile_pass_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTpSmem)
                                 : cudaFuncSetAttribute(tile_pass_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTpSmem);
        if (e != cudaSuccess) return status_of(e);
        attr_done[pm][dev] = true;
    }
    const uint64_t sms = (uint64_t)device_sms();
    const unsigned grid = (unsigned)(P.ntiles < sms ? P.ntiles : sms);
    if (pm) tile_pass_kernel<true><<<grid, kTpThreads, kTpSmem, s>>>(P, tre, tim);
    else tile_pass_kernel<false><<<grid, kTpThreads, kTpSmem, s>>>(P, tre, tim);
    return last_launch_status();
}

int fused_take_device_error() {
    int v = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&v, g_fused_error, sizeof(int));
    if (e != cudaSuccess) return status_of(e);
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_fused_error, &zero, sizeof(int));
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}

// LYTH_FUSED_STAGING=0 sends every group to the register pass (an A/B switch: both are bit-exact;
// groups then hold at most 6 qubits).
static bool staging_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("LYTH_FUSED_STAGING");
        on = !(v && v[0] == '0');
    }
    return on == 1;
}

static bool tile_path(uint64_t len, uint32_t &L) {
    if (!staging_enabled() || !len || (len & (len - 1))) return false;
    L = 0;
    while ((1ull << L) < len) L++;
    return L >= kTpMinBits;
}

bool fused_fits(uint64_t len, const uint32_t *bits, int k) {
    if (k < 1 || k > kFuseMaxQubits) return false;
    uint32_t L = 0;
    if (!tile_path(len, L)) return k <= kFuseRegisterQubits;
    int nhigh = 0;
    for (int l = 0; l < k; l++) nhigh += bits[l] >= 5;
    return nhigh <= kTpHighBits;
}

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s) {
    uint32_t L = 0;
    if (tile_path(len, L) && !(((uintptr_t)re | (uintptr_t)im) & 15)) {
        TpPlan P;
        if (plan_tile(g, L, P)) {
            const int st = launch_tile(P, L, re, im, s);
            if (st != LYTH_E_UNSUPPORTED) return st;
        }
    }
    if (g.k > kFuseRegisterQubits) return LYTH_E_UNSUPPORTED;
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

// A permutation pass: the amplitude at index i moves to the index whose bit dst[j] is bit src[j]
// of i (j < k; dst a permutation of src; other bits unchanged). The tile pass with no gates and
// each tile bit written at its image: the permuted bits are tile bits, so every tile maps onto
// itself and the pass runs in place. LYTH_E_UNSUPPORTED when the state is too small for tiles.
bool permute_supported(uint64_t len, const uint32_t *src, int k) {
    uint32_t L = 0;
    if (k < 1 || k > kPermuteMaxBits || !tile_path(len, L)) return false;
    TpPlan P;
    return plan_tile_permute(src, src, k, L, P);
}

int launch_permute(uint64_t len, const uint32_t *src, const uint32_t *dst, int k, float *re, float *im,
                   cudaStream_t s) {
    uint32_t L = 0;
    if (k < 1 || k > kPermuteMaxBits || !tile_path(len, L) || (((uintptr_t)re | (uintptr_t)im) & 15))
        return LYTH_E_UNSUPPORTED;
    TpPlan P;
    if (!plan_tile_permute(src, dst, k, L, P)) return LYTH_E_UNSUPPORTED;
    return launch_tile(P, L, re, im, s);
}

}  // namespace lyth

// ------------------------------------------------------------------ host-only layout self-test
// The tile pass is correct only if its planner's maps agree. For random groups (and permutations)
// it checks: the boxes' words cover the tile exactly once with the word positions the plan uses,
// the tensor-map coordinates rebuild each box origin (inner coordinate 0: 16-byte aligned), every
// segment's 128-bit accesses cover each word of the tile exactly once and reach all 32 banks in
// every quarter-warp (with the swizzle), each gate's target is a register level of its segment and
// its control where the gate says, and a permutation's writes send each word to its image. No
// device is touched.
namespace lyth {
namespace {
struct SplitMix {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    uint32_t below(uint32_t n) { return (uint32_t)(next() % n); }
};

// The swizzled word of a logical word.
uint32_t phys_word(uint32_t w) { return w ^ (((w >> 5) & 7u) << 2); }

int check_tile(const uint32_t *gbits, int k, const FusedGroup *g, const uint32_t *dst, uint32_t L, const TpPlan &P,
               SplitMix &rng) {
    // logical word -> address offset, from the boxes (dimension order, iterated boxes on top)
    std::vector<int64_t> off_of(kTpTile, -1);
    if (P.box_words * P.nbox != (uint32_t)kTpTile) return -10;
    for (uint32_t b = 0; b < P.nbox; b++)
        for (uint32_t e = 0; e < P.box_words; e++) {
            uint32_t rest = e;
            uint64_t a = P.box_off[b];
            for (int d = 0; d < 5; d++) {
                if (!P.dim_len[d]) continue;
                a += (uint64_t)(rest & ((1u << P.dim_box[d]) - 1)) << P.dim_lo[d];
                rest >>= P.dim_box[d];
            }
            const uint32_t w = b * P.box_words + e;
            if (off_of[w] != -1) return -11;
            off_of[w] = (int64_t)a;
        }
    // the offsets are exactly the tile's index space; dims partition [0, L); strides 16-byte aligned
    std::vector<int> cover(L, 0);
    for (int d = 0; d < 5; d++) {
        if (!P.dim_len[d]) continue;
        if (d > 0 && P.dim_lo[d] < 2) return -12;
        for (uint32_t x = 0; x < P.dim_len[d]; x++) {
            if (P.dim_lo[d] + x >= L) return -13;
            cover[P.dim_lo[d] + x]++;
        }
    }
    for (uint32_t x = 0; x < L; x++)
        if (cover[x] != 1) return -14;
    std::vector<uint8_t> seen(kTpTile, 0);
    for (uint32_t w = 0; w < (uint32_t)kTpTile; w++) {
        uint32_t idx = 0;
        for (int t = 0; t < kTpTileBits; t++)
            if ((off_of[w] >> P.tile_bits[t]) & 1) idx |= 1u << t;
        uint64_t back = 0;
        for (int t = 0; t < kTpTileBits; t++)
            if ((idx >> t) & 1) back |= 1ull << P.tile_bits[t];
        if (back != (uint64_t)off_of[w] || seen[idx]++) return -15;
    }
    uint64_t base = rng.next() % P.ntiles;
    for (int t = 0; t < kTpTileBits; t++) base = insert_bit(base, P.tile_bits[t], 0);
    for (uint32_t b = 0; b < P.nbox; b++) {
        const uint64_t a = base + P.box_off[b];
        uint64_t back = 0;
        for (int d = 0; d < 5; d++) {
            if (!P.dim_len[d]) continue;
            const uint64_t c = (a >> P.dim_lo[d]) & ((1ull << P.dim_len[d]) - 1);
            if (c & ((1ull << P.dim_box[d]) - 1)) return -16;  // a box origin off its box
            back += c << P.dim_lo[d];
        }
        if (back != a) return -17;
    }
    // physical word -> address offset
    std::vector<int64_t> off_phys(kTpTile, -1);
    for (uint32_t w = 0; w < (uint32_t)kTpTile; w++) off_phys[phys_word(w)] = off_of[w];
    // address bit -> its word image, recovered from the logical words
    auto img_of_bit = [&](uint32_t bit) -> uint32_t {
        for (uint32_t w = 0; w < (uint32_t)kTpTile; w++)
            if (off_of[w] == (int64_t)(1ull << bit)) return phys_word(w);
        return 0xffffffffu;
    };
    for (uint32_t s = 0; s < P.nseg; s++) {
        const TpSeg &S = P.segs[s];
        std::vector<uint8_t> hit(kTpTile, 0);
        for (int wp = 0; wp < kTpGroupWarps; wp++)
            for (int q = 0; q < 8; q++) {
                uint32_t chunks[4] = {0, 0, 0, 0};
                for (int lane = 0; lane < 32; lane++) {
                    uint32_t a = 0;
                    for (int b = 0; b < kTpLaneBits; b++) if ((lane >> b) & 1) a ^= S.lane_img[b];
                    for (int b = 0; b < kTpWarpBits; b++) if ((wp >> b) & 1) a ^= S.warp_img[b];
                    for (int l = 0; l < 3; l++) if ((q >> l) & 1) a ^= S.reg_img[l];
                    if (a & 3u || a >= (uint32_t)kTpTile) return -18;
                    for (int e = 0; e < 4; e++) {
                        if (hit[a + e]++) return -19;
                        // element e of the chunk holds address bits 0, 1 = e
                        if ((off_phys[a + e] & 3) != e) return -20;
                    }
                    chunks[lane >> 3] |= 1u << ((a >> 2) & 7u);
                }
                for (int h = 0; h < 4; h++)
                    if (chunks[h] != 0xffu) return -21;  // a quarter-warp reaches 8 distinct chunks
            }
        for (uint32_t i = S.g0; i < S.g1; i++) {
            if (!g) return -22;
            const TpGate &tg = P.gates[i];
            const int T = tg.case_ / 8, C = tg.case_ % 8 - 1;
            auto reg_bit = [&](int l) -> int64_t {
                if (l == 0) return 0;
                if (l == 1) return 1;
                for (uint32_t bit = 0; bit < L; bit++)
                    if (img_of_bit(bit) == S.reg_img[l - 2]) return bit;
                return -1;
            };
            if (reg_bit(T) != (int64_t)g->bits[g->gates[i].t]) return -23;
            int64_t cb = -1;
            if (C >= 0) cb = reg_bit(C);
            if (tg.cl >= 0) {
                if (C >= 0) return -24;
                const uint32_t im = tg.cl < kTpLaneBits ? S.lane_img[tg.cl] : S.warp_img[tg.cl - kTpLaneBits];
                for (uint32_t bit = 0; bit < L; bit++)
                    if (img_of_bit(bit) == im) cb = bit;
            }
            if (cb != (g->gates[i].c >= 0 ? (int64_t)g->bits[g->gates[i].c] : -1)) return -25;
        }
    }
    if (g) {
        uint32_t covered = 0;
        for (uint32_t s = 0; s < P.nseg; s++) {
            if (P.segs[s].g0 != covered) return -26;
            covered = P.segs[s].g1;
        }
        if (covered != g->ngates) return -27;
    }
    if (P.permute) {
        std::vector<uint8_t> hit(kTpTile, 0);
        auto image = [&](uint64_t a) {
            uint64_t o = 0;
            for (uint32_t bit = 0; bit < L; bit++) {
                if (!((a >> bit) & 1)) continue;
                uint32_t to = bit;
                for (int j = 0; j < k; j++)
                    if (gbits[j] == bit) to = dst[j];
                o |= 1ull << to;
            }
            return o;
        };
        const TpSeg &S = P.segs[0];
        for (int wp = 0; wp < kTpGroupWarps; wp++)
            for (int lane = 0; lane < 32; lane++)
                for (int q = 0; q < 8; q++)
                    for (int e = 0; e < 4; e++) {
                        uint32_t r = (uint32_t)e, wr = 0;
                        for (int b = 0; b < kTpLaneBits; b++)
                            if ((lane >> b) & 1) { r ^= S.lane_img[b]; wr ^= P.wlane_img[b]; }
                        for (int b = 0; b < kTpWarpBits; b++)
                            if ((wp >> b) & 1) { r ^= S.warp_img[b]; wr ^= P.wwarp_img[b]; }
                        for (int l = 0; l < 3; l++)
                            if ((q >> l) & 1) { r ^= S.reg_img[l]; wr ^= P.wreg_img[2 + l]; }
                        if (e & 1) wr ^= P.wreg_img[0];
                        if (e & 2) wr ^= P.wreg_img[1];
                        if (wr >= (uint32_t)kTpTile || hit[wr]++) return -28;
                        if (off_phys[wr] != (int64_t)image((uint64_t)off_phys[r])) return -29;
                    }
    }
    return LYTH_OK;
}
}  // namespace
}  // namespace lyth

using namespace lyth;

extern "C" int lyth_b200_fused_layout_selftest(uint64_t seed, uint32_t groups, uint32_t *planned,
                                               uint32_t *boxes) {
    SplitMix rng{seed};
    uint32_t n_planned = 0, n_boxes = 0;
    for (uint32_t it = 0; it < groups; it++) {
        const uint32_t L = kTpMinBits + rng.below(34 - kTpMinBits);
        // at most 8 bits above bit 4, at most 13 in all; a third of the groups on the low bits
        const uint32_t span = (it % 3 == 0) ? (L < 16 ? L : 16) : L;
        FusedGroup g{};
        g.k = 1 + (int32_t)rng.below(kFuseMaxQubits);
        uint64_t used = 0;
        int nhigh = 0, tries = 0;
        for (int l = 0; l < g.k && tries < 1000; tries++) {
            const uint32_t b = rng.below(span);
            if ((used >> b) & 1) continue;
            if (b >= 5 && nhigh == kTpHighBits) continue;
            used |= 1ull << b;
            nhigh += b >= 5;
            g.bits[l++] = b;
        }
        int have = 0;
        for (uint32_t b = 0; b < 64; b++) have += (used >> b) & 1;
        g.k = have;
        g.ngates = 1 + rng.below(kFuseMaxGates);
        for (uint32_t i = 0; i < g.ngates; i++) {
            g.gates[i].t = (int8_t)rng.below((uint32_t)g.k);
            g.gates[i].c = (int8_t)(g.k > 1 && rng.below(2) ? (g.gates[i].t + 1 + rng.below((uint32_t)g.k - 1)) % g.k : -1);
            for (int e = 0; e < 8; e++) g.gates[i].m[e] = 0.0f;
        }
        TpPlan P;
        if (!plan_tile(g, L, P)) return LYTH_E_UNSUPPORTED;  // every such group must plan
        n_planned++;
        n_boxes += P.nbox;
        int st = check_tile(g.bits, g.k, &g, nullptr, L, P, rng);
        if (st) return st;
        // a permutation of up to kPermuteMaxBits of the group's bits (a random cycle)
        const int pk = 1 + (int)rng.below((uint32_t)(g.k < kPermuteMaxBits ? g.k : kPermuteMaxBits));
        uint32_t src[kPermuteMaxBits], dst[kPermuteMaxBits];
        for (int j = 0; j < pk; j++) src[j] = g.bits[j];
        for (int j = 0; j < pk; j++) dst[j] = src[(j + 1) % pk];
        if (!plan_tile_permute(src, dst, pk, L, P)) return LYTH_E_UNSUPPORTED;
        if ((st = check_tile(src, pk, nullptr, dst, L, P, rng))) return st;
    }
    if (planned) *planned = n_planned;
    if (boxes) *boxes = n_boxes;
    return LYTH_OK;
}
