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

// ------------------------------------------------------------------ the staged pass
// For states of 2^14 amplitudes and more. The register pass above loads a whole tuple, computes,
// and stores, so at most its resident warps' loads are in flight: it streams well below HBM
// speed, and a group on the low address bits makes every warp load touch 32 lines. The staged
// pass moves the state through shared memory in tiles instead:
//
//  * a tile is 2^13 amplitudes whose indices differ in 13 "tile bits": 5 lane bits, 5 register
//    levels and 3 warp bits. Lane bits are address bits 0..4, except that when all six group
//    bits are >= 5 the highest one takes lane bit 4: every warp access is then 64 contiguous
//    bytes or more per lane half. Register levels are the group's other bits, filled up to five
//    with the lowest free bits ("batch" levels: independent tuples side by side). Warp bits are
//    the next free bits.
//  * one persistent CTA per SM, 16 warps in two groups of 8 that take alternate tiles. A tile is
//    copied into a 3-stage ring of shared memory, completing on an mbarrier: as 1-D bulk copies
//    of its contiguous runs (cp.async.bulk) when the runs are >= 2 KiB, else as one to eight
//    rank-5 tensor-map boxes (cp.async.bulk.tensor.5d, one box dimension per range of
//    consecutive tile bits; many short runs cost one request each, a box one request for all),
//    never with multicast. Each warp reads its 32
//    amplitudes per lane from shared memory and releases the stage, and warp 0 of the group,
//    once its whole group has read the stage, issues the tile three ahead into it. The gates
//    then run in registers and the results go to global memory directly (coalesced streaming
//    stores). Up to three tiles (192 KiB) are in flight per SM whatever the warps are doing,
//    and no warp is set aside for copies (16 warps x 128 registers fill the register file).
//  * with a group bit on lane bit 4, the two lane halves read disjoint banks: as runs, those
//    whose copy of that bit is 1 sit 16 words further along modulo 32 (a 32-word pad after every
//    two runs, that bit the lowest run-index bit); as boxes, that bit is the box dimension right
//    after address bits 0..3, 16 words.
//  * with no gates and each tile bit stored at its image under a permutation of the group's bits,
//    the same pass permutes the state in place (launch_permute: every tile maps onto itself).
//  * gates on register levels run the packed chains above; a gate on a lane bit fetches both
//    values of each pair from the two lanes by indexed shuffles and computes this lane's row.
//    The arithmetic per amplitude is the same chain in the same order, so the result is
//    bit-identical.
constexpr int kStTileBits = 13;
constexpr int kStTile = 1 << kStTileBits;            // amplitudes per tile
constexpr int kStRegs = 5;                           // register levels: 32 amplitudes per lane
constexpr int kStWarpBits = kStTileBits - 5 - kStRegs;
constexpr int kStGroupWarps = 1 << kStWarpBits;      // consumer warps per tile
constexpr int kStGroups = 2;                         // consumer groups, alternate tiles
constexpr int kStStages = 3;
constexpr int kStConsumers = kStGroups * kStGroupWarps;
constexpr int kStThreads = kStConsumers * 32;      // no separate producer warp
constexpr int kStMaxRuns = 64;
constexpr int kStCompWords = kStTile + 32 * (kStMaxRuns / 2);  // one component of a stage, padded
constexpr size_t kStBufBytes = (size_t)kStStages * 2 * kStCompWords * sizeof(float);
constexpr size_t kStSmem = kStBufBytes + (kStGroups + 1) * kStStages * sizeof(uint64_t) +
                          2 * kStGroups * kStStages * sizeof(uint32_t);
constexpr uint32_t kStMinBits = 14;                  // local bits from which the staged pass runs

// A gate of the staged pass. case_: target register level t and control register level c
// (or -1) as t * 8 + c + 1; 64 + c + 1 for a target on lane bit `lt`. lc: a control on a lane
// bit, or -1.
struct StagedGate {
    int16_t case_;
    int8_t lt, lc;
    float m[8];
};

struct StagedPlan {
    uint32_t tile_bits[kStTileBits];  // the tile's address bits, ascending (for the tile base)
    uint32_t run_bits;                // a run is address bits 0..run_bits-1: 2^run_bits amplitudes
    uint32_t nruns;
    uint32_t lane_w[5], reg_w[kStRegs], warp_w[kStWarpBits];  // shared-memory word weights
    uint32_t lane_addr[5], reg_addr[kStRegs], warp_addr[kStWarpBits];
    // Where each lane / register / warp bit's value is stored: the bit itself, or for a
    // permutation pass its image (a permutation of tile bits keeps every tile in place).
    uint32_t dlane_addr[5], dreg_addr[kStRegs], dwarp_addr[kStWarpBits];
    uint32_t run_word[kStMaxRuns];  // shared-memory word of run r
    // Box copies (tma = 1): dimension k of the tensor maps covers address bits
    // [dim_lo[k], dim_lo[k] + dim_len[k]) and its box the lowest dim_box[k] of them; nbox boxes
    // per component, box b at word b * box_words with the address bits box_off[b] set.
    uint32_t tma;
    uint32_t dim_lo[5], dim_len[5], dim_box[5];
    uint32_t nbox, box_words;
    uint64_t box_off[8];
    uint64_t run_off[kStMaxRuns];   // element offset of run r within a tile
    uint64_t ntiles;
    uint32_t ngates;
    StagedGate gates[kFuseMaxGates];
};

__device__ int g_fused_error;

LYTH_D uint64_t st_tile_base(const StagedPlan &P, uint64_t tile) {
    uint64_t b = tile;
#pragma unroll
    for (int k = 0; k < kStTileBits; k++) b = insert_bit(b, P.tile_bits[k], 0);
    return b;
}

// A gate on a lane bit: lane `lo` holds the pair's p0 and lane `hi` its p1 (lo = this lane with
// the bit clear, hi = with it set); r = this lane's row coefficients in row-0 form. CL as in
// split_gate. Pairs a register control excludes neither shuffle nor compute.
template <int KL, int CL>
LYTH_D void lane_gate(const U8 &r, int lo, int hi, bool on, float2 (&X)[1 << (KL - 1)], float2 (&Y)[1 << (KL - 1)]) {
#pragma unroll
    for (int i = 0; i < (1 << (KL - 1)); i++) {
        if (CL >= 1 && !(i & (1 << (CL - 1)))) continue;
        if (CL == 0) {
            const float p0r = __shfl_sync(0xffffffffu, X[i].y, lo), p0i = __shfl_sync(0xffffffffu, Y[i].y, lo);
            const float p1r = __shfl_sync(0xffffffffu, X[i].y, hi), p1i = __shfl_sync(0xffffffffu, Y[i].y, hi);
            float a, b;
            row0(r, p0r, p0i, p1r, p1i, a, b);
            if (on) { X[i].y = a; Y[i].y = b; }
        } else {
            float2 p0r, p0i, p1r, p1i;
            p0r.x = __shfl_sync(0xffffffffu, X[i].x, lo); p0r.y = __shfl_sync(0xffffffffu, X[i].y, lo);
            p0i.x = __shfl_sync(0xffffffffu, Y[i].x, lo); p0i.y = __shfl_sync(0xffffffffu, Y[i].y, lo);
            p1r.x = __shfl_sync(0xffffffffu, X[i].x, hi); p1r.y = __shfl_sync(0xffffffffu, X[i].y, hi);
            p1i.x = __shfl_sync(0xffffffffu, Y[i].x, hi); p1i.y = __shfl_sync(0xffffffffu, Y[i].y, hi);
            float2 a, b;
            row0_2(r, p0r, p0i, p1r, p1i, a, b);
            if (on) { X[i] = a; Y[i] = b; }
        }
    }
}

#define LYTH_ST_REG(T, C) \
    case (T) * 8 + (C) + 1: gate_case<kStRegs, T, C>(m, X, Y); break;
#define LYTH_ST_REG_T(T) \
    LYTH_ST_REG(T, -1) LYTH_ST_C0(T) LYTH_ST_C1(T) LYTH_ST_C2(T) LYTH_ST_C3(T) LYTH_ST_C4(T)
#define LYTH_ST_C0(T) LYTH_ST_IF(T, 0)
#define LYTH_ST_C1(T) LYTH_ST_IF(T, 1)
#define LYTH_ST_C2(T) LYTH_ST_IF(T, 2)
#define LYTH_ST_C3(T) LYTH_ST_IF(T, 3)
#define LYTH_ST_C4(T) LYTH_ST_IF(T, 4)
// (T, C) with C == T never occurs; its label maps to no work
#define LYTH_ST_IF(T, C) \
    case (T) * 8 + (C) + 1: if constexpr ((T) != (C)) gate_case<kStRegs, T, ((T) != (C) ? (C) : -1)>(m, X, Y); break;
#define LYTH_ST_LANE(C) \
    case 64 + (C) + 1: lane_gate<kStRegs, C>(r, lo, hi, on, X, Y); break;

// Issue tile `t`'s bulk copies into stage `stage` (the whole warp: lane 0 arms the barrier with
// the tile's byte count, every lane issues its share of the runs).
LYTH_D void st_issue(const StagedPlan &P, const CUtensorMap *tre, const CUtensorMap *tim, uint64_t t, float *sre,
                     float *sim, uint32_t bar, const float *re, const float *im, int lane) {
    if (lane == 0) mbar_expect_tx(bar, 2u * kStTile * (uint32_t)sizeof(float));
    __syncwarp();
    const uint64_t base = st_tile_base(P, t);
    if (P.tma) {
        if ((uint32_t)lane < P.nbox) {
            const uint64_t a = base + P.box_off[lane];
            int c[5];
#pragma unroll
            for (int k = 0; k < 5; k++) c[k] = (int)((a >> P.dim_lo[k]) & ((1ull << P.dim_len[k]) - 1));
            const uint32_t w = (uint32_t)lane * P.box_words;
            tensor_load_5d(smem_u32(sre + w), tre, c[0], c[1], c[2], c[3], c[4], bar);
            tensor_load_5d(smem_u32(sim + w), tim, c[0], c[1], c[2], c[3], c[4], bar);
        }
        return;
    }
    const uint32_t run_bytes = (1u << P.run_bits) * (uint32_t)sizeof(float);
    for (uint32_t r = lane; r < P.nruns; r += 32) {
        const uint64_t g = base + P.run_off[r];
        bulk_load(smem_u32(sre + P.run_word[r]), re + g, run_bytes, bar);
        bulk_load(smem_u32(sim + P.run_word[r]), im + g, run_bytes, bar);
    }
}

__global__ void __launch_bounds__(kStThreads, 1)
    staged_fused_kernel(const __grid_constant__ StagedPlan P, const __grid_constant__ CUtensorMap tre,
                        const __grid_constant__ CUtensorMap tim, float *re, float *im) {
    constexpr int NP = 1 << (kStRegs - 1);  // float2 pairs per lane
    extern __shared__ __align__(128) uint8_t st_smem[];
    float *buf = reinterpret_cast<float *>(st_smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(st_smem + kStBufBytes);
    // Tiles of this CTA: t_j = blockIdx.x + j * gridDim.x. Tile j lives in stage j % 3 and is
    // consumed by group j % 2; warp 0 of that group issues tile j + 3 into the same stage once
    // all its warps have read tile j (the stage's `empty` barrier). A tile's arrival is signalled
    // on the barrier of its (stage, group): a group consumes the uses of its barriers in order,
    // so it never waits more than one phase ahead of one it has seen complete, however far the
    // two groups drift apart.
    auto full = [&](uint64_t j) { return smem_u32(bars + (j % kStStages) * kStGroups + (j % kStGroups)); };
    auto full_parity = [&](uint64_t j) { return (uint32_t)(j / (kStStages * kStGroups)) & 1u; };
    auto empty = [&](uint32_t s) { return smem_u32(bars + kStGroups * kStStages + s); };
    auto sre_of = [&](uint32_t s) { return buf + (size_t)s * 2 * kStCompWords; };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / kStGroupWarps, wid = warp % kStGroupWarps;
    const uint64_t ntiles = P.ntiles > blockIdx.x ? (P.ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    // Uses of each full barrier armed and consumed, for the wind-down: every use up to the last
    // has completed except possibly the last armed one, so its parity is unambiguous.
    constexpr int NB = kStStages * kStGroups;
    uint32_t *n_armed = reinterpret_cast<uint32_t *>(bars + (kStGroups + 1) * kStStages);
    uint32_t *n_used = n_armed + NB;
    auto bar_of = [&](uint64_t j) { return (uint32_t)((j % kStStages) * kStGroups + (j % kStGroups)); };
    if (warp == 0) {
        if (lane == 0) {
            for (int b = 0; b < NB; b++) {
                mbar_init(smem_u32(bars + b), 1);
                n_armed[b] = 0;
                n_used[b] = 0;
            }
            for (int s = 0; s < kStStages; s++) mbar_init(empty(s), kStGroupWarps);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        for (uint32_t j = 0; j < (uint32_t)kStStages && j < ntiles; j++) {
            st_issue(P, &tre, &tim, blockIdx.x + (uint64_t)j * gridDim.x, sre_of(j), sre_of(j) + kStCompWords, full(j),
                     re, im, lane);
            if (lane == 0) n_armed[bar_of(j)]++;
        }
    }
    __syncthreads();

    uint32_t lane_s = 0, warp_s = 0;
    uint64_t lane_g = 0, warp_g = 0;
#pragma unroll
    for (int b = 0; b < 5; b++)
        if ((lane >> b) & 1) { lane_s += P.lane_w[b]; lane_g += 1ull << P.dlane_addr[b]; }
#pragma unroll
    for (int b = 0; b < kStWarpBits; b++)
        if ((wid >> b) & 1) { warp_s += P.warp_w[b]; warp_g += 1ull << P.dwarp_addr[b]; }
    for (uint64_t j = grp; j < ntiles; j += kStGroups) {
        const uint64_t t = blockIdx.x + j * gridDim.x;
        const uint32_t stage = (uint32_t)(j % kStStages), phase = (uint32_t)(j / kStStages) & 1u;
        const bool ok = mbar_wait(full(j), full_parity(j), &g_fused_error);
        if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform: the gates below shuffle
        if (wid == 0 && lane == 0) n_used[bar_of(j)]++;
        const float *sre = sre_of(stage);
        const float *sim = sre + kStCompWords;
        uint32_t ss[kStRegs];
#pragma unroll
        for (int l = 0; l < kStRegs; l++) {
            ss[l] = P.reg_w[l];
            asm volatile("" : "+r"(ss[l]));
        }
        float2 X[NP], Y[NP];
#pragma unroll
        for (int i = 0; i < NP; i++) {
            uint32_t o = lane_s + warp_s;
#pragma unroll
            for (int l = 1; l < kStRegs; l++)
                if (i & (1 << (l - 1))) o += ss[l];
            X[i] = make_float2(sre[o], sre[o + ss[0]]);
            Y[i] = make_float2(sim[o], sim[o + ss[0]]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(stage));  // release: the reads above are ordered before
        if (wid == 0 && j + kStStages < ntiles) {
            // refill: wait until the whole group has read this stage, then issue tile j + 3
            const bool free_ok = mbar_wait(empty(stage), phase, &g_fused_error);
            if (!__all_sync(0xffffffffu, free_ok)) break;
            st_issue(P, &tre, &tim, t + (uint64_t)kStStages * gridDim.x, sre_of(stage), sre_of(stage) + kStCompWords,
                     full(j + kStStages), re, im, lane);
            if (lane == 0) n_armed[bar_of(j + kStStages)]++;
        }

        for (uint32_t g = 0; g < P.ngates; g++) {
            const StagedGate &sg = P.gates[g];
            const U8 m{sg.m[0], sg.m[1], sg.m[2], sg.m[3], sg.m[4], sg.m[5], sg.m[6], sg.m[7]};
            const bool on = sg.lc < 0 || ((lane >> sg.lc) & 1);
            if (sg.case_ < 64) {
                if (!on) continue;
                switch (sg.case_) {
                    LYTH_ST_REG_T(0) LYTH_ST_REG_T(1) LYTH_ST_REG_T(2) LYTH_ST_REG_T(3) LYTH_ST_REG_T(4)
                    default: break;
                }
            } else {
                const int h = (lane >> sg.lt) & 1;
                const int lo = lane & ~(1 << sg.lt), hi = lane | (1 << sg.lt);
                const U8 r{h ? m.cr : m.ar, h ? m.ci : m.ai, h ? m.dr : m.br, h ? m.di : m.bi, 0.f, 0.f, 0.f, 0.f};
                switch (sg.case_) {
                    LYTH_ST_LANE(-1) LYTH_ST_LANE(0) LYTH_ST_LANE(1) LYTH_ST_LANE(2) LYTH_ST_LANE(3) LYTH_ST_LANE(4)
                    default: break;
                }
            }
        }

        uint64_t gs[kStRegs];
#pragma unroll
        for (int l = 0; l < kStRegs; l++) {
            gs[l] = 1ull << P.dreg_addr[l];
            asm volatile("" : "+l"(gs[l]));
        }
        const uint64_t base = st_tile_base(P, t) + lane_g + warp_g;
#pragma unroll
        for (int i = 0; i < NP; i++) {
            uint64_t a = base;
#pragma unroll
            for (int l = 1; l < kStRegs; l++)
                if (i & (1 << (l - 1))) a += gs[l];
            __stcs(re + a, X[i].x);
            __stcs(re + a + gs[0], X[i].y);
            __stcs(im + a, Y[i].x);
            __stcs(im + a + gs[0], Y[i].y);
        }
    }
    // Every armed tile has landed before the block may leave. Normally each was consumed; after
    // a timed-out wait, one use per barrier may be outstanding (bounded wait for it).
    __syncthreads();
    if (threadIdx.x == 0)
        for (int b = 0; b < NB; b++)
            if (n_armed[b] != n_used[b]) mbar_wait(smem_u32(bars + b), (n_armed[b] - 1u) & 1u, &g_fused_error);
}
#undef LYTH_ST_REG
#undef LYTH_ST_REG_T
#undef LYTH_ST_C0
#undef LYTH_ST_C1
#undef LYTH_ST_C2
#undef LYTH_ST_C3
#undef LYTH_ST_C4
#undef LYTH_ST_IF
#undef LYTH_ST_LANE

// The staged layout of a group over L local bits (false: the register pass runs instead).
// Box layout of the tile bits (tensor-map copies): dimension 0 = address bits 0..3 (with a lane
// group bit) or the contiguous tile bits from 0, then the lane group bit (so the two lane halves
// sit 16 words apart), then each further range of consecutive tile bits; beyond five dimensions
// the smallest ranges are iterated as separate boxes (at most 8). Fills weight[] (word weight of
// each tile bit) and the plan's dim / box fields; false when the tile does not fit the form.
static bool layout_boxes(const bool *tile, int star, uint32_t L, uint32_t *weight, StagedPlan &P) {
    struct Dim { uint32_t lo, box; };
    Dim d[kStTileBits];
    int nd = 0;
    bool placed[64] = {false};
    uint32_t b0 = 0;
    if (star >= 0) b0 = 4;
    else while (b0 < 8 && tile[b0]) b0++;
    for (uint32_t b = 0; b < b0; b++) if (!tile[b]) return false;
    d[nd++] = {0, b0};
    for (uint32_t b = 0; b < b0; b++) placed[b] = true;
    if (star >= 0) { d[nd++] = {(uint32_t)star, 1}; placed[star] = true; }
    for (uint32_t b = 0; b < 64; b++) {
        if (!tile[b] || placed[b]) continue;
        uint32_t e = b;
        while (e < 64 && tile[e] && !placed[e] && e - b < 8) e++;
        d[nd++] = {b, e - b};
        for (uint32_t x = b; x < e; x++) placed[x] = true;
    }
    uint32_t iter[3];
    int ni = 0;
    while (nd > 5) {  // iterate the smallest range (ties: the highest), never dimension 0 or the star
        int pick = -1;
        for (int k = (star >= 0 ? 2 : 1); k < nd; k++)
            if (pick < 0 || d[k].box < d[pick].box || (d[k].box == d[pick].box && d[k].lo > d[pick].lo)) pick = k;
        if (ni + (int)d[pick].box > 3) return false;
        for (uint32_t i = 0; i < d[pick].box; i++) iter[ni++] = d[pick].lo + i;
        for (int k = pick; k + 1 < nd; k++) d[k] = d[k + 1];
        nd--;
    }
    // coverage: from each dimension's first bit to the next dimension's first bit in address order
    for (int k = 0; k < nd; k++) {
        uint32_t hi = L;
        for (int q = 0; q < nd; q++)
            if (d[q].lo > d[k].lo && d[q].lo < hi) hi = d[q].lo;
        if (hi - d[k].lo < d[k].box || hi - d[k].lo > 31) return false;
        P.dim_lo[k] = d[k].lo;
        P.dim_len[k] = hi - d[k].lo;
        P.dim_box[k] = d[k].box;
    }
    if (d[0].box < 2) return false;  // the inner box must span >= 16 bytes
    for (int k = nd; k < 5; k++) { P.dim_lo[k] = 0; P.dim_len[k] = 0; P.dim_box[k] = 0; }
    uint32_t w = 1;
    for (int k = 0; k < nd; k++)
        for (uint32_t i = 0; i < d[k].box; i++) { weight[d[k].lo + i] = w; w <<= 1; }
    P.box_words = w;
    P.nbox = 1u << ni;
    for (int i = 0; i < ni; i++) weight[iter[i]] = w << i;
    for (uint32_t bx = 0; bx < P.nbox; bx++) {
        uint64_t off = 0;
        for (int i = 0; i < ni; i++)
            if ((bx >> i) & 1) off += 1ull << iter[i];
        P.box_off[bx] = off;
    }
    P.tma = 1;
    return true;
}

// boxes: 0 = runs only, 1 = boxes where runs would be short (< 2 KiB), 2 = boxes where they fit.
static bool plan_staged(const FusedGroup &g, uint32_t L, int boxes, StagedPlan &P) {
    if (L < kStMinBits || g.k < 1 || g.k > kFuseMaxQubits) return false;
    const int k = g.k;
    int use[kFuseMaxQubits] = {0};
    for (uint32_t i = 0; i < g.ngates; i++) {
        use[g.gates[i].t]++;
        if (g.gates[i].c >= 0) use[g.gates[i].c]++;
    }
    bool group[64] = {false};
    for (int l = 0; l < k; l++) group[g.bits[l]] = true;
    int code[kFuseMaxQubits];  // group level -> kernel level (0..4 register, 5 + b lane bit b)
    for (int l = 0; l < k; l++) code[l] = g.bits[l] < 5 ? 5 + (int)g.bits[l] : -1;
    // a sixth group bit >= 5 goes to lane bit 4: the highest one (it splits the fewest runs)
    int nhi = 0, top_l = -1;
    for (int l = 0; l < k; l++)
        if (g.bits[l] >= 5) {
            nhi++;
            if (top_l < 0 || g.bits[l] > g.bits[top_l]) top_l = l;
        }
    const int nstar = nhi > kStRegs ? 1 : 0;
    uint32_t lane_addr[5] = {0, 1, 2, 3, 4};
    bool star[64] = {false};
    if (nstar) {
        lane_addr[4] = g.bits[top_l];
        code[top_l] = 5 + 4;
        star[g.bits[top_l]] = true;
    }
    bool used[64] = {false};
    for (int b = 0; b < 5; b++) used[lane_addr[b]] = true;
    auto next_free = [&]() -> uint32_t {
        for (uint32_t b = 0; b < 64; b++)
            if (!used[b] && !group[b]) { used[b] = true; return b; }
        return 64;
    };
    // register levels: level 0 a batch bit when there is one (no gate touches it, so every gate
    // runs on packed pairs), else the group bit used least
    int regs_l[kStRegs], nreg = 0;
    for (int l = 0; l < k; l++)
        if (code[l] < 0) regs_l[nreg++] = l;
    uint32_t reg_addr[kStRegs];
    int r = 0;
    if (nreg < kStRegs) {
        reg_addr[r++] = next_free();
    } else {
        int best = 0;
        for (int i = 1; i < nreg; i++)
            if (use[regs_l[i]] < use[regs_l[best]]) best = i;
        const int t = regs_l[0]; regs_l[0] = regs_l[best]; regs_l[best] = t;
    }
    for (int i = 0; i < nreg; i++) {
        code[regs_l[i]] = r;
        reg_addr[r++] = g.bits[regs_l[i]];
        used[g.bits[regs_l[i]]] = true;
    }
    while (r < kStRegs) reg_addr[r++] = next_free();
    uint32_t warp_addr[kStWarpBits];
    for (int b = 0; b < kStWarpBits; b++) warp_addr[b] = next_free();

    uint32_t all[kStTileBits];
    int n = 0;
    for (int b = 0; b < 5; b++) all[n++] = lane_addr[b];
    for (int b = 0; b < kStRegs; b++) all[n++] = reg_addr[b];
    for (int b = 0; b < kStWarpBits; b++) all[n++] = warp_addr[b];
    for (int i = 0; i < n; i++)
        if (all[i] >= L) return false;
    for (int i = 1; i < n; i++)
        for (int j = i; j > 0 && all[j - 1] > all[j]; j--) { const uint32_t t = all[j]; all[j] = all[j - 1]; all[j - 1] = t; }
    for (int i = 1; i < n; i++)
        if (all[i] == all[i - 1]) return false;
    bool tile[64] = {false};
    for (int i = 0; i < n; i++) tile[all[i]] = true;
    memset(&P, 0, sizeof P);
    for (int i = 0; i < n; i++) P.tile_bits[i] = all[i];
    uint32_t weight[64] = {0};  // shared-memory word weight of each tile bit
    // Runs of >= 2 KiB copy fastest as plain bulk copies; shorter ones (a tile of many small
    // runs) as tensor-map boxes, one or a few per component.
    uint32_t m_runs = 0;
    while (m_runs < 64 && tile[m_runs] && !star[m_runs]) m_runs++;
    if (boxes == 1 && m_runs >= 9) boxes = 0;
    if (!(boxes && layout_boxes(tile, nstar ? (int)lane_addr[4] : -1, L, weight, P))) {
        // runs: address bits 0..m-1, all tile bits and none the lane group bit
        P.tma = 0;
        uint32_t m = 0;
        while (m < 64 && tile[m] && !star[m]) m++;
        // run-index bits: the lane group bit first, then the other tile bits above the run
        uint32_t ridx[kStTileBits];
        int nr = 0;
        if (nstar) ridx[nr++] = lane_addr[4];
        for (int i = 0; i < n; i++)
            if (all[i] >= m && !star[all[i]]) ridx[nr++] = all[i];
        if (m < 7 || (1 << nr) > kStMaxRuns || (uint32_t)nr + m != (uint32_t)kStTileBits) return false;
        const uint32_t RL = 1u << m;
        const uint32_t gstride = nstar ? 2 * RL + 32u : RL, jstride = RL + 16u;
        for (uint32_t b = 0; b < m; b++) weight[b] = 1u << b;
        for (int q = 0; q < nr; q++)
            weight[ridx[q]] = q < nstar ? jstride : (1u << (q - nstar)) * gstride;
        P.run_bits = m;
        P.nruns = 1u << nr;
        uint32_t top = 0;
        for (uint32_t run = 0; run < P.nruns; run++) {
            uint64_t off = 0;
            uint32_t w = 0;
            for (int q = 0; q < nr; q++)
                if ((run >> q) & 1) { off += 1ull << ridx[q]; w += weight[ridx[q]]; }
            P.run_off[run] = off;
            P.run_word[run] = w;
            if (w + RL > top) top = w + RL;
        }
        if (top > (uint32_t)kStCompWords) return false;
    }
    for (int b = 0; b < 5; b++) { P.lane_addr[b] = lane_addr[b]; P.lane_w[b] = weight[lane_addr[b]]; }
    for (int b = 0; b < 5; b++) P.dlane_addr[b] = lane_addr[b];
    for (int b = 0; b < kStRegs; b++) P.dreg_addr[b] = reg_addr[b];
    for (int b = 0; b < kStWarpBits; b++) P.dwarp_addr[b] = warp_addr[b];
    for (int b = 0; b < kStRegs; b++) { P.reg_addr[b] = reg_addr[b]; P.reg_w[b] = weight[reg_addr[b]]; }
    for (int b = 0; b < kStWarpBits; b++) { P.warp_addr[b] = warp_addr[b]; P.warp_w[b] = weight[warp_addr[b]]; }
    P.ntiles = 1ull << (L - kStTileBits);
    P.ngates = g.ngates;
    for (uint32_t i = 0; i < g.ngates; i++) {
        const FusedGate &fg = g.gates[i];
        StagedGate &sg = P.gates[i];
        const int t = code[fg.t], c = fg.c >= 0 ? code[fg.c] : -1;
        const int creg = c >= 0 && c < kStRegs ? c : -1;
        sg.lc = (int8_t)(c >= kStRegs ? c - 5 : -1);
        if (t < kStRegs) {
            sg.case_ = (int16_t)(t * 8 + creg + 1);
            sg.lt = -1;
        } else {
            sg.case_ = (int16_t)(64 + creg + 1);
            sg.lt = (int8_t)(t - 5);
        }
        memcpy(sg.m, fg.m, sizeof sg.m);
    }
    return true;
}

// The two tensor maps of a box plan (re and im over 2^L f32 amplitudes). Unused dimensions have
// extent 1.
static bool encode_boxes(const StagedPlan &P, uint32_t L, float *re, float *im, CUtensorMap &tre, CUtensorMap &tim) {
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
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    return one(tre, re) && one(tim, im);
}

static int launch_staged(const StagedPlan &P, const CUtensorMap &tre, const CUtensorMap &tim, float *re, float *im,
                         cudaStream_t s) {
    static bool attr_done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LYTH_E_INVALID;
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(staged_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStSmem);
        if (e != cudaSuccess) return status_of(e);
        attr_done[dev] = true;
    }
    const uint64_t sms = (uint64_t)device_sms();
    const unsigned grid = (unsigned)(P.ntiles < sms ? P.ntiles : sms);
    staged_fused_kernel<<<grid, kStThreads, kStSmem, s>>>(P, tre, tim, re, im);
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

// LYTH_FUSED_STAGING=0 sends every group to the register pass (an A/B switch: both are bit-exact).
static bool staging_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("LYTH_FUSED_STAGING");
        on = !(v && v[0] == '0');
    }
    return on == 1;
}

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s) {
    if (staging_enabled() && len && !(len & (len - 1)) && !(((uintptr_t)re | (uintptr_t)im) & 15)) {
        uint32_t L = 0;
        while ((1ull << L) < len) L++;
        StagedPlan P;
        CUtensorMap tre, tim;
        memset(&tre, 0, sizeof tre);
        memset(&tim, 0, sizeof tim);
        bool ok = plan_staged(g, L, 1, P);
        if (ok && P.tma && !encode_boxes(P, L, re, im, tre, tim)) ok = plan_staged(g, L, 0, P);  // runs instead
        if (ok) return launch_staged(P, tre, tim, re, im, s);
    }
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
// of i (j < k <= 6; dst a permutation of src; other bits unchanged). The staged pass with no gates
// and each tile bit stored at its image: the permuted bits are tile bits, so every tile maps onto
// itself and the pass runs in place. LYTH_E_UNSUPPORTED when the state is too small for tiles.
bool permute_supported(uint64_t len, const uint32_t *src, int k) {
    if (k < 1 || k > kFuseMaxQubits || !len || (len & (len - 1))) return false;
    uint32_t L = 0;
    while ((1ull << L) < len) L++;
    FusedGroup g{};
    g.k = k;
    for (int j = 0; j < k; j++) g.bits[j] = src[j];
    StagedPlan P;
    return plan_staged(g, L, 0, P);
}

int launch_permute(uint64_t len, const uint32_t *src, const uint32_t *dst, int k, float *re, float *im,
                   cudaStream_t s) {
    if (k < 1 || k > kFuseMaxQubits || !len || (len & (len - 1)) || (((uintptr_t)re | (uintptr_t)im) & 15))
        return LYTH_E_UNSUPPORTED;
    uint32_t L = 0;
    while ((1ull << L) < len) L++;
    FusedGroup g{};
    g.k = k;
    for (int j = 0; j < k; j++) g.bits[j] = src[j];
    g.ngates = 0;
    StagedPlan P;
    CUtensorMap tre, tim;
    memset(&tre, 0, sizeof tre);
    memset(&tim, 0, sizeof tim);
    bool ok = plan_staged(g, L, 1, P);
    if (ok && P.tma && !encode_boxes(P, L, re, im, tre, tim)) ok = plan_staged(g, L, 0, P);
    if (!ok) return LYTH_E_UNSUPPORTED;
    auto image = [&](uint32_t a) {
        for (int j = 0; j < k; j++)
            if (src[j] == a) return dst[j];
        return a;
    };
    for (int b = 0; b < 5; b++) P.dlane_addr[b] = image(P.lane_addr[b]);
    for (int b = 0; b < kStRegs; b++) P.dreg_addr[b] = image(P.reg_addr[b]);
    for (int b = 0; b < kStWarpBits; b++) P.dwarp_addr[b] = image(P.warp_addr[b]);
    return launch_staged(P, tre, tim, re, im, s);
}

}  // namespace lyth

// ------------------------------------------------------------------ host-only layout self-test
// The staged pass is correct only if its planner's maps agree: for random groups it checks that
// every tile element has exactly one shared-memory word, that the copies (runs or tensor-map
// boxes, with the box coordinates rebuilt from the tile base) and the warps' reads agree on it,
// that the tensor-map dimensions partition the index space with 16-byte-aligned box origins,
// that no warp read hits a bank twice, and that every gate's target / control land on the
// group's bits. No device is touched.
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

int check_layout(const FusedGroup &g, uint32_t L, const StagedPlan &P, SplitMix &rng) {
    std::vector<int64_t> word2off(kStCompWords, -1);
    if (P.tma) {
        if (P.box_words * P.nbox != (uint32_t)kStTile) return -10;
        std::vector<int> cover(L, 0);
        for (int d = 0; d < 5; d++) {
            if (!P.dim_len[d]) continue;
            if (d > 0 && P.dim_lo[d] < 2) return -11;  // global strides must be multiples of 16 B
            for (uint32_t x = 0; x < P.dim_len[d]; x++) {
                if (P.dim_lo[d] + x >= L) return -12;
                cover[P.dim_lo[d] + x]++;
            }
        }
        for (uint32_t x = 0; x < L; x++)
            if (cover[x] != 1) return -13;
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
                if (word2off[w] != -1) return -14;
                word2off[w] = (int64_t)a;
            }
        uint64_t base = rng.next() % P.ntiles;
        for (int t = 0; t < kStTileBits; t++) base = insert_bit(base, P.tile_bits[t], 0);
        for (uint32_t b = 0; b < P.nbox; b++) {
            const uint64_t a = base + P.box_off[b];
            uint64_t back = 0;
            for (int d = 0; d < 5; d++) {
                if (!P.dim_len[d]) continue;
                const uint64_t c = (a >> P.dim_lo[d]) & ((1ull << P.dim_len[d]) - 1);
                if (c & ((1ull << P.dim_box[d]) - 1)) return -15;  // box origin off its alignment
                back += c << P.dim_lo[d];
            }
            if (back != a) return -16;
        }
    } else {
        for (uint32_t r = 0; r < P.nruns; r++)
            for (uint32_t o = 0; o < (1u << P.run_bits); o++) {
                const uint32_t w = P.run_word[r] + o;
                if (w >= (uint32_t)kStCompWords || word2off[w] != -1) return -17;
                word2off[w] = (int64_t)(P.run_off[r] + o);
            }
    }
    std::vector<uint8_t> hit(kStTile, 0);
    for (int wp = 0; wp < kStGroupWarps; wp++)
        for (int i = 0; i < (1 << kStRegs); i++) {
            uint32_t banks = 0;
            for (int lane = 0; lane < 32; lane++) {
                uint32_t w = 0;
                uint64_t a = 0;
                for (int b = 0; b < 5; b++)
                    if ((lane >> b) & 1) { w += P.lane_w[b]; a += 1ull << P.lane_addr[b]; }
                for (int b = 0; b < kStWarpBits; b++)
                    if ((wp >> b) & 1) { w += P.warp_w[b]; a += 1ull << P.warp_addr[b]; }
                for (int b = 0; b < kStRegs; b++)
                    if ((i >> b) & 1) { w += P.reg_w[b]; a += 1ull << P.reg_addr[b]; }
                if (w >= (uint32_t)kStCompWords || word2off[w] != (int64_t)a) return -18;
                uint32_t idx = 0;  // the element's position among the tile bits
                for (int t = 0; t < kStTileBits; t++)
                    if ((a >> P.tile_bits[t]) & 1) idx |= 1u << t;
                if (hit[idx]++) return -19;
                banks |= 1u << (w % 32);
            }
            if (banks != 0xffffffffu) return -20;
        }
    for (uint32_t gi = 0; gi < g.ngates; gi++) {
        const StagedGate &sg = P.gates[gi];
        int64_t tb, cb = -1;
        if (sg.case_ < 64) {
            tb = P.reg_addr[sg.case_ / 8];
            if (sg.case_ % 8 > 0) cb = P.reg_addr[sg.case_ % 8 - 1];
        } else {
            tb = P.lane_addr[sg.lt];
            if (sg.case_ > 64) cb = P.reg_addr[sg.case_ - 65];
        }
        if (sg.lc >= 0) {
            if (cb >= 0) return -21;
            cb = P.lane_addr[sg.lc];
        }
        if (tb != (int64_t)g.bits[g.gates[gi].t]) return -22;
        if (cb != (g.gates[gi].c >= 0 ? (int64_t)g.bits[g.gates[gi].c] : -1)) return -23;
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
        const uint32_t L = kStMinBits + rng.below(34 - kStMinBits);
        FusedGroup g{};
        g.k = 1 + (int32_t)rng.below(kFuseMaxQubits);
        // a third of the groups on the low bits, where lanes hold group bits
        const uint32_t span = (it % 3 == 0) ? 12 : L;
        uint32_t used = 0;
        for (int l = 0; l < g.k;) {
            const uint32_t b = rng.below(span);
            if (b >= 32 || (used >> b) & 1) continue;
            used |= 1u << b;
            g.bits[l++] = b;
        }
        g.ngates = 1 + rng.below(12);
        for (uint32_t i = 0; i < g.ngates; i++) {
            g.gates[i].t = (int8_t)rng.below((uint32_t)g.k);
            g.gates[i].c = (int8_t)(g.k > 1 && rng.below(2) ? (g.gates[i].t + 1 + rng.below((uint32_t)g.k - 1)) % g.k : -1);
        }
        StagedPlan P;
        if (!plan_staged(g, L, (int)(it % 3), P)) return LYTH_E_UNSUPPORTED;  // every such group must plan
        n_planned++;
        n_boxes += P.tma;
        const int st = check_layout(g, L, P, rng);
        if (st) return st;
    }
    if (planned) *planned = n_planned;
    if (boxes) *boxes = n_boxes;
    return LYTH_OK;
}
