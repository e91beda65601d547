// Fused state-vector passes (lyth-circuit Group, crates/lyth-circuit/src/lib.rs:72-208 and
// docs/ADR-0030): one pass over the state applies a run of consecutive gates that together
// touch at most K <= 5 qubits.
//
// A thread owns the 2^K amplitudes that differ only in the group's K bits: it loads them
// (2^K coalesced loads per component: consecutive threads take consecutive values of the
// other bits), applies the group's gates in circuit order with the same fma chains as the
// unfused passes, and stores them back in place. The values between two gates are exactly the
// values the unfused passes would write and read back, so fused equals unfused bit for bit
// (the reference's claim, ADR-0030 Q1).
//
// Registers, not memory: the target (and control) of each gate is a run-time level of the
// group, but every case is a separate, fully unrolled code path selected by a uniform branch,
// so the 2^K amplitudes are only ever indexed by compile-time constants.
#include "fused.cuh"

namespace lyth {

template <int K, int T>
LYTH_D void apply_u(const U8 &m, float (&xr)[1 << K], float (&xi)[1 << K]) {
#pragma unroll
    for (int j = 0; j < (1 << K); j++) {
        if (j & (1 << T)) continue;
        const int j1 = j | (1 << T);
        float a, b, c, d;
        row0(m, xr[j], xi[j], xr[j1], xi[j1], a, b);
        row1(m, xr[j], xi[j], xr[j1], xi[j1], c, d);
        xr[j] = a; xi[j] = b; xr[j1] = c; xi[j1] = d;
    }
}

template <int K, int C, int T>
LYTH_D void apply_cu(const U8 &m, float (&xr)[1 << K], float (&xi)[1 << K]) {
#pragma unroll
    for (int j = 0; j < (1 << K); j++) {
        if ((j & (1 << T)) || !(j & (1 << C))) continue;
        const int j1 = j | (1 << T);
        float a, b, c, d;
        row0(m, xr[j], xi[j], xr[j1], xi[j1], a, b);
        row1(m, xr[j], xi[j], xr[j1], xi[j1], c, d);
        xr[j] = a; xi[j] = b; xr[j1] = c; xi[j1] = d;
    }
}

template <int K, int T = 0>
LYTH_D void dispatch_u(int t, const U8 &m, float (&xr)[1 << K], float (&xi)[1 << K]) {
    if constexpr (T < K) {
        if (t == T) apply_u<K, T>(m, xr, xi);
        else dispatch_u<K, T + 1>(t, m, xr, xi);
    }
}

template <int K, int C, int T = 0>
LYTH_D void dispatch_cu_t(int t, const U8 &m, float (&xr)[1 << K], float (&xi)[1 << K]) {
    if constexpr (T < K) {
        if constexpr (T != C) {
            if (t == T) {
                apply_cu<K, C, T>(m, xr, xi);
                return;
            }
        }
        dispatch_cu_t<K, C, T + 1>(t, m, xr, xi);
    }
}

template <int K, int C = 0>
LYTH_D void dispatch_cu(int c, int t, const U8 &m, float (&xr)[1 << K], float (&xi)[1 << K]) {
    if constexpr (C < K) {
        if (c == C) dispatch_cu_t<K, C>(t, m, xr, xi);
        else dispatch_cu<K, C + 1>(c, t, m, xr, xi);
    }
}

// Blocks per SM the register budget should allow: the 2^K amplitudes of a tuple live in
// registers (2^(K+1) floats), and a second resident block doubles the loads in flight.
template <int K>
constexpr int fused_min_blocks() {
    return K >= 5 ? 1 : (K == 4 ? 2 : 4);
}

template <int K>
__global__ void __launch_bounds__(256, fused_min_blocks<K>())
    fused_pass_kernel(uint64_t len, const __grid_constant__ FusedGroup G, float *re, float *im) {
    constexpr int S = 1 << K;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t rest = len >> K;
    for (uint64_t r = tid; r < rest; r += nthreads) {
        uint64_t base = r;
#pragma unroll
        for (int l = 0; l < K; l++) base = insert_bit(base, G.sorted[l], 0);
        // The per-level strides are re-read from the parameter space each iteration (an
        // empty asm keeps the compiler from hoisting 2^K 64-bit offsets into registers).
        uint64_t stride[K];
#pragma unroll
        for (int l = 0; l < K; l++) {
            stride[l] = 1ull << G.bits[l];
            asm volatile("" : "+l"(stride[l]));
        }
        float xr[S], xi[S];
#pragma unroll
        for (int j = 0; j < S; j++) {
            uint64_t off = 0;
#pragma unroll
            for (int l = 0; l < K; l++)
                if (j & (1 << l)) off += stride[l];
            xr[j] = re[base + off];
            xi[j] = im[base + off];
        }
        for (uint32_t g = 0; g < G.ngates; g++) {
            const FusedGate &fg = G.gates[g];
            const U8 m{fg.m[0], fg.m[1], fg.m[2], fg.m[3], fg.m[4], fg.m[5], fg.m[6], fg.m[7]};
            if (fg.c < 0) dispatch_u<K>(fg.t, m, xr, xi);
            else dispatch_cu<K>(fg.c, fg.t, m, xr, xi);
        }
#pragma unroll
        for (int j = 0; j < S; j++) {
            uint64_t off = 0;
#pragma unroll
            for (int l = 0; l < K; l++)
                if (j & (1 << l)) off += stride[l];
            re[base + off] = xr[j];
            im[base + off] = xi[j];
        }
    }
}

// ---- the same pass with each tuple split over a lane pair (lane l and l ^ 16 of a warp).
// Level K-1 of the group is the "split" level: lane half h = lane >> 4 holds the 2^(K-1)
// amplitudes whose split bit is h. Gates on the other levels run inside each lane as above; a
// gate targeting the split level swaps the partner's values in with one shuffle per amplitude
// and each lane computes its own row (row 0 with p0 = own, p1 = partner; row 1 with p0 =
// partner, p1 = own) -- the same chains on the same values, so the results are unchanged; a
// CU controlled by the split level runs only on the h = 1 lanes. Half the registers per thread
// triples the resident warps, and K = 6 fits.
template <int K>
LYTH_D void split_u(const U8 &m, int h, float (&xr)[1 << K], float (&xi)[1 << K], int cmask) {
#pragma unroll
    for (int j = 0; j < (1 << K); j++) {
        const float orr = __shfl_xor_sync(0xffffffffu, xr[j], 16);
        const float oi = __shfl_xor_sync(0xffffffffu, xi[j], 16);
        if (cmask >= 0 && !(j & cmask)) continue;
        float a, b;
        if (h == 0) row0(m, xr[j], xi[j], orr, oi, a, b);
        else row1(m, orr, oi, xr[j], xi[j], a, b);
        xr[j] = a;
        xi[j] = b;
    }
}

// Split-level gate with a local control at level C of the lane's half.
template <int K, int C = 0>
LYTH_D void dispatch_split_cu(int c, const U8 &m, int h, float (&xr)[1 << K], float (&xi)[1 << K]) {
    if constexpr (C < K) {
        if (c == C) split_u<K>(m, h, xr, xi, 1 << C);
        else dispatch_split_cu<K, C + 1>(c, m, h, xr, xi);
    }
}

template <int K>
constexpr int pair_min_blocks() {
    return K >= 6 ? 2 : 3;
}

template <int K>
__global__ void __launch_bounds__(256, pair_min_blocks<K>()) fused_pair_kernel(uint64_t len, const __grid_constant__ FusedGroup G,
                                                            float *re, float *im) {
    constexpr int KL = K - 1;  // levels inside a lane
    constexpr int S = 1 << KL;
    const int lane = threadIdx.x & 31, h = lane >> 4;
    const uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint64_t rest = len >> K;
    // A warp covers 16 tuples per step; every lane of the warp runs every step (shuffles).
    for (uint64_t r0 = warp * 16; r0 < rest; r0 += nwarps * 16) {
        const uint64_t r = r0 + (lane & 15);
        const bool live = r < rest;
        uint64_t base = live ? r : 0;
#pragma unroll
        for (int l = 0; l < K; l++) base = insert_bit(base, G.sorted[l], 0);
        uint64_t stride[K];
#pragma unroll
        for (int l = 0; l < K; l++) {
            stride[l] = 1ull << G.bits[l];
            asm volatile("" : "+l"(stride[l]));
        }
        if (h) base += stride[KL];
        float xr[S], xi[S];
#pragma unroll
        for (int j = 0; j < S; j++) {
            uint64_t off = 0;
#pragma unroll
            for (int l = 0; l < KL; l++)
                if (j & (1 << l)) off += stride[l];
            xr[j] = live ? re[base + off] : 0.0f;
            xi[j] = live ? im[base + off] : 0.0f;
        }
        for (uint32_t g = 0; g < G.ngates; g++) {
            const FusedGate &fg = G.gates[g];
            const U8 m{fg.m[0], fg.m[1], fg.m[2], fg.m[3], fg.m[4], fg.m[5], fg.m[6], fg.m[7]};
            if (fg.t == KL) {
                if (fg.c < 0) split_u<KL>(m, h, xr, xi, -1);
                else dispatch_split_cu<KL>(fg.c, m, h, xr, xi);
            } else if (fg.c == KL) {
                if (h) dispatch_u<KL>(fg.t, m, xr, xi);
            } else if (fg.c < 0) {
                dispatch_u<KL>(fg.t, m, xr, xi);
            } else {
                dispatch_cu<KL>(fg.c, fg.t, m, xr, xi);
            }
        }
        if (live) {
#pragma unroll
            for (int j = 0; j < S; j++) {
                uint64_t off = 0;
#pragma unroll
                for (int l = 0; l < KL; l++)
                    if (j & (1 << l)) off += stride[l];
                re[base + off] = xr[j];
                im[base + off] = xi[j];
            }
        }
    }
}

// Put the level with the fewest gates targeting it last (the split level of the pair kernel).
static FusedGroup with_split_level_last(const FusedGroup &g) {
    int cost[kFuseMaxQubits] = {0};
    for (uint32_t i = 0; i < g.ngates; i++) cost[g.gates[i].t]++;
    int best = g.k - 1;
    for (int l = 0; l < g.k; l++)
        if (cost[l] < cost[best]) best = l;
    FusedGroup o = g;
    const int last = g.k - 1;
    if (best == last) return o;
    auto swap_level = [&](int8_t &x) {
        if (x == best) x = (int8_t)last;
        else if (x == last) x = (int8_t)best;
    };
    o.bits[best] = g.bits[last];
    o.bits[last] = g.bits[best];
    for (uint32_t i = 0; i < o.ngates; i++) {
        swap_level(o.gates[i].t);
        swap_level(o.gates[i].c);
    }
    return o;
}

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s) {
    const unsigned grid = stream_grid(len >> g.k, kStreamBlock);
    switch (g.k) {
        case 1: fused_pass_kernel<1><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 2: fused_pass_kernel<2><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 3: fused_pass_kernel<3><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 4: fused_pass_kernel<4><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 5: {
            const FusedGroup o = with_split_level_last(g);
            const unsigned grid2 = stream_grid((len >> 5) * 2, kStreamBlock);
            fused_pair_kernel<5><<<grid2, kStreamBlock, 0, s>>>(len, o, re, im);
            break;
        }
        case 6: {
            const FusedGroup o = with_split_level_last(g);
            const unsigned grid2 = stream_grid((len >> 6) * 2, kStreamBlock);
            fused_pair_kernel<6><<<grid2, kStreamBlock, 0, s>>>(len, o, re, im);
            break;
        }
        default: return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}

}  // namespace lyth
