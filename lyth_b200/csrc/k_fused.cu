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

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s) {
    const unsigned grid = stream_grid(len >> g.k, kStreamBlock);
    switch (g.k) {
        case 1: fused_pass_kernel<1><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 2: fused_pass_kernel<2><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 3: fused_pass_kernel<3><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 4: fused_pass_kernel<4><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        case 5: fused_pass_kernel<5><<<grid, kStreamBlock, 0, s>>>(len, g, re, im); break;
        default: return LYTH_E_UNSUPPORTED;
    }
    return last_launch_status();
}

}  // namespace lyth
