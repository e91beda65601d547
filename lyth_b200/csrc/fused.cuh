// A fused group of state-vector gates (see k_fused.cu).
#pragma once

#include "gates.cuh"

namespace lyth {

constexpr int kFuseMaxQubits = 13;       // a group's bits (the tile pass: at most 8 of them above bit 4)
constexpr int kFuseRegisterQubits = 6;   // the register pass (states below 2^14 amplitudes)
constexpr int kFuseMaxGates = 48;
constexpr int kPermuteMaxBits = 6;       // bits one permutation pass moves

// A gate inside a group: target level t, control level c (-1 for a plain U), levels index the
// group's bits; the matrix as lyth-circuit's f32s gives it.
struct FusedGate {
    int8_t t, c;
    int16_t pad;
    float m[8];
};

struct FusedGroup {
    int32_t k;              // number of bits (levels)
    uint32_t bits[kFuseMaxQubits];    // level l <-> amplitude bit bits[l]
    uint32_t sorted[kFuseMaxQubits];  // the same bits ascending (for the zero insertion)
    uint32_t ngates;
    FusedGate gates[kFuseMaxGates];
};

int launch_fused(uint64_t len, const FusedGroup &g, float *re, float *im, cudaStream_t s);
// Whether a group on these bits runs as one pass at this state size (the tile pass: at most 8
// bits above bit 4; the register pass below 2^14 amplitudes: at most 6 bits).
bool fused_fits(uint64_t len, const uint32_t *bits, int k);
// Move the amplitude at i to the index whose bit dst[j] is bit src[j] of i (k <= 6 bits, dst a
// permutation of src), in one in-place pass. LYTH_E_UNSUPPORTED below the tile pass's size.
int launch_permute(uint64_t len, const uint32_t *src, const uint32_t *dst, int k, float *re, float *im,
                   cudaStream_t s);
// Whether launch_permute takes these bits at this size (host only, no launch).
bool permute_supported(uint64_t len, const uint32_t *src, int k);
// LYTH_E_TIMEOUT (and clears the flag) if a tile pass gave up a bounded wait; else LYTH_OK.
int fused_take_device_error();

}  // namespace lyth
