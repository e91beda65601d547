// Shared helpers for the sm_100a kernels of liblyth_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "lyth_b200.h"

#define LYTH_HD __host__ __device__ __forceinline__
#define LYTH_D __device__ __forceinline__

namespace lyth {

// B200: 148 SMs, 2048 resident threads each. A grid-stride launch of 256-thread blocks fills
// the machine with this many blocks; kernels never need more for a streaming pass.
constexpr int kSMs = 148;
constexpr int kStreamBlock = 256;
constexpr int kStreamBlocksPerSM = 8;

inline int device_sms() {
    int dev = 0, sms = kSMs;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : kSMs;
}

// Blocks for a grid-stride streaming kernel that processes `units` per block-iteration.
inline unsigned stream_grid(uint64_t units_total, uint64_t units_per_block) {
    uint64_t need = (units_total + units_per_block - 1) / units_per_block;
    uint64_t cap = (uint64_t)device_sms() * kStreamBlocksPerSM;
    if (need > cap) need = cap;
    if (need == 0) need = 1;
    return (unsigned)need;
}

// LYTH_E_TIMEOUT (and the flag cleared) if a bounded device wait of that file's kernels ran
// out since the last call, else LYTH_OK (k_gemv.cu, k_probe.cu, k_stream.cu; the fused pass's in
// fused.cuh).
int gemv_take_device_error();
int probe_take_device_error();
int transpose_take_device_error();

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// cudaError_t passes through as a positive status; LYTH's own refusals are negative.
inline int status_of(cudaError_t e) { return e == cudaSuccess ? LYTH_OK : (int)e; }
inline int last_launch_status() { return status_of(cudaGetLastError()); }

// Streaming loads that do not allocate in L1: every element is touched once per pass. Not
// .nc, so they stay correct when a caller aliases an output onto this input.
LYTH_D float4 ld_stream4(const float *p) {
    float4 v;
    asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
// A load that may alias a later store of the same kernel (in-place passes): no .nc.
LYTH_D float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
LYTH_D void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
LYTH_D void st_stream4(float *p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// Insert a bit of value `v` at position `b` of k: bits of k at and above b move up by one.
LYTH_HD uint64_t insert_bit(uint64_t k, unsigned b, uint64_t v) {
    uint64_t low = k & ((1ull << b) - 1);
    return ((k >> b) << (b + 1)) | (v << b) | low;
}

// ir.rs:78-81: element k of a split view is (k / w) * 2w + part * w + (k % w) of its base.
LYTH_HD uint64_t view_index(uint64_t w, uint64_t part, uint64_t k) {
    return (k / w) * 2 * w + part * w + (k % w);
}

}  // namespace lyth
