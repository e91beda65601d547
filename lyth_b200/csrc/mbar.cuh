// mbarrier, bulk-copy and tensor-copy helpers shared by the TMA-fed kernels (inline PTX, sm_100a).
//
// Every wait is bounded twice -- by a poll count and by wall time on the global timer, since
// one try_wait may itself suspend for an implementation-defined interval -- and a wait that
// runs out sets the caller's device error flag and returns false, so a kernel winds down
// instead of hanging. No copy here uses cluster multicast.
#pragma once

#include "common.cuh"

namespace lyth {

constexpr uint32_t kWaitPolls = 1u << 24;        // try_wait polls before giving up
constexpr uint64_t kWaitNs = 2000000000ull;      // or 2 s of wall time, whichever first

LYTH_D uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

LYTH_D void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
LYTH_D uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase of parity `parity` to complete, giving up after `polls` polls or `ns` of
// global-timer time; on the limit set *err and return false.
LYTH_D bool mbar_wait_limited(uint32_t bar, uint32_t parity, int *err, uint32_t polls, uint64_t ns) {
    uint64_t t0 = 0;
    for (uint32_t i = 0; i < polls; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 255u) == 0) {
            const uint64_t t = global_ns();
            if (i == 0) t0 = t;
            else if (t - t0 > ns) break;
        }
    }
    atomicExch(err, 1);
    return false;
}
// The kernels' wait: 2^24 polls or 2 s.
LYTH_D bool mbar_wait(uint32_t bar, uint32_t parity, int *err) {
    return mbar_wait_limited(bar, parity, err, kWaitPolls, kWaitNs);
}

// Wait until a 64-bit flag in global memory (this GPU's or a peer's, system scope) reaches
// `target`, polling with acquire loads; on `ns` of global-timer time set *err and return false.
LYTH_D bool flag_wait_bounded(const uint64_t *flag, uint64_t target, uint64_t ns, int *err) {
    const uint64_t t0 = global_ns();
    for (;;) {
        uint64_t v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
        if (v >= target) return true;
        if (global_ns() - t0 > ns) {
            atomicExch(err, 1);
            return false;
        }
        __nanosleep(200);
    }
}

// Cluster-scope forms, for CTA pairs that share barriers (the 2-SM tensor-core contraction).
// The address of this CTA's shared-memory word `addr` in the shared memory of cluster CTA `rank`.
LYTH_D uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
LYTH_D uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of every CTA of the cluster (warp-aligned).
LYTH_D void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive (and expect `bytes`) on a barrier given by its shared::cluster address (this CTA's or
// the partner's). The data a barrier guards is ordered by the copy's complete_tx or, for tensor
// memory, by the tcgen05 fences around the arrive and the wait, so the default semantics suffice
// (a cluster-scope acquire in every poll of a wait would cost each poll a cluster-wide fence).
LYTH_D void mbar_expect_tx_cluster(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
LYTH_D void mbar_arrive_cluster(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
LYTH_D void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
LYTH_D void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completion counted in bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
LYTH_D void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"((uint64_t)src), "r"(bytes), "r"(bar)
        : "memory");
}

// Tiled tensor-map copy of a rank-5 box into this CTA's shared memory (no multicast).
LYTH_D void tensor_load_5d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2, int c3, int c4,
                           uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5, %6}], [%7];" ::"r"(dst),
        "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
        : "memory");
}

// Tiled tensor-map store of a rank-5 box from this CTA's shared memory (bulk group of the issuing
// thread; commit and wait below).
LYTH_D void tensor_store_5d(const CUtensorMap *map, int c0, int c1, int c2, int c3, int c4, uint32_t src) {
    asm volatile(
        "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}], [%6];" ::"l"(
            (uint64_t)map),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(src)
        : "memory");
}
LYTH_D void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's committed bulk stores have finished reading shared memory.
LYTH_D void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's committed bulk stores have completed.
LYTH_D void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- host: tensor maps through the driver entry point (no link-time libcuda).
typedef CUresult (*PFN_encode_tiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                     const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                     CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                     CUtensorMapFloatOOBfill);

inline PFN_encode_tiled tensor_map_encoder() {
    static PFN_encode_tiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encode_tiled>(p);
    }
    return fn;
}

}  // namespace lyth
