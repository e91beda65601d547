// bf16 contraction on the sm_100a tensor cores: C (f32) = A (bf16, m x k, row-major) *
// B (bf16, k x n, row-major), f32 accumulation in tensor memory.
//
// The reference never uses tensor cores (its contraction is scalar mul.rn + add.rn,
// crates/lyth-ptx/src/contracted.rs); this is the class the north star assigns to tcgen05.
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0       TMA producer: per K step, one 128 x 64 box of A (K-major, 128-byte swizzle)
//                and four 64 x 64 boxes of B (N-major, 128-byte swizzle) into a 4-stage ring,
//                completion tracked by an mbarrier with an expected byte count. No multicast:
//                every CTA fetches its own tiles.
//   warp 1       MMA issuer: one thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128,
//                N=256, K=16) four times per stage, accumulating into one of two 256-column
//                f32 accumulators in TMEM, and tcgen05.commit frees the stage / hands a
//                finished accumulator to the epilogue.
//   warps 2..5   epilogue: tcgen05.ld 32x32b (each warp reads its 32-lane quadrant: one row of
//                the tile per thread), 128-bit stores of f32 C. Two accumulators let the
//                epilogue of tile i overlap the main loop of tile i+1.
// (m a multiple of 256 takes the 2-SM form below instead.)
// Every wait on an mbarrier is bounded; one that runs out sets a device flag (read by
// lyth_b200_device_error) and the kernel winds down instead of hanging.
#include <cuda.h>

#include "fused.cuh"
#include "mbar.cuh"

namespace lyth {

constexpr int MM_BM = 128, MM_BN = 256, MM_BK = 64, MM_STAGES = 4;
constexpr int MM_A_BYTES = MM_BM * MM_BK * 2;               // 16 KiB
constexpr int MM_B_BOX_BYTES = 64 * MM_BK * 2;              // one 64(N) x 64(K) box: 8 KiB
constexpr int MM_B_BYTES = MM_BN * MM_BK * 2;               // 32 KiB
constexpr int MM_STAGE_BYTES = MM_A_BYTES + MM_B_BYTES;     // 48 KiB
constexpr int MM_TMEM_COLS = 2 * MM_BN;                     // two f32 accumulators
constexpr int MM_THREADS = 192;
constexpr size_t MM_SMEM = 1024 + (size_t)MM_STAGES * MM_STAGE_BYTES + 256;

__device__ int g_device_error;

// Instruction descriptor, kind::f16: D f32 (bit 4), A bf16 (bits 7-9 = 1), B bf16 (bits
// 10-12 = 1), A K-major (bit 15 = 0), B MN-major (bit 16 = 1), N >> 3 at bits 17-22, M >> 4
// at bits 24-28.
constexpr uint32_t MM_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                              ((uint32_t)(MM_BN >> 3) << 17) | ((uint32_t)(MM_BM >> 4) << 24);

// Bounded mbarrier wait (mbar.cuh) reporting to this kernel's error flag.
LYTH_D bool mm_wait(uint32_t bar, uint32_t parity) { return mbar_wait(bar, parity, &g_device_error); }
LYTH_D void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor (sm_100): start >> 4 at bits 0-13, leading byte offset >> 4
// at 16-29, stride byte offset >> 4 at 32-45, version 1 at 46-47, base offset 0, layout
// SWIZZLE_128B (2) at 61-63.
LYTH_D uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

LYTH_D void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(MM_IDESC), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
LYTH_D void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
LYTH_D void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LYTH_D void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

LYTH_D void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(MM_THREADS, 1)
    mma_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, float *C,
                    uint32_t M, uint32_t N, uint32_t K) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + MM_STAGES * MM_A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sB + MM_STAGES * MM_B_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * MM_STAGES + 4);
    auto full = [&](int s) { return smem_u32(bars + s); };
    auto empty = [&](int s) { return smem_u32(bars + MM_STAGES + s); };
    auto tfull = [&](int b) { return smem_u32(bars + 2 * MM_STAGES + b); };
    auto tempty = [&](int b) { return smem_u32(bars + 2 * MM_STAGES + 2 + b); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tiles_m = M / MM_BM, tiles_n = N / MM_BN, ntiles = tiles_m * tiles_n, kblocks = K / MM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < MM_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull(b), 1);
            mbar_init(tempty(b), 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(MM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int m0 = (int)((tile % tiles_m) * MM_BM), n0 = (int)((tile / tiles_m) * MM_BN);
                for (uint32_t kb = 0; kb < kblocks; kb++) {
                    if (!mm_wait(empty(stage), phase ^ 1)) { ok = false; break; }
                    mbar_expect_tx(full(stage), MM_STAGE_BYTES);
                    const int k0 = (int)(kb * MM_BK);
                    tma_load_2d(smem_u32(sA + stage * MM_A_BYTES), &tmA, k0, m0, full(stage));
#pragma unroll
                    for (int j = 0; j < MM_BN / 64; j++)
                        tma_load_2d(smem_u32(sB + stage * MM_B_BYTES + j * MM_B_BOX_BYTES), &tmB, n0 + 64 * j, k0,
                                    full(stage));
                    if (++stage == MM_STAGES) { stage = 0; phase ^= 1; }
                }
            }
            // Normally every load has been consumed by the MMAs before the block-wide sync
            // below. After a timed-out wait, give the stages this thread may have in flight a
            // bounded chance to land before the block leaves.
            if (!ok) {
                for (int s = 0; s < MM_STAGES; s++) {
                    mm_wait(full(stage), phase);
                    if (++stage == MM_STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, local = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, local++) {
                const uint32_t ab = local & 1, aphase = (local >> 1) & 1;
                if (!mm_wait(tempty(ab), aphase ^ 1)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + ab * MM_BN;
                for (uint32_t kb = 0; kb < kblocks; kb++) {
                    if (!mm_wait(full(stage), phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + stage * MM_A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * MM_B_BYTES);
#pragma unroll
                    for (int k = 0; k < MM_BK / 16; k++) {
                        // A: K-major rows of 128 B, 8-row groups 1024 B apart; step K by 32 B.
                        const uint64_t da = smem_desc(a_base + k * 32, 16, 1024);
                        // B: N-major rows (one per k) of 128 B; 64-wide N blocks one box
                        // (8 KiB) apart, 8-row K groups 1024 B apart; step K by 16 rows.
                        const uint64_t db = smem_desc(b_base + k * 16 * 128, MM_B_BOX_BYTES, 1024);
                        umma_bf16(d_tmem, da, db, (kb | (uint32_t)k) != 0);
                    }
                    umma_commit(empty(stage));
                    if (++stage == MM_STAGES) { stage = 0; phase ^= 1; }
                }
                if (ok) umma_commit(tfull(ab));
            }
        }
    } else {
        const uint32_t quad = (uint32_t)(warp & 3);  // the TMEM lane quadrant this warp may read
        uint32_t local = 0;
        for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, local++) {
            const uint32_t ab = local & 1, aphase = (local >> 1) & 1;
            if (!mm_wait(tfull(ab), aphase)) break;
            tc_fence_after();
            const uint32_t m0 = (tile % tiles_m) * MM_BM, n0 = (tile / tiles_m) * MM_BN;
            const uint32_t row = m0 + quad * 32 + lane;
            float *crow = C + (uint64_t)row * N + n0;
#pragma unroll 1
            for (int c = 0; c < MM_BN / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tmem_base + ab * MM_BN + ((quad * 32) << 16) + c * 32, r);
#pragma unroll
                for (int v = 0; v < 8; v++) {
                    float4 f = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                           __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                    *reinterpret_cast<float4 *>(crow + c * 32 + 4 * v) = f;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(ab));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(MM_TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// The 2-SM form: a cluster of two CTAs (a CTA pair on neighbouring SMs) computes a 256 x 256 tile
// with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16). Each CTA stages only its half of the
// operands -- A rows 128c .. 128c+127 and B columns 128c .. 128c+127 of the tile, c = its rank in
// the pair -- and the pair's MMA reads both halves, so a CTA moves 32 KiB per 64-deep K step
// where the 1-SM kernel moves 48 KiB for the same 128 x 256 x 64 of arithmetic per SM: the L2 ->
// shared-memory traffic per flop drops by a third.
//
//   both CTAs, warp 0   TMA producer: waits on its own `empty` barrier, arrives with the byte
//                       count on the leader's `full` barrier and loads its halves (no multicast;
//                       the .cta_group::2 form lets the copy complete on the leader's barrier).
//   leader, warp 1      MMA issuer: waits for both halves (`full` counts two arrivals and 64 KiB),
//                       issues four MMAs and frees the stage in both CTAs with one commit
//                       (tcgen05.commit .multicast::cluster, mask 0b11); a finished accumulator is
//                       handed to both CTAs' epilogues the same way.
//   both CTAs, warps 2-5 epilogue: tcgen05.ld of this CTA's 128 accumulator rows (its own TMEM),
//                       f32 stores of C, then an arrival on the leader's `tempty` barrier (8 warps).
// TMEM: 512 columns (two 256-column accumulators) allocated by warp 1 of both CTAs
// (tcgen05.alloc.cta_group::2). Every barrier wait is bounded; a CTA pair meets at a cluster
// barrier at the start (barrier initialisation and TMEM allocation seen by both) and at the end
// (no CTA leaves while its partner may still read its shared memory or signal its barriers).
constexpr int M2_BM = 256, M2_BN = 256, M2_STAGES = 6;
constexpr int M2_A_BYTES = 128 * MM_BK * 2;                 // this CTA's 128 rows: 16 KiB
constexpr int M2_B_BYTES = 128 * MM_BK * 2;                 // this CTA's 128 columns: 16 KiB
constexpr int M2_STAGE_BYTES = M2_A_BYTES + M2_B_BYTES;     // 32 KiB
constexpr size_t M2_SMEM = 1024 + (size_t)M2_STAGES * M2_STAGE_BYTES + 256;
constexpr uint32_t M2_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(M2_BN >> 3) << 17) |
                              ((uint32_t)(M2_BM >> 4) << 24);

LYTH_D void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(dst),
        "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar_cluster)
        : "memory");
}
LYTH_D void umma2_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(M2_IDESC), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z),
        "r"(z));
}
// Arrive on the barrier at this shared-memory offset in both CTAs of the pair once every MMA this
// thread issued has completed.
LYTH_D void umma2_commit_both(uint32_t bar) {
    const uint16_t mask = 3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(mask)
        : "memory");
}

__global__ void __launch_bounds__(MM_THREADS, 1)
    mma2_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, float *C,
                     uint32_t M, uint32_t N, uint32_t K) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + M2_STAGES * M2_A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sB + M2_STAGES * M2_B_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * M2_STAGES + 4);
    auto full = [&](int s) { return smem_u32(bars + s); };
    auto empty = [&](int s) { return smem_u32(bars + M2_STAGES + s); };
    auto tfull = [&](int b) { return smem_u32(bars + 2 * M2_STAGES + b); };
    auto tempty = [&](int b) { return smem_u32(bars + 2 * M2_STAGES + 2 + b); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();
    uint32_t pair, npairs;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(pair));
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(npairs));
    const uint32_t tiles_m = M / M2_BM, tiles_n = N / M2_BN, ntiles = tiles_m * tiles_n, kblocks = K / MM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < M2_STAGES; s++) {
            mbar_init(full(s), 2);  // the two producers' arrivals (the leader's barrier is the one used)
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull(b), 1);
            mbar_init(tempty(b), 8);  // four epilogue warps in each CTA (the leader's is the one used)
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(MM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t tile = pair; tile < ntiles && ok; tile += npairs) {
                const int m0 = (int)((tile % tiles_m) * M2_BM + 128 * crank);
                const int n0 = (int)((tile / tiles_m) * M2_BN + 128 * crank);
                for (uint32_t kb = 0; kb < kblocks; kb++) {
                    if (!mm_wait(empty(stage), phase ^ 1)) { ok = false; break; }
                    const uint32_t lf = mapa_shared(full(stage), 0);
                    mbar_expect_tx_cluster(lf, M2_STAGE_BYTES);
                    const int k0 = (int)(kb * MM_BK);
                    tma_load_2d_pair(smem_u32(sA + stage * M2_A_BYTES), &tmA, k0, m0, lf);
                    tma_load_2d_pair(smem_u32(sB + stage * M2_B_BYTES), &tmB, n0, k0, lf);
                    tma_load_2d_pair(smem_u32(sB + stage * M2_B_BYTES + MM_B_BOX_BYTES), &tmB, n0 + 64, k0, lf);
                    if (++stage == M2_STAGES) { stage = 0; phase ^= 1; }
                }
            }
            // Tail: every stage released by the MMA's commit, so no arrival is still on its way to
            // this CTA's barriers when it leaves.
            if (ok)
                for (int s = 0; s < M2_STAGES; s++) {
                    if (!mm_wait(empty(stage), phase ^ 1)) break;
                    if (++stage == M2_STAGES) { stage = 0; phase ^= 1; }
                }
        }
    } else if (warp == 1) {
        if (lane == 0 && crank == 0) {
            uint32_t stage = 0, phase = 0, local = 0;
            bool ok = true;
            for (uint32_t tile = pair; tile < ntiles && ok; tile += npairs, local++) {
                const uint32_t ab = local & 1, aphase = (local >> 1) & 1;
                if (!mm_wait(tempty(ab), aphase ^ 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + ab * M2_BN;
                for (uint32_t kb = 0; kb < kblocks; kb++) {
                    if (!mm_wait(full(stage), phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + stage * M2_A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * M2_B_BYTES);
#pragma unroll
                    for (int k = 0; k < MM_BK / 16; k++) {
                        const uint64_t da = smem_desc(a_base + k * 32, 16, 1024);
                        const uint64_t db = smem_desc(b_base + k * 16 * 128, MM_B_BOX_BYTES, 1024);
                        umma2_bf16(d_tmem, da, db, (kb | (uint32_t)k) != 0);
                    }
                    umma2_commit_both(empty(stage));
                    if (++stage == M2_STAGES) { stage = 0; phase ^= 1; }
                }
                if (ok) umma2_commit_both(tfull(ab));
            }
            // After a timed-out wait, give the stages the producers may have in flight a bounded
            // chance to land (both CTAs' copies complete on these barriers) before the pair leaves.
            if (!ok) {
                for (int s = 0; s < M2_STAGES; s++) {
                    mm_wait(full(stage), phase);
                    if (++stage == M2_STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else {
        const uint32_t quad = (uint32_t)(warp & 3);  // the TMEM lane quadrant this warp may read
        const uint32_t lead_tempty[2] = {mapa_shared(tempty(0), 0), mapa_shared(tempty(1), 0)};
        uint32_t local = 0;
        for (uint32_t tile = pair; tile < ntiles; tile += npairs, local++) {
            const uint32_t ab = local & 1, aphase = (local >> 1) & 1;
            if (!mm_wait(tfull(ab), aphase)) break;
            tc_fence_after();
            const uint32_t m0 = (tile % tiles_m) * M2_BM + 128 * crank, n0 = (tile / tiles_m) * M2_BN;
            const uint32_t row = m0 + quad * 32 + lane;
            float *crow = C + (uint64_t)row * N + n0;
#pragma unroll 1
            for (int c = 0; c < M2_BN / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tmem_base + ab * M2_BN + ((quad * 32) << 16) + c * 32, r);
#pragma unroll
                for (int v = 0; v < 8; v++) {
                    float4 f = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                           __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                    *reinterpret_cast<float4 *>(crow + c * 32 + 4 * v) = f;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead_tempty[ab]);
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(MM_TMEM_COLS)
                     : "memory");
    }
}

// A 2-D bf16 tensor map: inner extent `inner` (contiguous), outer `outer`, box inner 64
// (128 bytes, the swizzle span) x box_outer, 128-byte swizzle.
static bool make_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
    PFN_encode_tiled enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace lyth

using namespace lyth;

// CTA pairs of the pair kernel resident at once on device `dev` (a GPC with an odd count of SMs
// holds one pair fewer than half its SMs), asked once per device. `cfg` is the launch's
// configuration (block, shared memory, cluster shape); its grid is overwritten.
static int mma2_pairs(int dev, int sms, cudaLaunchConfig_t &cfg) {
    static int fit_of[64] = {0};
    const int pairs = sms / 2;
    if (dev < 0 || dev >= 64) return pairs;
    if (fit_of[dev] == 0) {
        cfg.gridDim = dim3(2u * (unsigned)pairs);
        int fit = 0;
        if (cudaOccupancyMaxActiveClusters(&fit, mma2_bf16_kernel, &cfg) != cudaSuccess || fit < 1) fit = pairs;
        cudaGetLastError();
        fit_of[dev] = fit < pairs ? fit : pairs;
    }
    return fit_of[dev];
}

// pair: 1 = the 2-SM kernel (m a multiple of 256), 0 = the 1-SM kernel, -1 = the 2-SM kernel
// where the shape allows it.
static int matmul_bf16_launch(uint32_t m, uint32_t n, uint32_t k, const uint16_t *a, const uint16_t *b, float *c,
                              cudaStream_t s, int pair) {
    if (!a || !b || !c) return LYTH_E_INVALID;
    if (m == 0 || n == 0 || k == 0) return LYTH_E_INVALID;
    if (m % MM_BM || n % MM_BN || k % MM_BK) return LYTH_E_UNSUPPORTED;
    if ((((uintptr_t)a) | ((uintptr_t)b) | ((uintptr_t)c)) & 15u) return LYTH_E_UNSUPPORTED;
    if (pair < 0) pair = m % M2_BM == 0;
    if (pair && m % M2_BM) return LYTH_E_UNSUPPORTED;
    CUtensorMap ta, tb;
    if (!make_map(&ta, a, k, m, MM_BM)) return LYTH_E_UNSUPPORTED;  // A: inner K, outer M, box 64 x 128
    if (!make_map(&tb, b, n, k, MM_BK)) return LYTH_E_UNSUPPORTED;  // B: inner N, outer K, box 64 x 64
    static bool attr_done[2][64] = {{false}};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[pair][dev]) {
        cudaError_t e = pair ? cudaFuncSetAttribute(mma2_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)M2_SMEM)
                             : cudaFuncSetAttribute(mma_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)MM_SMEM);
        if (e != cudaSuccess) return status_of(e);
        attr_done[pair][dev] = true;
    }
    const int sms = device_sms();
    if (!pair) {
        const uint32_t tiles = (m / MM_BM) * (n / MM_BN);
        const unsigned grid = tiles < (uint32_t)sms ? tiles : (unsigned)sms;
        mma_bf16_kernel<<<grid, MM_THREADS, MM_SMEM, s>>>(ta, tb, c, m, n, k);
        return last_launch_status();
    }
    const uint32_t tiles = (m / M2_BM) * (n / M2_BN);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(MM_THREADS);
    cfg.dynamicSmemBytes = M2_SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int pairs = mma2_pairs(dev, sms, cfg);
    if ((uint32_t)pairs > tiles) pairs = (int)tiles;
    cfg.gridDim = dim3(2u * (unsigned)pairs);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, mma2_bf16_kernel, ta, tb, c, m, n, k);
    if (e != cudaSuccess) return status_of(e);
    return last_launch_status();
}

extern "C" int lyth_b200_matmul_bf16(uint32_t m, uint32_t n, uint32_t k, const uint16_t *a, const uint16_t *b,
                                     float *c, cudaStream_t s) {
    return matmul_bf16_launch(m, n, k, a, b, c, s, -1);
}

extern "C" int lyth_b200_matmul_bf16_pairs(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LYTH_E_INVALID;
    const cudaError_t e =
        cudaFuncSetAttribute(mma2_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)M2_SMEM);
    if (e != cudaSuccess) return status_of(e);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(MM_THREADS);
    cfg.dynamicSmemBytes = M2_SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return mma2_pairs(dev, device_sms(), cfg);
}

extern "C" int lyth_b200_matmul_bf16_form(int pair, uint32_t m, uint32_t n, uint32_t k, const uint16_t *a,
                                          const uint16_t *b, float *c, cudaStream_t s) {
    if (pair != 0 && pair != 1) return LYTH_E_INVALID;
    return matmul_bf16_launch(m, n, k, a, b, c, s, pair);
}

extern "C" int lyth_b200_device_error(void) {
    // every flag is read (and cleared) whichever reports first
    const int fused = fused_take_device_error();
    const int gemv = gemv_take_device_error();
    const int probe = probe_take_device_error();
    const int tx = transpose_take_device_error();
    if (fused != LYTH_OK) return fused;
    if (gemv != LYTH_OK) return gemv;
    if (probe != LYTH_OK) return probe;
    if (tx != LYTH_OK) return tx;
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
    if (e != cudaSuccess) return status_of(e);
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}
