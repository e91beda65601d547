// The state vector (lyth-circuit, crates/lyth-circuit/src/lib.rs:327-371), re-designed for B200.
//
// The reference ping-pongs two full state buffers and launches one pass per gate on one GPU.
// This engine:
//  * updates the state in place (one copy of 2^q amplitudes: 33 qubits is 64 GiB, which leaves
//    room on a 180 GB part), with the same fma chains as the out-of-place kernels, so every
//    amplitude is bit-identical to the reference's;
//  * fuses consecutive local gates on at most 13 qubits into one pass (k_fused.cu), applying
//    them in circuit order, bit-identical to the unfused passes (lyth-circuit fuse, lib.rs:72-100);
//  * keeps a logical -> physical qubit map, so a SWAP moves no data: it relabels two qubits.
//    The map is undone by real permutation passes only when the state is read out, which is
//    exact because a swap is a permutation;
//  * skips the control=0 half of a CU (it is a copy in the reference: identity in place);
//  * shards 2^q amplitudes over 2^g ranks on the g highest physical bits: rank r holds physical
//    indices [r * 2^L, (r+1) * 2^L), L = q - g. A gate on a local bit is a local (fusable) pass.
//    A CU whose control is a rank bit runs (as a local U) only on the ranks whose bit is 1. A
//    diagonal gate whose target is a rank bit is a scalar on each shard and moves no data. Any
//    other gate whose target is a rank bit first swaps that qubit into a local bit (the local bit
//    needed furthest ahead leaves): half the shard is packed, moved to the partner and unpacked into
//    the positions it vacated, chunk by chunk, the move through CUDA IPC mappings ordered by
//    sequence flags -- copy-engine pulls (cudaMemcpyAsync), SM peer loads fused with the unpack,
//    or SM stores into the partners' shards -- or over NCCL. With remap off the pair exchanges
//    whole shards instead and each computes its own row of the gate as chunks land. Peer memory
//    is touched only by those copies and plain loads and stores: no TMA, no multicast.
//
// NCCL is opened with dlopen on first use by a multi-rank handle, so the library itself loads
// (and serves every single-GPU entry point) without it.
#include <dlfcn.h>
#include <time.h>
#include <unistd.h>
#include <math.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "fused.cuh"
#include "mbar.cuh"

namespace lyth {

// ------------------------------------------------------------------ NCCL, loaded on demand
struct NcclApi {
    bool tried = false, ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
};
static NcclApi g_nccl;

static bool load_nccl() {
    if (g_nccl.tried) return g_nccl.ok;
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return false;
#define LYTH_SYM(field, name) g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name))
    LYTH_SYM(GetUniqueId, "ncclGetUniqueId");
    LYTH_SYM(CommInitRank, "ncclCommInitRank");
    LYTH_SYM(CommDestroy, "ncclCommDestroy");
    LYTH_SYM(CommAbort, "ncclCommAbort");
    LYTH_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    LYTH_SYM(GroupStart, "ncclGroupStart");
    LYTH_SYM(GroupEnd, "ncclGroupEnd");
    LYTH_SYM(Send, "ncclSend");
    LYTH_SYM(Recv, "ncclRecv");
    LYTH_SYM(AllReduce, "ncclAllReduce");
    LYTH_SYM(AllGather, "ncclAllGather");
#undef LYTH_SYM
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.GroupStart &&
                g_nccl.GroupEnd && g_nccl.Send && g_nccl.Recv && g_nccl.AllReduce;
    return g_nccl.ok;
}

// ------------------------------------------------------------------ kernels of the engine
__global__ void set_one_kernel(float *re, float *im, uint64_t i) {
    re[i] = 1.0f;
    im[i] = 0.0f;
}

// re = U(stream 2g), im = U(stream 2g + 1), g the global index; f64 partial of |a|^2 per block.
__global__ void __launch_bounds__(256) init_random_kernel(uint64_t len, uint64_t base, uint64_t seed, float *re,
                                                          float *im, double *partial) {
    __shared__ double sh[256];
    double acc = 0.0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t g = base + i;
        uint64_t z0 = seed + (2 * g + 1) * 0x9E3779B97F4A7C15ull;
        uint64_t z1 = seed + (2 * g + 2) * 0x9E3779B97F4A7C15ull;
        z0 = (z0 ^ (z0 >> 30)) * 0xBF58476D1CE4E5B9ull; z0 = (z0 ^ (z0 >> 27)) * 0x94D049BB133111EBull; z0 ^= z0 >> 31;
        z1 = (z1 ^ (z1 >> 30)) * 0xBF58476D1CE4E5B9ull; z1 = (z1 ^ (z1 >> 27)) * 0x94D049BB133111EBull; z1 ^= z1 >> 31;
        const float r = __fsub_rn(__fmul_rn(__fmul_rn((float)(z0 >> 40), 1.0f / 16777216.0f), 2.0f), 1.0f);
        const float m = __fsub_rn(__fmul_rn(__fmul_rn((float)(z1 >> 40), 1.0f / 16777216.0f), 2.0f), 1.0f);
        re[i] = r;
        im[i] = m;
        acc += (double)r * (double)r + (double)m * (double)m;
    }
    sh[threadIdx.x] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[blockIdx.x] = sh[0];
}

__global__ void sum_partials_kernel(const double *partial, int count, double *out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        double s = 0.0;
        for (int i = 0; i < count; i++) s += partial[i];
        *out = s;
    }
}

__global__ void __launch_bounds__(256) scale_kernel(uint64_t len, const double *norm2, float *re, float *im) {
    const float f = (float)(1.0 / sqrt(*norm2));
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (uint64_t)gridDim.x * blockDim.x) {
        re[i] = __fmul_rn(re[i], f);
        im[i] = __fmul_rn(im[i], f);
    }
}

// A swap of k local bits with k rank bits: the shard splits into 2^k subsets by the values of the
// local bits, one per partner rank (and the one this rank keeps); subset `pattern` is the local
// indices whose bits vs[0..k) (ascending) equal the pattern's bits. Partner y = blockIdx.y takes
// elements [k0, k0 + count) of its subset, in ascending order of the other bits, to / from slice y
// of the chunk buffers. With vs[0] >= 2 four consecutive elements are four consecutive indices.
struct MultiPat {
    uint32_t k;
    uint32_t vs[8];
    uint32_t pattern[64];  // per partner: bit s = value at vs[s]
};
LYTH_D uint64_t insert_pattern(uint64_t x, const MultiPat &mp, uint32_t pat) {
    for (uint32_t s = 0; s < mp.k; s++) x = insert_bit(x, mp.vs[s], (pat >> s) & 1u);
    return x;
}
__global__ void __launch_bounds__(1024) pack_multi_kernel(uint64_t count, uint64_t k0, const __grid_constant__ MultiPat mp,
                                                         const float *re, const float *im, float *ore, float *oim) {
    const uint32_t y = blockIdx.y, pat = mp.pattern[y];
    ore += (uint64_t)y * count;
    oim += (uint64_t)y * count;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    if (mp.vs[0] >= 2 && (count & 3) == 0 && (k0 & 3) == 0) {
        for (uint64_t g = tid; g < (count >> 2); g += nth) {
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat);
            st4(ore + 4 * g, ld_stream4(re + i));
            st4(oim + 4 * g, ld_stream4(im + i));
        }
        return;
    }
    for (uint64_t e = tid; e < count; e += nth) {
        const uint64_t i = insert_pattern(k0 + e, mp, pat);
        ore[e] = re[i];
        oim[e] = im[i];
    }
}
__global__ void __launch_bounds__(1024) unpack_multi_kernel(uint64_t count, uint64_t k0, const __grid_constant__ MultiPat mp,
                                                           float *re, float *im, const float *ire, const float *iim) {
    const uint32_t y = blockIdx.y, pat = mp.pattern[y];
    ire += (uint64_t)y * count;
    iim += (uint64_t)y * count;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    if (mp.vs[0] >= 2 && (count & 3) == 0 && (k0 & 3) == 0) {
        for (uint64_t g = tid; g < (count >> 2); g += nth) {
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat);
            st4(re + i, ld_stream4(ire + 4 * g));
            st4(im + i, ld_stream4(iim + 4 * g));
        }
        return;
    }
    for (uint64_t e = tid; e < count; e += nth) {
        const uint64_t i = insert_pattern(k0 + e, mp, pat);
        re[i] = ire[e];
        im[i] = iim[e];
    }
}

// A 128-bit load of a partner's memory through its CUDA IPC mapping (peer access over NVLink):
// cached at L2 level only, so no L1 line of an earlier chunk in the same slot is ever read.
LYTH_D float4 ld_peer4(const float *p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
LYTH_D float ld_peer(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
// Where partner y's packed slice for this rank starts in that partner's send slot (both
// components), for the peer-load transport.
struct PeerSrc {
    const float *re[64];
    const float *im[64];
};
// The peer-load transport's pull, fused with the unpack: block row y reads partner y's packed
// slice straight out of the partner's memory (plain loads issued by the SMs: no copy engine, no
// TMA, no multicast) and stores it into this rank's subset pattern[y], the positions whose own
// amplitudes that partner takes from this rank's send slot -- packed there before this runs. No
// receive buffer, and no separate unpack pass over HBM. Two groups of four per thread per trip
// keep four 16-byte peer loads in flight.
__global__ void __launch_bounds__(512) pull_unpack_kernel(uint64_t count, uint64_t k0, const __grid_constant__ MultiPat mp,
                                                          const __grid_constant__ PeerSrc src, float *re, float *im) {
    const uint32_t y = blockIdx.y, pat = mp.pattern[y];
    const float *pre = src.re[y], *pim = src.im[y];
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    if (mp.vs[0] >= 2 && (count & 3) == 0 && (k0 & 3) == 0) {
        const uint64_t groups = count >> 2;
        uint64_t g = tid;
        for (; g + nth < groups; g += 2 * nth) {
            const uint64_t h = g + nth;
            const float4 a = ld_peer4(pre + 4 * g), b = ld_peer4(pim + 4 * g);
            const float4 c = ld_peer4(pre + 4 * h), d = ld_peer4(pim + 4 * h);
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat), j = insert_pattern(k0 + 4 * h, mp, pat);
            st4(re + i, a);
            st4(im + i, b);
            st4(re + j, c);
            st4(im + j, d);
        }
        if (g < groups) {
            const float4 a = ld_peer4(pre + 4 * g), b = ld_peer4(pim + 4 * g);
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat);
            st4(re + i, a);
            st4(im + i, b);
        }
        return;
    }
    for (uint64_t e = tid; e < count; e += nth) {
        const uint64_t i = insert_pattern(k0 + e, mp, pat);
        re[i] = ld_peer(pre + e);
        im[i] = ld_peer(pim + e);
    }
}

// Partner y's shard (both components), for the push form.
struct PeerDst {
    float *re[64];
    float *im[64];
};
// The push form of a swap-in: block row y reads this rank's packed slice y (local, contiguous)
// and stores it into partner y's shard at the positions of subset `pat` there -- the subset whose
// own amplitudes that partner packed for this rank before this runs (plain SM stores over NVLink
// through the CUDA IPC mapping: no copy engine, no TMA, no multicast). Every partner takes this
// rank's data at the same pattern. Two groups of four per thread per trip.
__global__ void __launch_bounds__(512) push_kernel(uint64_t count, uint64_t k0, const __grid_constant__ MultiPat mp,
                                                   uint32_t pat, const float *sre, const float *sim,
                                                   const __grid_constant__ PeerDst dst) {
    const uint32_t y = blockIdx.y;
    sre += (uint64_t)y * count;
    sim += (uint64_t)y * count;
    float *dre = dst.re[y], *dim = dst.im[y];
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    if (mp.vs[0] >= 2 && (count & 3) == 0 && (k0 & 3) == 0) {
        const uint64_t groups = count >> 2;
        uint64_t g = tid;
        for (; g + nth < groups; g += 2 * nth) {
            const uint64_t h = g + nth;
            const float4 a = ld_stream4(sre + 4 * g), b = ld_stream4(sim + 4 * g);
            const float4 c = ld_stream4(sre + 4 * h), d = ld_stream4(sim + 4 * h);
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat), j = insert_pattern(k0 + 4 * h, mp, pat);
            st4(dre + i, a);
            st4(dim + i, b);
            st4(dre + j, c);
            st4(dim + j, d);
        }
        if (g < groups) {
            const float4 a = ld_stream4(sre + 4 * g), b = ld_stream4(sim + 4 * g);
            const uint64_t i = insert_pattern(k0 + 4 * g, mp, pat);
            st4(dre + i, a);
            st4(dim + i, b);
        }
        return;
    }
    for (uint64_t e = tid; e < count; e += nth) {
        const uint64_t i = insert_pattern(k0 + e, mp, pat);
        dre[i] = sre[e];
        dim[i] = sim[e];
    }
}

// Cross-GPU sequence flags of the copy-engine transport. Every rank polls only its own flag block
// and peers signal it by remote stores into it, so every remote write is awaited by the rank it
// targets before that rank frees anything.
__device__ int g_sv_error;

struct FlagPut {
    uint32_t n;
    uint64_t *flag[64];
};
// Thread t stores `value` into flag t (a peer's block), after this stream's earlier writes.
__global__ void flags_put_kernel(const __grid_constant__ FlagPut fp, uint64_t value) {
    const uint32_t t = threadIdx.x;
    if (t >= fp.n) return;
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(fp.flag[t]), "l"(value) : "memory");
}

struct FlagSet {
    uint32_t n;
    const uint64_t *flag[64];
};
// Wait until every flag is >= target (thread t polls flag t). Bounded by 2 s of global-timer time;
// on the limit set g_sv_error and return.
__global__ void flag_wait_kernel(const __grid_constant__ FlagSet fs, uint64_t target) {
    const uint32_t t = threadIdx.x;
    if (t >= fs.n) return;
    flag_wait_bounded(fs.flag[t], target, kWaitNs, &g_sv_error);
}

// ---- host waits with a deadline (the NCCL transport's failure path)
// query(): 0 = the awaited work is done, 1 = not yet, anything else a CUDA status to return.
// async_error(): nonzero once the communicator reports an error (ncclCommGetAsyncError). On an
// async error the communicator is aborted and LYTH_E_NCCL returned; past `deadline_ms` it is
// aborted and LYTH_E_TIMEOUT returned. ncclCommAbort makes the NCCL kernels a dead peer left
// waiting return, so the streams drain afterwards.
struct WaitHooks {
    void *ctx;
    int (*query)(void *);
    int (*async_error)(void *);
    void (*abort)(void *);
};

int wait_with_deadline(const WaitHooks &h, double deadline_ms, uint32_t poll_us, uint64_t *polls) {
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (uint64_t i = 0;; i++) {
        if (polls) *polls = i + 1;
        const int q = h.query(h.ctx);
        if (q == 0) return LYTH_OK;
        if (q != 1) return q;
        if (h.async_error && h.async_error(h.ctx)) {
            if (h.abort) h.abort(h.ctx);
            return LYTH_E_NCCL;
        }
        clock_gettime(CLOCK_MONOTONIC, &t1);
        const double ms = (t1.tv_sec - t0.tv_sec) * 1e3 + (t1.tv_nsec - t0.tv_nsec) * 1e-6;
        if (ms > deadline_ms) {
            if (h.abort) h.abort(h.ctx);
            return LYTH_E_TIMEOUT;
        }
        if (poll_us) usleep(poll_us);
    }
}

// One rank's CUDA IPC handles, all-gathered at set-up of the IPC transports.
struct IpcRec {
    int32_t ok, pad;
    cudaIpcMemHandle_t h[7];  // sre[0], sre[1], sim[0], sim[1], flags, re, im
};
}  // namespace lyth

using namespace lyth;

struct lyth_sv {
    uint32_t qubits = 0, local_bits = 0, global_bits = 0;
    int device = 0, rank = 0, nranks = 1;
    uint64_t local_len = 0, chunk = 0;
    float *re = nullptr, *im = nullptr;
    float *rre[2] = {nullptr, nullptr}, *rim[2] = {nullptr, nullptr};  // receive chunks
    float *sre[2] = {nullptr, nullptr}, *sim[2] = {nullptr, nullptr};  // packed send chunks
    double *scratch = nullptr;  // norm partials
    cudaStream_t stream = nullptr, comm_stream = nullptr;
    cudaStream_t copy_stream = nullptr;  // second copy-engine queue (the im halves of the pulls)
    cudaEvent_t ev_pull = nullptr, ev_copied = nullptr;
    // Further copy-engine queues: a pull is cut into `pull_queues` pieces per component, issued
    // round-robin over comm_stream, copy_stream and these (lyth_sv_set_pull_queues); 0 (the
    // default) gives every partner's two slices a queue of their own, up to 8 queues.
    static constexpr int kExtraQueues = 6;
    cudaStream_t xq[kExtraQueues] = {};
    cudaEvent_t ev_xq[kExtraQueues] = {};
    int pull_queues = 0;
    cudaEvent_t ev_recv[2] = {nullptr, nullptr}, ev_done[2] = {nullptr, nullptr}, ev_start = nullptr;
    cudaEvent_t ev_packed[2] = {nullptr, nullptr};
    ncclComm_t comm = nullptr;
    // The communicator was aborted (an NCCL async error, or a host wait past the deadline): every
    // later collective step of this handle refuses with LYTH_E_NCCL, and teardown skips
    // ncclCommDestroy (the abort freed the communicator).
    bool comm_aborted = false;
    double deadline_ms = 300000.0;  // lyth_sv_set_deadline
    std::vector<uint32_t> pos;  // logical qubit -> physical bit
    std::vector<uint32_t> inv;  // physical bit -> logical qubit
    uint64_t passes = 0, exchanges = 0, bytes_sent = 0, launches = 0;
    // Per-class device timing (lyth_sv_set_timing): pending event pairs, folded totals.
    bool timing = false;
    struct Mark { int cls; cudaEvent_t a, b; };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> pool;
    uint64_t t_count[5] = {0, 0, 0, 0, 0};
    double t_ms[5] = {0, 0, 0, 0, 0};
    // Fusion (lyth_sv_set_fusion): the open group of consecutive local gates, on physical bits.
    int fuse_k = kFuseMaxQubits;
    FusedGroup open{};
    // Rank-bit gates: 1 = swap the qubit into a local bit first (default), 0 = pairwise
    // exchange of the whole shard and compute this rank's row.
    int remap = 1;
    // Most rank-bit qubits one swap-in may bring in together (lyth_sv_set_swap_batch). With
    // diagonal rank-bit gates moving no data, the swap-ins left are the rank-bit qubits' non-
    // diagonal gates, which a batch takes in one exchange among 2^k ranks: fewer bytes than k
    // single swaps, and no single-gate passes squeezed between consecutive swap-ins.
    int swap_batch = 6;
    // Diagonal gates on rank bits (lyth_sv_set_diagonal): 1 = no exchange -- on a shard whose
    // rank bit is v the gate is the scalar u_vv (under its control, when it has one), applied as
    // a local gate diag(u_vv, u_vv); 0 = swap-in or exchange like any other gate.
    int diag = 1;
    // Copy-engine transport for swap-ins (multi-rank): every rank's send chunks and flag block
    // mapped through CUDA IPC; a rank pulls its partners' packed slices with cudaMemcpyAsync on
    // the copy engines. Flag block (kFlagWords u64): [r * 2 + b] = last chunk rank r packed for
    // this rank into its send slot b; [kPulledAt + r * 2 + b] = last chunk rank r pulled from this
    // rank's send slot b.
    bool ce = false;
    // With `ce`, how swap-ins move (lyth_sv_set_transport 1-4): kPeerNone -- copy-engine pulls
    // into the receive chunks; kPeerLoad -- SM-issued peer loads fused with the unpack
    // (pull_unpack_kernel); kPeerMixed -- copy engines pairwise, peer loads for batched swap-ins
    // (several partners); kPeerStore -- SM stores of this rank's packed chunks straight into the
    // partners' shards (push_kernel). Every form leaves the flags and send slots as the next one
    // expects, so they mix freely.
    int peer_mode = 0;
    uint64_t *flags = nullptr;
    std::vector<float *> peer_sre[2], peer_sim[2];
    std::vector<uint64_t *> peer_flags;  // every rank's flag block (own included)
    std::vector<float *> peer_re, peer_im;  // every rank's shard (the push form's destinations)
    // every rank's IPC handles from set-up: the shards are opened only when the push form is
    // selected (lyth_sv_set_transport 4), so the other forms map just the chunks and flags
    std::vector<IpcRec> ipc_all;
    std::vector<void *> ipc_opened;
    uint64_t xseq = 0;                       // chunk sequence number, identical on every rank
    uint64_t slot_seq[2] = {0, 0};           // last chunk packed into send slot b
    std::vector<int> slot_partners[2];       // the ranks that pull it
    // Plan handle (lyth_sv_plan_create): no device state; each step is appended here instead.
    bool plan = false;
    std::vector<lyth_sv_op> ops;
};
static_assert(kFuseMaxQubits == LYTH_SV_FUSE_MAX_QUBITS && kFuseMaxGates == LYTH_SV_FUSE_MAX_GATES,
              "plan op layout");

namespace {

// Exchange chunk: 256 Mi amplitudes (1 GiB per component, 2 GiB per NCCL group each way).
// NCCL's point-to-point bandwidth on B200 NVLink grows with the message: measured per direction
// 277 GB/s at 64 MiB, 332 at 256 MiB, 639 at 1 GiB. The four chunk buffers (send and receive,
// double-buffered, both components) take 8 GiB per rank, next to a shard of 8-32 GiB.
constexpr uint64_t kChunk = 1ull << 28;
constexpr int kInitBlocks = 1184;

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    explicit DeviceGuard(const lyth_sv *sv) {
        if (sv->plan) return;  // a plan handle makes no CUDA call
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(sv->device);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int nccl_status(ncclResult_t r) { return r == ncclSuccess ? LYTH_OK : LYTH_E_NCCL; }

// Synchronise `stream` of a handle. With a live communicator the wait polls the stream and the
// communicator's async error and gives up at the handle's deadline (wait_with_deadline): a peer
// that died leaves this rank with LYTH_E_NCCL or LYTH_E_TIMEOUT and an aborted communicator
// instead of a hang. Without one it is a plain synchronisation.
struct SyncCtx {
    lyth_sv *sv;
    cudaStream_t stream;
};
int sync_stream(lyth_sv *sv, cudaStream_t stream) {
    if (!stream) return LYTH_OK;
    if (!sv->comm || sv->comm_aborted || !g_nccl.CommGetAsyncError) return status_of(cudaStreamSynchronize(stream));
    SyncCtx c{sv, stream};
    WaitHooks h;
    h.ctx = &c;
    h.query = [](void *p) {
        const cudaError_t e = cudaStreamQuery(static_cast<SyncCtx *>(p)->stream);
        if (e == cudaSuccess) return 0;
        if (e == cudaErrorNotReady) return 1;
        return status_of(e);
    };
    h.async_error = [](void *p) {
        ncclResult_t r = ncclSuccess;
        if (g_nccl.CommGetAsyncError(static_cast<SyncCtx *>(p)->sv->comm, &r) != ncclSuccess) return 1;
        return (r != ncclSuccess && r != ncclInProgress) ? 1 : 0;
    };
    h.abort = [](void *p) {
        lyth_sv *v = static_cast<SyncCtx *>(p)->sv;
        if (g_nccl.CommAbort && v->comm) g_nccl.CommAbort(v->comm);
        v->comm_aborted = true;
    };
    return wait_with_deadline(h, sv->deadline_ms, 50, nullptr);
}

// Every queue of the handle drained: the communication and copy queues first (pulls and NCCL),
// then the compute stream. The pulls on the extra queues are also joined into the communication
// stream by events; draining them here keeps that from being the only guarantee.
int drain_all(lyth_sv *sv) {
    int st = sync_stream(sv, sv->comm_stream);
    if (!st && sv->copy_stream) st = sync_stream(sv, sv->copy_stream);
    for (int i = 0; !st && i < lyth_sv::kExtraQueues; i++)
        if (sv->xq[i]) st = sync_stream(sv, sv->xq[i]);
    if (!st) st = sync_stream(sv, sv->stream);
    return st;
}

void reset_map(lyth_sv *sv) {
    sv->pos.resize(sv->qubits);
    sv->inv.resize(sv->qubits);
    for (uint32_t q = 0; q < sv->qubits; q++) sv->pos[q] = sv->inv[q] = q;
}

cudaEvent_t take_event(lyth_sv *sv) {
    if (!sv->pool.empty()) {
        cudaEvent_t e = sv->pool.back();
        sv->pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Opens a timed region of class `cls` on the compute stream (no-op when timing is off).
int mark_begin(lyth_sv *sv, int cls) {
    if (!sv->timing || sv->plan) return -1;
    sv->marks.push_back({cls, take_event(sv), take_event(sv)});
    cudaEventRecord(sv->marks.back().a, sv->stream);
    return (int)sv->marks.size() - 1;
}
void mark_end(lyth_sv *sv, int idx) {
    if (idx >= 0) cudaEventRecord(sv->marks[idx].b, sv->stream);
}

int fold_timing(lyth_sv *sv) {
    if (sv->marks.empty()) return LYTH_OK;
    int st = status_of(cudaStreamSynchronize(sv->stream));
    if (st) return st;
    for (auto &mk : sv->marks) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, mk.a, mk.b) == cudaSuccess) {
            sv->t_count[mk.cls]++;
            sv->t_ms[mk.cls] += ms;
        }
        sv->pool.push_back(mk.a);
        sv->pool.push_back(mk.b);
    }
    sv->marks.clear();
    return LYTH_OK;
}

lyth_sv_op &record(lyth_sv *sv, int kind, int a, int b, int c) {
    sv->ops.emplace_back();
    lyth_sv_op &op = sv->ops.back();
    memset(&op, 0, sizeof op);
    op.kind = kind;
    op.a = a;
    op.b = b;
    op.c = c;
    return op;
}
void set_m(lyth_sv_op &op, const U8 &m) {
    const float v[8] = {m.ar, m.ai, m.br, m.bi, m.cr, m.ci, m.dr, m.di};
    memcpy(op.m, v, sizeof v);
}

// The rank bit b of this rank.
inline int rank_bit(const lyth_sv *sv, uint32_t b) { return (sv->rank >> b) & 1; }

// Off-diagonal entries all zero (either sign).
inline bool is_diag(const U8 &m) { return m.br == 0.f && m.bi == 0.f && m.cr == 0.f && m.ci == 0.f; }

// Row v of a diagonal gate as the local gate diag(u_vv, u_vv). Its fma chains give every
// amplitude the value the full gate gives it (u_vv times the amplitude): the terms dropped are
// products with the zero off-diagonal entries, which change no nonzero sum, only the sign an
// exactly-zero result takes (and NaN from a non-finite partner).
inline U8 scalar_row(const U8 &m, int v) {
    const float r = v ? m.dr : m.ar, i = v ? m.di : m.ai;
    return U8{r, i, 0.f, 0.f, 0.f, 0.f, r, i};
}
inline bool is_one(const U8 &s) { return s.ar == 1.f && s.ai == 0.f; }

// A local bit to carry a scalar gate: one the open fused group already holds (so the group does
// not widen), else bit 0 / 1; never `avoid` (the control of a controlled scalar).
uint32_t carrier(const lyth_sv *sv, int avoid) {
    for (int l = 0; l < sv->open.k; l++)
        if ((int)sv->open.bits[l] != avoid) return sv->open.bits[l];
    return avoid == 0 ? 1u : 0u;
}

// A gate whose target is rank bit b: chunked pairwise exchange, then this rank's row.
int exchange_gate(lyth_sv *sv, uint32_t b, const U8 &m, int ctrl_bit) {
    if (sv->plan) {
        set_m(record(sv, LYTH_SV_OP_EXCHANGE, (int)b, 0, ctrl_bit), m);
        sv->bytes_sent += 2 * sv->local_len * sizeof(float);
        sv->exchanges++;
        sv->passes++;
        return LYTH_OK;
    }
    const int partner = sv->rank ^ (1 << b);
    const int side = rank_bit(sv, b);
    const int mk = mark_begin(sv, LYTH_SV_T_EXCHANGE);
    int st = status_of(cudaEventRecord(sv->ev_start, sv->stream));
    if (st) return st;
    st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_start, 0));
    if (st) return st;
    const uint64_t nchunks = (sv->local_len + sv->chunk - 1) / sv->chunk;
    for (uint64_t c = 0; c < nchunks; c++) {
        const int buf = (int)(c & 1);
        const uint64_t off = c * sv->chunk;
        const uint64_t len = (sv->local_len - off) < sv->chunk ? (sv->local_len - off) : sv->chunk;
        if (c >= 2) {
            st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_done[buf], 0));
            if (st) return st;
        }
        if ((st = nccl_status(g_nccl.GroupStart()))) return st;
        g_nccl.Send(sv->re + off, len, ncclFloat32, partner, sv->comm, sv->comm_stream);
        g_nccl.Send(sv->im + off, len, ncclFloat32, partner, sv->comm, sv->comm_stream);
        g_nccl.Recv(sv->rre[buf], len, ncclFloat32, partner, sv->comm, sv->comm_stream);
        g_nccl.Recv(sv->rim[buf], len, ncclFloat32, partner, sv->comm, sv->comm_stream);
        if ((st = nccl_status(g_nccl.GroupEnd()))) return st;
        if ((st = status_of(cudaEventRecord(sv->ev_recv[buf], sv->comm_stream)))) return st;
        if ((st = status_of(cudaStreamWaitEvent(sv->stream, sv->ev_recv[buf], 0)))) return st;
        if ((st = launch_exchange_u(len, off, side, ctrl_bit, m, sv->re + off, sv->im + off, sv->rre[buf],
                                    sv->rim[buf], sv->stream)))
            return st;
        if ((st = status_of(cudaEventRecord(sv->ev_done[buf], sv->stream)))) return st;
        sv->bytes_sent += 2 * len * sizeof(float);
        sv->launches++;
    }
    mark_end(sv, mk);
    sv->exchanges++;
    sv->passes++;
    return LYTH_OK;
}

// A local 1-qubit or 2-qubit pass, counted and (when on) timed.
int local_u(lyth_sv *sv, uint32_t p, const U8 &m) {
    if (sv->plan) {
        set_m(record(sv, LYTH_SV_OP_U, (int)p, 0, 0), m);
        sv->passes++;
        return LYTH_OK;
    }
    const int mk = mark_begin(sv, LYTH_SV_T_U);
    const int st = launch_u(sv->local_len, p, m, sv->re, sv->im, sv->re, sv->im, sv->stream);
    mark_end(sv, mk);
    sv->passes++;
    sv->launches++;
    return st;
}
int local_cu(lyth_sv *sv, uint32_t pc, uint32_t pt, const U8 &m) {
    if (sv->plan) {
        set_m(record(sv, LYTH_SV_OP_CU, (int)pc, (int)pt, 0), m);
        sv->passes++;
        return LYTH_OK;
    }
    const int mk = mark_begin(sv, LYTH_SV_T_CU);
    const int st = launch_cu(sv->local_len, pc, pt, m, sv->re, sv->im, sv->re, sv->im, sv->stream);
    mark_end(sv, mk);
    sv->passes++;
    sv->launches++;
    return st;
}

// ---- fusion: lyth-circuit's greedy in-order rule (lib.rs:72-100) on physical local bits. A
// gate joins the open group while the union of bits stays within fuse_k (and the group has
// room); otherwise the group is run and the gate opens the next. A group of one gate runs the
// specialised single-gate pass (the in-place CU then skips its control=0 half).
int level_of(FusedGroup &g, uint32_t bit) {
    for (int l = 0; l < g.k; l++)
        if (g.bits[l] == bit) return l;
    return -1;
}

int flush_group(lyth_sv *sv) {
    FusedGroup &g = sv->open;
    if (g.ngates == 0) return LYTH_OK;
    int st;
    if (g.ngates == 1) {
        const FusedGate &fg = g.gates[0];
        const U8 m{fg.m[0], fg.m[1], fg.m[2], fg.m[3], fg.m[4], fg.m[5], fg.m[6], fg.m[7]};
        st = fg.c < 0 ? local_u(sv, g.bits[fg.t], m) : local_cu(sv, g.bits[fg.c], g.bits[fg.t], m);
    } else {
        for (int l = 0; l < g.k; l++) g.sorted[l] = g.bits[l];
        for (int i = 1; i < g.k; i++)
            for (int j = i; j > 0 && g.sorted[j - 1] > g.sorted[j]; j--) {
                const uint32_t t = g.sorted[j];
                g.sorted[j] = g.sorted[j - 1];
                g.sorted[j - 1] = t;
            }
        if (sv->plan) {
            lyth_sv_op &op = record(sv, LYTH_SV_OP_FUSED, 0, 0, 0);
            op.k = g.k;
            for (int l = 0; l < g.k; l++) op.bits[l] = g.bits[l];
            op.ngates = g.ngates;
            for (uint32_t i = 0; i < g.ngates; i++) {
                op.gt[i] = g.gates[i].t;
                op.gc[i] = g.gates[i].c;
                memcpy(op.gm[i], g.gates[i].m, sizeof op.gm[i]);
            }
            st = LYTH_OK;
        } else {
            const int mk = mark_begin(sv, LYTH_SV_T_FUSED);
            st = launch_fused(sv->local_len, g, sv->re, sv->im, sv->stream);
            mark_end(sv, mk);
            sv->launches++;
        }
        sv->passes++;
    }
    g.k = 0;
    g.ngates = 0;
    return st;
}

// Queue a local gate: c < 0 for a U on bit t, else a CU (control c, target t).
int add_local(lyth_sv *sv, int c, uint32_t t, const U8 &m) {
    if (sv->fuse_k <= 1) return c < 0 ? local_u(sv, t, m) : local_cu(sv, (uint32_t)c, t, m);
    FusedGroup &g = sv->open;
    int extra = (level_of(g, t) < 0) + (c >= 0 && level_of(g, (uint32_t)c) < 0);
    bool fits = g.k + extra <= sv->fuse_k;
    if (fits && extra) {  // the union must also run as one pass at this size (fused_fits)
        uint32_t u[kFuseMaxQubits];
        int n = 0;
        for (int l = 0; l < g.k; l++) u[n++] = g.bits[l];
        if (level_of(g, t) < 0) u[n++] = t;
        if (c >= 0 && level_of(g, (uint32_t)c) < 0) u[n++] = (uint32_t)c;
        fits = fused_fits(sv->local_len, u, n);
    }
    if (g.ngates > 0 && (!fits || g.ngates == (uint32_t)kFuseMaxGates)) {
        int st = flush_group(sv);
        if (st) return st;
    }
    if (level_of(g, t) < 0) g.bits[g.k++] = t;
    if (c >= 0 && level_of(g, (uint32_t)c) < 0) g.bits[g.k++] = (uint32_t)c;
    FusedGate &fg = g.gates[g.ngates++];
    fg.t = (int8_t)level_of(g, t);
    fg.c = (int8_t)(c >= 0 ? level_of(g, (uint32_t)c) : -1);
    fg.pad = 0;
    fg.m[0] = m.ar; fg.m[1] = m.ai; fg.m[2] = m.br; fg.m[3] = m.bi;
    fg.m[4] = m.cr; fg.m[5] = m.ci; fg.m[6] = m.dr; fg.m[7] = m.di;
    return LYTH_OK;
}

// [kLandedAt + r * 2 + b]: last chunk rank r stored into this rank's shard from its send slot b
// (the push form).
constexpr int kFlagRanks = 64, kPulledAt = 2 * kFlagRanks, kLandedAt = 4 * kFlagRanks, kFlagWords = 6 * kFlagRanks;
constexpr int kPeerNone = 0, kPeerLoad = 1, kPeerMixed = 2, kPeerStore = 3;

// Wait on `stream` until this rank's own flags [base + r * 2 + b] for the listed ranks are >= target.
int wait_own(lyth_sv *sv, cudaStream_t stream, const std::vector<int> &ranks, int base, int b, uint64_t target) {
    FlagSet fs{};
    fs.n = (uint32_t)ranks.size();
    for (uint32_t i = 0; i < fs.n; i++) fs.flag[i] = sv->flags + base + ranks[i] * 2 + b;
    flag_wait_kernel<<<1, 64, 0, stream>>>(fs, target);
    sv->launches++;
    return last_launch_status();
}
// Store `value` into flag [base + rank * 2 + b] of each listed rank's block (after `stream`'s work).
int put_peers(lyth_sv *sv, cudaStream_t stream, const std::vector<int> &ranks, int base, int b, uint64_t value) {
    FlagPut fp{};
    fp.n = (uint32_t)ranks.size();
    for (uint32_t i = 0; i < fp.n; i++) fp.flag[i] = sv->peer_flags[ranks[i]] + base + sv->rank * 2 + b;
    flags_put_kernel<<<1, 64, 0, stream>>>(fp, value);
    sv->launches++;
    return last_launch_status();
}

// Swap of local bits V[j] with physical rank bits Gp[j], j < k: one exchange among the 2^k ranks
// that differ only in those rank bits. Rank r keeps the subset whose local bits equal its own rank
// bits and trades subset q with the rank whose rank bits are q, into the same positions:
// (2^k - 1) / 2^k of the shard each way (half for k = 1). Pipelined chunk by chunk on two streams:
// pack(c + 1) on the compute stream while chunk c moves on the communication stream, unpack(c) as
// it lands, send and receive chunks double-buffered.
//
// Transport: with the copy-engine path (CUDA IPC maps every rank's send chunks and flags), a rank
// pulls its slice of each partner's packed chunk with cudaMemcpyAsync -- copy engines over NVLink,
// no SMs -- after the partner's `packed` flag reaches the chunk's sequence number, then raises its
// own `pulled` flag; a rank re-packs a send slot only after every partner that pulls from it has
// raised `pulled` past it. The peer-load form keeps that protocol with pull_unpack_kernel in place
// of the copies and the unpack (it also waits for this rank's own pack of the chunk, whose
// positions it overwrites). The push form reads `packed` as "these positions are free": once
// every partner has packed chunk c, a rank stores its packed slices into their shards
// (push_kernel) and raises `landed` in each; the swap-in ends on the compute stream when every
// partner's last `landed` has arrived. Otherwise NCCL send / recv in one group per chunk. NCCL's transfer runs
// on SMs: measured on B200, its point-to-point bandwidth halves when a memory-bound kernel shares
// every SM with it, so on that path pack / unpack take half the SMs.
int physical_swap_multi(lyth_sv *sv, const std::vector<uint32_t> &V, const std::vector<uint32_t> &Gp) {
    const uint32_t k = (uint32_t)V.size(), L = sv->local_bits;
    const uint32_t P = (1u << k) - 1;
    const uint64_t sub = sv->local_len >> k;
    uint32_t qself = 0;
    for (uint32_t j = 0; j < k; j++) qself |= (uint32_t)rank_bit(sv, Gp[j] - L) << j;
    MultiPat mp{};
    mp.k = k;
    uint32_t order[8];
    for (uint32_t j = 0; j < k; j++) order[j] = j;
    for (uint32_t a = 1; a < k; a++)
        for (uint32_t b = a; b > 0 && V[order[b - 1]] > V[order[b]]; b--) { const uint32_t t = order[b]; order[b] = order[b - 1]; order[b - 1] = t; }
    for (uint32_t s = 0; s < k; s++) mp.vs[s] = V[order[s]];
    std::vector<int> partner;
    std::vector<uint32_t> myslice;  // the slice of partner y's send chunk that holds this rank's data
    for (uint32_t q = 0; q <= P; q++) {
        if (q == qself) continue;
        int r = sv->rank;
        uint32_t pat = 0;
        for (uint32_t j = 0; j < k; j++)
            r = (r & ~(1 << (Gp[j] - L))) | (int)(((q >> j) & 1u) << (Gp[j] - L));
        for (uint32_t s = 0; s < k; s++) pat |= ((q >> order[s]) & 1u) << s;
        mp.pattern[partner.size()] = pat;
        partner.push_back(r);
        myslice.push_back(qself < q ? qself : qself - 1);
    }
    auto remap_bits = [&]() {
        for (uint32_t j = 0; j < k; j++) {
            const uint32_t p1 = V[j], p2 = Gp[j];
            const uint32_t q1 = sv->inv[p1], q2 = sv->inv[p2];
            sv->pos[q1] = p2; sv->pos[q2] = p1;
            sv->inv[p1] = q2; sv->inv[p2] = q1;
        }
    };
    if (sv->plan) {
        if (k == 1) {
            record(sv, LYTH_SV_OP_SWAP_LR, (int)V[0], (int)(Gp[0] - L), 0);
        } else {
            lyth_sv_op &op = record(sv, LYTH_SV_OP_SWAP_MULTI, 0, 0, 0);
            op.k = (int32_t)k;
            for (uint32_t j = 0; j < k; j++) { op.bits[j] = V[j]; op.rbits[j] = Gp[j] - L; }
        }
        sv->bytes_sent += 2 * P * sub * sizeof(float);
        sv->exchanges++;
        remap_bits();
        return LYTH_OK;
    }
    // elements per partner per chunk: a chunk buffer holds P slices
    uint64_t C = sv->chunk >> (k == 1 ? 0 : k);
    if (C > sub) C = sub;
    // Over the copy engines a swap-in is cut into at least 8 chunks (of >= 2^24 amplitudes), so
    // the first pack and the last unpack, the parts the pipeline cannot hide, stay short; copy-
    // engine pulls keep their bandwidth at that size.
    if (sv->ce) {
        uint64_t c8 = sub >> 3;
        if (c8 < (1ull << 24)) c8 = 1ull << 24;
        if (C > c8) C = c8;
    }
    const uint64_t nchunks = sub / C;
    const unsigned gx_cap = sv->ce ? (unsigned)device_sms() * 2u : (unsigned)device_sms() / 2u;
    unsigned gx = stream_grid(C / 4 + 1, 1024);
    if (gx * P > gx_cap) gx = gx_cap / P > 0 ? gx_cap / P : 1;
    const dim3 grid(gx, P);
    const bool pl = sv->ce && (sv->peer_mode == kPeerLoad || (sv->peer_mode == kPeerMixed && P > 1));
    // the push form: this rank stores its packed slices into the partners' shards once their own
    // pack of the chunk has read the positions it overwrites
    const bool ps = sv->ce && sv->peer_mode == kPeerStore;
    uint32_t patself = 0;  // the subset pattern this rank's data takes in every partner's shard
    for (uint32_t s = 0; s < k; s++) patself |= ((qself >> order[s]) & 1u) << s;
    // the peer-load pull and the push: about two 512-thread blocks per SM over all partners, next
    // to the pack
    const unsigned pgx = std::max(1u, (unsigned)device_sms() * 2u / P);
    const dim3 pgrid(std::min<unsigned>(pgx, stream_grid(C / 8 + 1, 512)), P);
    const int mk = mark_begin(sv, LYTH_SV_T_SWAP);
    int st = status_of(cudaEventRecord(sv->ev_start, sv->stream));
    if (st) return st;
    if ((st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_start, 0)))) return st;
    const uint64_t seq0 = sv->xseq;
    auto pack = [&](uint64_t c) -> int {
        const int b = (int)(c & 1);
        int r;
        // the send slot is re-packed once every rank that pulls its last chunk has done so
        if (sv->ce && sv->slot_seq[b] && (r = wait_own(sv, sv->stream, sv->slot_partners[b], kPulledAt, b, sv->slot_seq[b])))
            return r;
        // (the push form's own push of chunk c - 2 from this slot is ordered before this on the
        // compute stream: see the wait on ev_recv below)
        pack_multi_kernel<<<grid, 1024, 0, sv->stream>>>(C, c * C, mp, sv->re, sv->im, sv->sre[b], sv->sim[b]);
        sv->launches++;
        if ((r = last_launch_status())) return r;
        if (sv->ce) {
            // "packed": the slot holds chunk c, and this rank's chunk-c positions are free
            if ((r = put_peers(sv, sv->stream, partner, 0, b, seq0 + c + 1))) return r;
            sv->slot_seq[b] = ps ? 0 : seq0 + c + 1;  // nobody pulls a pushed slot
            if (ps) sv->slot_partners[b].clear();
            else sv->slot_partners[b] = partner;
        }
        return status_of(cudaEventRecord(sv->ev_packed[b], sv->stream));
    };
    if ((st = pack(0))) return st;
    for (uint64_t c = 0; c < nchunks; c++) {
        const int b = (int)(c & 1);
        const uint64_t seq = seq0 + c + 1;
        // receive slot b is free once unpack(c - 2) has drained it
        if (c >= 2 && !pl && !ps && (st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_done[b], 0)))) return st;
        if (ps) {
            // this rank's slices of chunk c are packed, and every partner has packed (read) the
            // positions they go to
            if ((st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_packed[b], 0)))) return st;
            if ((st = wait_own(sv, sv->comm_stream, partner, 0, b, seq))) return st;
            PeerDst pd{};
            for (uint32_t y = 0; y < P; y++) {
                pd.re[y] = sv->peer_re[partner[y]];
                pd.im[y] = sv->peer_im[partner[y]];
            }
            push_kernel<<<pgrid, 512, 0, sv->comm_stream>>>(C, c * C, mp, patself, sv->sre[b], sv->sim[b], pd);
            sv->launches++;
            if ((st = last_launch_status())) return st;
            if ((st = put_peers(sv, sv->comm_stream, partner, kLandedAt, b, seq))) return st;
        } else if (pl) {
            // the pull overwrites the positions pack(c) read on the compute stream
            if ((st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_packed[b], 0)))) return st;
            if ((st = wait_own(sv, sv->comm_stream, partner, 0, b, seq))) return st;
            PeerSrc srcs{};
            for (uint32_t y = 0; y < P; y++) {
                srcs.re[y] = sv->peer_sre[b][partner[y]] + (uint64_t)myslice[y] * C;
                srcs.im[y] = sv->peer_sim[b][partner[y]] + (uint64_t)myslice[y] * C;
            }
            pull_unpack_kernel<<<pgrid, 512, 0, sv->comm_stream>>>(C, c * C, mp, srcs, sv->re, sv->im);
            sv->launches++;
            if ((st = last_launch_status())) return st;
            if ((st = put_peers(sv, sv->comm_stream, partner, kPulledAt, b, seq))) return st;
        } else if (sv->ce) {
            // re halves on the communication stream, im halves on a second stream: two copy
            // engines in flight
            if ((st = wait_own(sv, sv->comm_stream, partner, 0, b, seq))) return st;
            if ((st = status_of(cudaEventRecord(sv->ev_pull, sv->comm_stream)))) return st;
            // the queues: comm_stream, copy_stream, then the extra ones. A set count cuts each
            // component's slice into Q pieces; by default (0) every partner's two slices get a
            // queue each, up to all of them, so the pulls from several partners run at once.
            const int Q = sv->pull_queues > 0 ? sv->pull_queues
                                               : (int)std::min<uint32_t>(2u * P, 2u + lyth_sv::kExtraQueues);
            cudaStream_t qs[2 + lyth_sv::kExtraQueues] = {sv->comm_stream, sv->copy_stream};
            for (int i = 0; i < lyth_sv::kExtraQueues; i++) qs[2 + i] = sv->xq[i];
            for (int i = 1; i < Q; i++)
                if ((st = status_of(cudaStreamWaitEvent(qs[i], sv->ev_pull, 0)))) return st;
            const uint64_t piece = sv->pull_queues > 0 ? (C + (uint64_t)Q - 1) / (uint64_t)Q : C;
            int next = 0;
            for (uint32_t y = 0; y < P; y++) {
                const uint64_t off = (uint64_t)y * C, src = (uint64_t)myslice[y] * C;
                for (int comp = 0; comp < 2; comp++) {
                    float *dst = (comp ? sv->rim[b] : sv->rre[b]) + off;
                    const float *from = (comp ? sv->peer_sim[b][partner[y]] : sv->peer_sre[b][partner[y]]) + src;
                    for (uint64_t p0 = 0; p0 < C; p0 += piece) {
                        const uint64_t len = C - p0 < piece ? C - p0 : piece;
                        if ((st = status_of(cudaMemcpyAsync(dst + p0, from + p0, len * sizeof(float),
                                                            cudaMemcpyDeviceToDevice, qs[next]))))
                            return st;
                        next = (next + 1) % Q;
                    }
                }
            }
            for (int i = 1; i < Q; i++) {
                cudaEvent_t ev = i == 1 ? sv->ev_copied : sv->ev_xq[i - 2];
                if ((st = status_of(cudaEventRecord(ev, qs[i])))) return st;
                if ((st = status_of(cudaStreamWaitEvent(sv->comm_stream, ev, 0)))) return st;
            }
            if ((st = put_peers(sv, sv->comm_stream, partner, kPulledAt, b, seq))) return st;
        } else {
            if ((st = status_of(cudaStreamWaitEvent(sv->comm_stream, sv->ev_packed[b], 0)))) return st;
            if ((st = nccl_status(g_nccl.GroupStart()))) return st;
            for (uint32_t y = 0; y < P; y++) {
                const uint64_t off = (uint64_t)y * C;
                g_nccl.Send(sv->sre[b] + off, C, ncclFloat32, partner[y], sv->comm, sv->comm_stream);
                g_nccl.Send(sv->sim[b] + off, C, ncclFloat32, partner[y], sv->comm, sv->comm_stream);
                g_nccl.Recv(sv->rre[b] + off, C, ncclFloat32, partner[y], sv->comm, sv->comm_stream);
                g_nccl.Recv(sv->rim[b] + off, C, ncclFloat32, partner[y], sv->comm, sv->comm_stream);
            }
            if ((st = nccl_status(g_nccl.GroupEnd()))) return st;
        }
        if ((st = status_of(cudaEventRecord(sv->ev_recv[b], sv->comm_stream)))) return st;
        sv->bytes_sent += 2 * P * C * sizeof(float);
        if (c + 1 < nchunks && (st = pack(c + 1))) return st;
        if ((st = status_of(cudaStreamWaitEvent(sv->stream, sv->ev_recv[b], 0)))) return st;
        if (!pl && !ps) {
            unpack_multi_kernel<<<grid, 1024, 0, sv->stream>>>(C, c * C, mp, sv->re, sv->im, sv->rre[b], sv->rim[b]);
            sv->launches++;
            if ((st = last_launch_status())) return st;
            if ((st = status_of(cudaEventRecord(sv->ev_done[b], sv->stream)))) return st;
        }
    }
    if (ps) {
        // every partner's stores into this shard have landed: a partner raises "landed" for its
        // chunks in order, so the last chunk of each slot covers the earlier ones
        const int bl = (int)((nchunks - 1) & 1);
        if ((st = wait_own(sv, sv->stream, partner, kLandedAt, bl, seq0 + nchunks))) return st;
        if (nchunks >= 2 && (st = wait_own(sv, sv->stream, partner, kLandedAt, bl ^ 1, seq0 + nchunks - 1))) return st;
    }
    sv->xseq = seq0 + nchunks;
    mark_end(sv, mk);
    sv->exchanges++;
    remap_bits();
    return LYTH_OK;
}

// Physical swap of rank bits b1, b2: ranks whose two bits differ trade whole shards with the
// rank that has them exchanged.
int physical_swap_global_global(lyth_sv *sv, uint32_t b1, uint32_t b2) {
    if (sv->plan) {
        record(sv, LYTH_SV_OP_SWAP_RR, (int)b1, (int)b2, 0);
        if (rank_bit(sv, b1) != rank_bit(sv, b2)) {
            sv->bytes_sent += 2 * sv->local_len * sizeof(float);
            sv->exchanges++;
        }
        return LYTH_OK;
    }
    if (rank_bit(sv, b1) == rank_bit(sv, b2)) return LYTH_OK;
    const int partner = sv->rank ^ (1 << b1) ^ (1 << b2);
    int st = LYTH_OK;
    for (uint64_t off = 0; off < sv->local_len; off += sv->chunk) {
        const uint64_t len = (sv->local_len - off) < sv->chunk ? (sv->local_len - off) : sv->chunk;
        if ((st = status_of(cudaStreamSynchronize(sv->stream)))) return st;
        if ((st = nccl_status(g_nccl.GroupStart()))) return st;
        g_nccl.Send(sv->re + off, len, ncclFloat32, partner, sv->comm, sv->stream);
        g_nccl.Send(sv->im + off, len, ncclFloat32, partner, sv->comm, sv->stream);
        g_nccl.Recv(sv->rre[0], len, ncclFloat32, partner, sv->comm, sv->stream);
        g_nccl.Recv(sv->rim[0], len, ncclFloat32, partner, sv->comm, sv->stream);
        if ((st = nccl_status(g_nccl.GroupEnd()))) return st;
        if ((st = status_of(cudaMemcpyAsync(sv->re + off, sv->rre[0], len * 4, cudaMemcpyDeviceToDevice, sv->stream)))) return st;
        if ((st = status_of(cudaMemcpyAsync(sv->im + off, sv->rim[0], len * 4, cudaMemcpyDeviceToDevice, sv->stream)))) return st;
        sv->bytes_sent += 2 * len * sizeof(float);
    }
    sv->exchanges++;
    return LYTH_OK;
}

// Swap physical bits p1 < p2 with real data motion, and update the map to match.
int physical_swap(lyth_sv *sv, uint32_t p1, uint32_t p2) {
    if (p1 == p2) return LYTH_OK;
    if (p1 > p2) { uint32_t t = p1; p1 = p2; p2 = t; }
    const uint32_t L = sv->local_bits;
    int st;
    if (p2 < L && sv->plan) {
        record(sv, LYTH_SV_OP_SWAP_LOCAL, (int)p1, (int)p2, 0);
        sv->passes++;
        st = LYTH_OK;
    } else if (p2 < L) {
        st = launch_swap(sv->local_len, p1, p2, sv->re, sv->im, sv->re, sv->im, sv->stream);
        sv->passes++;
        sv->launches++;
    } else if (p1 < L) {
        return physical_swap_multi(sv, std::vector<uint32_t>{p1}, std::vector<uint32_t>{p2});  // updates the map
    } else {
        st = physical_swap_global_global(sv, p1 - L, p2 - L);
    }
    if (st) return st;
    const uint32_t q1 = sv->inv[p1], q2 = sv->inv[p2];
    sv->pos[q1] = p2; sv->pos[q2] = p1;
    sv->inv[p1] = q2; sv->inv[p2] = q1;
    return LYTH_OK;
}

// Move local bits src[j] -> dst[j] (j < k <= 6, dst a permutation of src) in one in-place pass
// and update the map. LYTH_E_UNSUPPORTED: the state is below the tile pass's size.
int permute_local(lyth_sv *sv, const std::vector<uint32_t> &src, const std::vector<uint32_t> &dst) {
    const int k = (int)src.size();
    if (sv->plan) {
        if (!permute_supported(sv->local_len, src.data(), k)) return LYTH_E_UNSUPPORTED;  // as the engine
        lyth_sv_op &op = record(sv, LYTH_SV_OP_PERMUTE, 0, 0, 0);
        op.k = k;
        for (int j = 0; j < k; j++) { op.bits[j] = src[j]; op.rbits[j] = dst[j]; }
    } else {
        const int st = launch_permute(sv->local_len, src.data(), dst.data(), k, sv->re, sv->im, sv->stream);
        if (st) return st;
        sv->launches++;
    }
    sv->passes++;
    std::vector<uint32_t> moved(k);
    for (int j = 0; j < k; j++) moved[j] = sv->inv[src[j]];
    for (int j = 0; j < k; j++) {
        sv->inv[dst[j]] = moved[j];
        sv->pos[moved[j]] = dst[j];
    }
    return LYTH_OK;
}

// Undo the qubit map, so physical bit q holds logical qubit q. The qubits that belong on rank bits
// come home first by swaps; the local bits then hold a permutation of the local qubits, applied by
// permutation passes of up to 6 bits each (a cycle of the permutation, several short ones
// together, or a piece of a long one) instead of one swap pass per transposition.
int normalize(lyth_sv *sv) {
    const uint32_t L = sv->local_bits;
    int st;
    for (uint32_t q = L; q < sv->qubits; q++)
        if (sv->pos[q] != q && (st = physical_swap(sv, q, sv->pos[q]))) return st;
    // the cycles of sigma on the local bits (physical bit a's value belongs at bit inv[a]), all
    // taken from the map before any pass
    std::vector<std::vector<uint32_t>> cycles;
    std::vector<bool> seen(L, false);
    for (uint32_t p = 0; p < L; p++) {
        if (seen[p] || sv->inv[p] == p) continue;
        std::vector<uint32_t> cyc{p};
        seen[p] = true;
        for (uint32_t a = sv->inv[p]; a != p; a = sv->inv[a]) {
            cyc.push_back(a);
            seen[a] = true;
        }
        cycles.push_back(cyc);
    }
    std::vector<uint32_t> src, dst;
    auto flush = [&]() -> int {
        if (src.empty()) return LYTH_OK;
        const int r = permute_local(sv, src, dst);
        src.clear();
        dst.clear();
        return r;
    };
    st = LYTH_OK;
    for (auto &cyc : cycles) {
        while (cyc.size() > 1 && !st) {
            const size_t m = cyc.size() < (size_t)kPermuteMaxBits ? cyc.size() : (size_t)kPermuteMaxBits;
            if (src.size() + m > (size_t)kPermuteMaxBits && (st = flush())) break;
            // bits cyc[0..m) rotate: cyc[i] -> cyc[i + 1], cyc[m - 1] -> cyc[0]
            for (size_t i = 0; i < m; i++) {
                src.push_back(cyc[i]);
                dst.push_back(cyc[(i + 1) % m]);
            }
            if (m == cyc.size()) break;
            // a longer cycle: cyc[0] now holds what belongs at cyc[m], and the rest is still a
            // cycle through cyc[0], which needs a later pass
            st = flush();
            cyc.erase(cyc.begin() + 1, cyc.begin() + (long)m);
        }
        if (st) break;
    }
    if (!st) st = flush();
    if (st && st != LYTH_E_UNSUPPORTED) return st;
    // below the tile pass's size: one swap pass per transposition
    for (uint32_t q = 0; q < L; q++)
        if (sv->pos[q] != q && (st = physical_swap(sv, q, sv->pos[q]))) return st;
    return LYTH_OK;
}

// Bring the qubit on physical rank bit gp into a local bit. The victim is the local bit whose
// logical qubit is next used furthest ahead in gates[i..count) (never used: best), ties to the
// highest bit. With a swap batch > 1, other rank-bit qubits come in with it, soonest-used first,
// each while its next use precedes the next use of the victim it would displace (the next-furthest
// local bit): one exchange among 2^k ranks then replaces k single swaps. Every choice depends only
// on the map and the gate list, so every rank makes it.
int swap_in(lyth_sv *sv, uint32_t gp, const lyth_gate *gates, uint64_t count, uint64_t i) {
    int st = flush_group(sv);
    if (st) return st;
    const uint32_t L = sv->local_bits;
    // next[p] = the first gate from i on that needs physical bit p to be local: the target of a
    // gate that is not a rank-bit-free diagonal. SWAPs move the labels, not the data, so the
    // walk follows each bit's logical qubit through them; controls never need a local bit.
    std::vector<uint64_t> next(sv->qubits, UINT64_MAX);
    std::vector<uint32_t> at = sv->pos;
    uint32_t seen = 0;
    for (uint64_t j = i; j < count && seen < sv->qubits; j++) {
        const lyth_gate &h = gates[j];
        if (h.q0 >= sv->qubits || (h.kind != LYTH_GATE_U && h.q1 >= sv->qubits)) break;
        if (h.kind == LYTH_GATE_SWAP) {
            std::swap(at[h.q0], at[h.q1]);
            continue;
        }
        if (sv->diag && is_diag(u8_of(h.m))) continue;
        const uint32_t p = at[h.kind == LYTH_GATE_U ? h.q0 : h.q1];
        if (next[p] == UINT64_MAX) {
            next[p] = j;
            seen++;
        }
    }
    // local bits by next use, furthest first (ties: highest bit)
    std::vector<uint32_t> loc(L);
    for (uint32_t b = 0; b < L; b++) loc[b] = L - 1 - b;
    std::stable_sort(loc.begin(), loc.end(), [&](uint32_t x, uint32_t y) { return next[x] > next[y]; });
    // the other rank bits by next use, soonest first
    std::vector<uint32_t> glob;
    for (uint32_t b = L; b < sv->qubits; b++)
        if (b != gp) glob.push_back(b);
    std::stable_sort(glob.begin(), glob.end(), [&](uint32_t x, uint32_t y) { return next[x] < next[y]; });
    std::vector<uint32_t> V{loc[0]}, G{gp};
    for (uint32_t j = 0; j < glob.size() && (int)V.size() < sv->swap_batch && V.size() < L; j++) {
        if (next[glob[j]] < next[loc[V.size()]]) {
            V.push_back(loc[V.size()]);
            G.push_back(glob[j]);
        } else {
            break;
        }
    }
    if (V.size() == 1) return physical_swap(sv, V[0], gp);
    return physical_swap_multi(sv, V, G);
}

int apply_one(lyth_sv *sv, const lyth_gate *gates, uint64_t count, uint64_t i) {
    const lyth_gate &g = gates[i];
    const uint32_t L = sv->local_bits;
    if (g.q0 >= sv->qubits || (g.kind != LYTH_GATE_U && (g.q1 >= sv->qubits || g.q1 == g.q0))) return LYTH_E_INVALID;
    const U8 m = u8_of(g.m);
    switch (g.kind) {
        case LYTH_GATE_SWAP: {
            const uint32_t pa = sv->pos[g.q0], pb = sv->pos[g.q1];
            sv->pos[g.q0] = pb; sv->pos[g.q1] = pa;
            sv->inv[pa] = g.q1; sv->inv[pb] = g.q0;
            return LYTH_OK;
        }
        case LYTH_GATE_U: {
            uint32_t p = sv->pos[g.q0];
            if (p >= L && sv->diag && is_diag(m)) {  // this shard's row: a scalar, no exchange
                const U8 s = scalar_row(m, rank_bit(sv, p - L));
                return is_one(s) ? LYTH_OK : add_local(sv, -1, carrier(sv, -1), s);
            }
            if (p >= L && sv->remap) {
                int st = swap_in(sv, p, gates, count, i);
                if (st) return st;
                p = sv->pos[g.q0];
            }
            if (p < L) return add_local(sv, -1, p, m);
            int st = flush_group(sv);
            if (st) return st;
            return exchange_gate(sv, p - L, m, -1);
        }
        case LYTH_GATE_CU: {
            const bool diag = sv->diag && is_diag(m);
            if (sv->pos[g.q1] >= L && sv->remap && !diag) {
                int st = swap_in(sv, sv->pos[g.q1], gates, count, i);
                if (st) return st;
            }
            const uint32_t pc = sv->pos[g.q0], pt = sv->pos[g.q1];
            if (pc < L && pt < L) return add_local(sv, (int)pc, pt, m);
            if (pc >= L && !rank_bit(sv, pc - L)) return LYTH_OK;  // control 0 on this whole shard
            if (pt < L) return add_local(sv, -1, pt, m);
            if (diag) {  // diagonal on a rank-bit target: this shard's row is a scalar
                const U8 s = scalar_row(m, rank_bit(sv, pt - L));
                if (is_one(s)) return LYTH_OK;
                if (pc >= L) return add_local(sv, -1, carrier(sv, -1), s);  // control 1 here
                return add_local(sv, (int)pc, carrier(sv, (int)pc), s);      // under the local control
            }
            int st = flush_group(sv);
            if (st) return st;
            return exchange_gate(sv, pt - L, m, pc < L ? (int)pc : -1);
        }
        default:
            return LYTH_E_INVALID;
    }
}

// IPC transport set-up (collective over the handle's ranks): all-gather every rank's handles and
// map every rank's send chunks and flag block through CUDA IPC (the shards wait for open_shards).
// Every rank ends with the same `ce` (false: NCCL for swaps).

void close_ipc(lyth_sv *sv) {
    for (void *p : sv->ipc_opened) cudaIpcCloseMemHandle(p);
    sv->ipc_opened.clear();
    for (int b = 0; b < 2; b++) { sv->peer_sre[b].clear(); sv->peer_sim[b].clear(); }
    sv->peer_flags.clear();
    sv->peer_re.clear();
    sv->peer_im.clear();
    sv->ipc_all.clear();
    sv->ce = false;
    sv->peer_mode = kPeerNone;
}

int setup_ce(lyth_sv *sv) {
    const int n = sv->nranks;
    IpcRec mine{};
    mine.ok = 1;
    if (cudaMalloc(&sv->flags, kFlagWords * sizeof(uint64_t)) != cudaSuccess) {
        sv->flags = nullptr;
        mine.ok = 0;
    } else if (cudaMemset(sv->flags, 0, kFlagWords * sizeof(uint64_t)) != cudaSuccess) {
        mine.ok = 0;
    }
    void *exported[7] = {sv->sre[0], sv->sre[1], sv->sim[0], sv->sim[1], sv->flags, sv->re, sv->im};
    for (int i = 0; i < 7 && mine.ok; i++)
        if (cudaIpcGetMemHandle(&mine.h[i], exported[i]) != cudaSuccess) mine.ok = 0;
    if (n > kFlagRanks) mine.ok = 0;
    cudaGetLastError();
    IpcRec *d = nullptr;
    if (cudaMalloc(&d, sizeof(IpcRec) * (n + 1)) != cudaSuccess) {
        cudaGetLastError();
        return LYTH_E_OOM;
    }
    int st = status_of(cudaMemcpy(d + n, &mine, sizeof mine, cudaMemcpyHostToDevice));
    if (!st) st = nccl_status(g_nccl.AllGather(d + n, d, sizeof(IpcRec), ncclUint8, sv->comm, sv->stream));
    if (!st) st = status_of(cudaStreamSynchronize(sv->stream));
    std::vector<IpcRec> all(n);
    if (!st) st = status_of(cudaMemcpy(all.data(), d, sizeof(IpcRec) * n, cudaMemcpyDeviceToHost));
    if (st) { cudaFree(d); return st; }
    bool every = true;
    for (int r = 0; r < n; r++) every = every && all[r].ok;
    int32_t opened = every ? 1 : 0;
    if (every) {
        for (int b = 0; b < 2; b++) { sv->peer_sre[b].assign(n, nullptr); sv->peer_sim[b].assign(n, nullptr); }
        sv->peer_flags.assign(n, nullptr);
        for (int r = 0; r < n && opened; r++) {
            if (r == sv->rank) {
                for (int b = 0; b < 2; b++) { sv->peer_sre[b][r] = sv->sre[b]; sv->peer_sim[b][r] = sv->sim[b]; }
                sv->peer_flags[r] = sv->flags;
                continue;
            }
            void *p[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
            for (int i = 0; i < 5; i++) {
                if (cudaIpcOpenMemHandle(&p[i], all[r].h[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                    cudaGetLastError();
                    opened = 0;
                    break;
                }
                sv->ipc_opened.push_back(p[i]);
            }
            if (!opened) break;
            sv->peer_sre[0][r] = (float *)p[0]; sv->peer_sre[1][r] = (float *)p[1];
            sv->peer_sim[0][r] = (float *)p[2]; sv->peer_sim[1][r] = (float *)p[3];
            sv->peer_flags[r] = (uint64_t *)p[4];
        }
    }
    // every rank must agree: the transport is used only if every rank mapped every peer
    int32_t *dok = reinterpret_cast<int32_t *>(d);
    st = status_of(cudaMemcpy(dok, &opened, sizeof opened, cudaMemcpyHostToDevice));
    if (!st) st = nccl_status(g_nccl.AllReduce(dok, dok, 1, ncclInt32, ncclMin, sv->comm, sv->stream));
    if (!st) st = status_of(cudaStreamSynchronize(sv->stream));
    int32_t agreed = 0;
    if (!st) st = status_of(cudaMemcpy(&agreed, dok, sizeof agreed, cudaMemcpyDeviceToHost));
    cudaFree(d);
    if (st) { close_ipc(sv); return st; }
    // mixed by default: copy engines for pairwise swap-ins, peer loads for batched ones (measured
    // on 4 B200s: a batched swap-in 5 % shorter with peer loads, a pairwise one 20 % longer)
    if (agreed) {
        sv->ce = true;
        sv->peer_mode = kPeerMixed;
        sv->ipc_all = all;
    } else {
        close_ipc(sv);
    }
    return LYTH_OK;
}

// Map every partner's shard for the push form (collective: lyth_sv_set_transport 4 on every rank,
// after the drain). Every rank agrees through an NCCL min, as at set-up; on a refusal nothing
// stays mapped and LYTH_E_UNSUPPORTED is returned on every rank.
int open_shards(lyth_sv *sv) {
    if (!sv->peer_re.empty()) return LYTH_OK;
    if (sv->comm_aborted) return LYTH_E_NCCL;
    const int n = sv->nranks;
    int32_t opened = (int)sv->ipc_all.size() == n ? 1 : 0;
    std::vector<void *> mapped;
    std::vector<float *> pre(n, nullptr), pim(n, nullptr);
    for (int r = 0; r < n && opened; r++) {
        if (r == sv->rank) { pre[r] = sv->re; pim[r] = sv->im; continue; }
        void *p[2] = {nullptr, nullptr};
        for (int i = 0; i < 2; i++) {
            if (cudaIpcOpenMemHandle(&p[i], sv->ipc_all[r].h[5 + i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                opened = 0;
                break;
            }
            mapped.push_back(p[i]);
        }
        if (opened) { pre[r] = (float *)p[0]; pim[r] = (float *)p[1]; }
    }
    // the norm scratch holds the vote (nothing is in flight after the drain)
    int32_t *dok = reinterpret_cast<int32_t *>(sv->scratch);
    int st = status_of(cudaMemcpy(dok, &opened, sizeof opened, cudaMemcpyHostToDevice));
    if (!st) st = nccl_status(g_nccl.AllReduce(dok, dok, 1, ncclInt32, ncclMin, sv->comm, sv->stream));
    if (!st) st = sync_stream(sv, sv->stream);
    int32_t agreed = 0;
    if (!st) st = status_of(cudaMemcpy(&agreed, dok, sizeof agreed, cudaMemcpyDeviceToHost));
    if (st || !agreed) {
        for (void *p : mapped) cudaIpcCloseMemHandle(p);
        return st ? st : LYTH_E_UNSUPPORTED;
    }
    sv->peer_re = pre;
    sv->peer_im = pim;
    sv->ipc_opened.insert(sv->ipc_opened.end(), mapped.begin(), mapped.end());
    return LYTH_OK;
}

int device_sv_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_sv_error, sizeof v) != cudaSuccess) return LYTH_E_INVALID;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_sv_error, &zero, sizeof zero);
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}

// Before a rank's buffers and flag block go: every partner has pulled the last chunk of each send
// slot (the pulled flags arrive in this rank's own block, so no peer writes to it afterwards, and
// every flag this rank wrote to a peer was awaited by that peer before its own teardown).
void teardown_ce(lyth_sv *sv) {
    if (!sv->ce) return;
    cudaStreamSynchronize(sv->stream);
    cudaStreamSynchronize(sv->comm_stream);
    cudaStreamSynchronize(sv->copy_stream);
    for (int i = 0; i < lyth_sv::kExtraQueues; i++)
        if (sv->xq[i]) cudaStreamSynchronize(sv->xq[i]);
    for (int b = 0; b < 2; b++)
        if (sv->slot_seq[b]) wait_own(sv, sv->stream, sv->slot_partners[b], kPulledAt, b, sv->slot_seq[b]);
    cudaStreamSynchronize(sv->stream);
    // After a timed-out wait a peer may still be inside its own bounded waits: outlast them.
    if (device_sv_error() != LYTH_OK) usleep(5000000);
    close_ipc(sv);
}

void free_all(lyth_sv *sv) {
    teardown_ce(sv);
    if (sv->comm && !sv->comm_aborted && g_nccl.CommDestroy) g_nccl.CommDestroy(sv->comm);
    cudaFree(sv->flags);
    cudaFree(sv->re);
    cudaFree(sv->im);
    for (int b = 0; b < 2; b++) {
        cudaFree(sv->rre[b]);
        cudaFree(sv->rim[b]);
        cudaFree(sv->sre[b]);
        cudaFree(sv->sim[b]);
        if (sv->ev_packed[b]) cudaEventDestroy(sv->ev_packed[b]);
        if (sv->ev_recv[b]) cudaEventDestroy(sv->ev_recv[b]);
        if (sv->ev_done[b]) cudaEventDestroy(sv->ev_done[b]);
    }
    cudaFree(sv->scratch);
    for (auto &mk : sv->marks) { cudaEventDestroy(mk.a); cudaEventDestroy(mk.b); }
    for (auto e : sv->pool) cudaEventDestroy(e);
    if (sv->ev_start) cudaEventDestroy(sv->ev_start);
    if (sv->ev_pull) cudaEventDestroy(sv->ev_pull);
    if (sv->ev_copied) cudaEventDestroy(sv->ev_copied);
    if (sv->stream) cudaStreamDestroy(sv->stream);
    if (sv->comm_stream) cudaStreamDestroy(sv->comm_stream);
    if (sv->copy_stream) cudaStreamDestroy(sv->copy_stream);
    for (int i = 0; i < lyth_sv::kExtraQueues; i++) {
        if (sv->xq[i]) cudaStreamDestroy(sv->xq[i]);
        if (sv->ev_xq[i]) cudaEventDestroy(sv->ev_xq[i]);
    }
}

}  // namespace

extern "C" {

int lyth_sv_unique_id(unsigned char id[LYTH_SV_ID_BYTES]) {
    if (!id) return LYTH_E_INVALID;
    if (!load_nccl()) return LYTH_E_NO_NCCL;
    ncclUniqueId u;
    int st = nccl_status(g_nccl.GetUniqueId(&u));
    if (st) return st;
    memcpy(id, u.internal, LYTH_SV_ID_BYTES);
    return LYTH_OK;
}

int lyth_sv_create(lyth_sv **out, uint32_t qubits, int device, int rank, int nranks, const unsigned char *id) {
    if (!out) return LYTH_E_INVALID;
    *out = nullptr;
    if (nranks < 1 || (nranks & (nranks - 1)) || rank < 0 || rank >= nranks) return LYTH_E_INVALID;
    uint32_t g = 0;
    while ((1 << g) < nranks) g++;
    if (qubits < g + 2 || qubits > 40) return LYTH_E_INVALID;
    if (nranks > 1 && !id) return LYTH_E_INVALID;
    if (nranks > 1 && !load_nccl()) return LYTH_E_NO_NCCL;
    DeviceGuard guard(device);
    lyth_sv *sv = new lyth_sv();
    sv->qubits = qubits;
    sv->global_bits = g;
    sv->local_bits = qubits - g;
    sv->device = device;
    sv->rank = rank;
    sv->nranks = nranks;
    sv->local_len = 1ull << sv->local_bits;
    sv->chunk = sv->local_len < kChunk ? sv->local_len : kChunk;
    reset_map(sv);
    int st = LYTH_OK;
    auto fail = [&](int code) {
        free_all(sv);
        delete sv;
        return code;
    };
    if (cudaMalloc(&sv->re, sv->local_len * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&sv->im, sv->local_len * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&sv->scratch, (kInitBlocks + 2) * sizeof(double)) != cudaSuccess) {
        cudaGetLastError();
        return fail(LYTH_E_OOM);
    }
    if (nranks > 1) {
        for (int b = 0; b < 2; b++) {
            if (cudaMalloc(&sv->rre[b], sv->chunk * sizeof(float)) != cudaSuccess ||
                cudaMalloc(&sv->rim[b], sv->chunk * sizeof(float)) != cudaSuccess ||
                cudaMalloc(&sv->sre[b], sv->chunk * sizeof(float)) != cudaSuccess ||
                cudaMalloc(&sv->sim[b], sv->chunk * sizeof(float)) != cudaSuccess) {
                cudaGetLastError();
                return fail(LYTH_E_OOM);
            }
        }
    }
    if ((st = status_of(cudaStreamCreateWithFlags(&sv->stream, cudaStreamNonBlocking)))) return fail(st);
    // The communication stream runs NCCL's kernels beside the pack / unpack of the next chunk;
    // at the highest priority their blocks are placed first as SM slots come free.
    int prio_lo = 0, prio_hi = 0;
    cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi);
    if ((st = status_of(cudaStreamCreateWithPriority(&sv->comm_stream, cudaStreamNonBlocking, prio_hi)))) return fail(st);
    if ((st = status_of(cudaStreamCreateWithPriority(&sv->copy_stream, cudaStreamNonBlocking, prio_hi)))) return fail(st);
    if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_pull, cudaEventDisableTiming)))) return fail(st);
    if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_copied, cudaEventDisableTiming)))) return fail(st);
    for (int i = 0; i < lyth_sv::kExtraQueues; i++) {
        if ((st = status_of(cudaStreamCreateWithPriority(&sv->xq[i], cudaStreamNonBlocking, prio_hi)))) return fail(st);
        if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_xq[i], cudaEventDisableTiming)))) return fail(st);
    }
    for (int b = 0; b < 2; b++) {
        if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_recv[b], cudaEventDisableTiming)))) return fail(st);
        if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_done[b], cudaEventDisableTiming)))) return fail(st);
        if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_packed[b], cudaEventDisableTiming)))) return fail(st);
    }
    if ((st = status_of(cudaEventCreateWithFlags(&sv->ev_start, cudaEventDisableTiming)))) return fail(st);
    if (nranks > 1) {
        ncclUniqueId u;
        memcpy(u.internal, id, LYTH_SV_ID_BYTES);
        if (g_nccl.CommInitRank(&sv->comm, nranks, u, rank) != ncclSuccess) {
            sv->comm = nullptr;
            return fail(LYTH_E_NCCL);
        }
        if ((st = setup_ce(sv))) return fail(st);
    }
    *out = sv;
    return LYTH_OK;
}

int lyth_sv_destroy(lyth_sv *sv) {
    if (!sv) return LYTH_OK;
    if (sv->plan) {
        delete sv;
        return LYTH_OK;
    }
    DeviceGuard guard(sv);
    sync_stream(sv, sv->stream);
    sync_stream(sv, sv->comm_stream);
    free_all(sv);
    delete sv;
    return LYTH_OK;
}

uint64_t lyth_sv_local_len(const lyth_sv *sv) { return sv ? sv->local_len : 0; }
cudaStream_t lyth_sv_stream(const lyth_sv *sv) { return sv ? sv->stream : nullptr; }

int lyth_sv_init_basis(lyth_sv *sv, uint64_t index) {
    if (!sv) return LYTH_E_INVALID;
    if (index >> sv->qubits) return LYTH_E_INVALID;
    DeviceGuard guard(sv);
    reset_map(sv);
    if (sv->plan) return LYTH_OK;
    int st;
    if ((st = status_of(cudaMemsetAsync(sv->re, 0, sv->local_len * 4, sv->stream)))) return st;
    if ((st = status_of(cudaMemsetAsync(sv->im, 0, sv->local_len * 4, sv->stream)))) return st;
    if ((index >> sv->local_bits) == (uint64_t)sv->rank) {
        set_one_kernel<<<1, 1, 0, sv->stream>>>(sv->re, sv->im, index & (sv->local_len - 1));
        return last_launch_status();
    }
    return LYTH_OK;
}

int lyth_sv_init_random(lyth_sv *sv, uint64_t seed) {
    if (!sv) return LYTH_E_INVALID;
    DeviceGuard guard(sv);
    reset_map(sv);
    if (sv->plan) return LYTH_OK;
    const uint64_t base = (uint64_t)sv->rank * sv->local_len;
    init_random_kernel<<<kInitBlocks, 256, 0, sv->stream>>>(sv->local_len, base, seed, sv->re, sv->im, sv->scratch);
    int st = last_launch_status();
    if (st) return st;
    double *norm2 = sv->scratch + kInitBlocks;
    sum_partials_kernel<<<1, 32, 0, sv->stream>>>(sv->scratch, kInitBlocks, norm2);
    if ((st = last_launch_status())) return st;
    if (sv->nranks > 1) {
        if ((st = nccl_status(g_nccl.AllReduce(norm2, norm2, 1, ncclFloat64, ncclSum, sv->comm, sv->stream)))) return st;
    }
    scale_kernel<<<stream_grid(sv->local_len, 256), 256, 0, sv->stream>>>(sv->local_len, norm2, sv->re, sv->im);
    return last_launch_status();
}

int lyth_sv_set_local(lyth_sv *sv, const float *re, const float *im) {
    if (!sv) return LYTH_E_INVALID;
    if (sv->plan) {
        reset_map(sv);
        return LYTH_OK;
    }
    if (!re || !im) return LYTH_E_INVALID;
    DeviceGuard guard(sv);
    reset_map(sv);
    int st;
    if ((st = status_of(cudaMemcpyAsync(sv->re, re, sv->local_len * 4, cudaMemcpyDefault, sv->stream)))) return st;
    if ((st = status_of(cudaMemcpyAsync(sv->im, im, sv->local_len * 4, cudaMemcpyDefault, sv->stream)))) return st;
    return status_of(cudaStreamSynchronize(sv->stream));
}

int lyth_sv_get_local(lyth_sv *sv, float *re, float *im) {
    if (!sv) return LYTH_E_INVALID;
    if (sv->plan) return normalize(sv);
    if (!re || !im) return LYTH_E_INVALID;
    if (sv->comm_aborted) return LYTH_E_NCCL;
    DeviceGuard guard(sv);
    int st = normalize(sv);
    if (st) return st;
    if ((st = status_of(cudaMemcpyAsync(re, sv->re, sv->local_len * 4, cudaMemcpyDefault, sv->stream)))) return st;
    if ((st = status_of(cudaMemcpyAsync(im, sv->im, sv->local_len * 4, cudaMemcpyDefault, sv->stream)))) return st;
    return status_of(cudaStreamSynchronize(sv->stream));
}

int lyth_sv_apply(lyth_sv *sv, const lyth_gate *gates, uint64_t count) {
    if (!sv || (count && !gates)) return LYTH_E_INVALID;
    if (sv->comm_aborted) return LYTH_E_NCCL;
    DeviceGuard guard(sv);
    for (uint64_t i = 0; i < count; i++) {
        int st = apply_one(sv, gates, count, i);
        if (st) {
            sv->open.k = 0;
            sv->open.ngates = 0;
            return st;
        }
    }
    return flush_group(sv);
}

int lyth_sv_set_transport(lyth_sv *sv, int kind) {
    if (!sv) return LYTH_E_INVALID;
    if (kind < 0 || kind > 4) return LYTH_E_INVALID;
    if (kind && sv->peer_flags.empty()) return LYTH_E_UNSUPPORTED;
    if (!sv->plan) {
        DeviceGuard guard(sv);
        // drain the current transport before switching: partners must have pulled every chunk,
        // and this rank's own pulls on the copy stream must have landed
        int st = drain_all(sv);
        if (st) return st;
        if (sv->ce && !kind)
            for (int b = 0; b < 2; b++)
                if (sv->slot_seq[b]) wait_own(sv, sv->stream, sv->slot_partners[b], kPulledAt, b, sv->slot_seq[b]);
        if ((st = status_of(cudaStreamSynchronize(sv->stream)))) return st;
        if (kind == 4 && (st = open_shards(sv))) return st;
    }
    sv->ce = kind != 0;
    sv->peer_mode = kind == 2 ? kPeerLoad : kind == 3 ? kPeerMixed : kind == 4 ? kPeerStore : kPeerNone;
    return LYTH_OK;
}

int lyth_sv_transport(const lyth_sv *sv) { return sv && sv->ce ? 1 + sv->peer_mode : 0; }

int lyth_sv_set_chunk(lyth_sv *sv, uint64_t elements) {
    if (!sv) return LYTH_E_INVALID;
    const uint64_t cap = sv->local_len < kChunk ? sv->local_len : kChunk;
    if (elements < 1024 || (elements & (elements - 1)) || elements > cap) return LYTH_E_UNSUPPORTED;
    if (!sv->plan) {
        DeviceGuard guard(sv);
        const int st = drain_all(sv);
        if (st) return st;
    }
    sv->chunk = elements;
    return LYTH_OK;
}

int lyth_sv_set_swap_batch(lyth_sv *sv, int max_qubits) {
    if (!sv) return LYTH_E_INVALID;
    if (max_qubits < 1 || max_qubits > 6) return LYTH_E_UNSUPPORTED;
    sv->swap_batch = max_qubits;
    return LYTH_OK;
}

int lyth_sv_set_remap(lyth_sv *sv, int on) {
    if (!sv) return LYTH_E_INVALID;
    sv->remap = on != 0;
    return LYTH_OK;
}

int lyth_sv_set_diagonal(lyth_sv *sv, int on) {
    if (!sv) return LYTH_E_INVALID;
    sv->diag = on != 0;
    return LYTH_OK;
}

int lyth_sv_set_fusion(lyth_sv *sv, int max_qubits) {
    if (!sv) return LYTH_E_INVALID;
    if (max_qubits < 1 || max_qubits > kFuseMaxQubits) return LYTH_E_UNSUPPORTED;
    sv->fuse_k = max_qubits;
    return LYTH_OK;
}

int lyth_sv_sync(lyth_sv *sv) {
    if (!sv) return LYTH_E_INVALID;
    if (sv->plan) return LYTH_OK;
    DeviceGuard guard(sv);
    if (sv->comm_aborted) return LYTH_E_NCCL;
    int st = drain_all(sv);
    if (st) return st;
    if ((st = fused_take_device_error())) return st;  // a tile pass that gave up a bounded wait
    return sv->ce ? device_sv_error() : LYTH_OK;       // a transport flag wait that did
}

uint64_t lyth_sv_launches(const lyth_sv *sv) { return sv ? sv->launches : 0; }

int lyth_sv_set_timing(lyth_sv *sv, int on) {
    if (!sv) return LYTH_E_INVALID;
    sv->timing = on != 0;
    return LYTH_OK;
}

int lyth_sv_timing(lyth_sv *sv, int cls, uint64_t *count, double *ms) {
    if (!sv || cls < 0 || cls > LYTH_SV_T_SWAP) return LYTH_E_INVALID;
    DeviceGuard guard(sv);
    int st = fold_timing(sv);
    if (st) return st;
    if (count) *count = sv->t_count[cls];
    if (ms) *ms = sv->t_ms[cls];
    return LYTH_OK;
}

int lyth_sv_reset_timing(lyth_sv *sv) {
    if (!sv) return LYTH_E_INVALID;
    DeviceGuard guard(sv);
    int st = fold_timing(sv);
    for (int c = 0; c <= LYTH_SV_T_SWAP; c++) { sv->t_count[c] = 0; sv->t_ms[c] = 0.0; }
    return st;
}

int lyth_sv_stats(const lyth_sv *sv, uint64_t *passes, uint64_t *exchanges, uint64_t *bytes_sent) {
    if (!sv) return LYTH_E_INVALID;
    if (passes) *passes = sv->passes;
    if (exchanges) *exchanges = sv->exchanges;
    if (bytes_sent) *bytes_sent = sv->bytes_sent;
    return LYTH_OK;
}

int lyth_sv_plan_create(lyth_sv **out, uint32_t qubits, int rank, int nranks) {
    if (!out) return LYTH_E_INVALID;
    *out = nullptr;
    if (nranks < 1 || (nranks & (nranks - 1)) || rank < 0 || rank >= nranks) return LYTH_E_INVALID;
    uint32_t g = 0;
    while ((1 << g) < nranks) g++;
    if (qubits < g + 2 || qubits > 40) return LYTH_E_INVALID;
    lyth_sv *sv = new lyth_sv();
    sv->plan = true;
    sv->qubits = qubits;
    sv->global_bits = g;
    sv->local_bits = qubits - g;
    sv->device = -1;
    sv->rank = rank;
    sv->nranks = nranks;
    sv->local_len = 1ull << sv->local_bits;
    sv->chunk = sv->local_len < kChunk ? sv->local_len : kChunk;
    reset_map(sv);
    *out = sv;
    return LYTH_OK;
}

uint64_t lyth_sv_plan_count(const lyth_sv *sv) { return sv ? (uint64_t)sv->ops.size() : 0; }

int lyth_sv_plan_op(const lyth_sv *sv, uint64_t index, lyth_sv_op *out) {
    if (!sv || !out || !sv->plan || index >= sv->ops.size()) return LYTH_E_INVALID;
    *out = sv->ops[index];
    return LYTH_OK;
}

int lyth_sv_plan_clear(lyth_sv *sv) {
    if (!sv || !sv->plan) return LYTH_E_INVALID;
    sv->ops.clear();
    return LYTH_OK;
}

}  // extern "C"

int lyth_sv_set_pull_queues(lyth_sv *sv, int queues) {
    if (!sv) return LYTH_E_INVALID;
    if (queues < 0 || queues > 2 + lyth_sv::kExtraQueues) return LYTH_E_UNSUPPORTED;
    if (!sv->plan) {
        DeviceGuard guard(sv);
        const int st = drain_all(sv);
        if (st) return st;
    }
    sv->pull_queues = queues;
    return LYTH_OK;
}

int lyth_sv_set_deadline(lyth_sv *sv, double ms) {
    if (!sv) return LYTH_E_INVALID;
    if (!(ms >= 1.0)) return LYTH_E_UNSUPPORTED;
    sv->deadline_ms = ms;
    return LYTH_OK;
}

// Host-only check of wait_with_deadline with fake hooks (no device, no NCCL): scenario 0 = the
// work completes after 3 polls; 1 = the communicator reports an async error at the 2nd poll;
// 2 = the work never completes (the deadline passes); 3 = the stream reports a CUDA error.
extern "C" int lyth_sv_deadline_selftest(int scenario, double deadline_ms, int *aborts, uint64_t *polls) {
    struct Fake {
        int scenario, n, aborts;
    } f{scenario, 0, 0};
    WaitHooks h;
    h.ctx = &f;
    h.query = [](void *p) {
        Fake *x = static_cast<Fake *>(p);
        x->n++;
        if (x->scenario == 0) return x->n >= 3 ? 0 : 1;
        if (x->scenario == 3) return x->n >= 2 ? (int)cudaErrorLaunchFailure : 1;
        return 1;
    };
    h.async_error = [](void *p) {
        Fake *x = static_cast<Fake *>(p);
        return (x->scenario == 1 && x->n >= 2) ? 1 : 0;
    };
    h.abort = [](void *p) { static_cast<Fake *>(p)->aborts++; };
    const int st = wait_with_deadline(h, deadline_ms, 100, polls);
    if (aborts) *aborts = f.aborts;
    return st;
}
