// Bounded-wait self-test: the library's two kinds of device-side wait -- an mbarrier phase wait
// (the TMA-fed kernels: fused pass, bf16 contraction, GEMV ring) and a flag wait (the state
// vector's cross-GPU transport) -- run here on something that never completes, with a short
// limit, through the same device functions the kernels use (mbar_wait_limited,
// flag_wait_bounded). The wait gives up, sets this file's error flag and the kernel returns, so
// lyth_b200_device_error reports LYTH_E_TIMEOUT and the context stays usable. No fault, trap or
// unbounded loop is involved.
#include "common.cuh"
#include "mbar.cuh"

namespace lyth {

__device__ int g_probe_error;
__device__ uint64_t g_probe_flag;  // never raised: stays 0

__global__ void wait_probe_kernel(int which, uint64_t ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    if (which == 0) {
        mbar_init(smem_u32(&bar), 1);  // one arrival expected; none ever comes
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_wait_limited(smem_u32(&bar), 0, &g_probe_error, 0xffffffffu, ns);
    } else {
        flag_wait_bounded(&g_probe_flag, 1, ns, &g_probe_error);
    }
}

int probe_take_device_error() {
    int v = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&v, g_probe_error, sizeof(int));
    if (e != cudaSuccess) return status_of(e);
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_probe_error, &zero, sizeof(int));
        return LYTH_E_TIMEOUT;
    }
    return LYTH_OK;
}

}  // namespace lyth

using namespace lyth;

extern "C" int lyth_b200_wait_selftest(int which, uint32_t limit_us, cudaStream_t s) {
    if ((which != 0 && which != 1) || limit_us == 0 || limit_us > 2000000u) return LYTH_E_INVALID;
    wait_probe_kernel<<<1, 32, 0, s>>>(which, (uint64_t)limit_us * 1000ull);
    return last_launch_status();
}
