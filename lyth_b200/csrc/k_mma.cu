// bf16 contraction on the tcgen05 tensor cores (examples/matmul.lyth with bf16 storage).
// Entry point only; the kernel lands in a following change.
#include "common.cuh"

extern "C" int lyth_b200_matmul_bf16(uint32_t m, uint32_t n, uint32_t k, const uint16_t *a, const uint16_t *b,
                                     float *c, cudaStream_t s) {
    (void)m; (void)n; (void)k; (void)a; (void)b; (void)c; (void)s;
    return LYTH_E_UNSUPPORTED;
}
