// ref_gpu_harness.cu — COMPARISON ARM (test and benchmark infrastructure only).
//
// Compiles the reference executor's own CUDA translation unit
// (src/mono27b_executor.cu, included in place from the reference checkout;
// nothing is copied) for sm_100a with the reference's CUDA flags
// (CMakeLists.txt:36-40: --use_fast_math, --default-stream=per-thread), and
// exposes its activation quantizer and batch-1 matvec kernels with the
// reference's launch shapes, so that they can be timed on a B200 next to this
// project's kernels:
//   k_quant_q8_1        <<<n/32, 32>>>                 (l_quant_q8_n, :2022-2030)
//   k_q4k_mv_q8_dp4a    <<<rows, (32, 4), 32*8*4 B>>>  (l_mv_q8_on, :2061-2065)
//   k_q6k_mv_q8_dp4a    <<<rows, 128>>>                (:2069-2071)
//   k_q80_mv_q8_dp4a    <<<rows, (32, 4)>>>            (:2072-2074)
// Weights are the reference's raw GGUF blocks; activations its q8_1 blocks
// (36 bytes per 32 values).  Built by oracle/build.py into oracle/_ref/.
// Never part of the product library.  Built with hidden visibility: only
// the two refgpu_* entries are exported (the reference's own extern "C"
// executor API stays inside this library).
#include "mono27b_executor.cu"

bool g_mono27b_verbose = false;
Mono27BKernelConfig g_kernel_cfg;

#define REFGPU_API __attribute__((visibility("default")))

extern "C" {

// x: n fp32 values (n a multiple of 32) -> n/32 q8_1 blocks at q8.
REFGPU_API int refgpu_quant_q8_1(const float *x, void *q8, int n, cudaStream_t st) {
    k_quant_q8_1<<<n / 32, 32, 0, st>>>(x, (BlockQ8_1 *)q8, n);
    return (int)cudaGetLastError();
}

// y[r] = W[r] . x for `rows` rows of `rb` blocks; type 12 (q4_K), 14 (q6_K)
// or 8 (q8_0); q8 from refgpu_quant_q8_1.
REFGPU_API int refgpu_matvec(int type, const void *W, const void *q8, float *y, int rb, int rows, cudaStream_t st) {
    switch (type) {
    case 12:
        k_q4k_mv_q8_dp4a<<<rows, dim3(32, g_kernel_cfg.q4k_q8_warp_count),
                           32 * (size_t)g_kernel_cfg.q4k_q8_smem_per_warp * sizeof(float), st>>>(
            (const BlockQ4K *)W, (const BlockQ8_1 *)q8, y, nullptr, rb, rows);
        break;
    case 14:
        k_q6k_mv_q8_dp4a<<<rows, 128, 0, st>>>((const BlockQ6K *)W, (const BlockQ8_1 *)q8, y, rb, rows);
        break;
    case 8:
        k_q80_mv_q8_dp4a<<<rows, dim3(32, 4), 0, st>>>((const BlockQ8 *)W, (const BlockQ8_1 *)q8, y, rb, rows);
        break;
    default:
        return -1;
    }
    return (int)cudaGetLastError();
}

}  // extern "C"
