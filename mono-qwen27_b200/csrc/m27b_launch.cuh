// m27b_launch.cuh — host-side launchers shared between the kernel files and
// the C ABI (capi.cu).  Internal to libm27b.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace m27b {

// Launch with programmatic stream serialization (see pdl_wait / pdl_trigger).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

enum ActMode { ACT_PLAIN = 0, ACT_GATED = 1, ACT_RMSNORM = 2, ACT_RMSNORM_SUM = 3, ACT_SWIGLU = 4 };

struct ActArgs {
    const float *x;
    const float *gate;  // ACT_GATED, ACT_SWIGLU (the gate projection)
    const float *w;     // ACT_RMSNORM / ACT_RMSNORM_SUM (may be null: weight 1.0)
    float eps;
    int k;
    int ldx;
    void *out;
    // ACT_RMSNORM_SUM (q8_K, one token): the consumer half of a fused
    // all-reduce.  x is the sum, in ascending s, of the epoch-tagged words
    // words[s * src_stride + i] that the nsrc ranks stored; it is also written
    // to x_out, then normalised and quantized.  ss_words ([k / 256]) carries
    // the per-CTA sums of squares between the CTAs.
    const uint2 *words;
    int nsrc;
    int src_stride;
    uint2 *ss_words;
    const unsigned *epoch_base;  // epoch = *epoch_base * epoch_mul + epoch_add
    unsigned epoch_mul, epoch_add;
    float *x_out;
    int *status;
    unsigned long long wait_ns;  // bound on each word wait (0: M27B_WAIT_NS)
};

cudaError_t launch_act_quant(int act_type, int mode, const ActArgs &a, int n_tok, cudaStream_t st);

// Device address of the library status word on the current device (cached).
int *status_ptr_current();
size_t planar_row_bytes(int type, int rb);
cudaError_t launch_repack(int type, const void *raw, int rb, int rows, void *out, cudaStream_t st);
cudaError_t launch_dequant_rows(int type, bool planar, const void *w, size_t row_stride, int rb, int row_count, int k,
                                const int32_t *rows, int n, float *out, int ldo, cudaStream_t st);

}  // namespace m27b
