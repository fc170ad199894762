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

enum ActMode { ACT_PLAIN = 0, ACT_GATED = 1, ACT_RMSNORM = 2 };

struct ActArgs {
    const float *x;
    const float *gate;  // ACT_GATED
    const float *w;     // ACT_RMSNORM (may be null: weight 1.0)
    float eps;
    int k;
    int ldx;
    void *out;
};

cudaError_t launch_act_quant(int act_type, int mode, const ActArgs &a, int n_tok, cudaStream_t st);
size_t planar_row_bytes(int type, int rb);
cudaError_t launch_repack(int type, const void *raw, int rb, int rows, void *out, cudaStream_t st);
cudaError_t launch_dequant_rows(int type, bool planar, const void *w, size_t row_stride, int rb, int row_count, int k,
                                const int32_t *rows, int n, float *out, int ldo, cudaStream_t st);

}  // namespace m27b
