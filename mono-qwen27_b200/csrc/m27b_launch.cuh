// m27b_launch.cuh — host-side launchers shared between the kernel files and
// the C ABI (capi.cu).  Internal to libm27b.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace m27b {

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
