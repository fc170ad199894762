// read_probe.cu — m27b_hbm_read_probe: a plain stream of a buffer into
// shared memory with bulk asynchronous copies (the copy engine the matvec
// kernels use), nothing computed: the time of one launch is the read ceiling
// a weight-streaming launch of that size can reach on this GPU, launch,
// ramp-up and drain included.  Measurement support for the benchmark's
// roofline; no counterpart in the reference.
#include <cuda_runtime.h>

#include <cstdio>

#include "m27b_launch.cuh"
#include "m27b_qmv.h"
#include "qmv_blk.cuh"

namespace m27b {

constexpr int RP_CHUNK = 32768;  // bytes per bulk copy
constexpr int RP_STAGES = 6;     // copies in flight per CTA (192 KB)

// One CTA (one thread issues, the others leave) per SM: chunk c of the CTA's
// share goes into stage c % RP_STAGES once the copy that used the stage
// before has landed.  Every wait is bounded (status 6 on timeout); the copies
// still in flight are waited for (bounded) before the CTA exits.
__global__ void __launch_bounds__(32) k_read_probe(const uint8_t *p, size_t bytes, int *status) {
    extern __shared__ __align__(128) uint8_t rp_smem[];
    uint64_t *bar = (uint64_t *)(rp_smem + (size_t)RP_STAGES * RP_CHUNK);
    if (threadIdx.x != 0) return;
    const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t lo = (size_t)blockIdx.x * per;
    const size_t hi = lo + per < bytes ? lo + per : bytes;
    if (lo >= hi) return;
    for (int s = 0; s < RP_STAGES; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
    const int n = (int)((hi - lo + RP_CHUNK - 1) / RP_CHUNK);
    int issued = 0;
    bool ok = true;
    for (; issued < n; ++issued) {
        const int s = issued % RP_STAGES;
        if (issued >= RP_STAGES && !mbar_wait_bounded(&bar[s], (uint32_t)(((issued / RP_STAGES) - 1) & 1), status, 6)) {
            ok = false;
            break;
        }
        const size_t off = lo + (size_t)issued * RP_CHUNK;
        const uint32_t sz = (uint32_t)(hi - off < (size_t)RP_CHUNK ? hi - off : (size_t)RP_CHUNK);
        mbar_arrive_expect_tx(&bar[s], sz);
        bulk_copy_g2s(rp_smem + (size_t)s * RP_CHUNK, p + off, sz, &bar[s]);
    }
    // every copy issued and not yet waited for lands before the CTA exits
    (void)ok;  // after a timeout the same drain applies (the failed wait's copy included)
    for (int c = issued > RP_STAGES ? issued - RP_STAGES : 0; c < issued; ++c)
        mbar_wait_bounded(&bar[c % RP_STAGES], (uint32_t)((c / RP_STAGES) & 1), status, 6);
}

}  // namespace m27b

extern "C" {

bool m27b_hbm_read_probe(const void *p, size_t bytes, cudaStream_t stream, char *err, size_t err_cap) {
    auto fail = [&](const char *m) {
        if (err && err_cap) std::snprintf(err, err_cap, "m27b_hbm_read_probe: %s", m);
        return false;
    };
    if (!p || bytes < 16 || (bytes & 15) || ((uintptr_t)p & 15)) return fail("needs a 16-byte aligned buffer of 16k bytes");
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return fail("no CUDA device");
    int *status = m27b::status_ptr_current();
    if (!status) return fail("cannot resolve the device status word");
    const size_t smem = (size_t)m27b::RP_STAGES * m27b::RP_CHUNK + m27b::RP_STAGES * 8;
    static bool opted[64] = {};
    if (dev >= 64 || !opted[dev]) {
        if (cudaFuncSetAttribute(m27b::k_read_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return fail("shared-memory opt-in failed");
        if (dev < 64) opted[dev] = true;
    }
    m27b::k_read_probe<<<sms, 32, smem, stream>>>((const uint8_t *)p, bytes, status);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(cudaGetErrorString(e));
    if (err && err_cap) err[0] = '\0';
    return true;
}

}  // extern "C"
