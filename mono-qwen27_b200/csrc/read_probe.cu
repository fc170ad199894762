// read_probe.cu — m27b_hbm_read_probe: a plain stream of a buffer into
// shared memory with bulk asynchronous copies (the copy engine the matvec
// kernels use), nothing computed: the time of one launch is the read
// ceiling a weight-streaming launch of that size can reach on this GPU, launch,
// ramp-up and drain included.  The copy shape (issuing warps per CTA, copies
// in flight per warp, bytes per copy, CTAs per SM) is a parameter, so that a
// benchmark can take the fastest of several shapes as the ceiling.
// Measurement support for the benchmark's roofline; no counterpart in the
// reference.
#include <cuda_runtime.h>

#include <cstdio>

#include "m27b_launch.cuh"
#include "m27b_qmv.h"
#include "qmv_blk.cuh"

namespace m27b {

constexpr int RP_MAX_WARPS = 16;
constexpr int RP_MAX_STAGES = 8;
constexpr int RP_MAX_CHUNK = 65536;

// Lane 0 of every warp issues (the other lanes leave).  The buffer is split
// into one contiguous, 16-byte aligned share per warp of the grid; a warp
// streams its share in `chunk`-byte copies, copy c into stage c % stages
// once the copy that used the stage before has landed.  Every wait is
// bounded (status 6 on timeout); the copies still in flight are waited for
// (bounded) before the warp exits.  Launched like the matvec kernels (with
// programmatic dependent launch): the next launch may start its copies as
// soon as every CTA of this one has started, and a launch finishes only
// after its predecessor (griddepcontrol.wait before the exit), so a chain of
// probes keeps the ordering a chain of matvecs has.
__global__ void __launch_bounds__(RP_MAX_WARPS * 32) k_read_probe(const uint8_t *p, size_t bytes, int chunk, int stages,
                                                                  int *status) {
    extern __shared__ __align__(128) uint8_t rp_smem[];
    pdl_trigger();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) != 0) return;
    uint8_t *stage0 = rp_smem + (size_t)warp * stages * chunk;
    uint64_t *bar = (uint64_t *)(rp_smem + (size_t)nw * stages * chunk) + warp * RP_MAX_STAGES;
    const size_t tw = (size_t)gridDim.x * nw, gw = (size_t)blockIdx.x * nw + warp;
    const size_t per = ((bytes + tw - 1) / tw + 15) & ~(size_t)15;
    const size_t lo = gw * per;
    const size_t hi = lo + per < bytes ? lo + per : bytes;
    if (lo >= hi) {
        pdl_wait();
        return;
    }
    for (int s = 0; s < stages; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
    const int n = (int)((hi - lo + chunk - 1) / chunk);
    int issued = 0;
    for (; issued < n; ++issued) {
        const int s = issued % stages;
        if (issued >= stages && !mbar_wait_bounded(&bar[s], (uint32_t)(((issued / stages) - 1) & 1), status, 6)) break;
        const size_t off = lo + (size_t)issued * chunk;
        const uint32_t sz = (uint32_t)(hi - off < (size_t)chunk ? hi - off : (size_t)chunk);
        mbar_arrive_expect_tx(&bar[s], sz);
        bulk_copy_g2s(stage0 + (size_t)s * chunk, p + off, sz, &bar[s]);
    }
    // every copy issued and not yet waited for lands before the warp exits
    // (after a timeout too: the failed wait's copy is among them)
    for (int c = issued > stages ? issued - stages : 0; c < issued; ++c)
        mbar_wait_bounded(&bar[c % stages], (uint32_t)((c / stages) & 1), status, 6);
    pdl_wait();
}

}  // namespace m27b

extern "C" {

bool m27b_hbm_read_probe_shape(const void *p, size_t bytes, int warps, int stages, int chunk, int ctas_per_sm,
                               cudaStream_t stream, char *err, size_t err_cap) {
    auto fail = [&](const char *m) {
        if (err && err_cap) std::snprintf(err, err_cap, "m27b_hbm_read_probe: %s", m);
        return false;
    };
    if (!p || bytes < 16 || (bytes & 15) || ((uintptr_t)p & 15)) return fail("needs a 16-byte aligned buffer of 16k bytes");
    if (warps < 1 || warps > m27b::RP_MAX_WARPS || stages < 1 || stages > m27b::RP_MAX_STAGES || chunk < 16 ||
        chunk > m27b::RP_MAX_CHUNK || (chunk & 15) || ctas_per_sm < 1 || ctas_per_sm > 8)
        return fail("shape out of range (warps 1-16, stages 1-8, chunk 16-65536 bytes in steps of 16, 1-8 CTAs per SM)");
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return fail("no CUDA device");
    int *status = m27b::status_ptr_current();
    if (!status) return fail("cannot resolve the device status word");
    const size_t smem = (size_t)warps * stages * chunk + (size_t)warps * m27b::RP_MAX_STAGES * 8;
    static size_t opted[64] = {};
    if (smem > 48 * 1024 && (dev >= 64 || smem > opted[dev])) {
        if (cudaFuncSetAttribute(m27b::k_read_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess) {
            (void)cudaGetLastError();  // the refusal is reported here, not by a later launch check
            return fail("shared-memory opt-in failed (too many bytes in flight per CTA)");
        }
        if (dev < 64) opted[dev] = smem;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, m27b::k_read_probe, warps * 32, smem) != cudaSuccess) {
        (void)cudaGetLastError();
        return fail("occupancy query failed");
    }
    if (occ < ctas_per_sm) return fail("that many CTAs of this shape do not fit on one SM");
    const cudaError_t e = m27b::launch_pdl(m27b::k_read_probe, dim3(sms * ctas_per_sm), dim3(warps * 32), smem, stream,
                                           (const uint8_t *)p, bytes, chunk, stages, status);
    if (e != cudaSuccess) return fail(cudaGetErrorString(e));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_hbm_read_probe(const void *p, size_t bytes, cudaStream_t stream, char *err, size_t err_cap) {
    return m27b_hbm_read_probe_shape(p, bytes, 1, 6, 32768, 1, stream, err, err_cap);
}

}  // extern "C"
