// read_probe.cu — m27b_hbm_read_probe: a plain streaming read of a buffer, the
// measured ceiling a weight-streaming launch of the same size can reach on
// this GPU (launch, ramp-up and drain included).  Measurement support for the
// benchmark's roofline; no counterpart in the reference.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "m27b_device.cuh"
#include "m27b_qmv.h"

namespace m27b {

// grid-stride 16-byte streaming loads, four in flight per thread; the xor of
// everything read goes to sink[blockIdx.x] so nothing is optimised away
__global__ void __launch_bounds__(512) k_read_probe(const uint4 *p, size_t n16, unsigned *sink) {
    unsigned acc = 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        const uint4 a = ldg_stream16(p + i), b = ldg_stream16(p + i + stride);
        const uint4 c = ldg_stream16(p + i + 2 * stride), d = ldg_stream16(p + i + 3 * stride);
        acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n16; i += stride) {
        const uint4 a = ldg_stream16(p + i);
        acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicXor(sink + blockIdx.x, acc);
}

}  // namespace m27b

extern "C" {

bool m27b_hbm_read_probe(const void *p, size_t bytes, unsigned *sink, int ctas_per_sm, cudaStream_t stream, char *err,
                         size_t err_cap) {
    auto fail = [&](const char *m) {
        if (err && err_cap) std::snprintf(err, err_cap, "m27b_hbm_read_probe: %s", m);
        return false;
    };
    if (!p || !sink || bytes < 16 || (bytes & 15) || ((uintptr_t)p & 15)) return fail("16-byte aligned buffer of 16k bytes");
    if (ctas_per_sm < 1 || ctas_per_sm > 4) return fail("ctas_per_sm must be 1..4");
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return fail("no CUDA device");
    m27b::k_read_probe<<<sms * ctas_per_sm, 512, 0, stream>>>((const uint4 *)p, bytes / 16, sink);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(cudaGetErrorString(e));
    if (err && err_cap) err[0] = '\0';
    return true;
}

}  // extern "C"
