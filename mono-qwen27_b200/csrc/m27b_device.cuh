// m27b_device.cuh — device helpers shared by the sm_100a quantized matvec kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "m27b_blocks.h"

#define M27B_DI __device__ __forceinline__

namespace m27b {

// Streaming 128-bit load of weight bytes: read-only path, no L1 allocation
// (each weight byte is used once per call), 256-byte L2 prefetch hint so that
// the DRAM bursts stay full while the warp walks a row.
M27B_DI uint4 ldg_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

M27B_DI uint2 ldg_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

M27B_DI uint32_t ldg_stream_u16(const void *p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

M27B_DI float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu))); }

M27B_DI int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Sum of the four byte-lanes products of two uint4 (16 x int8 . int8).
M27B_DI int dot16(uint4 a, uint4 b) {
    int s = dp4a((int)a.x, (int)b.x, 0);
    s = dp4a((int)a.y, (int)b.y, s);
    s = dp4a((int)a.z, (int)b.z, s);
    return dp4a((int)a.w, (int)b.w, s);
}

M27B_DI float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Monotone map of a float to uint32 (total order on non-NaN values).
M27B_DI uint32_t float_order_key(float v) {
    uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Packed argmax key: larger value wins; on equal values the smaller index
// wins (the index is stored complemented in the low word).
M27B_DI unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}

// Programmatic dependent launch (sm_90+).  A kernel launched with the
// programmatic-stream-serialization attribute may start while the previous
// kernel in the stream is still running, once that kernel has executed
// pdl_trigger() in every CTA (or exited).  pdl_wait() blocks until the
// previous kernel has completed and its memory writes are visible: every read
// of data a previous kernel produced, and every global write, comes after it.
M27B_DI void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
M27B_DI void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- bounded waits and cross-GPU signalling ----
constexpr unsigned long long M27B_WAIT_NS = 2000000000ull;  // 2 s bound on any wait

M27B_DI unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- epoch-tagged words ----
// A value travels with its epoch in one aligned 8-byte word {bits, epoch}
// (bits in the low half), written by one relaxed system-scope 64-bit store
// and read by one relaxed system-scope 64-bit load.  Under the PTX memory
// model an aligned scalar b64 access at .sys scope is single-copy atomic and
// does not race with the writer, so a reader sees either the whole old word
// or the whole new one: a word whose epoch matches carries that epoch's
// value, with no fence or separate flag.  (A v2.b32 vector access would be two
// scalar accesses in unspecified order, and a weak one a data race.)  The
// relaxed .sys load is not served from L1, so a re-read sees a store made
// by another SM or another GPU.
M27B_DI void st_word(uint2 *p, uint32_t bits, uint32_t ep) {
    const unsigned long long w = (unsigned long long)bits | ((unsigned long long)ep << 32);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
M27B_DI uint2 ld_word(const uint2 *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}
// Re-read *p until its epoch is `ep`, for at most `limit_ns` nanoseconds
// (0: M27B_WAIT_NS) or until an earlier wait has failed (*status non-zero);
// on failure record `code` in *status and return the last word read.
M27B_DI uint2 wait_word(const uint2 *p, uint2 w, uint32_t ep, int *status, int code,
                        unsigned long long limit_ns = 0) {
    if (w.y == ep) return w;
    const unsigned long long lim = limit_ns ? limit_ns : M27B_WAIT_NS;
    const unsigned long long t0 = global_ns();
    for (unsigned it = 0;; ++it) {
        w = ld_word(p);
        if (w.y == ep) return w;
        if ((it & 31u) == 31u && (global_ns() - t0 > lim || (status && *(volatile int *)status != 0))) {
            if (status) atomicCAS(status, 0, code);
            return w;
        }
    }
}

// ---- prologue gathers ----
// A q8_K activation record (fp32 d, 256 codes, 16 int16 sub-block sums:
// 292 bytes) in 32-bit words, and the two signed halves of a word.
constexpr int Q8K_WORDS = 73;
M27B_DI int s16_lo(uint32_t v) { return (int)(int16_t)(v & 0xffffu); }
M27B_DI int s16_hi(uint32_t v) { return (int)(int16_t)(v >> 16); }

// Element i of n goes from global src(i) to shared dst(i, value), read
// through L2 (the previous kernel wrote it).  Each thread issues R loads
// before any of its stores: the compiler does not move a global load above a
// store through a generic pointer, so a plain load-store loop pays one L2
// round trip per iteration.
template <int R, class T, class Src, class Dst>
M27B_DI void gather_l2(int n, Src src, Dst dst) {
    for (int i0 = threadIdx.x; i0 < n; i0 += R * (int)blockDim.x) {
        T v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = i0 + r * (int)blockDim.x;
            if (i < n) v[r] = __ldcg(src(i));
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = i0 + r * (int)blockDim.x;
            if (i < n) dst(i, v[r]);
        }
    }
}

// ---- asynchronous copies ----
// Asynchronous global -> shared copies (cp.async; completion by
// cp_async_wait_all in the issuing thread).
M27B_DI void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
M27B_DI void cp_async8(void *smem, const void *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}
M27B_DI void cp_async4(void *smem, const void *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}
M27B_DI void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

}  // namespace m27b
