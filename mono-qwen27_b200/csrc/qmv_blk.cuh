// qmv_blk.cuh — k-quant matvec with one super-block per lane, weights
// streamed through shared memory with coalesced asynchronous copies: q4_K
// (the target's matrices), q5_K and IQ4_XS (the reference's other 256-value
// types, k_q5k_mv_q8 src/mono27b_executor.cu:499-531 and k_iq4xs_mv_q8_dp4a
// :647-686).  The block type enters only through a traits struct (bytes per
// block, how a lane loads it, its dot product); the description below uses
// q4_K's 144 bytes.
//
// Mapping: a warp owns groups of 8 consecutive rows; lane L works on row slot
// L/4 of the group and, in pass p, on super-block 4p + L%4 of that row.  A
// lane holds a whole 144-byte block, so the per-block work — the fp16 scales,
// the twelve packed bytes of 6-bit scales/mins (reference get_scale_min_k4,
// src/mono27b_executor.cu:690-693), and the min correction against the
// activation's bsums — is done once per 256 weights.  The four lanes of a row
// reduce with two shuffles at the end of the row.
//
// Streaming: one "item" of a warp is pass p of one group — the 4 consecutive
// blocks (576 contiguous bytes) of each of the 8 rows.  Lane 0 of the warp
// copies an item into the warp's shared-memory stage with ONE 2-D TMA tensor
// copy (cp.async.bulk.tensor.2d, box 8 rows x 576 bytes over a uint32 view of
// the weight rows, no multicast) that completes on the stage's mbarrier.
// Rows past the end and blocks past the end of a row read as zeros (the
// tensor map's bounds), so ragged tails need no special case; the copies of item i+1 are in flight while item i is
// multiplied (two stages per warp, or all of a warp's items for matrices with few row groups; the block is copied to registers and the
// stage handed back before the math).  Every mbarrier wait is bounded by the
// global timer (M27B_WAIT_NS); a wait that runs out records an error in the
// library's device status word and the kernel drains its own copies before
// it returns.  Lanes read their block from the stage: the 576-byte slot
// stride and 144-byte block stride put the 8 lanes of each shared-memory
// phase on distinct banks.
//
// Activations are staged per CTA as 272-byte records per (token, block):
// 256 codes | 8 int16 sums of each 32-value sub-block (bsum[2j]+bsum[2j+1]);
// the fp32 block scales follow in their own array.  The 272-byte stride puts
// the four blocks a phase reads on disjoint banks.
#pragma once

#include <cuda.h>

#include "qmv_kernels.cuh"
#include "q8k_warp.cuh"

namespace m27b {

#ifndef M27B_BLK_STAGES
#define M27B_BLK_STAGES 2
#endif
#ifndef M27B_BLK_WARPS
#define M27B_BLK_WARPS 16
#endif
#ifndef M27B_BLK_CTAS
#define M27B_BLK_CTAS 1
#endif
constexpr int BLK_XREC = 272;                 // bytes per staged (token, block) activation record
constexpr int BLK_STAGES = M27B_BLK_STAGES;   // stages per warp
constexpr int BLK_WARPS = M27B_BLK_WARPS;     // most warps per CTA
constexpr int BLK_CTAS = M27B_BLK_CTAS;       // resident CTAs per SM the launch plans for
constexpr int BLK_THREADS = BLK_WARPS * 32;
// the CTAs of an SM share its 228 KB of shared memory (1 KB reserved per CTA)
constexpr size_t BLK_SMEM_MAX = BLK_CTAS == 1 ? 226 * 1024 : 112 * 1024;

// One item: 8 rows x 4 consecutive blocks of `bytes` bytes (q4_K: 4608).
constexpr int blk_item(int bytes) { return 8 * 4 * bytes; }
// stages + barriers of one warp
// most stages per warp: a matrix with few row groups streams each group
// with one warp that has all of the group's items in flight at once
constexpr int BLK_MAX_STAGES = 8;
constexpr size_t blk_warp_bytes(int bytes, int nst = BLK_STAGES) {
    return (size_t)nst * blk_item(bytes) + (size_t)nst * 8;
}

inline size_t blk_x_bytes(int k, int nt) { return (size_t)nt * ((size_t)k / 256) * (BLK_XREC + 4); }

// Warps per CTA: as many as the shared memory left after the staged
// activations holds stages for (at most BLK_WARPS); 0 if not even one fits.
inline size_t blk_part_bytes(int nt) { return (size_t)BLK_WARPS * 8 * 2 * nt * 4; }

inline int blk_warps(int k, int nt, int bytes = 144) {
    const size_t x = blk_x_bytes(k, nt) + blk_part_bytes(nt);
    if (x + 16 >= BLK_SMEM_MAX) return 0;
    const size_t w = (BLK_SMEM_MAX - x - 16) / blk_warp_bytes(bytes);
    return (int)(w < (size_t)BLK_WARPS ? w : (size_t)BLK_WARPS);
}

inline size_t blk_smem_for(int nwarps, int k, int nt, int bytes = 144, int nst = BLK_STAGES) {
    return (size_t)nwarps * blk_warp_bytes(bytes, nst) + blk_x_bytes(k, nt) + blk_part_bytes(nt) + 16;
}
inline size_t blk_smem_bytes(int k, int nt, int bytes = 144) {
    return blk_smem_for(blk_warps(k, nt, bytes), k, nt, bytes);
}

// ---- mbarrier + bulk-copy helpers (sm_90+ PTX; no cluster multicast) ----
M27B_DI uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

M27B_DI void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
M27B_DI void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
M27B_DI void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

M27B_DI void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

M27B_DI void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 2-D tiled TMA load of the box at (x, y) of the tensor map into shared memory.
M27B_DI void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((unsigned long long)tm), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Test the phase; if it is not complete the thread may wait in hardware for a
// system-dependent time before the test returns false.  (No suspend-time
// hint: with a 20 us hint the tensor-core kernel's hand-offs ran ~4% slower.)
M27B_DI bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most
// M27B_WAIT_NS; returns false (and records `code` in *status) on timeout.
M27B_DI bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 8; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > M27B_WAIT_NS) {
            if (status) atomicCAS(status, 0, code);
            return false;
        }
    }
}

template <int NT>
M27B_DI void stage_x_blk(const QmvArgs &a, uint8_t *xrec, float *xd) {
    const int nb = a.k / 256;
    const uint8_t *src = (const uint8_t *)a.xq;  // NT*nb blocks of 292 bytes
    // a record is 73 words: d, 64 code words, 8 words of two bsums each
    gather_l2<8, unsigned>(NT * nb * Q8K_WORDS, [&](int i) { return (const unsigned *)src + i; },
                           [&](int i, unsigned v) {
                               const int blk = i / Q8K_WORDS, o = i - blk * Q8K_WORDS;
                               uint8_t *rec = xrec + (size_t)blk * BLK_XREC;
                               if (o == 0) xd[blk] = __uint_as_float(v);
                               else if (o <= 64) ((uint32_t *)rec)[o - 1] = v;
                               else ((int16_t *)(rec + 256))[o - 65] = (int16_t)(s16_lo(v) + s16_hi(v));
                           });
}

// The same records built from fp32 activations in the prologue (the fused
// quantize + matvec entries): warp w quantizes blocks w, w + nwarps, ... of
// the NT rows with the shared q8_K warp routine (the codes, sub-block sums
// and scale equal those m27b_act_quant produces).  A warp loads all of its
// blocks (up to QX_REGS) before any arithmetic, so the prologue pays one L2
// round trip.  With a.xnorm_on the rows are first RMSNormed with weights
// a.xnorm (may be null) and a.eps: each warp's sums of squares over the
// values it holds are reduced over the CTA in warp order (`red`: nwarps * NT
// floats).
constexpr int QX_REGS = 4;

M27B_DI void quant_x_rec(float (&v)[8], int lane, uint8_t *rec8, float *dslot) {
    uint32_t packed[2];
    int sum;
    float d;
    quant_q8K_lane(v, lane, packed, sum, d);
    uint32_t *rec = (uint32_t *)rec8;
    rec[2 * lane] = packed[0];
    rec[2 * lane + 1] = packed[1];
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);  // lanes 4s..4s+3 hold sub-block s
    if ((lane & 3) == 0) ((int16_t *)(rec8 + 256))[lane >> 2] = (int16_t)sum;
    if (lane == 0) *dslot = d;
}

template <int NT>
M27B_DI void quant_x_blk(const QmvArgs &a, uint8_t *xrec, float *xd, float *red) {
    const int nb = a.k / 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int total = NT * nb;
    if ((total + nw - 1) / nw <= QX_REGS) {
        float v[QX_REGS][8];
#pragma unroll
        for (int r = 0; r < QX_REGS; ++r) {
            const int i = warp + r * nw;
            if (i < total) {
                const int t = i / nb, b = i - t * nb;
                const float4 *xr = (const float4 *)(a.xf + (size_t)t * a.ldxf + b * 256 + lane * 8);
                const float4 p0 = __ldcg(xr), p1 = __ldcg(xr + 1);
                v[r][0] = p0.x; v[r][1] = p0.y; v[r][2] = p0.z; v[r][3] = p0.w;
                v[r][4] = p1.x; v[r][5] = p1.y; v[r][6] = p1.z; v[r][7] = p1.w;
            }
        }
        if (a.xnorm_on) {
            float ss[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) ss[t] = 0.0f;
#pragma unroll
            for (int r = 0; r < QX_REGS; ++r) {
                const int i = warp + r * nw;
                if (i < total) {
                    float s2 = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) s2 = fmaf(v[r][j], v[r][j], s2);
                    const int t = i / nb;
#pragma unroll
                    for (int t2 = 0; t2 < NT; ++t2)
                        if (t2 == t) ss[t2] += s2;
                }
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float w = warp_sum(ss[t]);
                if (lane == 0) red[warp * NT + t] = w;
            }
            __syncthreads();
            float ns[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float tot = 0.0f;
                for (int w = 0; w < nw; ++w) tot += red[w * NT + t];
                ns[t] = 1.0f / sqrtf(tot / (float)a.k + a.eps);
            }
            __syncthreads();  // red is reused by the caller
#pragma unroll
            for (int r = 0; r < QX_REGS; ++r) {
                const int i = warp + r * nw;
                if (i < total) {
                    const int t = i / nb, b = i - t * nb;
                    float nst = ns[0];
#pragma unroll
                    for (int t2 = 1; t2 < NT; ++t2)
                        if (t2 == t) nst = ns[t2];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        v[r][j] = v[r][j] * nst;
                        if (a.xnorm) v[r][j] = v[r][j] * a.xnorm[b * 256 + lane * 8 + j];
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < QX_REGS; ++r) {
            const int i = warp + r * nw;
            if (i < total) quant_x_rec(v[r], lane, xrec + (size_t)i * BLK_XREC, xd + i);
        }
        return;
    }
    // long rows: two passes (sum of squares, then quantize), block by block
    float ns[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) ns[t] = 1.0f;
    if (a.xnorm_on) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float4 *x4 = (const float4 *)(a.xf + (size_t)t * a.ldxf);
            float ss = 0.0f;
#pragma unroll 4
            for (int i = threadIdx.x; i < a.k / 4; i += blockDim.x) {
                const float4 q = x4[i];
                ss = fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, fmaf(q.w, q.w, ss))));
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.0f;
            for (int w = 0; w < nw; ++w) tot += red[w];
            ns[t] = 1.0f / sqrtf(tot / (float)a.k + a.eps);
            __syncthreads();
        }
    }
    for (int i = warp; i < total; i += nw) {
        const int t = i / nb, b = i - t * nb;
        const float4 *xr = (const float4 *)(a.xf + (size_t)t * a.ldxf + b * 256 + lane * 8);
        const float4 p0 = __ldcg(xr), p1 = __ldcg(xr + 1);
        float v[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        if (a.xnorm_on) {
            float nst = ns[0];
#pragma unroll
            for (int t2 = 1; t2 < NT; ++t2)
                if (t2 == t) nst = ns[t2];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[j] = v[j] * nst;
                if (a.xnorm) v[j] = v[j] * a.xnorm[b * 256 + lane * 8 + j];
            }
        }
        quant_x_rec(v, lane, xrec + (size_t)i * BLK_XREC, xd + i);
    }
}

// One block (held in registers) times NT staged activation blocks.
template <int NT>
M27B_DI void q4k_block_mac(const uint4 (&v)[9], const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
    const uint4 hd = v[0];
    // all eight 6-bit scales and mins of the block, one byte each
    const uint32_t sc03 = hd.y & 0x3f3f3f3fu;
    const uint32_t mn03 = hd.z & 0x3f3f3f3fu;
    const uint32_t sc47 = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
    const float dw = h2f(hd.x), dmw = h2f(hd.x >> 16);
    int isum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) isum[t] = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint4 qa = v[1 + 2 * g], qb = v[2 + 2 * g];  // qs bytes 32g .. 32g+31
        const uint32_t lo[8] = {qa.x & 0x0f0f0f0fu, qa.y & 0x0f0f0f0fu, qa.z & 0x0f0f0f0fu, qa.w & 0x0f0f0f0fu,
                                qb.x & 0x0f0f0f0fu, qb.y & 0x0f0f0f0fu, qb.z & 0x0f0f0f0fu, qb.w & 0x0f0f0f0fu};
        const uint32_t hi[8] = {qa.x & 0xf0f0f0f0u, qa.y & 0xf0f0f0f0u, qa.z & 0xf0f0f0f0u, qa.w & 0xf0f0f0f0u,
                                qb.x & 0xf0f0f0f0u, qb.y & 0xf0f0f0f0u, qb.z & 0xf0f0f0f0u, qb.w & 0xf0f0f0f0u};
        const uint32_t scw = g < 2 ? sc03 : sc47;
        const int sh = 16 * (g & 1);
        const int s_lo = (int)((scw >> sh) & 0xffu), s_hi = (int)((scw >> (sh + 8)) & 0xffu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint8_t *xr = xrec0 + (size_t)t * nb * BLK_XREC + 64 * g;
            const int4 x0 = *(const int4 *)(xr);
            const int4 x1 = *(const int4 *)(xr + 16);
            const int4 x2 = *(const int4 *)(xr + 32);
            const int4 x3 = *(const int4 *)(xr + 48);
            int dl = dp4a_us(lo[0], x0.x, 0);
            dl = dp4a_us(lo[1], x0.y, dl);
            dl = dp4a_us(lo[2], x0.z, dl);
            dl = dp4a_us(lo[3], x0.w, dl);
            dl = dp4a_us(lo[4], x1.x, dl);
            dl = dp4a_us(lo[5], x1.y, dl);
            dl = dp4a_us(lo[6], x1.z, dl);
            dl = dp4a_us(lo[7], x1.w, dl);
            int dh = dp4a_us(hi[0], x2.x, 0);  // 16 x the high-nibble dot
            dh = dp4a_us(hi[1], x2.y, dh);
            dh = dp4a_us(hi[2], x2.z, dh);
            dh = dp4a_us(hi[3], x2.w, dh);
            dh = dp4a_us(hi[4], x3.x, dh);
            dh = dp4a_us(hi[5], x3.y, dh);
            dh = dp4a_us(hi[6], x3.z, dh);
            dh = dp4a_us(hi[7], x3.w, dh);
            isum[t] += s_lo * dl + s_hi * (dh >> 4);
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t *xr = xrec0 + (size_t)t * nb * BLK_XREC;
        const int4 bs = *(const int4 *)(xr + 256);  // sub-block bsum pairs
        int msum = __dp2a_lo(bs.x, (int)mn03, 0);
        msum = __dp2a_hi(bs.y, (int)mn03, msum);
        msum = __dp2a_lo(bs.z, (int)mn47, msum);
        msum = __dp2a_hi(bs.w, (int)mn47, msum);
        const float dx = xd0[t * nb];
        acc[t] = fmaf(dw * dx, (float)isum[t], acc[t]);
        acc[t] = fmaf(-(dmw * dx), (float)msum, acc[t]);
    }
}

// One q5_K block (176 bytes: d, dmin, scales[12] | qh[32] | qs[128]) times
// NT staged activation blocks.  The nibbles and the 6-bit scales/mins are
// q4_K's; bit s of qh[l] is bit 4 of element l of sub-block s, merged into
// the byte lanes before the dp4a (codes 0..31), as k_q5k_mv_q8 and ggml's
// vec_dot_q5_K_q8_K define the value (src/mono27b_executor.cu:955-969).
template <int NT>
M27B_DI void q5k_block_mac(const uint4 (&v)[11], const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
    const uint4 hd = v[0];
    const uint32_t sc03 = hd.y & 0x3f3f3f3fu;
    const uint32_t mn03 = hd.z & 0x3f3f3f3fu;
    const uint32_t sc47 = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
    const float dw = h2f(hd.x), dmw = h2f(hd.x >> 16);
    const uint32_t qh[8] = {v[1].x, v[1].y, v[1].z, v[1].w, v[2].x, v[2].y, v[2].z, v[2].w};
    int isum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) isum[t] = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint4 qa = v[3 + 2 * g], qb = v[4 + 2 * g];  // qs bytes 32g .. 32g+31
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (w[i] & 0x0f0f0f0fu) | (((qh[i] >> (2 * g)) & 0x01010101u) << 4);
            hi[i] = ((w[i] >> 4) & 0x0f0f0f0fu) | (((qh[i] >> (2 * g + 1)) & 0x01010101u) << 4);
        }
        const uint32_t scw = g < 2 ? sc03 : sc47;
        const int sh = 16 * (g & 1);
        const int s_lo = (int)((scw >> sh) & 0xffu), s_hi = (int)((scw >> (sh + 8)) & 0xffu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint8_t *xr = xrec0 + (size_t)t * nb * BLK_XREC + 64 * g;
            const int4 x0 = *(const int4 *)(xr);
            const int4 x1 = *(const int4 *)(xr + 16);
            const int4 x2 = *(const int4 *)(xr + 32);
            const int4 x3 = *(const int4 *)(xr + 48);
            int dl = dp4a_us(lo[0], x0.x, 0);
            dl = dp4a_us(lo[1], x0.y, dl);
            dl = dp4a_us(lo[2], x0.z, dl);
            dl = dp4a_us(lo[3], x0.w, dl);
            dl = dp4a_us(lo[4], x1.x, dl);
            dl = dp4a_us(lo[5], x1.y, dl);
            dl = dp4a_us(lo[6], x1.z, dl);
            dl = dp4a_us(lo[7], x1.w, dl);
            int dh = dp4a_us(hi[0], x2.x, 0);
            dh = dp4a_us(hi[1], x2.y, dh);
            dh = dp4a_us(hi[2], x2.z, dh);
            dh = dp4a_us(hi[3], x2.w, dh);
            dh = dp4a_us(hi[4], x3.x, dh);
            dh = dp4a_us(hi[5], x3.y, dh);
            dh = dp4a_us(hi[6], x3.z, dh);
            dh = dp4a_us(hi[7], x3.w, dh);
            isum[t] += s_lo * dl + s_hi * dh;
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t *xr = xrec0 + (size_t)t * nb * BLK_XREC;
        const int4 bs = *(const int4 *)(xr + 256);
        int msum = __dp2a_lo(bs.x, (int)mn03, 0);
        msum = __dp2a_hi(bs.y, (int)mn03, msum);
        msum = __dp2a_lo(bs.z, (int)mn47, msum);
        msum = __dp2a_hi(bs.w, (int)mn47, msum);
        const float dx = xd0[t * nb];
        acc[t] = fmaf(dw * dx, (float)isum[t], acc[t]);
        acc[t] = fmaf(-(dmw * dx), (float)msum, acc[t]);
    }
}

M27B_DI uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// The IQ4_NL / IQ4_XS codebook (reference src/mono27b_executor.cu:51-55) as
// four words of signed bytes: entries 0-3, 4-7, 8-11, 12-15.
constexpr uint32_t iq4_word(int a, int b, int c, int d) {
    return (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c << 16) |
           ((uint32_t)(uint8_t)d << 24);
}
constexpr uint32_t IQ4_T0 = iq4_word(-127, -104, -83, -65), IQ4_T1 = iq4_word(-49, -35, -22, -10);
constexpr uint32_t IQ4_T2 = iq4_word(1, 13, 25, 38), IQ4_T3 = iq4_word(53, 69, 89, 113);

// The 8 codes of one qs word (4 bytes, low nibble = element j of the
// sub-block's first half, high nibble = element j of its second half) as
// codebook bytes: lo4 = the four low-nibble values, hi4 = the four high.
// prmt looks a nibble's low 3 bits up in entries 0-7 and in 8-15; a second
// prmt in sign-replicate mode turns each nibble's bit 3 into a byte mask that
// picks one of the two (selector nibble 0x9 replicates the sign of byte 1 =
// 0x80 -> 0xff, 0x0 takes byte 0 = 0x00); the lookups come out interleaved
// (l0 h0 l1 h1 | l2 h2 l3 h3) and two more prmt split them.
M27B_DI void iq4_lookup(uint32_t q, uint32_t &lo4, uint32_t &hi4) {
    const uint32_t s = q & 0x77777777u;
    const uint32_t m8 = q & 0x88888888u;
    const uint32_t sm = m8 | (m8 >> 3);
    const uint32_t a0 = prmt(IQ4_T0, IQ4_T1, s), b0 = prmt(IQ4_T2, IQ4_T3, s);
    const uint32_t a1 = prmt(IQ4_T0, IQ4_T1, s >> 16), b1 = prmt(IQ4_T2, IQ4_T3, s >> 16);
    const uint32_t k0 = prmt(0x8000u, 0u, sm), k1 = prmt(0x8000u, 0u, sm >> 16);
    const uint32_t v0 = (a0 & ~k0) | (b0 & k0), v1 = (a1 & ~k1) | (b1 & k1);
    lo4 = prmt(v0, v1, 0x6420u);
    hi4 = prmt(v0, v1, 0x7531u);
}

// One IQ4_XS block (136 bytes: d, scales_h | scales_l[4] | qs[128], read as
// 17 x 8 bytes) times NT staged activation blocks: per 32-value sub-block ib
// the signed dot of its codebook values with the q8_K codes, times the
// stored 6-bit scale minus 32, summed in integers over the block, then times
// d * d_x (ggml's vec_dot_iq4_xs_q8_K in integer form).
template <int NT>
M27B_DI void iq4xs_block_mac(const uint2 (&v)[17], const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
    const float dw = h2f(v[0].x);
    const uint32_t sh = v[0].x >> 16, sl = v[0].y;
    int isum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) isum[t] = 0;
#pragma unroll
    for (int ib = 0; ib < 8; ++ib) {
        const int ls = (int)(((sl >> (4 * ib)) & 0xfu) | (((sh >> (2 * ib)) & 3u) << 4)) - 32;
        const uint32_t q[4] = {v[1 + 2 * ib].x, v[1 + 2 * ib].y, v[2 + 2 * ib].x, v[2 + 2 * ib].y};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) iq4_lookup(q[i], lo[i], hi[i]);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint8_t *xr = xrec0 + (size_t)t * nb * BLK_XREC + 32 * ib;
            const int4 xl = *(const int4 *)(xr);       // values 0..15 of the sub-block
            const int4 xh = *(const int4 *)(xr + 16);  // values 16..31
            int dot = __dp4a((int)lo[0], xl.x, 0);
            dot = __dp4a((int)lo[1], xl.y, dot);
            dot = __dp4a((int)lo[2], xl.z, dot);
            dot = __dp4a((int)lo[3], xl.w, dot);
            dot = __dp4a((int)hi[0], xh.x, dot);
            dot = __dp4a((int)hi[1], xh.y, dot);
            dot = __dp4a((int)hi[2], xh.z, dot);
            dot = __dp4a((int)hi[3], xh.w, dot);
            isum[t] += ls * dot;
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = fmaf(dw * xd0[t * nb], (float)isum[t], acc[t]);
}

// Block traits: bytes per block, the lane's register copy of its block (read
// from the stage), and the block's dot product with the staged activations.
struct BlkQ4K {
    static constexpr int BYTES = 144;
    struct Reg { uint4 v[9]; };
    static M27B_DI void load(const uint8_t *p, Reg &r) {
#pragma unroll
        for (int j = 0; j < 9; ++j) r.v[j] = *(const uint4 *)(p + 16 * j);
    }
    template <int NT>
    static M27B_DI void mac(const Reg &r, const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
        q4k_block_mac<NT>(r.v, xrec0, xd0, nb, acc);
    }
};

struct BlkQ5K {
    static constexpr int BYTES = 176;
    struct Reg { uint4 v[11]; };
    static M27B_DI void load(const uint8_t *p, Reg &r) {
#pragma unroll
        for (int j = 0; j < 11; ++j) r.v[j] = *(const uint4 *)(p + 16 * j);
    }
    template <int NT>
    static M27B_DI void mac(const Reg &r, const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
        q5k_block_mac<NT>(r.v, xrec0, xd0, nb, acc);
    }
};

// 136-byte blocks sit at 8-byte offsets in the stage: 8-byte reads (the 16
// lanes of a 64-bit shared-memory phase land on distinct banks: 544-byte slot
// and 136-byte block strides).
struct BlkIQ4XS {
    static constexpr int BYTES = 136;
    struct Reg { uint2 v[17]; };
    static M27B_DI void load(const uint8_t *p, Reg &r) {
#pragma unroll
        for (int j = 0; j < 17; ++j) r.v[j] = *(const uint2 *)(p + 8 * j);
    }
    template <int NT>
    static M27B_DI void mac(const Reg &r, const uint8_t *xrec0, const float *xd0, int nb, float (&acc)[NT]) {
        iq4xs_block_mac<NT>(r.v, xrec0, xd0, nb, acc);
    }
};

// Work of a warp: items (group, pass, matrix) in that order, matrix fastest
// (SWIGLU streams the gate blocks, then the up blocks, of the same pass).
template <class BT, int NT, int EPI>
M27B_DI void qmv_kblk_body(const QmvArgs &a, const CUtensorMap *tm0, const CUtensorMap *tm1, int split, int nst) {
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    constexpr int ITEM = blk_item(BT::BYTES);
    extern __shared__ __align__(128) uint8_t kblk_smem[];
    uint8_t *smem = kblk_smem;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane >> 2, qd = lane & 3;
    const int nwarps = blockDim.x >> 5;
    const int ngroups = (a.rows + 7) >> 3;
    const int P = (a.rb + 3) >> 2;  // passes per row
    const int nb = a.rb;

    // split == 1: warp wg owns groups wg, wg+W, ...; all passes of each
    // split == nwarps: the CTA owns groups blockIdx.x, +gridDim.x, ...; warp
    // w takes passes [w*P/split, (w+1)*P/split) of each and the partial sums
    // are combined in warp order (deterministic).
    // (warp-major: the groups go round the CTAs first, so that every CTA,
    // and every SM, carries the same number of groups within one)
    const int wg = split == 1 ? warp * gridDim.x + blockIdx.x : blockIdx.x;
    const int W = split == 1 ? gridDim.x * nwarps : gridDim.x;
    const int my_groups = wg < ngroups ? (ngroups - 1 - wg) / W + 1 : 0;
    const int p_lo = split == 1 ? 0 : (warp * P) / split;
    const int my_passes = (split == 1 ? P : ((warp + 1) * P) / split) - p_lo;

    // [stages of all warps | activation records | block scales | partials | barriers]
    uint8_t *stage0 = smem + (size_t)warp * nst * ITEM;
    uint8_t *xrec = smem + (size_t)nwarps * nst * ITEM;
    float *xd = (float *)(xrec + (size_t)NT * nb * BLK_XREC);
    float *part = (float *)(((uintptr_t)(xd + NT * nb) + 15) & ~(uintptr_t)15);  // [BLK_WARPS][8][2][NT]
    uint64_t *bar = (uint64_t *)(part + (size_t)BLK_WARPS * 8 * 2 * NT) + (size_t)warp * nst;
    if (lane == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    // copy cursor: lane 0 issues one tensor copy per item; all lanes track it
    int lg = 0, lp = 0, lm = 0, li = 0, ls = 0;  // ls = li % nst
    auto issue_item = [&]() {
        if (lg < my_groups && my_passes > 0) {
            if (lane == 0) {
                uint64_t *b = &bar[ls];
                fence_proxy_async();  // the stage's previous reads precede the async writes
                mbar_arrive_expect_tx(b, ITEM);
                tma_load_2d(stage0 + ls * ITEM, (NM == 2 && lm == 1) ? tm1 : tm0, (p_lo + lp) * BT::BYTES,
                            (wg + lg * W) * 8, b);
            }
            ++li;
            if (++ls == nst) ls = 0;
            if (++lm == NM) {
                lm = 0;
                if (++lp == my_passes) { lp = 0; ++lg; }
            }
        }
    };

    // the stages' copies go out before the activations are staged
    for (int i = 0; i < nst; ++i) issue_item();
    // the weights are not produced by the previous kernel: their copies are
    // already in flight; the activations (and every global write) wait for it
    pdl_wait();
    if (a.xf)
        quant_x_blk<NT>(a, xrec, xd, part);
    else
        stage_x_blk<NT>(a, xrec, xd);
    pdl_trigger();
    __syncthreads();

    float acc[NM][NT];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[m][t] = 0.0f;
    unsigned long long best[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) best[t] = 0ull;

    int ci = 0, cs = 0;  // items consumed; cs = ci % nst
    uint32_t cph = 0;     // phase parity of stage cs
    bool ok = true;
    int g = 0;
    for (; g < my_groups; ++g) {
        const int row = (wg + g * W) * 8 + slot;
        for (int pt = 0; pt < my_passes; ++pt) {
            const int b = 4 * (p_lo + pt) + qd;
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                // every lane waits (bounded); the warp leaves together if any lane gave up
                const bool landed = mbar_wait_bounded(&bar[cs], cph, a.status, 1);
                if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
                // take this lane's block into registers, then hand the stage back
                // to the copy engine: a later item streams in during the math
                typename BT::Reg v;
                BT::load(stage0 + cs * ITEM + slot * (4 * BT::BYTES) + qd * BT::BYTES, v);
                __syncwarp();
                issue_item();
                ++ci;
                if (++cs == nst) { cs = 0; cph ^= 1u; }
                if (row < a.rows && b < nb) BT::template mac<NT>(v, xrec + (size_t)b * BLK_XREC, xd + b, nb, acc[m]);
            }
            if (!ok) break;
        }
        if (!ok) break;

        // group done: reduce the four lanes of each row (lane slot*4 keeps it)
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float s = acc[m][t];
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                acc[m][t] = s;
            }
        if (split > 1) {
            // combine the warps' partial sums in warp order
            if (qd == 0) {
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int t = 0; t < NT; ++t) part[(((size_t)warp * 8 + slot) * 2 + m) * NT + t] = acc[m][t];
            }
            __syncthreads();
            if (warp == 0 && qd == 0) {
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        float v = 0.0f;
                        for (int w = 0; w < split; ++w) v += part[(((size_t)w * 8 + slot) * 2 + m) * NT + t];
                        acc[m][t] = v;
                    }
            }
            __syncthreads();
        }
        if ((split == 1 || warp == 0) && qd == 0 && row < a.rows) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const size_t o = (size_t)t * a.ldy + row;
                const float s0 = acc[0][t];
                if constexpr (EPI == EPI_STORE) {
                    a.y[o] = a.residual ? s0 + a.residual[o] : s0;
                } else if constexpr (EPI == EPI_PUSH) {
                    push_row(a.push, o, a.residual ? s0 + a.residual[o] : s0);
                } else if constexpr (EPI == EPI_SWIGLU) {
                    a.y[o] = s0 / (1.0f + expf(-s0)) * acc[NM - 1][t];
                } else {
                    if (a.y) a.y[o] = s0;
                    const unsigned long long key = argmax_key(s0, (uint32_t)row + a.row_offset);
                    best[t] = key > best[t] ? key : best[t];
                }
            }
        }
        if constexpr (EPI == EPI_SWIGLU && NT == 1) {
            // q8_K of the SwiGLU rows for the next matvec (a.q8out set): the
            // warp that stores the last 8-row group of a 256-row block (an
            // arrival count per block) quantizes the block from L2, with the
            // routine and codes of m27b_act_quant, and resets the count
            if (a.q8out && (split == 1 || warp == 0)) {
                const int grp = wg + g * W, blk = grp >> 5;
                __threadfence();
                __syncwarp();
                unsigned prev = 0u;
                if (lane == 0) prev = atomicAdd(a.q8cnt + blk, 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == 31u) {
                    if (lane == 0) a.q8cnt[blk] = 0u;
                    __threadfence();
                    const float4 *src = (const float4 *)(a.y + (size_t)blk * 256 + lane * 8);
                    const float4 p0 = __ldcg(src), p1 = __ldcg(src + 1);
                    float v[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                    quant_q8K_warp(v, lane, (m27b_block_q8_K *)a.q8out + blk);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[m][t] = 0.0f;
    }
    if (!ok) {
        // a wait ran out: let every copy this warp issued land (bounded again)
        // before the CTA's shared memory is released
        for (; ci < li; ++ci) {
            mbar_wait_bounded(&bar[cs], cph, a.status, 2);
            if (++cs == nst) { cs = 0; cph ^= 1u; }
        }
        // keep the CTA-wide barriers of the cooperative split balanced
        if (split > 1)
            for (; g < my_groups; ++g) {
                __syncthreads();
                __syncthreads();
            }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (ok && qd == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (best[t] != 0ull) atomicMax(a.best + t, best[t]);
        }
    }
}

template <int NT, int EPI>
__global__ void __launch_bounds__(BLK_THREADS, BLK_CTAS)
    k_qmv_q4k_blk(const QmvArgs a, const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                  int split, int nst) {
    qmv_kblk_body<BlkQ4K, NT, EPI>(a, &tm0, &tm1, split, nst);
}

template <int NT, int EPI>
__global__ void __launch_bounds__(BLK_THREADS, BLK_CTAS)
    k_qmv_q5k_blk(const QmvArgs a, const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                  int split, int nst) {
    qmv_kblk_body<BlkQ5K, NT, EPI>(a, &tm0, &tm1, split, nst);
}

template <int NT, int EPI>
__global__ void __launch_bounds__(BLK_THREADS, BLK_CTAS)
    k_qmv_iq4xs_blk(const QmvArgs a, const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                    int split, int nst) {
    qmv_kblk_body<BlkIQ4XS, NT, EPI>(a, &tm0, &tm1, split, nst);
}

}  // namespace m27b
