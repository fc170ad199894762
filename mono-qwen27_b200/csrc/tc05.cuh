// tc05.cuh — 5th-generation tensor-core helpers shared by the verify-pass
// matvecs on the tensor cores (qmv_q4k_mma.cu, qmv_q6k_mma.cu): TMEM
// allocation, kind::i8 MMAs with A in TMEM and B in shared memory, TMEM
// loads and stores, descriptors, and the bounded mbarrier waits of the
// warp-specialized pipelines.
#pragma once

#include "qmv_blk.cuh"

namespace m27b {

// TMEM residency.  tcgen05.alloc has no bounded form, so the CTAs of the
// tensor-core matvecs that can be resident on one SM at once (of one launch,
// or of launches that programmatic dependent launch overlaps) never ask for
// more than the SM's 512 columns together.  Shared memory enforces it: every
// such CTA allocates all 512 columns and asks for at least MMA_SMEM_MIN of
// shared memory, more than half of what an SM has, so no two are resident
// on one SM.
constexpr size_t MMA_SMEM_LIMIT = 227 * 1024;
constexpr size_t MMA_SMEM_MIN = 116 * 1024;

// ---- tcgen05 helpers ----
M27B_DI void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
M27B_DI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
M27B_DI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
M27B_DI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
M27B_DI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]^T, s8 x s8 -> s32, one thread.
M27B_DI void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
// The MMAs issued so far by this thread arrive on `bar` when they complete.
M27B_DI void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Eight consecutive 32-bit TMEM columns of this thread's lane.
M27B_DI void tmem_ld8(uint32_t taddr, int (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
// Four consecutive 32-bit TMEM columns of this thread's lane.
M27B_DI void tmem_ld4(uint32_t taddr, int (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr)
                 : "memory");
}
M27B_DI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Eight consecutive 32-bit TMEM columns of this thread's lane.
M27B_DI void tmem_st8(uint32_t taddr, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, uint32_t v4, uint32_t v5,
                      uint32_t v6, uint32_t v7) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(v0),
                 "r"(v1), "r"(v2), "r"(v3), "r"(v4), "r"(v5), "r"(v6), "r"(v7)
                 : "memory");
}
M27B_DI void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, no swizzle, core matrices of
// 8 rows x 16 bytes; 128 bytes between the two 16-byte K halves of a 32-byte
// K slice (leading offset), 256 bytes between 8-row groups (stride offset).
M27B_DI uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46);
}

// Instruction descriptor: D s32, A s8, B s8, both K-major, M = 128, N = NB
// (the callers' A values are unsigned codes below 128).
template <int NB>
constexpr uint32_t umma_idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

M27B_DI void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that gives up at once when the CTA's abort flag is raised, and
// raises it (recording status 5) when its own 2 s run out.
M27B_DI bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    if (*abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 8; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > M27B_WAIT_NS) {
            *abort = 1;
            if (status) atomicCAS(status, 0, 5);
            return false;
        }
    }
}

// The same wait for a whole worker warp: every lane leaves with one answer,
// so a warp never runs its .sync.aligned TMEM accesses with lanes missing.
M27B_DI bool warp_wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort, status)) != 0;
}

// The tokens' q8_K activations of a tensor-core matvec's K range (nb blocks)
// into shared memory: the codes into the canonical K-major no-swizzle UMMA
// layout of B (`bsm`: per block and 32-value slice s, NB / 8 core-matrix
// groups of 8 tokens x 2 K halves x 16 bytes), the block scale and the
// bsum words through the callbacks.  A warp task is (block kl, group of 8
// tokens): lane l takes token 8 g + l / 4 and word l % 4 of each 16-byte code
// chunk, so a store instruction covers 8 tokens x 16 bytes = 128 consecutive
// bytes (no bank conflict); its loads (16 chunk words, the scale on lanes
// l % 4 == 0, bsum words 65 + l % 4 and 69 + l % 4) all go out before its
// stores, R tasks at a time.  Tokens n_tok .. NB-1 are zero.  src(t, kl)
// points at token t's record of block kl (73 words: d, 64 code words, 8
// words of two bsums each), read through L2.
template <int R, int NB, class Src, class PutD, class PutBs>
M27B_DI void gather_tiles(int n_tok, int nb, uint8_t *bsm, Src src, PutD put_d, PutBs put_bs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int tl = lane >> 2, w = lane & 3;
    const int ntask = nb * (NB / 8);
    for (int k0 = warp; k0 < ntask; k0 += R * nw) {
        uint32_t v[R][16], dv[R], b0[R], b1[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int task = k0 + r * nw, kl = task / (NB / 8), t = (task % (NB / 8)) * 8 + tl;
            const bool on = task < ntask && t < n_tok;
            const unsigned *p = on ? src(t, kl) : nullptr;
#pragma unroll
            for (int c = 0; c < 16; ++c) v[r][c] = on ? __ldcg(p + 1 + 4 * c + w) : 0u;
            dv[r] = on && w == 0 ? __ldcg(p) : 0u;
            b0[r] = on ? __ldcg(p + 65 + w) : 0u;
            b1[r] = on ? __ldcg(p + 69 + w) : 0u;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int task = k0 + r * nw, kl = task / (NB / 8), g = task % (NB / 8), t = g * 8 + tl;
            if (task >= ntask) continue;
#pragma unroll
            for (int c = 0; c < 16; ++c)
                *(uint32_t *)(bsm + ((size_t)(kl * 8 + (c >> 1)) * (NB / 8) + g) * 256 + (c & 1) * 128 + tl * 16 +
                              w * 4) = v[r][c];
            if (w == 0) put_d(t, kl, dv[r]);
            put_bs(t, kl, w, b0[r]);
            put_bs(t, kl, 4 + w, b1[r]);
        }
    }
}

// K split across CTAs: ks ranges per 128-row tile, partial sums in `part`,
// one arrival counter per (tile, 32-row epilogue slice) in `count`.
struct MmaSplit {
    float *part;
    unsigned *count;
    int ks;
};

}  // namespace m27b
