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
// more than the SM's 512 columns together.  Shared memory enforces it: a CTA
// of 512 columns asks for at least MMA_SMEM_MIN, more than an SM has beside
// any other such CTA; a CTA of 256 columns asks for MMA_SMEM_PAIR_MIN ..
// MMA_SMEM_PAIR, so at most two fit.
constexpr size_t MMA_SMEM_LIMIT = 227 * 1024;
constexpr size_t MMA_SMEM_MIN = 148 * 1024;
constexpr size_t MMA_SMEM_PAIR = 112 * 1024;
constexpr size_t MMA_SMEM_PAIR_MIN = 80 * 1024;

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

// The tokens' q8_K records of a tensor-core matvec's K range, a warp per
// record: record rec = t * nb + kl (token t < n_tok, local block kl < nb) is
// read from src(t, kl) (73 words, through L2) and word o of it handed to
// put(t, kl, o, value); lane l takes words l, l + 32 and l + 64 (l < 9).  A
// warp issues the loads of R records before any store, and the address
// arithmetic is per record, not per word.  Records of tokens n_tok .. NB-1
// are put as zeros.
template <int R, class Src, class Put>
M27B_DI void gather_records(int n_tok, int NB, int nb, Src src, Put put) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nrec = n_tok * nb;
    for (int r0 = warp; r0 < nrec; r0 += R * nw) {
        unsigned v[R][3];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int rec = r0 + j * nw;
            if (rec < nrec) {
                const int t = rec / nb;
                const unsigned *p = src(t, rec - t * nb);
                v[j][0] = __ldcg(p + lane);
                v[j][1] = __ldcg(p + 32 + lane);
                v[j][2] = lane < Q8K_WORDS - 64 ? __ldcg(p + 64 + lane) : 0u;
            }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int rec = r0 + j * nw;
            if (rec < nrec) {
                const int t = rec / nb, kl = rec - t * nb;
                put(t, kl, lane, v[j][0]);
                put(t, kl, 32 + lane, v[j][1]);
                if (lane < Q8K_WORDS - 64) put(t, kl, 64 + lane, v[j][2]);
            }
        }
    }
    for (int rec = nrec + warp; rec < NB * nb; rec += nw) {
        const int t = rec / nb, kl = rec - t * nb;
        put(t, kl, lane, 0u);
        put(t, kl, 32 + lane, 0u);
        if (lane < Q8K_WORDS - 64) put(t, kl, 64 + lane, 0u);
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
