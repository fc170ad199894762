// qmv_q4k_mma.cu — q4_K weights x 5..16 q8_K tokens on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in TMEM): the batched
// "verify" matvec of speculative decoding.
//
// Replaces, for 5..16 tokens, the reference's per-token dp4a matvec
// (k_q4k_mv_q8_dp4a, src/mono27b_executor.cu:320-364, called once per
// token).  Result semantics are ggml's vec_dot_q4_K_q8_K, as in the dp4a
// kernels (qmv_blk.cuh): per super-block the integer sum
//     isum = sum_s sc_s * dot(q4_s, q8_s)          (s = 8 sub-blocks of 32)
//     msum = sum_s m_s * bsum_s
// and y += d*dx*isum - dmin*dx*msum in fp32.
//
// Mapping onto the tensor cores.  One MMA of shape M=128 rows x N tokens x
// K=32 is exactly one q4_K sub-block: A = the sub-block's 4-bit values as
// bytes, B = the tokens' q8 codes, D = the 32-term integer dot products of
// every (row, token), each sub-block into its own TMEM accumulator.  The
// epilogue applies the 6-bit scales in integers (isum = sum_s sc_s * D_s,
// exactly ggml's), the min term with dp2a against the activation's bsums, and
// the fp16/fp32 block scales.  The A operand lives in TMEM: the thread that
// owns a row writes its bytes into its own TMEM lane (tcgen05.st), so the
// narrow MMAs (N = 8 or 16) do not re-read a 4 KB A tile from shared memory.
//
// Pipeline per CTA (one 128-row tile at a time, persistent over tiles, one
// CTA per SM), warp-specialized and synchronised only by mbarriers:
//   * warp 8 issues: TMA copies of one raw 128-row x 144-byte block column per
//     stage (2-D tensor map, no multicast), and, per half-block (4
//     sub-blocks), the 4 MMAs plus a commit;
//   * warps 0-7 unpack a half-block into one of two TMEM A buffers, and run
//     the epilogue of the previous block (tcgen05.ld of its 8 accumulators,
//     one row per thread, eight tokens per thread);
//   * hand-offs: stage full (TMA) -> stage empty (the unpacking warps have
//     read it), A buffer full -> MMAs done (the buffer is free again and the
//     block's accumulators are final), accumulators free (epilogue read).
// The activations (all K, all tokens) are staged once per CTA in the
// canonical K-major no-swizzle UMMA layout, with their scales and bsum
// pairs.  Every wait is bounded (2 s); a timeout records status 5 and raises
// the CTA's abort flag, every role leaves its loop, the issuing thread waits
// (bounded) for its own copies and MMAs, and the CTA frees its TMEM.
#include "qmv_blk.cuh"
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"

namespace m27b {

constexpr int MMA_ROWS = 128;
constexpr int MMA_WORKERS = 256;                 // warps 0-7: unpack + epilogue
constexpr int MMA_THREADS = MMA_WORKERS + 32;    // warp 8: TMA + MMA issue
constexpr int MMA_RAW_BYTES = MMA_ROWS * 144;    // one TMA box: 128 rows x one q4_K block
constexpr int MMA_TMEM_COLS = 512;               // D: 2 blocks x 8 sub-blocks x 16; A: 2 x 32
constexpr int MMA_ACOL = 256;                    // first TMEM column of the A buffers
constexpr int MMA_NA = 2;                        // A buffers (half-blocks the unpacking may run ahead)
constexpr size_t MMA_SMEM_LIMIT = 227 * 1024;
// Every CTA asks for more than half of an SM's shared memory, so no two CTAs
// of this kernel (of one launch, or of two launches that programmatic
// dependent launch overlaps) are ever resident on one SM: each allocates all
// 512 TMEM columns, and tcgen05.alloc has no bounded form — a second
// allocator on the SM would wait for the first CTA to exit, unbounded.
constexpr size_t MMA_SMEM_MIN = 116 * 1024;

struct MmaLayout {
    size_t b, dx, bs, raw, bar, flag, total;
    int stages;
};

// Shared memory plan for K = 256 * rb values and an MMA N of nb_tok (8 or 16).
__host__ __device__ inline MmaLayout mma_layout(int rb, int nb_tok, int stages) {
    MmaLayout L;
    size_t off = 0;
    L.b = off;
    off += (size_t)rb * 8 * nb_tok * 32;                     // codes, UMMA layout
    L.dx = off;
    off += (size_t)nb_tok * rb * 4;                          // block scales
    L.bs = off;
    off += (size_t)nb_tok * rb * 16;                         // bsum pairs
    off = (off + 127) & ~(size_t)127;
    L.raw = off;
    off += (size_t)stages * MMA_RAW_BYTES;
    L.bar = off;  // full[stages], empty[stages], a_full[NA], mma_done[NA], d_free[2], drain
    off += (size_t)(2 * stages + 2 * MMA_NA + 3) * 8;
    L.flag = off;  // abort flag, TMEM address slot
    off += 16;
    L.total = off;
    L.stages = stages;
    return L;
}

// Most stages (up to 4) that fit; 0 if not even two do.
inline int mma_stages(int rb, int nb_tok) {
    for (int s = 4; s >= 2; --s)
        if (mma_layout(rb, nb_tok, s).total + 1024 <= MMA_SMEM_LIMIT) return s;
    return 0;
}

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

// Instruction descriptor: D s32, A s8 (the planes are 0..105), B s8, both
// K-major, M = 128, N = NB.
template <int NB>
constexpr uint32_t umma_idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(MMA_ROWS >> 4) << 24);
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

template <int NB>
__global__ void __launch_bounds__(MMA_THREADS, 1)
    k_qmv_q4k_mma(const QmvArgs a, const __grid_constant__ CUtensorMap tm, int n_tok, int stages) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool issuer_warp = warp == 8;
    const int r = tid & (MMA_ROWS - 1);  // workers: row of the tile (TMEM lane)
    const int h = (tid >> 7) & 1;        // workers: which half of the row's work
    const int rb = a.rb;
    const MmaLayout L = mma_layout(rb, NB, stages);
    uint8_t *bsm = smem + L.b;
    float *dxs = (float *)(smem + L.dx);
    int4 *bss = (int4 *)(smem + L.bs);
    uint8_t *raw = smem + L.raw;
    uint64_t *full = (uint64_t *)(smem + L.bar);
    uint64_t *empty = full + stages;
    uint64_t *a_full = empty + stages;      // [MMA_NA]
    uint64_t *mma_done = a_full + MMA_NA;   // [MMA_NA]
    uint64_t *d_free = mma_done + MMA_NA;   // [2]
    uint64_t *drain = d_free + 2;
    volatile int *abort = (volatile int *)(smem + L.flag);
    uint32_t *tslot = (uint32_t *)(smem + L.flag + 8);

    const int ntiles = (a.rows + MMA_ROWS - 1) / MMA_ROWS;
    const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nblk = my_tiles * rb;  // block items of this CTA
    const int J = 2 * nblk;          // half-block items

    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        for (int b = 0; b < MMA_NA; ++b) {
            mbar_init(&a_full[b], 8);
            mbar_init(&mma_done[b], 1);
        }
        mbar_init(&d_free[0], 8);
        mbar_init(&d_free[1], 8);
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, MMA_TMEM_COLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    auto issue_block = [&](int bi) {
        const int tl = bi / rb, k = bi - tl * rb;
        const int row0 = ((int)blockIdx.x + tl * (int)gridDim.x) * MMA_ROWS;
        uint64_t *b = &full[bi % stages];
        fence_proxy_async();
        mbar_arrive_expect_tx(b, MMA_RAW_BYTES);
        tma_load_2d(raw + (size_t)(bi % stages) * MMA_RAW_BYTES, &tm, k * 36, row0, b);
    };
    // the first raw block columns go out at once: weights do not depend on the previous kernel
    int issued = 0;
    if (issuer_warp && lane == 0)
        for (; issued < stages && issued < nblk; ++issued) issue_block(issued);

    // activations: codes into the UMMA layout (tokens >= n_tok are zero),
    // block scales and sub-block bsum pairs
    pdl_wait();
    {
        const uint8_t *xq = (const uint8_t *)a.xq;
        const int nchunk = NB * rb * 16;  // 16-byte chunks of codes
        for (int c = tid; c < nchunk; c += MMA_THREADS) {
            const int t = c / (rb * 16), rem = c - t * rb * 16, blk = rem >> 4, ch = rem & 15;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (t < n_tok) {
                const uint32_t *src = (const uint32_t *)(xq + ((size_t)t * rb + blk) * 292 + 4 + 16 * ch);
                v = make_uint4(src[0], src[1], src[2], src[3]);
            }
            const int s = ch >> 1, j = ch & 1;
            *(uint4 *)(bsm + ((size_t)(blk * 8 + s) * (NB / 8) + (t >> 3)) * 256 + j * 128 + (t & 7) * 16) = v;
        }
        for (int c = tid; c < NB * rb; c += MMA_THREADS) {
            const int t = c / rb, blk = c - t * rb;
            float d = 0.0f;
            int4 p = make_int4(0, 0, 0, 0);
            if (t < n_tok) {
                const uint8_t *sb = xq + ((size_t)t * rb + blk) * 292;
                d = *(const float *)sb;
                const int16_t *bs = (const int16_t *)(sb + 260);
                int w[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int lo = bs[4 * q] + bs[4 * q + 1], hi = bs[4 * q + 2] + bs[4 * q + 3];
                    w[q] = (lo & 0xffff) | (hi << 16);
                }
                p = make_int4(w[0], w[1], w[2], w[3]);
            }
            dxs[c] = d;
            bss[c] = p;
        }
    }
    pdl_trigger();
    fence_proxy_async();  // the codes are read by the tensor cores (async proxy)
    __syncthreads();

    if (issuer_warp) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_i8<NB>();
            const uint32_t b_base = smem_u32(bsm);
            for (int j = 0; j < J; ++j) {
                const int bi = j >> 1, q = j & 1, ab = j % MMA_NA, db = bi & 1;
                // a block's first MMAs overwrite accumulators whose epilogue (block bi - 2) is done
                if (q == 0 && bi >= 2 && !wait_or_abort(&d_free[db], (uint32_t)(((bi - 2) >> 1) & 1), abort, a.status))
                    break;
                if (!wait_or_abort(&a_full[ab], (uint32_t)((j / MMA_NA) & 1), abort, a.status)) break;
                tc_fence_after();
                const int k = bi % rb;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t bd = umma_desc(b_base + (uint32_t)((k * 8 + 4 * q + s) * NB * 32));
                    umma_i8_ts(tmem + (uint32_t)(db * 128 + (4 * q + s) * 16),
                               tmem + (uint32_t)(MMA_ACOL + ab * 32 + s * 8), bd, idesc, 0u);
                }
                umma_commit(&mma_done[ab]);
                // the block's raw stage, once every worker warp has read it, takes block bi + stages
                if (q == 1 && issued < nblk) {
                    if (!wait_or_abort(&empty[bi % stages], (uint32_t)((bi / stages) & 1), abort, a.status)) break;
                    issue_block(issued++);
                }
            }
            // drain: every MMA issued above, and every copy still in flight (bounded, even after an abort)
            umma_commit(drain);
            mbar_wait_bounded(drain, 0u, a.status, 5);
            for (int bi = issued - stages < 0 ? 0 : issued - stages; bi < issued; ++bi)
                mbar_wait_bounded(&full[bi % stages], (uint32_t)((bi / stages) & 1), a.status, 5);
        }
        __syncwarp();
    } else {
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const bool epi_thread = NB == 16 || h == 0;
        const int toff = NB == 16 ? 8 * h : 0;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        // scales of the block being unpacked and of the previous one (its epilogue)
        float cur_d = 0.0f, cur_dm = 0.0f, prev_d = 0.0f, prev_dm = 0.0f;
        uint32_t sc03 = 0, sc47 = 0, cur_m03 = 0, cur_m47 = 0;
        uint32_t psc03 = 0, psc47 = 0, prev_m03 = 0, prev_m47 = 0;

        auto epilogue = [&](int bi) {
            const int tl = bi / rb, k = bi - tl * rb;
            if (epi_thread) {
                int v[8][8];
                const uint32_t dcol = tmem + lane_base + (uint32_t)((bi & 1) * 128 + toff);
#pragma unroll
                for (int s = 0; s < 8; ++s) tmem_ld8(dcol + (uint32_t)(s * 16), v[s]);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    int isum = 0;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const int sc = (int)(((s < 4 ? psc03 : psc47) >> (8 * (s & 3))) & 0xffu);
                        isum += sc * v[s][i];
                    }
                    const int t = toff + i;
                    const int4 bs = bss[t * rb + k];
                    int msum = __dp2a_lo(bs.x, (int)prev_m03, 0);
                    msum = __dp2a_hi(bs.y, (int)prev_m03, msum);
                    msum = __dp2a_lo(bs.z, (int)prev_m47, msum);
                    msum = __dp2a_hi(bs.w, (int)prev_m47, msum);
                    const float dx = dxs[t * rb + k];
                    acc[i] = fmaf(prev_d * dx, (float)isum, acc[i]);
                    acc[i] = fmaf(-(prev_dm * dx), (float)msum, acc[i]);
                }
            }
            if (k == rb - 1) {  // the tile's last block: write its rows
                const int row = ((int)blockIdx.x + tl * (int)gridDim.x) * MMA_ROWS + r;
                if (epi_thread && row < a.rows) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int t = toff + i;
                        if (t < n_tok) {
                            const size_t o = (size_t)t * a.ldy + row;
                            a.y[o] = a.residual ? acc[i] + a.residual[o] : acc[i];
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
            }
        };
        auto shift_scales = [&]() {
            prev_d = cur_d;
            prev_dm = cur_dm;
            prev_m03 = cur_m03;
            prev_m47 = cur_m47;
            psc03 = sc03;
            psc47 = sc47;
        };

        bool ok = true;
        for (int j = 0; j < J; ++j) {
            const int bi = j >> 1, q = j & 1, ab = j % MMA_NA;
            if (q == 0 && !warp_wait_or_abort(&full[bi % stages], (uint32_t)((bi / stages) & 1), abort, a.status)) {
                ok = false;
                break;
            }
            // A buffer ab is free once the MMAs of half-block j - MMA_NA are done.
            // This is also the only wait on those MMAs before the epilogue of
            // block bi - 1 (at q == 1 it covers that block's last half-block):
            // waiting again after this warp's a_full arrival below could find
            // half-block j's MMAs already complete, one phase past the awaited
            // one, and the parity test would then wait for the phase after.
            if (j >= MMA_NA &&
                !warp_wait_or_abort(&mma_done[ab], (uint32_t)(((j - MMA_NA) / MMA_NA) & 1), abort, a.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint8_t *rw = raw + (size_t)(bi % stages) * MMA_RAW_BYTES + (size_t)r * 144;
            if (q == 0) {
                const uint4 hd = *(const uint4 *)rw;
                shift_scales();
                cur_d = h2f(hd.x);
                cur_dm = h2f(hd.x >> 16);
                sc03 = hd.y & 0x3f3f3f3fu;
                cur_m03 = hd.z & 0x3f3f3f3fu;
                sc47 = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
                cur_m47 = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
            }
            {
                // qs group g = 2q + h of row r: low nibbles are sub-block 2g, high 2g+1,
                // i.e. sub-blocks 2h and 2h + 1 of the half-block
                const int g = 2 * q + h;
                const uint4 qa = *(const uint4 *)(rw + 16 + 32 * g), qb = *(const uint4 *)(rw + 32 + 32 * g);
                const uint32_t acol = tmem + lane_base + (uint32_t)(MMA_ACOL + ab * 32 + 2 * h * 8);
                tmem_st8(acol, qa.x & 0x0f0f0f0fu, qa.y & 0x0f0f0f0fu, qa.z & 0x0f0f0f0fu, qa.w & 0x0f0f0f0fu,
                         qb.x & 0x0f0f0f0fu, qb.y & 0x0f0f0f0fu, qb.z & 0x0f0f0f0fu, qb.w & 0x0f0f0f0fu);
                tmem_st8(acol + 8, (qa.x >> 4) & 0x0f0f0f0fu, (qa.y >> 4) & 0x0f0f0f0fu, (qa.z >> 4) & 0x0f0f0f0fu,
                         (qa.w >> 4) & 0x0f0f0f0fu, (qb.x >> 4) & 0x0f0f0f0fu, (qb.y >> 4) & 0x0f0f0f0fu,
                         (qb.z >> 4) & 0x0f0f0f0fu, (qb.w >> 4) & 0x0f0f0f0fu);
                tmem_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[ab]);
                if (q == 1) mbar_arrive(&empty[bi % stages]);  // this warp is done with the raw stage
            }
            if (q == 1 && bi >= 1) {
                // block bi - 1: both half-blocks' MMAs were awaited above (j - 3 at
                // q == 0, j - 2 at this q == 1), before this warp's arrival
                epilogue(bi - 1);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_free[(bi - 1) & 1]);
            }
        }
        if (ok && nblk > 0) {
            // the last block: its two half-blocks' MMAs, then its epilogue
            const bool done =
                warp_wait_or_abort(&mma_done[(J - 2) % MMA_NA], (uint32_t)(((J - 2) / MMA_NA) & 1), abort, a.status) &&
                warp_wait_or_abort(&mma_done[(J - 1) % MMA_NA], (uint32_t)(((J - 1) / MMA_NA) & 1), abort, a.status);
            if (done) {
                shift_scales();
                tc_fence_after();
                epilogue(nblk - 1);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, MMA_TMEM_COLS);
    }
}

// 1: launched; 0: shape not supported by this kernel (caller falls back).
template <int NB>
static cudaError_t run_mma(const QmvArgs &a, int n_tok, int sm_count, cudaStream_t st, bool *launched) {
    *launched = false;
    const int stages = mma_stages(a.rb, NB);
    if (stages == 0) return cudaSuccess;
    const MmaLayout L = mma_layout(a.rb, NB, stages);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool opted[64] = {};
    if (dev >= 64 || !opted[dev]) {
        e = cudaFuncSetAttribute(k_qmv_q4k_mma<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM_LIMIT);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = true;
    }
    CUtensorMap tm;
    if (!encode_rows_u32(&tm, a.w0, a.row_stride, a.rows, 36, MMA_ROWS)) return cudaErrorInvalidValue;
    const int ntiles = (a.rows + MMA_ROWS - 1) / MMA_ROWS;
    const int grid = ntiles < sm_count ? ntiles : sm_count;
    const size_t smem = L.total > MMA_SMEM_MIN ? L.total : MMA_SMEM_MIN;
    *launched = true;
    return launch_pdl(k_qmv_q4k_mma<NB>, dim3(grid), dim3(MMA_THREADS), smem, st, a, tm, n_tok, stages);
}

bool q4k_mma_supported(int rb, int n_tok) {
    return n_tok >= 5 && n_tok <= 16 && mma_stages(rb, n_tok <= 8 ? 8 : 16) > 0;
}

cudaError_t launch_q4k_mma(const QmvArgs &a, int n_tok, int sm_count, cudaStream_t st) {
    bool launched = false;
    const cudaError_t e = n_tok <= 8 ? run_mma<8>(a, n_tok, sm_count, st, &launched)
                                     : run_mma<16>(a, n_tok, sm_count, st, &launched);
    if (e != cudaSuccess) return e;
    return launched ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace m27b
