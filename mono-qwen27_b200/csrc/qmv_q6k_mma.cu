// qmv_q6k_mma.cu — q6_K weights x 1..8 q8_K tokens on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in TMEM): ffn_down and
// lm_head of the speculative verify pass.
//
// Replaces, for the drafted tokens of a verify pass, the reference's
// per-token q6_K matvec (k_q6k_mv_q8_dp4a, src/mono27b_executor.cu:630-645,
// called once per token).  Result semantics are ggml's vec_dot_q6_K_q8_K:
// per super-block the integer sum
//     isum = sum_g sc_g * (dot(q_g, x_g) - 32 * bsum_g)     (16 groups of 16)
// with q the unsigned 6-bit codes and sc_g the signed 8-bit scales, then
// y += d * dx * isum in fp32.
//
// Mapping onto the tensor cores.  A kind::i8 MMA has K = 32: two 16-value
// groups with different scales.  Each 32-value slice of a block is
// multiplied twice, with A = the slice's codes with its second group zeroed
// and with its first group zeroed, so that every group gets its own
// accumulator D_g = dot(q_g, x_g) for all (row, token).  The tensor pipe has
// room for the doubled MMAs; the codes are unpacked once, and the zero halves
// of the A buffers are written once at the start.  The A operand lives in
// TMEM: thread r (TMEM lane r) unpacks weight row r.  The epilogue applies
// the scales and the -32 offset in integers (exactly ggml's sums) and the
// fp16 / fp32 block scales in fp32.
//
// Weights: the repacked rows of 848-byte tiles (ql[4][128] | qh[4][64] |
// scales[4][16] | d[4] per 4 blocks, qmv_q6k_tile.cuh).  Per block and
// 128-row tile the producer issues four 2-D TMA copies into one stage: the
// block's ql (128 bytes per row, 128-byte swizzle), qh (64 bytes, 64-byte
// swizzle), scales (16 bytes) and the tile's four d words (16 bytes).  The
// swizzles spread the unpacking threads' 16-byte reads of rows 128 / 64
// bytes apart over all banks.  No multicast.
//
// Pipeline (one CTA of 15 warps per SM, 512 TMEM columns), synchronised by
// mbarriers only, every wait bounded (2 s; a timeout records status 5 and
// raises the CTA's abort flag, every role leaves its loop, the issuing
// threads wait for their own copies and MMAs, the CTA frees its TMEM):
//   * warp 13 streams the weights (a stage refilled once every unpacking and
//     epilogue warp has handed it back);
//   * warps 12 and 14 issue the MMAs of the first / second half of every
//     block (4 slices x 2 groups = 8 MMAs, M = 128, N = 8, K = 32);
//   * warps 0-3 unpack a half-block (ql nibble | qh bits << 4, four codes
//     per 32-bit word) into one of four A buffers;
//   * warps 4-11 run the epilogue of a half-block (tcgen05.ld of its 8 group
//     accumulators, integer scale sums; per block the fp32 combine), two
//     warps per TMEM lane quarter, 4 tokens each.
// TMEM: a ring of 4 half-block accumulator buffers (8 groups x 8 tokens = 64
// columns) and a ring of 4 half-block A buffers (4 slices x 2 x 8 columns).
//
// K split (few row tiles, long rows: ffn_down): ks ranges of blocks per tile,
// unit u = tile * ks + range, the grid a multiple of ks so that all units of
// a CTA lie in one range and the CTA stages only that range's activations;
// partial sums part[((tile * ks + range) * 8 + token) * 128 + row], the
// epilogue warp arriving last at count[tile * 8 + warp] adds its 32-row
// slice over the ranges in range order (deterministic).
#include "tc05.cuh"
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"
#include "qmv_q6k_tile.cuh"

namespace m27b {

constexpr int Q6M_NB = 8;      // MMA N: tokens per launch
constexpr int Q6M_ROWS = 128;  // MMA M: weight rows per tile
constexpr int Q6M_UNPACK = 4, Q6M_EPI = 8;
constexpr int Q6M_ISSUER = Q6M_UNPACK + Q6M_EPI, Q6M_PRODUCER = Q6M_ISSUER + 1, Q6M_ISSUER2 = Q6M_PRODUCER + 1;
constexpr int Q6M_THREADS = (Q6M_ISSUER2 + 1) * 32;
constexpr int Q6M_NA = 4, Q6M_ND = 4;          // A / accumulator ring slots (half-blocks)
constexpr int Q6M_HCOLS = 8 * Q6M_NB;          // accumulator columns of a half-block (8 groups)
constexpr int Q6M_ACOL = Q6M_ND * Q6M_HCOLS;   // first A column
constexpr int Q6M_TCOLS = 512;                 // Q6M_ACOL + Q6M_NA * 64
static_assert(Q6M_ACOL + Q6M_NA * 64 == Q6M_TCOLS, "TMEM plan");
// one stage: ql | qh | scales | d of 128 rows of one block
constexpr int Q6M_QL = 0, Q6M_QH = 128 * 128, Q6M_SC = Q6M_QH + 128 * 64, Q6M_D = Q6M_SC + 128 * 16;
constexpr int Q6M_RAW = Q6M_D + 128 * 16;  // 28672 bytes (a multiple of 1024: swizzle alignment)
constexpr int Q6M_MAX_KS = 8;

struct Q6mLayout {
    size_t b, dx, bs, raw, bar, flag, total;
};

// Shared memory for nbmax blocks of staged activations and `stages` stages.
__host__ __device__ inline Q6mLayout q6m_layout(int nbmax, int stages) {
    Q6mLayout L;
    size_t off = 0;
    L.b = off;
    off += (size_t)nbmax * 8 * Q6M_NB * 32;  // codes, UMMA K-major layout
    L.dx = off;
    off += (size_t)Q6M_NB * nbmax * 4;       // block scales
    L.bs = off;
    off += (size_t)Q6M_NB * nbmax * 32;      // 16 bsums per (token, block)
    off = (off + 1023) & ~(size_t)1023;
    L.raw = off;
    off += (size_t)stages * Q6M_RAW;
    L.bar = off;  // full, empty [stages]; a_full, mma_done [NA]; hb_done, d_free [ND]; drain
    off += (size_t)(2 * stages + 2 * Q6M_NA + 2 * Q6M_ND + 1) * 8;
    L.flag = off;  // abort flag, TMEM address slot
    off += 16;
    L.total = off;
    return L;
}

inline int q6m_stages(int nbmax) {
    for (int s = 4; s >= 2; --s)
        if (q6m_layout(nbmax, s).total + 1024 + 1024 <= MMA_SMEM_LIMIT) return s;  // + alignment slack
    return 0;
}

M27B_DI void tmem_st4(uint32_t taddr, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v0), "r"(v1), "r"(v2),
                 "r"(v3)
                 : "memory");
}

// Codes of slice m (0..3) of a half-block, four per word, from the half's ql
// words (l0: values 0..31 of the half's first 32 ql bytes, l1: the next 32)
// and qh words h: q = ql nibble | two qh bits << 4.
M27B_DI uint32_t q6_code_word(uint32_t l0, uint32_t l1, uint32_t h, int m) {
    switch (m) {
    case 0: return (l0 & 0x0f0f0f0fu) | ((h & 0x03030303u) << 4);
    case 1: return (l1 & 0x0f0f0f0fu) | ((h & 0x0c0c0c0cu) << 2);
    case 2: return ((l0 >> 4) & 0x0f0f0f0fu) | (h & 0x30303030u);
    default: return ((l1 >> 4) & 0x0f0f0f0fu) | ((h >> 2) & 0x30303030u);
    }
}

template <int EPI>
__global__ void __launch_bounds__(Q6M_THREADS, 1)
    k_qmv_q6k_mma(const QmvArgs a, const __grid_constant__ CUtensorMap tm_ql, const __grid_constant__ CUtensorMap tm_qh,
                  const __grid_constant__ CUtensorMap tm_sc, const __grid_constant__ CUtensorMap tm_d, int n_tok,
                  int stages, int nbmax, const MmaSplit sp) {
    constexpr int NB = Q6M_NB;
    extern __shared__ __align__(1024) uint8_t q6m_smem_raw[];
    // the dynamic shared memory base is 1024-aligned here (swizzled stages)
    uint8_t *smem = (uint8_t *)(((uintptr_t)q6m_smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = a.rb;
    const Q6mLayout L = q6m_layout(nbmax, stages);
    uint8_t *bsm = smem + L.b;
    float *dxs = (float *)(smem + L.dx);
    uint32_t *bss = (uint32_t *)(smem + L.bs);  // [token][nbmax][8] bsum pairs
    uint8_t *raw = smem + L.raw;
    uint64_t *full = (uint64_t *)(smem + L.bar);
    uint64_t *empty = full + stages;
    uint64_t *a_full = empty + stages;       // [NA]
    uint64_t *mma_done = a_full + Q6M_NA;    // [NA]: a half-block's MMAs (its A buffer is free)
    uint64_t *hb_done = mma_done + Q6M_NA;   // [ND]: a half-block's accumulators are final
    uint64_t *d_free = hb_done + Q6M_ND;     // [ND]: read by the epilogue
    uint64_t *drain = d_free + Q6M_ND;
    volatile int *abort = (volatile int *)(smem + L.flag);
    uint32_t *tslot = (uint32_t *)(smem + L.flag + 8);

    // this CTA's units: u = blockIdx.x + i * gridDim.x, tile u / ks, range
    // u % ks = blockIdx.x % ks (gridDim.x is a multiple of ks)
    const int ks = sp.ks, range = (int)blockIdx.x % ks;
    const int k0 = range * rb / ks, nbr = (range + 1) * rb / ks - k0;  // the range's blocks
    const int ntiles = (a.rows + Q6M_ROWS - 1) / Q6M_ROWS, nunits = ntiles * ks;
    const int my_units = (int)blockIdx.x < nunits ? (nunits - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nblk = my_units * nbr;  // block items
    const int J = 2 * nblk;           // half-block items
    auto tile_of = [&](int bi) { return ((int)blockIdx.x + (bi / nbr) * (int)gridDim.x) / ks; };

    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], Q6M_UNPACK + Q6M_EPI);
        }
        for (int b = 0; b < Q6M_NA; ++b) {
            mbar_init(&a_full[b], Q6M_UNPACK);
            mbar_init(&mma_done[b], 1);
        }
        for (int b = 0; b < Q6M_ND; ++b) {
            mbar_init(&hb_done[b], 1);
            mbar_init(&d_free[b], Q6M_EPI);
        }
        mbar_init(drain, 2);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, Q6M_TCOLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    auto issue_block = [&](int bi) {
        const int kb = k0 + bi % nbr, t4 = kb >> 2, b4 = kb & 3, row0 = tile_of(bi) * Q6M_ROWS;
        uint8_t *st = raw + (size_t)(bi % stages) * Q6M_RAW;
        uint64_t *bar = &full[bi % stages];
        mbar_arrive_expect_tx(bar, Q6M_RAW);
        const int x = t4 * (Q6T_TILE / 4);
        tma_load_2d(st + Q6M_QL, &tm_ql, x + 32 * b4, row0, bar);
        tma_load_2d(st + Q6M_QH, &tm_qh, x + 128 + 16 * b4, row0, bar);
        tma_load_2d(st + Q6M_SC, &tm_sc, x + 192 + 4 * b4, row0, bar);
        tma_load_2d(st + Q6M_D, &tm_d, x + 208, row0, bar);
    };
    // the first stages go out at once: weights do not depend on the previous kernel
    int issued = 0;
    if (warp == Q6M_PRODUCER && lane == 0)
        for (; issued < stages && issued < nblk; ++issued) issue_block(issued);
    // the zero halves of the A buffers: slice m of buffer ab occupies columns
    // ACOL + 64 ab + 16 m + [0, 16): codes of the first group then zeros, zeros
    // then codes of the second group
    if (warp < Q6M_UNPACK) {
        const uint32_t lb = (uint32_t)(32 * warp) << 16;
        for (int c = 0; c < Q6M_NA * 4; ++c) {
            tmem_st4(tmem + lb + (uint32_t)(Q6M_ACOL + 16 * c + 4), 0u, 0u, 0u, 0u);
            tmem_st4(tmem + lb + (uint32_t)(Q6M_ACOL + 16 * c + 8), 0u, 0u, 0u, 0u);
        }
        tmem_wait_st();
    }

    // activations of this CTA's range: the codes into the UMMA layout, the
    // block scales to dxs, the bsum words as they are; tokens >= n_tok zero
    pdl_wait();
    gather_tiles<2, NB>(
        n_tok, nbr, bsm, [&](int t, int kl) { return (const unsigned *)a.xq + ((size_t)t * rb + k0 + kl) * Q8K_WORDS; },
        [&](int t, int kl, unsigned v) { dxs[t * nbmax + kl] = __uint_as_float(v); },
        [&](int t, int kl, int m, unsigned v) { bss[(t * nbmax + kl) * 8 + m] = v; });
    pdl_trigger();
    fence_proxy_async();  // the codes are read by the tensor cores (async proxy)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == Q6M_ISSUER || warp == Q6M_ISSUER2) {
        if (lane == 0) {
            const int q = warp == Q6M_ISSUER ? 0 : 1;
            constexpr uint32_t idesc = umma_idesc_i8<NB>();
            const uint32_t b_base = smem_u32(bsm);
            for (int bi = 0; bi < nblk; ++bi) {
                const int j = 2 * bi + q, ab = j % Q6M_NA, db = j % Q6M_ND;
                // the accumulators of half-block j - ND have been read
                if (j >= Q6M_ND && !wait_or_abort(&d_free[db], (uint32_t)(((j - Q6M_ND) / Q6M_ND) & 1), abort, a.status))
                    break;
                if (!wait_or_abort(&a_full[ab], (uint32_t)((j / Q6M_NA) & 1), abort, a.status)) break;
                tc_fence_after();
                const int kl = bi % nbr;
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const uint64_t bd = umma_desc(b_base + (uint32_t)((kl * 8 + 4 * q + m) * NB * 32));
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        umma_i8_ts(tmem + (uint32_t)(db * Q6M_HCOLS + (2 * m + e) * NB),
                                   tmem + (uint32_t)(Q6M_ACOL + ab * 64 + 16 * m + 8 * e), bd, idesc, 0u);
                }
                umma_commit(&mma_done[ab]);
                umma_commit(&hb_done[db]);
            }
            umma_commit(drain);
            mbar_wait_bounded(drain, 0u, a.status, 5);
        }
        __syncwarp();
    } else if (warp == Q6M_PRODUCER) {
        if (lane == 0) {
            for (; issued < nblk; ++issued) {
                const int bi = issued;
                if (!wait_or_abort(&empty[bi % stages], (uint32_t)((bi / stages - 1) & 1), abort, a.status)) break;
                issue_block(bi);
            }
            // every copy in flight lands before the CTA's shared memory is released (bounded)
            for (int bi = issued - stages < 0 ? 0 : issued - stages; bi < issued; ++bi)
                mbar_wait_bounded(&full[bi % stages], (uint32_t)((bi / stages) & 1), a.status, 5);
        }
        __syncwarp();
    } else if (warp < Q6M_UNPACK) {
        // A operand: thread r = TMEM lane r = row r of the tile
        const int r = tid;
        const uint32_t lb = (uint32_t)(32 * warp) << 16;
        const int sw_ql = r & 7, sw_qh = (r >> 1) & 3;  // swizzle of row r's 16-byte chunks
        // a whole block per pass (both half-blocks into their A buffers): one
        // tcgen05.wait::st per block
        for (int bi = 0; bi < nblk; ++bi) {
            const int j0 = 2 * bi, ab0 = j0 % Q6M_NA, ab1 = (j0 + 1) % Q6M_NA;
            if (!warp_wait_or_abort(&full[bi % stages], (uint32_t)((bi / stages) & 1), abort, a.status)) break;
            if (j0 >= Q6M_NA &&
                !warp_wait_or_abort(&mma_done[ab0], (uint32_t)(((j0 - Q6M_NA) / Q6M_NA) & 1), abort, a.status))
                break;
            if (j0 + 1 >= Q6M_NA &&
                !warp_wait_or_abort(&mma_done[ab1], (uint32_t)(((j0 + 1 - Q6M_NA) / Q6M_NA) & 1), abort, a.status))
                break;
            tc_fence_after();
            const uint8_t *st = raw + (size_t)(bi % stages) * Q6M_RAW;
            const uint8_t *qlr = st + Q6M_QL + r * 128, *qhr = st + Q6M_QH + r * 64;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                // half q: ql bytes 64q .. 64q + 63 (chunks 4q .. 4q + 3), qh bytes 32q .. 32q + 31
                uint4 l[4], h[2];
#pragma unroll
                for (int c = 0; c < 4; ++c) l[c] = *(const uint4 *)(qlr + 16 * ((4 * q + c) ^ sw_ql));
#pragma unroll
                for (int c = 0; c < 2; ++c) h[c] = *(const uint4 *)(qhr + 16 * ((2 * q + c) ^ sw_qh));
                const uint32_t acol = tmem + lb + (uint32_t)(Q6M_ACOL + (q ? ab1 : ab0) * 64);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    // values 32 m + [0, 16) of the half: ql bytes [0, 16) (or [32, 48)), qh bytes [0, 16)
                    const uint4 a0 = l[0], a1 = l[1], b0 = l[2], b1 = l[3];
                    tmem_st4(acol + 16 * m, q6_code_word(a0.x, b0.x, h[0].x, m), q6_code_word(a0.y, b0.y, h[0].y, m),
                             q6_code_word(a0.z, b0.z, h[0].z, m), q6_code_word(a0.w, b0.w, h[0].w, m));
                    tmem_st4(acol + 16 * m + 12, q6_code_word(a1.x, b1.x, h[1].x, m),
                             q6_code_word(a1.y, b1.y, h[1].y, m), q6_code_word(a1.z, b1.z, h[1].z, m),
                             q6_code_word(a1.w, b1.w, h[1].w, m));
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[ab0]);
                mbar_arrive(&a_full[ab1]);
                mbar_arrive(&empty[bi % stages]);  // this warp is done with the stage
            }
        }
    } else {
        // epilogue: warp 4 + 4 th + quarter, thread lane of that quarter = row
        // r of the tile, tokens [4 th, 4 th + 4)
        constexpr int TPT = NB / 2;
        const int e = warp - Q6M_UNPACK, quarter = e & 3, th = e >> 2;
        const int r = 32 * quarter + lane, toff = th * TPT;
        const uint32_t lb = (uint32_t)(32 * quarter) << 16;
        float acc[TPT];
        int isum[TPT], msum[TPT];
#pragma unroll
        for (int i = 0; i < TPT; ++i) {
            acc[i] = 0.0f;
            isum[i] = 0;
            msum[i] = 0;
        }
        unsigned long long best[TPT];
#pragma unroll
        for (int i = 0; i < TPT; ++i) best[i] = 0ull;
        uint4 scw = make_uint4(0u, 0u, 0u, 0u);
        float dw = 0.0f;
        for (int j = 0; j < J; ++j) {
            const int bi = j >> 1, q = j & 1, db = j % Q6M_ND, kl = bi % nbr;
            if (q == 0) {
                // row r's 16 scales and the block's d, read before the stage is handed back
                if (!warp_wait_or_abort(&full[bi % stages], (uint32_t)((bi / stages) & 1), abort, a.status)) break;
                const uint8_t *st = raw + (size_t)(bi % stages) * Q6M_RAW;
                scw = *(const uint4 *)(st + Q6M_SC + r * 16);
                dw = h2f((uint16_t)*(const uint32_t *)(st + Q6M_D + r * 16 + 4 * ((k0 + kl) & 3)));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[bi % stages]);
            }
            if (!warp_wait_or_abort(&hb_done[db], (uint32_t)((j / Q6M_ND) & 1), abort, a.status)) break;
            tc_fence_after();
            int v[8][TPT];
            const uint32_t dcol = tmem + lb + (uint32_t)(db * Q6M_HCOLS + toff);
#pragma unroll
            for (int g = 0; g < 8; ++g) tmem_ld4(dcol + (uint32_t)(g * NB), v[g]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[db]);
            // the half's scales: groups 8q .. 8q + 7 = bytes of words 2q, 2q + 1
            const uint32_t s0 = q ? scw.z : scw.x, s1 = q ? scw.w : scw.y;
#pragma unroll
            for (int i = 0; i < TPT; ++i) {
                int is = isum[i];
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const int sc = (int)(int8_t)(((g < 4 ? s0 : s1) >> (8 * (g & 3))) & 0xffu);
                    is += sc * v[g][i];
                }
                isum[i] = is;
                const uint4 bp = *(const uint4 *)(bss + ((toff + i) * nbmax + kl) * 8 + 4 * q);
                int ms = msum[i];
                ms = __dp2a_lo((int)bp.x, (int)s0, ms);
                ms = __dp2a_hi((int)bp.y, (int)s0, ms);
                ms = __dp2a_lo((int)bp.z, (int)s1, ms);
                ms = __dp2a_hi((int)bp.w, (int)s1, ms);
                msum[i] = ms;
            }
            if (q == 0) continue;
            // block done: fp32 combine
#pragma unroll
            for (int i = 0; i < TPT; ++i) {
                acc[i] = fmaf(dw * dxs[(toff + i) * nbmax + kl], (float)(isum[i] - 32 * msum[i]), acc[i]);
                isum[i] = 0;
                msum[i] = 0;
            }
            if (kl != nbr - 1) continue;
            // the unit's last block
            const int tile = tile_of(bi), row = tile * Q6M_ROWS + r;
            bool write = true;
            if (ks > 1) {
                float *pt = sp.part + ((size_t)(tile * ks + range) * NB + toff) * Q6M_ROWS + r;
#pragma unroll
                for (int i = 0; i < TPT; ++i) pt[(size_t)i * Q6M_ROWS] = acc[i];
                __threadfence();
                __syncwarp();
                unsigned prev = 0u;
                unsigned *cnt = sp.count + (size_t)tile * 8 + e;
                if (lane == 0) prev = atomicAdd(cnt, 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                write = prev == (unsigned)(ks - 1);
                if (write) {
                    if (lane == 0) *cnt = 0u;
                    __threadfence();
#pragma unroll
                    for (int i = 0; i < TPT; ++i) {
                        float s = 0.0f;
                        for (int q2 = 0; q2 < ks; ++q2)
                            s += q2 == range ? acc[i]
                                             : __ldcg(sp.part + ((size_t)(tile * ks + q2) * NB + toff + i) * Q6M_ROWS + r);
                        acc[i] = s;
                    }
                }
            }
            if (write && row < a.rows) {
#pragma unroll
                for (int i = 0; i < TPT; ++i) {
                    const int t = toff + i;
                    if (t < n_tok) {
                        const size_t o = (size_t)t * a.ldy + row;
                        if constexpr (EPI == EPI_ARGMAX) {
                            if (a.y) a.y[o] = acc[i];
                            const unsigned long long key = argmax_key(acc[i], (uint32_t)row + a.row_offset);
                            best[i] = key > best[i] ? key : best[i];
                        } else {
                            a.y[o] = a.residual ? acc[i] + a.residual[o] : acc[i];
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < TPT; ++i) acc[i] = 0.0f;
        }
        if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
            for (int i = 0; i < TPT; ++i) {
                unsigned long long k = best[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
                    k = k2 > k ? k2 : k;
                }
                if (lane == 0 && toff + i < n_tok && k != 0ull) atomicMax(a.best + toff + i, k);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Q6M_TCOLS);
    }
}

// K ranges per tile: 1 when the tiles fill the SMs, else the most (at most
// Q6M_MAX_KS, ranges of at least 2 blocks) that keep one unit per SM.
static int q6m_ks(int ntiles, int rb, int sm_count) {
    if (ntiles >= sm_count) return 1;
    int best = 1;
    for (int k = 2; k <= Q6M_MAX_KS; ++k)
        if (rb / k >= 2 && ntiles * k <= sm_count) best = k;
    return best;
}

// K ranges of a launch over `rows` x rb blocks (split: with scratch).
static int q6m_plan_ks(int rows, int rb, bool split, int sm_count) {
    return split ? q6m_ks((rows + Q6M_ROWS - 1) / Q6M_ROWS, rb, sm_count) : 1;
}

// Whether the kernel serves n_tok tokens over rows x rb blocks (the staged
// activations of a CTA's K range and two stages fit its shared memory).
bool q6k_mma_supported(int rows, int rb, int n_tok, bool split, int sm_count) {
    if (n_tok < 1 || n_tok > Q6M_NB || rb < 1 || rows < 1) return false;
    const int ks = q6m_plan_ks(rows, rb, split, sm_count);
    return q6m_stages((rb + ks - 1) / ks) > 0;
}

// Scratch of the K-split launch (an upper bound over the splits it picks).
size_t q6k_mma_part_floats(int rows) {
    const int ntiles = (rows + Q6M_ROWS - 1) / Q6M_ROWS;
    return (size_t)ntiles * Q6M_MAX_KS * Q6M_NB * Q6M_ROWS;
}
size_t q6k_mma_count_words(int rows) { return (size_t)((rows + Q6M_ROWS - 1) / Q6M_ROWS) * 8; }

// epi: EPI_STORE (y, optional residual) or EPI_ARGMAX (a.best, optional
// logits in a.y).  part / count: K-split scratch (null: no split).
cudaError_t launch_q6k_mma(const QmvArgs &a, int n_tok, int epi, float *part, unsigned *count, int sm_count,
                           cudaStream_t st) {
    if (n_tok < 1 || n_tok > Q6M_NB || (epi != EPI_STORE && epi != EPI_ARGMAX)) return cudaErrorInvalidValue;
    const int ntiles = (a.rows + Q6M_ROWS - 1) / Q6M_ROWS;
    const int ks = q6m_plan_ks(a.rows, a.rb, part && count, sm_count);
    const int nbmax = (a.rb + ks - 1) / ks;
    const int stages = q6m_stages(nbmax);
    if (stages == 0) return cudaErrorInvalidValue;
    const Q6mLayout L = q6m_layout(nbmax, stages);
    size_t smem = L.total + 1024;  // + the base's alignment
    if (smem < MMA_SMEM_MIN) smem = MMA_SMEM_MIN;
    auto kern = epi == EPI_ARGMAX ? k_qmv_q6k_mma<EPI_ARGMAX> : k_qmv_q6k_mma<EPI_STORE>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool opted[2][64] = {};
    bool &op = opted[epi == EPI_ARGMAX][dev < 64 ? dev : 0];
    if (dev >= 64 || !op) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM_LIMIT);
        if (e != cudaSuccess) return e;
        if (dev < 64) op = true;
    }
    CUtensorMap tq, th, ts, td;
    if (!encode_rows_u32(&tq, a.w0, a.row_stride, a.rows, 32, Q6M_ROWS, 128) ||
        !encode_rows_u32(&th, a.w0, a.row_stride, a.rows, 16, Q6M_ROWS, 64) ||
        !encode_rows_u32(&ts, a.w0, a.row_stride, a.rows, 4, Q6M_ROWS) ||
        !encode_rows_u32(&td, a.w0, a.row_stride, a.rows, 4, Q6M_ROWS))
        return cudaErrorInvalidValue;
    const int units = ntiles * ks;
    const int grid = ks > 1 ? units : (units < sm_count ? units : sm_count);
    return launch_pdl(kern, dim3(grid), dim3(Q6M_THREADS), smem, st, a, tq, th, ts, td, n_tok, stages, nbmax,
                      MmaSplit{part, count, ks});
}

}  // namespace m27b
