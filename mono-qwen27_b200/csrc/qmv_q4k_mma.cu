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
// K=32 is exactly one q4_K sub-block.  The 6-bit scale cannot multiply the
// 4-bit weights inside an 8-bit operand (up to 945), so each sub-block is
// split into two 8-bit planes, q4 * (sc >> 3) and q4 * (sc & 7) (at most 105:
// a plain 32-bit multiply of four packed nibbles by the small factor forms
// them without carries between bytes).  The 16 MMAs of a super-block (8
// sub-blocks x 2 planes) accumulate into two TMEM accumulators D_hi, D_lo,
// and isum = 8 * D_hi + D_lo exactly.  The min term uses dp2a against the
// activation's bsums on the CUDA cores.
//
// Pipeline per CTA (one 128-row tile at a time, persistent over tiles; one
// CTA per SM):
//   * TMA streams one raw 128-row x 144-byte block column per stage (2-D
//     tensor map, no multicast) into a ring of stages;
//   * the activations (all K, all tokens) are staged once in the canonical
//     K-major no-swizzle UMMA layout, with their scales and bsum pairs;
//   * work advances in half-blocks (4 sub-blocks): all 256 threads unpack a
//     half-block into one of two A buffers (32 KB each: 4 sub-blocks x 2
//     planes x 128 rows x 32 bytes), one thread issues its 8 MMAs and
//     commits them to that buffer's mbarrier; the next half-block is
//     unpacked into the other buffer meanwhile;
//   * D accumulators are double-buffered per block: the epilogue of block b
//     (tcgen05.ld of D_hi / D_lo, one row per thread, eight tokens per
//     thread) runs while block b + 1 is in the tensor cores.
// Every wait is bounded (2 s); a timeout records status 5, the CTA leaves
// together, waits (bounded) for its own copies and MMAs, frees its TMEM and
// returns.
#include "qmv_blk.cuh"
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"

namespace m27b {

constexpr int MMA_ROWS = 128;
constexpr int MMA_THREADS = 256;
constexpr int MMA_RAW_BYTES = MMA_ROWS * 144;  // one TMA box: 128 rows x one q4_K block
constexpr int MMA_ABUF = 8 * 4096;             // 4 sub-blocks x 2 planes x 4 KB
constexpr int MMA_TMEM_COLS = 64;              // 2 blocks x (D_hi, D_lo) x 16 columns
constexpr size_t MMA_SMEM_LIMIT = 227 * 1024;

struct MmaLayout {
    size_t b, dx, bs, raw, bar, tslot, total;
    int stages;
};

// Shared memory plan for K = 256 * rb values and an MMA N of nb_tok (8 or 16).
__host__ __device__ inline MmaLayout mma_layout(int rb, int nb_tok, int stages) {
    MmaLayout L;
    size_t off = 2 * (size_t)MMA_ABUF;                       // two A buffers
    L.b = off;
    off += (size_t)rb * 8 * nb_tok * 32;                     // codes, UMMA layout
    L.dx = off;
    off += (size_t)nb_tok * rb * 4;                          // block scales
    L.bs = off;
    off += (size_t)nb_tok * rb * 16;                         // bsum pairs
    off = (off + 127) & ~(size_t)127;
    L.raw = off;
    off += (size_t)stages * MMA_RAW_BYTES;
    L.bar = off;
    off += (size_t)(stages + 2) * 8;
    L.tslot = off;
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

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, s8 x s8 -> s32, one thread.
M27B_DI void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
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

template <int NB>
__global__ void __launch_bounds__(MMA_THREADS, 1)
    k_qmv_q4k_mma(const QmvArgs a, const __grid_constant__ CUtensorMap tm, int n_tok, int stages) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (MMA_ROWS - 1);  // row of the tile (TMEM lane)
    const int h = tid >> 7;              // which half of the work on that row
    const int rb = a.rb;
    const MmaLayout L = mma_layout(rb, NB, stages);
    uint8_t *abuf = smem;
    uint8_t *bsm = smem + L.b;
    float *dxs = (float *)(smem + L.dx);
    int4 *bss = (int4 *)(smem + L.bs);
    uint8_t *raw = smem + L.raw;
    uint64_t *full = (uint64_t *)(smem + L.bar);
    uint64_t *mma_bar = full + stages;  // [2]: one per A buffer
    uint32_t *tslot = (uint32_t *)(smem + L.tslot);

    const int ntiles = (a.rows + MMA_ROWS - 1) / MMA_ROWS;
    const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nblk = my_tiles * rb;  // block items of this CTA
    const int J = 2 * nblk;          // half-block items

    if (tid == 0) {
        for (int s = 0; s < stages + 2; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, MMA_TMEM_COLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    // raw block columns go out first: the weights do not depend on the previous kernel
    auto issue_block = [&](int bi) {
        const int tl = bi / rb, k = bi - tl * rb;
        const int row0 = ((int)blockIdx.x + tl * (int)gridDim.x) * MMA_ROWS;
        uint64_t *b = &full[bi % stages];
        fence_proxy_async();
        mbar_arrive_expect_tx(b, MMA_RAW_BYTES);
        tma_load_2d(raw + (size_t)(bi % stages) * MMA_RAW_BYTES, &tm, k * 36, row0, b);
    };
    int issued = 0;
    if (tid == 0)
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

    constexpr uint32_t idesc = umma_idesc_i8<NB>();
    const uint32_t a_base = smem_u32(abuf), b_base = smem_u32(bsm);
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const bool epi_thread = NB == 16 || h == 0;

    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    // scales of the block being unpacked and of the previous one (its epilogue)
    float cur_d = 0.0f, cur_dm = 0.0f, prev_d = 0.0f, prev_dm = 0.0f;
    uint32_t cur_m03 = 0, cur_m47 = 0, prev_m03 = 0, prev_m47 = 0, sc03 = 0, sc47 = 0;

    // epilogue of block item bi (its MMAs have completed)
    auto epilogue = [&](int bi) {
        const int tl = bi / rb, k = bi - tl * rb;
        if (epi_thread) {
            int dh[8], dl[8];
            const uint32_t col = (uint32_t)((bi & 1) * 32 + (NB == 16 ? 8 * h : 0));
            tmem_ld8(tmem + lane_base + col, dh);
            tmem_ld8(tmem + lane_base + col + 16, dl);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int t = (NB == 16 ? 8 * h : 0) + i;
                const int4 bs = bss[t * rb + k];
                int msum = __dp2a_lo(bs.x, (int)prev_m03, 0);
                msum = __dp2a_hi(bs.y, (int)prev_m03, msum);
                msum = __dp2a_lo(bs.z, (int)prev_m47, msum);
                msum = __dp2a_hi(bs.w, (int)prev_m47, msum);
                const int isum = dh[i] * 8 + dl[i];
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
                    const int t = (NB == 16 ? 8 * h : 0) + i;
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

    bool ok = true;
    int waited = 0;  // block items whose raw stage has been waited for
    int j = 0;
    for (; j < J; ++j) {
        const int bi = j >> 1, q = j & 1, ab = j & 1;
        bool landed = true;
        if (q == 0) {
            landed = mbar_wait_bounded(&full[bi % stages], (uint32_t)((bi / stages) & 1), a.status, 5);
            if (landed) ++waited;
        }
        if (j >= 2) landed = mbar_wait_bounded(&mma_bar[ab], (uint32_t)(((j - 2) >> 1) & 1), a.status, 5) && landed;
        // unpack qs group g = 2q + h of row r: low nibbles are sub-block 2g, high 2g+1
        const uint8_t *rw = raw + (size_t)(bi % stages) * MMA_RAW_BYTES + (size_t)r * 144;
        if (q == 0) {
            const uint4 hd = *(const uint4 *)rw;
            prev_d = cur_d;
            prev_dm = cur_dm;
            prev_m03 = cur_m03;
            prev_m47 = cur_m47;
            cur_d = h2f(hd.x);
            cur_dm = h2f(hd.x >> 16);
            sc03 = hd.y & 0x3f3f3f3fu;
            cur_m03 = hd.z & 0x3f3f3f3fu;
            sc47 = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
            cur_m47 = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
        }
        {
            const int g = 2 * q + h;
            const uint4 qa = *(const uint4 *)(rw + 16 + 32 * g), qb = *(const uint4 *)(rw + 32 + 32 * g);
            const uint32_t nib[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const uint32_t scw = g < 2 ? sc03 : sc47;
            const int sh = 16 * (g & 1);
            uint8_t *dst0 = abuf + (size_t)ab * MMA_ABUF + (size_t)(r >> 3) * 256 + (r & 7) * 16;
#pragma unroll
            for (int part = 0; part < 2; ++part) {  // 0: low nibbles (sub-block 2g), 1: high (2g+1)
                const uint32_t sc = (scw >> (sh + 8 * part)) & 0xffu;
                const uint32_t fh = sc >> 3, fl = sc & 7u;
                const int sl = 2 * h + part;  // sub-block within the half-block
                uint32_t qv[8];
#pragma unroll
                for (int w = 0; w < 8; ++w) qv[w] = part ? (nib[w] >> 4) & 0x0f0f0f0fu : nib[w] & 0x0f0f0f0fu;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    *(uint4 *)(dst0 + (size_t)(0 * 4 + sl) * 4096 + c * 128) =
                        make_uint4(qv[4 * c] * fh, qv[4 * c + 1] * fh, qv[4 * c + 2] * fh, qv[4 * c + 3] * fh);
                    *(uint4 *)(dst0 + (size_t)(1 * 4 + sl) * 4096 + c * 128) =
                        make_uint4(qv[4 * c] * fl, qv[4 * c + 1] * fl, qv[4 * c + 2] * fl, qv[4 * c + 3] * fl);
                }
            }
        }
        if (q == 1 && bi >= 1) {
            tc_fence_after();
            epilogue(bi - 1);
        }
        fence_proxy_async();
        tc_fence_before();
        ok = __syncthreads_and(landed) != 0;
        if (!ok) break;
        if (tid == 0) {
            tc_fence_after();
            if (q == 1 && issued < nblk) issue_block(issued++);  // this raw stage has been read
            const uint32_t d_hi = tmem + (uint32_t)((bi & 1) * 32), d_lo = d_hi + 16;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = bi % rb;
                const uint64_t bd = umma_desc(b_base + (uint32_t)((k * 8 + 4 * q + s) * NB * 32));
                const uint32_t acc_in = (q > 0 || s > 0) ? 1u : 0u;
                umma_i8(d_hi, umma_desc(a_base + (uint32_t)(ab * MMA_ABUF + (0 * 4 + s) * 4096)), bd, idesc, acc_in);
                umma_i8(d_lo, umma_desc(a_base + (uint32_t)(ab * MMA_ABUF + (1 * 4 + s) * 4096)), bd, idesc, acc_in);
            }
            umma_commit(&mma_bar[ab]);
        }
    }

    if (ok) {
        // the last two half-blocks' MMAs, then the last block's epilogue
        bool landed = true;
        if (J >= 2) landed = mbar_wait_bounded(&mma_bar[(J - 2) & 1], (uint32_t)(((J - 2) >> 1) & 1), a.status, 5);
        if (J >= 1) landed = mbar_wait_bounded(&mma_bar[(J - 1) & 1], (uint32_t)(((J - 1) >> 1) & 1), a.status, 5) && landed;
        if (__syncthreads_and(landed) && nblk > 0) {
            // the last block's scales moved to prev_* only when a next block began
            prev_d = cur_d;
            prev_dm = cur_dm;
            prev_m03 = cur_m03;
            prev_m47 = cur_m47;
            tc_fence_after();
            epilogue(nblk - 1);
        }
    } else if (tid == 0) {
        // a wait ran out: let this CTA's copies and MMAs finish (bounded) before
        // its shared memory and TMEM are released
        for (int bi = waited; bi < issued; ++bi)
            mbar_wait_bounded(&full[bi % stages], (uint32_t)((bi / stages) & 1), a.status, 5);
        if (j >= 2) mbar_wait_bounded(&mma_bar[j & 1], (uint32_t)(((j - 2) >> 1) & 1), a.status, 5);
        if (j >= 1) mbar_wait_bounded(&mma_bar[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), a.status, 5);
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
    *launched = true;
    return launch_pdl(k_qmv_q4k_mma<NB>, dim3(grid), dim3(MMA_THREADS), L.total, st, a, tm, n_tok, stages);
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
