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
//   * warp 13 streams the weights: one TMA copy of a raw 128-row x 144-byte
//     block column per stage (2-D tensor map, no multicast; up to 10 stages
//     in flight), refilling a stage once every reader has handed it back;
//   * warps 12 and 14 issue the MMAs, one per half-block of every block
//     (4 sub-blocks: 4 MMAs plus two commits);
//   * warps 0-3 unpack: thread r (TMEM lane r) writes row r's block into
//     two of eight TMEM A buffers (one per half-block), a block per
//     tcgen05.wait::st;
//   * warps 4-11 run the epilogue, concurrently with the unpacking of the
//     next block: two warps per TMEM lane quarter, each for half of the
//     tokens (tcgen05.ld of the block's 8 accumulators, one row per thread);
//   * hand-offs: stage full (TMA) -> stage empty (the unpacking warps have
//     read the nibbles and the epilogue warps the block header), A buffer
//     full -> half-block MMAs done (the buffer is free again), block MMAs
//     done (its accumulators are final) -> accumulators free (epilogue read).
// The activations of the CTA's K range (all tokens) are staged once per CTA
// in the canonical K-major no-swizzle UMMA layout, with their scales and
// bsum pairs.  Every wait is bounded (2 s); a timeout records status 5 and raises
// the CTA's abort flag, every role leaves its loop, the issuing thread waits
// (bounded) for its own copies and MMAs, and the CTA frees its TMEM.
#include "tc05.cuh"
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"

namespace m27b {

constexpr int MMA_ROWS = 128;
constexpr int MMA_UNPACK_WARPS = 4;              // warps 0-3: A unpack, one row per thread
constexpr int MMA_EPI_WARPS = 8;                 // warps 4-11: epilogue, two per lane quarter
constexpr int MMA_ISSUER = MMA_UNPACK_WARPS + MMA_EPI_WARPS;  // warp 12: MMAs of first half-blocks
constexpr int MMA_PRODUCER = MMA_ISSUER + 1;                    // warp 13: TMA weight copies
constexpr int MMA_ISSUER2 = MMA_PRODUCER + 1;                   // warp 14: MMAs of second half-blocks
constexpr int MMA_THREADS = (MMA_ISSUER2 + 1) * 32;
constexpr int MMA_MAX_STAGES = 10;
constexpr int MMA_MAX_KS = 8;
constexpr uint32_t MMA_TCOLS = 512;
// Work moves through the roles in items of PB consecutive blocks of a unit
// (PB = 2 at 8 tokens, 1 at 16): one TMA stage (a 128-row box of PB blocks),
// one unpack pass with one tcgen05.wait::st, one A-buffer hand-off, one MMA
// commit, one accumulator hand-off per item — every mbarrier hand-off costs
// ~0.2 us of wake-up latency, which bounded the one-block pipeline.
// TMEM per CTA (all 512 columns): a ring of 2 accumulator items (PB blocks x
// 8 sub-blocks x NB columns: 256 together) and a ring of NAI A items (2 PB
// half-blocks of 32 columns each: 256 together).  One CTA per SM: every CTA
// asks for at least MMA_SMEM_MIN of shared memory, more than an SM has beside
// any other tensor-core CTA (of one launch, or of two launches that
// programmatic dependent launch overlaps), so its tcgen05.alloc of all
// columns never contends — the instruction has no bounded form.
template <int NB> constexpr int mma_pb() { return NB == 8 ? 2 : 1; }
template <int NB> constexpr int mma_ditem() { return mma_pb<NB>() * 8 * NB; }   // accumulator columns per item
template <int NB> constexpr int mma_aitem() { return mma_pb<NB>() * 64; }       // A columns per item
template <int NB> constexpr int mma_nai() { return 256 / mma_aitem<NB>(); }     // A ring slots
constexpr int MMA_ACOL = 256;                                                    // first A column
static_assert(2 * mma_ditem<8>() == MMA_ACOL && 2 * mma_ditem<16>() == MMA_ACOL, "TMEM plan");
__host__ __device__ constexpr int mma_raw_bytes(int nb_tok) { return MMA_ROWS * 144 * (nb_tok <= 8 ? 2 : 1); }  // one stage

// K split across CTAs (verify pass, few row tiles): ks ranges of blocks per
// 128-row tile, unit u = tile * ks + range, the grid a multiple of ks so that
// all units of a CTA lie in one range and the CTA stages only that range's
// activations; the ranges' partial sums go to
// part[((tile * ks + range) * NB + token) * 128 + row] and the epilogue warp
// that arrives last at count[tile * 8 + epilogue warp] adds its 32-row slice
// over the ranges in range order (ks = 1: no scratch, rows written directly).
struct MmaLayout {
    size_t b, dx, bs, raw, bar, flag, total;
    int stages;
};

// Shared memory plan for nbmax blocks of staged activations (a K range) and
// an MMA N of nb_tok (8 or 16).
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
    off += (size_t)stages * mma_raw_bytes(nb_tok);
    L.bar = off;  // full[stages], empty[stages], a_full[NAI], idone[NAI], d_free[2], drain
    off += (size_t)(2 * stages + 2 * 4 + 3) * 8;
    L.flag = off;  // abort flag, TMEM address slot
    off += 16;
    L.total = off;
    L.stages = stages;
    return L;
}

// Most stages (up to MMA_MAX_STAGES) that fit beside nbmax blocks of
// activations; 0 if not even two do.
inline int mma_stages(int nbmax, int nb_tok) {
    for (int s = MMA_MAX_STAGES; s >= 2; --s)
        if (mma_layout(nbmax, nb_tok, s).total + 1024 <= MMA_SMEM_LIMIT) return s;
    return 0;
}


template <int NB>
__global__ void __launch_bounds__(MMA_THREADS, 1)
    k_qmv_q4k_mma(const QmvArgs a, const __grid_constant__ CUtensorMap tm, int n_tok, int stages, int nbmax,
                  const MmaSplit sp) {
    constexpr int PB = mma_pb<NB>(), DITEM = mma_ditem<NB>(), AITEM = mma_aitem<NB>(), NAI = mma_nai<NB>();
    constexpr int RS = 144 * PB, RAW = MMA_ROWS * RS;  // stage row stride, stage bytes
    extern __shared__ __align__(1024) uint8_t mma_smem[];
    uint8_t *smem = mma_smem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = a.rb;
    const MmaLayout L = mma_layout(nbmax, NB, stages);
    uint8_t *bsm = smem + L.b;
    float *dxs = (float *)(smem + L.dx);
    int4 *bss = (int4 *)(smem + L.bs);
    uint8_t *raw = smem + L.raw;
    uint64_t *full = (uint64_t *)(smem + L.bar);
    uint64_t *empty = full + stages;
    uint64_t *a_full = empty + stages;   // [NAI]: an item's A operand written
    uint64_t *idone = a_full + NAI;      // [NAI]: an item's MMAs complete (accumulators final, A slot free)
    uint64_t *d_free = idone + NAI;      // [2]: an accumulator item read by the epilogue
    uint64_t *drain = d_free + 2;
    volatile int *abort = (volatile int *)(smem + L.flag);
    uint32_t *tslot = (uint32_t *)(smem + L.flag + 8);

    // units of this CTA: u = blockIdx.x + i * gridDim.x, tile u / ks, range
    // u % ks = blockIdx.x % ks (gridDim.x is a multiple of ks): blocks
    // [k0, k0 + nbr) of the tile's rows
    const int ks = sp.ks, range = (int)blockIdx.x % ks;
    const int k0 = range * rb / ks, nbr = (range + 1) * rb / ks - k0;
    const int ntiles = (a.rows + MMA_ROWS - 1) / MMA_ROWS, nunits = ntiles * ks;
    const int my_units = (int)blockIdx.x < nunits ? (nunits - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    // items: PB consecutive blocks of a unit, ng per unit (the last may be short)
    const int ng = (nbr + PB - 1) / PB, nitem = my_units * ng;
    auto item_tile = [&](int it) { return ((int)blockIdx.x + (it / ng) * (int)gridDim.x) / ks; };
    auto item_kl0 = [&](int it) { return (it % ng) * PB; };                         // first block in the range
    auto item_nb = [&](int it) { const int k = nbr - item_kl0(it); return k < PB ? k : PB; };

    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MMA_UNPACK_WARPS + MMA_EPI_WARPS);
        }
        for (int b = 0; b < NAI; ++b) {
            mbar_init(&a_full[b], MMA_UNPACK_WARPS);
            mbar_init(&idone[b], 1);  // one issuing thread per item
        }
        for (int b = 0; b < 2; ++b) mbar_init(&d_free[b], MMA_EPI_WARPS);
        mbar_init(drain, 2);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, MMA_TCOLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    // the readers' generic loads of a stage are ordered before its refill by
    // the empty barrier (arrive-release, wait-acquire) that the producer waits on
    // item it: blocks k0 + PB (it % ng) .. of unit it / ng (a box reaching
    // past the range reads blocks no one uses; past the row, zeros)
    auto issue_item = [&](int it) {
        uint64_t *b = &full[it % stages];
        mbar_arrive_expect_tx(b, RAW);
        tma_load_2d(raw + (size_t)(it % stages) * RAW, &tm, (k0 + item_kl0(it)) * 36, item_tile(it) * MMA_ROWS, b);
    };
    // the first raw block columns go out at once: weights do not depend on the previous kernel
    int issued = 0;
    if (warp == MMA_PRODUCER && lane == 0)
        for (; issued < stages && issued < nitem; ++issued) issue_item(issued);

    // activations of this CTA's range: the codes into the UMMA layout, the
    // block scales to dxs, the sums of sub-block pairs (2m, 2m + 1) to
    // halfword m of bss; tokens >= n_tok zero
    pdl_wait();
    gather_tiles<2, NB>(
        n_tok, nbr, bsm, [&](int t, int kl) { return (const unsigned *)a.xq + ((size_t)t * rb + k0 + kl) * Q8K_WORDS; },
        [&](int t, int kl, unsigned v) { dxs[t * nbmax + kl] = __uint_as_float(v); },
        [&](int t, int kl, int m, unsigned v) {
            ((int16_t *)&bss[t * nbmax + kl])[m] = (int16_t)(s16_lo(v) + s16_hi(v));
        });
    pdl_trigger();
    fence_proxy_async();  // the codes are read by the tensor cores (async proxy)
    __syncthreads();

    if (warp == MMA_ISSUER || warp == MMA_ISSUER2) {
        if (lane == 0) {
            // whole items, alternating between the two issuing threads: item
            // it accumulates into accumulator item it & 1 from A slot it % NAI
            const int w = warp == MMA_ISSUER ? 0 : 1;
            constexpr uint32_t idesc = umma_idesc_i8<NB>();
            const uint32_t b_base = smem_u32(bsm);
            for (int it = w; it < nitem; it += 2) {
                const int ds = it & 1, as = it % NAI;
                // the item's MMAs overwrite accumulators whose epilogue (item it - 2) is done
                if (it >= 2 && !wait_or_abort(&d_free[ds], (uint32_t)(((it - 2) >> 1) & 1), abort, a.status)) break;
                if (!wait_or_abort(&a_full[as], (uint32_t)((it / NAI) & 1), abort, a.status)) break;
                tc_fence_after();
                const int kl0 = item_kl0(it), nb = item_nb(it);
                for (int b = 0; b < nb; ++b)
#pragma unroll
                    for (int s8 = 0; s8 < 8; ++s8) {
                        const uint64_t bd = umma_desc(b_base + (uint32_t)(((kl0 + b) * 8 + s8) * NB * 32));
                        umma_i8_ts(tmem + (uint32_t)(ds * DITEM + (8 * b + s8) * NB),
                                   tmem + (uint32_t)(MMA_ACOL + as * AITEM + (2 * b + (s8 >> 2)) * 32 + (s8 & 3) * 8),
                                   bd, idesc, 0u);
                    }
                umma_commit(&idone[as]);
            }
            // drain: every MMA issued above (bounded, even after an abort)
            umma_commit(drain);
            mbar_wait_bounded(drain, 0u, a.status, 5);
        }
        __syncwarp();
    } else if (warp == MMA_PRODUCER) {
        if (lane == 0) {
            // block bi goes into the stage block bi - stages used, once every
            // unpacking and epilogue warp has handed that one back
            for (; issued < nitem; ++issued) {
                const int it = issued;
                if (!wait_or_abort(&empty[it % stages], (uint32_t)((it / stages - 1) & 1), abort, a.status)) break;
                issue_item(it);
            }
            // every copy still in flight lands before the CTA's shared memory is released (bounded)
            for (int it = issued - stages < 0 ? 0 : issued - stages; it < issued; ++it)
                mbar_wait_bounded(&full[it % stages], (uint32_t)((it / stages) & 1), a.status, 5);
        }
        __syncwarp();
    } else if (warp < MMA_UNPACK_WARPS) {
        // A operand: thread r = TMEM lane r = row r of the tile
        const int r = tid;
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        for (int it = 0; it < nitem; ++it) {
            const int as = it % NAI;
            if (!warp_wait_or_abort(&full[it % stages], (uint32_t)((it / stages) & 1), abort, a.status)) break;
            // A slot as is free once the MMAs of item it - NAI are done
            if (it >= NAI && !warp_wait_or_abort(&idone[as], (uint32_t)(((it - NAI) / NAI) & 1), abort, a.status))
                break;
            tc_fence_after();
            const uint8_t *rw0 = raw + (size_t)(it % stages) * RAW + (size_t)r * RS;
            const int nb = item_nb(it);
            for (int b = 0; b < nb; ++b) {
                const uint8_t *rw = rw0 + b * 144;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint32_t acol = tmem + lane_base + (uint32_t)(MMA_ACOL + as * AITEM + (2 * b + q) * 32);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // qs group g = 2q + h: low nibbles are sub-block 2g, high 2g+1,
                        // i.e. sub-blocks 2h and 2h + 1 of half-block q
                        const int g = 2 * q + h;
                        const uint4 qa = *(const uint4 *)(rw + 16 + 32 * g), qb = *(const uint4 *)(rw + 32 + 32 * g);
                        tmem_st8(acol + 16 * h, qa.x & 0x0f0f0f0fu, qa.y & 0x0f0f0f0fu, qa.z & 0x0f0f0f0fu,
                                 qa.w & 0x0f0f0f0fu, qb.x & 0x0f0f0f0fu, qb.y & 0x0f0f0f0fu, qb.z & 0x0f0f0f0fu,
                                 qb.w & 0x0f0f0f0fu);
                        tmem_st8(acol + 16 * h + 8, (qa.x >> 4) & 0x0f0f0f0fu, (qa.y >> 4) & 0x0f0f0f0fu,
                                 (qa.z >> 4) & 0x0f0f0f0fu, (qa.w >> 4) & 0x0f0f0f0fu, (qb.x >> 4) & 0x0f0f0f0fu,
                                 (qb.y >> 4) & 0x0f0f0f0fu, (qb.z >> 4) & 0x0f0f0f0fu, (qb.w >> 4) & 0x0f0f0f0fu);
                    }
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[as]);
                mbar_arrive(&empty[it % stages]);  // this warp is done with the stage
            }
        }
    } else {
        // epilogue: warp 4 + 4 * th + quarter; thread lane of that quarter = row r;
        // tokens [th * NB / 2, (th + 1) * NB / 2)
        constexpr int TPT = NB / 2;  // tokens per thread
        const int e = warp - MMA_UNPACK_WARPS, quarter = e & 3, th = e >> 2;
        const int r = 32 * quarter + lane;
        const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
        const int toff = th * TPT;
        float acc[TPT];
#pragma unroll
        for (int i = 0; i < TPT; ++i) acc[i] = 0.0f;
        for (int it = 0; it < nitem; ++it) {
            const int kl0 = item_kl0(it), nb = item_nb(it), ds = it & 1;
            // the block headers of row r (scales, mins), read before the stage is handed back
            if (!warp_wait_or_abort(&full[it % stages], (uint32_t)((it / stages) & 1), abort, a.status)) break;
            uint4 hd[PB];
#pragma unroll
            for (int b = 0; b < PB; ++b)
                hd[b] = b < nb ? *(const uint4 *)(raw + (size_t)(it % stages) * RAW + (size_t)r * RS + b * 144)
                               : make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[it % stages]);
            // the item's MMAs
            if (!warp_wait_or_abort(&idone[it % NAI], (uint32_t)((it / NAI) & 1), abort, a.status)) break;
            tc_fence_after();
            int v[PB][8][TPT];
            const uint32_t dcol = tmem + lane_base + (uint32_t)(ds * DITEM + toff);
#pragma unroll
            for (int b = 0; b < PB; ++b)
#pragma unroll
                for (int s8 = 0; s8 < 8; ++s8) {
                    if constexpr (TPT == 8) tmem_ld8(dcol + (uint32_t)((8 * b + s8) * NB), v[b][s8]);
                    else tmem_ld4(dcol + (uint32_t)((8 * b + s8) * NB), v[b][s8]);
                }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[ds]);  // the accumulators are in registers
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                if (b >= nb) continue;
                const int kl = kl0 + b;
                const float dw = h2f(hd[b].x), dmw = h2f(hd[b].x >> 16);
                const uint32_t sc03 = hd[b].y & 0x3f3f3f3fu, mn03 = hd[b].z & 0x3f3f3f3fu;
                const uint32_t sc47 = (hd[b].w & 0x0f0f0f0fu) | ((hd[b].y >> 2) & 0x30303030u);
                const uint32_t mn47 = ((hd[b].w >> 4) & 0x0f0f0f0fu) | ((hd[b].z >> 2) & 0x30303030u);
#pragma unroll
                for (int i = 0; i < TPT; ++i) {
                    int isum = 0;
#pragma unroll
                    for (int s8 = 0; s8 < 8; ++s8) {
                        const int sc = (int)(((s8 < 4 ? sc03 : sc47) >> (8 * (s8 & 3))) & 0xffu);
                        isum += sc * v[b][s8][i];
                    }
                    const int t = toff + i;
                    const int4 bs = bss[t * nbmax + kl];
                    int msum = __dp2a_lo(bs.x, (int)mn03, 0);
                    msum = __dp2a_hi(bs.y, (int)mn03, msum);
                    msum = __dp2a_lo(bs.z, (int)mn47, msum);
                    msum = __dp2a_hi(bs.w, (int)mn47, msum);
                    const float dx = dxs[t * nbmax + kl];
                    acc[i] = fmaf(dw * dx, (float)isum, acc[i]);
                    acc[i] = fmaf(-(dmw * dx), (float)msum, acc[i]);
                }
            }
            if (kl0 + nb == nbr) {  // the unit's last item
                const int tile = item_tile(it);
                const int row = tile * MMA_ROWS + r;
                bool write = true;
                if (ks > 1) {
                    // this range's partial sums; the warp arriving last for its
                    // 32-row slice of the tile adds the ranges in range order
                    float *pt = sp.part + ((size_t)(tile * ks + range) * NB + toff) * MMA_ROWS + r;
#pragma unroll
                    for (int i = 0; i < TPT; ++i) pt[(size_t)i * MMA_ROWS] = acc[i];
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
                            float v2 = 0.0f;
                            for (int q2 = 0; q2 < ks; ++q2)
                                v2 += q2 == range ? acc[i]
                                                  : __ldcg(sp.part + ((size_t)(tile * ks + q2) * NB + toff + i) * MMA_ROWS + r);
                            acc[i] = v2;
                        }
                    }
                }
                if (write && row < a.rows) {
#pragma unroll
                    for (int i = 0; i < TPT; ++i) {
                        const int t = toff + i;
                        if (t < n_tok) {
                            const size_t o = (size_t)t * a.ldy + row;
                            a.y[o] = a.residual ? acc[i] + a.residual[o] : acc[i];
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < TPT; ++i) acc[i] = 0.0f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, MMA_TCOLS);
    }
}

// K ranges per tile: 1 when the tiles fill the SMs, else the most (at most
// MMA_MAX_KS, ranges of at least 2 blocks) that keep one unit per SM.
static int mma_ks(int ntiles, int rb, int sm_count) {
    if (ntiles >= sm_count) return 1;
    int best = 1;
    for (int k = 2; k <= MMA_MAX_KS; ++k)
        if (rb / k >= 2 && ntiles * k <= sm_count) best = k;
    return best;
}

// 1: launched; 0: shape not supported by this kernel (caller falls back).
template <int NB>
static cudaError_t run_mma(const QmvArgs &a, int n_tok, int sm_count, cudaStream_t st, bool *launched, float *part,
                           unsigned *count) {
    *launched = false;
    const int ntiles = (a.rows + MMA_ROWS - 1) / MMA_ROWS;
    const int ks = part && count ? mma_ks(ntiles, a.rb, sm_count) : 1;
    const int nbmax = (a.rb + ks - 1) / ks;
    const int stages = mma_stages(nbmax, NB);
    if (stages == 0) return cudaSuccess;
    const MmaLayout L = mma_layout(nbmax, NB, stages);
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
    if (!encode_rows_u32(&tm, a.w0, a.row_stride, a.rows, 36 * mma_pb<NB>(), MMA_ROWS)) return cudaErrorInvalidValue;
    const int units = ntiles * ks;
    const int grid = ks > 1 ? units : (units < sm_count ? units : sm_count);
    const size_t smem = L.total > MMA_SMEM_MIN ? L.total : MMA_SMEM_MIN;
    *launched = true;
    return launch_pdl(k_qmv_q4k_mma<NB>, dim3(grid), dim3(MMA_THREADS), smem, st, a, tm, n_tok, stages, nbmax,
                      MmaSplit{part, count, ks});
}

// Whether 5..16 tokens over rows of rb blocks are served without a K split
// (the whole row's activations and two stages fit).
bool q4k_mma_supported(int rb, int n_tok) {
    return n_tok >= 5 && n_tok <= 16 && mma_stages(rb, n_tok <= 8 ? 8 : 16) > 0;
}

// Scratch of the K-split tensor-core path for `rows` x rb q4_K and n_tok
// tokens (an upper bound: the split the launch picks never needs more).
size_t q4k_mma_split_part_floats(int rows, int rb, int n_tok) {
    (void)rb;
    const int NB = n_tok <= 8 ? 8 : 16, ntiles = (rows + MMA_ROWS - 1) / MMA_ROWS;
    return (size_t)ntiles * MMA_MAX_KS * NB * MMA_ROWS;
}
size_t q4k_mma_split_count_words(int rows) { return (size_t)((rows + MMA_ROWS - 1) / MMA_ROWS) * 8; }

// part / count null: one unit per tile (no scratch).
cudaError_t launch_q4k_mma(const QmvArgs &a, int n_tok, int sm_count, cudaStream_t st, float *part,
                           unsigned *count) {
    bool launched = false;
    const cudaError_t e = n_tok <= 8 ? run_mma<8>(a, n_tok, sm_count, st, &launched, part, count)
                                     : run_mma<16>(a, n_tok, sm_count, st, &launched, part, count);
    if (e != cudaSuccess) return e;
    return launched ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace m27b
