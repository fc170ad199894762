// qmv_q6k_ksplit.cu — q6_K x 5..8 tokens with the K dimension split across
// CTAs: ffn_down (5120 x 17408) in a speculative verify pass.
//
// The one-pass q6_K kernel (qmv_q6k_tile.cuh) stages every token's whole
// activation row in each CTA; at 8 tokens x 17408 values that is 159 KB and
// leaves no room for the weight stages.  Here the K dimension is split into
// `ks` ranges of whole 4-block tiles and CTA c serves range c % ks only, so
// it stages just that slice of the activations (8 tokens x ~20 blocks =
// 47 KB) next to 8 warps x 2 stages of weight items.  Warp w of the CTAs of a
// range streams whole row groups (items of 8 rows x 1 tile, one 2-D TMA box
// each, as in the one-pass kernel) over the range's tiles, reduces each row
// over its lanes and stores the range's partial sums part[range][t][row].
// The warp whose range completes a row group last (an arrival counter per
// group) adds the ranges' partials in range order (+ residual) and writes y,
// then resets the counter for the next launch: the result is deterministic
// and no warp waits for another.  Integer sums and the fp32 combine per
// block follow ggml's vec_dot_q6_K_q8_K, as in the one-pass kernel (the
// reference's per-token k_q6k_mv_q8_dp4a, src/mono27b_executor.cu:630-645).
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"
#include "qmv_q6k_tile.cuh"

namespace m27b {

constexpr int KSP_WARPS = 8;
constexpr int KSP_MAX_RANGES = 8;
constexpr int KSP_TOKENS = 8;  // tokens of one launch (fewer are padded with zero activations)

struct KsplitArgs {
    float *part;      // [ks][KSP_TOKENS][rows] partial sums of the K ranges
    unsigned *count;  // [row groups] arrivals, zero at rest
    int ks;           // K ranges
    int n_tok;        // real tokens (<= KSP_TOKENS); rows past it are neither read nor written
};

inline int ksp_tiles_max(int rb, int ks) {
    const int P = (rb + 3) / 4;
    return (P + ks - 1) / ks;
}
inline size_t ksp_smem_bytes(int rb, int ks) {
    const size_t nbr = (size_t)4 * ksp_tiles_max(rb, ks);
    return (size_t)KSP_WARPS * Q6T_WARP_BYTES + (size_t)KSP_TOKENS * nbr * (Q6T_XREC + 4) + 32;
}

template <int NT>
__global__ void __launch_bounds__(KSP_WARPS * 32, 1)
    k_qmv_q6k_ksplit(const QmvArgs a, const __grid_constant__ CUtensorMap tm, const KsplitArgs ka) {
    extern __shared__ __align__(128) uint8_t ksp_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int qd = lane >> 3, c = lane & 7;
    const int half = c >> 2, rr = (c >> 1) & 1, lsub = c & 1;
    const int ngroups = (a.rows + 7) >> 3;
    const int P = (a.rb + 3) >> 2;
    const int KS = ka.ks;
    const int rg = (int)blockIdx.x % KS;                     // this CTA's K range
    const int cta = (int)blockIdx.x / KS, nctas = (int)gridDim.x / KS;
    const int t0 = (rg * P) / KS, ntl = ((rg + 1) * P) / KS - t0;
    const int b0 = 4 * t0;
    const int nbr = (4 * (t0 + ntl) < a.rb ? 4 * (t0 + ntl) : a.rb) - b0;  // blocks of the range
    const int gw = cta * nwarps + warp, W = nctas * nwarps;
    const int my_groups = gw < ngroups ? (ngroups - 1 - gw) / W + 1 : 0;

    // [stages of all warps | activation records of the range | block scales | barriers]
    uint8_t *stage0 = ksp_smem + (size_t)warp * Q6T_STAGES * Q6T_ITEM;
    uint8_t *xrec = ksp_smem + (size_t)nwarps * Q6T_STAGES * Q6T_ITEM;
    float *xd = (float *)(xrec + (size_t)NT * nbr * Q6T_XREC);
    uint64_t *bar = (uint64_t *)(((uintptr_t)(xd + NT * nbr) + 15) & ~(uintptr_t)15) + (size_t)warp * Q6T_STAGES;
    if (lane == 0) {
        for (int s = 0; s < Q6T_STAGES; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    int lg = 0, lp = 0, li = 0, ls = 0;
    auto issue_item = [&]() {
        if (lg < my_groups && ntl > 0) {
            if (lane == 0) {
                uint64_t *b = &bar[ls];
                fence_proxy_async();
                mbar_arrive_expect_tx(b, Q6T_ITEM);
                tma_load_2d(stage0 + ls * Q6T_ITEM, &tm, (t0 + lp) * (Q6T_TILE / 4), (gw + lg * W) * 8, b);
            }
            ++li;
            if (++ls == Q6T_STAGES) ls = 0;
            if (++lp == ntl) { lp = 0; ++lg; }
        }
    };
    for (int i = 0; i < Q6T_STAGES; ++i) issue_item();
    pdl_wait();
    // the range's activation blocks of every token (zero codes for padded tokens)
    {
        const uint8_t *src = (const uint8_t *)a.xq;
#pragma unroll 8
        for (int i = threadIdx.x; i < NT * nbr * 64; i += blockDim.x) {
            const int blk = i >> 6, r = i & 63, t = blk / nbr, bl = blk - t * nbr;
            const int hi = r >> 5, cc = (r >> 2) & 7, w = r & 3;
            const int e = 128 * (cc >> 2) + 32 * ((cc >> 1) & 1) + 16 * (cc & 1) + 64 * hi + 4 * w;
            const uint32_t v = t < ka.n_tok ? *(const uint32_t *)(src + ((size_t)t * a.rb + b0 + bl) * 292 + 4 + e) : 0u;
            ((uint32_t *)(xrec + (size_t)blk * Q6T_XREC))[hi * 32 + cc * 4 + w] = v;
        }
        for (int i = threadIdx.x; i < NT * nbr * 9; i += blockDim.x) {
            const int blk = i / 9, j = i - blk * 9, t = blk / nbr, bl = blk - t * nbr;
            const uint8_t *sb = src + ((size_t)t * a.rb + b0 + bl) * 292;
            if (j < 8) {
                uint32_t pr = 0u;
                if (t < ka.n_tok) {
                    const int16_t *bs = (const int16_t *)(sb + 260);
                    const int g = 8 * (j >> 2) + 2 * ((j >> 1) & 1) + (j & 1);
                    pr = (uint32_t)(uint16_t)bs[g] | ((uint32_t)(uint16_t)bs[g + 4] << 16);
                }
                ((uint32_t *)(xrec + (size_t)blk * Q6T_XREC + 256))[j] = pr;
            } else {
                xd[blk] = t < ka.n_tok ? *(const float *)sb : 0.0f;
            }
        }
    }
    pdl_trigger();
    __syncthreads();

    float acc[8][NT];
#pragma unroll
    for (int s = 0; s < 8; ++s)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[s][t] = 0.0f;
    bool ok = true;
    int cs = 0, ci = 0;
    uint32_t cph = 0;
    for (int g = 0; g < my_groups; ++g) {
        const int grp = gw + g * W, row0 = grp * 8;
        for (int pt = 0; pt < ntl; ++pt) {
            const int b = 4 * (t0 + pt) + qd;
            const bool vb = b < a.rb;
            const int bl = vb ? b - b0 : 0;
            const bool landed = mbar_wait_bounded(&bar[cs], cph, a.status, 1);
            if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
            const uint8_t *it = stage0 + cs * Q6T_ITEM;
            if (vb) {
                int4 xa[NT], xh[NT];
                int blo[NT], bhi[NT];
                float dx[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint8_t *xr = xrec + ((size_t)t * nbr + bl) * Q6T_XREC;
                    xa[t] = *(const int4 *)(xr + 16 * c);
                    xh[t] = *(const int4 *)(xr + 128 + 16 * c);
                    const uint32_t pr = *(const uint32_t *)(xr + 256 + 4 * c);
                    blo[t] = (int)(int16_t)(pr & 0xffffu);
                    bhi[t] = (int)(int16_t)(pr >> 16);
                    dx[t] = xd[t * nbr + bl];
                }
                q6t_item_mac<NT>(it, qd, c, half, rr, lsub, xa, xh, blo, bhi, dx, acc);
            }
            __syncwarp();  // every lane is done with this stage before it is refilled
            issue_item();
            ++ci;
            if (++cs == Q6T_STAGES) { cs = 0; cph ^= 1u; }
        }
        if (!ok) break;
        // the range's partial sum of each row of the group (lane s holds row slot s)
        float fin[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = 0.0f;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const float w = warp_sum(acc[s][t]);
                v = lane == s ? w : v;
                acc[s][t] = 0.0f;
            }
            fin[t] = v;
        }
        const int row = row0 + lane;
        if (lane < 8 && row < a.rows) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (t < ka.n_tok) ka.part[((size_t)rg * KSP_TOKENS + t) * a.rows + row] = fin[t];
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0u;
        if (lane == 0) prev = atomicAdd(ka.count + grp, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)(KS - 1)) {
            // every range of this row group is in: add them in range order
            if (lane == 0) ka.count[grp] = 0u;
            __threadfence();
            if (lane < 8 && row < a.rows) {
                for (int t = 0; t < ka.n_tok; ++t) {
                    float v = 0.0f;
                    for (int r2 = 0; r2 < KS; ++r2) v += __ldcg(ka.part + ((size_t)r2 * KSP_TOKENS + t) * a.rows + row);
                    const size_t o = (size_t)t * a.ldy + row;
                    a.y[o] = a.residual ? v + a.residual[o] : v;
                }
            }
        }
    }
    if (!ok) {
        // a wait ran out: let every copy this warp issued land (bounded again)
        for (; ci < li; ++ci) {
            mbar_wait_bounded(&bar[cs], cph, a.status, 2);
            if (++cs == Q6T_STAGES) { cs = 0; cph ^= 1u; }
        }
    }
}

// Most K ranges of a launch for a row of rb blocks (0: this kernel does not apply).
int q6k_ksplit_ranges(int rb) {
    const int P = (rb + 3) / 4;
    if (P < 8) return 0;  // short rows: the one-pass kernel stages little
    return P >= 16 ? 4 : 2;
}

size_t q6k_ksplit_part_floats(int rows, int ks) { return (size_t)ks * KSP_TOKENS * rows; }

cudaError_t launch_q6k_ksplit(const QmvArgs &a_in, int n_tok, float *part, unsigned *count, int sm_count,
                              cudaStream_t st) {
    const int ks = q6k_ksplit_ranges(a_in.rb);
    if (ks == 0 || n_tok < 1 || n_tok > KSP_TOKENS || !part || !count) return cudaErrorInvalidValue;
    QmvArgs a = a_in;
    const size_t smem = ksp_smem_bytes(a.rb, ks);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static size_t opted[64] = {0};
    if (dev >= 64 || smem > opted[dev]) {
        e = cudaFuncSetAttribute(k_qmv_q6k_ksplit<KSP_TOKENS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = smem;
    }
    CUtensorMap tm;
    if (!encode_rows_u32(&tm, a.w0, a.row_stride, a.rows, Q6T_TILE / 4)) return cudaErrorInvalidValue;
    KsplitArgs ka{part, count, ks, n_tok};
    const int grid = ks * (sm_count / ks);  // one CTA per SM, the same number per range
    return launch_pdl(k_qmv_q6k_ksplit<KSP_TOKENS>, dim3(grid), dim3(KSP_WARPS * 32), smem, st, a, tm, ka);
}

}  // namespace m27b
