// qmv_q6k_stream.cu — q6_K x one token for matrices with few, long rows
// (ffn_down, 5120 x 17408, in a decode step) with the work cut evenly over
// the warps of the grid.
//
// The one-pass kernel (qmv_q6k_tile.cuh) hands whole row groups to CTAs:
// ffn_down's 640 groups over 296 CTAs leave 48 CTAs with three groups and
// the rest with two, and the launch lasts as long as a three-group CTA; its
// two CTAs per SM also stage the 17408-value activation row twice, which
// leaves room for six warps each.  Here one CTA per SM stages the row once,
// next to the stages of up to 15 warps, and the items (row group, tile) are
// numbered group-major and cut into one contiguous run per warp of the grid:
// with at least as many warps as row groups, each group into 3-4 equal runs
// of its own (every warp in one group), else into runs of equal item counts
// across group boundaries (with fewer items than warps, one item per run and
// the other warps idle).  A warp accumulates the 8 rows of a
// group over the tiles of its run; when the run leaves the group (or ends)
// it reduces over its lanes.  A group that lies inside one run is written
// directly; otherwise the run's partial row sums go to slot (warp - first
// warp of the group) of part[group], and the warp that arrives last at the
// group's counter adds the slots in slot order (+ residual), writes y and
// resets the counter: the result does not depend on arrival order and no
// warp waits for another.  The arithmetic per item is the one-pass kernel's
// (q6t_item_mac: ggml's vec_dot_q6_K_q8_K, reference
// src/mono27b_executor.cu:630-645 for the per-token kernel it replaces).
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"
#include "qmv_q6k_tile.cuh"

namespace m27b {

constexpr int Q6S_MAX_WARPS = 16;
constexpr size_t Q6S_SMEM_MAX = 227 * 1024;
constexpr int Q6S_MIN_WARPS = 4;

inline size_t q6s_x_bytes(int k) { return ((size_t)k / 256) * (Q6T_XREC + 4); }
inline size_t q6s_smem_for(int nwarps, int k) { return (size_t)nwarps * Q6T_WARP_BYTES + q6s_x_bytes(k) + 32; }
int q6s_warps(int k) {
    const size_t fixed = q6s_x_bytes(k) + 32;
    if (fixed >= Q6S_SMEM_MAX) return 0;
    const size_t w = (Q6S_SMEM_MAX - fixed) / Q6T_WARP_BYTES;
    return (int)(w < (size_t)Q6S_MAX_WARPS ? w : (size_t)Q6S_MAX_WARPS);
}

struct StreamArgs {
    float *part;      // [row groups][tiles per row][8] partial row sums of the runs that share a group
    unsigned *count;  // [row groups] arrivals, zero at rest
};

// The warp (of Wt) whose run holds item i of T: runs are [w*T/Wt, (w+1)*T/Wt).
M27B_DI int q6s_warp_of(long long i, long long T, long long Wt) { return (int)(((i + 1) * Wt - 1) / T); }

// EPI_STORE: y[row] = sum (+ residual); EPI_PUSH: the same value as an
// epoch-tagged word into every rank's receive window (the fused all-reduce).
template <int EPI>
__global__ void __launch_bounds__(Q6S_MAX_WARPS * 32, 1)
    k_qmv_q6k_stream(const QmvArgs a, const __grid_constant__ CUtensorMap tm, const StreamArgs sa) {
    auto out = [&](int row, float v) {
        const float r = a.residual ? v + a.residual[row] : v;
        if constexpr (EPI == EPI_PUSH)
            push_row(a.push, (size_t)row, r);
        else
            a.y[row] = r;
    };
    extern __shared__ __align__(128) uint8_t q6s_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int qd = lane >> 3, c = lane & 7;
    const int half = c >> 2, rr = (c >> 1) & 1, lsub = c & 1;
    const int ngroups = (a.rows + 7) >> 3;
    const int P = (a.rb + 3) >> 2;  // tiles per row
    const int nb = a.rb;
    // runs: Wt = min(warps of the grid, items), so that no run is empty (a
    // group's contributors are then consecutive runs); run r belongs to warp
    // r / gridDim.x of CTA r % gridDim.x (consecutive runs on different SMs).
    // With at least as many runs as groups every group gets kg = Wt / G or
    // Wt / G + 1 runs of equal tile counts (each run inside one group: one
    // hand-off per warp); otherwise the items are cut into equal runs
    // regardless of group boundaries.
    const long long T = (long long)ngroups * P;
    const long long Wt = (long long)gridDim.x * nwarps < T ? (long long)gridDim.x * nwarps : T;
    const int gw = warp * (int)gridDim.x + (int)blockIdx.x;
    const bool aligned = Wt >= ngroups && Wt / ngroups <= P;
    long long i_lo = 0, i_hi = 0;
    int a_first = 0, a_n = 0;  // aligned: this run's group's first run and run count
    if (gw < Wt) {
        if (aligned) {
            const int k = (int)(Wt / ngroups), m = (int)(Wt % ngroups);  // m groups take k + 1 runs
            int g, p, kg;
            if (gw < m * (k + 1)) {
                g = gw / (k + 1);
                p = gw - g * (k + 1);
                kg = k + 1;
                a_first = g * (k + 1);
            } else {
                const int r = gw - m * (k + 1);
                g = m + r / k;
                p = r - (g - m) * k;
                kg = k;
                a_first = m * (k + 1) + (g - m) * k;
            }
            a_n = kg;
            i_lo = (long long)g * P + (long long)p * P / kg;
            i_hi = (long long)g * P + (long long)(p + 1) * P / kg;
        } else {
            i_lo = gw * T / Wt;
            i_hi = (gw + 1) * T / Wt;
        }
    }

    // [stages of all warps | activation records | block scales | barriers]
    uint8_t *stage0 = q6s_smem + (size_t)warp * Q6T_STAGES * Q6T_ITEM;
    uint8_t *xrec = q6s_smem + (size_t)nwarps * Q6T_STAGES * Q6T_ITEM;
    float *xd = (float *)(xrec + (size_t)nb * Q6T_XREC);
    uint64_t *bar = (uint64_t *)(((uintptr_t)(xd + nb) + 15) & ~(uintptr_t)15) + (size_t)warp * Q6T_STAGES;
    if (lane == 0) {
        for (int s = 0; s < Q6T_STAGES; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    long long li_item = i_lo;  // next item to issue
    int li = 0, ls = 0;
    auto issue_item = [&]() {
        if (li_item < i_hi) {
            if (lane == 0) {
                const int grp = (int)(li_item / P), tile = (int)(li_item - (long long)grp * P);
                uint64_t *b = &bar[ls];
                fence_proxy_async();
                mbar_arrive_expect_tx(b, Q6T_ITEM);
                tma_load_2d(stage0 + ls * Q6T_ITEM, &tm, tile * (Q6T_TILE / 4), grp * 8, b);
            }
            ++li_item;
            ++li;
            if (++ls == Q6T_STAGES) ls = 0;
        }
    };
    // the weights are not produced by the previous kernel: their copies go
    // out first; the activations (and every global write) wait for it
    for (int i = 0; i < Q6T_STAGES; ++i) issue_item();
    pdl_wait();
    if (a.xf)
        quant_x_q6t<1>(a, xrec, xd);
    else
        stage_x_q6t<1>(a, xrec, xd);
    pdl_trigger();
    __syncthreads();

    float acc[8][1];
#pragma unroll
    for (int s = 0; s < 8; ++s) acc[s][0] = 0.0f;
    bool ok = true;
    int cs = 0, ci = 0;
    uint32_t cph = 0;
    long long i = i_lo;
    while (i < i_hi) {
        const int grp = (int)(i / P);
        const long long g_lo = (long long)grp * P, g_end = g_lo + P;
        const long long run_end = g_end < i_hi ? g_end : i_hi;
        for (; i < run_end; ++i) {
            const int b = 4 * (int)(i - g_lo) + qd;
            const bool vb = b < nb;
            int4 xa[1], xh[1];
            int blo[1], bhi[1];
            float dx[1];
            {
                const uint8_t *xr = xrec + (size_t)(vb ? b : 0) * Q6T_XREC;
                xa[0] = *(const int4 *)(xr + 16 * c);
                xh[0] = *(const int4 *)(xr + 128 + 16 * c);
                const uint32_t pr = *(const uint32_t *)(xr + 256 + 4 * c);
                blo[0] = (int)(int16_t)(pr & 0xffffu);
                bhi[0] = (int)(int16_t)(pr >> 16);
                dx[0] = xd[vb ? b : 0];
            }
            // every lane waits (bounded); the warp leaves together if any lane gave up
            const bool landed = mbar_wait_bounded(&bar[cs], cph, a.status, 1);
            if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
            if (vb) q6t_item_mac<1>(stage0 + cs * Q6T_ITEM, qd, c, half, rr, lsub, xa, xh, blo, bhi, dx, acc);
            __syncwarp();  // every lane is done with this stage before it is refilled
            issue_item();
            ++ci;
            if (++cs == Q6T_STAGES) { cs = 0; cph ^= 1u; }
        }
        if (!ok) break;
        // the run's sum of each row of the group (lane s < 8 holds row slot s)
        float fin = 0.0f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const float w = warp_sum(acc[s][0]);
            fin = lane == s ? w : fin;
            acc[s][0] = 0.0f;
        }
        const int row = grp * 8 + lane;
        const int w_first = aligned ? a_first : q6s_warp_of(g_lo, T, Wt);
        const int w_last = aligned ? a_first + a_n - 1 : q6s_warp_of(g_end - 1, T, Wt);
        if (w_first == w_last) {
            // the whole group lies in this run
            if (lane < 8 && row < a.rows) out(row, fin);
            continue;
        }
        const int n = w_last - w_first + 1;
        float *gp = sa.part + (size_t)grp * P * 8;
        if (lane < 8) gp[(gw - w_first) * 8 + lane] = fin;
        __threadfence();
        __syncwarp();
        unsigned prev = 0u;
        if (lane == 0) prev = atomicAdd(sa.count + grp, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)(n - 1)) {
            // every run of this group is in: add the slots in order
            if (lane == 0) sa.count[grp] = 0u;
            __threadfence();
            if (lane < 8 && row < a.rows) {
                float v = 0.0f;
                for (int k = 0; k < n; ++k) v += __ldcg(gp + k * 8 + lane);
                out(row, v);
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

// Scratch of a launch: part floats and counter words for a matrix of `rows`
// rows of `rb` q6_K blocks (tiles of 4 blocks).
size_t q6k_stream_part_floats(int rows, int rb) { return (size_t)((rows + 7) / 8) * ((rb + 3) / 4) * 8; }
size_t q6k_stream_count_words(int rows) { return (size_t)(rows + 7) / 8; }

// Whether the stream kernel applies (one token, rows long enough that the
// staged activation row leaves room for Q6S_MIN_WARPS warps).
bool q6k_stream_applies(int k) { return q6s_warps(k) >= Q6S_MIN_WARPS; }

template <int EPI>
static cudaError_t launch_stream_epi(const QmvArgs &a, float *part, unsigned *count, int sm_count, cudaStream_t st) {
    const int nw = q6s_warps(a.k);
    if (nw < Q6S_MIN_WARPS || !part || !count) return cudaErrorInvalidValue;
    const size_t smem = q6s_smem_for(nw, a.k);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static size_t opted[64] = {0};
    if (dev >= 64 || smem > opted[dev]) {
        e = cudaFuncSetAttribute(k_qmv_q6k_stream<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = smem;
    }
    CUtensorMap tm;
    if (!encode_rows_u32(&tm, a.w0, a.row_stride, a.rows, Q6T_TILE / 4)) return cudaErrorInvalidValue;
    const StreamArgs sa{part, count};
    return launch_pdl(k_qmv_q6k_stream<EPI>, dim3(sm_count), dim3(nw * 32), smem, st, a, tm, sa);
}

// epi: EPI_STORE or EPI_PUSH (a.push set).
cudaError_t launch_q6k_stream(const QmvArgs &a, float *part, unsigned *count, int sm_count, cudaStream_t st,
                              int epi) {
    if (epi == EPI_PUSH) return launch_stream_epi<EPI_PUSH>(a, part, count, sm_count, st);
    if (epi == EPI_STORE) return launch_stream_epi<EPI_STORE>(a, part, count, sm_count, st);
    return cudaErrorInvalidValue;
}

}  // namespace m27b
