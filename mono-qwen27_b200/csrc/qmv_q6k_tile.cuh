// qmv_q6k_tile.cuh — q6_K matvec over the tiled layout written by m27b_repack.
//
// Layout (lossless, +8 bytes per 4 blocks): a row is ceil(rb/4) tiles of 848
// bytes, tile t holding blocks 4t..4t+3 as
//     ql[4][128] | qh[4][64] | scales[4][16] | d[4] (fp16 + 2 pad bytes)
// (blocks past the end of the row are zero).  GGUF q6_K blocks are 210 bytes
// and only 2-byte aligned (reference BlockQ6K, src/mono27b_executor.cu:57-62);
// the tiles are 16-byte aligned so that one 2-D TMA box of 8 rows x 848 bytes
// fetches a whole work item.
//
// Item = (group of 8 rows, tile p).  Lane L = 8*qd + c works on block
// 4p + qd, 16-byte ql chunk c, for all 8 rows of the item: ql chunk c holds,
// in its low nibbles, values 128*half + 32*rr + 16*lsub + [0,16) (c = 4*half
// + 2*rr + lsub) and, in its high nibbles, the same + 64; their top two bits
// are bits 2rr and 2rr+4 of qh chunk 2*half+lsub (q6k_val, reference
// :1026-1048).  The lane's activation slice is the same for the 8 rows, so it
// is read from shared memory once per item.  The 8 lanes of a shared-memory
// phase read 8 consecutive 16-byte chunks (conflict-free).
//
// Integer sums follow ggml's vec_dot_q6_K_q8_K: per 16-value group,
// sc * (<q, x> - 32 * bsum) with q the unsigned 6-bit code; fp32 combine with
// d_w * d_x per block.
//
// Work split: with enough row groups every warp streams its own groups
// (split 1); for matrices with few rows and long rows (e.g. ffn_down,
// 5120 x 17408) all warps of a CTA split the tiles of one group and combine
// their partial sums in shared memory in a fixed order (deterministic).
#pragma once

#include "qmv_blk.cuh"

namespace m27b {

constexpr int Q6T_TILE = 848;            // bytes per 4-block tile of a row
constexpr int Q6T_ITEM = 8 * Q6T_TILE;   // 6784 bytes: one item (8 rows x 1 tile)
constexpr int Q6T_STAGES = 2;
constexpr int Q6T_WARPS = 8;             // most warps per CTA
constexpr int Q6T_XREC = 288;            // per (token, block): 8 lo chunks | 8 hi chunks | 8 bsum pairs
constexpr size_t Q6T_SMEM_MAX = 112 * 1024;  // two CTAs per SM
// With several tokens and long rows (ffn_down: 4 tokens x 17408 values of
// staged activations = 79 KB) two CTAs per SM would leave room for too few
// warps; such shapes run one CTA per SM with up to this much.
constexpr size_t Q6T_SMEM_BIG = 220 * 1024;
constexpr int Q6T_MIN_WARPS = 4;

inline size_t q6t_x_bytes(int k, int nt) { return (size_t)nt * ((size_t)k / 256) * (Q6T_XREC + 4); }
constexpr size_t Q6T_WARP_BYTES = (size_t)Q6T_STAGES * Q6T_ITEM + (size_t)Q6T_STAGES * 8;
// partial sums for the cooperative split: [warps][8 rows][2 matrices][NT]
inline size_t q6t_part_bytes(int nt) { return (size_t)Q6T_WARPS * 8 * 2 * nt * 4; }

inline int q6t_warps_within(int k, int nt, size_t limit) {
    const size_t fixed = q6t_x_bytes(k, nt) + q6t_part_bytes(nt) + 32;
    if (fixed >= limit) return 0;
    const size_t w = (limit - fixed) / Q6T_WARP_BYTES;
    return (int)(w < (size_t)Q6T_WARPS ? w : (size_t)Q6T_WARPS);
}
// CTAs per SM for a shape: 2 within Q6T_SMEM_MAX, else 1 within Q6T_SMEM_BIG.
inline int q6t_ctas_per_sm(int k, int nt) { return q6t_warps_within(k, nt, Q6T_SMEM_MAX) >= Q6T_MIN_WARPS ? 2 : 1; }
inline int q6t_warps(int k, int nt) {
    return q6t_warps_within(k, nt, q6t_ctas_per_sm(k, nt) == 2 ? Q6T_SMEM_MAX : Q6T_SMEM_BIG);
}
inline size_t q6t_smem_bytes(int k, int nt) {
    return (size_t)q6t_warps(k, nt) * Q6T_WARP_BYTES + q6t_x_bytes(k, nt) + q6t_part_bytes(nt) + 32;
}

// Stage NT activation rows (q8_K) as per-block records for the lane mapping
// above: [8 lo chunks (16 codes each) | 8 hi chunks | 8 packed bsum pairs].
template <int NT>
M27B_DI void stage_x_q6t(const QmvArgs &a, uint8_t *xrec, float *xd) {
    const int nb = a.k / 256;
    const uint8_t *src = (const uint8_t *)a.xq;  // NT*nb blocks of 292 bytes
    // codes: 64 words per block; word w of chunk c (lo/hi) comes from element
    // e_lo(c) (+64 for hi) + 4w
    // a record is 73 words: d, 64 code words, 8 words of two bsums each.
    // Code element e = 4 (o - 1) goes to word hi * 32 + c * 4 + w of the
    // staged record, where e = 128 (c / 4) + 32 ((c / 2) % 2) + 16 (c % 2)
    // + 64 hi + 4 w; pack word j holds the sums of 16-value groups
    // g(j) = 8 (j / 4) + 2 ((j / 2) % 2) + j % 2 (low half) and g(j) + 4.
    gather_l2<8, unsigned>(NT * nb * Q8K_WORDS, [&](int i) { return (const unsigned *)src + i; },
                           [&](int i, unsigned v) {
                               const int blk = i / Q8K_WORDS, o = i - blk * Q8K_WORDS;
                               uint8_t *rec = xrec + (size_t)blk * Q6T_XREC;
                               if (o == 0) {
                                   xd[blk] = __uint_as_float(v);
                               } else if (o <= 64) {
                                   const int e = 4 * (o - 1), hi = (e >> 6) & 1, w = (e >> 2) & 3;
                                   const int c = 4 * (e >> 7) + 2 * ((e >> 5) & 1) + ((e >> 4) & 1);
                                   ((uint32_t *)rec)[hi * 32 + c * 4 + w] = v;
                               } else {
                                   uint16_t *pk = (uint16_t *)(rec + 256);
#pragma unroll
                                   for (int h = 0; h < 2; ++h) {
                                       const int b = 2 * (o - 65) + h;          // bsum index 0..15
                                       const int hb = (b >> 2) & 1, g = b - 4 * hb;  // high half of g's word?
                                       const int j = g < 4 ? g : g - 4;
                                       pk[2 * j + hb] = (uint16_t)(h ? (v >> 16) : v);
                                   }
                               }
                           });
}

// The same records built from fp32 activations (the fused quantize + matvec
// entries, e.g. ffn_down's input silu(gate) * up): warp w quantizes blocks
// w, w + nwarps, ... of the NT rows with the shared q8_K warp routine (the
// codes, group sums and scale m27b_act_quant writes), QX_REGS blocks' loads
// in flight before any arithmetic.  Lane l holds values 8l .. 8l+7 of a
// block: they land in chunk c (below) at word offset ((8l >> 2) & 3); the
// 16-value group l/2 sum goes to bsum pair word j, half h.
template <int NT>
M27B_DI void quant_x_q6t(const QmvArgs &a, uint8_t *xrec, float *xd) {
    const int nb = a.k / 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int e = 8 * lane;
    const int c = 4 * (e >> 7) + 2 * ((e >> 5) & 1) + ((e >> 4) & 1);
    const int word = ((e >> 6) & 1) * 32 + c * 4 + ((e >> 2) & 3);
    const int m = lane >> 1;
    const int bj = 4 * (m >> 3) + 2 * ((m >> 1) & 1) + (m & 1), bh = (m >> 2) & 1;
    const int total = NT * nb;
    for (int i0 = warp; i0 < total; i0 += nw * QX_REGS) {
        float v[QX_REGS][8];
#pragma unroll
        for (int r = 0; r < QX_REGS; ++r) {
            const int i = i0 + r * nw;
            if (i < total) {
                const int t = i / nb, b = i - t * nb;
                const float4 *xr = (const float4 *)(a.xf + (size_t)t * a.ldxf + b * 256 + lane * 8);
                const float4 p0 = __ldcg(xr), p1 = __ldcg(xr + 1);
                v[r][0] = p0.x; v[r][1] = p0.y; v[r][2] = p0.z; v[r][3] = p0.w;
                v[r][4] = p1.x; v[r][5] = p1.y; v[r][6] = p1.z; v[r][7] = p1.w;
            }
        }
#pragma unroll
        for (int r = 0; r < QX_REGS; ++r) {
            const int i = i0 + r * nw;
            if (i < total) {
                uint32_t packed[2];
                int sum;
                float d;
                quant_q8K_lane(v[r], lane, packed, sum, d);
                uint8_t *rec = xrec + (size_t)i * Q6T_XREC;
                ((uint32_t *)rec)[word] = packed[0];
                ((uint32_t *)rec)[word + 1] = packed[1];
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                if ((lane & 1) == 0) ((int16_t *)(rec + 256 + 4 * bj))[bh] = (int16_t)sum;
                if (lane == 0) xd[i] = d;
            }
        }
    }
}

// One lane's share of one item (8 rows x 1 tile at `it` in shared memory):
// block 4p + qd, ql chunk c of every row, against this lane's activation
// slice of that block (xa / xh: low / high chunk codes, blo / bhi: their
// 16-value group sums, dx: the block scale) for NT tokens, accumulated into
// acc[row slot][token].
template <int NT>
M27B_DI void q6t_item_mac(const uint8_t *it, int qd, int c, int half, int rr, int lsub, const int4 (&xa)[NT],
                          const int4 (&xh)[NT], const int (&blo)[NT], const int (&bhi)[NT], const float (&dx)[NT],
                          float (&acc)[8][NT]) {
    // the code's two high bits (qh bits 2rr, 2rr + 1 for the low nibbles,
    // 2rr + 4, 2rr + 5 for the high ones) moved to bits 4-5 of each byte
    // with one shift inside the byte: << (4 - 2rr), >> 2rr
    const int sl = 4 - 2 * rr, sh = 2 * rr;
    const int sc_byte = 8 * half + 2 * rr + lsub;  // scale of the low chunk; the high one is +4
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const uint8_t *tl = it + s * Q6T_TILE;
        const uint4 ql = *(const uint4 *)(tl + qd * 128 + 16 * c);
        const uint4 qh = *(const uint4 *)(tl + 512 + qd * 64 + 16 * (2 * half + lsub));
        const uint4 scw = *(const uint4 *)(tl + 768 + qd * 16);
        const float dw = h2f(*(const uint32_t *)(tl + 832 + qd * 4));
        const uint32_t sw_lo = sc_byte < 4 ? scw.x : sc_byte < 8 ? scw.y : sc_byte < 12 ? scw.z : scw.w;
        const uint32_t sw_hi = sc_byte < 4 ? scw.y : sc_byte < 8 ? scw.z : scw.w;
        const int scl = (int)(int8_t)((sw_lo >> (8 * (sc_byte & 3))) & 0xffu);
        const int sch = (int)(int8_t)((sw_hi >> (8 * (sc_byte & 3))) & 0xffu);
        uint32_t lo[4], hi[4];
        lo[0] = (ql.x & 0x0f0f0f0fu) | ((qh.x << sl) & 0x30303030u);
        lo[1] = (ql.y & 0x0f0f0f0fu) | ((qh.y << sl) & 0x30303030u);
        lo[2] = (ql.z & 0x0f0f0f0fu) | ((qh.z << sl) & 0x30303030u);
        lo[3] = (ql.w & 0x0f0f0f0fu) | ((qh.w << sl) & 0x30303030u);
        hi[0] = ((ql.x >> 4) & 0x0f0f0f0fu) | ((qh.x >> sh) & 0x30303030u);
        hi[1] = ((ql.y >> 4) & 0x0f0f0f0fu) | ((qh.y >> sh) & 0x30303030u);
        hi[2] = ((ql.z >> 4) & 0x0f0f0f0fu) | ((qh.z >> sh) & 0x30303030u);
        hi[3] = ((ql.w >> 4) & 0x0f0f0f0fu) | ((qh.w >> sh) & 0x30303030u);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            int dl = dp4a_us(lo[0], xa[t].x, 0);
            dl = dp4a_us(lo[1], xa[t].y, dl);
            dl = dp4a_us(lo[2], xa[t].z, dl);
            dl = dp4a_us(lo[3], xa[t].w, dl);
            int dh = dp4a_us(hi[0], xh[t].x, 0);
            dh = dp4a_us(hi[1], xh[t].y, dh);
            dh = dp4a_us(hi[2], xh[t].z, dh);
            dh = dp4a_us(hi[3], xh[t].w, dh);
            // codes are stored +32: <q-32, x> = <q, x> - 32 * bsum
            const int isum = scl * (dl - 32 * blo[t]) + sch * (dh - 32 * bhi[t]);
            acc[s][t] = fmaf(dw * dx[t], (float)isum, acc[s][t]);
        }
    }
}

template <int NT, int EPI>
__global__ void __launch_bounds__(Q6T_WARPS * 32, 2)
    k_qmv_q6k_tile(const QmvArgs a, const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                   int split) {
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    extern __shared__ __align__(128) uint8_t q6t_smem[];
    uint8_t *smem = q6t_smem;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int qd = lane >> 3, c = lane & 7;
    const int half = c >> 2, rr = (c >> 1) & 1, lsub = c & 1;
    const int nwarps = blockDim.x >> 5;
    const int ngroups = (a.rows + 7) >> 3;
    const int P = (a.rb + 3) >> 2;  // tiles per row
    const int nb = a.rb;

    // split == 1: warp wg owns groups wg, wg+W, ...; all tiles of each.
    // split == nwarps: the CTA owns groups blockIdx.x, +gridDim.x, ...; warp
    // w takes tiles [w*P/split, (w+1)*P/split) of each.
    const int wg = split == 1 ? blockIdx.x * nwarps + warp : blockIdx.x;
    const int W = split == 1 ? gridDim.x * nwarps : gridDim.x;
    const int my_groups = wg < ngroups ? (ngroups - 1 - wg) / W + 1 : 0;
    const int p_lo = split == 1 ? 0 : (warp * P) / split;
    const int p_hi = split == 1 ? P : ((warp + 1) * P) / split;
    const int my_tiles = p_hi - p_lo;

    // [stages | activation records | block scales | partials | barriers]
    uint8_t *stage0 = smem + (size_t)warp * Q6T_STAGES * Q6T_ITEM;
    uint8_t *xrec = smem + (size_t)nwarps * Q6T_STAGES * Q6T_ITEM;
    float *xd = (float *)(xrec + (size_t)NT * nb * Q6T_XREC);
    float *part = (float *)(((uintptr_t)(xd + NT * nb) + 15) & ~(uintptr_t)15);  // [nwarps][8][NT]
    uint64_t *bar = (uint64_t *)(part + (size_t)Q6T_WARPS * 8 * 2 * NT) + (size_t)warp * Q6T_STAGES;
    if (lane == 0) {
        for (int s = 0; s < Q6T_STAGES; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    int lg = 0, lp = 0, lm = 0, li = 0, ls = 0;
    auto issue_item = [&]() {
        if (lg < my_groups && my_tiles > 0) {
            if (lane == 0) {
                uint64_t *b = &bar[ls];
                fence_proxy_async();
                mbar_arrive_expect_tx(b, Q6T_ITEM);
                tma_load_2d(stage0 + ls * Q6T_ITEM, (NM == 2 && lm == 1) ? &tm1 : &tm0, (p_lo + lp) * (Q6T_TILE / 4),
                            (wg + lg * W) * 8, b);
            }
            ++li;
            if (++ls == Q6T_STAGES) ls = 0;
            if (++lm == NM) {
                lm = 0;
                if (++lp == my_tiles) { lp = 0; ++lg; }
            }
        }
    };

    for (int i = 0; i < Q6T_STAGES; ++i) issue_item();
    // the weights are not produced by the previous kernel: their copies are
    // already in flight; the activations (and every global write) wait for it
    pdl_wait();
    if (a.xf)
        quant_x_q6t<NT>(a, xrec, xd);
    else
        stage_x_q6t<NT>(a, xrec, xd);
    pdl_trigger();
    __syncthreads();

    float acc[NM][8][NT];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int s = 0; s < 8; ++s)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[m][s][t] = 0.0f;
    unsigned long long best[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) best[t] = 0ull;

    bool ok = true;
    int cs = 0;
    uint32_t cph = 0;
    int ci = 0;
    int g = 0;
    for (; g < my_groups; ++g) {
        const int row0 = (wg + g * W) * 8;
        for (int pt = 0; pt < my_tiles; ++pt) {
            const int b = 4 * (p_lo + pt) + qd;
            const bool vb = b < nb;
            // this lane's activation slice for block b, once for the 8 rows
            int4 xa[NT], xh[NT];
            int blo[NT], bhi[NT];
            float dx[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint8_t *xr = xrec + ((size_t)t * nb + (vb ? b : 0)) * Q6T_XREC;
                xa[t] = *(const int4 *)(xr + 16 * c);
                xh[t] = *(const int4 *)(xr + 128 + 16 * c);
                const uint32_t pr = *(const uint32_t *)(xr + 256 + 4 * c);
                blo[t] = (int)(int16_t)(pr & 0xffffu);
                bhi[t] = (int)(int16_t)(pr >> 16);
                dx[t] = xd[t * nb + (vb ? b : 0)];
            }
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                const bool landed = mbar_wait_bounded(&bar[cs], cph, a.status, 1);
                if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
                const uint8_t *it = stage0 + cs * Q6T_ITEM;
                if (vb) q6t_item_mac<NT>(it, qd, c, half, rr, lsub, xa, xh, blo, bhi, dx, acc[m]);
                __syncwarp();  // all lanes done with this stage before it is refilled
                issue_item();
                ++ci;
                if (++cs == Q6T_STAGES) { cs = 0; cph ^= 1u; }
            }
            if (!ok) break;
        }
        if (!ok) break;

        // group done: each row's sum over the 32 lanes of this warp
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int s = 0; s < 8; ++s)
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[m][s][t] = warp_sum(acc[m][s][t]);
        // lane s (< 8) finalises row slot s
        float fin[NM][NT];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float v = acc[m][0][t];
#pragma unroll
                for (int s = 1; s < 8; ++s)
                    if (lane == s) v = acc[m][s][t];
                fin[m][t] = v;
            }
        if (split > 1) {
            // cooperative split: combine the warps' partials in warp order
            if (lane < 8) {
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int t = 0; t < NT; ++t) part[((size_t)warp * 8 + lane) * NT * NM + m * NT + t] = fin[m][t];
            }
            __syncthreads();
            if (warp == 0 && lane < 8) {
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        float v = 0.0f;
                        for (int w = 0; w < split; ++w) v += part[((size_t)w * 8 + lane) * NT * NM + m * NT + t];
                        fin[m][t] = v;
                    }
            }
            __syncthreads();
        }
        const int row = row0 + lane;
        if ((split == 1 || warp == 0) && lane < 8 && row < a.rows) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const size_t o = (size_t)t * a.ldy + row;
                const float s0 = fin[0][t];
                if constexpr (EPI == EPI_STORE) {
                    a.y[o] = a.residual ? s0 + a.residual[o] : s0;
                } else if constexpr (EPI == EPI_PUSH) {
                    push_row(a.push, o, a.residual ? s0 + a.residual[o] : s0);
                } else if constexpr (EPI == EPI_SWIGLU) {
                    a.y[o] = s0 / (1.0f + expf(-s0)) * fin[NM - 1][t];
                } else {
                    if (a.y) a.y[o] = s0;
                    const unsigned long long key = argmax_key(s0, (uint32_t)row + a.row_offset);
                    best[t] = key > best[t] ? key : best[t];
                }
            }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int s = 0; s < 8; ++s)
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[m][s][t] = 0.0f;
    }
    if (!ok) {
        // a wait ran out: let every copy this warp issued land (bounded again)
        for (; ci < li; ++ci) {
            mbar_wait_bounded(&bar[cs], cph, a.status, 2);
            if (++cs == Q6T_STAGES) { cs = 0; cph ^= 1u; }
        }
        // keep the CTA-wide barriers of the cooperative split balanced: the
        // other warps still meet two per remaining group, this one included
        if (split > 1)
            for (; g < my_groups; ++g) {
                __syncthreads();
                __syncthreads();
            }
    }
    if constexpr (EPI == EPI_ARGMAX) {
        if (ok && lane < 8) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (best[t] != 0ull) atomicMax(a.best + t, best[t]);
        }
    }
}

}  // namespace m27b
