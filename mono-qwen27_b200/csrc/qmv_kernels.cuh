// qmv_kernels.cuh — the persistent streaming matvec kernel and its per-format
// slice arithmetic (see qmv.cu for the design).
#pragma once

#include "m27b_device.cuh"

namespace m27b {

constexpr int QMV_WARPS = 8;
constexpr int QMV_THREADS = QMV_WARPS * 32;

enum WeightKind { W_Q4K = 0, W_Q6KP = 1, W_Q80P = 2, W_Q5K = 3, W_IQ4XS = 4, W_F16 = 5, W_F32 = 6 };
enum Epilogue { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_ARGMAX = 2, EPI_PUSH = 3 };

// EPI_PUSH: the matvec half of a fused matvec + all-reduce over NVLink.  Row
// r of token t (plus the residual, if any) goes, as the epoch-tagged word
// {value, epoch}, to dst[p][t * ldy + r] for every rank p < npeers (dst[p]
// lies in rank p's receive window, mapped into this process).  The consumer
// polls the words themselves; nothing else signals completion.
constexpr int M27B_MAX_PEERS = 8;
struct PushArgs {
    uint2 *dst[M27B_MAX_PEERS];
    const unsigned *epoch_base;  // epoch = *epoch_base * epoch_mul + epoch_add
    unsigned epoch_mul, epoch_add;
    int npeers;
};

struct QmvArgs {
    const uint8_t *w0;         // weight rows (gate for SWIGLU)
    const uint8_t *w1;         // up rows (SWIGLU only)
    const void *xq;            // NT activation rows (q8_K or q8_0 blocks)
    float *y;                  // [NT][ldy] output (ARGMAX: logits, may be null)
    const float *residual;     // [NT][ldy] added to y (STORE only; may be null)
    unsigned long long *best;  // [NT] packed argmax keys (ARGMAX)
    size_t row_stride;         // bytes per weight row in its layout
    int ldy;
    int rows;
    int rb;                    // blocks per row
    int k;                     // values per row
    int passes;                // 1024-value passes per row
    int segs;                  // units per row = ceil(passes / PS)
    uint32_t row_offset;       // added to argmax indices
    int *status;               // device status word: set non-zero if a bounded wait runs out
    PushArgs push;             // EPI_PUSH only
    // activations quantized in the prologue (q4_K kernel) instead of read as
    // q8_K blocks from xq: fp32 rows xf (stride ldxf), optionally RMSNormed
    const float *xf;
    int ldxf;
    int xnorm_on;
    const float *xnorm;        // RMSNorm weights (may be null: 1.0)
    float eps;
    // SWIGLU, one token, rows a multiple of 256: also write the rows as q8_K
    // blocks (the next matvec's input); q8cnt holds one zeroed word per block
    void *q8out;
    unsigned *q8cnt;
};

// EPI_PUSH row store: one epoch-tagged value to every rank's receive window.
M27B_DI void push_row(const PushArgs &p, size_t o, float v) {
    const uint32_t ep = *p.epoch_base * p.epoch_mul + p.epoch_add;
#pragma unroll
    for (int i = 0; i < M27B_MAX_PEERS; ++i)
        if (i < p.npeers) st_word(p.dst[i] + o, __float_as_uint(v), ep);
}

// Planar view of the staged activations in shared memory.
struct XStage {
    const int8_t *q;     // [NT][k] codes
    const uint32_t *pk;  // [NT][nb*8] the two bsums each lane slice needs, packed as int16 pairs (q8_K only)
    const float *d;      // [NT][nb] block scales
    int k;
    int nb;
};

// u8 x s8 four-way dot product (dp4a.u32.s32): a's bytes unsigned, b's signed.
M27B_DI int dp4a_us(uint32_t a, int b, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// ---------------------------------------------------------------------------
// q4_K, GGUF layout (144-byte blocks).  Pass p, lane L: block b = 4p + L/8,
// 16-byte nibble chunk c = L%8 = 2g + h of qs: the low nibbles are values
// 64g + 16h + [0,16) of sub-block 2g, the high nibbles values 64g + 32 + 16h
// + [0,16) of sub-block 2g+1 (reference :930-942 / official_dequant.c:57-61).
struct WQ4K {
    static constexpr int NL = 2;
    static constexpr int PER_PASS = 4;  // blocks per pass
    // index of the first of the two bsums lane slice c needs (second is +2)
    M27B_DI static int bsum_lo(int c) { return 2 * c - (c & 1); }
    static constexpr int BSUM_GAP = 2;
    M27B_DI static void load(const uint8_t *row, int rb, int p, int lane, uint4 (&v)[NL]) {
        const int b = PER_PASS * p + (lane >> 3);
        if (b < rb) {
            const uint8_t *blk = row + (size_t)b * 144;
            v[0] = ldg_stream16(blk + 16 + 16 * (lane & 7));
            v[1] = ldg_stream16(blk);
        }
    }
    template <int NT>
    M27B_DI static void mac(const uint4 (&v)[NL], int rb, int p, int lane, const XStage &xs, float (&acc)[NT]) {
        const int b = PER_PASS * p + (lane >> 3);
        if (b >= rb) return;
        const int c = lane & 7, g = c >> 1, h = c & 1;
        const uint4 q = v[0], hd = v[1];
        // 6-bit scale/min of sub-blocks 2g and 2g+1 as byte pairs in the low
        // 16 bits (get_scale_min_k4, reference :690-693).
        const int sh = 16 * (g & 1);
        const uint32_t A = hd.y >> sh, B = hd.z >> sh, C = hd.w >> sh;
        uint32_t scp, mnp;
        if (g < 2) {
            scp = A & 0x3f3fu;
            mnp = B & 0x3f3fu;
        } else {
            scp = (C & 0x0f0fu) | ((A >> 2) & 0x3030u);
            mnp = ((C >> 4) & 0x0f0fu) | ((B >> 2) & 0x3030u);
        }
        const float dw = h2f(hd.x), dmw = h2f(hd.x >> 16);
        const uint32_t l0 = q.x & 0x0f0f0f0fu, l1 = q.y & 0x0f0f0f0fu, l2 = q.z & 0x0f0f0f0fu, l3 = q.w & 0x0f0f0f0fu;
        const uint32_t h0 = q.x & 0xf0f0f0f0u, h1 = q.y & 0xf0f0f0f0u, h2 = q.z & 0xf0f0f0f0u, h3 = q.w & 0xf0f0f0f0u;
        const int e0 = b * 256 + 64 * g + 16 * h;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int8_t *xt = xs.q + (size_t)t * xs.k;
            const int4 xa = *(const int4 *)(xt + e0);
            const int4 xb = *(const int4 *)(xt + e0 + 32);
            int dl = dp4a_us(l0, xa.x, 0);
            dl = dp4a_us(l1, xa.y, dl);
            dl = dp4a_us(l2, xa.z, dl);
            dl = dp4a_us(l3, xa.w, dl);
            int dh = dp4a_us(h0, xb.x, 0);  // 16 x the high-nibble dot
            dh = dp4a_us(h1, xb.y, dh);
            dh = dp4a_us(h2, xb.z, dh);
            dh = dp4a_us(h3, xb.w, dh);
            // |dl|, |dh>>4| <= 16*15*127 fit int16: pack and weight by the byte-pair scales
            const int pair = (dl & 0xffff) | ((dh >> 4) << 16);
            const int isum = __dp2a_lo(pair, (int)scp, 0);
            const int msum = __dp2a_lo((int)xs.pk[t * xs.nb * 8 + b * 8 + c], (int)mnp, 0);
            const float v2 = fmaf(dw, (float)isum, -dmw * (float)msum);
            acc[t] = fmaf(v2, xs.d[t * xs.nb + b], acc[t]);
        }
    }
};

// ---------------------------------------------------------------------------
// q6_K, planar layout from m27b_repack: row = [ql rb*128 | qh rb*64 |
// scales rb*16 | d rb*2, padded to 16].  Pass p, lane L: block b = 4p + L/8,
// c = L%8 = 4*half + 2*rr + lsub: ql chunk c holds, in its low nibbles,
// values 128*half + 32*rr + 16*lsub + [0,16) and, in its high nibbles, the
// same + 64; their high bits are bits 2rr and 2rr+4 of qh chunk 2*half+lsub
// (q6k_val, reference :1026-1048).
struct WQ6KP {
    static constexpr int NL = 3;
    static constexpr int PER_PASS = 4;
    M27B_DI static int bsum_lo(int c) { return c + 4 * (c >> 2); }
    static constexpr int BSUM_GAP = 4;
    M27B_DI static void load(const uint8_t *row, int rb, int p, int lane, uint4 (&v)[NL]) {
        const int b = PER_PASS * p + (lane >> 3);
        if (b < rb) {
            const int c = lane & 7, half = c >> 2, lsub = c & 1;
            v[0] = ldg_stream16(row + (size_t)b * 128 + 16 * c);
            v[1] = ldg_stream16(row + (size_t)rb * 128 + (size_t)b * 64 + 16 * (2 * half + lsub));
            const uint2 s = ldg_stream8(row + (size_t)rb * 192 + (size_t)b * 16 + 8 * half);
            v[2] = make_uint4(s.x, s.y, ldg_stream_u16(row + (size_t)rb * 208 + 2 * b), 0u);
        }
    }
    template <int NT>
    M27B_DI static void mac(const uint4 (&v)[NL], int rb, int p, int lane, const XStage &xs, float (&acc)[NT]) {
        const int b = PER_PASS * p + (lane >> 3);
        if (b >= rb) return;
        const int c = lane & 7, half = c >> 2, rr = (c >> 1) & 1, lsub = c & 1;
        const int sb = 8 * (2 * rr + lsub);
        const int sc_lo = (int)(int8_t)((v[2].x >> sb) & 0xffu);
        const int sc_hi = (int)(int8_t)((v[2].y >> sb) & 0xffu);
        const float dw = h2f(v[2].z);
        const uint4 ql = v[0], qh = v[1];
        // qh bits 2rr, 2rr + 1 (low nibbles) and 2rr + 4, 2rr + 5 (high) to
        // bits 4-5 of each byte with one shift inside the byte
        const int sl = 4 - 2 * rr, sh = 2 * rr;
        uint4 lo, hi;
        lo.x = (ql.x & 0x0f0f0f0fu) | ((qh.x << sl) & 0x30303030u);
        lo.y = (ql.y & 0x0f0f0f0fu) | ((qh.y << sl) & 0x30303030u);
        lo.z = (ql.z & 0x0f0f0f0fu) | ((qh.z << sl) & 0x30303030u);
        lo.w = (ql.w & 0x0f0f0f0fu) | ((qh.w << sl) & 0x30303030u);
        hi.x = ((ql.x >> 4) & 0x0f0f0f0fu) | ((qh.x >> sh) & 0x30303030u);
        hi.y = ((ql.y >> 4) & 0x0f0f0f0fu) | ((qh.y >> sh) & 0x30303030u);
        hi.z = ((ql.z >> 4) & 0x0f0f0f0fu) | ((qh.z >> sh) & 0x30303030u);
        hi.w = ((ql.w >> 4) & 0x0f0f0f0fu) | ((qh.w >> sh) & 0x30303030u);
        const int e_lo = b * 256 + 128 * half + 32 * rr + 16 * lsub;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int8_t *xt = xs.q + (size_t)t * xs.k;
            const int4 xa = *(const int4 *)(xt + e_lo);
            const int4 xb = *(const int4 *)(xt + e_lo + 64);
            int dl = dp4a_us(lo.x, xa.x, 0);
            dl = dp4a_us(lo.y, xa.y, dl);
            dl = dp4a_us(lo.z, xa.z, dl);
            dl = dp4a_us(lo.w, xa.w, dl);
            int dh = dp4a_us(hi.x, xb.x, 0);
            dh = dp4a_us(hi.y, xb.y, dh);
            dh = dp4a_us(hi.z, xb.z, dh);
            dh = dp4a_us(hi.w, xb.w, dh);
            // codes are stored +32: <q-32, x> = <q, x> - 32 * bsum (up to 16*32*127 in
            // magnitude, so kept in 32-bit integers)
            const uint32_t pr = xs.pk[t * xs.nb * 8 + b * 8 + c];
            const int blo = (int)(int16_t)(pr & 0xffffu), bhi = (int)(int16_t)(pr >> 16);
            const int isum = sc_lo * (dl - 32 * blo) + sc_hi * (dh - 32 * bhi);
            acc[t] = fmaf(dw * xs.d[t * xs.nb + b], (float)isum, acc[t]);
        }
    }
};

// ---------------------------------------------------------------------------
// q8_0, planar layout from m27b_repack: row = [qs rb*32 | d rb*2, padded to
// 16].  Pass p, lane L: block b = 32p + L, all 32 codes.
struct WQ80P {
    static constexpr int NL = 3;
    static constexpr int PER_PASS = 32;
    M27B_DI static void load(const uint8_t *row, int rb, int p, int lane, uint4 (&v)[NL]) {
        const int b = PER_PASS * p + lane;
        if (b < rb) {
            v[0] = ldg_stream16(row + (size_t)b * 32);
            v[1] = ldg_stream16(row + (size_t)b * 32 + 16);
            v[2].x = ldg_stream_u16(row + (size_t)rb * 32 + 2 * b);
        }
    }
    template <int NT>
    M27B_DI static void mac(const uint4 (&v)[NL], int rb, int p, int lane, const XStage &xs, float (&acc)[NT]) {
        const int b = PER_PASS * p + lane;
        if (b >= rb) return;
        const float dw = h2f(v[2].x);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int8_t *xt = xs.q + (size_t)t * xs.k + b * 32;
            const int dot = dot16(v[0], *(const uint4 *)xt) + dot16(v[1], *(const uint4 *)(xt + 16));
            acc[t] = fmaf((float)dot, dw * xs.d[t * xs.nb + b], acc[t]);
        }
    }
};

template <int WT> struct WTraits;
template <> struct WTraits<W_Q4K> { using T = WQ4K; };
template <> struct WTraits<W_Q6KP> { using T = WQ6KP; };
template <> struct WTraits<W_Q80P> { using T = WQ80P; };

// Copy NT activation rows into shared memory in planar form: codes, the
// bsum pair of every (block, lane slice), block scales.
template <int WT, int NT>
M27B_DI XStage stage_x(const QmvArgs &a, uint8_t *smem) {
    XStage xs;
    xs.k = a.k;
    if constexpr (WT == W_Q80P) {
        const int nb = a.k / 32;
        int8_t *q = (int8_t *)smem;
        float *d = (float *)(smem + (size_t)NT * a.k);
        const uint16_t *src = (const uint16_t *)a.xq;  // 17 halfwords per block
        gather_l2<8, unsigned short>(
            NT * nb * 17, [&](int i) { return (const unsigned short *)src + i; },
            [&](int i, unsigned short hw) {
                const int blk = i / 17, o = i - blk * 17;
                if (o == 0) d[blk] = h2f(hw);
                else *(uint16_t *)(q + (size_t)blk * 32 + 2 * (o - 1)) = hw;
            });
        xs.q = q;
        xs.pk = nullptr;
        xs.d = d;
        xs.nb = nb;
    } else {
        using T = typename WTraits<WT>::T;
        const int nb = a.k / 256;
        int8_t *q = (int8_t *)smem;
        uint32_t *pk = (uint32_t *)(smem + (size_t)NT * a.k);
        float *d = (float *)(smem + (size_t)NT * a.k + (size_t)NT * nb * 32);
        const uint8_t *src = (const uint8_t *)a.xq;  // 292-byte blocks
        const int total = NT * nb * 65;                // d + 64 code words per block
        gather_l2<8, unsigned>(
            total, [&](int i) { return (const unsigned *)(src + (size_t)(i / 65) * 292) + (i % 65); },
            [&](int i, unsigned w) {
                const int blk = i / 65, o = i - blk * 65;
                if (o == 0) d[blk] = __uint_as_float(w);
                else ((uint32_t *)q)[(size_t)blk * 64 + (o - 1)] = w;
            });
        for (int i = threadIdx.x; i < NT * nb * 8; i += blockDim.x) {
            const int blk = i >> 3, c = i & 7, lo = T::bsum_lo(c);
            const int16_t *bs = (const int16_t *)(src + (size_t)blk * 292 + 260);
            pk[i] = (uint32_t)(uint16_t)__ldcg(bs + lo) | ((uint32_t)(uint16_t)__ldcg(bs + lo + T::BSUM_GAP) << 16);
        }
        xs.q = q;
        xs.pk = pk;
        xs.d = d;
        xs.nb = nb;
    }
    return xs;
}

template <int EPI, int NT, int NM>
M27B_DI void finish_row(const QmvArgs &a, int row, float (&acc)[NM][NT], int lane, unsigned long long &best) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        float s0 = warp_sum(acc[0][t]);
        float s1 = 0.0f;
        if constexpr (NM == 2) s1 = warp_sum(acc[1][t]);
        if (lane == t) {
            const size_t o = (size_t)t * a.ldy + row;
            if constexpr (EPI == EPI_STORE) {
                a.y[o] = a.residual ? s0 + a.residual[o] : s0;
            } else if constexpr (EPI == EPI_SWIGLU) {
                a.y[o] = s0 / (1.0f + expf(-s0)) * s1;
            } else {
                if (a.y) a.y[o] = s0;
                const unsigned long long key = argmax_key(s0, (uint32_t)row + a.row_offset);
                best = key > best ? key : best;
            }
        }
        acc[0][t] = 0.0f;
        if constexpr (NM == 2) acc[1][t] = 0.0f;
    }
}

// The warp's work is a sequence of units (row, segment); a segment is PS
// passes of a row.  Units are double-buffered in registers: the loads of unit
// u+1 are issued before unit u is multiplied.
template <int WT, int NT, int EPI, int PS>
__global__ void __launch_bounds__(QMV_THREADS, 2) k_qmv(const QmvArgs a) {
    using T = typename WTraits<WT>::T;
    constexpr int NM = EPI == EPI_SWIGLU ? 2 : 1;
    extern __shared__ __align__(16) uint8_t smem[];

    const int lane = threadIdx.x & 31;
    const int wg = blockIdx.x * QMV_WARPS + (threadIdx.x >> 5);
    const int W = gridDim.x * QMV_WARPS;
    const int P = a.passes, S = a.segs;
    const int my_rows = wg < a.rows ? (a.rows - 1 - wg) / W + 1 : 0;

    uint4 bufA[PS][NM][T::NL];
    uint4 bufB[PS][NM][T::NL];
    int lrow = 0, lseg = 0;  // load cursor
    int crow = 0, cseg = 0;  // compute cursor

    auto load_unit = [&](uint4 (&buf)[PS][NM][T::NL]) {
        if (lrow < my_rows) {
            const size_t r = (size_t)wg + (size_t)lrow * W;
            const uint8_t *r0 = a.w0 + r * a.row_stride;
            const uint8_t *r1 = NM == 2 ? a.w1 + r * a.row_stride : nullptr;
#pragma unroll
            for (int j = 0; j < PS; ++j) {
                const int p = lseg * PS + j;
                if (p < P) {
                    T::load(r0, a.rb, p, lane, buf[j][0]);
                    if constexpr (NM == 2) T::load(r1, a.rb, p, lane, buf[j][1]);
                }
            }
            if (++lseg == S) { lseg = 0; ++lrow; }
        }
    };

    // First loads go out before the activations are staged (weights are not
    // produced by the previous kernel; activations and writes wait for it).
    load_unit(bufA);
    pdl_wait();
    const XStage xs = stage_x<WT, NT>(a, smem);
    pdl_trigger();
    __syncthreads();

    float acc[NM][NT];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[m][t] = 0.0f;
    unsigned long long best = 0ull;

    auto compute_unit = [&](const uint4 (&buf)[PS][NM][T::NL]) {
#pragma unroll
        for (int j = 0; j < PS; ++j) {
            const int p = cseg * PS + j;
            if (p < P) {
                T::template mac<NT>(buf[j][0], a.rb, p, lane, xs, acc[0]);
                if constexpr (NM == 2) T::template mac<NT>(buf[j][1], a.rb, p, lane, xs, acc[1]);
            }
        }
        if (++cseg == S) {
            finish_row<EPI, NT, NM>(a, wg + crow * W, acc, lane, best);
            cseg = 0;
            ++crow;
        }
    };

    while (crow < my_rows) {
        load_unit(bufB);
        compute_unit(bufA);
        if (crow >= my_rows) break;
        load_unit(bufA);
        compute_unit(bufB);
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (lane < NT && best != 0ull) atomicMax(a.best + lane, best);
    }
}

// Largest unit (passes held per register buffer) that double-buffers
// without spilling: per pass and lane a q4_K slice holds 8 registers, a q6_K
// slice 11, a q8_0 slice 9; SWIGLU holds two matrices.
constexpr int max_ps(int wt, int epi, int nt) {
    return epi == EPI_SWIGLU ? (wt == W_Q4K ? (nt == 1 ? 3 : nt == 2 ? 2 : 1) : (nt == 1 ? 2 : 1))
         : wt == W_Q4K ? (nt <= 2 ? 6 : nt == 3 ? 5 : 4)
         : wt == W_Q6KP ? (nt <= 2 ? 4 : 3)
         : (nt <= 3 ? 5 : 4);
}

// Passes per unit for a row of P passes: the whole row when it fits the cap,
// else the unit size <= cap with the fewest idle passes (then the largest).
inline int pick_ps(int P, int cap) {
    if (P <= cap) return P;
    int best = cap, waste = 1 << 30;
    for (int ps = cap; ps >= 1; --ps) {
        const int s = (P + ps - 1) / ps, w = s * ps - P;
        if (w < waste) { waste = w; best = ps; }
    }
    return best;
}

size_t qmv_smem_bytes(int wtype, int k, int ntok);
cudaError_t launch_qmv(int wt, int epi, QmvArgs a, int nt, int sm_count, cudaStream_t st);
// f16 / f32 weights x fp32 activations (a.xf, a.ldxf), store epilogue (qmv_float.cu).
cudaError_t launch_qmv_float(int wt, const QmvArgs &a, int nt, int sm_count, cudaStream_t st);
// q4_K x 5..16 tokens on the tensor cores (qmv_q4k_mma.cu), store epilogue.
bool q4k_mma_supported(int rb, int n_tok);
// part / count (nullable): scratch for K split across CTAs (q4k_mma_split_*).
cudaError_t launch_q4k_mma(const QmvArgs &a, int n_tok, int sm_count, cudaStream_t st, float *part = nullptr,
                           unsigned *count = nullptr);
size_t q4k_mma_split_part_floats(int rows, int rb, int n_tok);
size_t q4k_mma_split_count_words(int rows);

}  // namespace m27b
