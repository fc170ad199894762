// engine_kernels.cu — fp32 glue of the decode step around the quantized
// matvecs, and the seeded synthetic weight generator.
//
// Semantics follow the reference's attention layer (src/mono27b_executor.cu
// :2372-2479): per-head RMSNorm of q and k with their norm weights
// (k_rms_norm_mulw_batched :698-733), rotary embedding of the first n_rot
// dims as (p, p + n_rot/2) pairs with theta^(-2p/n_rot) (k_mrope :1147-1178,
// all position streams equal for text tokens), K/V cache append
// (k_mrope_and_cache :1180-1229), and decode attention over the cache
// (k_attn_decode_split_partial / _reduce :1339-1484) — here a plain
// max-subtracted softmax with no score clamp.
#include "m27b_device.cuh"
#include "m27b_launch.cuh"
#include "q8k_warp.cuh"
#include "attn_common.cuh"

namespace m27b {

// ---------------------------------------------------------------------------
// q/k RMSNorm + RoPE + KV-cache append.
// qkv (one matvec output row per token) = [local q/gate heads interleaved,
// 2*hd each | local k heads, hd each | local v heads, hd each].  Grid
// (nq + nkv, tokens): CTA (h < nq, t) handles q head h of token t (writes
// q[t][h] and gate[t][h]); CTA (nq + j, t) handles kv head j (writes the K/V
// cache at position *pos + t).  blockDim.x = hd.
__global__ void k_qk_norm_rope_cache(const float *qkv, const float *q_norm, const float *k_norm, float *q, float *gate,
                                     float *kc, float *vc, const int *pos_p, int nq, int nkv, int hd, int n_rot,
                                     float theta, float eps, int qkv_stride, int qg_stride) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float sh[];  // hd values + 32 partials
    const int h = blockIdx.x, d = threadIdx.x, t = blockIdx.y;
    const int pos = *pos_p + t;
    qkv += (size_t)t * qkv_stride;
    q += (size_t)t * qg_stride;
    gate += (size_t)t * qg_stride;
    const bool is_q = h < nq;
    const float *src = is_q ? qkv + (size_t)h * 2 * hd : qkv + (size_t)nq * 2 * hd + (size_t)(h - nq) * hd;
    const float v = src[d];
    // RMS over the head
    float s = warp_sum(v * v);
    if ((d & 31) == 0) sh[hd + (d >> 5)] = s;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (hd >> 5); ++i) tot += sh[hd + i];
    const float scale = rsqrtf(tot / (float)hd + eps);
    const float nw = is_q ? (q_norm ? q_norm[d] : 1.0f) : (k_norm ? k_norm[d] : 1.0f);
    const float xn = v * scale * nw;
    sh[d] = xn;
    __syncthreads();
    float out = xn;
    const int half = n_rot / 2;
    if (d < n_rot) {
        const int p = d < half ? d : d - half;
        const float ang = (float)pos * powf(theta, -2.0f * (float)p / (float)n_rot);
        float sn, cs;
        sincosf(ang, &sn, &cs);
        out = d < half ? xn * cs - sh[d + half] * sn : sh[d - half] * sn + xn * cs;
    }
    if (is_q) {
        q[(size_t)h * hd + d] = out;
        gate[(size_t)h * hd + d] = src[hd + d];
    } else {
        const int j = h - nq;
        const size_t off = ((size_t)pos * nkv + j) * hd + d;
        kc[off] = out;
        vc[off] = qkv[(size_t)nq * 2 * hd + (size_t)nkv * hd + (size_t)j * hd + d];
    }
}

// ---------------------------------------------------------------------------
// Decode attention, split over positions (flash-decoding).
//
// k_attn_partial: grid (nkv, S), 256 threads.  CTA (j, s) handles the
// G = nq/nkv query heads of kv head j over split s of the L = *pos + 1 cached
// positions; the number of active splits adapts to L on the device
// (att_splits: at least ATT_MIN_POS positions per split) so one captured graph
// serves every position.  Warp w takes every 8th position of the split; lane l
// holds dims [l*DPL, (l+1)*DPL) of a K/V row (vector loads), the query heads
// sit in shared memory.  Per (split, head) the partial record is
// acc[hd], max, sum (record stride hd + 4 keeps records 16-byte aligned).
// k_attn_reduce: grid nq, 256 threads: warp w combines splits w, w+8, ...
// rescaled to the global max, then the 8 warps are summed in shared memory.
template <int DPL>
__global__ void __launch_bounds__(256) k_attn_partial(const float *q, const float *kc, const float *vc, float *part,
                                                      const int *pos_p, int nq, int nkv, float scale, int q_stride,
                                                      int part_stride) {
    pdl_wait();
    pdl_trigger();
    constexpr int hd = DPL * 32, rec = hd + 4;
    const int j = blockIdx.x, s = blockIdx.y;
    const int G = nq / nkv;
    // token z of a batch sees the cache up to its own position *pos + z
    q += (size_t)blockIdx.z * q_stride;
    part += (size_t)blockIdx.z * part_stride;
    const int L = *pos_p + 1 + (int)blockIdx.z;
    const int S = att_splits(L, gridDim.y);
    if (s >= S) return;
    const int p0 = (int)(((long)L * s) / S), p1 = (int)(((long)L * (s + 1)) / S);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    extern __shared__ __align__(16) float sh[];  // q [G][hd] (pre-scaled), then [8 warps][G][rec]
    float *qs = sh;
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = q[(size_t)j * G * hd + i] * scale;
    __syncthreads();
    float acc[ATT_G][DPL], m[ATT_G], l[ATT_G];
#pragma unroll
    for (int g = 0; g < ATT_G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = 0.0f;
    }
    // software pipeline: the next position's K/V rows are in flight while
    // the current one is scored (one memory latency per warp, not one per position)
    float kv[DPL], vv[DPL], kn[DPL], vn[DPL];
    if (p0 + warp < p1) {
        ld_dims<DPL>(kc + ((size_t)(p0 + warp) * nkv + j) * hd + lane * DPL, kn);
        ld_dims<DPL>(vc + ((size_t)(p0 + warp) * nkv + j) * hd + lane * DPL, vn);
    }
    for (int p = p0 + warp; p < p1; p += 8) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            kv[i] = kn[i];
            vv[i] = vn[i];
        }
        if (p + 8 < p1) {
            ld_dims<DPL>(kc + ((size_t)(p + 8) * nkv + j) * hd + lane * DPL, kn);
            ld_dims<DPL>(vc + ((size_t)(p + 8) * nkv + j) * hd + lane * DPL, vn);
        }
#pragma unroll
        for (int g = 0; g < ATT_G; ++g) {
            if (g < G) {
                float qv[DPL];
                ld_dims<DPL>(qs + g * hd + lane * DPL, qv);
                float d = 0.0f;
#pragma unroll
                for (int i = 0; i < DPL; ++i) d = fmaf(qv[i], kv[i], d);
                d = warp_sum(d);
                const float mn = fmaxf(m[g], d);
                const float a = expf(m[g] - mn), b = expf(d - mn);
                l[g] = l[g] * a + b;
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[g][i] = acc[g][i] * a + b * vv[i];
                m[g] = mn;
            }
        }
    }
    float *cb = sh + G * hd;
#pragma unroll
    for (int g = 0; g < ATT_G; ++g) {
        if (g < G) {
            float *r = cb + ((size_t)warp * G + g) * rec;
#pragma unroll
            for (int i = 0; i < DPL; ++i) r[lane * DPL + i] = acc[g][i];
            if (lane == 0) {
                r[hd] = m[g];
                r[hd + 1] = l[g];
            }
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int g = idx / hd, dd = idx - g * hd;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w) M = fmaxf(M, cb[((size_t)w * G + g) * rec + hd]);
        float Lsum = 0.0f, A = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float *r = cb + ((size_t)w * G + g) * rec;
            const float f = r[hd] == -INFINITY ? 0.0f : expf(r[hd] - M);
            Lsum += r[hd + 1] * f;
            A += r[dd] * f;
        }
        float *o = part + ((size_t)s * nq + j * G + g) * rec;
        o[dd] = A;
        if (dd == 0) {
            o[hd] = M;
            o[hd + 1] = Lsum;
        }
    }
}

template <int DPL>
__global__ void __launch_bounds__(256) k_attn_reduce(const float *part, float *out, const int *pos_p, int nq, int smax,
                                                     int part_stride, int out_stride) {
    pdl_wait();
    pdl_trigger();
    constexpr int hd = DPL * 32, rec = hd + 4;
    __shared__ __align__(16) float red[8][rec];
    __shared__ float wmax[8];
    const int h = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    part += (size_t)blockIdx.y * part_stride;
    out += (size_t)blockIdx.y * out_stride;
    const int S = att_splits(*pos_p + 1 + (int)blockIdx.y, smax);
    float M = -INFINITY;
#pragma unroll 4
    for (int s = warp; s < S; s += 8) M = fmaxf(M, part[((size_t)s * nq + h) * rec + hd]);
    if (lane == 0) wmax[warp] = M;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wmax[w]);
    float A[DPL], Ls = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) A[i] = 0.0f;
#pragma unroll 4
    for (int s = warp; s < S; s += 8) {
        const float *r = part + ((size_t)s * nq + h) * rec;
        const float f = expf(r[hd] - M);  // every active split holds at least one position
        Ls = fmaf(f, r[hd + 1], Ls);
        float v[DPL];
        ld_dims<DPL>(r + lane * DPL, v);
#pragma unroll
        for (int i = 0; i < DPL; ++i) A[i] = fmaf(f, v[i], A[i]);
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) red[warp][lane * DPL + i] = A[i];
    if (lane == 0) red[warp][hd] = Ls;
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            o += red[w][d];
            L += red[w][hd];
        }
        out[(size_t)h * hd + d] = o / L;
    }
}

// ---------------------------------------------------------------------------
// Fused decode-layer attention for the engine: the two kernels below replace
// k_qk_norm_rope_cache + the split attention + the gated q8_K quantizer.
//
// Rotary table of the step's position: rope[p] = (cos, sin) of
// pos * theta^(-2p/n_rot) for p < n_rot/2 (the same for every layer), one
// thread per pair, computed once per step.
__global__ void k_rope_table(float2 *rope, const int *pos_p, int n_rot, float theta) {
    pdl_wait();
    pdl_trigger();
    const int p = threadIdx.x;
    if (p >= n_rot / 2) return;
    const float ang = (float)(*pos_p) * powf(theta, -2.0f * (float)p / (float)n_rot);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    rope[p] = make_float2(cs, sn);
}

// One warp applies RMSNorm (with its norm weights) and the rotary embedding
// (table from k_rope_table) to one head of `src` (hd = DPL * 32 values, lane
// l holding dims [l*DPL, (l+1)*DPL)) and leaves the result, times `mul`, in
// dst (shared).
template <int DPL>
M27B_DI void norm_rope_warp(const float *src, const float *nw, float *dst, float mul, const float2 *rope, int n_rot,
                            float eps, int lane) {
    constexpr int hd = DPL * 32;
    float v[DPL];
    ld_dims<DPL>(src + lane * DPL, v);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) ss = fmaf(v[i], v[i], ss);
    ss = warp_sum(ss);
    const float sc = rsqrtf(ss / (float)hd + eps);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane * DPL + i;
        v[i] = v[i] * sc * (nw ? nw[d] : 1.0f);
        dst[d] = v[i];
    }
    __syncwarp();
    const int half = n_rot / 2;
    float out[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane * DPL + i;
        out[i] = v[i];
        if (d < n_rot) {
            const float2 r = rope[d < half ? d : d - half];
            out[i] = d < half ? v[i] * r.x - dst[d + half] * r.y : dst[d - half] * r.y + v[i] * r.x;
        }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < DPL; ++i) dst[lane * DPL + i] = out[i] * mul;
    __syncwarp();
}

// Split attention with the q/k norm, RoPE and KV-cache append folded in.
// grid (nkv, splits), 256 threads, G = nq / nkv query heads per kv head (a
// template parameter: the heads' arithmetic is unrolled and interleaved).
// qkv = [nq heads of (q, gate) | nkv k heads | nkv v heads].  Warp g < G
// normalises and rotates query head j*G + g into shared memory.  The newest
// position L - 1 (= *pos) lies in the last active split only: there warp G
// (warp 0 after its query head when G = 8) also normalises and rotates kv
// head j's k and appends k and v at position L - 1 of the caches, which the
// CTA reads back after a barrier (no other CTA touches it).  Warp w scores
// positions p0 + w, p0 + w + 8, ...: the G dot products of a position are
// reduced over the lanes in interleaved butterflies, then the running (max,
// sum, acc) of each head is updated.  The warps' records
// are combined with per-(warp, head) scale factors computed once.
//
// Before griddepcontrol.wait the kernel reads only what the launch order has
// already completed (when this grid starts, its predecessor — the qkv
// projection — has passed its own wait, so every earlier kernel of the step,
// the position advance and the rotary table included, is done): the
// position, the K/V rows of this warp's first two positions unless one of
// them is the newest (appended below), and (into shared memory, once per
// CTA) the q/k norm weights and the rotary factors.  All of it is in flight
// while the projection drains; after the wait only the q (and k, v) rows
// are read.
constexpr int ATT_SLOTS = 4;  // positions per warp whose K/V rows are copied before the wait

size_t attn_qkv_smem_bytes(int G, int hd) {
    // q [G][hd] | k scratch / warp records [8][G][hd] | (m, l) [8][G][2] |
    // scale factors [8][G] | q_norm, k_norm [hd] each | rotary pairs (<= hd
    // floats) | K/V slots [8][ATT_SLOTS][2][hd]
    return (size_t)(G * hd + 8 * G * hd + 8 * G * 2 + 8 * G + 3 * hd + 8 * ATT_SLOTS * 2 * hd) * sizeof(float);
}

template <int DPL, int G>
__global__ void __launch_bounds__(256, 2) k_attn_partial_qkv(const float *qkv, const float *q_norm, const float *k_norm,
                                                             float *kc, float *vc, float *part, const int *pos_p,
                                                             int nq, int nkv, float scale, const float2 *rope,
                                                             int n_rot, float eps) {
    constexpr int hd = DPL * 32, rec = hd + 4;
    const int j = blockIdx.x, s = blockIdx.y;
    const int pos = *pos_p, L = pos + 1;
    const int S = att_splits(L, gridDim.y);
    if (s >= S) return;
    const int p0 = (int)(((long)L * s) / S), p1 = (int)(((long)L * (s + 1)) / S);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool appender = s == S - 1;
    const int kwarp = G < 8 ? G : 0;  // the warp that appends k, v (last split)
    extern __shared__ __align__(16) float sh[];
    float *qs = sh;                      // [G][hd] queries, normalised, rotated, times scale
    float *cb = sh + G * hd;             // k scratch, then the warps' records [8][G][hd]
    float *mlw = cb + 8 * G * hd;        // [8][G][2] (max, sum) per warp and head
    float *fw = mlw + 8 * G * 2;         // [8][G] scale factor of each warp's record
    float *wq = fw + 8 * G;              // q_norm [hd]
    float *wk = wq + hd;                 // k_norm [hd]
    float2 *rp = (float2 *)(wk + hd);    // rotary pairs [n_rot / 2]
    float *kvs = wk + 2 * hd;            // [8 warps][ATT_SLOTS][K, V][hd] prefetched rows
    // warp w's positions are pA + 8i; the first ATT_SLOTS of them (other
    // than the newest, appended below) are copied into its slots now
    const int pA = p0 + warp;
    float *myk = kvs + (size_t)warp * ATT_SLOTS * 2 * hd;
#pragma unroll
    for (int i = 0; i < ATT_SLOTS; ++i) {
        const int p = pA + 8 * i;
        if (p < p1 && p != pos) {
            cp_async_dims<DPL>(myk + (2 * i) * hd + lane * DPL, kc + ((size_t)p * nkv + j) * hd + lane * DPL);
            cp_async_dims<DPL>(myk + (2 * i + 1) * hd + lane * DPL, vc + ((size_t)p * nkv + j) * hd + lane * DPL);
        }
    }
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        wq[i] = q_norm ? q_norm[i] : 1.0f;
        wk[i] = k_norm ? k_norm[i] : 1.0f;
    }
    for (int i = threadIdx.x; i < n_rot / 2; i += blockDim.x) rp[i] = rope[i];
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (warp < G)
        norm_rope_apply<DPL>(qkv + (size_t)(j * G + warp) * 2 * hd, wq, rp, qs + warp * hd, scale, n_rot, eps, lane);
    if (appender && warp == kwarp) {
        const size_t off = ((size_t)pos * nkv + j) * hd;
        norm_rope_apply<DPL>(qkv + (size_t)nq * 2 * hd + (size_t)j * hd, wk, rp, cb, 1.0f, n_rot, eps, lane);
        const float *vsrc = qkv + (size_t)nq * 2 * hd + (size_t)nkv * hd + (size_t)j * hd;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane * DPL + i;
            kc[off + d] = cb[d];
            vc[off + d] = vsrc[d];
        }
    }
    cp_async_wait_all();  // this lane's slot rows (it reads only its own dims of them)
    __syncthreads();      // q in shared memory; the appended k/v visible to this CTA
    float acc[G][DPL], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = 0.0f;
    }
    // row r (0 = K, 1 = V) of position p = pA + 8i: from the warp's slot when
    // it was prefetched, else (the newest position, or beyond the slots) from
    // global memory
    auto row = [&](int i, int p, int r, float (&out)[DPL]) {
        if (i < ATT_SLOTS && p != pos)
            ld_dims<DPL>(myk + (2 * i + r) * hd + lane * DPL, out);
        else
            ld_dims<DPL>((r ? vc : kc) + ((size_t)p * nkv + j) * hd + lane * DPL, out);
    };
    auto update = [&](int g, float d, const float (&vv)[DPL]) {
        const float mn = fmaxf(m[g], d);
        const float a = expf(m[g] - mn), b = expf(d - mn);
        l[g] = l[g] * a + b;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] = acc[g][i] * a + b * vv[i];
        m[g] = mn;
    };
    // one position per step: G dot products, their lane sums in interleaved
    // butterflies, then each head's running update
    for (int i = 0; pA + 8 * i < p1; ++i) {
        const int p = pA + 8 * i;
        float dq[G];
        {
            float kr[DPL];
            row(i, p, 0, kr);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float qv[DPL];
                ld_dims<DPL>(qs + g * hd + lane * DPL, qv);
                float x = 0.0f;
#pragma unroll
                for (int d = 0; d < DPL; ++d) x = fmaf(qv[d], kr[d], x);
                dq[g] = x;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < G; ++g) dq[g] += __shfl_xor_sync(0xffffffffu, dq[g], o);
        float vv[DPL];
        row(i, p, 1, vv);
#pragma unroll
        for (int g = 0; g < G; ++g) update(g, dq[g], vv);
    }
    __syncthreads();  // the k scratch in cb is reused below
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float *r = cb + ((size_t)warp * G + g) * hd;
#pragma unroll
        for (int i = 0; i < DPL; ++i) r[lane * DPL + i] = acc[g][i];
    }
    if (lane < G) {
        // lane g publishes head g's (max, sum); the compile-time index keeps them in registers
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (lane == g) {
                mlw[(warp * G + g) * 2] = m[g];
                mlw[(warp * G + g) * 2 + 1] = l[g];
            }
    }
    __syncthreads();
    // scale factor of warp w's record of head g against the heads' maximum
    if (threadIdx.x < 8 * G) {
        const int w = threadIdx.x / G, g = threadIdx.x - w * G;
        float M = -INFINITY;
#pragma unroll
        for (int u = 0; u < 8; ++u) M = fmaxf(M, mlw[(u * G + g) * 2]);
        const float mw = mlw[(w * G + g) * 2];
        fw[w * G + g] = mw == -INFINITY ? 0.0f : expf(mw - M);
        if (w == 0) {
            float Lsum = 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float mu = mlw[(u * G + g) * 2];
                Lsum += mlw[(u * G + g) * 2 + 1] * (mu == -INFINITY ? 0.0f : expf(mu - M));
            }
            float *o = part + ((size_t)s * nq + j * G + g) * rec;
            o[hd] = M;
            o[hd + 1] = Lsum;
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int g = idx / hd, dd = idx - g * hd;
        float A = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) A += cb[((size_t)w * G + g) * hd + dd] * fw[w * G + g];
        part[((size_t)s * nq + j * G + g) * rec + dd] = A;
    }
}

// Split reduction + sigmoid gate + q8_K quantization: grid nq*hd/256 (hd
// divides 256), 256 threads; CTA b produces q8_K block b of the gated
// attention output o * sigmoid(gate) (heads b*256/hd ..), the input of o_proj.
// Warp w folds splits w, w + 8, ... into a running (max, sum, acc) in one
// pass over the records (the loads of a warp's splits are independent), then
// the 8 warps' results are combined against their common maximum.
template <int DPL>
__global__ void __launch_bounds__(256) k_attn_reduce_gate_q8K(const float *part, const float *qkv, void *xq,
                                                              const int *pos_p, int nq, int smax) {
    constexpr int hd = DPL * 32, rec = hd + 4, hpb = 256 / hd;
    __shared__ __align__(16) float red[8][rec];
    __shared__ __align__(16) float xs[256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the gate inputs come from the qkv projection, two launches back (done
    // when this grid starts): read before the wait for the split records
    float gv[hpb];
#pragma unroll
    for (int hh = 0; hh < hpb; ++hh)
        gv[hh] = threadIdx.x < hd ? qkv[(size_t)(blockIdx.x * hpb + hh) * 2 * hd + hd + threadIdx.x] : 0.0f;
    const int S = att_splits(*pos_p + 1, smax);
    pdl_wait();
    pdl_trigger();
#pragma unroll
    for (int hh = 0; hh < hpb; ++hh) {
        const int h = blockIdx.x * hpb + hh;
        float M = -INFINITY, Ls = 0.0f, A[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) A[i] = 0.0f;
#pragma unroll 4
        for (int s = warp; s < S; s += 8) {
            const float *r = part + ((size_t)s * nq + h) * rec;
            float v[DPL];
            ld_dims<DPL>(r + lane * DPL, v);
            const float mr = r[hd], lr = r[hd + 1];  // every active split holds at least one position
            const float mn = fmaxf(M, mr);
            const float a = expf(M - mn), b = expf(mr - mn);
            Ls = Ls * a + lr * b;
#pragma unroll
            for (int i = 0; i < DPL; ++i) A[i] = A[i] * a + b * v[i];
            M = mn;
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) red[warp][lane * DPL + i] = A[i];
        if (lane == 0) {
            red[warp][hd] = M;
            red[warp][hd + 1] = Ls;
        }
        __syncthreads();
        if (threadIdx.x < hd) {  // hd <= 256 = blockDim.x: one value per thread
            const int d = threadIdx.x;
            float Mx = -INFINITY;
#pragma unroll
            for (int w = 0; w < 8; ++w) Mx = fmaxf(Mx, red[w][hd]);
            float o = 0.0f, L = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const float f = red[w][hd] == -INFINITY ? 0.0f : expf(red[w][hd] - Mx);  // a warp with no split
                o += red[w][d] * f;
                L += red[w][hd + 1] * f;
            }
            xs[hh * hd + d] = (o / L) * (1.0f / (1.0f + expf(-gv[hh])));
        }
        __syncthreads();
    }
    if (warp == 0) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = xs[lane * 8 + i];
        quant_q8K_warp(v, lane, (m27b_block_q8_K *)xq + blockIdx.x);
    }
}

size_t attn_smem_bytes(int G, int hd) { return (size_t)(G * hd + 8 * G * (hd + 4)) * sizeof(float); }

template <int DPL>
static cudaError_t attn_run(const float *q, const float *kc, const float *vc, float *part, float *out, const int *pos,
                            int nq, int nkv, int S, float scale, int n_tok, cudaStream_t st) {
    constexpr int hd = DPL * 32;
    const size_t smem = attn_smem_bytes(nq / nkv, hd);
    const int q_stride = nq * hd, part_stride = S * nq * (hd + 4);
    cudaError_t e = launch_pdl(k_attn_partial<DPL>, dim3(nkv, S, n_tok), dim3(256), smem, st, q, kc, vc, part, pos, nq,
                               nkv, scale, q_stride, part_stride);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_attn_reduce<DPL>, dim3(nq, n_tok), dim3(256), 0, st, (const float *)part, out, pos, nq, S,
                      part_stride, q_stride);
}

template <int DPL, int G>
static cudaError_t attn_qkv_opt_in() {
    return cudaFuncSetAttribute(k_attn_partial_qkv<DPL, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_qkv_smem_bytes(G, DPL * 32));
}

template <int DPL>
static cudaError_t attn_opt_in() {
    const int smem = (int)attn_smem_bytes(ATT_G, DPL * 32);
    const cudaError_t e = cudaFuncSetAttribute(k_attn_partial<DPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if constexpr (DPL == 1 || DPL == 2 || DPL == 4 || DPL == 8) {
        for (cudaError_t r : {attn_qkv_opt_in<DPL, 1>(), attn_qkv_opt_in<DPL, 2>(), attn_qkv_opt_in<DPL, 3>(),
                              attn_qkv_opt_in<DPL, 4>(), attn_qkv_opt_in<DPL, 5>(), attn_qkv_opt_in<DPL, 6>(),
                              attn_qkv_opt_in<DPL, 7>(), attn_qkv_opt_in<DPL, 8>()})
            if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
}

template <int DPL, int G>
static cudaError_t attn_partial_qkv_run(const float *qkv, const float *q_norm, const float *k_norm, float *kc,
                                        float *vc, float *part, const int *pos, int nq, int nkv, int S, float scale,
                                        const float2 *rope, int n_rot, float eps, cudaStream_t st) {
    return launch_pdl(k_attn_partial_qkv<DPL, G>, dim3(nkv, S), dim3(256), attn_qkv_smem_bytes(G, DPL * 32), st, qkv,
                      q_norm, k_norm, kc, vc, part, pos, nq, nkv, scale, rope, n_rot, eps);
}

template <int DPL>
static cudaError_t attn_fused_run(const float *qkv, const float *q_norm, const float *k_norm, float *kc, float *vc,
                                  float *part, void *xq, const int *pos, int nq, int nkv, int S, float scale,
                                  const float2 *rope, int n_rot, float eps, cudaStream_t st) {
    cudaError_t e;
    switch (nq / nkv) {
#define M27B_ATT_G(GG)                                                                                                 \
    case GG:                                                                                                           \
        e = attn_partial_qkv_run<DPL, GG>(qkv, q_norm, k_norm, kc, vc, part, pos, nq, nkv, S, scale, rope, n_rot, eps, \
                                          st);                                                                         \
        break;
        M27B_ATT_G(1) M27B_ATT_G(2) M27B_ATT_G(3) M27B_ATT_G(4) M27B_ATT_G(5) M27B_ATT_G(6) M27B_ATT_G(7) M27B_ATT_G(8)
#undef M27B_ATT_G
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return launch_pdl(k_attn_reduce_gate_q8K<DPL>, dim3(nq * DPL * 32 / 256), dim3(256), 0, st, (const float *)part, qkv,
                      xq, pos, nq, S);
}

// Engine attention in two kernels: q/k norm + RoPE + KV append + split
// attention, then split reduce + gate + q8_K of o_proj's input.  head_dim
// must divide 256 (false: use the unfused kernels).
bool attn_fused_supported(int hd) { return hd == 32 || hd == 64 || hd == 128 || hd == 256; }

cudaError_t attn_fused_launch(const float *qkv, const float *q_norm, const float *k_norm, float *kc, float *vc,
                              float *part, void *xq, const int *pos, int nq, int nkv, int hd, int S, float scale,
                              const float2 *rope, int n_rot, float eps, cudaStream_t st) {
    switch (hd) {
        case 32: return attn_fused_run<1>(qkv, q_norm, k_norm, kc, vc, part, xq, pos, nq, nkv, S, scale, rope, n_rot, eps, st);
        case 64: return attn_fused_run<2>(qkv, q_norm, k_norm, kc, vc, part, xq, pos, nq, nkv, S, scale, rope, n_rot, eps, st);
        case 128: return attn_fused_run<4>(qkv, q_norm, k_norm, kc, vc, part, xq, pos, nq, nkv, S, scale, rope, n_rot, eps, st);
        case 256: return attn_fused_run<8>(qkv, q_norm, k_norm, kc, vc, part, xq, pos, nq, nkv, S, scale, rope, n_rot, eps, st);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Decode attention of a verify pass (several tokens) in ONE launch, after
// k_qk_norm_rope_cache has normalised and rotated every token's queries
// (q, gate rows of nq * hd) and appended its K/V: token t at position
// *pos + t attends to the cache up to its own position.  Grid (nkv, smax,
// tokens), 256 threads; the active splits of token t are ceil(L_t / ABT_CH)
// (at most smax), so a split usually holds one chunk.  CTA (j, s, t):
//   * puts its first chunk's K and V rows in flight (cp.async: every 16-byte
//     piece of a thread at once), then scales the G query heads of kv head j
//     into shared memory;
//   * per chunk of ABT_CH positions: warps score positions against every
//     head, warp g updates head g's running max / sum, each thread
//     accumulates its output values over the chunk's V rows;
//   * writes its partial record (acc, max, sum) and counts itself in
//     count[t][j]; the CTA that arrives last reduces the kv group's splits in
//     split order (vector loads from L2, eight in flight per thread), applies
//     the sigmoid gate, quantizes the G*hd values to q8_K (o_proj's input
//     row t) and resets count[t][j] to zero for the next launch.
// No CTA waits for another: the last arriver is decided by the atomic.  (As
// the single-token step's attention this design measured slower than the
// split + reduce pair above, 179 vs 189 tokens/s; the pair stays there.)
constexpr int ABT_CH = 32;  // positions per staged chunk

struct AttnBatchArgs {
    const float *q, *gate;  // [tokens][nq * hd]: normalised + rotated queries, gate rows
    const float *kc, *vc;
    float *part;            // [tokens][smax][nq][hd + 4]
    void *xq;               // [tokens] q8_K rows of nq * hd values
    const int *pos_p;
    unsigned *count;        // [tokens][nkv], zero between launches
    int nq, nkv, smax;
    float scale;
};

M27B_DI int abt_splits(int L, int smax) {
    const int s = (L + ABT_CH - 1) / ABT_CH;
    return s < smax ? s : smax;
}

size_t attn_batch_smem_bytes(int G, int hd) {
    return (size_t)(G * hd + 2 * ABT_CH * hd + ATT_G * ABT_CH + 4 * ATT_G) * sizeof(float);
}

template <int DPL, int G>
__global__ void __launch_bounds__(256) k_attn_batch(const AttnBatchArgs a) {
    constexpr int hd = DPL * 32, rec = hd + 4, CH = ABT_CH, Q4 = hd / 4;
    constexpr int NO = (G * hd + 255) / 256;  // output values per thread, at most
    const int j = blockIdx.x, s = blockIdx.y, tok = blockIdx.z;
    const int nq = a.nq, nkv = a.nkv;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = threadIdx.x;
    // the pass's first position is set before the pass starts; cache rows
    // below it are older than this launch, those at or past it are appended
    // by the previous kernel
    const int pos0 = *a.pos_p;
    const int L = pos0 + tok + 1;
    const int S = abt_splits(L, a.smax);
    if (s >= S) return;
    float *part = a.part + (size_t)tok * a.smax * nq * rec;
    unsigned *count = a.count + (size_t)tok * nkv;
    const int p0 = (int)(((long)L * s) / S), p1 = (int)(((long)L * (s + 1)) / S);
    extern __shared__ __align__(16) float sh[];
    float *qs = sh;               // [G][hd] queries times scale
    float *ks = qs + G * hd;      // [CH][hd] staged K rows
    float *vs = ks + CH * hd;     // [CH][hd] staged V rows
    float *sc = vs + CH * hd;     // [ATT_G][CH] scores, then softmax weights
    float *hm = sc + ATT_G * CH;  // [ATT_G] running max
    float *hl = hm + ATT_G;       // [ATT_G] running sum
    float *ha = hl + ATT_G;       // [ATT_G] rescale of the previous chunks
    float *hf = ha + ATT_G;       // flag: this CTA arrived last
    auto stage = [&](int c0, int n) {
        for (int idx = t; idx < n * Q4; idx += 256) {
            const int p = idx / Q4, c4 = idx - p * Q4;
            const size_t o = ((size_t)(c0 + p) * nkv + j) * hd + 4 * c4;
            cp_async16(ks + p * hd + 4 * c4, a.kc + o);
            cp_async16(vs + p * hd + 4 * c4, a.vc + o);
        }
    };
    // the first chunk's copies go out before the wait when all its rows are old
    const int n0 = p1 - p0 < CH ? p1 - p0 : CH;
    const bool early = p0 + n0 <= pos0;
    if (early) stage(p0, n0);
    pdl_wait();
    pdl_trigger();
    if (!early) stage(p0, n0);
    const float *qrow = a.q + (size_t)tok * nq * hd;
    if (warp < G) {
        float qv[DPL];
        ld_dims<DPL>(qrow + (size_t)(j * G + warp) * hd + lane * DPL, qv);
#pragma unroll
        for (int i = 0; i < DPL; ++i) qs[warp * hd + lane * DPL + i] = qv[i] * a.scale;
    }
    if (t < ATT_G) {
        hm[t] = -INFINITY;
        hl[t] = 0.0f;
    }
    float acc[NO];
#pragma unroll
    for (int i = 0; i < NO; ++i) acc[i] = 0.0f;
    for (int c0 = p0; c0 < p1; c0 += CH) {
        const int n = p1 - c0 < CH ? p1 - c0 : CH;
        __syncthreads();  // the previous chunk is consumed (the first chunk's copies are already in flight)
        if (c0 != p0) stage(c0, n);
        cp_async_wait_all();
        __syncthreads();
        for (int p = warp; p < n; p += 8) {
            float kv[DPL];
            ld_dims<DPL>(ks + p * hd + lane * DPL, kv);
            float d[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float qv[DPL];
                ld_dims<DPL>(qs + g * hd + lane * DPL, qv);
                float x = 0.0f;
#pragma unroll
                for (int i = 0; i < DPL; ++i) x = fmaf(qv[i], kv[i], x);
                d[g] = x;
            }
            // the G lane sums in interleaved butterflies
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int g = 0; g < G; ++g) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g < G; ++g) sc[g * CH + p] = d[g];
            }
        }
        __syncthreads();
        if (warp < G) {
            const float v = lane < n ? sc[warp * CH + lane] : -INFINITY;
            float cm = v;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mo = hm[warp], mn = fmaxf(mo, cm);
            const float w = lane < n ? expf(v - mn) : 0.0f;
            const float sum = warp_sum(w);
            const float al = mo == -INFINITY ? 0.0f : expf(mo - mn);
            if (lane < n) sc[warp * CH + lane] = w;
            __syncwarp();
            if (lane == 0) {
                hm[warp] = mn;
                hl[warp] = hl[warp] * al + sum;
                ha[warp] = al;
            }
        }
        __syncthreads();
        // P.V: the thread's outputs advance together, one position at a time
        // (independent chains; output slots past G heads use head 0's weights, unused)
        int wofs[NO], vofs[NO];
#pragma unroll
        for (int i = 0; i < NO; ++i) {
            const int o = t + 256 * i, g = o < G * hd ? o / hd : 0;
            wofs[i] = g * CH;
            vofs[i] = o - (o / hd) * hd;
            acc[i] *= ha[g];
        }
#pragma unroll 4
        for (int p = 0; p < n; ++p) {
#pragma unroll
            for (int i = 0; i < NO; ++i) acc[i] = fmaf(sc[wofs[i] + p], vs[p * hd + vofs[i]], acc[i]);
        }
    }
    // this split's partial record per head
#pragma unroll
    for (int i = 0; i < NO; ++i) {
        const int o = t + 256 * i;
        if (o < G * hd) {
            const int g = o / hd, d = o - g * hd;
            part[((size_t)s * nq + j * G + g) * rec + d] = acc[i];
        }
    }
    if (t < G) {
        float *r = part + ((size_t)s * nq + j * G + t) * rec;
        r[hd] = hm[t];
        r[hd + 1] = hl[t];
    }
    __threadfence();
    __syncthreads();
    if (t == 0) hf[0] = atomicAdd(count + j, 1u) == (unsigned)(S - 1) ? 1.0f : 0.0f;
    __syncthreads();
    if (hf[0] == 0.0f) return;
    // the last arriver: every split's record is visible (each CTA fenced its
    // writes before counting itself); read them from L2
    if (t == 0) count[j] = 0u;
    __threadfence();
    float *fm = ks;          // [S][G] split max, then split weight
    float *fl = ks + S * G;  // [S][G] split sum
    float *xs = vs;          // [G * hd] gated output
    for (int idx = t; idx < S * G; idx += 256) {
        const int s2 = idx / G, g = idx - s2 * G;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(part + ((size_t)s2 * nq + j * G + g) * rec + hd));
        fm[idx] = ml.x;
        fl[idx] = ml.y;
    }
    __syncthreads();
    for (int g = warp; g < G; g += 8) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, fm[s2 * G + g]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float Ls = 0.0f;
        for (int s2 = lane; s2 < S; s2 += 32) {
            const float f = expf(fm[s2 * G + g] - M);
            fm[s2 * G + g] = f;
            Ls = fmaf(f, fl[s2 * G + g], Ls);
        }
        Ls = warp_sum(Ls);
        if (lane == 0) hl[g] = Ls;
    }
    __syncthreads();
    const float *grow = a.gate + (size_t)tok * nq * hd;
    for (int q = t; q < G * Q4; q += 256) {
        const int g = q / Q4, c4 = q - g * Q4;
        const float *base = part + ((size_t)j * G + g) * rec + 4 * c4;
        const size_t sstride = (size_t)nq * rec;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int s2 = 0; s2 < S; s2 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                v[u] = s2 + u < S ? __ldcg(reinterpret_cast<const float4 *>(base + (size_t)(s2 + u) * sstride))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (s2 + u < S) {
                    const float f = fm[(s2 + u) * G + g];
                    x.x = fmaf(f, v[u].x, x.x);
                    x.y = fmaf(f, v[u].y, x.y);
                    x.z = fmaf(f, v[u].z, x.z);
                    x.w = fmaf(f, v[u].w, x.w);
                }
            }
        }
        const float4 gt = *reinterpret_cast<const float4 *>(grow + (size_t)(j * G + g) * hd + 4 * c4);
        const float il = 1.0f / hl[g];
        float *o = xs + g * hd + 4 * c4;
        o[0] = (x.x * il) * (1.0f / (1.0f + expf(-gt.x)));
        o[1] = (x.y * il) * (1.0f / (1.0f + expf(-gt.y)));
        o[2] = (x.z * il) * (1.0f / (1.0f + expf(-gt.z)));
        o[3] = (x.w * il) * (1.0f / (1.0f + expf(-gt.w)));
    }
    __syncthreads();
    const int nb = G * hd / 256;
    for (int b = warp; b < nb; b += 8) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = xs[b * 256 + lane * 8 + i];
        quant_q8K_warp(v, lane, (m27b_block_q8_K *)a.xq + (size_t)tok * (nq * hd / 256) + (size_t)j * nb + b);
    }
}

// The (head_dim, heads per kv head) pairs the batch kernel is built for:
// whole q8_K blocks per kv group, (G * hd) % 256 == 0.
#define M27B_ABT_SHAPES(X)                                                                                             \
    X(2, 4) X(2, 8) X(4, 2) X(4, 4) X(4, 6) X(4, 8) X(8, 1) X(8, 2) X(8, 3) X(8, 4) X(8, 5) X(8, 6) X(8, 7) X(8, 8)

static cudaError_t attn_batch_opt_in_all() {
    cudaError_t e = cudaSuccess;
#define M27B_ABT_OPT(D, GG)                                                                                            \
    if (e == cudaSuccess)                                                                                              \
        e = cudaFuncSetAttribute(k_attn_batch<D, GG>, cudaFuncAttributeMaxDynamicSharedMemorySize,                     \
                                 (int)attn_batch_smem_bytes(ATT_G, D * 32));
    M27B_ABT_SHAPES(M27B_ABT_OPT)
#undef M27B_ABT_OPT
    return e;
}

// head_dim 64 / 128 / 256, a kv group's heads filling whole q8_K blocks, and
// the reduction's split weights fitting the staging buffer.
bool attn_batch_supported(int hd, int G, int smax) {
    return (hd == 64 || hd == 128 || hd == 256) && G >= 1 && G <= ATT_G && (G * hd) % 256 == 0 &&
           2 * smax * G <= ABT_CH * hd;
}

// Token t at position *pos + t attends to the cache up to its own position;
// q and gate rows from k_qk_norm_rope_cache (stride nq * hd), K/V already
// appended; q8_K rows of o_proj's input in xq.  count holds n_tok * nkv
// words (zero at rest), part n_tok * S * nq * (hd + 4) floats.
cudaError_t attn_batch_launch(const float *q, const float *gate, const float *kc, const float *vc, float *part,
                              void *xq, const int *pos, unsigned *count, int nq, int nkv, int hd, int S, float scale,
                              int n_tok, cudaStream_t st) {
    AttnBatchArgs a{};
    a.q = q;
    a.gate = gate;
    a.kc = kc;
    a.vc = vc;
    a.part = part;
    a.xq = xq;
    a.pos_p = pos;
    a.count = count;
    a.nq = nq;
    a.nkv = nkv;
    a.smax = S;
    a.scale = scale;
    const size_t smem = attn_batch_smem_bytes(nq / nkv, hd);
    const dim3 grid(nkv, S, n_tok);
    const int dpl = hd / 32, G = nq / nkv;
#define M27B_ABT_RUN(D, GG)                                                                                            \
    if (dpl == D && G == GG) return launch_pdl(k_attn_batch<D, GG>, grid, dim3(256), smem, st, a);
    M27B_ABT_SHAPES(M27B_ABT_RUN)
#undef M27B_ABT_RUN
    return cudaErrorInvalidValue;
}

cudaError_t rope_table_launch(float2 *rope, const int *pos, int n_rot, float theta, cudaStream_t st) {
    return launch_pdl(k_rope_table, dim3(1), dim3(128), 0, st, rope, pos, n_rot, theta);
}

// Raise the shared-memory limit of every attention instantiation (once per
// device, before any capture).
cudaError_t attn_prepare() {
    cudaError_t e = cudaSuccess;
    for (cudaError_t r : {attn_opt_in<1>(), attn_opt_in<2>(), attn_opt_in<3>(), attn_opt_in<4>(), attn_opt_in<5>(),
                          attn_opt_in<6>(), attn_opt_in<7>(), attn_opt_in<8>(), attn_batch_opt_in_all()})
        if (r != cudaSuccess) e = r;
    return e;
}

// Enqueue decode attention for n_tok consecutive tokens (token t at position
// *pos + t, attending to the cache up to its own position): out[t][h][:] for
// the nq local query heads of each token.  q holds n_tok rows of nq * hd,
// part n_tok * S * nq * (hd + 4) floats; hd is a multiple of 32, at most 256.
cudaError_t attn_launch(const float *q, const float *kc, const float *vc, float *part, float *out, const int *pos,
                        int nq, int nkv, int hd, int S, float scale, cudaStream_t st, int n_tok) {
    switch (hd / 32) {
        case 1: return attn_run<1>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 2: return attn_run<2>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 3: return attn_run<3>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 4: return attn_run<4>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 5: return attn_run<5>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 6: return attn_run<6>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 7: return attn_run<7>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        case 8: return attn_run<8>(q, kc, vc, part, out, pos, nq, nkv, S, scale, n_tok, st);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Seeded synthetic GGUF blocks, generated in global tensor coordinates so
// every tensor-parallel shard is a slice of the same global tensor.

M27B_DI uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Fill rows x nblk blocks (raw GGUF layout, row stride nblk*bsize) of global
// rows row0.., global blocks blk0.. of tensor `tid`.  type: 12 q4_K, 14 q6_K,
// 8 q8_0.  fp16 scales are chosen so the values have std ~= sigma.
__global__ void k_fill_blocks(uint8_t *out, int type, int rows, int nblk, long row0, int blk0, uint64_t seed, int tid,
                              float sigma) {
    const int bsize = type == M27B_TYPE_Q4_K ? 144 : type == M27B_TYPE_Q6_K ? 210 : 34;
    const long total = (long)rows * nblk;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long r = i / nblk;
        const int b = (int)(i - r * nblk);
        const uint64_t key = mix64(seed ^ mix64((uint64_t)tid * 0x100000001b3ull ^ (uint64_t)(row0 + r) << 20 ^
                                                 (uint64_t)(blk0 + b)));
        uint8_t *blk = out + i * bsize;
        uint64_t st = key;
        for (int o = 0; o < bsize; o += 8) {
            st = mix64(st);
            for (int k = 0; k < 8 && o + k < bsize; ++k) blk[o + k] = (uint8_t)(st >> (8 * k));
        }
        const float u = 0.5f + (float)(key >> 40) * (1.0f / 16777216.0f);  // [0.5, 1.5)
        if (type == M27B_TYPE_Q4_K) {
            const unsigned short d = __half_as_ushort(__float2half_rn(u * sigma / 250.0f));
            const unsigned short m = __half_as_ushort(__float2half_rn(u * sigma / 120.0f));
            blk[0] = d & 0xff; blk[1] = d >> 8; blk[2] = m & 0xff; blk[3] = m >> 8;
        } else if (type == M27B_TYPE_Q6_K) {
            const unsigned short d = __half_as_ushort(__float2half_rn(u * sigma / 1300.0f));
            blk[208] = d & 0xff; blk[209] = d >> 8;
        } else {
            const unsigned short d = __half_as_ushort(__float2half_rn(u * sigma / 74.0f));
            blk[0] = d & 0xff; blk[1] = d >> 8;
        }
    }
}

// End of a decode step: the argmax key becomes the next step's token, the
// position advances, and the token is appended to hist (greedy generation
// without a host round trip).  ctl = [token, pos, count, step].
__global__ void k_advance(const unsigned long long *best, int *ctl, int *hist, int cap) {
    if (threadIdx.x != 0) return;
    const int next = (int)(0xffffffffu - (uint32_t)(*best & 0xffffffffull));
    const int c = ctl[2];
    if (c < cap) hist[c] = next;
    ctl[0] = next;
    ctl[1] += 1;
    ctl[2] = c + 1;
    ctl[3] += 1;
}

// Tensor-parallel variant of k_advance: exchange the ranks' argmax keys over
// NVLink as two epoch-tagged words per rank (each rank stores its key into
// slot `rank` of every rank's window), wait for every rank's key (bounded),
// and take the largest.  ctl[3] counts steps.
struct BestExchange {
    uint2 *dst[8];       // slot `rank` ([2] words) in every rank's window
    const uint2 *slots;  // this rank's slots [npeers][2]
    int npeers;
    int *status;
};

__global__ void k_advance_p2p(unsigned long long *best, int *ctl, int *hist, int cap, BestExchange b) {
    if (threadIdx.x != 0) return;
    const uint32_t ep = (uint32_t)ctl[3] + 1u;
    const unsigned long long key = *best;
    for (int p = 0; p < b.npeers; ++p) {
        st_word(b.dst[p], (uint32_t)key, ep);
        st_word(b.dst[p] + 1, (uint32_t)(key >> 32), ep);
    }
    unsigned long long m = 0ull;
    for (int s = 0; s < b.npeers; ++s) {
        const uint2 *q = b.slots + 2 * s;
        const uint2 lo = wait_word(q, ld_word(q), ep, b.status, 4);
        const uint2 hi = wait_word(q + 1, ld_word(q + 1), ep, b.status, 4);
        const unsigned long long v = ((unsigned long long)hi.x << 32) | lo.x;
        m = v > m ? v : m;
    }
    *best = m;  // the global key, as the NCCL max all-reduce leaves it
    const int next = (int)(0xffffffffu - (uint32_t)(m & 0xffffffffull));
    const int c = ctl[2];
    if (c < cap) hist[c] = next;
    ctl[0] = next;
    ctl[1] += 1;
    ctl[2] = c + 1;
    ctl[3] += 1;
}

__global__ void k_fill_f32(float *out, long n, float v) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) out[i] = v;
}

}  // namespace m27b
