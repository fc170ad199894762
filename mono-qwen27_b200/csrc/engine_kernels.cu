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

namespace m27b {

// ---------------------------------------------------------------------------
// q/k RMSNorm + RoPE + KV-cache append.
// qkv (one matvec output) = [local q/gate heads interleaved, 2*hd each |
// local k heads, hd each | local v heads, hd each].  CTA h < nq handles q head
// h (writes q[h] and gate[h]); CTA nq + j handles kv head j (writes K/V cache
// at position *pos).  blockDim.x = hd.
__global__ void k_qk_norm_rope_cache(const float *qkv, const float *q_norm, const float *k_norm, float *q, float *gate,
                                     float *kc, float *vc, const int *pos_p, int nq, int nkv, int hd, int n_rot,
                                     float theta, float eps) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float sh[];  // hd values + 32 partials
    const int h = blockIdx.x, d = threadIdx.x;
    const int pos = *pos_p;
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
// Decode attention, split over positions.  Grid (nkv, splits), 256 threads:
// CTA (j, s) handles the G = nq/nkv query heads of kv head j over positions
// [s*L/S, (s+1)*L/S) of the L = *pos + 1 cached positions; warp w takes every
// 8th position, lanes hold hd/32 dims.  Partials (max, sum, acc[hd]) per
// (split, q head) go to `part`; k_attn_reduce combines them.
constexpr int ATT_G = 8;  // most query heads per kv head

__global__ void __launch_bounds__(256) k_attn_partial(const float *q, const float *kc, const float *vc, float *part,
                                                      const int *pos_p, int nq, int nkv, int hd, float scale) {
    pdl_wait();
    pdl_trigger();
    const int j = blockIdx.x, s = blockIdx.y, S = gridDim.y;
    const int G = nq / nkv;
    const int L = *pos_p + 1;
    const int p0 = (int)(((long)L * s) / S), p1 = (int)(((long)L * (s + 1)) / S);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int DPL = hd / 32;  // dims per lane (<= 8)
    float qr[ATT_G][8], acc[ATT_G][8], m[ATT_G], l[ATT_G];
#pragma unroll
    for (int g = 0; g < ATT_G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            acc[g][i] = 0.0f;
            qr[g][i] = (g < G && i < DPL) ? q[(size_t)(j * G + g) * hd + lane * DPL + i] * scale : 0.0f;
        }
    }
    for (int p = p0 + warp; p < p1; p += 8) {
        const float *kr = kc + ((size_t)p * nkv + j) * hd + lane * DPL;
        const float *vr = vc + ((size_t)p * nkv + j) * hd + lane * DPL;
        float kv[8], vv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            kv[i] = i < DPL ? kr[i] : 0.0f;
            vv[i] = i < DPL ? vr[i] : 0.0f;
        }
#pragma unroll
        for (int g = 0; g < ATT_G; ++g) {
            if (g >= G) continue;
            float d = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) d = fmaf(qr[g][i], kv[i], d);
            d = warp_sum(d);
            const float mn = fmaxf(m[g], d);
            const float a = expf(m[g] - mn), b = expf(d - mn);
            l[g] = l[g] * a + b;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[g][i] = acc[g][i] * a + b * vv[i];
            m[g] = mn;
        }
    }
    // combine the 8 warps in shared memory: per warp (m, l, acc[hd]) per head
    extern __shared__ float sh[];  // [8 warps][G][hd + 2]
    const int rec = hd + 2;
#pragma unroll
    for (int g = 0; g < ATT_G; ++g) {
        if (g < G) {
            float *r = sh + ((size_t)warp * G + g) * rec;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < DPL) r[lane * DPL + i] = acc[g][i];
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
        for (int w = 0; w < 8; ++w) M = fmaxf(M, sh[((size_t)w * G + g) * rec + hd]);
        float Lsum = 0.0f, A = 0.0f;
        for (int w = 0; w < 8; ++w) {
            const float *r = sh + ((size_t)w * G + g) * rec;
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

// Combine the split partials: out[h][d] = sum_s e^(m_s-M) acc_s / sum_s e^(m_s-M) l_s.
__global__ void k_attn_reduce(const float *part, float *out, int nq, int hd, int S) {
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x, d = threadIdx.x;
    const int rec = hd + 2;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, part[((size_t)s * nq + h) * rec + hd]);
    float Lsum = 0.0f, A = 0.0f;
    for (int s = 0; s < S; ++s) {
        const float *r = part + ((size_t)s * nq + h) * rec;
        const float f = r[hd] == -INFINITY ? 0.0f : expf(r[hd] - M);
        Lsum += r[hd + 1] * f;
        A += r[d] * f;
    }
    out[(size_t)h * hd + d] = A / Lsum;
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
// without a host round trip).  ctl = [token, pos, count].
__global__ void k_advance(const unsigned long long *best, int *ctl, int *hist, int cap) {
    if (threadIdx.x != 0) return;
    const int next = (int)(0xffffffffu - (uint32_t)(*best & 0xffffffffull));
    const int c = ctl[2];
    if (c < cap) hist[c] = next;
    ctl[0] = next;
    ctl[1] += 1;
    ctl[2] = c + 1;
}

__global__ void k_fill_f32(float *out, long n, float v) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) out[i] = v;
}

}  // namespace m27b
