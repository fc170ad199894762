// attn_common.cuh — device helpers of the decode step's attention kernels
// (engine_kernels.cu): split counts, per-lane row loads, asynchronous row
// copies, and the q/k RMSNorm + rotary embedding of one head by one warp.
#pragma once

#include "m27b_device.cuh"

namespace m27b {

constexpr int ATT_G = 8;         // most query heads per kv head
constexpr int ATT_MIN_POS = 16;  // fewest positions per split

M27B_DI int att_splits(int L, int smax) {
    const int s = (L + ATT_MIN_POS - 1) / ATT_MIN_POS;
    return s < smax ? s : smax;
}

template <int DPL>
M27B_DI void ld_dims(const float *p, float (&v)[DPL]) {
    if constexpr (DPL % 4 == 0) {
#pragma unroll
        for (int c = 0; c < DPL / 4; ++c) {
            const float4 t = reinterpret_cast<const float4 *>(p)[c];
            v[4 * c] = t.x; v[4 * c + 1] = t.y; v[4 * c + 2] = t.z; v[4 * c + 3] = t.w;
        }
    } else if constexpr (DPL % 2 == 0) {
#pragma unroll
        for (int c = 0; c < DPL / 2; ++c) {
            const float2 t = reinterpret_cast<const float2 *>(p)[c];
            v[2 * c] = t.x; v[2 * c + 1] = t.y;
        }
    } else {
#pragma unroll
        for (int c = 0; c < DPL; ++c) v[c] = p[c];
    }
}

// A lane's DPL consecutive floats of a row (16-, 8- or 4-byte aligned as DPL allows).
template <int DPL>
M27B_DI void cp_async_dims(float *dst, const float *src) {
    if constexpr (DPL % 4 == 0) {
#pragma unroll
        for (int c = 0; c < DPL / 4; ++c) cp_async16(dst + 4 * c, src + 4 * c);
    } else if constexpr (DPL == 2) {
        cp_async8(dst, src);
    } else {
#pragma unroll
        for (int c = 0; c < DPL; ++c) cp_async4(dst + c, src + c);
    }
}

// As norm_rope_warp, with the norm weights (nw, hd values) and the rotary
// factors (rope, n_rot / 2 pairs) already in shared memory.
template <int DPL>
M27B_DI void norm_rope_apply(const float *src, const float *nw, const float2 *rope, float *dst, float mul, int n_rot,
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
        v[i] = v[i] * sc * nw[lane * DPL + i];
        dst[lane * DPL + i] = v[i];
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

}  // namespace m27b
