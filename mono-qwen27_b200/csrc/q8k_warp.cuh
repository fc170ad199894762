// q8k_warp.cuh — ggml q8_K quantization of one 256-value super-block by one
// warp (shared by the activation quantizers, the fused attention epilogue and
// the matvec prologues that quantize their own activations, so that every
// path produces the same codes).
#pragma once

#include "m27b_blocks.h"
#include "m27b_device.cuh"

namespace m27b {

// ggml q8_K of one super-block, 8 values per lane (lane l holds values
// 8l..8l+7): m = signed value of largest |x| (first one on ties),
// iscale = -127/m, q = min(127, rne(iscale*x)), d = 1/iscale.  Returns the
// lane's 8 codes packed in two words, their sum, and d.
M27B_DI void quant_q8K_lane(const float (&v)[8], int lane, uint32_t (&packed)[2], int &sum, float &d) {
    float best_a = 0.0f, best_v = 0.0f;
    int best_i = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float av = fabsf(v[j]);
        if (av > best_a) { best_a = av; best_v = v[j]; best_i = lane * 8 + j; }
    }
    // (|x| desc, index asc) is a total order, so the butterfly converges on
    // the first element of largest magnitude in every lane.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, best_a, o);
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (oa > best_a || (oa == best_a && oi < best_i)) { best_a = oa; best_v = ov; best_i = oi; }
    }
    packed[0] = packed[1] = 0u;
    sum = 0;
    d = 0.0f;
    if (best_a != 0.0f) {
        const float iscale = -127.0f / best_v;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int q = __float2int_rn(iscale * v[j]);
            q = q > 127 ? 127 : q;
            sum += q;
            packed[j >> 2] |= ((uint32_t)q & 0xffu) << (8 * (j & 3));
        }
        d = 1.0f / iscale;
    }
}

// ... written as ggml's block_q8_K (codes, d, bsums of 16).
M27B_DI void quant_q8K_warp(const float (&v)[8], int lane, m27b_block_q8_K *ob) {
    uint32_t packed[2];
    int s;
    float d;
    quant_q8K_lane(v, lane, packed, s, d);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint32_t *qw = (uint32_t *)((uint8_t *)ob + 4 + 8 * lane);  // 4-byte aligned
    qw[0] = packed[0];
    qw[1] = packed[1];
    if ((lane & 1) == 0) ob->bsums[lane >> 1] = (int16_t)s;
    if (lane == 0) ob->d = d;
}

}  // namespace m27b
