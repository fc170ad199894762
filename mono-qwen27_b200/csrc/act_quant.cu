// act_quant.cu — fp32 activations -> ggml q8_K / q8_0 blocks on sm_100a.
//
// Replaces the reference's q8_1 activation quantizers k_quant_q8_1 and
// k_quant_q8_1_fused_gate (src/mono27b_executor.cu:84-138).  The output is
// ggml's block_q8_K / block_q8_0, bit for bit what quantize_row_q8_K_ref /
// quantize_row_q8_0_ref produce on the CPU, so the matvec results follow
// ggml's vec_dot_q4_K_q8_K / q6_K_q8_K / q8_0_q8_0 semantics.
//
// q8_K (per 256 values, one warp, 8 values per lane):
//   m = signed value of largest |x| (first one on ties); iscale = -127/m;
//   q = min(127, round_half_even(iscale*x)); d = 1/iscale; bsums = sums of 16.
// q8_0 (per 32 values, one warp, one value per lane):
//   d = amax/127 (stored fp16, round-to-nearest-even); q = roundf(x * (1/d)).
//
// Modes: plain x; x * sigmoid(gate) (the gated attention output feeding
// o_proj, reference :2452-2473); RMSNorm(x) * w (the norm that precedes every
// projection, reference l_rms :2139-2141).  IEEE division and expf are used
// (no fast-math) so plain-mode output is bit-exact.
#include "m27b_device.cuh"
#include "m27b_launch.cuh"

namespace m27b {

// Row scale for ACT_RMSNORM: 1/sqrt(mean(x^2) + eps), block-wide reduction.
template <int MODE>
M27B_DI float row_norm_scale(const ActArgs &a, const float *xr) {
    if (MODE != ACT_RMSNORM) return 1.0f;
    __shared__ float red[32];
    // independent partial sums over 16-byte loads keep several loads in flight
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    const int bd = blockDim.x;
    if ((a.k & 3) == 0 && ((uintptr_t)xr & 15) == 0) {
        const float4 *x4 = (const float4 *)xr;
        const int n4 = a.k >> 2;
        int i = threadIdx.x;
        for (; i + 3 * bd < n4; i += 4 * bd) {
            const float4 v0 = x4[i], v1 = x4[i + bd], v2 = x4[i + 2 * bd], v3 = x4[i + 3 * bd];
            s0 = fmaf(v0.x, v0.x, fmaf(v0.y, v0.y, fmaf(v0.z, v0.z, fmaf(v0.w, v0.w, s0))));
            s1 = fmaf(v1.x, v1.x, fmaf(v1.y, v1.y, fmaf(v1.z, v1.z, fmaf(v1.w, v1.w, s1))));
            s2 = fmaf(v2.x, v2.x, fmaf(v2.y, v2.y, fmaf(v2.z, v2.z, fmaf(v2.w, v2.w, s2))));
            s3 = fmaf(v3.x, v3.x, fmaf(v3.y, v3.y, fmaf(v3.z, v3.z, fmaf(v3.w, v3.w, s3))));
        }
        for (; i < n4; i += bd) {
            const float4 v0 = x4[i];
            s0 = fmaf(v0.x, v0.x, fmaf(v0.y, v0.y, fmaf(v0.z, v0.z, fmaf(v0.w, v0.w, s0))));
        }
    } else {
        for (int i = threadIdx.x; i < a.k; i += bd) s0 = fmaf(xr[i], xr[i], s0);
    }
    float s = warp_sum((s0 + s1) + (s2 + s3));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.0f;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) tot += red[i];
    return 1.0f / sqrtf(tot / (float)a.k + a.eps);
}

template <int MODE>
M27B_DI float act_value(const ActArgs &a, const float *xr, const float *gr, int i, float nscale) {
    float v = xr[i];
    if (MODE == ACT_GATED) {
        const float g = gr[i];
        v = v * (1.0f / (1.0f + expf(-g)));
    } else if (MODE == ACT_RMSNORM) {
        v = v * nscale;
        if (a.w) v = v * a.w[i];
    }
    return v;
}

// grid (ceil(nblocks/8), n_tok), block 256: warp w of CTA c quantizes
// super-block 8c + w of token blockIdx.y.
template <int MODE>
__global__ void __launch_bounds__(256) k_act_quant_q8K(ActArgs a) {
    pdl_trigger();
    pdl_wait();  // x is produced by the previous kernel
    const int t = blockIdx.y;
    const float *xr = a.x + (size_t)t * a.ldx;
    const float *gr = a.gate ? a.gate + (size_t)t * a.ldx : nullptr;
    const float ns = row_norm_scale<MODE>(a, xr);
    const int nb = a.k / 256;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nb) return;
    m27b_block_q8_K *ob = (m27b_block_q8_K *)a.out + (size_t)t * nb + b;

    float v[8];
    float best_a = 0.0f, best_v = 0.0f;
    int best_i = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = act_value<MODE>(a, xr, gr, b * 256 + lane * 8 + j, ns);
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
    uint32_t packed[2] = {0u, 0u};
    int s = 0;
    float d = 0.0f;
    if (best_a != 0.0f) {
        const float iscale = -127.0f / best_v;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int q = __float2int_rn(iscale * v[j]);
            q = q > 127 ? 127 : q;
            s += q;
            packed[j >> 2] |= ((uint32_t)q & 0xffu) << (8 * (j & 3));
        }
        d = 1.0f / iscale;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint32_t *qw = (uint32_t *)((uint8_t *)ob + 4 + 8 * lane);  // 4-byte aligned
    qw[0] = packed[0];
    qw[1] = packed[1];
    if ((lane & 1) == 0) ob->bsums[lane >> 1] = (int16_t)s;
    if (lane == 0) ob->d = d;
}

// grid (ceil(nblocks/8), n_tok), block 256: warp w of CTA c quantizes q8_0
// block 8c + w (32 values, one per lane).
template <int MODE>
__global__ void __launch_bounds__(256) k_act_quant_q80(ActArgs a) {
    pdl_trigger();
    pdl_wait();  // x is produced by the previous kernel
    const int t = blockIdx.y;
    const float *xr = a.x + (size_t)t * a.ldx;
    const float *gr = a.gate ? a.gate + (size_t)t * a.ldx : nullptr;
    const float ns = row_norm_scale<MODE>(a, xr);
    const int nb = a.k / 32;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nb) return;
    const float v = act_value<MODE>(a, xr, gr, b * 32 + lane, ns);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    m27b_block_q8_0 *ob = (m27b_block_q8_0 *)a.out + (size_t)t * nb + b;
    ob->qs[lane] = (int8_t)roundf(v * id);
    if (lane == 0) ob->d = __half_as_ushort(__float2half_rn(d));
}

cudaError_t launch_act_quant(int act_type, int mode, const ActArgs &a, int n_tok, cudaStream_t st) {
    const int nb = act_type == M27B_TYPE_Q8_K ? a.k / 256 : a.k / 32;
    dim3 grid((nb + 7) / 8, n_tok);
    if (act_type == M27B_TYPE_Q8_K) {
        if (mode == ACT_PLAIN) return launch_pdl(k_act_quant_q8K<ACT_PLAIN>, grid, dim3(256), 0, st, a);
        if (mode == ACT_GATED) return launch_pdl(k_act_quant_q8K<ACT_GATED>, grid, dim3(256), 0, st, a);
        return launch_pdl(k_act_quant_q8K<ACT_RMSNORM>, grid, dim3(256), 0, st, a);
    }
    if (mode == ACT_PLAIN) return launch_pdl(k_act_quant_q80<ACT_PLAIN>, grid, dim3(256), 0, st, a);
    if (mode == ACT_GATED) return launch_pdl(k_act_quant_q80<ACT_GATED>, grid, dim3(256), 0, st, a);
    return launch_pdl(k_act_quant_q80<ACT_RMSNORM>, grid, dim3(256), 0, st, a);
}

}  // namespace m27b
