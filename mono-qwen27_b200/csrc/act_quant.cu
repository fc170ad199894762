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
// projection, reference l_rms :2139-2141); silu(gate) * x (the FFN activation
// feeding ffn_down when gate and up were computed as separate matvecs; the
// same fp32 expression as the matvec SwiGLU epilogue).  IEEE division and expf are used
// (no fast-math) so plain-mode output is bit-exact.
#include "m27b_device.cuh"
#include "m27b_launch.cuh"
#include "q8k_warp.cuh"

namespace m27b {

// Row scale for ACT_RMSNORM: 1/sqrt(mean(x^2) + eps), block-wide reduction
// (used when the row cannot be staged in shared memory).
template <int MODE>
M27B_DI float row_norm_scale(const ActArgs &a, const float *xr) {
    if (MODE != ACT_RMSNORM) return 1.0f;
    __shared__ float red[32];
    float s0 = 0.0f;
    for (int i = threadIdx.x; i < a.k; i += blockDim.x) s0 = fmaf(xr[i], xr[i], s0);
    float s = warp_sum(s0);
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
    } else if (MODE == ACT_SWIGLU) {
        const float g = gr[i];
        v = g / (1.0f + expf(-g)) * v;
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
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = act_value<MODE>(a, xr, gr, b * 256 + lane * 8 + j, ns);
    quant_q8K_warp(v, lane, (m27b_block_q8_K *)a.out + (size_t)t * nb + b);
}

// RMSNorm(x) * w -> q8_K with the row staged once in shared memory: every
// value is read from global memory once (all loads issued up front), the sum
// of squares reduced over the CTA, and each warp quantizes a super-block from
// shared memory.  grid (ceil(nblocks/8), n_tok), block 256.
constexpr int NQ_MAX_K = 16384;  // largest row staged in shared memory (64 KB)
constexpr int M27B_MAX_SRC = 8;   // most source ranks of the fused all-reduce

__global__ void __launch_bounds__(256) k_norm_quant_q8K(ActArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();  // x is produced by the previous kernel
    const int t = blockIdx.y;
    const float4 *x4 = (const float4 *)(a.x + (size_t)t * a.ldx);
    float4 *xs4 = (float4 *)xs;
    const int n4 = a.k >> 2;
    float ss = 0.0f;
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += 256) {
        const float4 v = x4[i];
        xs4[i] = v;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    ss = warp_sum(ss);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float ns = 1.0f / sqrtf(tot / (float)a.k + a.eps);
    const int nb = a.k / 256;
    const int b = blockIdx.x * 8 + warp;
    if (b >= nb) return;
    float v[8];
    const float4 *p = (const float4 *)(xs + b * 256 + lane * 8);
    const float4 p0 = p[0], p1 = p[1];
    const float raw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float u = raw[j] * ns;
        if (a.w) u = u * a.w[b * 256 + lane * 8 + j];
        v[j] = u;
    }
    quant_q8K_warp(v, lane, (m27b_block_q8_K *)a.out + (size_t)t * nb + b);
}

// Consumer half of the fused all-reduce (ACT_RMSNORM_SUM): grid k/256, block
// 256; CTA b owns super-block b, thread i value 256b + i.  Each thread reads
// its value's word from every source rank (all loads in flight), re-reads any
// word whose epoch has not arrived yet (bounded), and sums them in rank order.
// The CTA's sum of squares goes to ss_words[b] as an epoch-tagged word; every
// CTA waits for all of them and adds them in CTA order, so every CTA (and
// every rank) computes the same norm.  Then warp 0 quantizes the super-block.
// The words order everything this kernel reads and writes against the
// producing matvec (which has staged its activations and read its residual
// before storing a row), so it does not wait for that grid to retire: it
// starts once the grid has triggered, when every producer CTA is resident.
// It triggers its own dependents at once; they launch only after all of its
// CTAs are resident, so none of them can be starved of an SM.
__global__ void __launch_bounds__(256) k_allreduce_norm_quant_q8K(ActArgs a) {
    __shared__ __align__(16) float xs[256];
    __shared__ float red[8];
    __shared__ float css[256];
    pdl_trigger();
    const uint32_t ep = *a.epoch_base * a.epoch_mul + a.epoch_add;
    const int b = blockIdx.x, nb = gridDim.x, i = b * 256 + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint2 w[M27B_MAX_SRC];
#pragma unroll
    for (int s = 0; s < M27B_MAX_SRC; ++s)
        if (s < a.nsrc) w[s] = ld_word(a.words + (size_t)s * a.src_stride + i);
    float v = 0.0f;
#pragma unroll
    for (int s = 0; s < M27B_MAX_SRC; ++s)
        if (s < a.nsrc) {
            w[s] = wait_word(a.words + (size_t)s * a.src_stride + i, w[s], ep, a.status, 3, a.wait_ns);
            v = s == 0 ? __uint_as_float(w[s].x) : v + __uint_as_float(w[s].x);
        }
    a.x_out[i] = v;
    xs[threadIdx.x] = v;
    const float sq = warp_sum(v * v);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        float c = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) c += red[k];
        st_word(a.ss_words + b, __float_as_uint(c), ep);
    }
    if ((int)threadIdx.x < nb) {
        const uint2 *q = a.ss_words + threadIdx.x;
        css[threadIdx.x] = __uint_as_float(wait_word(q, ld_word(q), ep, a.status, 3, a.wait_ns).x);
    }
    __syncthreads();
    if (warp != 0) return;
    float tot = 0.0f;
    for (int k = 0; k < nb; ++k) tot += css[k];
    const float ns = 1.0f / sqrtf(tot / (float)a.k + a.eps);
    const float4 *p = (const float4 *)(xs + lane * 8);
    const float4 p0 = p[0], p1 = p[1];
    const float raw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    float q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float u = raw[j] * ns;
        if (a.w) u = u * a.w[b * 256 + lane * 8 + j];
        q[j] = u;
    }
    quant_q8K_warp(q, lane, (m27b_block_q8_K *)a.out + b);
}

bool norm_quant_staged(const ActArgs &a) {
    return a.k <= NQ_MAX_K && (a.k & 3) == 0 && (a.ldx & 3) == 0 && ((uintptr_t)a.x & 15) == 0;
}

cudaError_t launch_norm_quant(const ActArgs &a, int n_tok, cudaStream_t st) {
    const int nb = a.k / 256;
    const dim3 grid((nb + 7) / 8, n_tok);
    const size_t smem = (size_t)a.k * sizeof(float);
    static bool opted[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (smem > 48 * 1024 && (dev >= 64 || !opted[dev])) {
        e = cudaFuncSetAttribute(k_norm_quant_q8K, cudaFuncAttributeMaxDynamicSharedMemorySize, NQ_MAX_K * 4);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = true;
    }
    return launch_pdl(k_norm_quant_q8K, grid, dim3(256), smem, st, a);
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
        if (mode == ACT_SWIGLU) return launch_pdl(k_act_quant_q8K<ACT_SWIGLU>, grid, dim3(256), 0, st, a);
        if (mode == ACT_RMSNORM_SUM) {
            if (n_tok != 1 || a.nsrc < 1 || a.nsrc > M27B_MAX_SRC || !a.words || !a.ss_words || !a.epoch_base ||
                !a.x_out || nb > 256)
                return cudaErrorInvalidValue;
            return launch_pdl(k_allreduce_norm_quant_q8K, dim3(nb), dim3(256), 0, st, a);
        }
        if (norm_quant_staged(a)) return launch_norm_quant(a, n_tok, st);
        return launch_pdl(k_act_quant_q8K<ACT_RMSNORM>, grid, dim3(256), 0, st, a);
    }
    if (mode == ACT_RMSNORM_SUM) return cudaErrorInvalidValue;
    if (mode == ACT_PLAIN) return launch_pdl(k_act_quant_q80<ACT_PLAIN>, grid, dim3(256), 0, st, a);
    if (mode == ACT_GATED) return launch_pdl(k_act_quant_q80<ACT_GATED>, grid, dim3(256), 0, st, a);
    if (mode == ACT_SWIGLU) return launch_pdl(k_act_quant_q80<ACT_SWIGLU>, grid, dim3(256), 0, st, a);
    return launch_pdl(k_act_quant_q80<ACT_RMSNORM>, grid, dim3(256), 0, st, a);
}

}  // namespace m27b
