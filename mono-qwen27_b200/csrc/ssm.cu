// ssm.cu — the Gated DeltaNet block of the hybrid model's recurrent layers
// (reference decode step src/mono27b_executor.cu:2484-2548), one token.
//
//   k_rmsnorm_row    x -> RMSNorm(x) * w                    (l_rms, :2491)
//   k_ssm_conv_qk    causal conv + SiLU over the q|k|v channels with the
//                    per-layer conv state (k_ssm_conv1d_u :1488-1501), L2
//                    norm of each q and k group (k_l2_norm_g :1118-1133), and
//                    beta = sigmoid(b), g = softplus(a + dt_bias) * ssm_a
//                    (k_ssm_params_fused :816-826)
//   k_ssm_delta      the gated delta rule per value head (k_deltanet_ggml
//                    :1526-1603), then RMSNorm(o) * ssm_norm * silu(z)
//                    (k_rms_norm_mulw_mul_batched :735-765) quantized to
//                    q8_K for ssm_out — one kernel, so the 6144-wide output
//                    never round-trips through global memory in fp32
//
// Layout: the conv channels are [q: n_group x 128 | k: n_group x 128 |
// v: dt_rank x 128]; value head j uses q/k group j % n_group (ggml's
// broadcast, as the reference kernel indexes it); the state of head j is
// S_j[col][i] (col = value dim, i = key dim), 128 x 128 fp32, the reference's
// transposed layout.  Key and value heads are 128 wide (the reference's
// S_v = 128).  Arithmetic is fp32 as in the reference; the L2 norm's sum of
// squares is accumulated in fp64 as there.
#include "m27b_device.cuh"
#include "m27b_launch.cuh"
#include "q8k_warp.cuh"

namespace m27b {

constexpr int SSM_HD = 128;  // key / value head width

M27B_DI float silu_f(float x) { return x / (1.0f + expf(-x)); }

// y = RMSNorm(x) * w over n values; one CTA of 512 threads.
__global__ void __launch_bounds__(512) k_rmsnorm_row(const float *x, const float *w, float eps, int n, float *y) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float scale = 1.0f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = scale * x[i] * w[i];
}

// grid = conv_ch / 128, block 128: thread = channel.  CTAs [0, 2*ng) hold
// the q and k groups and L2-normalise them; CTA 0 also turns the beta/alpha
// projections ba = [b (dr) | a (dr)] into bg = [beta (dr) | g (dr)].
__global__ void __launch_bounds__(SSM_HD) k_ssm_conv_qk(const float *x, const float *w, float *cstate, float *out,
                                                         const float *ba, const float *dt_bias, const float *ssm_a,
                                                         float *bg, int K, int n_qk_ctas, int dr, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ double red[SSM_HD];
    const int c = blockIdx.x * SSM_HD + threadIdx.x;
    const int sl = K - 1;
    float *st = cstate + (size_t)c * sl;
    const float *wc = w + (size_t)c * K;
    float s = 0.0f;
    for (int j = 0; j < sl; ++j) s += st[j] * wc[j];
    const float xin = x[c];
    s += xin * wc[sl];
    for (int j = 0; j + 1 < sl; ++j) st[j] = st[j + 1];
    if (sl > 0) st[sl - 1] = xin;
    float v = silu_f(s);
    if ((int)blockIdx.x < n_qk_ctas) {
        red[threadIdx.x] = (double)v * (double)v;
        __syncthreads();
        for (int step = SSM_HD / 2; step > 0; step >>= 1) {
            if ((int)threadIdx.x < step) red[threadIdx.x] += red[threadIdx.x + step];
            __syncthreads();
        }
        v *= 1.0f / sqrtf(fmaxf((float)red[0], eps * eps));
    }
    out[c] = v;
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < dr; i += blockDim.x) {
            bg[i] = 1.0f / (1.0f + expf(-ba[i]));
            const float z = ba[dr + i] + dt_bias[i];
            const float sp = z > 20.0f ? z : logf(1.0f + expf(z));
            bg[dr + i] = sp * ssm_a[i];
        }
}

// grid = dr / 2 (a CTA owns value heads 2b, 2b+1 = q8_K block b of the
// output), block 512 = 16 warps: warp w takes head 2b + w/8 and its 16 value
// columns (w%8)*16 .. +15; lane holds key rows lane + 32r of a column.
__global__ void __launch_bounds__(512) k_ssm_delta(const float *xc, const float *bg, const float *z,
                                                    const float *ssm_norm, float *S, m27b_block_q8_K *out, int ng,
                                                    int dr, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float qs[2][SSM_HD], ks[2][SSM_HD], vs[2][SSM_HD], os[2][SSM_HD];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h0 = 2 * blockIdx.x;
    if (tid < 2 * SSM_HD) {
        const int hh = tid >> 7, i = tid & (SSM_HD - 1), gi = (h0 + hh) % ng;
        qs[hh][i] = xc[(size_t)gi * SSM_HD + i];
        ks[hh][i] = xc[(size_t)(ng + gi) * SSM_HD + i];
        vs[hh][i] = xc[(size_t)2 * ng * SSM_HD + (size_t)(h0 + hh) * SSM_HD + i];
    }
    __syncthreads();
    {
        const int hh = warp >> 3, col0 = (warp & 7) * 16, h = h0 + hh;
        const float beta = bg[h], gv = expf(bg[dr + h]);
        float kr[4], qr[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            kr[r] = ks[hh][lane + 32 * r];
            qr[r] = qs[hh][lane + 32 * r];
        }
        float *Sh = S + (size_t)h * SSM_HD * SSM_HD;
        float sv[16][4];
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) sv[j][r] = Sh[(size_t)(col0 + j) * SSM_HD + lane + 32 * r];
        const float oscale = 1.0f / sqrtf((float)SSM_HD);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            float kv = 0.0f;
#pragma unroll
            for (int r = 0; r < 4; ++r) kv += sv[j][r] * kr[r];
            kv = warp_sum(kv);
            const float delta = (vs[hh][col0 + j] - gv * kv) * beta;
            float att = 0.0f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                sv[j][r] = gv * sv[j][r] + kr[r] * delta;
                att += sv[j][r] * qr[r];
            }
            att = warp_sum(att);
            if (lane == 0) os[hh][col0 + j] = att * oscale;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) Sh[(size_t)(col0 + j) * SSM_HD + lane + 32 * r] = sv[j][r];
    }
    __syncthreads();
    if (warp == 0) {
        // lanes 0-15: head 2b, lanes 16-31: head 2b+1; 8 values each
        const int hh = lane >> 4, base = (lane & 15) * 8, h = h0 + hh;
        float v[8];
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = os[hh][base + j];
            ss = fmaf(v[j], v[j], ss);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float scale = 1.0f / sqrtf(ss / (float)SSM_HD + eps);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            v[j] = (scale * v[j] * ssm_norm[base + j]) * silu_f(z[(size_t)h * SSM_HD + base + j]);
        quant_q8K_warp(v, lane, out + blockIdx.x);
    }
}

// Seeded pseudo-random fp32 fill, uniform in [offset - scale, offset + scale]
// (synthetic weights for the benchmark's hybrid model).
__global__ void k_fill_f32_rand(float *out, long n, uint64_t seed, float scale, float offset) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        uint64_t s = seed ^ (0x9e3779b97f4a7c15ull * (uint64_t)(i + 1));
        s ^= s >> 30;
        s *= 0xbf58476d1ce4e5b9ull;
        s ^= s >> 27;
        s *= 0x94d049bb133111ebull;
        s ^= s >> 31;
        const float u = (float)(s >> 40) * (1.0f / 16777216.0f);  // [0, 1)
        out[i] = offset + scale * (2.0f * u - 1.0f);
    }
}

cudaError_t ssm_rmsnorm_launch(const float *x, const float *w, float eps, int n, float *y, cudaStream_t st) {
    return launch_pdl(k_rmsnorm_row, dim3(1), dim3(512), 0, st, x, w, eps, n, y);
}

cudaError_t ssm_conv_launch(const float *x, const float *w, float *cstate, float *out, const float *ba,
                            const float *dt_bias, const float *ssm_a, float *bg, int conv_ch, int K, int ng, int dr,
                            float eps, cudaStream_t st) {
    if (conv_ch % SSM_HD) return cudaErrorInvalidValue;
    return launch_pdl(k_ssm_conv_qk, dim3(conv_ch / SSM_HD), dim3(SSM_HD), 0, st, x, w, cstate, out, ba, dt_bias,
                      ssm_a, bg, K, 2 * ng, dr, eps);
}

cudaError_t ssm_delta_launch(const float *xc, const float *bg, const float *z, const float *ssm_norm, float *S,
                             void *xq, int ng, int dr, float eps, cudaStream_t st) {
    if (dr % 2) return cudaErrorInvalidValue;
    return launch_pdl(k_ssm_delta, dim3(dr / 2), dim3(512), 0, st, xc, bg, z, ssm_norm, S, (m27b_block_q8_K *)xq, ng,
                      dr, eps);
}

}  // namespace m27b
