// qmv_float.cu — f16 / f32 weight rows times fp32 activations, the
// reference's k_f16_mv and k_f32_mv (src/mono27b_executor.cu:900-916,
// :1101-1114; reached through l_mv_fallback, :2127-2137) for the small
// unquantized matrices of the hybrid model.  Semantics are ggml's: for f16
// weights the activation is rounded to fp16 first (the f16 vec_dot type);
// every product of two fp16 values is exact in fp32.  Sums are fp32 (ggml's
// generic code sums in double: the difference is fp32 rounding order).
//
// Streaming: each lane reads 16 bytes of a row per step (8 halves or 4
// floats), a warp 512 contiguous bytes, FV_UNROLL steps in flight per lane.
// Many rows: one warp per row (persistent over rows).  Few rows: one CTA per
// row, its warps take interleaved 16-byte chunks and their sums are combined
// in warp order (deterministic).  The activations are read from global
// memory (L1/L2 resident: at most 4 rows of k floats).
#include <algorithm>

#include "m27b_launch.cuh"
#include "qmv_kernels.cuh"

namespace m27b {

constexpr int FV_WARPS = 8;
constexpr int FV_THREADS = FV_WARPS * 32;
constexpr int FV_UNROLL = 4;

template <int WT>
struct FloatRow;

template <>
struct FloatRow<W_F16> {
    static constexpr int N = 8;  // values per 16 bytes
    static M27B_DI void vals(const uint4 &q, float (&v)[8]) {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = h2f(w[i]);
            v[2 * i + 1] = h2f(w[i] >> 16);
        }
    }
    static M27B_DI float xval(float x) { return __half2float(__float2half_rn(x)); }
};

template <>
struct FloatRow<W_F32> {
    static constexpr int N = 4;
    static M27B_DI void vals(const uint4 &q, float (&v)[4]) {
        v[0] = __uint_as_float(q.x);
        v[1] = __uint_as_float(q.y);
        v[2] = __uint_as_float(q.z);
        v[3] = __uint_as_float(q.w);
    }
    static M27B_DI float xval(float x) { return x; }
};

template <int WT, int NT>
__global__ void __launch_bounds__(FV_THREADS) k_qmv_float(const QmvArgs a, int split) {
    using R = FloatRow<WT>;
    constexpr int N = R::N;
    __shared__ float part[FV_WARPS][NT];
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunks = a.k / N;
    const int row0 = split == 1 ? (int)blockIdx.x * FV_WARPS + warp : (int)blockIdx.x;
    const int rstep = split == 1 ? (int)gridDim.x * FV_WARPS : (int)gridDim.x;
    const int c0 = split == 1 ? lane : warp * 32 + lane;
    const int cstep = split == 1 ? 32 : 32 * FV_WARPS;
    for (int row = row0; row < a.rows; row += rstep) {
        const uint4 *wr = (const uint4 *)(a.w0 + (size_t)row * a.row_stride);
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        for (int c = c0; c < chunks; c += cstep * FV_UNROLL) {
            uint4 q[FV_UNROLL];
#pragma unroll
            for (int u = 0; u < FV_UNROLL; ++u) {
                const int cc = c + u * cstep;
                q[u] = cc < chunks ? __ldcs(wr + cc) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < FV_UNROLL; ++u) {
                const int cc = c + u * cstep;
                if (cc < chunks) {
                    float v[N];
                    R::vals(q[u], v);
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float4 *xr = (const float4 *)(a.xf + (size_t)t * a.ldxf + (size_t)cc * N);
#pragma unroll
                        for (int j = 0; j < N / 4; ++j) {
                            const float4 x4 = xr[j];
                            acc[t] = fmaf(v[4 * j], R::xval(x4.x), acc[t]);
                            acc[t] = fmaf(v[4 * j + 1], R::xval(x4.y), acc[t]);
                            acc[t] = fmaf(v[4 * j + 2], R::xval(x4.z), acc[t]);
                            acc[t] = fmaf(v[4 * j + 3], R::xval(x4.w), acc[t]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = warp_sum(acc[t]);
        if (split > 1) {
            if (lane == 0)
#pragma unroll
                for (int t = 0; t < NT; ++t) part[warp][t] = acc[t];
            __syncthreads();
            if (warp == 0)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float s = 0.0f;
                    for (int w = 0; w < FV_WARPS; ++w) s += part[w][t];
                    acc[t] = s;
                }
            __syncthreads();
        }
        if (lane == 0 && (split == 1 || warp == 0)) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const size_t o = (size_t)t * a.ldy + row;
                a.y[o] = a.residual ? acc[t] + a.residual[o] : acc[t];
            }
        }
    }
}

template <int WT, int NT>
static cudaError_t run_float(const QmvArgs &a, int sm_count, cudaStream_t st) {
    // many rows: a warp per row over a grid of up to 8 CTAs per SM; few rows
    // (fewer than 16 per SM): a CTA per row
    const long slots = (long)sm_count * 8;
    if ((long)a.rows >= (long)sm_count * 16) {
        const long grid = std::min(slots, ((long)a.rows + FV_WARPS - 1) / FV_WARPS);
        return launch_pdl(k_qmv_float<WT, NT>, dim3((unsigned)grid), dim3(FV_THREADS), 0, st, a, 1);
    }
    const long grid = std::min(slots, (long)a.rows);
    return launch_pdl(k_qmv_float<WT, NT>, dim3((unsigned)grid), dim3(FV_THREADS), 0, st, a, FV_WARPS);
}

template <int WT>
static cudaError_t run_float_nt(int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return run_float<WT, 1>(a, sm_count, st);
    case 2: return run_float<WT, 2>(a, sm_count, st);
    case 3: return run_float<WT, 3>(a, sm_count, st);
    case 4: return run_float<WT, 4>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_qmv_float(int wt, const QmvArgs &a, int nt, int sm_count, cudaStream_t st) {
    if (wt == W_F16) return run_float_nt<W_F16>(nt, a, sm_count, st);
    if (wt == W_F32) return run_float_nt<W_F32>(nt, a, sm_count, st);
    return cudaErrorInvalidValue;
}

}  // namespace m27b
