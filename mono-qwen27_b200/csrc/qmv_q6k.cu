// qmv_q6k.cu — q6_K matvec instantiations over the tiled layout
// (qmv_q6k_tile.cuh), batch 1..4, store / SwiGLU / argmax epilogues.
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"
#include "qmv_q6k_tile.cuh"

namespace m27b {

static size_t q6t_smem_for(int nwarps, int k, int nt) {
    return (size_t)nwarps * Q6T_WARP_BYTES + q6t_x_bytes(k, nt) + q6t_part_bytes(nt) + 32;
}

template <int NT, int EPI>
static cudaError_t run_q6t(const QmvArgs &a, int sm_count, cudaStream_t st) {
    auto kern = k_qmv_q6k_tile<NT, EPI>;
    const int nw = q6t_warps(a.k, NT);
    if (nw < 1) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static size_t opted[64] = {0};
    const size_t smem_max = q6t_smem_for(nw, a.k, NT);
    if (smem_max > 48 * 1024 && (dev >= 64 || smem_max > opted[dev])) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = smem_max;
    }
    const long groups = (a.rows + 7) / 8;
    const int P = (a.rb + 3) / 4;
    // two resident CTAs per SM (shared memory <= 112 KB each), or one for
    // shapes whose staged activations leave two CTAs too few warps
    const long slots = (long)sm_count * q6t_ctas_per_sm(a.k, NT);
    int split, nthreads;
    long grid;
    size_t smem;
    const bool one_per_sm = q6t_ctas_per_sm(a.k, NT) == 1;
    if (P < 2 || (one_per_sm ? groups >= 4 * slots * nw : 2 * groups >= slots * nw)) {
        // every warp streams whole row groups
        split = 1;
        const long max_warps = slots * nw;
        const long gpw = (groups + max_warps - 1) / max_warps;
        const long warps = (groups + gpw - 1) / gpw;
        grid = (warps + nw - 1) / nw;
        nthreads = nw * 32;
        smem = smem_max;
    } else {
        // few row groups: the warps of a CTA split each group's tiles
        split = P < nw ? P : nw;
        // one CTA per resident slot; CTA c takes groups c, c + grid, ...: the
        // two CTAs an SM holds then carry (nearly) the same number of groups,
        // and the SMs differ by at most one group
        grid = groups < slots ? groups : slots;
        nthreads = split * 32;
        smem = q6t_smem_for(split, a.k, NT);
    }
    CUtensorMap tm0, tm1;
    if (!encode_rows_u32(&tm0, a.w0, a.row_stride, a.rows, Q6T_TILE / 4)) return cudaErrorInvalidValue;
    if (EPI == EPI_SWIGLU) {
        if (!encode_rows_u32(&tm1, a.w1, a.row_stride, a.rows, Q6T_TILE / 4)) return cudaErrorInvalidValue;
    } else {
        tm1 = tm0;
    }
    return launch_pdl(kern, dim3((unsigned)grid), dim3(nthreads), smem, st, a, tm0, tm1, split);
}

template <int EPI>
static cudaError_t run_q6t_nt(int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return run_q6t<1, EPI>(a, sm_count, st);
    case 2: return run_q6t<2, EPI>(a, sm_count, st);
    case 3: return run_q6t<3, EPI>(a, sm_count, st);
    case 4: return run_q6t<4, EPI>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

template <>
cudaError_t run_qmv_format<W_Q6KP>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (epi) {
    case EPI_STORE: return run_q6t_nt<EPI_STORE>(nt, a, sm_count, st);
    case EPI_SWIGLU: return run_q6t_nt<EPI_SWIGLU>(nt, a, sm_count, st);
    case EPI_ARGMAX: return run_q6t_nt<EPI_ARGMAX>(nt, a, sm_count, st);
    case EPI_PUSH: return nt == 1 ? run_q6t<1, EPI_PUSH>(a, sm_count, st) : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
