// qmv_launch.cuh — launch one instantiation of k_qmv with a balanced
// persistent grid.  Included by the per-format instantiation files.
#pragma once

#include <cuda.h>

#include "m27b_launch.cuh"
#include "qmv_kernels.cuh"

namespace m27b {

size_t qmv_smem_bytes(int wtype, int k, int ntok);

// Tensor map over weight rows viewed as [rows][row_bytes/4] uint32 with a box
// of box_rows rows x box_u32 words (one TMA copy per (row group, tile)).
// 2-D map over rows of uint32 words, box of box_u32 words x box_rows rows;
// swizzle 0 (none) or 32 / 64 / 128: the shared-memory swizzle span in bytes
// (16-byte chunk c of row r lands at chunk c ^ (r mod span / 16) for the
// 128-byte pattern; the box row must fit in the span).
bool encode_rows_u32(CUtensorMap *tm, const void *w, size_t row_bytes, int rows, int box_u32, int box_rows = 8,
                     int swizzle = 0);

template <int WT, int NT, int EPI, int PS>
cudaError_t run_qmv(const QmvArgs &a, int sm_count, cudaStream_t st) {
    auto kern = k_qmv<WT, NT, EPI, PS>;
    const size_t smem = qmv_smem_bytes(WT == W_Q80P ? M27B_TYPE_Q8_0 : M27B_TYPE_Q6_K, a.k, NT);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    // per device: largest dynamic smem opted in, and the resident CTAs per SM
    // for the last smem size queried
    static size_t opted[64] = {0};
    static size_t occ_smem[64] = {0};
    static int occ_val[64] = {0};
    if (smem > 48 * 1024 && (dev >= 64 || smem > opted[dev])) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = smem;
    }
    int occ = 0;
    if (dev < 64 && occ_val[dev] > 0 && occ_smem[dev] == smem) {
        occ = occ_val[dev];
    } else {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, QMV_THREADS, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) { occ_smem[dev] = smem; occ_val[dev] = occ; }
    }
    if (occ < 1) return cudaErrorInvalidConfiguration;
    // Balanced persistent grid: the fewest rows per warp that the resident
    // warps allow, then just enough warps for every warp to get that many.
    const long max_warps = (long)sm_count * occ * QMV_WARPS;
    const long rpw = (a.rows + max_warps - 1) / max_warps;
    const long warps = (a.rows + rpw - 1) / rpw;
    const long grid = (warps + QMV_WARPS - 1) / QMV_WARPS;
    return launch_pdl(kern, dim3((unsigned)grid), dim3(QMV_THREADS), smem, st, a);
}

template <int WT, int NT, int EPI, int PS>
cudaError_t run_qmv_capped(const QmvArgs &a, int sm_count, cudaStream_t st) {
    if constexpr (PS <= max_ps(WT, EPI, NT)) return run_qmv<WT, NT, EPI, PS>(a, sm_count, st);
    else return cudaErrorInvalidValue;
}

template <int WT, int NT, int EPI>
cudaError_t run_qmv_ps(QmvArgs a, int sm_count, cudaStream_t st) {
    const int ps = pick_ps(a.passes, max_ps(WT, EPI, NT));
    a.segs = (a.passes + ps - 1) / ps;
    switch (ps) {
    case 1: return run_qmv_capped<WT, NT, EPI, 1>(a, sm_count, st);
    case 2: return run_qmv_capped<WT, NT, EPI, 2>(a, sm_count, st);
    case 3: return run_qmv_capped<WT, NT, EPI, 3>(a, sm_count, st);
    case 4: return run_qmv_capped<WT, NT, EPI, 4>(a, sm_count, st);
    case 5: return run_qmv_capped<WT, NT, EPI, 5>(a, sm_count, st);
    case 6: return run_qmv_capped<WT, NT, EPI, 6>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

template <int WT, int EPI>
cudaError_t run_qmv_nt(int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return run_qmv_ps<WT, 1, EPI>(a, sm_count, st);
    case 2: return run_qmv_ps<WT, 2, EPI>(a, sm_count, st);
    case 3: return run_qmv_ps<WT, 3, EPI>(a, sm_count, st);
    case 4: return run_qmv_ps<WT, 4, EPI>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

// Defined once per weight format (qmv_q4k.cu, qmv_q6k.cu, qmv_q80.cu).
template <int WT>
cudaError_t run_qmv_format(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st);

#define M27B_DEFINE_QMV_FORMAT(WT)                                                                                     \
    template <>                                                                                                        \
    cudaError_t run_qmv_format<WT>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {                \
        switch (epi) {                                                                                                 \
        case EPI_STORE: return run_qmv_nt<WT, EPI_STORE>(nt, a, sm_count, st);                                         \
        case EPI_SWIGLU: return run_qmv_nt<WT, EPI_SWIGLU>(nt, a, sm_count, st);                                       \
        case EPI_ARGMAX: return run_qmv_nt<WT, EPI_ARGMAX>(nt, a, sm_count, st);                                       \
        default: return cudaErrorInvalidValue;                                                                         \
        }                                                                                                              \
    }

}  // namespace m27b
