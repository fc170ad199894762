// qmv_q4k.cu — q4_K matvec instantiations: one super-block per lane
// (qmv_blk.cuh), batch 1..4, store / SwiGLU / argmax epilogues.
#include <cudaTypedefs.h>

#include "qmv_blk.cuh"
#include "qmv_launch.cuh"

namespace m27b {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// Tensor map over q4_K rows viewed as [rows][row_bytes/4] uint32 with a box of
// 8 rows x 144 uint32 (4 blocks): one TMA copy per (8-row group, pass).
static bool encode_rows(CUtensorMap *tm, const void *w, size_t row_bytes, int rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t gdim[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {144, 8};
    const cuuint32_t estride[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), gdim, gstride, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int EPI>
static cudaError_t run_blk(const QmvArgs &a, int sm_count, cudaStream_t st) {
    auto kern = k_qmv_q4k_blk<NT, EPI>;
    const int nw = blk_warps(a.k, NT);
    if (nw < 1) return cudaErrorInvalidValue;
    const size_t smem = blk_smem_bytes(a.k, NT);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
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
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, nw * 32, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) { occ_smem[dev] = smem; occ_val[dev] = occ; }
    }
    if (occ < 1) return cudaErrorInvalidConfiguration;
    // balanced persistent grid over groups of 8 rows
    const long groups = (a.rows + 7) / 8;
    const long max_warps = (long)sm_count * occ * nw;
    const long gpw = (groups + max_warps - 1) / max_warps;
    const long warps = (groups + gpw - 1) / gpw;
    const long grid = (warps + nw - 1) / nw;
    CUtensorMap tm0, tm1;
    if (!encode_rows(&tm0, a.w0, a.row_stride, a.rows)) return cudaErrorInvalidValue;
    if (EPI == EPI_SWIGLU) {
        if (!encode_rows(&tm1, a.w1, a.row_stride, a.rows)) return cudaErrorInvalidValue;
    } else {
        tm1 = tm0;
    }
    kern<<<(unsigned)grid, nw * 32, smem, st>>>(a, tm0, tm1);
    return cudaGetLastError();
}

template <int EPI>
static cudaError_t run_blk_nt(int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return run_blk<1, EPI>(a, sm_count, st);
    case 2: return run_blk<2, EPI>(a, sm_count, st);
    case 3: return run_blk<3, EPI>(a, sm_count, st);
    case 4: return run_blk<4, EPI>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

template <>
cudaError_t run_qmv_format<W_Q4K>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (epi) {
    case EPI_STORE: return run_blk_nt<EPI_STORE>(nt, a, sm_count, st);
    case EPI_SWIGLU: return run_blk_nt<EPI_SWIGLU>(nt, a, sm_count, st);
    case EPI_ARGMAX: return run_blk_nt<EPI_ARGMAX>(nt, a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
