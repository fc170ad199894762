// qmv.cu — batch 1..4 quantized matvec over GGUF k-quant blocks on sm_100a.
//
// Replaces the reference's one-row-per-CTA dp4a kernels
//   k_q4k_mv_q8_dp4a       src/mono27b_executor.cu:320-364
//   k_q4k_q4k_swiglu_dp4a  src/mono27b_executor.cu:369-417
//   k_q6k_mv_q8_dp4a       src/mono27b_executor.cu:630-645
//   k_q80_mv_q8_dp4a       src/mono27b_executor.cu:533-580
//   lm_head + k_argmax     src/mono27b_executor.cu:2577-2593, :209-239
// with a persistent, HBM-streaming design:
//
//  * grid = just enough 8-warp CTAs (at most #SMs x resident CTAs) for every
//    warp to own the same number of rows; warp w owns rows w, w + W, ... so
//    that all warps sweep the matrix front to back together;
//  * a row is walked in "passes" of 1024 values: in each pass lane L owns one
//    16-byte slice of super-block 4p + L/8 (q4_K / q6_K) or block 32p + L
//    (q8_0) — 32 weights — and fetches it with a 128-bit streaming load;
//  * a warp's work is a sequence of units of PS passes (a whole row when it
//    has at most 6 passes); units are double-buffered in registers, so the
//    loads of the next unit are in flight while the current one is multiplied;
//  * the activations (ggml q8_K / q8_0 blocks of up to 4 tokens) are staged
//    once per CTA in shared memory in planar form (codes | bsum pairs |
//    scales), and every weight slice is reused for all tokens from registers;
//  * integer dot products per 16-value group (dp4a; u8 x s8 for the unsigned
//    nibbles), the 6-bit q4_K scale/min unpacking and the q6_K 2-bit
//    high-plane merge happen in registers; dp2a applies the two sub-block
//    scales (and the two mins against the bsums) in one instruction each.
//    Integer partial sums equal ggml's vec_dot_q4_K_q8_K / q6_K_q8_K /
//    q8_0_q8_0; only the order of the fp32 accumulation differs.
//
// q6_K and q8_0 tensors are read in the planar layout written by m27b_repack
// (repack.cu), because their GGUF blocks (210 B / 34 B) are only 2-byte
// aligned; q4_K blocks (144 B) are read in place.
#include <cudaTypedefs.h>

#include "qmv_blk.cuh"
#include "qmv_launch.cuh"
#include "qmv_q6k_tile.cuh"

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

bool encode_rows_u32(CUtensorMap *tm, const void *w, size_t row_bytes, int rows, int box_u32, int box_rows,
                     int swizzle) {
    auto enc = tensor_map_encoder();
    if (!enc || (row_bytes & 15) != 0 || ((uintptr_t)w & 15) != 0) return false;
    const CUtensorMapSwizzle sw = swizzle == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : swizzle == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle && box_u32 * 4 > swizzle) return false;
    const cuuint64_t gdim[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_u32, (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), gdim, gstride, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Dynamic shared memory bytes for the staged activations.
size_t qmv_smem_bytes(int wtype, int k, int ntok) {
    if (wtype == M27B_TYPE_Q8_0) return (size_t)ntok * k + (size_t)ntok * (k / 32) * 4;
    if (wtype == M27B_TYPE_Q4_K) return blk_warps(k, ntok) > 0 ? blk_smem_bytes(k, ntok) : 0;  // qmv_blk.cuh
    if (wtype == M27B_TYPE_Q5_K) return blk_warps(k, ntok, 176) > 0 ? blk_smem_bytes(k, ntok, 176) : 0;
    if (wtype == M27B_TYPE_IQ4_XS) return blk_warps(k, ntok, 136) > 0 ? blk_smem_bytes(k, ntok, 136) : 0;
    if (wtype == M27B_TYPE_Q6_K) return q6t_warps(k, ntok) > 0 ? q6t_smem_bytes(k, ntok) : 0;   // qmv_q6k_tile.cuh
    return (size_t)ntok * k + (size_t)ntok * (k / 256) * 32 + (size_t)ntok * (k / 256) * 4;
}

cudaError_t launch_qmv(int wt, int epi, QmvArgs a, int nt, int sm_count, cudaStream_t st) {
    switch (wt) {
    case W_Q4K: return run_qmv_format<W_Q4K>(epi, nt, a, sm_count, st);
    case W_Q6KP: return run_qmv_format<W_Q6KP>(epi, nt, a, sm_count, st);
    case W_Q80P: return run_qmv_format<W_Q80P>(epi, nt, a, sm_count, st);
    case W_Q5K: return run_qmv_format<W_Q5K>(epi, nt, a, sm_count, st);
    case W_IQ4XS: return run_qmv_format<W_IQ4XS>(epi, nt, a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
