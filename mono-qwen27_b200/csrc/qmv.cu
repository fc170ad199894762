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
//  * grid = (#SMs x resident CTAs), 8 warps per CTA; warp w of the grid owns
//    rows w, w + W, w + 2W, ... so that all warps sweep the matrix front to
//    back together;
//  * a row is walked in "passes" of 1024 values: in each pass lane L owns one
//    16-byte slice of super-block 4p + L/8 (q4_K / q6_K) or block 32p + L
//    (q8_0) — 32 weights — and fetches it with a 128-bit streaming load;
//  * each warp keeps a software pipeline of PM passes of loads in registers
//    (two register buffers, ping-pong) across row boundaries, so the loads of
//    the next rows are in flight while the current ones are multiplied;
//  * the activations (ggml q8_K / q8_0 blocks of up to 4 tokens) are staged
//    once per CTA in shared memory in planar form (codes | bsums | scales),
//    and every weight slice is reused for all tokens from registers;
//  * integer dp4a dot products per 16-value group, the 6-bit q4_K scale/min
//    unpacking and the q6_K 2-bit high-plane merge happen in registers;
//    per-slice integer sums are combined in fp32 exactly as ggml's
//    vec_dot_q4_K_q8_K / q6_K_q8_K / q8_0_q8_0 (same integer partial sums,
//    only the order of fp32 accumulation differs).
//
// q6_K and q8_0 tensors are read in the planar layout written by m27b_repack
// (repack.cu), because their GGUF blocks (210 B / 34 B) are only 2-byte
// aligned; q4_K blocks (144 B) are read in place.
#include "m27b_device.cuh"
#include "qmv_kernels.cuh"

namespace m27b {

// Dynamic shared memory bytes for the staged activations.
size_t qmv_smem_bytes(int wtype, int k, int ntok) {
    if (wtype == M27B_TYPE_Q8_0) return (size_t)ntok * k + (size_t)ntok * (k / 32) * 4;
    return (size_t)ntok * k + (size_t)ntok * (k / 16) * 2 + (size_t)ntok * (k / 256) * 4;
}

template <int WT, int NT, int EPI>
static cudaError_t launch_one(const QmvArgs &a, int sm_count, cudaStream_t st) {
    auto kern = k_qmv<WT, NT, EPI>;
    const size_t smem = qmv_smem_bytes(WT == W_Q80P ? M27B_TYPE_Q8_0 : M27B_TYPE_Q4_K, a.k, NT);
    static size_t configured[64] = {0};  // largest dynamic smem opted in so far, per device
    int dev = 0;
    cudaError_t ge = cudaGetDevice(&dev);
    if (ge != cudaSuccess) return ge;
    if (smem > 48 * 1024 && (dev >= 64 || smem > configured[dev])) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev] = smem;
    }
    // resident CTAs per SM for this smem size, cached per device (last size)
    static size_t occ_smem[64];
    static int occ_val[64] = {0};
    int occ = 0;
    if (dev < 64 && occ_val[dev] > 0 && occ_smem[dev] == smem) {
        occ = occ_val[dev];
    } else {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, QMV_THREADS, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) { occ_smem[dev] = smem; occ_val[dev] = occ; }
    }
    if (occ < 1) return cudaErrorInvalidConfiguration;
    const long warps_needed = (long)a.rows;
    long grid = (long)sm_count * occ;
    const long max_grid = (warps_needed + QMV_WARPS - 1) / QMV_WARPS;
    if (grid > max_grid) grid = max_grid;
    if (grid < 1) grid = 1;
    kern<<<(unsigned)grid, QMV_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

template <int WT, int EPI>
static cudaError_t launch_nt(const QmvArgs &a, int nt, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return launch_one<WT, 1, EPI>(a, sm_count, st);
    case 2: return launch_one<WT, 2, EPI>(a, sm_count, st);
    case 3: return launch_one<WT, 3, EPI>(a, sm_count, st);
    case 4: return launch_one<WT, 4, EPI>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

template <int EPI>
static cudaError_t launch_wt(int wt, const QmvArgs &a, int nt, int sm_count, cudaStream_t st) {
    switch (wt) {
    case W_Q4K: return launch_nt<W_Q4K, EPI>(a, nt, sm_count, st);
    case W_Q6KP: return launch_nt<W_Q6KP, EPI>(a, nt, sm_count, st);
    case W_Q80P: return launch_nt<W_Q80P, EPI>(a, nt, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_qmv(int wt, int epi, const QmvArgs &a, int nt, int sm_count, cudaStream_t st) {
    switch (epi) {
    case EPI_STORE: return launch_wt<EPI_STORE>(wt, a, nt, sm_count, st);
    case EPI_SWIGLU: return launch_wt<EPI_SWIGLU>(wt, a, nt, sm_count, st);
    case EPI_ARGMAX: return launch_wt<EPI_ARGMAX>(wt, a, nt, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
