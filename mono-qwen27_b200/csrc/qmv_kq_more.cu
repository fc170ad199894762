// qmv_kq_more.cu — q5_K and IQ4_XS matvec instantiations on the q4_K
// streaming design (qmv_blk.cuh): batch 1..4, store / SwiGLU / argmax
// epilogues.  They replace the reference's k_q5k_mv_q8
// (src/mono27b_executor.cu:499-531) and k_iq4xs_mv_q8_dp4a (:674-686), which
// the dispatcher l_mv_q8_on calls for these types (:2066-2077).
#include "qmv_blk_launch.cuh"

namespace m27b {

template <class BT>
static cudaError_t run_kq(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (epi) {
    case EPI_STORE: return run_blk_nt<BT, EPI_STORE>(nt, a, sm_count, st);
    case EPI_SWIGLU: return run_blk_nt<BT, EPI_SWIGLU>(nt, a, sm_count, st);
    case EPI_ARGMAX: return run_blk_nt<BT, EPI_ARGMAX>(nt, a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

template <>
cudaError_t run_qmv_format<W_Q5K>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    return run_kq<BlkQ5K>(epi, nt, a, sm_count, st);
}

template <>
cudaError_t run_qmv_format<W_IQ4XS>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    return run_kq<BlkIQ4XS>(epi, nt, a, sm_count, st);
}

}  // namespace m27b
