// qmv_q4k.cu — q4_K matvec instantiations: one super-block per lane
// (qmv_blk.cuh), batch 1..4, store / SwiGLU / argmax / all-reduce push
// epilogues.
#include "qmv_blk_launch.cuh"

namespace m27b {

template <>
cudaError_t run_qmv_format<W_Q4K>(int epi, int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (epi) {
    case EPI_STORE: return run_blk_nt<BlkQ4K, EPI_STORE>(nt, a, sm_count, st);
    case EPI_SWIGLU: return run_blk_nt<BlkQ4K, EPI_SWIGLU>(nt, a, sm_count, st);
    case EPI_ARGMAX: return run_blk_nt<BlkQ4K, EPI_ARGMAX>(nt, a, sm_count, st);
    case EPI_PUSH: return nt == 1 ? run_blk<BlkQ4K, 1, EPI_PUSH>(a, sm_count, st) : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
