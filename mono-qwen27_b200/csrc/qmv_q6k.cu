// qmv_q6k.cu — instantiations of the streaming matvec for W_Q6KP (one file per
// weight format so the instantiations compile in parallel).
#include "qmv_launch.cuh"

namespace m27b {
M27B_DEFINE_QMV_FORMAT(W_Q6KP)
}  // namespace m27b
