/*
 * m27b_allreduce.h — the consumer half of the fused NVLink all-reduce of the
 * tensor-parallel decode step, as a standalone entry.
 *
 * The reference is single-GPU; its counterpart is the residual add plus the
 * RMSNorm and activation quantization that follow o_proj and ffn_down
 * (src/mono27b_executor.cu:2452-2479, l_rms + l_quant_q8_n :2139-2141,
 * :2022-2030).  In the tensor-parallel engine each rank's o_proj / ffn_down
 * kernel stores its partial output rows straight into every rank's receive
 * window; this entry is the kernel that then sums them and prepares the next
 * matvec's input.
 *
 * Word format: every value travels as one aligned 8-byte word, value bits in
 * the low 32 bits and an epoch in the high 32, written and read as one 64-bit
 * relaxed system-scope access.  A word whose epoch equals the one awaited
 * carries that epoch's value; no flag or fence accompanies it.
 *
 * Same conventions as m27b_qmv.h: bool + error buffer; device pointers;
 * enqueued on `stream`, never synchronised.
 */
#ifndef M27B_ALLREDUCE_H
#define M27B_ALLREDUCE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#include "m27b_qmv.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Most source ranks one consumer sums. */
#define M27B_ALLREDUCE_MAX_SRC 8

/* x_out[i] = sum over s = 0 .. nsrc-1 (in that order) of the value of word
 * words[s * src_stride + i], for i < k, once that word's epoch equals
 * *epoch; then xq = q8_K(RMSNorm(x_out) * norm_w) (norm_w may be NULL for
 * weight 1.0), as m27b_act_quant_rmsnorm of x_out would quantize it except
 * that the sum of squares is added per 256-value block and then over the
 * blocks in order (the same on every rank, so every rank quantizes the same
 * codes).  x_out is bit for bit the rank-ordered fp32 sum.  One token;
 * k a multiple of 256, at most 65536.  ss_words is k/256 words of scratch
 * the CTAs exchange their sums of squares through (with the same epoch): its
 * words must not already carry *epoch.  Every wait gives up after wait_ns
 * nanoseconds (0: 2 s) and then records status 3 in the library's device
 * status word (m27b_device_status); the kernel always returns and the output
 * of such a launch is invalid. */
M27B_API bool m27b_allreduce_norm_quant(const void *words, int nsrc, int src_stride, void *ss_words,
                                        const unsigned *epoch, const float *norm_w, float eps, int k, float *x_out,
                                        void *xq, unsigned long long wait_ns, cudaStream_t stream, char *err,
                                        size_t err_cap);

#ifdef __cplusplus
}
#endif

#endif /* M27B_ALLREDUCE_H */
