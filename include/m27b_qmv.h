/*
 * m27b_qmv.h — C ABI of the B200 (sm_100a) quantized weight-streaming kernels.
 *
 * This is the seam the reference executor's matvec dispatch calls through.
 * It replaces, one for one:
 *
 *   m27b_act_quant      <- l_quant_q8_n + k_quant_q8_1          src/mono27b_executor.cu:2022-2030, :84-107
 *                          (activations are quantized to ggml's q8_K / q8_0, not q8_1,
 *                          so that results follow ggml's CPU vec_dot semantics)
 *   m27b_act_quant_gated<- k_quant_q8_1_fused_gate              src/mono27b_executor.cu:109-138, :2460
 *   m27b_act_quant_swiglu<- k_elem_swiglu + l_quant_q8_n         src/mono27b_executor.cu:833-838, :2022-2030
 *                          (gate and up computed as separate matvecs, e.g. a verify batch)
 *   m27b_qmv            <- l_mv_q8_on / l_mv_quant_residual     src/mono27b_executor.cu:2054-2102
 *                          (k_q4k_mv_q8_dp4a :320-364, k_q6k_mv_q8_dp4a :630-645,
 *                          k_q80_mv_q8_dp4a :533-580, k_q5k_mv_q8 :499-531,
 *                          k_iq4xs_mv_q8_dp4a :674-686)
 *   m27b_qmv_f32        <- l_mv_quant / l_mv_fallback           src/mono27b_executor.cu:2033-2050, :2127-2137
 *                          (f16 / f32 weights: k_f16_mv :900-916, k_f32_mv :1101-1114)
 *   m27b_qmv_swiglu     <- l_ffn_gate_up_swiglu                 src/mono27b_executor.cu:2239-2261
 *                          (k_q4k_q4k_swiglu_dp4a :369-417)
 *   m27b_qmv_argmax     <- lm_head block + k_argmax             src/mono27b_executor.cu:2577-2593, :209-239
 *   m27b_dequant_rows   <- k_q4k_embed / mono27b_engine_embed   src/mono27b_executor.cu:1233-1254, :2641-2664
 *   m27b_repack         <- (new) optional load-time repack of q6_K / q8_0 rows
 *                          into 16-byte aligned planes; lossless.
 *
 * Conventions (kept from the reference, include/mono27b_config.h:155-184):
 *   - every entry returns bool; on failure it writes a message into
 *     err[0..err_cap) and returns false; on success err[0] is set to '\0'.
 *   - every pointer argument that names tensor data is a DEVICE pointer on the
 *     current CUDA device; the work is enqueued on `stream` (0 = the default
 *     stream) and nothing is synchronised, so every entry is usable inside CUDA
 *     graph capture.  No entry allocates device memory.
 *
 * Weight rows: a WeightView {ptr, ggml_type, row_blocks, row_count} as the
 * reference loader fills it (include/mono27b_config.h:63-68, filled at
 * src/mono27b_executor.cu:1695-1716): row_count rows of row_blocks blocks.
 * q4_K, q5_K and IQ4_XS rows are read in their GGUF layout (IQ4_XS rows need
 * an even block count, so that rows stay 16-byte aligned).  q6_K and q8_0
 * rows must first be repacked with m27b_repack; the repacked view carries
 * ggml_type | M27B_LAYOUT_PLANAR.  f16 / f32 rows (row_blocks = values per
 * row, as the reference loader sets it; a multiple of 8 / 4) take fp32
 * activations through m27b_qmv_f32 only.  ptr must be 16-byte aligned
 * (cudaMalloc gives 256).
 *
 * Activations: m27b_act_quant writes n_tok rows of m27b_act_bytes(type, k)
 * bytes, ggml block_q8_K (for q4_K / q6_K weights) or block_q8_0 (for q8_0
 * weights), bit for bit what ggml's quantize_row_q8_K_ref / q8_0_ref produce.
 */
#ifndef M27B_QMV_H
#define M27B_QMV_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#include "m27b_blocks.h"

#if defined(__GNUC__)
#define M27B_API __attribute__((visibility("default")))
#else
#define M27B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#ifndef M27B_EXTERNAL_WEIGHTVIEW
/* Identical layout to the reference's WeightView (include/mono27b_config.h:63-68).
 * Define M27B_EXTERNAL_WEIGHTVIEW after including the reference's header to
 * use its declaration instead. */
struct WeightView {
    void *ptr;
    uint32_t ggml_type;
    uint32_t row_blocks;
    uint32_t row_count;
};
#endif

/* Largest batch (tokens per call) the matvec entries accept. */
#define M27B_MAX_TOKENS 16

/* Library version string. */
M27B_API const char *m27b_version(void);

/* Read the current device's status word (synchronous): 0 when every bounded
 * wait inside the kernels completed; non-zero when a kernel gave up waiting
 * for its own shared-memory copies (the results of that launch are invalid).
 * clear != 0 resets it.  No counterpart in the reference, whose kernels have
 * no waits. */
M27B_API bool m27b_device_status(int *status, int clear, char *err, size_t err_cap);

/* Bytes of one quantized activation row of k values: k/256*292 for
 * M27B_TYPE_Q8_K, k/32*34 for M27B_TYPE_Q8_0; 0 if k is not a multiple of
 * the block size or the type is not an activation type. */
M27B_API size_t m27b_act_bytes(uint32_t act_type, int k);

/* Activation type a weight type is multiplied against (q8_0 for q8_0 weights,
 * q8_K for q4_K / q5_K / q6_K / IQ4_XS); 0 for f16 / f32 weights (fp32
 * activations, m27b_qmv_f32) and unsupported types. */
M27B_API uint32_t m27b_act_type_for(uint32_t ggml_type);

/* Quantize n_tok rows of k fp32 values (row stride ldx floats) into
 * n_tok * m27b_act_bytes(act_type, k) contiguous bytes at xq. */
M27B_API bool m27b_act_quant(const float *x, int k, int n_tok, int ldx, uint32_t act_type, void *xq,
                    cudaStream_t stream, char *err, size_t err_cap);

/* As m27b_act_quant, of x[i] * sigmoid(gate[i]) — the gated attention output
 * that feeds o_proj. */
M27B_API bool m27b_act_quant_gated(const float *x, const float *gate, int k, int n_tok, int ldx,
                          uint32_t act_type, void *xq, cudaStream_t stream, char *err, size_t err_cap);

/* Quantize silu(gate[i]) * up[i] (the FFN activation that feeds ffn_down),
 * n_tok rows of k values with row stride ldx in both inputs; the same fp32
 * expression as the SwiGLU epilogue of m27b_qmv_swiglu. */
M27B_API bool m27b_act_quant_swiglu(const float *gate, const float *up, int k, int n_tok, int ldx, uint32_t act_type,
                                   void *xq, cudaStream_t stream, char *err, size_t err_cap);

/* As m27b_act_quant, of RMSNorm(x) * w (w may be NULL for weight 1.0) with
 * the given eps; the norm is taken over each row of k values. */
M27B_API bool m27b_act_quant_rmsnorm(const float *x, const float *w, float eps, int k, int n_tok, int ldx,
                            uint32_t act_type, void *xq, cudaStream_t stream, char *err, size_t err_cap);

/* Bytes m27b_repack writes for a tensor (0 if the type is not repackable). */
M27B_API size_t m27b_repacked_bytes(uint32_t ggml_type, uint32_t row_blocks, uint32_t row_count);

/* Repack row_count GGUF rows of q6_K or q8_0 (row_blocks blocks each) from
 * `raw` into the aligned layout at `out` (m27b_repacked_bytes bytes, 16-byte
 * aligned); lossless.  The view for the result is {out, ggml_type |
 * M27B_LAYOUT_PLANAR, row_blocks, row_count}.  A q6_K row becomes
 * ceil(row_blocks/4) tiles of 848 bytes, each holding 4 blocks as
 * ql[4][128] | qh[4][64] | scales[4][16] | d[4] (fp16 + 2 zero bytes), blocks
 * past the row end zero; a q8_0 row becomes [qs | d, padded to 16 B]. */
M27B_API bool m27b_repack(const void *raw, uint32_t ggml_type, uint32_t row_blocks, uint32_t row_count,
                 void *out, cudaStream_t stream, char *err, size_t err_cap);

/* y[t*ldy + r] = W[r] . x[t] (+ residual[t*ldy + r] when residual != NULL)
 * for t < n_tok (1..M27B_MAX_TOKENS), r < row_count.  xq holds n_tok
 * activation rows from m27b_act_quant of type m27b_act_type_for(W type) and
 * k = row_blocks * block size.  residual may alias y. */
M27B_API bool m27b_qmv(const struct WeightView *w, const void *xq, int n_tok, float *y, int ldy,
              const float *residual, cudaStream_t stream, char *err, size_t err_cap);

/* y[t*ldy + r] = silu(G[r] . x[t]) * (U[r] . x[t]); gate and up must have the
 * same type and shape. */
M27B_API bool m27b_qmv_swiglu(const struct WeightView *gate, const struct WeightView *up, const void *xq,
                     int n_tok, float *y, int ldy, cudaStream_t stream, char *err, size_t err_cap);

/* Matvec with a fused argmax over rows: best[t] receives a packed key whose
 * index m27b_argmax_key_index() decodes (largest value, ties to the smallest
 * row index); logits (may be NULL) receive the values with stride ldl.
 * row_offset is added to every index, so that ranks holding a slice of the
 * vocabulary produce keys comparable across ranks. */
M27B_API bool m27b_qmv_argmax(const struct WeightView *w, const void *xq, int n_tok, float *logits, int ldl,
                     unsigned long long *best, uint32_t row_offset, cudaStream_t stream, char *err,
                     size_t err_cap);

/* q6_K matvec for 5..16 tokens with the K dimension split across CTAs: the
 * speculative verify pass's ffn_down (5120 x 17408), where the one-pass
 * kernel's staged activations (8 tokens x 17408 values) crowd out its weight
 * stages.  Same result semantics as m27b_qmv (per-range partial sums added
 * in range order; within fp32 rounding of the one-pass kernel).  Needs the
 * repacked q6_K layout and rows of at least 32 blocks; the caller passes
 * m27b_qmv_q6k_ksplit_part_bytes scratch for partial sums and
 * m27b_qmv_q6k_ksplit_count_bytes of counters that must be zero before the
 * first call (each call leaves them zero).  Calls overlapping on the GPU
 * with the same scratch race.  The reference runs this product token by
 * token (k_q6k_mv_q8_dp4a, src/mono27b_executor.cu:630-645). */
M27B_API size_t m27b_qmv_q6k_ksplit_part_bytes(const struct WeightView *w);
M27B_API size_t m27b_qmv_q6k_ksplit_count_bytes(const struct WeightView *w);
M27B_API bool m27b_qmv_q6k_ksplit(const struct WeightView *w, const void *xq, int n_tok, float *y, int ldy,
                                  const float *residual, void *part, void *count, cudaStream_t stream, char *err,
                                  size_t err_cap);

/* q4_K matvec for 5..16 tokens on the tensor cores (as m27b_qmv does for
 * them) with each 128-row tile's K dimension cut into ranges handled by
 * different CTAs, two CTAs per SM at up to 8 tokens: more, shorter
 * block-column chains in flight than the one-unit-per-tile launch (17408
 * rows are only 136 tiles for 148 SMs).  The ranges' partial sums are added
 * in range order by the last-arriving range of each 32-row slice
 * (deterministic; within fp32 rounding of m27b_qmv).  The caller passes
 * m27b_qmv_mma_split_part_bytes of scratch and m27b_qmv_mma_split_count_bytes
 * of counters that must be zero before the first call (each call leaves them
 * zero); calls overlapping on the GPU with the same scratch race.  Replaces,
 * for a verify pass, the reference's per-token k_q4k_mv_q8_dp4a
 * (src/mono27b_executor.cu:320-364). */
M27B_API size_t m27b_qmv_mma_split_part_bytes(const struct WeightView *w, int n_tok);
M27B_API size_t m27b_qmv_mma_split_count_bytes(const struct WeightView *w);
M27B_API bool m27b_qmv_mma_split(const struct WeightView *w, const void *xq, int n_tok, float *y, int ldy,
                                 const float *residual, void *part, void *count, cudaStream_t stream, char *err,
                                 size_t err_cap);

/* q6_K matvec for 1..8 tokens on the tensor cores (tcgen05 kind::i8, one
 * MMA per 16-value group: each 32-value slice is multiplied with either
 * group's codes zeroed), y = W.xq (+ residual): the speculative verify
 * pass's ffn_down.  Integer sums per super-block exactly as ggml's
 * vec_dot_q6_K_q8_K, fp32 combine per block (within fp32 rounding of
 * m27b_qmv).  Needs the repacked q6_K layout.  With part / count (both
 * non-NULL: m27b_qmv_q6k_mma_part_bytes of scratch, m27b_qmv_q6k_mma_count_bytes
 * of counters zero before the first call, left zero by every call) a matrix
 * of few row tiles has its K dimension split across CTAs, the ranges' partial
 * sums added in range order (deterministic); calls overlapping on the GPU
 * with the same scratch race.  Replaces, for a verify pass, the reference's
 * per-token k_q6k_mv_q8_dp4a (src/mono27b_executor.cu:630-645). */
M27B_API size_t m27b_qmv_q6k_mma_part_bytes(const struct WeightView *w);
M27B_API size_t m27b_qmv_q6k_mma_count_bytes(const struct WeightView *w);
M27B_API bool m27b_qmv_q6k_mma(const struct WeightView *w, const void *xq, int n_tok, float *y, int ldy,
                               const float *residual, void *part, void *count, cudaStream_t stream, char *err,
                               size_t err_cap);

/* The same kernel with m27b_qmv_argmax's epilogue (best[t] receives token
 * t's packed key; logits, may be NULL, with stride ldl): the
 * verify pass's lm_head for up to 8 tokens in one weight pass.  Replaces the
 * reference's lm_head block + k_argmax (src/mono27b_executor.cu:2577-2593,
 * :209-239) for the drafted tokens. */
M27B_API bool m27b_qmv_q6k_mma_argmax(const struct WeightView *w, const void *xq, int n_tok, float *logits, int ldl,
                                      unsigned long long *best, uint32_t row_offset, cudaStream_t stream, char *err,
                                      size_t err_cap);

/* q6_K matvec for ONE token over a matrix of few, long rows (a decode step's
 * ffn_down, 5120 x 17408), y = W.xq (+ residual): the (8-row group, 4-block
 * tile) items are cut into equal runs, one per warp of a one-CTA-per-SM grid,
 * so that no SM carries more row groups than another; a group shared by
 * several runs is summed by the run that finishes it last, in run order
 * (deterministic; within fp32 rounding of m27b_qmv).  Needs the repacked
 * q6_K layout and rows of at most 609 blocks (the staged activation row must
 * leave room for 4 warps' stages); the caller passes
 * m27b_qmv_q6k_stream_part_bytes of scratch for partial sums and
 * m27b_qmv_q6k_stream_count_bytes of counters that must be zero before the
 * first call (each call leaves them zero).  Calls overlapping on the GPU
 * with the same scratch race.  Replaces, for one token, the reference's
 * k_q6k_mv_q8_dp4a (src/mono27b_executor.cu:630-645). */
M27B_API size_t m27b_qmv_q6k_stream_part_bytes(const struct WeightView *w);
M27B_API size_t m27b_qmv_q6k_stream_count_bytes(const struct WeightView *w);
M27B_API bool m27b_qmv_q6k_stream(const struct WeightView *w, const void *xq, float *y, const float *residual,
                                  void *part, void *count, cudaStream_t stream, char *err, size_t err_cap);

/* fp32 activations in, like the reference's l_mv_quant(W, x, y)
 * (src/mono27b_executor.cu:2033-2050, its quantizer k_quant_q8_1 :84-107):
 * x rows (n_tok of them, stride ldx floats) are quantized to q8_K / q8_0 and
 * multiplied, y = W.x (+ residual).  For a q4_K, q5_K, IQ4_XS or (repacked)
 * q6_K matrix and up to 4 tokens (x 16-byte aligned, ldx a multiple of 4)
 * the matvec kernel quantizes the rows in its own prologue (one launch, same
 * codes as m27b_act_quant; with m27b_qmv_f32_rmsnorm not for q6_K);
 * otherwise the rows are first quantized into xq_scratch
 * (n_tok * m27b_act_bytes(m27b_act_type_for(type), k) bytes; may be NULL on
 * the one-launch path).  f16 / f32 matrices multiply the fp32 rows directly
 * (x 16-byte aligned, ldx a multiple of 4; the f16 path rounds x to fp16
 * first, as ggml does; xq_scratch unused). */
M27B_API bool m27b_qmv_f32(const struct WeightView *w, const float *x, int ldx, int n_tok, void *xq_scratch, float *y,
                           int ldy, const float *residual, cudaStream_t stream, char *err, size_t err_cap);

/* The same with RMSNorm(x) * norm_w (eps; norm_w may be NULL: 1.0) before
 * the quantization, the reference's l_rms + MV pair (:2139-2141).  With
 * w_up non-NULL the epilogue is SwiGLU, y = silu(W.x) * (W_up.x) (no
 * residual) — the FFN's gate/up after the post-attention norm.  Quantized
 * weight types only. */
M27B_API bool m27b_qmv_f32_rmsnorm(const struct WeightView *w, const struct WeightView *w_up, const float *x, int ldx,
                                   const float *norm_w, float eps, int n_tok, void *xq_scratch, float *y, int ldy,
                                   const float *residual, cudaStream_t stream, char *err, size_t err_cap);

/* out[i*ldo + j] = dequant(W[rows[i]])[j] for i < n, j < k; rows is a device
 * array of n row indices; an index outside [0, row_count) yields a zero row
 * (the reference embed zeroes the hidden state for such tokens). */
M27B_API bool m27b_dequant_rows(const struct WeightView *w, const int32_t *rows, int n, float *out, int ldo,
                       cudaStream_t stream, char *err, size_t err_cap);

/* Measurement support (no counterpart in the reference): stream `bytes`
 * (16-byte aligned, a multiple of 16) from device memory p into shared memory
 * with bulk asynchronous copies, nothing computed.  The time of one launch is
 * the read ceiling a weight-streaming launch of that size can reach.  Shape:
 * `ctas_per_sm` CTAs on every SM, `warps` issuing warps per CTA (1-16), each
 * streaming its contiguous share of the buffer in `chunk`-byte copies
 * (16-65536, a multiple of 16) with `stages` copies in flight (1-8).  Launched
 * with programmatic dependent launch, like the matvec kernels: back-to-back
 * probes overlap one launch's start with the previous one's drain.  A shape
 * whose CTAs do not fit `ctas_per_sm` to an SM is refused.  A wait that runs
 * out records status 6 (m27b_device_status). */
M27B_API bool m27b_hbm_read_probe_shape(const void *p, size_t bytes, int warps, int stages, int chunk, int ctas_per_sm,
                                        cudaStream_t stream, char *err, size_t err_cap);
/* m27b_hbm_read_probe_shape with one warp per CTA, six 32 KB copies in flight,
 * one CTA per SM. */
M27B_API bool m27b_hbm_read_probe(const void *p, size_t bytes, cudaStream_t stream, char *err, size_t err_cap);

/* Packed argmax key helpers (host side). */
static inline int64_t m27b_argmax_key_index(unsigned long long key) {
    return (int64_t)(0xffffffffull - (key & 0xffffffffull));
}

#ifdef __cplusplus
}
#endif

#endif /* M27B_QMV_H */
