/*
 * m27b_attn.h — decode attention over an fp32 KV cache (split over positions).
 *
 * Replaces the reference's decode attention pair k_attn_decode_split_partial
 * + k_attn_decode_split_reduce and its call site
 * (src/mono27b_executor.cu:1339-1484, :2441-2449).  The KV cache layout is the
 * reference's (k_mrope_and_cache, :1180-1229): element d of kv head j at
 * position p is cache[(p * n_kv + j) * head_dim + d], fp32.  The position is
 * read from device memory (the reference reads the __device__ global
 * g_kv_pos), so a captured graph serves every position.
 *
 * For query head h (kv head h / (n_q / n_kv)) and L = *pos + 1 cached
 * positions: out[h] = softmax(scale * q[h] . K[0..L)) V[0..L), the softmax
 * max-subtracted, accumulated in fp32.  Same conventions as m27b_qmv.h: bool +
 * error buffer; enqueues on `stream`, never synchronises.
 */
#ifndef M27B_ATTN_H
#define M27B_ATTN_H

#include <stdbool.h>
#include <stddef.h>

#include <cuda_runtime_api.h>

#include "m27b_qmv.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Bytes of split scratch m27b_attn_decode needs for n_q query heads of
 * head_dim values over `splits` position splits (0 for an invalid shape). */
M27B_API size_t m27b_attn_part_bytes(int n_q, int head_dim, int splits);

/* out[h * head_dim + d] for the n_q query heads q[h * head_dim + d] over the
 * cache positions [0, *pos].  head_dim: multiple of 32, 32..256; n_q a
 * multiple of n_kv with at most 8 query heads per kv head.  `splits` bounds
 * the position splits (short contexts use fewer: at least 16 positions per
 * split); a grid of n_kv * splits CTAs should not exceed one wave (148 on
 * B200).  `part` is caller scratch of m27b_attn_part_bytes(n_q, head_dim,
 * splits) bytes, 16-byte aligned; its contents need no initialisation.  The
 * first call on a device raises the kernels' shared-memory limit (a
 * per-device setting): make it before any stream capture. */
M27B_API bool m27b_attn_decode(const float *q, const float *k_cache, const float *v_cache, const int *pos, int n_q,
                               int n_kv, int head_dim, int splits, float scale, float *part, float *out,
                               cudaStream_t stream, char *err, size_t err_cap);

/* Capacity of the static scratch m27b_attn_decode_noalloc uses (1 MiB): enough
 * for 24 query heads of 256 values over 37 splits (37 * 24 * (256 + 4) * 4 =
 * 923,520 bytes by m27b_attn_part_bytes, the single-GPU Qwen-27B shape). */
#define M27B_ATTN_NOALLOC_SCRATCH_BYTES (1u << 20)

/* M27B_ATTN_NOALLOC_SCRATCH_BYTES as compiled into the library, for bindings
 * that do not read this header. */
M27B_API size_t m27b_attn_noalloc_scratch_bytes(void);

/* m27b_attn_decode without the `part` argument: the split partials live in a
 * file-scope __device__ array of M27B_ATTN_NOALLOC_SCRATCH_BYTES inside the
 * library, so neither the caller nor the library allocates device memory
 * (no cudaMalloc, cudaFree or allocating library routine).  This entry has no
 * counterpart in the reference; it is for callers that have no scratch
 * buffer to pass: a call site with a fixed signature (the reference's
 * attention call passes only q, the caches and out), or a host that plans all
 * device memory once at load time and cannot allocate on the decode path.
 * Results equal m27b_attn_decode's for the same arguments.
 *   - Shapes whose m27b_attn_part_bytes(n_q, head_dim, splits) exceeds
 *     M27B_ATTN_NOALLOC_SCRATCH_BYTES are rejected with an error (use fewer
 *     splits, or m27b_attn_decode with a larger buffer).
 *   - The first call on a device does the set-up (looks up the scratch's
 *     device address with cudaGetSymbolAddress and raises the kernels'
 *     shared-memory limit); make it before any stream capture.
 *   - Nothing in the scratch needs to start at zero: every active split writes
 *     its record before the reduction reads it.
 *   - There is one scratch per device: calls on the same device whose
 *     executions overlap (other streams, other host threads) race on it and
 *     give wrong results.  Order them on one stream. */
M27B_API bool m27b_attn_decode_noalloc(const float *q, const float *k_cache, const float *v_cache, const int *pos,
                                       int n_q, int n_kv, int head_dim, int splits, float scale, float *out,
                                       cudaStream_t stream, char *err, size_t err_cap);

#ifdef __cplusplus
}
#endif

#endif /* M27B_ATTN_H */
