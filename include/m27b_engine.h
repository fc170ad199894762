/*
 * m27b_engine.h — decode engine around the quantized matvec C ABI.
 *
 * Mirrors the lifecycle of the reference executor's C API
 * (include/mono27b_config.h:155-184: load_weights / init_state / embed /
 * decode_step / argmax / free_*) for a Qwen-27B-shaped attention model:
 * every layer is RMSNorm -> fused q/gate/k/v projection (q4_K) -> q/k head
 * RMSNorm + rotary embedding -> decode attention over an fp32 KV cache ->
 * sigmoid(gate)-gated o_proj (q4_K) + residual -> RMSNorm -> gate/up SwiGLU
 * (q4_K) -> down (q6_K) + residual; then output RMSNorm -> lm_head (q6_K) with
 * fused argmax (greedy).  Tensor names are the reference loader's
 * (src/mono27b_executor.cu:1739-1831): token_embd.weight, output_norm.weight,
 * output.weight, blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output,
 * attn_q_norm, attn_k_norm, post_attention_norm, ffn_gate, ffn_up,
 * ffn_down}.weight.
 *
 * Hybrid models (attn_interval > 0, the reference's Qwen3.5/3.6 layout:
 * layer il is attention iff (il + 1) % attn_interval == 0) run the other
 * layers as the reference's Gated DeltaNet block (:2484-2548): RMSNorm ->
 * qkv (conv channels) and z projections -> beta / alpha projections ->
 * causal conv + SiLU with a per-layer conv state -> L2-normalised q / k ->
 * gated delta rule with a per-layer 128 x 128 state per value head ->
 * RMSNorm * ssm_norm * silu(z) -> ssm_out + residual -> the FFN.  Their
 * tensors: blk.N.{attn_qkv | attn_q | ssm_in}.weight (qkv),
 * blk.N.{attn_gate | attn_k | ssm_in_gate}.weight (z), ssm_beta.weight,
 * ssm_alpha.weight (f16 / f32 or quantized, same type), ssm_conv1d.weight
 * (f32 / f16, conv_kern values per channel), ssm_dt.bias | ssm_dt_bias,
 * ssm_a | ssm_a_log (f32, the negative decay rates), ssm_norm.weight (f32,
 * 128), ssm_out.weight, plus attn_norm, post_attention_norm and the FFN.
 * Hybrid models run on one GPU (tp_size 1) and without the verify pass
 * (rolling the recurrent state back after a rejected draft is not built).
 *
 * Tensor parallelism over tp_size GPUs (one process per GPU): q/gate by
 * heads, k/v by the kv heads the local q heads use (replicated when
 * tp_size > n_kv_head), gate/up by 256-value blocks of the FFN dimension,
 * o_proj and down split along their input dimension, lm_head by vocabulary
 * rows.  The 5120-wide hidden state is summed after o_proj and after down
 * (rank 0 adds the residual) with an NCCL all-reduce, or with the fused
 * NVLink path of m27b_engine_enable_p2p; the argmax keys likewise.  The
 * reference itself is single-GPU.
 *
 * Same conventions as m27b_qmv.h: bool + error buffer; no exceptions.
 */
#ifndef M27B_ENGINE_H
#define M27B_ENGINE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "m27b_qmv.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct M27BModelConfig {
    int n_layers;     /* 64 */
    int hidden;       /* 5120 */
    int ffn;          /* 17408 */
    int n_head;       /* 24 */
    int n_kv_head;    /* 4 */
    int head_dim;     /* 256 (<= 256, multiple of 32) */
    int vocab;        /* 248320 */
    int n_rot;        /* rotary dims per head, 64 */
    float rope_theta; /* 1e7 */
    float rms_eps;    /* 1e-6 */
    int max_ctx;      /* KV cache positions */
    int tp_rank;      /* this process's tensor-parallel rank */
    int tp_size;      /* 1, 2, 4 or 8 */
    uint32_t weight_type; /* m27b_engine_random_weights: 0 = the q4_k_m mix
                             (q4_K, q6_K for ffn_down and output), 8 = q8_0
                             everywhere (a draft model) */
    int attn_interval;    /* 0: every layer is attention; k > 0: layer il is
                             attention iff (il + 1) % k == 0, the others
                             Gated DeltaNet (4 in the reference model) */
    int ssm_d_inner;      /* value channels, ssm_dt_rank x 128 (6144) */
    int ssm_d_state;      /* key head width, 128 */
    int ssm_dt_rank;      /* value heads, even (48) */
    int ssm_n_group;      /* q / k groups; value head j uses group j % n (16) */
    int ssm_conv_kern;    /* causal conv width, 2..8 (4) */
} M27BModelConfig;

typedef struct M27BEngine M27BEngine;

/* The slice of the model one tensor-parallel rank holds (pure host logic). */
typedef struct M27BPartition {
    int q_lo, n_q;    /* local query heads [q_lo, q_lo + n_q) */
    int kv_lo, n_kv;  /* local kv heads (the ones those query heads use) */
    int f_lo, n_f;    /* local FFN values (whole 256-value blocks) */
    int v_lo, n_v;    /* local vocabulary rows */
} M27BPartition;

/* Compute rank cfg->tp_rank's partition; false (with a message) if the shape
 * cannot be split over cfg->tp_size ranks.  No CUDA call. */
M27B_API bool m27b_engine_partition(const M27BModelConfig *cfg, M27BPartition *out, char *err, size_t err_cap);

/* Size of an NCCL unique id (bytes). */
#define M27B_NCCL_ID_BYTES 128

/* Fill `id` (M27B_NCCL_ID_BYTES bytes) with a new NCCL unique id; rank 0
 * calls this and distributes the bytes to the other ranks. */
M27B_API bool m27b_nccl_unique_id(void *id, char *err, size_t err_cap);

/* Create an engine on the current CUDA device: validates the shapes, and
 * allocates this rank's weight shards, the KV cache and the workspace. */
M27B_API bool m27b_engine_create(const M27BModelConfig *cfg, M27BEngine **out, char *err, size_t err_cap);

/* Create a second engine (tp_size 1) on the current device that shares src's
 * weights and has its own KV cache of max_ctx positions, DeltaNet states,
 * workspace and CUDA graphs: several independent sequences over one copy of
 * the weights (the reference keeps weights and state apart the same way,
 * include/mono27b_config.h:155-166).  src must outlive it and must not load
 * further tensors meanwhile; this engine never frees the weights. */
M27B_API bool m27b_engine_create_sharing(const M27BEngine *src, int max_ctx, M27BEngine **out, char *err,
                                         size_t err_cap);

/* Join the tensor-parallel group (tp_size > 1): id from m27b_nccl_unique_id. */
M27B_API bool m27b_engine_set_nccl(M27BEngine *e, const void *id, char *err, size_t err_cap);

/* Switch the hidden-state all-reduces to the fused NVLink path (tp_size 2..8,
 * after m27b_engine_set_nccl, before the first decode step; all ranks call
 * it).  o_proj and ffn_down then store their output rows straight into every
 * rank's receive window (CUDA IPC mappings, exchanged once over NCCL) and
 * publish an epoch with a system-scope release store; the next kernel waits
 * (bounded) for every rank's epoch, sums the partials in rank order and
 * applies the following RMSNorm + q8_K quantization.  The argmax keys are
 * exchanged the same way.  No NCCL call remains in the decode step. */
M27B_API bool m27b_engine_enable_p2p(M27BEngine *e, char *err, size_t err_cap);

/* Load one FULL tensor (host bytes in GGUF layout, or fp32 for norms) by its
 * GGUF name; the engine keeps this rank's shard (and repacks it). */
M27B_API bool m27b_engine_load_tensor(M27BEngine *e, const char *name, uint32_t ggml_type, uint32_t row_elems,
                                      uint32_t row_count, const void *host, char *err, size_t err_cap);

/* Load every entry of an opened `.m27b` blob (m27b_blob.h) whose
 * source_model equals `source` (M27B_SOURCE_TARGET for this engine) through
 * m27b_engine_load_tensor, by its GGUF name.  An entry the engine does not
 * know, or whose payload is shorter than its shape, is an error. */
struct M27BBlob;
M27B_API bool m27b_engine_load_blob(M27BEngine *e, const struct M27BBlob *blob, uint32_t source, char *err,
                                    size_t err_cap);

/* Fill every weight with seeded synthetic GGUF blocks generated on the GPU
 * in global coordinates (identical tensors for every tp_size); norms = 1.
 * The q4_K / q6_K values have standard deviation ~ sigma. */
M27B_API bool m27b_engine_random_weights(M27BEngine *e, uint64_t seed, float sigma, char *err, size_t err_cap);

/* Bytes of weights this rank streams per token (its shards, as stored). */
M27B_API size_t m27b_engine_weight_bytes_per_token(const M27BEngine *e);

/* Forget the KV cache (next position 0). */
M27B_API bool m27b_engine_reset(M27BEngine *e, char *err, size_t err_cap);

/* One decode step for `token` at position `pos` (pos == number of tokens
 * already in the cache).  Writes the greedy next token to *next (all ranks
 * agree).  If logits != NULL (tp_size == 1 only) the vocabulary logits are
 * copied to the host buffer.  The first step captures the step into a CUDA
 * graph that later steps replay; synchronises before returning. */
M27B_API bool m27b_engine_decode_step(M27BEngine *e, int token, int pos, int *next, float *logits, char *err,
                                      size_t err_cap);

/* Most tokens m27b_engine_verify takes in one pass. */
#define M27B_VERIFY_MAX 16

/* Speculative verification: run the n (1..M27B_VERIFY_MAX) tokens tokens[0..n)
 * at positions pos .. pos+n-1 in one pass — their K/V appended, token i
 * attending to the cache up to position pos+i — and write the greedy next
 * token after each to next[i] (the target's choice at every drafted
 * position; tokens a caller rejects leave K/V behind that later steps simply
 * overwrite).  q4_K matrices run 5+ tokens on the tensor cores.  logits
 * (tp_size 1 only, may be NULL) receive n rows of vocab floats.  The pass is
 * captured into a CUDA graph per n on first use.  At tp_size > 1 its
 * all-reduces (n rows each) run on the engine's NCCL communicator, also when
 * the decode step uses the fused NVLink all-reduce.  Synchronises before
 * returning. */
M27B_API bool m27b_engine_verify(M27BEngine *e, const int *tokens, int n, int pos, int *next, float *logits, char *err,
                                 size_t err_cap);

/* Counters and host times of m27b_engine_speculative_generate. */
typedef struct M27BSpecStats {
    int iterations;    /* draft + verify rounds */
    int proposed;      /* drafted tokens (iterations x k) */
    int accepted;      /* drafted tokens the target's greedy choice agreed with */
    double prefill_ms; /* feeding the prompt to both engines */
    double draft_ms;   /* the draft's generation calls */
    double verify_ms;  /* the target's verify passes */
} M27BSpecStats;

/* Greedy speculative decoding (the loop the reference lists as next,
 * README.md:41-45): feeds prompt[0 .. n_prompt-2] to both engines at
 * positions 0 .., then repeats: the draft proposes k tokens (1 <= k <
 * M27B_VERIFY_MAX) by greedy generation on the device, the target verifies
 * the last token and the k proposals in one pass, and the longest agreeing
 * prefix plus the target's own next token are kept.  out_tokens receives
 * exactly n_new tokens, the target's plain greedy continuation of the prompt
 * (lossless).  Both engines must have tp_size 1 or use NCCL (the verify
 * pass's all-reduce) and hold nothing else: positions from 0 are rewritten;
 * both need n_prompt + n_new + k positions of cache.  Hybrid (DeltaNet)
 * targets are refused by the verify pass.  stats may be NULL. */
M27B_API bool m27b_engine_speculative_generate(M27BEngine *target, M27BEngine *draft, const int *prompt, int n_prompt,
                                               int n_new, int k, int *out_tokens, M27BSpecStats *stats, char *err,
                                               size_t err_cap);

/* Greedy generation of n tokens on the device: step i (position pos + i)
 * consumes the token step i-1 produced (`token` for i = 0), with no host
 * round trip between steps (the captured step ends by writing its argmax as
 * the next token and advancing the position).  tokens[i] receives the token
 * step i produced.  Needs pos + n <= max_ctx; synchronises before returning. */
M27B_API bool m27b_engine_generate(M27BEngine *e, int token, int pos, int n, int *tokens, char *err, size_t err_cap);

/* Copy the current hidden state (after the last decode step, before the
 * output norm) to the host (hidden floats). */
M27B_API bool m27b_engine_hidden(M27BEngine *e, float *host, char *err, size_t err_cap);

/* The CUDA stream every engine call enqueues on (a cudaStream_t), so that a
 * caller can order its own work after the engine's or time the engine's work
 * with events recorded on it. */
M27B_API void *m27b_engine_stream(M27BEngine *e);

M27B_API void m27b_engine_destroy(M27BEngine *e);

#ifdef __cplusplus
}
#endif

#endif /* M27B_ENGINE_H */
