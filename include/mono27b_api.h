/*
 * mono27b_api.h — the reference executor's C API, served by libm27b.
 *
 * The reference executor exports these entry points
 * (include/mono27b_config.h:155-184, implemented in
 * src/mono27b_executor.cu:1727-2664) and its chat driver calls them
 * (src/mono27b_chat.cpp:352-391, :407, :467-471).  libm27b exports the same
 * symbols with the same signatures, so a program built against the
 * reference's own headers links against libm27b instead of the reference's
 * executor object with no source change.  This header restates the
 * reference's types in this project's code, field for field, for callers
 * that do not have the reference's headers (the types have to be alike: the
 * binary interface is the structs' layout).  Do not include it together with
 * the reference's mono27b_config.h; include one or the other.
 *
 * What the entries do here (each backed by the decode engine of
 * m27b_engine.h, tensor-parallel size 1):
 *   load_weights   infers the model shape from the tensor descriptors
 *                  (hidden, vocab, layers, heads, FFN, DeltaNet sizes; which
 *                  layers are attention), creates an engine and loads every
 *                  tensor it knows by its GGUF name (src/mono27b_executor.cu
 *                  :1739-1831; unknown names are skipped, as there).  The
 *                  WeightViews of *gpu_weights then describe the engine's own
 *                  device tensors (q6_K / q8_0 repacked: ggml_type carries
 *                  M27B_LAYOUT_PLANAR; q, k and v are row ranges of one fused
 *                  matrix; the attention output gate rows are interleaved in
 *                  wq, so `gate` stays empty).  Rotary dims (64, or head_dim
 *                  if smaller), theta 1e7 and eps 1e-6 are the reference's
 *                  constants.
 *   init_state     records max_ctx; the engine that holds this state's KV
 *                  cache, DeltaNet states and CUDA graphs is created at the
 *                  first decode step, sharing the weights'
 *                  (m27b_engine_create_sharing).
 *   decode_step    one step (captured into a CUDA graph, then replayed);
 *                  output->logits points at the vocabulary logits in device
 *                  memory (owned by the state, like the reference's work
 *                  buffer); state->kv_len = position + 1.  kv_cache_k/v,
 *                  ssm_state and conv_state point at the engine's buffers.
 *   embed          the fp32 embedding row of a token into device memory
 *                  (zeros for an out-of-range token), on the legacy default
 *                  stream, not synchronised.
 *   argmax         index of the largest of n device floats, ties to the
 *                  smallest index (synchronises).
 *   free_logits    clears output->logits (nothing to free).
 *   print_timing / reset_timing   the mean host time per decode step since
 *                  the last reset (the reference prints per-kernel timings
 *                  when built with MONO27B_TIMING).
 * The weights may be freed before a state that uses them; they are released
 * when the last such state is.  The library is built without
 * MONO27B_TIMING: a caller built with it keeps its extra state fields, which
 * the library never touches.  Errors: false + a message in error[0..cap),
 * as the reference does.
 */
#ifndef M27B_MONO27B_API_H
#define M27B_MONO27B_API_H

#ifndef __cplusplus
#error "mono27b_api.h declares the reference's C++ types (std::string in Mono27BGgufTensorInfo)"
#endif

#include <cstddef>
#include <cstdint>
#include <string>

#include "m27b_qmv.h" /* struct WeightView, the reference's layout */

/* Model constants the reference's structs are sized by
 * (include/mono27b_format.h:9, include/mono27b_config.h:42-54). */
constexpr uint32_t MONO27B_TARGET_LAYERS = 64U;
constexpr int MONO27B_TARGET_FA_INTERVAL = 4;
constexpr int MONO27B_TARGET_FA_LAYERS = MONO27B_TARGET_LAYERS / MONO27B_TARGET_FA_INTERVAL;

/* One tensor of a GGUF file (include/mono27b_gguf.h:45-52): dims[0] is the
 * innermost extent (values per row). */
struct Mono27BGgufTensorInfo {
    std::string name;
    uint32_t ggml_type = 0;
    uint64_t offset = 0;
    uint64_t size_bytes = 0;
    uint32_t n_dims = 0;
    uint64_t dims[4] = {};
};

/* include/mono27b_config.h:70-84 */
struct Mono27BAttentionLayerWeights {
    WeightView attn_norm, wq, wk, wv, wo, gate, q_norm, k_norm, post_norm, ffn_gate, ffn_up, ffn_down;
};

/* include/mono27b_config.h:86-101 */
struct Mono27BSSMLayerWeights {
    WeightView attn_norm, wqkv, wqkv_gate, ssm_conv1d, ssm_beta, ssm_alpha, ssm_dt_bias, ssm_a_log, ssm_norm, ssm_out,
        post_norm, ffn_gate, ffn_up, ffn_down;
};

/* include/mono27b_config.h:103-114 */
struct Mono27BExecutorWeights {
    struct {
        bool is_attention;
        union {
            Mono27BAttentionLayerWeights attn;
            Mono27BSSMLayerWeights ssm;
        };
    } layers[MONO27B_TARGET_LAYERS];
    WeightView output_norm;
    WeightView lm_head;
    WeightView tok_embd;
};

/* include/mono27b_config.h:116-150 (without the MONO27B_TIMING fields) */
struct Mono27BExecutorState {
    float *kv_cache_k[MONO27B_TARGET_FA_LAYERS];
    float *kv_cache_v[MONO27B_TARGET_FA_LAYERS];
    float *ssm_state[MONO27B_TARGET_LAYERS - MONO27B_TARGET_FA_LAYERS];
    float *conv_state[MONO27B_TARGET_LAYERS - MONO27B_TARGET_FA_LAYERS];
    float *attn_split_o;
    float *attn_split_m;
    float *attn_split_l;
    float *work_buf;
    size_t work_buf_size;
    void *q8_scratch;
    int *argmax_result;
    void *cuda_graph;
    void *cuda_graph_exec;
    int graph_captured;
    int max_ctx;
    int kv_len;
    void *stream1;
    void *sync_event;
};

/* include/mono27b_config.h:152-154 */
struct Mono27BLogitsOutput {
    float *logits;
};

extern "C" {

M27B_API bool mono27b_engine_load_weights(const unsigned char *gguf_data, uint64_t data_offset,
                                          const struct Mono27BGgufTensorInfo *tensors, size_t tensor_count,
                                          Mono27BExecutorWeights *gpu_weights, char *error, size_t error_cap);
M27B_API void mono27b_engine_free_weights(Mono27BExecutorWeights *w);
M27B_API bool mono27b_engine_init_state(int max_ctx, Mono27BExecutorState *state, char *error, size_t error_cap);
M27B_API void mono27b_engine_free_state(Mono27BExecutorState *state);
M27B_API bool mono27b_engine_embed(const Mono27BExecutorWeights *we, int token_id, float *hidden, char *error,
                                   size_t error_cap);
M27B_API bool mono27b_engine_decode_step(const Mono27BExecutorWeights *weights, Mono27BExecutorState *state,
                                         int token_id, int position, Mono27BLogitsOutput *output, char *error,
                                         size_t error_cap);
M27B_API void mono27b_engine_free_logits(Mono27BLogitsOutput *output);
M27B_API int mono27b_engine_argmax(Mono27BExecutorState *st, const float *logits, int n);
M27B_API void mono27b_engine_print_timing(Mono27BExecutorState *st);
M27B_API void mono27b_engine_reset_timing(Mono27BExecutorState *st);

} /* extern "C" */

#endif /* M27B_MONO27B_API_H */
