// api_probe.cpp — test program for the reference-executor API that libm27b
// exports (test infrastructure).
//
// Built twice by tests/test_ref_api.py: with -DM27B_PROBE_REFERENCE_HEADERS
// against the reference's own include/mono27b_config.h and
// include/mono27b_gguf.h (read in place), and without it against this
// project's include/mono27b_api.h.  Both builds print the size of every
// struct of the interface and the offset of every field; the two listings
// must be identical.  The reference-header build is also linked against
// libm27b and, with the matvec header included under
// M27B_EXTERNAL_WEIGHTVIEW (the reference's WeightView in both APIs), calls
// entry points whose argument checks answer before any CUDA call, printing
// what they return.
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <vector>

#ifdef M27B_PROBE_REFERENCE_HEADERS
#include "mono27b_config.h"
#include "mono27b_gguf.h"
#define M27B_EXTERNAL_WEIGHTVIEW
#include "m27b_qmv.h"
#else
#include "mono27b_api.h"
#endif

#define SZ(T) std::printf("sizeof %s %zu\n", #T, sizeof(T))
#define OFF(T, f) std::printf("offsetof %s.%s %zu\n", #T, #f, offsetof(T, f))

int main(int argc, char **argv) {
    SZ(WeightView);
    OFF(WeightView, ptr); OFF(WeightView, ggml_type); OFF(WeightView, row_blocks); OFF(WeightView, row_count);
    SZ(Mono27BGgufTensorInfo);
    OFF(Mono27BGgufTensorInfo, name); OFF(Mono27BGgufTensorInfo, ggml_type); OFF(Mono27BGgufTensorInfo, offset);
    OFF(Mono27BGgufTensorInfo, size_bytes); OFF(Mono27BGgufTensorInfo, n_dims); OFF(Mono27BGgufTensorInfo, dims);
    SZ(Mono27BAttentionLayerWeights);
    OFF(Mono27BAttentionLayerWeights, wq); OFF(Mono27BAttentionLayerWeights, gate);
    OFF(Mono27BAttentionLayerWeights, post_norm); OFF(Mono27BAttentionLayerWeights, ffn_down);
    SZ(Mono27BSSMLayerWeights);
    OFF(Mono27BSSMLayerWeights, wqkv_gate); OFF(Mono27BSSMLayerWeights, ssm_a_log);
    OFF(Mono27BSSMLayerWeights, ssm_out); OFF(Mono27BSSMLayerWeights, ffn_down);
    SZ(Mono27BExecutorWeights);
    OFF(Mono27BExecutorWeights, layers); OFF(Mono27BExecutorWeights, output_norm);
    OFF(Mono27BExecutorWeights, lm_head); OFF(Mono27BExecutorWeights, tok_embd);
    std::printf("offsetof layers[1] %zu\n", (size_t)((const char *)&((Mono27BExecutorWeights *)0)->layers[1] -
                                                     (const char *)0));
    std::printf("offsetof layers[0].attn %zu\n",
                (size_t)((const char *)&((Mono27BExecutorWeights *)0)->layers[0].attn - (const char *)0));
    SZ(Mono27BExecutorState);
    OFF(Mono27BExecutorState, kv_cache_v); OFF(Mono27BExecutorState, ssm_state); OFF(Mono27BExecutorState, conv_state);
    OFF(Mono27BExecutorState, attn_split_o); OFF(Mono27BExecutorState, work_buf);
    OFF(Mono27BExecutorState, work_buf_size); OFF(Mono27BExecutorState, q8_scratch);
    OFF(Mono27BExecutorState, argmax_result); OFF(Mono27BExecutorState, cuda_graph_exec);
    OFF(Mono27BExecutorState, graph_captured); OFF(Mono27BExecutorState, max_ctx); OFF(Mono27BExecutorState, kv_len);
    OFF(Mono27BExecutorState, stream1); OFF(Mono27BExecutorState, sync_event);
    SZ(Mono27BLogitsOutput);
#ifdef M27B_PROBE_REFERENCE_HEADERS
    if (argc > 1 && std::strcmp(argv[1], "--call") == 0) {
        char err[256];
        // a tensor table without token_embd: rejected before any device work
        std::vector<Mono27BGgufTensorInfo> ts(1);
        ts[0].name = "blk.0.attn_norm.weight";
        unsigned char data[16] = {};
        Mono27BExecutorWeights *w = new Mono27BExecutorWeights();
        const bool lw = mono27b_engine_load_weights(data, 0, ts.data(), ts.size(), w, err, sizeof(err));
        std::printf("load_weights %d %s\n", (int)lw, err);
        Mono27BLogitsOutput out{};
        out.logits = (float *)16;
        mono27b_engine_free_logits(&out);
        std::printf("free_logits %d\n", out.logits == nullptr ? 1 : 0);
        Mono27BExecutorState *st = new Mono27BExecutorState();
        mono27b_engine_free_state(st);  // a zeroed state: nothing to release
        std::printf("free_state ok\n");
        std::printf("argmax %d\n", mono27b_engine_argmax(st, nullptr, 0));
        mono27b_engine_free_weights(w);
        // the matvec seam with the reference's WeightView
        WeightView v{};
        v.ptr = (void *)256;
        v.ggml_type = 12;
        v.row_blocks = 20;
        v.row_count = 8;
        const bool q = m27b_qmv(&v, nullptr, 1, nullptr, 8, nullptr, 0, err, sizeof(err));
        std::printf("m27b_qmv %d %s\n", (int)q, err);
        delete st;
        delete w;
    }
#endif
    return 0;
}
