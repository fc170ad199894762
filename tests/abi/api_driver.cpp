// api_driver.cpp — drives the reference-executor API of libm27b the way the
// reference's chat driver does (src/mono27b_chat.cpp:352-391, :467-471):
// init_state, load_weights from an in-memory GGUF-style tensor table,
// decode_step per token with the logits read back from the device, argmax,
// embed, timing, free_weights then free_state.  Test infrastructure for
// tests/test_ref_api_gpu.py.
//
// usage: api_driver MODEL OUT max_ctx tok0 tok1 ...
// MODEL: "M27T", u32 count, then per tensor u32 name length, name bytes,
// u32 ggml_type, u32 n_dims, u64 dims[4], u64 offset, u64 size_bytes; the
// tensor data follows (offsets relative to its start).
// OUT: float logits[n][vocab], int32 argmax[n], float embed[hidden],
// float embed_out_of_range[hidden].
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "mono27b_api.h"

#define CHECK(c, ...)                          \
    do {                                       \
        if (!(c)) {                            \
            std::fprintf(stderr, __VA_ARGS__); \
            std::fprintf(stderr, "\n");        \
            return 1;                          \
        }                                      \
    } while (0)

int main(int argc, char **argv) {
    CHECK(argc >= 5, "usage: api_driver MODEL OUT max_ctx tokens...");
    FILE *f = std::fopen(argv[1], "rb");
    CHECK(f, "cannot open %s", argv[1]);
    std::vector<unsigned char> file;
    unsigned char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) file.insert(file.end(), buf, buf + n);
    std::fclose(f);
    size_t at = 0;
    auto rd = [&](void *dst, size_t bytes) {
        std::memcpy(dst, file.data() + at, bytes);
        at += bytes;
    };
    char magic[4];
    rd(magic, 4);
    CHECK(std::memcmp(magic, "M27T", 4) == 0, "bad model file");
    uint32_t count = 0;
    rd(&count, 4);
    std::vector<Mono27BGgufTensorInfo> ts(count);
    for (auto &t : ts) {
        uint32_t len = 0;
        rd(&len, 4);
        t.name.assign((const char *)file.data() + at, len);
        at += len;
        rd(&t.ggml_type, 4);
        rd(&t.n_dims, 4);
        rd(t.dims, 32);
        rd(&t.offset, 8);
        rd(&t.size_bytes, 8);
    }
    const uint64_t data_offset = at;
    const int max_ctx = std::atoi(argv[3]);
    std::vector<int> toks;
    for (int i = 4; i < argc; ++i) toks.push_back(std::atoi(argv[i]));

    char err[512] = {};
    Mono27BExecutorState *state = new Mono27BExecutorState();
    CHECK(mono27b_engine_init_state(max_ctx, state, err, sizeof(err)), "init_state: %s", err);
    Mono27BExecutorWeights *w = new Mono27BExecutorWeights();
    CHECK(mono27b_engine_load_weights(file.data(), data_offset, ts.data(), ts.size(), w, err, sizeof(err)),
          "load_weights: %s", err);
    const int vocab = (int)w->tok_embd.row_count;
    const int hidden = (int)w->tok_embd.row_blocks * 256;
    int n_layers = 0, n_attn = 0;
    for (uint32_t l = 0; l < MONO27B_TARGET_LAYERS; ++l)
        if (w->layers[l].is_attention ? w->layers[l].attn.wo.ptr != nullptr : w->layers[l].ssm.ssm_out.ptr != nullptr) {
            ++n_layers;
            n_attn += w->layers[l].is_attention ? 1 : 0;
        }
    std::printf("vocab %d hidden %d layers %d attention %d lm_head_type 0x%x\n", vocab, hidden, n_layers, n_attn,
                w->lm_head.ggml_type);

    FILE *o = std::fopen(argv[2], "wb");
    CHECK(o, "cannot open %s", argv[2]);
    std::vector<float> lg(vocab);
    std::vector<int32_t> am;
    mono27b_engine_reset_timing(state);
    for (size_t i = 0; i < toks.size(); ++i) {
        Mono27BLogitsOutput out{};
        CHECK(mono27b_engine_decode_step(w, state, toks[i], (int)i, &out, err, sizeof(err)), "decode_step %zu: %s", i,
              err);
        CHECK(out.logits && state->kv_len == (int)i + 1, "decode_step %zu: no logits / kv_len %d", i, state->kv_len);
        CHECK(cudaMemcpy(lg.data(), out.logits, (size_t)vocab * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy");
        std::fwrite(lg.data(), 4, vocab, o);
        am.push_back(mono27b_engine_argmax(state, out.logits, vocab));
        mono27b_engine_free_logits(&out);
        CHECK(out.logits == nullptr, "free_logits");
    }
    mono27b_engine_print_timing(state);
    std::fwrite(am.data(), 4, am.size(), o);
    float *dh = nullptr;
    CHECK(cudaMalloc(&dh, (size_t)hidden * 4) == cudaSuccess, "cudaMalloc");
    std::vector<float> row(hidden);
    for (int tok : {5, vocab + 3}) {
        CHECK(mono27b_engine_embed(w, tok, dh, err, sizeof(err)), "embed: %s", err);
        CHECK(cudaDeviceSynchronize() == cudaSuccess, "embed sync");
        CHECK(cudaMemcpy(row.data(), dh, (size_t)hidden * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy");
        std::fwrite(row.data(), 4, hidden, o);
    }
    std::fclose(o);
    cudaFree(dh);
    // the weights are released while the state still uses them: further
    // steps are refused, and the state's free releases them for good
    mono27b_engine_free_weights(w);
    Mono27BLogitsOutput out{};
    const bool after = mono27b_engine_decode_step(w, state, toks[0], 0, &out, err, sizeof(err));
    std::printf("decode_after_free %d %s\n", (int)after, err);
    mono27b_engine_free_state(state);
    std::printf("done\n");
    delete w;
    delete state;
    return 0;
}
