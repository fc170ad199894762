// spec.cpp — greedy speculative decoding over two engines (see
// m27b_engine_speculative_generate in include/m27b_engine.h).
//
// The reference lists the speculative loop as its next step and has no
// implementation of it (README.md:41-45); its draft model constants are in
// include/mono27b_format.h:10,17,19,27.  The loop: the draft proposes k
// tokens by greedy decoding on the device (m27b_engine_generate), the target
// scores the last accepted token and the k proposals in one verify pass of
// k + 1 tokens (m27b_engine_verify), and the longest prefix on which the
// target's greedy choice equals the proposal is kept, followed by the
// target's own choice after it.  The output therefore equals the target's
// plain greedy decoding.  KV entries past a rejection are left in place:
// positions index the caches, so later steps overwrite them.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "m27b_engine.h"

namespace {

bool sfail(char *err, size_t cap, const char *fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(err, cap, fmt, ap);
        va_end(ap);
    }
    return false;
}

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

extern "C" {

bool m27b_engine_speculative_generate(M27BEngine *target, M27BEngine *draft, const int *prompt, int n_prompt,
                                      int n_new, int k, int *out_tokens, M27BSpecStats *stats, char *err,
                                      size_t err_cap) {
    if (err && err_cap) err[0] = '\0';
    if (!target || !draft || !prompt || !out_tokens)
        return sfail(err, err_cap, "m27b_engine_speculative_generate: null argument");
    if (n_prompt < 1 || n_new < 1) return sfail(err, err_cap, "m27b_engine_speculative_generate: empty prompt or output");
    if (k < 1 || k >= M27B_VERIFY_MAX)
        return sfail(err, err_cap, "m27b_engine_speculative_generate: k must be in [1, %d] (got %d)", M27B_VERIFY_MAX - 1,
                     k);
    M27BSpecStats st{};
    using clk = std::chrono::steady_clock;
    char e2[512];
    auto t0 = clk::now();
    // the prompt except its last token, into both caches
    for (int pos = 0; pos + 1 < n_prompt; ++pos) {
        int nx = 0;
        if (!m27b_engine_decode_step(target, prompt[pos], pos, &nx, nullptr, err, err_cap)) return false;
        if (!m27b_engine_decode_step(draft, prompt[pos], pos, &nx, nullptr, err, err_cap)) return false;
    }
    st.prefill_ms = ms_since(t0);
    std::vector<int> props(k), nxt(k + 1), ver(k + 1);
    int last = prompt[n_prompt - 1], pos = n_prompt - 1, made = 0;
    while (made < n_new) {
        t0 = clk::now();
        // draft K/V at pos .. pos+k-1; props[i] is its choice after position pos+i
        if (!m27b_engine_generate(draft, last, pos, k, props.data(), err, err_cap)) return false;
        st.draft_ms += ms_since(t0);
        ver[0] = last;
        for (int i = 0; i < k; ++i) ver[i + 1] = props[i];
        t0 = clk::now();
        // target K/V at pos .. pos+k; nxt[i] is its choice after position pos+i
        if (!m27b_engine_verify(target, ver.data(), k + 1, pos, nxt.data(), nullptr, err, err_cap)) return false;
        st.verify_ms += ms_since(t0);
        int j = 0;
        while (j < k && props[j] == nxt[j]) ++j;
        if (j == k) {
            // every proposal kept: the draft has not yet seen its own last one
            t0 = clk::now();
            int nx = 0;
            if (!m27b_engine_decode_step(draft, props[k - 1], pos + k, &nx, nullptr, e2, sizeof(e2)))
                return sfail(err, err_cap, "%s", e2);
            st.draft_ms += ms_since(t0);
        }
        for (int i = 0; i < j && made < n_new; ++i) out_tokens[made++] = props[i];
        if (made < n_new) out_tokens[made++] = nxt[j];
        ++st.iterations;
        st.proposed += k;
        st.accepted += j;
        last = nxt[j];
        pos += j + 1;
    }
    if (stats) *stats = st;
    return true;
}

}  // extern "C"
