// mono27b_api.cu — the reference executor's C API (include/mono27b_api.h)
// over the decode engine.
//
// Replaces src/mono27b_executor.cu:1727-1833 (load / free weights),
// :1858-1984 (init / free state), :2294-2623 (decode step), :2625-2664
// (free_logits, argmax, embed).  The reference keeps weights and per-sequence
// state apart; here a "weights" engine holds the tensors and every state gets
// its own engine that borrows them (m27b_engine_create_sharing), created at
// its first decode step because the reference's driver initialises the state
// before it loads the weights (src/mono27b_chat.cpp:352-367).
#include <cuda_runtime.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "m27b_device.cuh"
#include "m27b_engine.h"
#include "mono27b_api.h"
#include "engine_state.h"

using namespace m27b;

namespace {

bool afail(char *err, size_t cap, const char *fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(err, cap, fmt, ap);
        va_end(ap);
    }
    return false;
}

// A loaded set of weights: the engine that owns them, and how many states
// borrow them.  Keyed by the token-embedding device pointer, which a copy of
// the caller's Mono27BExecutorWeights carries too.
struct WeightsEntry {
    M27BEngine *e = nullptr;
    int refs = 0;
    bool released = false;  // free_weights was called while states still use it
};

struct StateEntry {
    M27BEngine *e = nullptr;    // this state's engine (KV cache, graphs)
    M27BEngine *src = nullptr;  // the weights engine it borrows from
    int max_ctx = 0;
    double ms = 0.0;  // host time of decode steps since the last reset
    long steps = 0;
};

std::mutex g_mu;
std::map<const void *, WeightsEntry> g_weights;  // tok_embd.ptr -> entry
std::map<const Mono27BExecutorState *, StateEntry> g_states;
int32_t *g_tok_word[64] = {};  // per device: the row index of mono27b_engine_embed

void release_weights_locked(M27BEngine *src) {
    for (auto it = g_weights.begin(); it != g_weights.end(); ++it)
        if (it->second.e == src) {
            if (--it->second.refs <= 0 && it->second.released) {
                m27b_engine_destroy(it->second.e);
                g_weights.erase(it);
            }
            return;
        }
}

using TensorMap = std::map<std::string, const Mono27BGgufTensorInfo *>;

const Mono27BGgufTensorInfo *find(const TensorMap &by, const std::string &n) {
    auto it = by.find(n);
    return it == by.end() || it->second->size_bytes == 0 ? nullptr : it->second;
}

uint64_t rows_of(const Mono27BGgufTensorInfo *t) { return t->n_dims > 1 ? t->dims[1] : 1; }

WeightView f32_view(const float *p, uint32_t n) {
    WeightView v{};
    v.ptr = (void *)p;
    v.ggml_type = p ? M27B_TYPE_F32 : 0;
    v.row_blocks = p ? n : 0;
    v.row_count = p ? 1 : 0;
    return v;
}

// rows [r0, r0 + n) of a stored matrix as a view of its own
WeightView row_view(const QMat &m, int r0, int n) {
    if (!m.d) return WeightView{};
    WeightView v = m.v;
    v.ptr = (uint8_t *)m.d + stored_row_bytes(m) * (size_t)r0;
    v.row_count = (uint32_t)n;
    return v;
}

// Model shape from the tensor descriptors (the reference reads the same
// tensors by name, src/mono27b_executor.cu:1739-1831).  Rotary dims, theta
// and eps are the reference's constants (include/mono27b_config.h:20-21, :57).
bool infer_config(const TensorMap &by, M27BModelConfig &c, char *err, size_t cap) {
    std::memset(&c, 0, sizeof(c));
    const Mono27BGgufTensorInfo *emb = find(by, "token_embd.weight");
    if (!emb) return afail(err, cap, "mono27b_engine_load_weights: token_embd.weight not found");
    c.hidden = (int)emb->dims[0];
    c.vocab = (int)rows_of(emb);
    int nl = 0;
    for (const auto &kv : by) {
        int l = -1;
        if (std::sscanf(kv.first.c_str(), "blk.%d.", &l) == 1 && l + 1 > nl) nl = l + 1;
    }
    if (nl < 1) return afail(err, cap, "mono27b_engine_load_weights: no blk.N tensors");
    if (nl > (int)MONO27B_TARGET_LAYERS)
        return afail(err, cap, "mono27b_engine_load_weights: %d layers; Mono27BExecutorWeights holds %u", nl,
                     MONO27B_TARGET_LAYERS);
    c.n_layers = nl;
    auto name = [](int l, const char *s) { return "blk." + std::to_string(l) + "." + s; };
    std::vector<bool> attn(nl);
    int first_attn = -1, first_ssm = -1;
    for (int l = 0; l < nl; ++l) {
        attn[l] = find(by, name(l, "ssm_out.weight")) == nullptr;
        if (attn[l] && first_attn < 0) first_attn = l;
        if (!attn[l] && first_ssm < 0) first_ssm = l;
    }
    if (first_attn < 0) return afail(err, cap, "mono27b_engine_load_weights: no attention layer");
    c.attn_interval = 0;
    if (first_ssm >= 0) {
        for (int k = 2; k <= nl && !c.attn_interval; ++k) {
            bool ok = true;
            for (int l = 0; l < nl && ok; ++l) ok = attn[l] == ((l + 1) % k == 0);
            if (ok) c.attn_interval = k;
        }
        if (!c.attn_interval)
            return afail(err, cap, "mono27b_engine_load_weights: attention layers are not every k-th layer");
    }
    const Mono27BGgufTensorInfo *qn = find(by, name(first_attn, "attn_q_norm.weight"));
    const Mono27BGgufTensorInfo *wq = find(by, name(first_attn, "attn_q.weight"));
    const Mono27BGgufTensorInfo *wk = find(by, name(first_attn, "attn_k.weight"));
    const Mono27BGgufTensorInfo *fg = find(by, name(0, "ffn_gate.weight"));
    if (!qn || !wq || !wk || !fg)
        return afail(err, cap, "mono27b_engine_load_weights: layer %d: attention or FFN tensors missing", first_attn);
    c.head_dim = (int)qn->dims[0];
    if (c.head_dim <= 0) return afail(err, cap, "mono27b_engine_load_weights: bad attn_q_norm");
    c.n_head = (int)(rows_of(wq) / (2 * (uint64_t)c.head_dim));
    c.n_kv_head = (int)(rows_of(wk) / (uint64_t)c.head_dim);
    c.ffn = (int)rows_of(fg);
    c.n_rot = c.head_dim < 64 ? c.head_dim : 64;
    c.rope_theta = 10000000.0f;
    c.rms_eps = 1e-6f;
    c.tp_rank = 0;
    c.tp_size = 1;
    if (first_ssm >= 0) {
        const Mono27BGgufTensorInfo *so = find(by, name(first_ssm, "ssm_out.weight"));
        const Mono27BGgufTensorInfo *cv = find(by, name(first_ssm, "ssm_conv1d.weight"));
        const Mono27BGgufTensorInfo *sa = find(by, name(first_ssm, "ssm_a"));
        if (!sa) sa = find(by, name(first_ssm, "ssm_a_log"));
        if (!so || !cv || !sa)
            return afail(err, cap, "mono27b_engine_load_weights: layer %d: DeltaNet tensors missing", first_ssm);
        c.ssm_d_inner = (int)so->dims[0];
        c.ssm_dt_rank = (int)sa->dims[0];
        c.ssm_d_state = 128;
        c.ssm_conv_kern = (int)cv->dims[0];
        c.ssm_n_group = ((int)rows_of(cv) - c.ssm_d_inner) / (2 * c.ssm_d_state);
    }
    return true;
}

// Names the reference loader reads (src/mono27b_executor.cu:1739-1831),
// under the engine's spelling; everything else is skipped as there.
bool wanted(const std::string &n, bool ssm_layer) {
    static const char *attn_names[] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
                                       "attn_output.weight", "attn_gate.weight", "attn_q_norm.weight",
                                       "attn_k_norm.weight", "post_attention_norm.weight", "ffn_gate.weight",
                                       "ffn_up.weight", "ffn_down.weight"};
    static const char *ssm_names[] = {"attn_norm.weight", "attn_qkv.weight", "attn_q.weight", "ssm_in.weight",
                                      "attn_gate.weight", "attn_k.weight", "ssm_in_gate.weight", "ssm_conv1d.weight",
                                      "ssm_beta.weight", "ssm_alpha.weight", "ssm_dt_bias", "ssm_dt.bias",
                                      "ssm_a_log", "ssm_a", "ssm_norm.weight", "ssm_out.weight",
                                      "post_attention_norm.weight", "ffn_gate.weight", "ffn_up.weight",
                                      "ffn_down.weight"};
    if (ssm_layer) {
        for (const char *s : ssm_names)
            if (n == s) return true;
    } else {
        for (const char *s : attn_names)
            if (n == s) return true;
    }
    return false;
}

// Describe the engine's tensors in the reference's weight struct.
void fill_views(const M27BEngine *e, Mono27BExecutorWeights *w) {
    std::memset(w, 0, sizeof(*w));
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim;
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer &L = e->L[l];
        auto &d = w->layers[l];
        d.is_attention = !L.ssm;
        if (!L.ssm) {
            Mono27BAttentionLayerWeights &a = d.attn;
            a.attn_norm = f32_view(L.attn_norm, c.hidden);
            a.wq = row_view(L.wqkv, 0, c.n_head * 2 * hd);
            a.wk = row_view(L.wqkv, c.n_head * 2 * hd, c.n_kv_head * hd);
            a.wv = row_view(L.wqkv, c.n_head * 2 * hd + c.n_kv_head * hd, c.n_kv_head * hd);
            a.wo = L.wo.v;
            a.q_norm = f32_view(L.q_norm, hd);
            a.k_norm = f32_view(L.k_norm, hd);
            a.post_norm = f32_view(L.post_norm, c.hidden);
            a.ffn_gate = L.wg.v;
            a.ffn_up = L.wu.v;
            a.ffn_down = L.wd.v;
        } else {
            Mono27BSSMLayerWeights &s = d.ssm;
            const int dr = c.ssm_dt_rank;
            s.attn_norm = f32_view(L.attn_norm, c.hidden);
            s.wqkv = L.wqs.v;
            s.wqkv_gate = L.wz.v;
            s.ssm_conv1d = f32_view(L.conv_w, (uint32_t)c.ssm_conv_kern);
            s.ssm_conv1d.row_count = L.conv_w ? (uint32_t)e->conv_ch : 0;
            s.ssm_beta = row_view(L.wba, 0, dr);
            s.ssm_alpha = row_view(L.wba, dr, dr);
            s.ssm_dt_bias = f32_view(L.dt_bias, dr);
            s.ssm_a_log = f32_view(L.ssm_a, dr);
            s.ssm_norm = f32_view(L.ssm_norm, 128);
            s.ssm_out = L.wso.v;
            s.post_norm = f32_view(L.post_norm, c.hidden);
            s.ffn_gate = L.wg.v;
            s.ffn_up = L.wu.v;
            s.ffn_down = L.wd.v;
        }
    }
    w->output_norm = f32_view(e->out_norm, c.hidden);
    w->lm_head = e->lmh.v;
    w->tok_embd = e->embd.v;
}

// The state's pointers into its engine (the reference's fields, same roles).
void fill_state(const M27BEngine *e, Mono27BExecutorState *st) {
    int fa = 0, ss = 0;
    for (const Layer &L : e->L) {
        if (!L.ssm && fa < MONO27B_TARGET_FA_LAYERS) {
            st->kv_cache_k[fa] = L.kc;
            st->kv_cache_v[fa++] = L.vc;
        } else if (L.ssm && ss < (int)MONO27B_TARGET_LAYERS - MONO27B_TARGET_FA_LAYERS) {
            st->ssm_state[ss] = L.S;
            st->conv_state[ss++] = L.cstate;
        }
    }
    st->attn_split_o = e->part;
    st->work_buf = e->logits;
    st->work_buf_size = (size_t)e->V * sizeof(float);
    st->q8_scratch = e->xq;
    st->cuda_graph_exec = (void *)e->gexec;
    st->graph_captured = e->gexec ? 1 : 0;
    st->stream1 = (void *)e->st;
}

// Packed-key argmax over n floats (ties to the smallest index).
__global__ void k_argmax_f32(const float *v, int n, unsigned long long *best) {
    unsigned long long b = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(v[i], (uint32_t)i);
        b = k > b ? k : b;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, b, o);
        b = x > b ? x : b;
    }
    if ((threadIdx.x & 31) == 0 && b) atomicMax(best, b);
}

}  // namespace

extern "C" {

bool mono27b_engine_load_weights(const unsigned char *gguf_data, uint64_t data_offset,
                                 const Mono27BGgufTensorInfo *tensors, size_t tensor_count,
                                 Mono27BExecutorWeights *gpu_weights, char *error, size_t error_cap) {
    if (error && error_cap) error[0] = '\0';
    if (!gguf_data || !tensors || !gpu_weights)
        return afail(error, error_cap, "mono27b_engine_load_weights: null argument");
    std::memset(gpu_weights, 0, sizeof(*gpu_weights));
    TensorMap by;
    for (size_t i = 0; i < tensor_count; ++i) by[tensors[i].name] = &tensors[i];
    M27BModelConfig c;
    if (!infer_config(by, c, error, error_cap)) return false;
    c.max_ctx = 16;  // the weights engine never decodes; each state has its own cache
    M27BEngine *e = nullptr;
    if (!m27b_engine_create(&c, &e, error, error_cap)) return false;
    for (const auto &kv : by) {
        const Mono27BGgufTensorInfo *t = kv.second;
        if (!t->size_bytes) continue;
        std::string n = t->name;
        int l = -1, off = 0;
        if (std::sscanf(n.c_str(), "blk.%d.%n", &l, &off) == 1 && off > 0) {
            std::string what = n.substr(off);
            if (what == "attn_o.weight") what = "attn_output.weight";  // the reference's first spelling
            if (!wanted(what, e->L[l].ssm)) continue;
            n = "blk." + std::to_string(l) + "." + what;
        } else if (n != "token_embd.weight" && n != "output_norm.weight" && n != "output.weight") {
            continue;
        }
        const uint64_t rows = rows_of(t);
        if (t->dims[0] > 0xffffffffull || rows > 0xffffffffull) {
            m27b_engine_destroy(e);
            return afail(error, error_cap, "mono27b_engine_load_weights: %s: shape too large", n.c_str());
        }
        if (!m27b_engine_load_tensor(e, n.c_str(), t->ggml_type, (uint32_t)t->dims[0], (uint32_t)rows,
                                     gguf_data + data_offset + t->offset, error, error_cap)) {
            m27b_engine_destroy(e);
            return false;
        }
    }
    fill_views(e, gpu_weights);
    if (!gpu_weights->tok_embd.ptr) {
        m27b_engine_destroy(e);
        return afail(error, error_cap, "mono27b_engine_load_weights: token_embd.weight was not loaded");
    }
    std::lock_guard<std::mutex> lk(g_mu);
    g_weights[gpu_weights->tok_embd.ptr] = WeightsEntry{e, 0, false};
    return true;
}

void mono27b_engine_free_weights(Mono27BExecutorWeights *w) {
    if (!w) return;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_weights.find(w->tok_embd.ptr);
        if (it != g_weights.end()) {
            if (it->second.refs > 0) {
                it->second.released = true;  // the last state using them frees them
            } else {
                m27b_engine_destroy(it->second.e);
                g_weights.erase(it);
            }
        }
    }
    std::memset(w, 0, sizeof(*w));
}

bool mono27b_engine_init_state(int max_ctx, Mono27BExecutorState *state, char *error, size_t error_cap) {
    if (error && error_cap) error[0] = '\0';
    if (!state) return afail(error, error_cap, "mono27b_engine_init_state: null state");
    if (max_ctx < 1) return afail(error, error_cap, "mono27b_engine_init_state: max_ctx must be >= 1 (got %d)", max_ctx);
    std::memset(state, 0, sizeof(*state));
    int *am = nullptr;
    const cudaError_t ce = cudaMalloc(&am, sizeof(unsigned long long));
    if (ce != cudaSuccess) {
        cudaGetLastError();
        return afail(error, error_cap, "mono27b_engine_init_state: %s", cudaGetErrorString(ce));
    }
    state->argmax_result = am;
    state->max_ctx = max_ctx;
    state->kv_len = 0;
    std::lock_guard<std::mutex> lk(g_mu);
    g_states[state] = StateEntry{nullptr, nullptr, max_ctx, 0.0, 0};
    return true;
}

void mono27b_engine_free_state(Mono27BExecutorState *state) {
    if (!state) return;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_states.find(state);
        if (it != g_states.end()) {
            if (it->second.e) m27b_engine_destroy(it->second.e);
            if (it->second.src) release_weights_locked(it->second.src);
            g_states.erase(it);
        }
    }
    if (state->argmax_result) cudaFree(state->argmax_result);
    std::memset(state, 0, sizeof(*state));
}

bool mono27b_engine_embed(const Mono27BExecutorWeights *we, int token_id, float *hidden, char *error, size_t error_cap) {
    if (error && error_cap) error[0] = '\0';
    if (!we || !hidden) return afail(error, error_cap, "mono27b_engine_embed: null argument");
    const WeightView &v = we->tok_embd;
    if (!v.ptr) return afail(error, error_cap, "mono27b_engine_embed: no token embedding loaded");
    // a token outside the table gives a zero row, as in the reference; the
    // index reaches the device through a pageable host word (the copy
    // completes before cudaMemcpyAsync returns)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return afail(error, error_cap, "mono27b_engine_embed: no CUDA device");
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_tok_word[dev] && cudaMalloc(&g_tok_word[dev], sizeof(int32_t)) != cudaSuccess)
            return afail(error, error_cap, "mono27b_engine_embed: cannot allocate the index word");
    }
    const int32_t t = token_id;
    if (cudaMemcpyAsync(g_tok_word[dev], &t, sizeof(t), cudaMemcpyHostToDevice, 0) != cudaSuccess)
        return afail(error, error_cap, "mono27b_engine_embed: copying the token failed");
    const int k = (int)v.row_blocks * ((v.ggml_type & M27B_TYPE_MASK) == M27B_TYPE_Q8_0 ? 32 : 256);
    return m27b_dequant_rows(&v, g_tok_word[dev], 1, hidden, k, 0, error, error_cap);
}

bool mono27b_engine_decode_step(const Mono27BExecutorWeights *weights, Mono27BExecutorState *state, int token_id,
                                int position, Mono27BLogitsOutput *output, char *error, size_t error_cap) {
    if (error && error_cap) error[0] = '\0';
    if (!weights || !state || !output) return afail(error, error_cap, "mono27b_engine_decode_step: null argument");
    M27BEngine *e = nullptr;
    StateEntry *se = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto wit = g_weights.find(weights->tok_embd.ptr);
        if (wit == g_weights.end() || wit->second.released)
            return afail(error, error_cap,
                         "mono27b_engine_decode_step: weights not loaded by mono27b_engine_load_weights");
        auto sit = g_states.find(state);
        if (sit == g_states.end())
            return afail(error, error_cap,
                         "mono27b_engine_decode_step: state not initialised (mono27b_engine_init_state)");
        se = &sit->second;
        M27BEngine *src = wit->second.e;
        const int want_ctx = state->max_ctx > 0 ? state->max_ctx : se->max_ctx;
        if (se->e && (se->src != src || se->max_ctx < want_ctx)) {
            // other weights, or a longer context than this state's engine holds
            m27b_engine_destroy(se->e);
            release_weights_locked(se->src);
            se->e = nullptr;
            se->src = nullptr;
        }
        if (!se->e) {
            if (!m27b_engine_create_sharing(src, want_ctx, &se->e, error, error_cap)) return false;
            se->src = src;
            se->max_ctx = want_ctx;
            ++wit->second.refs;
        }
        e = se->e;
    }
    const auto t0 = std::chrono::steady_clock::now();
    int next = 0;
    if (!m27b_engine_decode_step(e, token_id, position, &next, nullptr, error, error_cap)) return false;
    const auto t1 = std::chrono::steady_clock::now();
    se->ms += std::chrono::duration<double, std::milli>(t1 - t0).count();
    ++se->steps;
    fill_state(e, state);
    state->kv_len = position + 1;
    output->logits = e->logits;
    return true;
}

void mono27b_engine_free_logits(Mono27BLogitsOutput *output) {
    if (output) output->logits = nullptr;  // the logits belong to the state's engine
}

int mono27b_engine_argmax(Mono27BExecutorState *st, const float *logits, int n) {
    if (!st || !st->argmax_result || !logits || n <= 0) return 0;
    unsigned long long *best = (unsigned long long *)st->argmax_result;
    if (cudaMemsetAsync(best, 0, sizeof(*best), 0) != cudaSuccess) return 0;
    const int want = (n + 255) / 256, blocks = want < 148 * 4 ? want : 148 * 4;
    k_argmax_f32<<<blocks, 256>>>(logits, n, best);
    unsigned long long key = 0;
    if (cudaMemcpy(&key, best, sizeof(key), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    return key ? (int)m27b_argmax_key_index(key) : 0;
}

void mono27b_engine_print_timing(Mono27BExecutorState *st) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_states.find(st);
    if (it == g_states.end() || it->second.steps == 0) {
        std::fprintf(stderr, "m27b: no decode steps timed\n");
        return;
    }
    std::fprintf(stderr, "m27b: %ld decode steps, %.3f ms per step (host time: graph replay + synchronise)\n",
                 it->second.steps, it->second.ms / (double)it->second.steps);
}

void mono27b_engine_reset_timing(Mono27BExecutorState *st) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_states.find(st);
    if (it != g_states.end()) {
        it->second.ms = 0.0;
        it->second.steps = 0;
    }
}

}  // extern "C"
