// engine.cu — decode engine (see include/m27b_engine.h).
//
// Host-side counterpart of the reference executor's load / state / decode
// functions (src/mono27b_executor.cu:1674-2664) for the attention layers of
// a Qwen-27B-shaped model, built on the sm_100a quantized matvec C ABI and
// extended with tensor parallelism over NCCL.  One engine per process and
// GPU; the whole decode step (64 layers, lm_head, argmax, all-reduces) is
// captured once into a CUDA graph and replayed (the reference captures its
// step the same way, :2353-2360); token and position live in device memory so
// that the replayed graph reads the current ones.
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "m27b_device.cuh"
#include "m27b_blob.h"
#include "m27b_engine.h"
#include "m27b_launch.cuh"
#include "qmv_kernels.cuh"
#include "engine_state.h"

namespace m27b {
__global__ void k_qk_norm_rope_cache(const float *qkv, const float *q_norm, const float *k_norm, float *q, float *gate,
                                     float *kc, float *vc, const int *pos_p, int nq, int nkv, int hd, int n_rot,
                                     float theta, float eps, int qkv_stride, int qg_stride);
cudaError_t attn_prepare();
bool attn_fused_supported(int hd);
cudaError_t attn_fused_launch(const float *qkv, const float *q_norm, const float *k_norm, float *kc, float *vc,
                              float *part, void *xq, const int *pos, int nq, int nkv, int hd, int S, float scale,
                              const float2 *rope, int n_rot, float eps, cudaStream_t st);
cudaError_t rope_table_launch(float2 *rope, const int *pos, int n_rot, float theta, cudaStream_t st);
bool attn_batch_supported(int hd, int G, int smax);
cudaError_t attn_batch_launch(const float *q, const float *gate, const float *kc, const float *vc, float *part,
                              void *xq, const int *pos, unsigned *count, int nq, int nkv, int hd, int S, float scale,
                              int n_tok, cudaStream_t st);

cudaError_t attn_launch(const float *q, const float *kc, const float *vc, float *part, float *out, const int *pos,
                        int nq, int nkv, int hd, int S, float scale, cudaStream_t st, int n_tok = 1);
__global__ void k_fill_blocks(uint8_t *out, int type, int rows, int nblk, long row0, int blk0, uint64_t seed, int tid,
                              float sigma);
__global__ void k_fill_f32(float *out, long n, float v);
__global__ void k_advance(const unsigned long long *best, int *ctl, int *hist, int cap);
struct BestExchange {
    uint2 *dst[8];
    const uint2 *slots;
    int npeers;
    int *status;
};
__global__ void k_advance_p2p(unsigned long long *best, int *ctl, int *hist, int cap, BestExchange b);
bool qmv_push(const WeightView *w, const void *xq, const float *residual, const PushArgs &push, cudaStream_t stream,
              char *err, size_t cap, const float *xf = nullptr);
bool qmv_q6k_ksplit(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                    float *part, unsigned *count, cudaStream_t stream, char *err, size_t cap);
bool qmv_swiglu_q8(const WeightView *gate, const WeightView *up, const void *xq, const float *xf, const float *norm_w,
                   float eps, float *y, void *q8out, unsigned *q8cnt, cudaStream_t stream, char *err, size_t cap);
int q6k_ksplit_ranges(int rb);
bool q4k_mma_supported(int rb, int n_tok);
size_t q4k_mma_split_part_floats(int rows, int rb, int n_tok);
size_t q4k_mma_split_count_words(int rows);
bool qmv_mma_split(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                   float *part, unsigned *count, cudaStream_t stream, char *err, size_t cap);
size_t q6k_stream_part_floats(int rows, int rb);
size_t q6k_stream_count_words(int rows);
bool q6k_stream_applies(int k);
bool qmv_q6k_stream(const WeightView *w, const void *xq, const float *xf, float *y, const float *residual, float *part,
                    unsigned *count, cudaStream_t stream, char *err, size_t cap, const PushArgs *push);
size_t q6k_ksplit_part_floats(int rows, int ks);
// q6_K on the tensor cores (qmv_q6k_mma.cu, capi.cu)
bool q6k_mma_supported(int rows, int rb, int n_tok, bool split, int sm_count);
size_t q6k_mma_part_floats(int rows);
size_t q6k_mma_count_words(int rows);
bool qmv_q6k_mma(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                 unsigned long long *best, uint32_t row_offset, int epi, float *part, unsigned *count,
                 cudaStream_t stream, char *err, size_t cap);
// Gated DeltaNet block (ssm.cu)
cudaError_t ssm_rmsnorm_launch(const float *x, const float *w, float eps, int n, float *y, cudaStream_t st);
cudaError_t ssm_conv_launch(const float *x, const float *w, float *cstate, float *out, const float *ba,
                            const float *dt_bias, const float *ssm_a, float *bg, int conv_ch, int K, int ng, int dr,
                            float eps, cudaStream_t st);
cudaError_t ssm_delta_launch(const float *xc, const float *bg, const float *z, const float *ssm_norm, float *S,
                             void *xq, int ng, int dr, float eps, cudaStream_t st);
__global__ void k_fill_f32_rand(float *out, long n, uint64_t seed, float scale, float offset);
}  // namespace m27b

using namespace m27b;

namespace {

bool efail(char *err, size_t cap, const char *fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(err, cap, fmt, ap);
        va_end(ap);
    }
    return false;
}

#define ECUDA(call)                                                                                        \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess) return efail(err, err_cap, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                            __FILE__, __LINE__);                                           \
    } while (0)
#define ENCCL(call)                                                                                          \
    do {                                                                                                     \
        ncclResult_t r_ = (call);                                                                            \
        if (r_ != ncclSuccess) return efail(err, err_cap, "%s: %s", #call, ncclGetErrorString(r_));          \
    } while (0)
#define ECALL(call)                 \
    do {                            \
        if (!(call)) return false;  \
    } while (0)

// IEEE binary16 bits -> float (host; exact).
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (ex == 0x1f) bits = sign | 0x7f800000u | (man << 13);
    else if (ex != 0) bits = sign | ((ex + 112u) << 23) | (man << 13);
    else {
        const float v = (float)man * 5.9604644775390625e-08f;  // subnormal: man * 2^-24
        return sign ? -v : v;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

size_t block_bytes(uint32_t t) {
    switch (t) {
    case M27B_TYPE_F32: return 4;
    case M27B_TYPE_F16: return 2;
    case M27B_TYPE_Q4_K: return 144;
    case M27B_TYPE_Q5_K: return 176;
    case M27B_TYPE_Q6_K: return 210;
    case M27B_TYPE_IQ4_XS: return 136;
    case M27B_TYPE_Q8_0: return 34;
    default: return 0;
    }
}
int block_elems(uint32_t t) {
    return t == M27B_TYPE_Q8_0 ? 32 : (t == M27B_TYPE_F16 || t == M27B_TYPE_F32) ? 1 : 256;
}
// q4_K, q5_K, IQ4_XS, f16 and f32 rows are read in their GGUF layout; q6_K and q8_0 are repacked.
bool raw_layout(uint32_t t) {
    return t == M27B_TYPE_Q4_K || t == M27B_TYPE_Q5_K || t == M27B_TYPE_IQ4_XS || t == M27B_TYPE_F16 ||
           t == M27B_TYPE_F32;
}
// layer il of a hybrid model is attention iff (il + 1) % attn_interval == 0 (reference :2372)
bool is_attention_layer(const M27BModelConfig &c, int il) {
    return c.attn_interval <= 0 || (il + 1) % c.attn_interval == 0;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// q8_0 matrices take q8_0 activations, the k-quants q8_K (ggml's pairing).
uint32_t act_type_of(uint32_t weight_type) {
    return weight_type == M27B_TYPE_Q8_0 ? M27B_TYPE_Q8_0 : M27B_TYPE_Q8_K;
}

// Receive window of the fused all-reduce (same layout on every rank), in
// epoch-tagged 8-byte words {value bits, epoch}:
//   recv  [2 parities][N source ranks][hidden]  partial rows
//   ss    [2 parities][hidden / 256]             the consumer CTAs' sums of squares
//   best  [N][2]                                 argmax keys (low word, high word)
// o_proj uses parity 0 and ffn_down parity 1, so a rank that runs one
// all-reduce ahead never overwrites words a slower rank is still reading.
struct WinLayout {
    size_t recv, ss, best, total;
};
WinLayout win_layout(int N, int hidden) {
    WinLayout w;
    size_t off = 0;
    w.recv = off;
    off = align256(off + (size_t)2 * N * hidden * sizeof(uint2));
    w.ss = off;
    off = align256(off + (size_t)2 * (hidden / 256) * sizeof(uint2));
    w.best = off;
    off = align256(off + (size_t)N * 2 * sizeof(uint2));
    w.total = off;
    return w;
}

}  // namespace


namespace {

bool dalloc(M27BEngine *e, void **p, size_t n, char *err, size_t err_cap) {
    ECUDA(cudaMalloc(p, n ? n : 16));
    e->allocs.push_back(*p);
    return true;
}

// Make sure a matrix of `type` with rows x k values exists (allocated on first use).
bool ensure_mat(M27BEngine *e, QMat &m, uint32_t type, int rows, int k, char *err, size_t err_cap) {
    if (m.d) {
        if (m.type != type || m.rows != rows || m.k != k)
            return efail(err, err_cap, "tensor shape/type differs from the first load (%u %dx%d vs %u %dx%d)", type, rows,
                         k, m.type, m.rows, m.k);
        return true;
    }
    if (block_bytes(type) == 0)
        return efail(err, err_cap, "unsupported matrix type %u (q4_K, q5_K, q6_K, IQ4_XS, q8_0)", type);
    if (k % block_elems(type)) return efail(err, err_cap, "k=%d not a multiple of the block size", k);
    const uint32_t rb = (uint32_t)(k / block_elems(type));
    if (type == M27B_TYPE_IQ4_XS && (rb & 1u))
        return efail(err, err_cap, "IQ4_XS matrices need an even number of blocks per (rank's) row, got %u", rb);
    const size_t raw = (size_t)rows * rb * block_bytes(type);
    const size_t n = raw_layout(type) ? raw : m27b_repacked_bytes(type, rb, (uint32_t)rows);
    ECALL(dalloc(e, &m.d, n, err, err_cap));
    m.type = type;
    m.rows = rows;
    m.k = k;
    m.gguf_bytes = raw;
    m.v.ptr = m.d;
    m.v.ggml_type = raw_layout(type) ? type : (type | M27B_LAYOUT_PLANAR);
    m.v.row_blocks = rb;
    m.v.row_count = (uint32_t)rows;
    return true;
}

bool ensure_scratch(M27BEngine *e, size_t n, char *err, size_t err_cap) {
    if (e->scratch_bytes >= n) return true;
    if (e->scratch) ECUDA(cudaFree(e->scratch));
    e->scratch = nullptr;
    ECUDA(cudaMalloc(&e->scratch, n));
    e->scratch_bytes = n;
    return true;
}

// Place raw GGUF rows (device, `rows` x row_blocks blocks) at row `row_at` of m.
bool place_rows(M27BEngine *e, QMat &m, const uint8_t *raw_dev, int rows, int row_at, char *err, size_t err_cap) {
    const size_t rowb = (size_t)m.v.row_blocks * block_bytes(m.type);
    if (raw_layout(m.type)) {
        ECUDA(cudaMemcpyAsync((uint8_t *)m.d + (size_t)row_at * rowb, raw_dev, rowb * rows, cudaMemcpyDeviceToDevice, e->st));
        return true;
    }
    const size_t prow = m27b_repacked_bytes(m.type, m.v.row_blocks, 1);
    char e2[256];
    if (!m27b_repack(raw_dev, m.type, m.v.row_blocks, (uint32_t)rows, (uint8_t *)m.d + (size_t)row_at * prow, e->st, e2,
                     sizeof(e2)))
        return efail(err, err_cap, "%s", e2);
    return true;
}

// Copy host GGUF rows [r0, r0+nr) x blocks [b0, b0+nb) of a full tensor
// (row_blocks blocks per row) into m at row row_at.
bool load_slice(M27BEngine *e, QMat &m, const uint8_t *host, uint32_t full_rb, int r0, int nr, int b0, int row_at,
                char *err, size_t err_cap) {
    const size_t bb = block_bytes(m.type);
    const size_t srow = (size_t)full_rb * bb, drow = (size_t)m.v.row_blocks * bb;
    std::vector<uint8_t> tmp(drow * nr);
    for (int r = 0; r < nr; ++r) std::memcpy(tmp.data() + drow * r, host + srow * (r0 + r) + bb * b0, drow);
    ECALL(ensure_scratch(e, tmp.size(), err, err_cap));
    ECUDA(cudaMemcpyAsync(e->scratch, tmp.data(), tmp.size(), cudaMemcpyHostToDevice, e->st));
    ECALL(place_rows(e, m, e->scratch, nr, row_at, err, err_cap));
    ECUDA(cudaStreamSynchronize(e->st));  // tmp and the scratch are reused
    return true;
}

// Generate seeded blocks for rows [r0, r0+nr) x blocks [b0, b0+nb) of global tensor `tid` into m at row row_at.
bool fill_slice(M27BEngine *e, QMat &m, int tid, uint64_t seed, float sigma, long r0, int nr, int b0, int row_at,
                char *err, size_t err_cap) {
    const size_t raw = (size_t)nr * m.v.row_blocks * block_bytes(m.type);
    ECALL(ensure_scratch(e, raw, err, err_cap));
    k_fill_blocks<<<1184, 256, 0, e->st>>>(e->scratch, (int)m.type, nr, (int)m.v.row_blocks, r0, b0, seed, tid, sigma);
    ECUDA(cudaGetLastError());
    ECALL(place_rows(e, m, e->scratch, nr, row_at, err, err_cap));
    ECUDA(cudaStreamSynchronize(e->st));
    return true;
}

bool load_f32(M27BEngine *e, float **dst, const void *host, size_t n, char *err, size_t err_cap) {
    if (!*dst) ECALL(dalloc(e, (void **)dst, n * 4, err, err_cap));
    ECUDA(cudaMemcpyAsync(*dst, host, n * 4, cudaMemcpyHostToDevice, e->st));
    ECUDA(cudaStreamSynchronize(e->st));
    return true;
}

bool mv(M27BEngine *e, const QMat &m, const uint8_t *xq, float *y, const float *res, char *err, size_t err_cap) {
    return m27b_qmv(&m.v, xq, 1, y, m.rows, res, e->st, err, err_cap);
}

// Most rows of the verify pass's q4_K projections (qkv, o_proj, gate/up).
int mma_rows_max(const M27BEngine *e) {
    const int qkv_rows = (2 * e->H + 2 * e->KV) * e->c.head_dim;
    return std::max(std::max(e->c.hidden, e->F), qkv_rows);
}

// Scratch of the verify pass's K-split tensor-core projections: the largest
// of qkv, o_proj and gate/up at 16 tokens.
size_t mma_scratch_floats(const M27BEngine *e) {
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim, qkv_rows = (2 * e->H + 2 * e->KV) * hd;
    size_t m = q4k_mma_split_part_floats(qkv_rows, c.hidden / 256, 16);
    m = std::max(m, q4k_mma_split_part_floats(c.hidden, std::max(1, e->H * hd / 256), 16));
    m = std::max(m, q4k_mma_split_part_floats(e->F, c.hidden / 256, 16));
    return m;
}

// A q4_K projection of a verify pass (5..16 tokens): on the tensor cores
// with K split across CTAs where the kernel serves the shape, else m27b_qmv.
bool vmv(M27BEngine *e, const QMat &m, const uint8_t *xq, int n, float *y, int ldy, const float *res, char *err,
         size_t err_cap) {
    if (e->mma_part && m.v.ggml_type == M27B_TYPE_Q4_K && q4k_mma_supported((int)m.v.row_blocks, n) &&
        q4k_mma_split_part_floats(m.rows, (int)m.v.row_blocks, n) <= mma_scratch_floats(e) &&
        m.rows <= mma_rows_max(e))
        return qmv_mma_split(&m.v, xq, n, y, ldy, res, e->mma_part, e->mma_count, e->st, err, err_cap);
    return m27b_qmv(&m.v, xq, n, y, ldy, res, e->st, err, err_cap);
}

// A repacked q6_K matrix of a verify pass (ffn_down with K split, lm_head
// without) that the tensor-core kernel serves for chunks of up to 8 tokens.
bool q6_verify_mma(const M27BEngine *e, const QMat &m, int n, bool split) {
    if (m.v.ggml_type != (M27B_TYPE_Q6_K | M27B_LAYOUT_PLANAR) || (split && !e->q6m_part)) return false;
    if (split && (size_t)m.rows > (size_t)e->c.hidden) return false;  // the scratch is sized for hidden rows
    for (int t0 = 0; t0 < n; t0 += 8)
        if (!q6k_mma_supported(m.rows, (int)m.v.row_blocks, std::min(8, n - t0), split, e->sms)) return false;
    return true;
}

// The down projection of one token (rows = hidden, long rows): a repacked
// q6_K matrix goes to the kernel that cuts its items evenly over the warps
// (its few row groups do not spread evenly over the SMs as whole groups),
// anything else to the one-pass matvec.
bool down_stream_ok(const M27BEngine *e, const QMat &m) {
    return e->sk_part && m.v.ggml_type == (M27B_TYPE_Q6_K | M27B_LAYOUT_PLANAR) && m.rows <= e->c.hidden &&
           (int)m.v.row_blocks <= e->F / 256 + 1 && q6k_stream_applies((int)m.v.row_blocks * 256);
}

bool down_mv(M27BEngine *e, const QMat &m, const uint8_t *xq, float *y, const float *res, char *err, size_t err_cap) {
    if (down_stream_ok(e, m))
        return qmv_q6k_stream(&m.v, xq, nullptr, y, res, e->sk_part, e->sk_count, e->st, err, err_cap, nullptr);
    return mv(e, m, xq, y, res, err, err_cap);
}

// The same into every rank's window (the fused all-reduce's producer).
bool down_push(M27BEngine *e, const QMat &m, const uint8_t *xq, const float *res, const PushArgs &push, char *err,
               size_t err_cap) {
    if (down_stream_ok(e, m))
        return qmv_q6k_stream(&m.v, xq, nullptr, nullptr, res, e->sk_part, e->sk_count, e->st, err, err_cap, &push);
    return qmv_push(&m.v, xq, res, push, e->st, err, err_cap);
}

bool allreduce_hidden(M27BEngine *e, float *buf, char *err, size_t err_cap) {
    if (e->c.tp_size == 1) return true;
    ENCCL(ncclAllReduce(buf, buf, (size_t)e->c.hidden, ncclFloat32, ncclSum, e->comm, e->st));
    return true;
}

// Producer half of the fused all-reduce: rows of `m` (+ residual) to every
// rank's window, parity `par`, instance `idx` of the step.
PushArgs push_args(M27BEngine *e, int par, unsigned idx) {
    const int N = e->c.tp_size, r = e->c.tp_rank;
    const WinLayout lay = win_layout(N, e->c.hidden);
    PushArgs p{};
    for (int q = 0; q < N; ++q) p.dst[q] = (uint2 *)(e->peer_win[q] + lay.recv) + ((size_t)par * N + r) * e->c.hidden;
    p.epoch_base = (const unsigned *)(e->ctl + 3);
    p.epoch_mul = 2u * (unsigned)e->c.n_layers;
    p.epoch_add = idx + 1u;
    p.npeers = N;
    return p;
}

// Consumer half: every rank's rows of parity `par`, summed in rank order into
// x_out (the replicated hidden state), then RMSNorm with `norm_w` and q8_K
// for the next matvec.
bool consume(M27BEngine *e, int par, unsigned idx, const float *norm_w, float *x_out, char *err, size_t err_cap) {
    const int N = e->c.tp_size;
    const WinLayout lay = win_layout(N, e->c.hidden);
    ActArgs a{};
    a.w = norm_w;
    a.eps = e->c.rms_eps;
    a.k = e->c.hidden;
    a.ldx = e->c.hidden;
    a.out = e->xq;
    a.words = (const uint2 *)(e->win + lay.recv) + (size_t)par * N * e->c.hidden;
    a.nsrc = N;
    a.src_stride = e->c.hidden;
    a.ss_words = (uint2 *)(e->win + lay.ss) + (size_t)par * (e->c.hidden / 256);
    a.epoch_base = (const unsigned *)(e->ctl + 3);
    a.epoch_mul = 2u * (unsigned)e->c.n_layers;
    a.epoch_add = idx + 1u;
    a.x_out = x_out;
    a.status = status_ptr_current();
    if (!a.status) return efail(err, err_cap, "cannot resolve the device status word");
    ECUDA(launch_act_quant(M27B_TYPE_Q8_K, ACT_RMSNORM_SUM, a, 1, e->st));
    return true;
}

// Enqueue one decode step on e->st (token / position read from device memory).
bool enqueue_step(M27BEngine *e, char *err, size_t err_cap) {
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim;
    const bool r0 = c.tp_rank == 0;
    const bool p2p = e->p2p;
    if (p2p) {
        // the fused all-reduce's consumer hands its successors q8_K activations
        bool k_quants = e->lmh.type != M27B_TYPE_Q8_0;
        bool push_types = true;  // o_proj / down store into the windows: q4_K or q6_K kernels
        for (const Layer &Ly : e->L) {
            k_quants = k_quants && Ly.wqkv.type != M27B_TYPE_Q8_0 && Ly.wg.type != M27B_TYPE_Q8_0;
            push_types = push_types && (Ly.wo.type == M27B_TYPE_Q4_K || Ly.wo.type == M27B_TYPE_Q6_K) &&
                         (Ly.wd.type == M27B_TYPE_Q4_K || Ly.wd.type == M27B_TYPE_Q6_K);
        }
        if (!k_quants) return efail(err, err_cap, "the fused NVLink all-reduce needs k-quant (not q8_0) matrices");
        if (!push_types)
            return efail(err, err_cap, "the fused NVLink all-reduce needs q4_K or q6_K attn_output / ffn_down matrices");
    }
    const int *pos = e->ctl + 1;
    // the FFN's gate/up kernel also writes silu(gate) * up as q8_K blocks
    // (into xq2, the down projection's input) when the types allow: no
    // separate quantizer launch
    auto ffn_q8 = [&](const Layer &Ly) {
        const uint32_t g = Ly.wg.v.ggml_type;
        return e->xq2 && e->ffn_cnt && (g == M27B_TYPE_Q4_K || g == M27B_TYPE_Q5_K || g == M27B_TYPE_IQ4_XS) &&
               e->F % 256 == 0 && act_type_of(Ly.wd.type) == M27B_TYPE_Q8_K;
    };
    ECALL(m27b_dequant_rows(&e->embd.v, e->ctl, 1, e->h, c.hidden, e->st, err, err_cap));
    ECUDA(rope_table_launch(e->rope, pos, c.n_rot, c.rope_theta, e->st));  // this step's rotary table
    // with the fused all-reduce the consumer kernel hands each projection its
    // normalised, quantized input; otherwise the projection normalises and
    // quantizes h itself (q4_K: in its prologue)
    if (p2p)
        ECALL(m27b_act_quant_rmsnorm(e->h, e->L[0].attn_norm, c.rms_eps, c.hidden, 1, c.hidden, M27B_TYPE_Q8_K, e->xq,
                                     e->st, err, err_cap));
    for (int l = 0; l < c.n_layers; ++l) {
        Layer &Ly = e->L[l];
        if (Ly.ssm) {
            // Gated DeltaNet block (single GPU): norm, four projections, conv + q/k norm,
            // delta rule + gated norm + q8_K, ssm_out + residual, then the FFN
            const int dr = c.ssm_dt_rank;
            ECUDA(ssm_rmsnorm_launch(e->h, Ly.attn_norm, c.rms_eps, c.hidden, e->hn, e->st));
            ECALL(m27b_qmv_f32(&Ly.wqs.v, e->hn, c.hidden, 1, e->xq, e->sx, e->conv_ch, nullptr, e->st, err, err_cap));
            ECALL(m27b_qmv_f32(&Ly.wz.v, e->hn, c.hidden, 1, e->xq, e->sz, c.ssm_d_inner, nullptr, e->st, err, err_cap));
            ECALL(m27b_qmv_f32(&Ly.wba.v, e->hn, c.hidden, 1, e->xq, e->sba, 2 * dr, nullptr, e->st, err, err_cap));
            ECUDA(ssm_conv_launch(e->sx, Ly.conv_w, Ly.cstate, e->sxc, e->sba, Ly.dt_bias, Ly.ssm_a, e->sbg, e->conv_ch,
                                  c.ssm_conv_kern, c.ssm_n_group, dr, c.rms_eps, e->st));
            ECUDA(ssm_delta_launch(e->sxc, e->sbg, e->sz, Ly.ssm_norm, Ly.S, e->xq, c.ssm_n_group, dr, c.rms_eps, e->st));
            ECALL(mv(e, Ly.wso, e->xq, e->h2, e->h, err, err_cap));
            if (ffn_q8(Ly)) {
                ECALL(qmv_swiglu_q8(&Ly.wg.v, &Ly.wu.v, nullptr, e->h2, Ly.post_norm, c.rms_eps, e->a, e->xq2,
                                    e->ffn_cnt, e->st, err, err_cap));
                ECALL(down_mv(e, Ly.wd, e->xq2, e->h, e->h2, err, err_cap));
                continue;
            }
            ECALL(m27b_qmv_f32_rmsnorm(&Ly.wg.v, &Ly.wu.v, e->h2, c.hidden, Ly.post_norm, c.rms_eps, 1, e->xq, e->a, e->F,
                                       nullptr, e->st, err, err_cap));
            ECALL(m27b_act_quant(e->a, e->F, 1, e->F, act_type_of(Ly.wd.type), e->xq, e->st, err, err_cap));
            ECALL(down_mv(e, Ly.wd, e->xq, e->h, e->h2, err, err_cap));
            continue;
        }
        if (p2p)
            ECALL(mv(e, Ly.wqkv, e->xq, e->qkv, nullptr, err, err_cap));
        else
            ECALL(m27b_qmv_f32_rmsnorm(&Ly.wqkv.v, nullptr, e->h, c.hidden, Ly.attn_norm, c.rms_eps, 1, e->xq, e->qkv,
                                       Ly.wqkv.rows, nullptr, e->st, err, err_cap));
        if (attn_fused_supported(hd) && act_type_of(Ly.wo.type) == M27B_TYPE_Q8_K) {
            // q/k norm + RoPE + KV append + attention, then reduce + gate + q8_K for o_proj
            ECUDA(attn_fused_launch(e->qkv, Ly.q_norm, Ly.k_norm, Ly.kc, Ly.vc, e->part, e->xq, pos, e->H, e->KV, hd,
                                    e->S, 1.0f / sqrtf((float)hd), e->rope, c.n_rot, c.rms_eps, e->st));
        } else {
            ECUDA(launch_pdl(k_qk_norm_rope_cache, dim3(e->H + e->KV), dim3(hd), (size_t)(hd + 32) * 4, e->st,
                             (const float *)e->qkv, (const float *)Ly.q_norm, (const float *)Ly.k_norm, e->q, e->gate,
                             Ly.kc, Ly.vc, pos, e->H, e->KV, hd, c.n_rot, c.rope_theta, c.rms_eps, 0, 0));
            ECUDA(attn_launch(e->q, Ly.kc, Ly.vc, e->part, e->o, pos, e->H, e->KV, hd, e->S, 1.0f / sqrtf((float)hd),
                              e->st));
            ECALL(m27b_act_quant_gated(e->o, e->gate, e->H * hd, 1, e->H * hd, act_type_of(Ly.wo.type), e->xq, e->st,
                                       err, err_cap));
        }
        // o_proj partial (+ residual on rank 0), summed over ranks -> h2, then
        // post-attention RMSNorm -> gate/up SwiGLU; its epilogue writes the
        // down projection's q8_K input (xq2), else a quantizer launch does
        // (quantizing it in the prologue of every down CTA instead, 68 blocks
        // each at K = 17408, measured slower)
        const bool fq = ffn_q8(Ly);
        uint8_t *dxq = fq ? e->xq2 : e->xq;
        if (p2p) {
            ECALL(qmv_push(&Ly.wo.v, e->xq, r0 ? e->h : nullptr, push_args(e, 0, 2u * l), e->st, err, err_cap));
            ECALL(consume(e, 0, 2u * l, Ly.post_norm, e->h2, err, err_cap));
            if (fq)
                ECALL(qmv_swiglu_q8(&Ly.wg.v, &Ly.wu.v, e->xq, nullptr, nullptr, 0.0f, e->a, e->xq2, e->ffn_cnt, e->st,
                                    err, err_cap));
            else
                ECALL(m27b_qmv_swiglu(&Ly.wg.v, &Ly.wu.v, e->xq, 1, e->a, e->F, e->st, err, err_cap));
        } else {
            ECALL(mv(e, Ly.wo, e->xq, e->h2, r0 ? e->h : nullptr, err, err_cap));
            ECALL(allreduce_hidden(e, e->h2, err, err_cap));
            if (fq)
                ECALL(qmv_swiglu_q8(&Ly.wg.v, &Ly.wu.v, nullptr, e->h2, Ly.post_norm, c.rms_eps, e->a, e->xq2,
                                    e->ffn_cnt, e->st, err, err_cap));
            else
                ECALL(m27b_qmv_f32_rmsnorm(&Ly.wg.v, &Ly.wu.v, e->h2, c.hidden, Ly.post_norm, c.rms_eps, 1, e->xq, e->a,
                                           e->F, nullptr, e->st, err, err_cap));
        }
        if (!fq) ECALL(m27b_act_quant(e->a, e->F, 1, e->F, act_type_of(Ly.wd.type), e->xq, e->st, err, err_cap));
        // down partial (+ residual on rank 0), summed over ranks -> h, then the
        // next layer's input RMSNorm (the output norm after the last layer) -> xq
        const float *next_norm = l + 1 < c.n_layers ? e->L[l + 1].attn_norm : e->out_norm;
        if (p2p) {
            ECALL(down_push(e, Ly.wd, dxq, r0 ? e->h2 : nullptr, push_args(e, 1, 2u * l + 1u), err, err_cap));
            ECALL(consume(e, 1, 2u * l + 1u, next_norm, e->h, err, err_cap));
        } else {
            ECALL(down_mv(e, Ly.wd, dxq, e->h, r0 ? e->h2 : nullptr, err, err_cap));
            ECALL(allreduce_hidden(e, e->h, err, err_cap));
        }
    }
    if (!p2p)
        ECALL(m27b_act_quant_rmsnorm(e->h, e->out_norm, c.rms_eps, c.hidden, 1, c.hidden, act_type_of(e->lmh.type),
                                     e->xq, e->st, err, err_cap));
    ECALL(m27b_qmv_argmax(&e->lmh.v, e->xq, 1, e->logits, e->V, e->best, (uint32_t)e->v_lo, e->st, err, err_cap));
    // next token and position for the following step (greedy generation on the device)
    if (p2p) {
        const int N = c.tp_size, r = c.tp_rank;
        const WinLayout lay = win_layout(N, c.hidden);
        BestExchange b{};
        for (int q = 0; q < N; ++q) b.dst[q] = (uint2 *)(e->peer_win[q] + lay.best) + 2 * r;
        b.slots = (const uint2 *)(e->win + lay.best);
        b.npeers = N;
        b.status = status_ptr_current();
        if (!b.status) return efail(err, err_cap, "cannot resolve the device status word");
        k_advance_p2p<<<1, 32, 0, e->st>>>(e->best, e->ctl, e->hist, c.max_ctx, b);
    } else {
        if (c.tp_size > 1) ENCCL(ncclAllReduce(e->best, e->best, 1, ncclUint64, ncclMax, e->comm, e->st));
        k_advance<<<1, 32, 0, e->st>>>(e->best, e->ctl, e->hist, c.max_ctx);
    }
    ECUDA(cudaGetLastError());
    return true;
}

// Enqueue a verify pass over n tokens (device e->vtok, positions ctl[1] ..
// ctl[1]+n-1): the same layer arithmetic as enqueue_step on n rows, with the
// unfused attention (each token at its own position) and the NCCL all-reduce
// of n rows at once — also on an engine whose decode step uses the fused
// NVLink all-reduce (it has the communicator; the verify pass leaves the
// fused path's step counter, ctl[3], alone).
bool enqueue_verify(M27BEngine *e, int n, char *err, size_t err_cap) {
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim, D = c.hidden;
    const bool r0 = c.tp_rank == 0;
    const int *pos = e->ctl + 1;
    const int qkv_rows = e->H * 2 * hd + 2 * e->KV * hd;
    ECALL(m27b_dequant_rows(&e->embd.v, e->vtok, n, e->h, D, e->st, err, err_cap));
    for (int l = 0; l < c.n_layers; ++l) {
        Layer &Ly = e->L[l];
        if (n >= 5 && Ly.wqkv.v.ggml_type == M27B_TYPE_Q4_K) {
            // quantize once, then the tensor cores with K split across CTAs
            ECALL(m27b_act_quant_rmsnorm(e->h, Ly.attn_norm, c.rms_eps, D, n, D, M27B_TYPE_Q8_K, e->xq, e->st, err,
                                         err_cap));
            ECALL(vmv(e, Ly.wqkv, e->xq, n, e->qkv, qkv_rows, nullptr, err, err_cap));
        } else {
            ECALL(m27b_qmv_f32_rmsnorm(&Ly.wqkv.v, nullptr, e->h, D, Ly.attn_norm, c.rms_eps, n, e->xq, e->qkv,
                                       qkv_rows, nullptr, e->st, err, err_cap));
        }
        ECUDA(launch_pdl(k_qk_norm_rope_cache, dim3(e->H + e->KV, n), dim3(hd), (size_t)(hd + 32) * 4, e->st,
                         (const float *)e->qkv, (const float *)Ly.q_norm, (const float *)Ly.k_norm, e->q, e->gate, Ly.kc,
                         Ly.vc, pos, e->H, e->KV, hd, c.n_rot, c.rope_theta, c.rms_eps, qkv_rows, e->H * hd));
        if (attn_batch_supported(hd, e->G, e->S) && act_type_of(Ly.wo.type) == M27B_TYPE_Q8_K) {
            // every token's split attention, reduction, gate and q8_K in one launch
            ECUDA(attn_batch_launch(e->q, e->gate, Ly.kc, Ly.vc, e->part, e->xq, pos, e->attn_count, e->H, e->KV, hd,
                                    e->S, 1.0f / sqrtf((float)hd), n, e->st));
        } else {
            ECUDA(attn_launch(e->q, Ly.kc, Ly.vc, e->part, e->o, pos, e->H, e->KV, hd, e->S, 1.0f / sqrtf((float)hd),
                              e->st, n));
            ECALL(m27b_act_quant_gated(e->o, e->gate, e->H * hd, n, e->H * hd, act_type_of(Ly.wo.type), e->xq, e->st,
                                       err, err_cap));
        }
        ECALL(vmv(e, Ly.wo, e->xq, n, e->h2, D, r0 ? e->h : nullptr, err, err_cap));
        if (c.tp_size > 1) ENCCL(ncclAllReduce(e->h2, e->h2, (size_t)n * D, ncclFloat32, ncclSum, e->comm, e->st));
        if (n >= 5 && Ly.wg.type == M27B_TYPE_Q4_K) {
            // 5+ tokens: gate and up on the tensor cores, then silu(gate) * up -> q8 for down
            ECALL(m27b_act_quant_rmsnorm(e->h2, Ly.post_norm, c.rms_eps, D, n, D, M27B_TYPE_Q8_K, e->xq, e->st, err,
                                         err_cap));
            ECALL(vmv(e, Ly.wg, e->xq, n, e->a, e->F, nullptr, err, err_cap));
            ECALL(vmv(e, Ly.wu, e->xq, n, e->a2, e->F, nullptr, err, err_cap));
            ECALL(m27b_act_quant_swiglu(e->a, e->a2, e->F, n, e->F, act_type_of(Ly.wd.type), e->xq, e->st, err,
                                        err_cap));
        } else {
            ECALL(m27b_qmv_f32_rmsnorm(&Ly.wg.v, &Ly.wu.v, e->h2, D, Ly.post_norm, c.rms_eps, n, e->xq, e->a, e->F,
                                       nullptr, e->st, err, err_cap));
            ECALL(m27b_act_quant(e->a, e->F, n, e->F, act_type_of(Ly.wd.type), e->xq, e->st, err, err_cap));
        }
        if (n >= 5 && q6_verify_mma(e, Ly.wd, n, true)) {
            // 5+ tokens of a q6_K down: the tensor cores, K split across CTAs, up to 8 tokens per weight pass
            const size_t xrow = m27b_act_bytes(M27B_TYPE_Q8_K, e->F);
            for (int t0 = 0; t0 < n; t0 += 8) {
                const int nt = std::min(8, n - t0);
                ECALL(qmv_q6k_mma(&Ly.wd.v, e->xq + t0 * xrow, nt, e->h + (size_t)t0 * D, D,
                                  r0 ? e->h2 + (size_t)t0 * D : nullptr, nullptr, 0u, EPI_STORE, e->q6m_part,
                                  e->q6m_count, e->st, err, err_cap));
            }
        } else if (n >= 5 && Ly.wd.v.ggml_type == (M27B_TYPE_Q6_K | M27B_LAYOUT_PLANAR) &&
                   q6k_ksplit_ranges((int)Ly.wd.v.row_blocks) > 0 && Ly.wd.rows == D)
            // 5+ tokens of a q6_K down: K split across CTAs, 8 tokens per weight pass
            ECALL(qmv_q6k_ksplit(&Ly.wd.v, e->xq, n, e->h, D, r0 ? e->h2 : nullptr, e->ksp_part, e->ksp_count, e->st,
                                 err, err_cap));
        else
            ECALL(m27b_qmv(&Ly.wd.v, e->xq, n, e->h, D, r0 ? e->h2 : nullptr, e->st, err, err_cap));
        if (c.tp_size > 1) ENCCL(ncclAllReduce(e->h, e->h, (size_t)n * D, ncclFloat32, ncclSum, e->comm, e->st));
    }
    ECALL(m27b_act_quant_rmsnorm(e->h, e->out_norm, c.rms_eps, D, n, D, act_type_of(e->lmh.type), e->xq, e->st, err,
                                 err_cap));
    if (n >= 5 && q6_verify_mma(e, e->lmh, n, false)) {
        // 5+ tokens: lm_head on the tensor cores, up to 8 tokens per weight pass
        const size_t xrow = m27b_act_bytes(M27B_TYPE_Q8_K, D);
        for (int t0 = 0; t0 < n; t0 += 8)
            ECALL(qmv_q6k_mma(&e->lmh.v, e->xq + t0 * xrow, std::min(8, n - t0), e->logits + (size_t)t0 * e->V, e->V,
                              nullptr, e->best + t0, (uint32_t)e->v_lo, EPI_ARGMAX, nullptr, nullptr, e->st, err,
                              err_cap));
    } else {
        ECALL(m27b_qmv_argmax(&e->lmh.v, e->xq, n, e->logits, e->V, e->best, (uint32_t)e->v_lo, e->st, err, err_cap));
    }
    if (c.tp_size > 1) ENCCL(ncclAllReduce(e->best, e->best, (size_t)n, ncclUint64, ncclMax, e->comm, e->st));
    return true;
}

bool set_ctl(M27BEngine *e, int token, int pos, char *err, size_t err_cap) {
    e->h_ctl[0] = token;
    e->h_ctl[1] = pos;
    e->h_ctl[2] = 0;
    // ctl[3] (the step counter, the fused all-reduce's epoch) is left alone
    ECUDA(cudaMemcpyAsync(e->ctl, e->h_ctl, 12, cudaMemcpyHostToDevice, e->st));
    return true;
}

// Capture the decode step into a graph on first use.  The step runs eagerly
// once before the capture (module loading and first-use set-up then happen
// outside it); the caller sets the control words again afterwards.  Re-running
// a step at one position rewrites the same KV-cache entries.
// Bytes of every DeltaNet layer's conv and delta-rule state.
size_t ssm_state_bytes(const M27BEngine *e, size_t *conv_b, size_t *delta_b) {
    const M27BModelConfig &c = e->c;
    *conv_b = (size_t)e->conv_ch * (c.ssm_conv_kern - 1) * 4;
    *delta_b = (size_t)c.ssm_dt_rank * 128 * 128 * 4;
    return (size_t)e->n_ssm * (*conv_b + *delta_b);
}

// Copy the DeltaNet states into buf (restore = false) or back from it.
bool ssm_state_copy(M27BEngine *e, uint8_t *buf, bool restore, char *err, size_t err_cap) {
    size_t cb, db, off = 0;
    ssm_state_bytes(e, &cb, &db);
    for (Layer &Ly : e->L) {
        if (!Ly.ssm) continue;
        ECUDA(cudaMemcpyAsync(restore ? (void *)Ly.cstate : buf + off, restore ? buf + off : (void *)Ly.cstate, cb,
                              cudaMemcpyDeviceToDevice, e->st));
        off += cb;
        ECUDA(cudaMemcpyAsync(restore ? (void *)Ly.S : buf + off, restore ? buf + off : (void *)Ly.S, db,
                              cudaMemcpyDeviceToDevice, e->st));
        off += db;
    }
    return true;
}

bool ensure_graph(M27BEngine *e, char *err, size_t err_cap) {
    if (e->gexec) return true;
    // the eager run advances the DeltaNet states (attention only rewrites one
    // KV-cache entry): keep a copy and put it back before the capture
    uint8_t *bk = nullptr;
    size_t cb, db;
    if (e->n_ssm) {
        ECUDA(cudaMalloc(&bk, ssm_state_bytes(e, &cb, &db)));
        if (!ssm_state_copy(e, bk, false, err, err_cap)) {
            cudaFree(bk);
            return false;
        }
    }
    const bool eager = enqueue_step(e, err, err_cap);
    const cudaError_t se = cudaStreamSynchronize(e->st);
    if (bk) {
        const bool back = eager && se == cudaSuccess && ssm_state_copy(e, bk, true, err, err_cap) &&
                          cudaStreamSynchronize(e->st) == cudaSuccess;
        cudaFree(bk);
        if (eager && se == cudaSuccess && !back) return efail(err, err_cap, "restoring the DeltaNet states failed");
    }
    if (!eager) return false;
    ECUDA(se);
    ECUDA(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    const bool ok = enqueue_step(e, err, err_cap);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    if (!ok) {
        if (g) cudaGraphDestroy(g);
        return false;
    }
    ECUDA(ce);
    const cudaError_t ie = cudaGraphInstantiate(&e->gexec, g, 0);
    cudaGraphDestroy(g);
    ECUDA(ie);
    return true;
}

bool check_ready(M27BEngine *e, int pos, int n, char *err, size_t err_cap) {
    const M27BModelConfig &c = e->c;
    if (pos < 0 || n < 1 || pos + n > c.max_ctx)
        return efail(err, err_cap, "positions %d..%d outside the cache (max_ctx %d)", pos, pos + n - 1, c.max_ctx);
    if (c.tp_size > 1 && !e->comm) return efail(err, err_cap, "m27b_engine_set_nccl was not called");
    for (const Layer &Ly : e->L) {
        if (!Ly.wg.d || !Ly.wu.d || !Ly.wd.d || !Ly.attn_norm || !Ly.post_norm)
            return efail(err, err_cap, "weights are not loaded");
        if (Ly.ssm ? (!Ly.wqs.d || !Ly.wz.d || !Ly.wba.d || !Ly.wso.d || !Ly.conv_w || !Ly.dt_bias || !Ly.ssm_a ||
                      !Ly.ssm_norm)
                   : (!Ly.wqkv.d || !Ly.wo.d || !Ly.q_norm || !Ly.k_norm))
            return efail(err, err_cap, "weights are not loaded");
    }
    if (!e->embd.d || !e->lmh.d || !e->out_norm) return efail(err, err_cap, "weights are not loaded");
    return true;
}

bool check_status(char *err, size_t err_cap) {
    int status = 0;
    char e2[256];
    if (!m27b_device_status(&status, 1, e2, sizeof(e2))) return efail(err, err_cap, "%s", e2);
    if (status) return efail(err, err_cap, "a kernel's bounded wait ran out (status %d)", status);
    return true;
}

bool parse_layer(const char *name, int *layer, std::string *what) {
    int l = -1;
    char rest[128];
    if (std::sscanf(name, "blk.%d.%127s", &l, rest) != 2) return false;
    *layer = l;
    *what = rest;
    return true;
}

}  // namespace

extern "C" {

bool m27b_nccl_unique_id(void *id, char *err, size_t err_cap) {
    if (!id) return efail(err, err_cap, "m27b_nccl_unique_id: null output");
    static_assert(sizeof(ncclUniqueId) == M27B_NCCL_ID_BYTES, "NCCL unique id size");
    ENCCL(ncclGetUniqueId((ncclUniqueId *)id));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_partition(const M27BModelConfig *cfg, M27BPartition *out, char *err, size_t err_cap) {
    if (!cfg || !out) return efail(err, err_cap, "m27b_engine_partition: null argument");
    const M27BModelConfig &c = *cfg;
    const int t = c.tp_size, r = c.tp_rank;
    if (t < 1 || r < 0 || r >= t) return efail(err, err_cap, "bad tensor-parallel rank %d of %d", r, t);
    if (c.n_layers < 1 || c.hidden < 256 || c.hidden % 256 || c.ffn % 256 || c.head_dim % 32 || c.head_dim > 256 ||
        c.head_dim < 32)
        return efail(err, err_cap, "unsupported shape (hidden and ffn must be multiples of 256, head_dim 32..256)");
    if (c.n_kv_head < 1 || c.n_head % t || c.n_head % c.n_kv_head || c.n_head / c.n_kv_head > 8)
        return efail(err, err_cap, "n_head must divide by tp_size and by n_kv_head (<= 8 q heads per kv head)");
    if (((c.n_head / t) * c.head_dim) % 256) return efail(err, err_cap, "local heads x head_dim must be a multiple of 256");
    if (c.n_rot < 2 || c.n_rot > c.head_dim || c.n_rot % 2) return efail(err, err_cap, "bad n_rot");
    if (c.ffn / 256 < t || c.vocab < t || c.max_ctx < 1) return efail(err, err_cap, "shape too small for tp_size");
    if (c.attn_interval < 0) return efail(err, err_cap, "attn_interval must be >= 0");
    if (c.attn_interval > 0) {
        if (t != 1) return efail(err, err_cap, "hybrid (Gated DeltaNet) models run with tp_size 1");
        if (c.ssm_d_state != 128 || c.ssm_dt_rank < 2 || c.ssm_dt_rank % 2 || c.ssm_d_inner != c.ssm_dt_rank * 128)
            return efail(err, err_cap,
                         "DeltaNet shape: ssm_d_state must be 128, ssm_dt_rank even, ssm_d_inner = ssm_dt_rank x 128");
        if (c.ssm_n_group < 1 || c.ssm_n_group > c.ssm_dt_rank || c.ssm_conv_kern < 2 || c.ssm_conv_kern > 8)
            return efail(err, err_cap, "DeltaNet shape: 1 <= ssm_n_group <= ssm_dt_rank, 2 <= ssm_conv_kern <= 8");
    }
    const int G = c.n_head / c.n_kv_head;
    M27BPartition p;
    p.n_q = c.n_head / t;
    p.q_lo = r * p.n_q;
    p.kv_lo = p.q_lo / G;
    p.n_kv = (p.q_lo + p.n_q - 1) / G - p.kv_lo + 1;
    if (p.n_q % p.n_kv || p.n_q / p.n_kv > 8) return efail(err, err_cap, "unsupported head split");
    // the attention kernel maps local query head h to local kv head h / (n_q / n_kv)
    for (int h = 0; h < p.n_q; ++h)
        if ((p.q_lo + h) / G - p.kv_lo != h / (p.n_q / p.n_kv))
            return efail(err, err_cap, "query heads of rank %d straddle kv heads unevenly", r);
    const int fb = c.ffn / 256;
    p.f_lo = (int)((long)fb * r / t) * 256;
    p.n_f = (int)((long)fb * (r + 1) / t) * 256 - p.f_lo;
    p.v_lo = (int)((long)c.vocab * r / t);
    p.n_v = (int)((long)c.vocab * (r + 1) / t) - p.v_lo;
    *out = p;
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_create(const M27BModelConfig *cfg, M27BEngine **out, char *err, size_t err_cap) {
    if (!cfg || !out) return efail(err, err_cap, "m27b_engine_create: null argument");
    *out = nullptr;
    M27BPartition pt;
    if (!m27b_engine_partition(cfg, &pt, err, err_cap)) return false;
    const M27BModelConfig &c = *cfg;
    M27BEngine *e = new M27BEngine();
    e->c = c;
    e->allocs.reserve(64);
    auto bail = [&](bool) {
        m27b_engine_destroy(e);
        return false;
    };
    if (cudaGetDevice(&e->dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&e->sms, cudaDevAttrMultiProcessorCount, e->dev) != cudaSuccess)
        return bail(efail(err, err_cap, "no CUDA device"));
    e->H = pt.n_q;
    e->q_lo = pt.q_lo;
    e->KV = pt.n_kv;
    e->kv_lo = pt.kv_lo;
    e->G = e->H / e->KV;  // local q heads per local kv head
    e->F = pt.n_f;
    e->f_lo = pt.f_lo;
    e->V = pt.n_v;
    e->v_lo = pt.v_lo;
    e->S = std::max(1, 148 / e->KV);  // attention splits: one wave of (kv head, split) CTAs
    if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess)
        return bail(efail(err, err_cap, "stream creation failed"));
    const int hd = c.head_dim;
    e->L.resize(c.n_layers);
    char e2[512];
    auto A = [&](void **p, size_t n) { return dalloc(e, p, n, e2, sizeof(e2)); };
    int xmax = std::max(std::max(c.hidden, e->F), e->H * hd);
    for (int l = 0; l < c.n_layers; ++l) e->L[l].ssm = !is_attention_layer(c, l);
    e->n_ssm = 0;
    for (const Layer &Ly : e->L) e->n_ssm += Ly.ssm ? 1 : 0;
    e->conv_ch = c.attn_interval > 0 ? c.ssm_d_inner + 2 * c.ssm_n_group * c.ssm_d_state : 0;
    if (e->n_ssm) xmax = std::max(xmax, c.ssm_d_inner);
    const size_t VM = M27B_VERIFY_MAX;  // activation buffers hold a whole verify pass
    bool ok = A((void **)&e->h, VM * c.hidden * 4) && A((void **)&e->h2, VM * c.hidden * 4) &&
              A((void **)&e->qkv, VM * (e->H * 2 + e->KV * 2) * hd * 4) && A((void **)&e->q, VM * e->H * hd * 4) &&
              A((void **)&e->gate, VM * e->H * hd * 4) && A((void **)&e->o, VM * e->H * hd * 4) &&
              A((void **)&e->a, VM * e->F * 4) && A((void **)&e->a2, VM * e->F * 4) &&
              A((void **)&e->part, VM * e->S * e->H * (hd + 4) * 4) &&
              A((void **)&e->logits, VM * e->V * 4) && A((void **)&e->xq, VM * m27b_act_bytes(M27B_TYPE_Q8_K, xmax)) &&
              A((void **)&e->best, VM * 8) && A((void **)&e->ctl, 16) && A((void **)&e->hist, (size_t)c.max_ctx * 4) &&
              A((void **)&e->rope, (size_t)c.n_rot / 2 * sizeof(float2)) && A((void **)&e->vtok, VM * 4) &&
              A((void **)&e->attn_count, VM * e->KV * sizeof(unsigned)) &&
              cudaMemset(e->attn_count, 0, VM * e->KV * sizeof(unsigned)) == cudaSuccess &&
              A((void **)&e->xq2, m27b_act_bytes(M27B_TYPE_Q8_K, e->F) + 16) &&
              A((void **)&e->ffn_cnt, (size_t)(e->F / 256 + 1) * sizeof(unsigned)) &&
              cudaMemset(e->ffn_cnt, 0, (size_t)(e->F / 256 + 1) * sizeof(unsigned)) == cudaSuccess &&
              A((void **)&e->ksp_part, q6k_ksplit_part_floats(c.hidden, 4) * sizeof(float)) &&
              A((void **)&e->ksp_count, (size_t)(c.hidden / 8) * sizeof(unsigned)) &&
              cudaMemset(e->ksp_count, 0, (size_t)(c.hidden / 8) * sizeof(unsigned)) == cudaSuccess &&
              A((void **)&e->mma_part, mma_scratch_floats(e) * sizeof(float)) &&
              A((void **)&e->mma_count, q4k_mma_split_count_words(mma_rows_max(e)) * sizeof(unsigned)) &&
              cudaMemset(e->mma_count, 0, q4k_mma_split_count_words(mma_rows_max(e)) * sizeof(unsigned)) ==
                  cudaSuccess &&
              A((void **)&e->q6m_part, q6k_mma_part_floats(c.hidden) * sizeof(float)) &&
              A((void **)&e->q6m_count, q6k_mma_count_words(c.hidden) * sizeof(unsigned)) &&
              cudaMemset(e->q6m_count, 0, q6k_mma_count_words(c.hidden) * sizeof(unsigned)) == cudaSuccess &&
              A((void **)&e->sk_part, q6k_stream_part_floats(c.hidden, e->F / 256 + 1) * sizeof(float)) &&
              A((void **)&e->sk_count, q6k_stream_count_words(c.hidden) * sizeof(unsigned)) &&
              cudaMemset(e->sk_count, 0, q6k_stream_count_words(c.hidden) * sizeof(unsigned)) == cudaSuccess;
    for (int l = 0; ok && l < c.n_layers; ++l) {
        Layer &Ly = e->L[l];
        if (Ly.ssm) {
            const size_t cs = (size_t)e->conv_ch * (c.ssm_conv_kern - 1) * 4, ss = (size_t)c.ssm_dt_rank * 128 * 128 * 4;
            ok = A((void **)&Ly.cstate, cs) && A((void **)&Ly.S, ss) && cudaMemset(Ly.cstate, 0, cs) == cudaSuccess &&
                 cudaMemset(Ly.S, 0, ss) == cudaSuccess;
            continue;
        }
        const size_t kvb = (size_t)c.max_ctx * e->KV * hd * 4;
        ok = A((void **)&Ly.kc, kvb) && A((void **)&Ly.vc, kvb) && cudaMemset(Ly.kc, 0, kvb) == cudaSuccess &&
             cudaMemset(Ly.vc, 0, kvb) == cudaSuccess;
    }
    if (ok && e->n_ssm)
        ok = A((void **)&e->hn, (size_t)c.hidden * 4) && A((void **)&e->sx, (size_t)e->conv_ch * 4) &&
             A((void **)&e->sxc, (size_t)e->conv_ch * 4) && A((void **)&e->sz, (size_t)c.ssm_d_inner * 4) &&
             A((void **)&e->sba, (size_t)2 * c.ssm_dt_rank * 4) && A((void **)&e->sbg, (size_t)2 * c.ssm_dt_rank * 4);
    ok = ok && cudaMemset(e->ctl, 0, 16) == cudaSuccess;
    if (!ok) return bail(efail(err, err_cap, "%s", e2));
    if (cudaMallocHost((void **)&e->h_ctl, 16) != cudaSuccess || cudaMallocHost((void **)&e->h_best, 8) != cudaSuccess ||
        cudaMallocHost((void **)&e->h_hist, (size_t)c.max_ctx * 4) != cudaSuccess ||
        cudaMallocHost((void **)&e->h_vtok, M27B_VERIFY_MAX * 4) != cudaSuccess ||
        cudaMallocHost((void **)&e->h_vbest, M27B_VERIFY_MAX * 8) != cudaSuccess)
        return bail(efail(err, err_cap, "pinned allocation failed"));
    if (attn_prepare() != cudaSuccess)
        return bail(efail(err, err_cap, "attention shared-memory opt-in failed"));
    *out = e;
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_create_sharing(const M27BEngine *src, int max_ctx, M27BEngine **out, char *err, size_t err_cap) {
    if (!src || !out) return efail(err, err_cap, "m27b_engine_create_sharing: null argument");
    *out = nullptr;
    if (src->c.tp_size != 1) return efail(err, err_cap, "m27b_engine_create_sharing: tp_size must be 1");
    M27BModelConfig c = src->c;
    c.max_ctx = max_ctx;
    M27BEngine *e = nullptr;
    if (!m27b_engine_create(&c, &e, err, err_cap)) return false;
    if (e->dev != src->dev) {
        m27b_engine_destroy(e);
        return efail(err, err_cap, "m27b_engine_create_sharing: the source engine lives on device %d, current is %d",
                     src->dev, e->dev);
    }
    // the weights are borrowed: they are not in e->allocs, so this engine never frees them
    for (size_t l = 0; l < e->L.size(); ++l) {
        Layer &d = e->L[l];
        const Layer &s = src->L[l];
        d.wqkv = s.wqkv, d.wo = s.wo, d.wg = s.wg, d.wu = s.wu, d.wd = s.wd;
        d.attn_norm = s.attn_norm, d.post_norm = s.post_norm, d.q_norm = s.q_norm, d.k_norm = s.k_norm;
        d.wqs = s.wqs, d.wz = s.wz, d.wba = s.wba, d.wso = s.wso;
        d.conv_w = s.conv_w, d.dt_bias = s.dt_bias, d.ssm_a = s.ssm_a, d.ssm_norm = s.ssm_norm;
    }
    e->embd = src->embd;
    e->lmh = src->lmh;
    e->out_norm = src->out_norm;
    *out = e;
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_set_nccl(M27BEngine *e, const void *id, char *err, size_t err_cap) {
    if (!e || !id) return efail(err, err_cap, "m27b_engine_set_nccl: null argument");
    if (e->c.tp_size == 1) return efail(err, err_cap, "tp_size is 1");
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ENCCL(ncclCommInitRank(&e->comm, e->c.tp_size, u, e->c.tp_rank));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_enable_p2p(M27BEngine *e, char *err, size_t err_cap) {
    if (!e) return efail(err, err_cap, "m27b_engine_enable_p2p: null engine");
    const int N = e->c.tp_size, r = e->c.tp_rank;
    if (N < 2) return efail(err, err_cap, "m27b_engine_enable_p2p: tp_size is 1");
    if (N > 8) return efail(err, err_cap, "m27b_engine_enable_p2p: at most 8 ranks");
    if (!e->comm) return efail(err, err_cap, "m27b_engine_enable_p2p: call m27b_engine_set_nccl first");
    if (e->gexec) return efail(err, err_cap, "m27b_engine_enable_p2p: call it before the first decode step");
    if (e->p2p) return efail(err, err_cap, "m27b_engine_enable_p2p: already enabled");
    const WinLayout lay = win_layout(N, e->c.hidden);
    ECUDA(cudaMalloc(&e->win, lay.total));
    ECUDA(cudaMemset(e->win, 0, lay.total));  // epochs start at 1: a zero word is "nothing yet"
    // every rank's IPC handle, gathered over the NCCL communicator
    cudaIpcMemHandle_t mine;
    ECUDA(cudaIpcGetMemHandle(&mine, e->win));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t *dh = nullptr;
    ECUDA(cudaMalloc(&dh, (size_t)N * 64));
    std::vector<uint8_t> all((size_t)N * 64);
    bool ok = cudaMemcpyAsync(dh + (size_t)r * 64, &mine, 64, cudaMemcpyHostToDevice, e->st) == cudaSuccess &&
              ncclAllGather(dh + (size_t)r * 64, dh, 64, ncclUint8, e->comm, e->st) == ncclSuccess &&
              cudaMemcpyAsync(all.data(), dh, all.size(), cudaMemcpyDeviceToHost, e->st) == cudaSuccess &&
              cudaStreamSynchronize(e->st) == cudaSuccess;
    cudaFree(dh);
    if (!ok) return efail(err, err_cap, "m27b_engine_enable_p2p: exchanging IPC handles failed");
    for (int q = 0; q < N; ++q) {
        if (q == r) {
            e->peer_win[q] = e->win;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + (size_t)q * 64, 64);
        void *p = nullptr;
        const cudaError_t ie = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (ie != cudaSuccess)
            return efail(err, err_cap, "m27b_engine_enable_p2p: mapping rank %d's window: %s", q, cudaGetErrorString(ie));
        e->peer_win[q] = (uint8_t *)p;
    }
    // every rank has mapped every window before any rank stores into one
    int *one = nullptr;
    ECUDA(cudaMalloc(&one, sizeof(int)));
    ok = cudaMemsetAsync(one, 0, sizeof(int), e->st) == cudaSuccess &&
         ncclAllReduce(one, one, 1, ncclInt32, ncclSum, e->comm, e->st) == ncclSuccess &&
         cudaStreamSynchronize(e->st) == cudaSuccess;
    cudaFree(one);
    if (!ok) return efail(err, err_cap, "m27b_engine_enable_p2p: barrier failed");
    e->p2p = true;
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_load_tensor(M27BEngine *e, const char *name, uint32_t type, uint32_t row_elems, uint32_t row_count,
                             const void *host, char *err, size_t err_cap) {
    if (!e || !name || !host) return efail(err, err_cap, "m27b_engine_load_tensor: null argument");
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim;
    const uint8_t *hb = (const uint8_t *)host;
    auto is_f32 = [&](size_t n) { return type == M27B_TYPE_F32 && row_elems * (size_t)row_count == n; };
    const std::string nm = name;
    if (nm == "token_embd.weight") {
        if (row_count != (uint32_t)c.vocab || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "token_embd shape");
        if (type != M27B_TYPE_Q4_K && type != M27B_TYPE_Q6_K && type != M27B_TYPE_Q8_0)
            return efail(err, err_cap, "token_embd must be q4_K, q6_K or q8_0 (got type %u)", type);
        ECALL(ensure_mat(e, e->embd, type, c.vocab, c.hidden, err, err_cap));
        return load_slice(e, e->embd, hb, e->embd.v.row_blocks, 0, c.vocab, 0, 0, err, err_cap);
    }
    if (nm == "output_norm.weight") {
        if (!is_f32(c.hidden)) return efail(err, err_cap, "output_norm must be f32[%d]", c.hidden);
        return load_f32(e, &e->out_norm, host, c.hidden, err, err_cap);
    }
    if (nm == "output.weight") {
        if (row_count != (uint32_t)c.vocab || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "output shape");
        ECALL(ensure_mat(e, e->lmh, type, e->V, c.hidden, err, err_cap));
        return load_slice(e, e->lmh, hb, e->lmh.v.row_blocks, e->v_lo, e->V, 0, 0, err, err_cap);
    }
    int l = -1;
    std::string what;
    if (!parse_layer(name, &l, &what) || l < 0 || l >= c.n_layers) return efail(err, err_cap, "unknown tensor %s", name);
    Layer &Ly = e->L[l];
    const uint32_t be = (uint32_t)block_elems(type);
    if (what == "attn_norm.weight" || what == "post_attention_norm.weight") {
        if (!is_f32(c.hidden)) return efail(err, err_cap, "%s must be f32[%d]", name, c.hidden);
        return load_f32(e, what[0] == 'a' ? &Ly.attn_norm : &Ly.post_norm, host, c.hidden, err, err_cap);
    }
    if (Ly.ssm && what.compare(0, 4, "ffn_") != 0) {
        // Gated DeltaNet tensors, under the reference loader's names (:1775-1825)
        const int dr = c.ssm_dt_rank, K = c.ssm_conv_kern;
        auto mat = [&](QMat &m, int rows, int k, int row_at) -> bool {
            ECALL(ensure_mat(e, m, type, rows, k, err, err_cap));
            return load_slice(e, m, hb, row_elems / be, 0, (int)row_count, 0, row_at, err, err_cap);
        };
        if (what == "attn_qkv.weight" || what == "attn_q.weight" || what == "ssm_in.weight") {
            if (row_count != (uint32_t)e->conv_ch || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "%s shape", name);
            return mat(Ly.wqs, e->conv_ch, c.hidden, 0);
        }
        if (what == "attn_gate.weight" || what == "attn_k.weight" || what == "ssm_in_gate.weight") {
            if (row_count != (uint32_t)c.ssm_d_inner || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "%s shape", name);
            return mat(Ly.wz, c.ssm_d_inner, c.hidden, 0);
        }
        if (what == "ssm_beta.weight" || what == "ssm_alpha.weight") {
            if (row_count != (uint32_t)dr || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "%s shape", name);
            ECALL(ensure_mat(e, Ly.wba, type, 2 * dr, c.hidden, err, err_cap));  // rows: beta | alpha
            return load_slice(e, Ly.wba, hb, row_elems / be, 0, dr, 0, what[4] == 'b' ? 0 : dr, err, err_cap);
        }
        if (what == "ssm_out.weight") {
            if (row_count != (uint32_t)c.hidden || row_elems != (uint32_t)c.ssm_d_inner) return efail(err, err_cap, "%s shape", name);
            if (act_type_of(type) != M27B_TYPE_Q8_K || type == M27B_TYPE_F16 || type == M27B_TYPE_F32)
                return efail(err, err_cap, "%s must be a 256-value k-quant (q4_K, q5_K, q6_K, IQ4_XS)", name);
            return mat(Ly.wso, c.hidden, c.ssm_d_inner, 0);
        }
        if (what == "ssm_conv1d.weight") {
            if (row_elems != (uint32_t)K || row_count != (uint32_t)e->conv_ch ||
                (type != M27B_TYPE_F32 && type != M27B_TYPE_F16))
                return efail(err, err_cap, "%s must be f32 / f16 [%d x %d]", name, e->conv_ch, K);
            std::vector<float> w((size_t)K * e->conv_ch);
            for (size_t i = 0; i < w.size(); ++i)
                w[i] = type == M27B_TYPE_F32 ? ((const float *)host)[i] : half_bits_to_float(((const uint16_t *)host)[i]);
            return load_f32(e, &Ly.conv_w, w.data(), w.size(), err, err_cap);
        }
        if (what == "ssm_dt.bias" || what == "ssm_dt_bias" || what == "ssm_a" || what == "ssm_a_log") {
            if (!is_f32(dr)) return efail(err, err_cap, "%s must be f32[%d]", name, dr);
            return load_f32(e, what.compare(0, 6, "ssm_dt") == 0 ? &Ly.dt_bias : &Ly.ssm_a, host, dr, err, err_cap);
        }
        if (what == "ssm_norm.weight") {
            if (!is_f32(128)) return efail(err, err_cap, "%s must be f32[128]", name);
            return load_f32(e, &Ly.ssm_norm, host, 128, err, err_cap);
        }
        return efail(err, err_cap, "unknown tensor %s for a DeltaNet layer", name);
    }
    if (what == "attn_q_norm.weight" || what == "attn_k_norm.weight") {
        if (!is_f32(hd)) return efail(err, err_cap, "%s must be f32[%d]", name, hd);
        return load_f32(e, what[5] == 'q' ? &Ly.q_norm : &Ly.k_norm, host, hd, err, err_cap);
    }
    const int qkv_rows = e->H * 2 * hd + 2 * e->KV * hd;
    if (what == "attn_q.weight") {
        if (row_count != (uint32_t)(c.n_head * 2 * hd) || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "attn_q shape");
        ECALL(ensure_mat(e, Ly.wqkv, type, qkv_rows, c.hidden, err, err_cap));
        return load_slice(e, Ly.wqkv, hb, row_elems / be, e->q_lo * 2 * hd, e->H * 2 * hd, 0, 0, err, err_cap);
    }
    if (what == "attn_k.weight" || what == "attn_v.weight") {
        if (row_count != (uint32_t)(c.n_kv_head * hd) || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "attn_k/v shape");
        ECALL(ensure_mat(e, Ly.wqkv, type, qkv_rows, c.hidden, err, err_cap));
        const int at = e->H * 2 * hd + (what[5] == 'k' ? 0 : e->KV * hd);
        return load_slice(e, Ly.wqkv, hb, row_elems / be, e->kv_lo * hd, e->KV * hd, 0, at, err, err_cap);
    }
    if (what == "attn_output.weight") {
        if (row_count != (uint32_t)c.hidden || row_elems != (uint32_t)(c.n_head * hd)) return efail(err, err_cap, "attn_output shape");
        ECALL(ensure_mat(e, Ly.wo, type, c.hidden, e->H * hd, err, err_cap));
        return load_slice(e, Ly.wo, hb, row_elems / be, 0, c.hidden, e->q_lo * hd / (int)be, 0, err, err_cap);
    }
    if (what == "ffn_gate.weight" || what == "ffn_up.weight") {
        if (row_count != (uint32_t)c.ffn || row_elems != (uint32_t)c.hidden) return efail(err, err_cap, "ffn gate/up shape");
        QMat &m = what[4] == 'g' ? Ly.wg : Ly.wu;
        ECALL(ensure_mat(e, m, type, e->F, c.hidden, err, err_cap));
        return load_slice(e, m, hb, row_elems / be, e->f_lo, e->F, 0, 0, err, err_cap);
    }
    if (what == "ffn_down.weight") {
        if (row_count != (uint32_t)c.hidden || row_elems != (uint32_t)c.ffn) return efail(err, err_cap, "ffn_down shape");
        ECALL(ensure_mat(e, Ly.wd, type, c.hidden, e->F, err, err_cap));
        return load_slice(e, Ly.wd, hb, row_elems / be, 0, c.hidden, e->f_lo / (int)be, 0, err, err_cap);
    }
    return efail(err, err_cap, "unknown tensor %s", name);
}

bool m27b_engine_load_blob(M27BEngine *e, const M27BBlob *blob, uint32_t source, char *err, size_t err_cap) {
    if (!e || !blob) return efail(err, err_cap, "m27b_engine_load_blob: null argument");
    const size_t n = m27b_blob_count(blob);
    size_t loaded = 0;
    for (size_t i = 0; i < n; ++i) {
        M27BWeightEntry en;
        const void *data = nullptr;
        if (!m27b_blob_entry(blob, i, &en, &data, err, err_cap)) return false;
        if (en.source_model != source) continue;
        // the payload of an entry must hold the tensor its shape describes
        const uint32_t base = en.ggml_type;
        const uint64_t need = base == M27B_TYPE_F32 ? (uint64_t)en.row_elems * en.row_count * 4
                                                    : (uint64_t)en.row_count * (en.row_elems / block_elems(base)) *
                                                          block_bytes(base);
        if (need == 0 || en.data_bytes < need)
            return efail(err, err_cap, "m27b_engine_load_blob: entry %s: %llu bytes for a %ux%u type-%u tensor",
                         en.name, (unsigned long long)en.data_bytes, en.row_count, en.row_elems, en.ggml_type);
        ECALL(m27b_engine_load_tensor(e, en.name, en.ggml_type, en.row_elems, en.row_count, data, err, err_cap));
        ++loaded;
    }
    if (loaded == 0) return efail(err, err_cap, "m27b_engine_load_blob: no entry of source %u", source);
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_random_weights(M27BEngine *e, uint64_t seed, float sigma, char *err, size_t err_cap) {
    if (!e) return efail(err, err_cap, "null engine");
    const M27BModelConfig &c = e->c;
    const int hd = c.head_dim;
    if (c.weight_type != 0 && c.weight_type != M27B_TYPE_Q8_0)
        return efail(err, err_cap, "weight_type must be 0 (q4_k_m mix) or 8 (q8_0)");
    const bool q80 = c.weight_type == M27B_TYPE_Q8_0;
    const uint32_t Q4 = q80 ? M27B_TYPE_Q8_0 : M27B_TYPE_Q4_K, Q6 = q80 ? M27B_TYPE_Q8_0 : M27B_TYPE_Q6_K;
    auto ones = [&](float **p, size_t n) -> bool {
        if (!*p) ECALL(dalloc(e, (void **)p, n * 4, err, err_cap));
        k_fill_f32<<<64, 256, 0, e->st>>>(*p, (long)n, 1.0f);
        ECUDA(cudaGetLastError());
        return true;
    };
    ECALL(ensure_mat(e, e->embd, Q4, c.vocab, c.hidden, err, err_cap));
    // the embedding in slices (the staging buffer stays small)
    for (int r = 0; r < c.vocab; r += 16384) {
        const int n = std::min(16384, c.vocab - r);
        ECALL(fill_slice(e, e->embd, 1 << 20, seed, sigma, r, n, 0, r, err, err_cap));
    }
    ECALL(ensure_mat(e, e->lmh, Q6, e->V, c.hidden, err, err_cap));
    for (int r = 0; r < e->V; r += 16384) {
        const int n = std::min(16384, e->V - r);
        ECALL(fill_slice(e, e->lmh, (1 << 20) + 1, seed, sigma, e->v_lo + r, n, 0, r, err, err_cap));
    }
    ECALL(ones(&e->out_norm, c.hidden));
    const int qkv_rows = e->H * 2 * hd + 2 * e->KV * hd;
    for (int l = 0; l < c.n_layers; ++l) {
        Layer &Ly = e->L[l];
        const int tid = 16 * l;
        if (Ly.ssm) {
            // DeltaNet: projections in the matrix mix (beta / alpha as one q4_K matrix), random conv
            // taps, dt_bias 0, ssm_a -1 (decay e^-softplus(a)), unit norms
            const int dr = c.ssm_dt_rank;
            ECALL(ensure_mat(e, Ly.wqs, Q4, e->conv_ch, c.hidden, err, err_cap));
            ECALL(fill_slice(e, Ly.wqs, tid + 8, seed, sigma, 0, e->conv_ch, 0, 0, err, err_cap));
            ECALL(ensure_mat(e, Ly.wz, Q4, c.ssm_d_inner, c.hidden, err, err_cap));
            ECALL(fill_slice(e, Ly.wz, tid + 9, seed, sigma, 0, c.ssm_d_inner, 0, 0, err, err_cap));
            ECALL(ensure_mat(e, Ly.wba, Q4, 2 * dr, c.hidden, err, err_cap));
            ECALL(fill_slice(e, Ly.wba, tid + 10, seed, sigma, 0, 2 * dr, 0, 0, err, err_cap));
            ECALL(ensure_mat(e, Ly.wso, Q4, c.hidden, c.ssm_d_inner, err, err_cap));
            ECALL(fill_slice(e, Ly.wso, tid + 11, seed, sigma, 0, c.hidden, 0, 0, err, err_cap));
            const size_t ncw = (size_t)e->conv_ch * c.ssm_conv_kern;
            if (!Ly.conv_w) ECALL(dalloc(e, (void **)&Ly.conv_w, ncw * 4, err, err_cap));
            k_fill_f32_rand<<<64, 256, 0, e->st>>>(Ly.conv_w, (long)ncw, seed * 131 + (uint64_t)tid, 0.5f, 0.0f);
            ECUDA(cudaGetLastError());
            auto fill = [&](float **p, size_t n, float v) -> bool {
                if (!*p) ECALL(dalloc(e, (void **)p, n * 4, err, err_cap));
                k_fill_f32<<<64, 256, 0, e->st>>>(*p, (long)n, v);
                ECUDA(cudaGetLastError());
                return true;
            };
            ECALL(fill(&Ly.dt_bias, dr, 0.0f));
            ECALL(fill(&Ly.ssm_a, dr, -1.0f));
            ECALL(fill(&Ly.ssm_norm, 128, 1.0f));
        } else {
            ECALL(ensure_mat(e, Ly.wqkv, Q4, qkv_rows, c.hidden, err, err_cap));
            ECALL(fill_slice(e, Ly.wqkv, tid + 1, seed, sigma, (long)e->q_lo * 2 * hd, e->H * 2 * hd, 0, 0, err,
                             err_cap));
            ECALL(fill_slice(e, Ly.wqkv, tid + 2, seed, sigma, (long)e->kv_lo * hd, e->KV * hd, 0, e->H * 2 * hd, err,
                             err_cap));
            ECALL(fill_slice(e, Ly.wqkv, tid + 3, seed, sigma, (long)e->kv_lo * hd, e->KV * hd, 0,
                             e->H * 2 * hd + e->KV * hd, err, err_cap));
            ECALL(ensure_mat(e, Ly.wo, Q4, c.hidden, e->H * hd, err, err_cap));
            ECALL(fill_slice(e, Ly.wo, tid + 4, seed, sigma, 0, c.hidden, e->q_lo * hd / block_elems(Q4), 0, err,
                             err_cap));
            ECALL(ones(&Ly.q_norm, hd));
            ECALL(ones(&Ly.k_norm, hd));
        }
        ECALL(ensure_mat(e, Ly.wg, Q4, e->F, c.hidden, err, err_cap));
        ECALL(fill_slice(e, Ly.wg, tid + 5, seed, sigma, e->f_lo, e->F, 0, 0, err, err_cap));
        ECALL(ensure_mat(e, Ly.wu, Q4, e->F, c.hidden, err, err_cap));
        ECALL(fill_slice(e, Ly.wu, tid + 6, seed, sigma, e->f_lo, e->F, 0, 0, err, err_cap));
        ECALL(ensure_mat(e, Ly.wd, Q6, c.hidden, e->F, err, err_cap));
        ECALL(fill_slice(e, Ly.wd, tid + 7, seed, sigma, 0, c.hidden, e->f_lo / block_elems(Q6), 0, err, err_cap));
        ECALL(ones(&Ly.attn_norm, c.hidden));
        ECALL(ones(&Ly.post_norm, c.hidden));
    }
    ECUDA(cudaStreamSynchronize(e->st));
    if (err && err_cap) err[0] = '\0';
    return true;
}

size_t m27b_engine_weight_bytes_per_token(const M27BEngine *e) {
    if (!e) return 0;
    size_t n = e->lmh.gguf_bytes + (e->embd.rows ? e->embd.gguf_bytes / e->embd.rows : 0);
    for (const Layer &Ly : e->L)
        n += Ly.wqkv.gguf_bytes + Ly.wo.gguf_bytes + Ly.wg.gguf_bytes + Ly.wu.gguf_bytes + Ly.wd.gguf_bytes +
             Ly.wqs.gguf_bytes + Ly.wz.gguf_bytes + Ly.wba.gguf_bytes + Ly.wso.gguf_bytes;
    return n;
}

bool m27b_engine_reset(M27BEngine *e, char *err, size_t err_cap) {
    if (!e) return efail(err, err_cap, "null engine");
    // attention: positions index the cache, a new sequence simply starts at pos 0;
    // DeltaNet: the recurrent states start from zero
    size_t cb, db;
    ssm_state_bytes(e, &cb, &db);
    for (Layer &Ly : e->L) {
        if (!Ly.ssm) continue;
        ECUDA(cudaMemsetAsync(Ly.cstate, 0, cb, e->st));
        ECUDA(cudaMemsetAsync(Ly.S, 0, db, e->st));
    }
    ECUDA(cudaStreamSynchronize(e->st));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_decode_step(M27BEngine *e, int token, int pos, int *next, float *logits, char *err, size_t err_cap) {
    if (!e || !next) return efail(err, err_cap, "m27b_engine_decode_step: null argument");
    if (logits && e->c.tp_size != 1) return efail(err, err_cap, "logits are only returned with tp_size 1");
    if (token < 0 || token >= e->c.vocab) return efail(err, err_cap, "token %d outside the vocabulary", token);
    ECALL(check_ready(e, pos, 1, err, err_cap));
    ECALL(set_ctl(e, token, pos, err, err_cap));
    if (!e->gexec) {
        ECALL(ensure_graph(e, err, err_cap));
        ECALL(set_ctl(e, token, pos, err, err_cap));
    }
    ECUDA(cudaGraphLaunch(e->gexec, e->st));
    ECUDA(cudaMemcpyAsync(e->h_best, e->best, 8, cudaMemcpyDeviceToHost, e->st));
    if (logits) ECUDA(cudaMemcpyAsync(logits, e->logits, (size_t)e->V * 4, cudaMemcpyDeviceToHost, e->st));
    ECUDA(cudaStreamSynchronize(e->st));
    *next = (int)m27b_argmax_key_index(*e->h_best);
    ECALL(check_status(err, err_cap));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_generate(M27BEngine *e, int token, int pos, int n, int *tokens, char *err, size_t err_cap) {
    if (!e || !tokens) return efail(err, err_cap, "m27b_engine_generate: null argument");
    if (token < 0 || token >= e->c.vocab) return efail(err, err_cap, "token %d outside the vocabulary", token);
    ECALL(check_ready(e, pos, n, err, err_cap));
    ECALL(set_ctl(e, token, pos, err, err_cap));
    if (!e->gexec) {
        ECALL(ensure_graph(e, err, err_cap));
        ECALL(set_ctl(e, token, pos, err, err_cap));
    }
    for (int i = 0; i < n; ++i) ECUDA(cudaGraphLaunch(e->gexec, e->st));
    ECUDA(cudaMemcpyAsync(e->h_hist, e->hist, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st));
    ECUDA(cudaStreamSynchronize(e->st));
    std::memcpy(tokens, e->h_hist, (size_t)n * 4);
    ECALL(check_status(err, err_cap));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_verify(M27BEngine *e, const int *tokens, int n, int pos, int *next, float *logits, char *err,
                        size_t err_cap) {
    if (!e || !tokens || !next) return efail(err, err_cap, "m27b_engine_verify: null argument");
    if (n < 1 || n > M27B_VERIFY_MAX) return efail(err, err_cap, "m27b_engine_verify: n must be in [1, %d]", M27B_VERIFY_MAX);
    if (e->n_ssm)
        return efail(err, err_cap,
                     "m27b_engine_verify: not for hybrid models (the DeltaNet state cannot be rolled back after a "
                     "rejected draft)");
    if (logits && e->c.tp_size != 1) return efail(err, err_cap, "logits are only returned with tp_size 1");
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= e->c.vocab)
            return efail(err, err_cap, "token %d outside the vocabulary", tokens[i]);
    ECALL(check_ready(e, pos, n, err, err_cap));
    std::memcpy(e->h_vtok, tokens, (size_t)n * 4);
    ECUDA(cudaMemcpyAsync(e->vtok, e->h_vtok, (size_t)n * 4, cudaMemcpyHostToDevice, e->st));
    ECALL(set_ctl(e, tokens[0], pos, err, err_cap));
    if (!e->vgraph[n]) {
        // eager once (module loading, first-use set-up), then capture; the
        // replay rewrites the same KV-cache entries
        ECALL(enqueue_verify(e, n, err, err_cap));
        ECUDA(cudaStreamSynchronize(e->st));
        ECUDA(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
        const bool ok = enqueue_verify(e, n, err, err_cap);
        cudaGraph_t g = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
        if (!ok) {
            if (g) cudaGraphDestroy(g);
            return false;
        }
        ECUDA(ce);
        const cudaError_t ie = cudaGraphInstantiate(&e->vgraph[n], g, 0);
        cudaGraphDestroy(g);
        ECUDA(ie);
    }
    ECUDA(cudaGraphLaunch(e->vgraph[n], e->st));
    ECUDA(cudaMemcpyAsync(e->h_vbest, e->best, (size_t)n * 8, cudaMemcpyDeviceToHost, e->st));
    if (logits) ECUDA(cudaMemcpyAsync(logits, e->logits, (size_t)n * e->V * 4, cudaMemcpyDeviceToHost, e->st));
    ECUDA(cudaStreamSynchronize(e->st));
    for (int i = 0; i < n; ++i) next[i] = (int)m27b_argmax_key_index(e->h_vbest[i]);
    ECALL(check_status(err, err_cap));
    if (err && err_cap) err[0] = '\0';
    return true;
}

bool m27b_engine_hidden(M27BEngine *e, float *host, char *err, size_t err_cap) {
    if (!e || !host) return efail(err, err_cap, "null argument");
    ECUDA(cudaMemcpyAsync(host, e->h, (size_t)e->c.hidden * 4, cudaMemcpyDeviceToHost, e->st));
    ECUDA(cudaStreamSynchronize(e->st));
    if (err && err_cap) err[0] = '\0';
    return true;
}

void *m27b_engine_stream(M27BEngine *e) { return e ? (void *)e->st : nullptr; }

void m27b_engine_destroy(M27BEngine *e) {
    if (!e) return;
    if (e->st) cudaStreamSynchronize(e->st);
    // graphs before the communicator they hold
    if (e->gexec) cudaGraphExecDestroy(e->gexec);
    for (cudaGraphExec_t g : e->vgraph)
        if (g) cudaGraphExecDestroy(g);
    for (int q = 0; q < 8; ++q)
        if (e->peer_win[q] && e->peer_win[q] != e->win) cudaIpcCloseMemHandle(e->peer_win[q]);
    if (e->win) cudaFree(e->win);
    if (e->comm) ncclCommDestroy(e->comm);
    for (void *p : e->allocs) cudaFree(p);
    if (e->scratch) cudaFree(e->scratch);
    if (e->h_vtok) cudaFreeHost(e->h_vtok);
    if (e->h_vbest) cudaFreeHost(e->h_vbest);
    if (e->h_ctl) cudaFreeHost(e->h_ctl);
    if (e->h_hist) cudaFreeHost(e->h_hist);
    if (e->h_best) cudaFreeHost(e->h_best);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

}  // extern "C"

namespace m27b {
size_t stored_row_bytes(const QMat &m) {
    if (!m.d || m.rows <= 0) return 0;
    const uint32_t rb = m.v.row_blocks;
    return raw_layout(m.type) ? (size_t)rb * block_bytes(m.type) : m27b_repacked_bytes(m.type, rb, 1);
}
}  // namespace m27b
