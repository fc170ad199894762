// capi.cu — extern "C" entry points of libm27b (declared in include/m27b_qmv.h).
//
// Error convention kept from the reference executor (include/mono27b_config.h:
// 155-184, e.g. src/mono27b_executor.cu:1711): bool return, message written
// with snprintf into the caller's buffer, err[0] == '\0' on success.
#include <cstdarg>
#include <cstdio>

#include "m27b_device.cuh"
#include "m27b_qmv.h"
#include "m27b_allreduce.h"
#include "qmv_kernels.cuh"

#include "m27b_launch.cuh"

using namespace m27b;

// Library status word, one per device: kernels set it non-zero when one of
// their bounded waits runs out (1: a stage never filled, 2: draining after
// such a failure, 3: a rank's all-reduce partial never arrived, 4: a rank's
// argmax key never arrived).  Read and cleared with m27b_device_status().
__device__ int g_m27b_status;

namespace m27b {
int *status_ptr_current() {
    static int *cache[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
    if (dev < 64 && cache[dev]) return cache[dev];
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_m27b_status) != cudaSuccess) return nullptr;
    if (dev < 64) cache[dev] = (int *)p;
    return (int *)p;
}
}  // namespace m27b

namespace {

bool fail(char *err, size_t cap, const char *fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(err, cap, fmt, ap);
        va_end(ap);
    }
    return false;
}

bool ok(char *err, size_t cap) {
    if (err && cap) err[0] = '\0';
    return true;
}

bool cuda_ok(cudaError_t e, const char *what, char *err, size_t cap) {
    if (e == cudaSuccess) return ok(err, cap);
    return fail(err, cap, "%s: %s", what, cudaGetErrorString(e));
}

int sm_count_current() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
    if (dev < 64 && cache[dev]) return cache[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (dev < 64) cache[dev] = n;
    return n;
}

// Values per block; 1 for f16 / f32, whose WeightView.row_blocks counts
// values (the reference loader's convention, src/mono27b_executor.cu:1704).
int block_elems(uint32_t base_type) {
    switch (base_type) {
    case M27B_TYPE_Q4_K:
    case M27B_TYPE_Q5_K:
    case M27B_TYPE_Q6_K:
    case M27B_TYPE_IQ4_XS:
    case M27B_TYPE_Q8_K: return 256;
    case M27B_TYPE_Q8_0: return 32;
    case M27B_TYPE_F16:
    case M27B_TYPE_F32: return 1;
    default: return 0;
    }
}

// Validated description of a weight view for the matvec kernels.
struct WDesc {
    int kind;       // W_Q4K / W_Q6KP / W_Q80P / W_Q5K / W_IQ4XS / W_F16 / W_F32
    int base;       // base ggml type
    int k;
    int passes;
    size_t row_stride;
};

bool is_float_kind(int kind) { return kind == W_F16 || kind == W_F32; }

bool describe(const WeightView *w, WDesc &d, const char *what, char *err, size_t cap) {
    if (!w) return fail(err, cap, "%s: null WeightView", what);
    if (!w->ptr) return fail(err, cap, "%s: null weight pointer", what);
    if (((uintptr_t)w->ptr & 15u) != 0) return fail(err, cap, "%s: weight pointer must be 16-byte aligned", what);
    if (w->row_blocks == 0 || w->row_count == 0) return fail(err, cap, "%s: empty weight (row_blocks=%u row_count=%u)", what,
                                                             w->row_blocks, w->row_count);
    if (w->row_count > 0x7fffffffu || w->row_blocks > 0x7fffffffu / 256u)
        return fail(err, cap, "%s: weight too large", what);
    const uint32_t base = w->ggml_type & M27B_TYPE_MASK;
    const bool planar = (w->ggml_type & M27B_LAYOUT_PLANAR) != 0;
    if ((w->ggml_type & ~(M27B_TYPE_MASK | M27B_LAYOUT_PLANAR)) != 0)
        return fail(err, cap, "%s: unknown layout flags in ggml_type 0x%x", what, w->ggml_type);
    d.base = (int)base;
    if (base == M27B_TYPE_Q4_K && !planar) {
        d.kind = W_Q4K;
        d.row_stride = (size_t)w->row_blocks * 144;
        d.passes = (int)((w->row_blocks + 3) / 4);
    } else if (base == M27B_TYPE_Q6_K && planar) {
        d.kind = W_Q6KP;
        d.row_stride = planar_row_bytes(M27B_TYPE_Q6_K, (int)w->row_blocks);
        d.passes = (int)((w->row_blocks + 3) / 4);
    } else if (base == M27B_TYPE_Q8_0 && planar) {
        d.kind = W_Q80P;
        d.row_stride = planar_row_bytes(M27B_TYPE_Q8_0, (int)w->row_blocks);
        d.passes = (int)((w->row_blocks + 31) / 32);
    } else if (base == M27B_TYPE_Q5_K && !planar) {
        d.kind = W_Q5K;
        d.row_stride = (size_t)w->row_blocks * 176;
        d.passes = (int)((w->row_blocks + 3) / 4);
    } else if (base == M27B_TYPE_IQ4_XS && !planar) {
        // 136-byte blocks: rows are 16-byte aligned (tensor-map rows) when the block count is even
        if (w->row_blocks & 1u)
            return fail(err, cap, "%s: IQ4_XS rows need an even number of blocks (got %u)", what, w->row_blocks);
        d.kind = W_IQ4XS;
        d.row_stride = (size_t)w->row_blocks * 136;
        d.passes = (int)((w->row_blocks + 3) / 4);
    } else if ((base == M27B_TYPE_F16 || base == M27B_TYPE_F32) && !planar) {
        const uint32_t per16 = base == M27B_TYPE_F16 ? 8u : 4u;
        if (w->row_blocks % per16)
            return fail(err, cap, "%s: %s rows need a multiple of %u values (got %u)", what,
                        base == M27B_TYPE_F16 ? "f16" : "f32", per16, w->row_blocks);
        d.kind = base == M27B_TYPE_F16 ? W_F16 : W_F32;
        d.row_stride = (size_t)w->row_blocks * (base == M27B_TYPE_F16 ? 2 : 4);
        d.passes = 0;
    } else if ((base == M27B_TYPE_Q6_K || base == M27B_TYPE_Q8_0) && !planar) {
        return fail(err, cap, "%s: ggml type %u must be repacked with m27b_repack before the matvec", what, base);
    } else {
        return fail(err, cap,
                    "%s: unsupported weight type 0x%x (q4_K, q5_K, IQ4_XS, f16, f32, planar q6_K and planar q8_0 are "
                    "supported)",
                    what, w->ggml_type);
    }
    d.k = (int)w->row_blocks * block_elems(base);
    return true;
}

size_t act_bytes(uint32_t act_type, int k) {
    if (k <= 0) return 0;
    if (act_type == M27B_TYPE_Q8_K) return (k % 256) ? 0 : (size_t)(k / 256) * sizeof(m27b_block_q8_K);
    if (act_type == M27B_TYPE_Q8_0) return (k % 32) ? 0 : (size_t)(k / 32) * sizeof(m27b_block_q8_0);
    return 0;
}

bool act_quant_common(int mode, const float *x, const float *gate, const float *w, float eps, int k, int n_tok, int ldx,
                      uint32_t act_type, void *xq, cudaStream_t stream, char *err, size_t cap, const char *what) {
    if (!x || !xq) return fail(err, cap, "%s: null pointer", what);
    if ((mode == ACT_GATED || mode == ACT_SWIGLU) && !gate) return fail(err, cap, "%s: null gate", what);
    if (n_tok < 1) return fail(err, cap, "%s: n_tok must be >= 1 (got %d)", what, n_tok);
    if (ldx < k) return fail(err, cap, "%s: ldx (%d) < k (%d)", what, ldx, k);
    if (act_bytes(act_type, k) == 0) return fail(err, cap, "%s: k=%d is not a multiple of the block size of type %u", what, k, act_type);
    if (((uintptr_t)xq & 3u) != 0) return fail(err, cap, "%s: output must be 4-byte aligned", what);
    if (n_tok > 65535) return fail(err, cap, "%s: n_tok too large", what);
    ActArgs a{x, gate, w, eps, k, ldx, xq};
    return cuda_ok(launch_act_quant((int)act_type, mode, a, n_tok, stream), what, err, cap);
}

// fp32 activations for the quantizing prologue of the q4_K kernel
struct XArgs {
    const float *xf;
    int ldxf;
    int norm_on;
    const float *norm_w;
    float eps;
};

// The SwiGLU rows also written as q8_K blocks (one token; the next matvec's input).
struct Q8Out {
    void *q8;
    unsigned *cnt;  // one zeroed word per 256-row block
};

bool qmv_common(int epi, const WeightView *w0, const WeightView *w1, const void *xq, int n_tok, float *y, int ldy,
                const float *residual, unsigned long long *best, uint32_t row_offset, cudaStream_t stream, char *err,
                size_t cap, const char *what, const PushArgs *push = nullptr, const XArgs *xa = nullptr,
                const Q8Out *qo = nullptr) {
    WDesc d0{}, d1{};
    if (!describe(w0, d0, what, err, cap)) return false;
    if (epi == EPI_SWIGLU) {
        if (!describe(w1, d1, what, err, cap)) return false;
        if (w1->ggml_type != w0->ggml_type || w1->row_blocks != w0->row_blocks || w1->row_count != w0->row_count)
            return fail(err, cap, "%s: gate and up must have the same type and shape", what);
    }
    if (!xq && !xa) return fail(err, cap, "%s: null activation pointer", what);
    if (n_tok < 1 || n_tok > M27B_MAX_TOKENS)
        return fail(err, cap, "%s: n_tok must be in [1, %d] (got %d)", what, M27B_MAX_TOKENS, n_tok);
    if (is_float_kind(d0.kind)) {
        // f16 / f32 weights take fp32 activations: the plain store epilogue only
        if (!xa) return fail(err, cap, "%s: f16 / f32 weights take fp32 activations (use m27b_qmv_f32)", what);
        if (epi != EPI_STORE || xa->norm_on)
            return fail(err, cap, "%s: f16 / f32 weights support the plain matvec (+ residual) only", what);
        if (!xa->xf || ((uintptr_t)xa->xf & 15) || (xa->ldxf & 3) || !y)
            return fail(err, cap, "%s: f16 / f32 matvec needs 16-byte aligned x rows (ldx a multiple of 4) and y",
                        what);
        if (ldy < (int)w0->row_count && n_tok > 1)
            return fail(err, cap, "%s: ldy (%d) < row_count (%u)", what, ldy, w0->row_count);
        const int sms = sm_count_current();
        if (sms <= 0) return fail(err, cap, "%s: no CUDA device", what);
        for (int t0 = 0; t0 < n_tok; t0 += 4) {
            const int nt = n_tok - t0 < 4 ? n_tok - t0 : 4;
            QmvArgs a{};
            a.w0 = (const uint8_t *)w0->ptr;
            a.xf = xa->xf + (size_t)t0 * xa->ldxf;
            a.ldxf = xa->ldxf;
            a.y = y + (size_t)t0 * ldy;
            a.residual = residual ? residual + (size_t)t0 * ldy : nullptr;
            a.row_stride = d0.row_stride;
            a.ldy = ldy;
            a.rows = (int)w0->row_count;
            a.k = d0.k;
            cudaError_t e = launch_qmv_float(d0.kind, a, nt, sms, stream);
            if (e != cudaSuccess) return cuda_ok(e, what, err, cap);
        }
        return ok(err, cap);
    }
    const bool kblk = d0.kind == W_Q4K || d0.kind == W_Q5K || d0.kind == W_IQ4XS;
    const bool q6_prologue = d0.kind == W_Q6KP && xa && !xa->norm_on;  // q6_K: plain quantization only
    if (xa && (!(kblk || q6_prologue) || n_tok > 4 || !xa->xf || ((uintptr_t)xa->xf & 15) || (xa->ldxf & 3)))
        return fail(err, cap,
                    "%s: in-kernel quantization needs q4_K / q5_K / IQ4_XS (or, without RMSNorm, q6_K) weights, "
                    "<= 4 tokens, 16-byte aligned rows",
                    what);
    if (epi == EPI_PUSH) {
        if (!push || push->npeers < 1 || push->npeers > M27B_MAX_PEERS || !push->epoch_base)
            return fail(err, cap, "%s: bad push descriptor", what);
        if (n_tok != 1) return fail(err, cap, "%s: the fused all-reduce takes one token", what);
        if (d0.kind == W_Q80P) return fail(err, cap, "%s: the fused all-reduce takes q4_K or q6_K weights", what);
    } else if (epi != EPI_ARGMAX && !y) {
        return fail(err, cap, "%s: null output", what);
    }
    if (epi == EPI_ARGMAX && !best) return fail(err, cap, "%s: null argmax output", what);
    if ((y || residual) && ldy < (int)w0->row_count && n_tok > 1)
        return fail(err, cap, "%s: ldy (%d) < row_count (%u)", what, ldy, w0->row_count);
    const uint32_t at = d0.base == M27B_TYPE_Q8_0 ? M27B_TYPE_Q8_0 : M27B_TYPE_Q8_K;
    const size_t xb = act_bytes(at, d0.k);
    if (((uintptr_t)xq & (at == M27B_TYPE_Q8_K ? 3u : 1u)) != 0) return fail(err, cap, "%s: misaligned activations", what);
    (void)xb;
    const size_t smem = qmv_smem_bytes(d0.base, d0.k, n_tok < 4 ? n_tok : 4);
    if (smem == 0 || smem > 227 * 1024)
        return fail(err, cap, "%s: activation staging does not fit in shared memory (k=%d too large)", what, d0.k);
    const int sms = sm_count_current();
    if (sms <= 0) return fail(err, cap, "%s: no CUDA device", what);
    int *status = status_ptr_current();
    if (!status) return fail(err, cap, "%s: cannot resolve the device status word", what);
    if (epi == EPI_ARGMAX) {
        cudaError_t e = cudaMemsetAsync(best, 0, sizeof(unsigned long long) * (size_t)n_tok, stream);
        if (e != cudaSuccess) return cuda_ok(e, what, err, cap);
    }
    // 5..16 tokens of a q4_K matrix: one pass on the tensor cores
    if (qo && (epi != EPI_SWIGLU || n_tok != 1 || (d0.kind != W_Q4K && d0.kind != W_Q5K && d0.kind != W_IQ4XS) ||
               (w0->row_count % 256) != 0 || !qo->q8 || !qo->cnt || ((uintptr_t)qo->q8 & 3)))
        return fail(err, cap, "%s: the q8_K epilogue takes one token of a 256-value k-quant SwiGLU, rows a multiple "
                              "of 256", what);
    const bool mma = !xa && d0.kind == W_Q4K && epi == EPI_STORE && q4k_mma_supported((int)w0->row_blocks, n_tok);
    for (int t0 = 0; t0 < n_tok; t0 += 4) {
        const int nt = mma ? n_tok : (n_tok - t0 < 4 ? n_tok - t0 : 4);
        QmvArgs a{};
        a.w0 = (const uint8_t *)w0->ptr;
        a.w1 = epi == EPI_SWIGLU ? (const uint8_t *)w1->ptr : nullptr;
        a.xq = xq ? (const uint8_t *)xq + (size_t)t0 * xb : nullptr;
        if (xa) {
            a.xf = xa->xf + (size_t)t0 * xa->ldxf;
            a.ldxf = xa->ldxf;
            a.xnorm_on = xa->norm_on;
            a.xnorm = xa->norm_w;
            a.eps = xa->eps;
        }
        a.y = y ? y + (size_t)t0 * ldy : nullptr;
        a.residual = residual ? residual + (size_t)t0 * ldy : nullptr;
        a.best = best ? best + t0 : nullptr;
        a.row_stride = d0.row_stride;
        a.ldy = ldy;
        a.rows = (int)w0->row_count;
        a.rb = (int)w0->row_blocks;
        a.k = d0.k;
        a.passes = d0.passes;
        a.row_offset = row_offset;
        a.status = status;
        if (push) a.push = *push;
        if (qo) {
            a.q8out = qo->q8;
            a.q8cnt = qo->cnt;
        }
        cudaError_t e = mma ? launch_q4k_mma(a, nt, sms, stream) : launch_qmv(d0.kind, epi, a, nt, sms, stream);
        if (e != cudaSuccess) return cuda_ok(e, what, err, cap);
        if (mma) break;
    }
    return ok(err, cap);
}

}  // namespace

namespace m27b {
size_t q6k_stream_part_floats(int rows, int rb);
size_t q6k_stream_count_words(int rows);
bool q6k_stream_applies(int k);
cudaError_t launch_q6k_stream(const QmvArgs &a, float *part, unsigned *count, int sm_count, cudaStream_t st,
                              int epi);

// q6_K x one token with the (row group, tile) items cut evenly over the
// grid's warps (ffn_down in a decode step): part holds
// q6k_stream_part_floats(rows, rb) floats, count one zeroed word per 8-row
// group.  q8_K activations xq, or fp32 x quantized in the prologue.
bool qmv_q6k_stream(const WeightView *w, const void *xq, const float *xf, float *y, const float *residual, float *part,
                    unsigned *count, cudaStream_t stream, char *err, size_t cap, const PushArgs *push) {
    const char *what = "qmv_q6k_stream";
    WDesc d{};
    if (!describe(w, d, what, err, cap)) return false;
    if (d.kind != W_Q6KP) return fail(err, cap, "%s: repacked q6_K weights only", what);
    if ((!xq && !xf) || (!y && !push) || !part || !count) return fail(err, cap, "%s: null pointer", what);
    if (!q6k_stream_applies(d.k)) return fail(err, cap, "%s: rows of %d values are too long to stage", what, d.k);
    const int sms = sm_count_current();
    int *status = status_ptr_current();
    if (sms <= 0 || !status) return fail(err, cap, "%s: no CUDA device", what);
    QmvArgs a{};
    a.w0 = (const uint8_t *)w->ptr;
    a.xq = xq;
    a.xf = xf;
    a.ldxf = d.k;
    a.y = y;
    a.residual = residual;
    a.row_stride = d.row_stride;
    a.ldy = (int)w->row_count;
    a.rows = (int)w->row_count;
    a.rb = (int)w->row_blocks;
    a.k = d.k;
    a.status = status;
    if (push) a.push = *push;
    return cuda_ok(launch_q6k_stream(a, part, count, sms, stream, push ? EPI_PUSH : EPI_STORE), what, err, cap) &&
           ok(err, cap);
}

// q4_K x 5..16 tokens on the tensor cores with K split across CTAs (the
// verify pass's q4_K projections): part holds q4k_mma_split_part_floats
// floats, count q4k_mma_split_count_words zeroed words.
bool qmv_mma_split(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                   float *part, unsigned *count, cudaStream_t stream, char *err, size_t cap) {
    const char *what = "qmv_mma_split";
    WDesc d{};
    if (!describe(w, d, what, err, cap)) return false;
    if (d.kind != W_Q4K) return fail(err, cap, "%s: q4_K weights only", what);
    if (!xq || !y || !part || !count) return fail(err, cap, "%s: null pointer", what);
    if (!q4k_mma_supported((int)w->row_blocks, n_tok))
        return fail(err, cap, "%s: %d tokens x %u blocks per row are not served by the tensor-core kernel", what, n_tok,
                    w->row_blocks);
    if (n_tok > 1 && ldy < (int)w->row_count) return fail(err, cap, "%s: ldy (%d) < row_count (%u)", what, ldy, w->row_count);
    const int sms = sm_count_current();
    int *status = status_ptr_current();
    if (sms <= 0 || !status) return fail(err, cap, "%s: no CUDA device", what);
    QmvArgs a{};
    a.w0 = (const uint8_t *)w->ptr;
    a.xq = xq;
    a.y = y;
    a.residual = residual;
    a.row_stride = d.row_stride;
    a.ldy = ldy;
    a.rows = (int)w->row_count;
    a.rb = (int)w->row_blocks;
    a.k = d.k;
    a.passes = d.passes;
    a.status = status;
    return cuda_ok(launch_q4k_mma(a, n_tok, sms, stream, part, count), what, err, cap) && ok(err, cap);
}

bool q6k_mma_supported(int rows, int rb, int n_tok, bool split, int sm_count);
size_t q6k_mma_part_floats(int rows);
size_t q6k_mma_count_words(int rows);
cudaError_t launch_q6k_mma(const QmvArgs &a, int n_tok, int epi, float *part, unsigned *count, int sm_count,
                           cudaStream_t st);

// q6_K x 1..8 tokens on the tensor cores (the verify pass's ffn_down and
// lm_head): EPI_STORE writes y (+ residual), EPI_ARGMAX sets best[t] to the
// packed argmax key of token t (logits into y when non-null).  part / count: K-split scratch
// (q6k_mma_part_floats floats, q6k_mma_count_words zeroed words) or null.
bool qmv_q6k_mma(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                 unsigned long long *best, uint32_t row_offset, int epi, float *part, unsigned *count,
                 cudaStream_t stream, char *err, size_t cap) {
    const char *what = epi == EPI_ARGMAX ? "qmv_q6k_mma_argmax" : "qmv_q6k_mma";
    WDesc d{};
    if (!describe(w, d, what, err, cap)) return false;
    if (d.kind != W_Q6KP) return fail(err, cap, "%s: repacked q6_K weights only", what);
    if (!xq || (epi == EPI_STORE && !y) || (epi == EPI_ARGMAX && !best))
        return fail(err, cap, "%s: null pointer", what);
    if ((part == nullptr) != (count == nullptr)) return fail(err, cap, "%s: part and count go together", what);
    const int sms = sm_count_current();
    int *status = status_ptr_current();
    if (sms <= 0 || !status) return fail(err, cap, "%s: no CUDA device", what);
    if (!q6k_mma_supported((int)w->row_count, (int)w->row_blocks, n_tok, part != nullptr, sms))
        return fail(err, cap, "%s: %d tokens x %u blocks per row are not served by the tensor-core kernel", what, n_tok,
                    w->row_blocks);
    if (n_tok > 1 && y && ldy < (int)w->row_count)
        return fail(err, cap, "%s: ldy (%d) < row_count (%u)", what, ldy, w->row_count);
    QmvArgs a{};
    a.w0 = (const uint8_t *)w->ptr;
    a.xq = xq;
    a.y = y;
    a.residual = epi == EPI_STORE ? residual : nullptr;
    a.best = best;
    a.row_offset = row_offset;
    a.row_stride = d.row_stride;
    a.ldy = y ? ldy : (int)w->row_count;
    a.rows = (int)w->row_count;
    a.rb = (int)w->row_blocks;
    a.k = d.k;
    a.status = status;
    if (epi == EPI_ARGMAX) {
        const cudaError_t e = cudaMemsetAsync(best, 0, sizeof(unsigned long long) * (size_t)n_tok, stream);
        if (e != cudaSuccess) return cuda_ok(e, what, err, cap);
    }
    return cuda_ok(launch_q6k_mma(a, n_tok, epi, part, count, sms, stream), what, err, cap) && ok(err, cap);
}

int q6k_ksplit_ranges(int rb);
size_t q6k_ksplit_part_floats(int rows, int ks);
cudaError_t launch_q6k_ksplit(const QmvArgs &a_in, int n_tok, float *part, unsigned *count, int sm_count,
                              cudaStream_t st);

// q6_K x 5..16 tokens with the K dimension split across CTAs (the verify
// pass's ffn_down): part holds q6k_ksplit_part_floats(rows, ranges) floats,
// count one zeroed word per 8-row group; 8 tokens per launch.
bool qmv_q6k_ksplit(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                    float *part, unsigned *count, cudaStream_t stream, char *err, size_t cap) {
    const char *what = "qmv_q6k_ksplit";
    WDesc d{};
    if (!describe(w, d, what, err, cap)) return false;
    if (d.kind != W_Q6KP) return fail(err, cap, "%s: repacked q6_K weights only", what);
    if (!xq || !y || !part || !count) return fail(err, cap, "%s: null pointer", what);
    if (n_tok < 1 || n_tok > M27B_MAX_TOKENS) return fail(err, cap, "%s: bad token count %d", what, n_tok);
    if (q6k_ksplit_ranges((int)w->row_blocks) == 0) return fail(err, cap, "%s: rows too short to split", what);
    const int sms = sm_count_current();
    int *status = status_ptr_current();
    if (sms <= 0 || !status) return fail(err, cap, "%s: no CUDA device", what);
    const size_t xb = act_bytes(M27B_TYPE_Q8_K, d.k);
    for (int t0 = 0; t0 < n_tok; t0 += 8) {
        const int nt = n_tok - t0 < 8 ? n_tok - t0 : 8;
        QmvArgs a{};
        a.w0 = (const uint8_t *)w->ptr;
        a.xq = (const uint8_t *)xq + (size_t)t0 * xb;
        a.y = y + (size_t)t0 * ldy;
        a.residual = residual ? residual + (size_t)t0 * ldy : nullptr;
        a.row_stride = d.row_stride;
        a.ldy = ldy;
        a.rows = (int)w->row_count;
        a.rb = (int)w->row_blocks;
        a.k = d.k;
        a.status = status;
        const cudaError_t e = launch_q6k_ksplit(a, nt, part, count, sms, stream);
        if (e != cudaSuccess) return cuda_ok(e, what, err, cap);
    }
    return ok(err, cap);
}

// Gate/up SwiGLU of one token whose epilogue also writes the rows as q8_K
// blocks into q8out (the down projection's input), from q8_K activations xq,
// or from fp32 rows xf RMSNormed with norm_w / eps in the kernel's prologue.
bool qmv_swiglu_q8(const WeightView *gate, const WeightView *up, const void *xq, const float *xf, const float *norm_w,
                   float eps, float *y, void *q8out, unsigned *q8cnt, cudaStream_t stream, char *err, size_t cap) {
    const Q8Out qo{q8out, q8cnt};
    const int rows = gate ? (int)gate->row_count : 0;
    if (xf) {
        const uint32_t base = gate ? (gate->ggml_type & M27B_TYPE_MASK) : 0;
        const int k = gate ? (int)gate->row_blocks * block_elems(base) : 0;
        XArgs xa{xf, k, 1, norm_w, eps};
        return qmv_common(EPI_SWIGLU, gate, up, nullptr, 1, y, rows, nullptr, nullptr, 0, stream, err, cap,
                          "qmv_swiglu_q8", nullptr, &xa, &qo);
    }
    return qmv_common(EPI_SWIGLU, gate, up, xq, 1, y, rows, nullptr, nullptr, 0, stream, err, cap, "qmv_swiglu_q8",
                      nullptr, nullptr, &qo);
}

// Matvec whose rows go to every rank's receive window (fused all-reduce,
// producer side); used by the tensor-parallel decode engine.
bool qmv_push(const WeightView *w, const void *xq, const float *residual, const PushArgs &push, cudaStream_t stream,
              char *err, size_t cap, const float *xf) {
    if (xf) {
        // fp32 activations quantized in the kernel's prologue (one row of k values)
        const uint32_t base = w ? (w->ggml_type & M27B_TYPE_MASK) : 0;
        const int k = w ? (int)w->row_blocks * block_elems(base) : 0;
        XArgs xa{xf, k, 0, nullptr, 0.0f};
        return qmv_common(EPI_PUSH, w, nullptr, nullptr, 1, nullptr, (int)(w ? w->row_count : 0), residual, nullptr, 0,
                          stream, err, cap, "qmv_push", &push, &xa);
    }
    return qmv_common(EPI_PUSH, w, nullptr, xq, 1, nullptr, (int)(w ? w->row_count : 0), residual, nullptr, 0, stream,
                      err, cap, "qmv_push", &push);
}
}  // namespace m27b

extern "C" {

const char *m27b_version(void) { return "m27b-b200 0.1 (sm_100a)"; }

bool m27b_device_status(int *status, int clear, char *err, size_t err_cap) {
    if (!status) return fail(err, err_cap, "m27b_device_status: null output");
    int *p = status_ptr_current();
    if (!p) return fail(err, err_cap, "m27b_device_status: no CUDA device");
    cudaError_t e = cudaMemcpy(status, p, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_ok(e, "m27b_device_status", err, err_cap);
    if (clear && *status) {
        const int zero = 0;
        e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_ok(e, "m27b_device_status", err, err_cap);
    }
    return ok(err, err_cap);
}

size_t m27b_act_bytes(uint32_t act_type, int k) { return act_bytes(act_type, k); }

uint32_t m27b_act_type_for(uint32_t ggml_type) {
    const uint32_t b = ggml_type & M27B_TYPE_MASK;
    if (b == M27B_TYPE_Q8_0) return M27B_TYPE_Q8_0;
    if (b == M27B_TYPE_Q4_K || b == M27B_TYPE_Q5_K || b == M27B_TYPE_Q6_K || b == M27B_TYPE_IQ4_XS)
        return M27B_TYPE_Q8_K;
    return 0;
}

bool m27b_act_quant(const float *x, int k, int n_tok, int ldx, uint32_t act_type, void *xq, cudaStream_t stream, char *err,
                    size_t err_cap) {
    return act_quant_common(ACT_PLAIN, x, nullptr, nullptr, 0.0f, k, n_tok, ldx, act_type, xq, stream, err, err_cap,
                            "m27b_act_quant");
}

bool m27b_act_quant_swiglu(const float *gate, const float *up, int k, int n_tok, int ldx, uint32_t act_type, void *xq,
                           cudaStream_t stream, char *err, size_t err_cap) {
    if (!gate) return fail(err, err_cap, "m27b_act_quant_swiglu: null gate");
    return act_quant_common(ACT_SWIGLU, up, gate, nullptr, 0.0f, k, n_tok, ldx, act_type, xq, stream, err, err_cap,
                            "m27b_act_quant_swiglu");
}

bool m27b_act_quant_gated(const float *x, const float *gate, int k, int n_tok, int ldx, uint32_t act_type, void *xq,
                          cudaStream_t stream, char *err, size_t err_cap) {
    return act_quant_common(ACT_GATED, x, gate, nullptr, 0.0f, k, n_tok, ldx, act_type, xq, stream, err, err_cap,
                            "m27b_act_quant_gated");
}

bool m27b_act_quant_rmsnorm(const float *x, const float *w, float eps, int k, int n_tok, int ldx, uint32_t act_type,
                            void *xq, cudaStream_t stream, char *err, size_t err_cap) {
    return act_quant_common(ACT_RMSNORM, x, nullptr, w, eps, k, n_tok, ldx, act_type, xq, stream, err, err_cap,
                            "m27b_act_quant_rmsnorm");
}

size_t m27b_repacked_bytes(uint32_t ggml_type, uint32_t row_blocks, uint32_t row_count) {
    const uint32_t b = ggml_type & M27B_TYPE_MASK;
    if (b != M27B_TYPE_Q6_K && b != M27B_TYPE_Q8_0) return 0;
    return planar_row_bytes((int)b, (int)row_blocks) * (size_t)row_count;
}

bool m27b_repack(const void *raw, uint32_t ggml_type, uint32_t row_blocks, uint32_t row_count, void *out,
                 cudaStream_t stream, char *err, size_t err_cap) {
    const uint32_t b = ggml_type & M27B_TYPE_MASK;
    if (!raw || !out) return fail(err, err_cap, "m27b_repack: null pointer");
    if (ggml_type != M27B_TYPE_Q6_K && ggml_type != M27B_TYPE_Q8_0)
        return fail(err, err_cap, "m27b_repack: only raw q6_K and q8_0 are repacked (got type 0x%x)", ggml_type);
    if (row_blocks == 0 || row_count == 0) return fail(err, err_cap, "m27b_repack: empty tensor");
    if (row_blocks > 65535u || row_count > 0x7fffffffu) return fail(err, err_cap, "m27b_repack: tensor too large");
    if (((uintptr_t)out & 15u) != 0) return fail(err, err_cap, "m27b_repack: output must be 16-byte aligned");
    return cuda_ok(launch_repack((int)b, raw, (int)row_blocks, (int)row_count, out, stream), "m27b_repack", err, err_cap);
}

bool m27b_qmv(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual, cudaStream_t stream,
              char *err, size_t err_cap) {
    return qmv_common(EPI_STORE, w, nullptr, xq, n_tok, y, ldy, residual, nullptr, 0, stream, err, err_cap, "m27b_qmv");
}

bool m27b_qmv_swiglu(const WeightView *gate, const WeightView *up, const void *xq, int n_tok, float *y, int ldy,
                     cudaStream_t stream, char *err, size_t err_cap) {
    return qmv_common(EPI_SWIGLU, gate, up, xq, n_tok, y, ldy, nullptr, nullptr, 0, stream, err, err_cap,
                      "m27b_qmv_swiglu");
}

bool m27b_qmv_argmax(const WeightView *w, const void *xq, int n_tok, float *logits, int ldl, unsigned long long *best,
                     uint32_t row_offset, cudaStream_t stream, char *err, size_t err_cap) {
    return qmv_common(EPI_ARGMAX, w, nullptr, xq, n_tok, logits, ldl, nullptr, best, row_offset, stream, err, err_cap,
                      "m27b_qmv_argmax");
}

// fp32 activations: quantized inside the q4_K kernel's prologue (<= 4 tokens),
// otherwise into xq_scratch by a separate quantizer launch first.
static bool qmv_f32_common(const WeightView *w, const WeightView *w_up, const float *x, int ldx, int norm_on,
                           const float *norm_w, float eps, int n_tok, void *xq_scratch, float *y, int ldy,
                           const float *residual, cudaStream_t stream, char *err, size_t cap, const char *what) {
    if (!w || !x) return fail(err, cap, "%s: null argument", what);
    if (w_up && residual) return fail(err, cap, "%s: the SwiGLU epilogue takes no residual", what);
    const int epi = w_up ? EPI_SWIGLU : EPI_STORE;
    const uint32_t base = w->ggml_type & M27B_TYPE_MASK;
    const int k = (int)w->row_blocks * block_elems(base);
    if (k <= 0) return fail(err, cap, "%s: unsupported weight type 0x%x", what, w->ggml_type);
    if (ldx < k) return fail(err, cap, "%s: ldx (%d) < k (%d)", what, ldx, k);
    if (base == M27B_TYPE_F16 || base == M27B_TYPE_F32) {
        // fp32 activations go straight into the f16 / f32 kernel
        XArgs xa{x, ldx, norm_on, norm_w, eps};
        return qmv_common(epi, w, w_up, nullptr, n_tok, y, ldy, residual, nullptr, 0, stream, err, cap, what, nullptr,
                          &xa);
    }
    const bool kblk = w->ggml_type == M27B_TYPE_Q4_K || w->ggml_type == M27B_TYPE_Q5_K ||
                      w->ggml_type == M27B_TYPE_IQ4_XS ||
                      (w->ggml_type == (M27B_TYPE_Q6_K | M27B_LAYOUT_PLANAR) && !norm_on);
    if (kblk && n_tok >= 1 && n_tok <= 4 && ((uintptr_t)x & 15) == 0 && (ldx & 3) == 0) {
        XArgs xa{x, ldx, norm_on, norm_w, eps};
        return qmv_common(epi, w, w_up, nullptr, n_tok, y, ldy, residual, nullptr, 0, stream, err, cap, what, nullptr,
                          &xa);
    }
    if (!xq_scratch) return fail(err, cap, "%s: this weight type / token count needs xq_scratch", what);
    const uint32_t at = base == M27B_TYPE_Q8_0 ? M27B_TYPE_Q8_0 : M27B_TYPE_Q8_K;
    if (!act_quant_common(norm_on ? ACT_RMSNORM : ACT_PLAIN, x, nullptr, norm_w, eps, k, n_tok, ldx, at, xq_scratch,
                          stream, err, cap, what))
        return false;
    return qmv_common(epi, w, w_up, xq_scratch, n_tok, y, ldy, residual, nullptr, 0, stream, err, cap, what);
}

bool m27b_qmv_f32(const WeightView *w, const float *x, int ldx, int n_tok, void *xq_scratch, float *y, int ldy,
                  const float *residual, cudaStream_t stream, char *err, size_t err_cap) {
    return qmv_f32_common(w, nullptr, x, ldx, 0, nullptr, 0.0f, n_tok, xq_scratch, y, ldy, residual, stream, err,
                          err_cap, "m27b_qmv_f32");
}

bool m27b_qmv_f32_rmsnorm(const WeightView *w, const WeightView *w_up, const float *x, int ldx, const float *norm_w,
                          float eps, int n_tok, void *xq_scratch, float *y, int ldy, const float *residual,
                          cudaStream_t stream, char *err, size_t err_cap) {
    return qmv_f32_common(w, w_up, x, ldx, 1, norm_w, eps, n_tok, xq_scratch, y, ldy, residual, stream, err, err_cap,
                          "m27b_qmv_f32_rmsnorm");
}

bool m27b_dequant_rows(const WeightView *w, const int32_t *rows, int n, float *out, int ldo, cudaStream_t stream, char *err,
                       size_t err_cap) {
    if (!w || !w->ptr || !rows || !out) return fail(err, err_cap, "m27b_dequant_rows: null pointer");
    if (n < 1) return fail(err, err_cap, "m27b_dequant_rows: n must be >= 1");
    const uint32_t base = w->ggml_type & M27B_TYPE_MASK;
    const bool planar = (w->ggml_type & M27B_LAYOUT_PLANAR) != 0;
    const int be = block_elems(base);
    if ((base != M27B_TYPE_Q4_K && base != M27B_TYPE_Q6_K && base != M27B_TYPE_Q8_0) ||
        (planar && base == M27B_TYPE_Q4_K))
        return fail(err, err_cap, "m27b_dequant_rows: unsupported weight type 0x%x (q4_K, q6_K, q8_0)", w->ggml_type);
    if (w->row_blocks == 0 || w->row_blocks > 0x7fffffffu / 256u) return fail(err, err_cap, "m27b_dequant_rows: bad row_blocks");
    const int k = (int)w->row_blocks * be;
    if (ldo < k) return fail(err, err_cap, "m27b_dequant_rows: ldo (%d) < k (%d)", ldo, k);
    size_t stride;
    if (planar) stride = planar_row_bytes((int)base, (int)w->row_blocks);
    else stride = (size_t)w->row_blocks * (base == M27B_TYPE_Q4_K ? 144 : base == M27B_TYPE_Q6_K ? 210 : 34);
    return cuda_ok(launch_dequant_rows((int)base, planar, w->ptr, stride, (int)w->row_blocks, (int)w->row_count, k, rows, n,
                                       out, ldo, stream),
                   "m27b_dequant_rows", err, err_cap);
}

bool m27b_allreduce_norm_quant(const void *words, int nsrc, int src_stride, void *ss_words, const unsigned *epoch,
                               const float *norm_w, float eps, int k, float *x_out, void *xq, unsigned long long wait_ns,
                               cudaStream_t stream, char *err, size_t err_cap) {
    const char *what = "m27b_allreduce_norm_quant";
    if (!words || !ss_words || !epoch || !x_out || !xq) return fail(err, err_cap, "%s: null pointer", what);
    if (nsrc < 1 || nsrc > M27B_ALLREDUCE_MAX_SRC)
        return fail(err, err_cap, "%s: nsrc must be in [1, %d] (got %d)", what, M27B_ALLREDUCE_MAX_SRC, nsrc);
    if (k < 256 || k % 256 || k > 65536) return fail(err, err_cap, "%s: k must be a multiple of 256 in [256, 65536]", what);
    if (src_stride < k) return fail(err, err_cap, "%s: src_stride (%d) < k (%d)", what, src_stride, k);
    if (((uintptr_t)words & 7u) || ((uintptr_t)ss_words & 7u))
        return fail(err, err_cap, "%s: words must be 8-byte aligned", what);
    if (((uintptr_t)xq & 3u) != 0) return fail(err, err_cap, "%s: output must be 4-byte aligned", what);
    ActArgs a{};
    a.w = norm_w;
    a.eps = eps;
    a.k = k;
    a.ldx = k;
    a.out = xq;
    a.words = (const uint2 *)words;
    a.nsrc = nsrc;
    a.src_stride = src_stride;
    a.ss_words = (uint2 *)ss_words;
    a.epoch_base = epoch;
    a.epoch_mul = 1u;
    a.epoch_add = 0u;
    a.x_out = x_out;
    a.status = status_ptr_current();
    a.wait_ns = wait_ns;
    if (!a.status) return fail(err, err_cap, "%s: cannot resolve the device status word", what);
    return cuda_ok(launch_act_quant(M27B_TYPE_Q8_K, ACT_RMSNORM_SUM, a, 1, stream), what, err, err_cap);
}

size_t m27b_qmv_q6k_ksplit_part_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    const int ks = q6k_ksplit_ranges((int)w->row_blocks);
    return ks ? q6k_ksplit_part_floats((int)w->row_count, ks) * sizeof(float) : 0;
}

size_t m27b_qmv_q6k_ksplit_count_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    return q6k_ksplit_ranges((int)w->row_blocks) ? (size_t)((w->row_count + 7) / 8) * sizeof(unsigned) : 0;
}

size_t m27b_qmv_mma_split_part_bytes(const WeightView *w, int n_tok) {
    if (!w || w->ggml_type != M27B_TYPE_Q4_K || n_tok < 5 || n_tok > 16) return 0;
    return q4k_mma_split_part_floats((int)w->row_count, (int)w->row_blocks, n_tok) * sizeof(float);
}

size_t m27b_qmv_mma_split_count_bytes(const WeightView *w) {
    if (!w || w->ggml_type != M27B_TYPE_Q4_K) return 0;
    return q4k_mma_split_count_words((int)w->row_count) * sizeof(unsigned);
}

bool m27b_qmv_mma_split(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                        void *part, void *count, cudaStream_t stream, char *err, size_t err_cap) {
    if (((uintptr_t)part & 15) || ((uintptr_t)count & 3))
        return fail(err, err_cap, "m27b_qmv_mma_split: misaligned scratch");
    return qmv_mma_split(w, xq, n_tok, y, ldy, residual, (float *)part, (unsigned *)count, stream, err, err_cap);
}

size_t m27b_qmv_q6k_mma_part_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    return q6k_mma_part_floats((int)w->row_count) * sizeof(float);
}

size_t m27b_qmv_q6k_mma_count_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    return q6k_mma_count_words((int)w->row_count) * sizeof(unsigned);
}

bool m27b_qmv_q6k_mma(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                      void *part, void *count, cudaStream_t stream, char *err, size_t err_cap) {
    if (((uintptr_t)part & 15) || ((uintptr_t)count & 3))
        return fail(err, err_cap, "m27b_qmv_q6k_mma: misaligned scratch");
    return qmv_q6k_mma(w, xq, n_tok, y, ldy, residual, nullptr, 0u, EPI_STORE, (float *)part, (unsigned *)count,
                       stream, err, err_cap);
}

bool m27b_qmv_q6k_mma_argmax(const WeightView *w, const void *xq, int n_tok, float *logits, int ldl,
                             unsigned long long *best, uint32_t row_offset, cudaStream_t stream, char *err,
                             size_t err_cap) {
    return qmv_q6k_mma(w, xq, n_tok, logits, ldl, nullptr, best, row_offset, EPI_ARGMAX, nullptr, nullptr, stream, err,
                       err_cap);
}

size_t m27b_qmv_q6k_stream_part_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    return q6k_stream_part_floats((int)w->row_count, (int)w->row_blocks) * sizeof(float);
}

size_t m27b_qmv_q6k_stream_count_bytes(const WeightView *w) {
    if (!w || (w->ggml_type & M27B_TYPE_MASK) != M27B_TYPE_Q6_K) return 0;
    return q6k_stream_count_words((int)w->row_count) * sizeof(unsigned);
}

bool m27b_qmv_q6k_stream(const WeightView *w, const void *xq, float *y, const float *residual, void *part, void *count,
                         cudaStream_t stream, char *err, size_t err_cap) {
    if (((uintptr_t)part & 15) || ((uintptr_t)count & 3))
        return fail(err, err_cap, "m27b_qmv_q6k_stream: misaligned scratch");
    if (!xq) return fail(err, err_cap, "m27b_qmv_q6k_stream: null pointer");
    return qmv_q6k_stream(w, xq, nullptr, y, residual, (float *)part, (unsigned *)count, stream, err, err_cap,
                          nullptr);
}

bool m27b_qmv_q6k_ksplit(const WeightView *w, const void *xq, int n_tok, float *y, int ldy, const float *residual,
                         void *part, void *count, cudaStream_t stream, char *err, size_t err_cap) {
    if (((uintptr_t)part & 15) || ((uintptr_t)count & 3))
        return fail(err, err_cap, "m27b_qmv_q6k_ksplit: misaligned scratch");
    if (w && n_tok > 1 && ldy < (int)w->row_count)
        return fail(err, err_cap, "m27b_qmv_q6k_ksplit: ldy (%d) < row_count (%u)", ldy, w->row_count);
    return qmv_q6k_ksplit(w, xq, n_tok, y, ldy, residual, (float *)part, (unsigned *)count, stream, err, err_cap);
}

}  // extern "C"
