// attn.cu — C ABI of the decode attention kernels (include/m27b_attn.h).
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "m27b_attn.h"

namespace m27b {
cudaError_t attn_prepare();
cudaError_t attn_launch(const float *q, const float *kc, const float *vc, float *part, float *out, const int *pos,
                        int nq, int nkv, int hd, int S, float scale, cudaStream_t st, int n_tok = 1);
}  // namespace m27b

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

constexpr int kMaxDevices = 64;

// Split partials of m27b_attn_decode_noalloc (one per device; see the header
// for the sharing rules).  Module-scope device memory: no allocation call.
constexpr size_t kNoallocFloats = M27B_ATTN_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoallocFloats];

// Device address of the static scratch on the current device (looked up once
// per device, with that device current).
bool noalloc_scratch(float **out, char *err, size_t cap) {
    static std::mutex mu;
    static float *ptr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return afail(err, cap, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return afail(err, cap, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!ptr[dev]) {
        float *p = nullptr;
        e = cudaGetSymbolAddress((void **)&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return afail(err, cap, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
        ptr[dev] = p;
    }
    *out = ptr[dev];
    return true;
}

// Raise the attention kernels' shared-memory limit once per device.
bool attn_ready(char *err, size_t cap) {
    static std::mutex mu;
    static bool done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return afail(err, cap, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return afail(err, cap, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev]) return true;
    e = m27b::attn_prepare();
    if (e != cudaSuccess) return afail(err, cap, "attention shared-memory opt-in: %s", cudaGetErrorString(e));
    done[dev] = true;
    return true;
}

}  // namespace

extern "C" {

size_t m27b_attn_part_bytes(int n_q, int head_dim, int splits) {
    if (n_q < 1 || head_dim < 32 || head_dim > 256 || head_dim % 32 || splits < 1) return 0;
    return (size_t)splits * n_q * (head_dim + 4) * sizeof(float);
}

bool m27b_attn_decode(const float *q, const float *k_cache, const float *v_cache, const int *pos, int n_q, int n_kv,
                      int head_dim, int splits, float scale, float *part, float *out, cudaStream_t stream, char *err,
                      size_t err_cap) {
    const char *what = "m27b_attn_decode";
    if (!q || !k_cache || !v_cache || !pos || !part || !out) return afail(err, err_cap, "%s: null pointer", what);
    if (head_dim < 32 || head_dim > 256 || head_dim % 32)
        return afail(err, err_cap, "%s: head_dim must be a multiple of 32 in [32, 256] (got %d)", what, head_dim);
    if (n_kv < 1 || n_q < n_kv || n_q % n_kv || n_q / n_kv > 8)
        return afail(err, err_cap, "%s: n_q (%d) must be a multiple of n_kv (%d), at most 8 per kv head", what, n_q, n_kv);
    if (splits < 1 || splits > 65535) return afail(err, err_cap, "%s: splits must be in [1, 65535] (got %d)", what, splits);
    if (((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)part | (uintptr_t)out) & 15u)
        return afail(err, err_cap, "%s: q, caches, part and out must be 16-byte aligned", what);
    if (!attn_ready(err, err_cap)) return false;
    const cudaError_t e = m27b::attn_launch(q, k_cache, v_cache, part, out, pos, n_q, n_kv, head_dim, splits, scale, stream);
    if (e != cudaSuccess) return afail(err, err_cap, "%s: launch: %s", what, cudaGetErrorString(e));
    if (err && err_cap) err[0] = '\0';
    return true;
}

size_t m27b_attn_noalloc_scratch_bytes(void) { return M27B_ATTN_NOALLOC_SCRATCH_BYTES; }

bool m27b_attn_decode_noalloc(const float *q, const float *k_cache, const float *v_cache, const int *pos, int n_q,
                              int n_kv, int head_dim, int splits, float scale, float *out, cudaStream_t stream, char *err,
                              size_t err_cap) {
    const char *what = "m27b_attn_decode_noalloc";
    const size_t need = m27b_attn_part_bytes(n_q, head_dim, splits);
    if (need > M27B_ATTN_NOALLOC_SCRATCH_BYTES)
        return afail(err, err_cap,
                     "%s: %d heads x %d values over %d splits need %zu bytes of scratch; the static scratch holds %u "
                     "(use fewer splits, or m27b_attn_decode with a caller buffer)",
                     what, n_q, head_dim, splits, need, (unsigned)M27B_ATTN_NOALLOC_SCRATCH_BYTES);
    float *scratch = nullptr;
    if (!noalloc_scratch(&scratch, err, err_cap)) return false;
    char e2[512];
    if (!m27b_attn_decode(q, k_cache, v_cache, pos, n_q, n_kv, head_dim, splits, scale, scratch, out, stream, e2,
                          sizeof(e2))) {
        // report under this entry's name
        const char *msg = e2;
        const size_t n = std::strlen("m27b_attn_decode");
        if (std::strncmp(msg, "m27b_attn_decode", n) == 0) msg += n;
        return afail(err, err_cap, "%s%s", what, msg);
    }
    return true;
}

}  // extern "C"
