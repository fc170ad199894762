/*
 * ggml_semantics.c — CPU ORACLE (test infrastructure only).
 *
 * This file is the checker for the CUDA quantized matvec path.  Only the
 * tests, the smoke check and bench.py's CPU-baseline leg may load it; the
 * product library never links or calls it.
 *
 * What it restates
 * ----------------
 * The named oracle is ggml's CPU path (llama.cpp, ggml/src/ggml-quants.c and
 * ggml/src/ggml-cpu/quants.c): quantize_row_q8_K_ref, quantize_row_q8_0_ref,
 * quantize_row_q4_K_ref / q5_K_ref (make_qkx2_quants), quantize_row_q6_K_ref
 * (make_qx_quants), dequantize_row_q4_K / q5_K / q6_K / q8_0 / iq4_xs and
 * the generic ggml_vec_dot_q4_K_q8_K / q5_K_q8_K / q6_K_q8_K / iq4_xs_q8_K /
 * q8_0_q8_0 / f16 / f32.  llama.cpp is vendored by the
 * reference as an EMPTY, git-ignored directory (reference .gitignore:3,
 * ref/llama.cpp/) with no pinned commit, so the algorithms below are written
 * from ggml's published block formats and quantization rules, not from a
 * copy of its source.
 *
 * Block layouts follow the reference's structs:
 *   BlockQ4K    src/mono27b_executor.cu:18-23   (144 B)
 *   BlockQ8     src/mono27b_executor.cu:25-28   (q8_0, 34 B)
 *   BlockQ5K    src/mono27b_executor.cu:30-36   (176 B)
 *   BlockQ8K    src/mono27b_executor.cu:38-42   (292 B)
 *   BlockIQ4XS  src/mono27b_executor.cu:44-49   (136 B; codebook :51-55)
 *   BlockQ6K    src/mono27b_executor.cu:57-62   (210 B)
 * Dequant formulas follow debug/official_dequant.c:47-65 (q4_K),
 * src/mono27b_executor.cu:955-969 (q5k_val), :1004-1011 (IQ4_XS) and
 * :1026-1048 (q6k_val), and get_scale_min_k4 at src/mono27b_executor.cu:690-693.
 * f16 / f32 weights (the reference's k_f16_mv / k_f32_mv, :900-916,
 * :1101-1114) take fp32 activations; ggml converts them to the weight's
 * vec_dot type first (fp16 for f16 weights, round to nearest even) and sums
 * the products in double.
 *
 * Pinning: dequant and the q8_0 quantizer are checked bit for bit against the
 * gguf 0.19.0 Python package (llama.cpp's gguf-py) through committed golden
 * fixtures, and the q4_K dequant against the 16 known outputs of
 * debug/official_dequant.c / debug/mono_give_current.debug.tsv:2.  The
 * IQ4_XS weight quantizer here is this oracle's own simple nearest-codebook
 * fit (ggml's search is not restated): it only generates test weights, and
 * the GPU and the CPU consume the same bytes.
 *
 * Build with -ffp-contract=off: every dequantized value is
 * fl(fl(d*sc)*q) - fl(dmin*m) with no fused multiply-add, which is the
 * bit-exact target for the GPU dequant.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 256

typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } orc_q4K;
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } orc_q6K;
typedef struct { uint16_t d; int8_t qs[32]; } orc_q80;
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } orc_q8K;
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qh[32]; uint8_t qs[128]; } orc_q5K;
typedef struct { uint16_t d; uint16_t scales_h; uint8_t scales_l[4]; uint8_t qs[128]; } orc_iq4xs;

/* The IQ4_NL / IQ4_XS codebook: the 16 signed values a 4-bit code stands for
 * (a format constant; reference src/mono27b_executor.cu:51-55). */
static const int8_t IQ4_VALUES[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

_Static_assert(sizeof(orc_q4K) == 144, "q4_K block is 144 bytes");
_Static_assert(sizeof(orc_q6K) == 210, "q6_K block is 210 bytes");
_Static_assert(sizeof(orc_q80) == 34, "q8_0 block is 34 bytes");
_Static_assert(sizeof(orc_q8K) == 292, "q8_K block is 292 bytes");
_Static_assert(sizeof(orc_q5K) == 176, "q5_K block is 176 bytes");
_Static_assert(sizeof(orc_iq4xs) == 136, "IQ4_XS block is 136 bytes");

/* ---- fp16 <-> fp32 ------------------------------------------------------ */

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE half -> single; exact for every input (normal, subnormal, inf, nan). */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1f) return bits_f32(sign | 0x7f800000u | (man << 13));
    if (exp == 0) {
        /* subnormal: man * 2^-24, exact in fp32 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* IEEE single -> half, round to nearest even (what F16C's vcvtps2ph with
 * rounding mode 0 and CUDA's __float2half_rn do). */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x = f32_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (ax < 0x38800000u) {
        /* result is subnormal (or zero): value / 2^-24, rounded to even */
        float a = bits_f32(ax);
        float q = a * 16777216.0f; /* exact scaling by 2^24 */
        float r = rintf(q);        /* default rounding mode: nearest even */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* carries into exp correctly */
    return (uint16_t)(sign | h);
}

/* Round to nearest, ties to even, for |v| < 2^22: ggml's nearest_int. */
static int rne_int(float v) { return (int)rintf(v); }

/* The 6-bit scale / min of sub-block j of a q4_K super-block
 * (src/mono27b_executor.cu:690-693). */
static void q4K_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) { *sc = s[j] & 63; *mn = s[j + 4] & 63; }
    else { *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4); *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

/* ---- dequantization ----------------------------------------------------- */

void orc_dequantize_row_q4_K(const void *vx, float *y, int64_t k) {
    const orc_q4K *x = (const orc_q4K *)vx;
    for (int64_t b = 0; b < k / QK; ++b) {
        const float d = orc_fp16_to_fp32(x[b].d), dmin = orc_fp16_to_fp32(x[b].dmin);
        for (int g = 0; g < 4; ++g) {
            int sc0, m0, sc1, m1;
            q4K_scale_min(2 * g, x[b].scales, &sc0, &m0);
            q4K_scale_min(2 * g + 1, x[b].scales, &sc1, &m1);
            const float d0 = d * (float)sc0, n0 = dmin * (float)m0;
            const float d1 = d * (float)sc1, n1 = dmin * (float)m1;
            const uint8_t *q = x[b].qs + 32 * g;
            float *o = y + b * QK + 64 * g;
            for (int l = 0; l < 32; ++l) o[l] = d0 * (float)(q[l] & 15) - n0;
            for (int l = 0; l < 32; ++l) o[32 + l] = d1 * (float)(q[l] >> 4) - n1;
        }
    }
}

/* element e of a q6_K block as the signed 6-bit code (q - 32) */
static int q6K_code(const orc_q6K *b, int e) {
    const int half = e / 128, r = (e % 128) / 32, l = e % 32;
    const uint8_t *ql = b->ql + 64 * half, *qh = b->qh + 32 * half;
    int lo = (r & 1) ? ql[l + 32] : ql[l];
    lo = (r & 2) ? (lo >> 4) : (lo & 15);
    int hi = (qh[l] >> (2 * r)) & 3;
    return (lo | (hi << 4)) - 32;
}

void orc_dequantize_row_q6_K(const void *vx, float *y, int64_t k) {
    const orc_q6K *x = (const orc_q6K *)vx;
    for (int64_t b = 0; b < k / QK; ++b) {
        const float d = orc_fp16_to_fp32(x[b].d);
        for (int e = 0; e < QK; ++e) {
            const float ds = d * (float)x[b].scales[e / 16];
            y[b * QK + e] = ds * (float)q6K_code(&x[b], e);
        }
    }
}

/* q5_K: sub-block s = 2g + h takes the low (h = 0) or high (h = 1) nibbles of
 * qs[32g .. 32g+31] plus 16 x bit s of qh[l]; value d*sc*q - dmin*m. */
void orc_dequantize_row_q5_K(const void *vx, float *y, int64_t k) {
    const orc_q5K *x = (const orc_q5K *)vx;
    for (int64_t b = 0; b < k / QK; ++b) {
        const float d = orc_fp16_to_fp32(x[b].d), dmin = orc_fp16_to_fp32(x[b].dmin);
        for (int g = 0; g < 4; ++g) {
            int sc0, m0, sc1, m1;
            q4K_scale_min(2 * g, x[b].scales, &sc0, &m0);
            q4K_scale_min(2 * g + 1, x[b].scales, &sc1, &m1);
            const float d0 = d * (float)sc0, n0 = dmin * (float)m0;
            const float d1 = d * (float)sc1, n1 = dmin * (float)m1;
            const uint8_t *q = x[b].qs + 32 * g;
            float *o = y + b * QK + 64 * g;
            for (int l = 0; l < 32; ++l)
                o[l] = d0 * (float)((q[l] & 15) + ((x[b].qh[l] >> (2 * g)) & 1 ? 16 : 0)) - n0;
            for (int l = 0; l < 32; ++l)
                o[32 + l] = d1 * (float)((q[l] >> 4) + ((x[b].qh[l] >> (2 * g + 1)) & 1 ? 16 : 0)) - n1;
        }
    }
}

/* The 6-bit scale of sub-block ib of an IQ4_XS block, as stored (0..63;
 * the multiplier is ls - 32). */
static int iq4xs_ls(const orc_iq4xs *b, int ib) {
    return ((b->scales_l[ib / 2] >> (4 * (ib % 2))) & 15) | (((b->scales_h >> (2 * ib)) & 3) << 4);
}

/* IQ4_XS: sub-block ib holds qs[16ib .. 16ib+15]; low nibbles are its
 * elements 0..15, high nibbles 16..31; value (d*(ls-32)) * codebook[q]. */
void orc_dequantize_row_iq4_xs(const void *vx, float *y, int64_t k) {
    const orc_iq4xs *x = (const orc_iq4xs *)vx;
    for (int64_t b = 0; b < k / QK; ++b) {
        const float d = orc_fp16_to_fp32(x[b].d);
        for (int ib = 0; ib < 8; ++ib) {
            const float dl = d * (float)(iq4xs_ls(&x[b], ib) - 32);
            const uint8_t *q = x[b].qs + 16 * ib;
            float *o = y + b * QK + 32 * ib;
            for (int j = 0; j < 16; ++j) {
                o[j] = dl * (float)IQ4_VALUES[q[j] & 15];
                o[16 + j] = dl * (float)IQ4_VALUES[q[j] >> 4];
            }
        }
    }
}

void orc_dequantize_row_f16(const void *vx, float *y, int64_t k) {
    const uint16_t *x = (const uint16_t *)vx;
    for (int64_t i = 0; i < k; ++i) y[i] = orc_fp16_to_fp32(x[i]);
}

void orc_dequantize_row_q8_0(const void *vx, float *y, int64_t k) {
    const orc_q80 *x = (const orc_q80 *)vx;
    for (int64_t b = 0; b < k / 32; ++b) {
        const float d = orc_fp16_to_fp32(x[b].d);
        for (int i = 0; i < 32; ++i) y[b * 32 + i] = (float)x[b].qs[i] * d;
    }
}

/* ---- activation quantizers ---------------------------------------------- */

/* q8_K: per 256 values, the signed value of largest magnitude m sets
 * iscale = -127/m; q = min(127, rne(iscale*x)); d = 1/iscale; bsums are the
 * sums of each 16 consecutive codes.  An all-zero block gives d = 0, q = 0. */
void orc_quantize_row_q8_K(const float *x, void *vy, int64_t k) {
    orc_q8K *y = (orc_q8K *)vy;
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        float amax = 0.0f, m = 0.0f;
        for (int j = 0; j < QK; ++j) {
            const float a = fabsf(x[j]);
            if (a > amax) { amax = a; m = x[j]; }
        }
        memset(&y[b], 0, sizeof(orc_q8K));
        if (amax == 0.0f) continue;
        const float iscale = -127.0f / m;
        for (int j = 0; j < QK; ++j) {
            int v = rne_int(iscale * x[j]);
            y[b].qs[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += y[b].qs[16 * g + i];
            y[b].bsums[g] = (int16_t)s;
        }
        y[b].d = 1.0f / iscale;
    }
}

/* q8_0: per 32 values, d = amax/127 stored as fp16, q = roundf(x * (1/d))
 * with ties away from zero. */
void orc_quantize_row_q8_0(const float *x, void *vy, int64_t k) {
    orc_q80 *y = (orc_q80 *)vy;
    for (int64_t b = 0; b < k / 32; ++b, x += 32) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[b].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 32; ++j) y[b].qs[j] = (int8_t)roundf(x[j] * id);
    }
}

/* ---- weight quantizers (used to GENERATE seeded test weights) ----------- */

/* Weighted asymmetric fit of n values to codes 0..nmax with a scale and a
 * non-positive offset: an initial min/max grid followed by nstep+1 trial
 * grids iscale = (nmax + rmin + rdelta*is)/(max-min), each refined by the
 * weighted least-squares scale/offset for its codes; the trial with the
 * smallest weighted squared error wins.  Returns the scale and stores -offset
 * in *neg_off.  (ggml's make_qkx2_quants with squared error; q4_K calls it
 * with rmin=-1, rdelta=0.1, nstep=20, q5_K with rmin=-0.5, rdelta=0.1,
 * nstep=15.) */
static float fit_asym(int n, int nmax, const float *x, const float *w, uint8_t *L,
                      float *neg_off, uint8_t *trial, float rmin, float rdelta, int nstep) {
    float lo = x[0], hi = x[0], sw = w[0], swx = w[0] * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
        sw += w[i];
        swx += w[i] * x[i];
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
        memset(L, 0, (size_t)n);
        *neg_off = -lo;
        return 0.0f;
    }
    float inv = (float)nmax / (hi - lo);
    float scale = 1.0f / inv;
    float err_best = 0.0f;
    for (int i = 0; i < n; ++i) {
        int l = rne_int(inv * (x[i] - lo));
        l = l < 0 ? 0 : (l > nmax ? nmax : l);
        L[i] = (uint8_t)l;
        const float r = scale * (float)l + lo - x[i];
        err_best += w[i] * (r * r);
    }
    for (int is = 0; is <= nstep; ++is) {
        inv = (rmin + rdelta * (float)is + (float)nmax) / (hi - lo);
        float sl = 0, sl2 = 0, sxl = 0;
        for (int i = 0; i < n; ++i) {
            int l = rne_int(inv * (x[i] - lo));
            l = l < 0 ? 0 : (l > nmax ? nmax : l);
            trial[i] = (uint8_t)l;
            sl += w[i] * (float)l;
            sl2 += w[i] * (float)l * (float)l;
            sxl += w[i] * (float)l * x[i];
        }
        const float det = sw * sl2 - sl * sl;
        if (det > 0) {
            float s = (sw * sxl - swx * sl) / det;
            float off = (sl2 * swx - sl * sxl) / det;
            if (off > 0) { off = 0; s = sxl / sl2; }
            float err = 0;
            for (int i = 0; i < n; ++i) {
                const float r = s * (float)trial[i] + off - x[i];
                err += w[i] * (r * r);
            }
            if (err < err_best) {
                memcpy(L, trial, (size_t)n);
                err_best = err;
                scale = s;
                lo = off;
            }
        }
    }
    *neg_off = -lo;
    return scale;
}

/* The shared part of the q4_K / q5_K weight quantizers for one super-block
 * of 256 values: fit each 32-value sub-block (weights rms + |x|) to codes
 * 0..nmax, quantize the 8 scales and 8 mins to 6 bits against the largest of
 * each (packed as get_scale_min_k4 reads them), then re-derive every code
 * from the stored scales: L[e] = clamp(rne((x + dmin*m)/(d*sc)), 0, nmax). */
static void quantize_kblock(const float *x, int nmax, float rmin, float rdelta, int nstep, uint8_t scales[12],
                            uint16_t *d16, uint16_t *dmin16, uint8_t L[QK]) {
    uint8_t trial[32];
    float w[32], sc[8], mn[8];
    float sc_max = 0, mn_max = 0;
    for (int j = 0; j < 8; ++j) {
        float s2 = 0;
        for (int l = 0; l < 32; ++l) s2 += x[32 * j + l] * x[32 * j + l];
        const float rms = sqrtf(s2 / 32.0f);
        for (int l = 0; l < 32; ++l) w[l] = rms + fabsf(x[32 * j + l]);
        sc[j] = fit_asym(32, nmax, x + 32 * j, w, L + 32 * j, &mn[j], trial, rmin, rdelta, nstep);
        if (sc[j] > sc_max) sc_max = sc[j];
        if (mn[j] > mn_max) mn_max = mn[j];
    }
    const float isc = sc_max > 0 ? 63.0f / sc_max : 0.0f;
    const float imn = mn_max > 0 ? 63.0f / mn_max : 0.0f;
    memset(scales, 0, 12);
    for (int j = 0; j < 8; ++j) {
        int ls = rne_int(isc * sc[j]), lm = rne_int(imn * mn[j]);
        ls = ls > 63 ? 63 : ls;
        lm = lm > 63 ? 63 : lm;
        if (j < 4) {
            scales[j] = (uint8_t)ls;
            scales[j + 4] = (uint8_t)lm;
        } else {
            scales[j + 4] = (uint8_t)((ls & 15) | ((lm & 15) << 4));
            scales[j - 4] |= (uint8_t)((ls >> 4) << 6);
            scales[j] |= (uint8_t)((lm >> 4) << 6);
        }
    }
    *d16 = orc_fp32_to_fp16(sc_max / 63.0f);
    *dmin16 = orc_fp32_to_fp16(mn_max / 63.0f);
    for (int j = 0; j < 8; ++j) {
        int s6, m6;
        q4K_scale_min(j, scales, &s6, &m6);
        const float d = orc_fp16_to_fp32(*d16) * (float)s6;
        if (d == 0.0f) continue;
        const float dm = orc_fp16_to_fp32(*dmin16) * (float)m6;
        for (int l = 0; l < 32; ++l) {
            int q = rne_int((x[32 * j + l] + dm) / d);
            L[32 * j + l] = (uint8_t)(q < 0 ? 0 : (q > nmax ? nmax : q));
        }
    }
}

void orc_quantize_row_q4_K(const float *x, void *vy, int64_t k) {
    orc_q4K *y = (orc_q4K *)vy;
    uint8_t L[QK];
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        quantize_kblock(x, 15, -1.0f, 0.1f, 20, y[b].scales, &y[b].d, &y[b].dmin, L);
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l)
                y[b].qs[32 * g + l] = (uint8_t)(L[64 * g + l] | (L[64 * g + 32 + l] << 4));
    }
}

/* q5_K: the q4_K procedure with codes 0..31 (ggml's quantize_row_q5_K_ref);
 * the low 4 bits go to the nibbles as in q4_K, bit 4 of sub-block s's code
 * for element l to bit s of qh[l]. */
void orc_quantize_row_q5_K(const float *x, void *vy, int64_t k) {
    orc_q5K *y = (orc_q5K *)vy;
    uint8_t L[QK];
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        quantize_kblock(x, 31, -0.5f, 0.1f, 15, y[b].scales, &y[b].d, &y[b].dmin, L);
        memset(y[b].qh, 0, 32);
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) {
                const int a = L[64 * g + l], c = L[64 * g + 32 + l];
                y[b].qs[32 * g + l] = (uint8_t)((a & 15) | ((c & 15) << 4));
                y[b].qh[l] |= (uint8_t)(((a >> 4) << (2 * g)) | ((c >> 4) << (2 * g + 1)));
            }
    }
}

/* IQ4_XS test-weight quantizer (this oracle's own fit, not ggml's search):
 * per sub-block the scale s = max|x| / 113 (so both signs stay inside the
 * codebook's range -127..113), the block scale d = max s / 31 in fp16, the
 * stored ls = clamp(rne(s/d) + 32, 0, 63), and each value takes the codebook
 * entry nearest to x / (d*(ls-32)) (first index on ties). */
void orc_quantize_row_iq4_xs(const float *x, void *vy, int64_t k) {
    orc_iq4xs *y = (orc_iq4xs *)vy;
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        float s[8], smax = 0.0f;
        for (int ib = 0; ib < 8; ++ib) {
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[32 * ib + j]));
            s[ib] = amax / 113.0f;
            smax = fmaxf(smax, s[ib]);
        }
        memset(&y[b], 0, sizeof(orc_iq4xs));
        y[b].d = orc_fp32_to_fp16(smax / 31.0f);
        const float d = orc_fp16_to_fp32(y[b].d);
        for (int ib = 0; ib < 8; ++ib) {
            int ls = d > 0.0f ? rne_int(s[ib] / d) + 32 : 32;
            ls = ls < 0 ? 0 : (ls > 63 ? 63 : ls);
            y[b].scales_l[ib / 2] |= (uint8_t)((ls & 15) << (4 * (ib % 2)));
            y[b].scales_h |= (uint16_t)((ls >> 4) << (2 * ib));
            const float dl = d * (float)(ls - 32);
            for (int j = 0; j < 32; ++j) {
                int best = 0;
                if (dl != 0.0f) {
                    const float t = x[32 * ib + j] / dl;
                    float err = fabsf(t - (float)IQ4_VALUES[0]);
                    for (int c = 1; c < 16; ++c) {
                        const float e2 = fabsf(t - (float)IQ4_VALUES[c]);
                        if (e2 < err) { err = e2; best = c; }
                    }
                }
                uint8_t *q = y[b].qs + 16 * ib + (j & 15);
                *q |= (uint8_t)(j < 16 ? best : best << 4);
            }
        }
    }
}

/* f16 weights: round to nearest even. */
void orc_quantize_row_f16(const float *x, void *vy, int64_t k) {
    uint16_t *y = (uint16_t *)vy;
    for (int64_t i = 0; i < k; ++i) y[i] = orc_fp32_to_fp16(x[i]);
}

/* Symmetric fit of n values to signed codes -nmax..nmax-1 with weights x^2:
 * start from iscale = -nmax/m (m = signed value of largest magnitude), then
 * try iscale = -(nmax + 0.1*is)/m for is in -9..9 and keep the grid whose
 * least-squares scale maximises sum(w*x*l)^2 / sum(w*l^2).  Codes are stored
 * biased by +nmax.  (ggml's make_qx_quants with rmse_type 1.) */
static float fit_sym(int n, int nmax, const float *x, int8_t *L) {
    float amax = 0, m = 0;
    for (int i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > amax) { amax = a; m = x[i]; }
    }
    if (amax < 1e-15f) {
        memset(L, 0, (size_t)n);
        return 0.0f;
    }
    float inv = -(float)nmax / m;
    float slx = 0, sl2 = 0;
    for (int i = 0; i < n; ++i) {
        int l = rne_int(inv * x[i]);
        l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
        L[i] = (int8_t)(l + nmax);
        const float w = x[i] * x[i];
        slx += w * x[i] * (float)l;
        sl2 += w * (float)l * (float)l;
    }
    float scale = sl2 != 0.0f ? slx / sl2 : 0.0f;
    float best = scale * slx;
    for (int is = -9; is <= 9; ++is) {
        if (is == 0) continue;
        inv = -((float)nmax + 0.1f * (float)is) / m;
        slx = sl2 = 0;
        for (int i = 0; i < n; ++i) {
            int l = rne_int(inv * x[i]);
            l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
            const float w = x[i] * x[i];
            slx += w * x[i] * (float)l;
            sl2 += w * (float)l * (float)l;
        }
        if (sl2 > 0 && slx * slx > best * sl2) {
            for (int i = 0; i < n; ++i) {
                int l = rne_int(inv * x[i]);
                L[i] = (int8_t)(nmax + (l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l)));
            }
            scale = slx / sl2;
            best = scale * slx;
        }
    }
    return scale;
}

void orc_quantize_row_q6_K(const float *x, void *vy, int64_t k) {
    orc_q6K *y = (orc_q6K *)vy;
    int8_t L[QK];
    float sc[16];
    for (int64_t b = 0; b < k / QK; ++b, x += QK) {
        float sc_big = 0, sc_abs = 0;
        for (int g = 0; g < 16; ++g) {
            sc[g] = fit_sym(16, 32, x + 16 * g, L + 16 * g);
            if (fabsf(sc[g]) > sc_abs) { sc_abs = fabsf(sc[g]); sc_big = sc[g]; }
        }
        memset(&y[b], 0, sizeof(orc_q6K));
        if (sc_abs < 1e-15f) continue;
        const float inv = -128.0f / sc_big;
        y[b].d = orc_fp32_to_fp16(1.0f / inv);
        for (int g = 0; g < 16; ++g) {
            int s = rne_int(inv * sc[g]);
            y[b].scales[g] = (int8_t)(s > 127 ? 127 : s);
        }
        for (int g = 0; g < 16; ++g) {
            const float d = orc_fp16_to_fp32(y[b].d) * (float)y[b].scales[g];
            if (d == 0.0f) continue;
            for (int i = 0; i < 16; ++i) {
                int q = rne_int(x[16 * g + i] / d);
                q = q < -32 ? -32 : (q > 31 ? 31 : q);
                L[16 * g + i] = (int8_t)(q + 32);
            }
        }
        for (int half = 0; half < 2; ++half) {
            const int8_t *Lh = L + 128 * half;
            uint8_t *ql = y[b].ql + 64 * half, *qh = y[b].qh + 32 * half;
            for (int l = 0; l < 32; ++l) {
                const int a = Lh[l], c = Lh[l + 32], e = Lh[l + 64], f = Lh[l + 96];
                ql[l] = (uint8_t)((a & 15) | ((e & 15) << 4));
                ql[l + 32] = (uint8_t)((c & 15) | ((f & 15) << 4));
                qh[l] = (uint8_t)((a >> 4) | ((c >> 4) << 2) | ((e >> 4) << 4) | ((f >> 4) << 6));
            }
        }
    }
}

/* ---- dot products ------------------------------------------------------- */
/* Each super-block contributes exact integer sums combined in fp32:
 *   q4_K:   (d_w*d_x) * sum_s sc_s*<q4,q8>_s  -  (dmin_w*d_x) * sum_s m_s*bsum_s
 *   q5_K:   the same with 5-bit codes
 *   q6_K:   (d_w*d_x) * sum_g sc_g*<q6-32,q8>_g
 *   IQ4_XS: (d_w*d_x) * sum_ib (ls_ib-32)*<codebook[q],q8>_ib
 *   q8_0:   sum_b <qw,qx>_b * (d_w*d_x)
 * (ggml's generic code adds the per-sub-block terms in float; the integer
 * form is exact and differs from it only in fp32 rounding order.)
 */

float orc_vec_dot_q4_K_q8_K(int64_t n, const void *vx, const void *vy) {
    const orc_q4K *x = (const orc_q4K *)vx;
    const orc_q8K *y = (const orc_q8K *)vy;
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int32_t isum = 0, msum = 0;
        for (int s = 0; s < 8; ++s) {
            int sc, mn;
            q4K_scale_min(s, x[b].scales, &sc, &mn);
            const uint8_t *q = x[b].qs + 32 * (s / 2);
            const int8_t *a = y[b].qs + 32 * s;
            int32_t dot = 0;
            for (int l = 0; l < 32; ++l) dot += (int32_t)((s & 1) ? (q[l] >> 4) : (q[l] & 15)) * a[l];
            isum += sc * dot;
            msum += mn * (y[b].bsums[2 * s] + y[b].bsums[2 * s + 1]);
        }
        const float dx = y[b].d;
        acc += orc_fp16_to_fp32(x[b].d) * dx * (float)isum;
        acc -= orc_fp16_to_fp32(x[b].dmin) * dx * (float)msum;
    }
    return acc;
}

float orc_vec_dot_q5_K_q8_K(int64_t n, const void *vx, const void *vy) {
    const orc_q5K *x = (const orc_q5K *)vx;
    const orc_q8K *y = (const orc_q8K *)vy;
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int32_t isum = 0, msum = 0;
        for (int s = 0; s < 8; ++s) {
            int sc, mn;
            q4K_scale_min(s, x[b].scales, &sc, &mn);
            const uint8_t *q = x[b].qs + 32 * (s / 2);
            const int8_t *a = y[b].qs + 32 * s;
            int32_t dot = 0;
            for (int l = 0; l < 32; ++l) {
                const int v = ((s & 1) ? (q[l] >> 4) : (q[l] & 15)) + (((x[b].qh[l] >> s) & 1) << 4);
                dot += v * a[l];
            }
            isum += sc * dot;
            msum += mn * (y[b].bsums[2 * s] + y[b].bsums[2 * s + 1]);
        }
        const float dx = y[b].d;
        acc += orc_fp16_to_fp32(x[b].d) * dx * (float)isum;
        acc -= orc_fp16_to_fp32(x[b].dmin) * dx * (float)msum;
    }
    return acc;
}

float orc_vec_dot_iq4_xs_q8_K(int64_t n, const void *vx, const void *vy) {
    const orc_iq4xs *x = (const orc_iq4xs *)vx;
    const orc_q8K *y = (const orc_q8K *)vy;
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int32_t isum = 0;
        for (int ib = 0; ib < 8; ++ib) {
            const uint8_t *q = x[b].qs + 16 * ib;
            const int8_t *a = y[b].qs + 32 * ib;
            int32_t dot = 0;
            for (int j = 0; j < 16; ++j) dot += IQ4_VALUES[q[j] & 15] * a[j] + IQ4_VALUES[q[j] >> 4] * a[16 + j];
            isum += (iq4xs_ls(&x[b], ib) - 32) * dot;
        }
        acc += orc_fp16_to_fp32(x[b].d) * y[b].d * (float)isum;
    }
    return acc;
}

/* f16 weights . fp32 activations: x rounded to fp16 (ggml's vec_dot type for
 * f16), each product exact in fp32, summed in double. */
float orc_vec_dot_f16_f32(int64_t n, const void *vx, const float *x) {
    const uint16_t *w = (const uint16_t *)vx;
    double acc = 0.0;
    for (int64_t i = 0; i < n; ++i)
        acc += (double)(orc_fp16_to_fp32(w[i]) * orc_fp16_to_fp32(orc_fp32_to_fp16(x[i])));
    return (float)acc;
}

/* f32 weights . fp32 activations: fp32 products summed in double. */
float orc_vec_dot_f32_f32(int64_t n, const float *w, const float *x) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; ++i) acc += (double)(w[i] * x[i]);
    return (float)acc;
}

float orc_vec_dot_q6_K_q8_K(int64_t n, const void *vx, const void *vy) {
    const orc_q6K *x = (const orc_q6K *)vx;
    const orc_q8K *y = (const orc_q8K *)vy;
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int32_t isum = 0;
        for (int g = 0; g < 16; ++g) {
            int32_t dot = 0;
            for (int i = 0; i < 16; ++i) dot += q6K_code(&x[b], 16 * g + i) * y[b].qs[16 * g + i];
            isum += x[b].scales[g] * dot;
        }
        acc += orc_fp16_to_fp32(x[b].d) * y[b].d * (float)isum;
    }
    return acc;
}

float orc_vec_dot_q8_0_q8_0(int64_t n, const void *vx, const void *vy) {
    const orc_q80 *x = (const orc_q80 *)vx, *y = (const orc_q80 *)vy;
    float acc = 0.0f;
    for (int64_t b = 0; b < n / 32; ++b) {
        int32_t dot = 0;
        for (int i = 0; i < 32; ++i) dot += (int32_t)x[b].qs[i] * y[b].qs[i];
        acc += (float)dot * (orc_fp16_to_fp32(x[b].d) * orc_fp16_to_fp32(y[b].d));
    }
    return acc;
}

/* ---- whole-matrix drivers (OpenMP over rows) ---------------------------- */

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_IQ4_XS = 23 };

static size_t row_bytes(int type, int64_t k) {
    switch (type) {
    case ORC_F32: return (size_t)k * 4;
    case ORC_F16: return (size_t)k * 2;
    case ORC_Q4_K: return (size_t)(k / QK) * sizeof(orc_q4K);
    case ORC_Q5_K: return (size_t)(k / QK) * sizeof(orc_q5K);
    case ORC_Q6_K: return (size_t)(k / QK) * sizeof(orc_q6K);
    case ORC_IQ4_XS: return (size_t)(k / QK) * sizeof(orc_iq4xs);
    case ORC_Q8_0: return (size_t)(k / 32) * sizeof(orc_q80);
    default: return 0;
    }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* y[t*rows + r] = W[r] . x[t] for t < ntok: W has `rows` rows of k values in
 * ggml type `type`, x holds ntok activation rows quantized to q8_K (k-quants,
 * IQ4_XS) or q8_0 (q8_0 weights), or plain fp32 rows (f16 / f32 weights).
 * Returns 0 on success, -1 on a bad type. */
int orc_matvec(int type, const void *W, int64_t rows, int64_t k, const void *xq, int ntok,
               float *y, int nthreads) {
    const size_t rb = row_bytes(type, k);
    if (!rb) return -1;
    const size_t xb = type == ORC_Q8_0 ? (size_t)(k / 32) * sizeof(orc_q80)
                    : (type == ORC_F16 || type == ORC_F32) ? (size_t)k * 4
                                                            : (size_t)(k / QK) * sizeof(orc_q8K);
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t *w = (const uint8_t *)W + (size_t)r * rb;
        for (int t = 0; t < ntok; ++t) {
            const uint8_t *a = (const uint8_t *)xq + (size_t)t * xb;
            float v = 0.0f;
            switch (type) {
            case ORC_Q4_K: v = orc_vec_dot_q4_K_q8_K(k, w, a); break;
            case ORC_Q5_K: v = orc_vec_dot_q5_K_q8_K(k, w, a); break;
            case ORC_Q6_K: v = orc_vec_dot_q6_K_q8_K(k, w, a); break;
            case ORC_IQ4_XS: v = orc_vec_dot_iq4_xs_q8_K(k, w, a); break;
            case ORC_F16: v = orc_vec_dot_f16_f32(k, w, (const float *)a); break;
            case ORC_F32: v = orc_vec_dot_f32_f32(k, (const float *)w, (const float *)a); break;
            default: v = orc_vec_dot_q8_0_q8_0(k, w, a); break;
            }
            y[(size_t)t * rows + r] = v;
        }
    }
    return 0;
}

/* Quantize `rows` rows of k fp32 values to `type` (weights) in parallel. */
int orc_quantize_rows(int type, const float *x, int64_t rows, int64_t k, void *out, int nthreads) {
    const size_t rb = row_bytes(type, k);
    if (!rb) return -1;
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * k;
        void *o = (uint8_t *)out + (size_t)r * rb;
        switch (type) {
        case ORC_Q4_K: orc_quantize_row_q4_K(xr, o, k); break;
        case ORC_Q5_K: orc_quantize_row_q5_K(xr, o, k); break;
        case ORC_Q6_K: orc_quantize_row_q6_K(xr, o, k); break;
        case ORC_IQ4_XS: orc_quantize_row_iq4_xs(xr, o, k); break;
        case ORC_F16: orc_quantize_row_f16(xr, o, k); break;
        case ORC_F32: memcpy(o, xr, (size_t)k * 4); break;
        default: orc_quantize_row_q8_0(xr, o, k); break;
        }
    }
    return 0;
}

/* Dequantize `rows` rows of `type` into fp32. */
int orc_dequantize_rows(int type, const void *W, int64_t rows, int64_t k, float *y) {
    const size_t rb = row_bytes(type, k);
    if (!rb) return -1;
    for (int64_t r = 0; r < rows; ++r) {
        const void *w = (const uint8_t *)W + (size_t)r * rb;
        float *o = y + (size_t)r * k;
        switch (type) {
        case ORC_Q4_K: orc_dequantize_row_q4_K(w, o, k); break;
        case ORC_Q5_K: orc_dequantize_row_q5_K(w, o, k); break;
        case ORC_Q6_K: orc_dequantize_row_q6_K(w, o, k); break;
        case ORC_IQ4_XS: orc_dequantize_row_iq4_xs(w, o, k); break;
        case ORC_F16: orc_dequantize_row_f16(w, o, k); break;
        case ORC_F32: memcpy(o, w, (size_t)k * 4); break;
        default: orc_dequantize_row_q8_0(w, o, k); break;
        }
    }
    return 0;
}

/* Index of the largest value, ties to the smallest index. */
int64_t orc_argmax(const float *v, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return n > 0 ? best : -1;
}

/* ---- vectorised q4_K . q8_K (the timed CPU baseline) -------------------- *
 * ggml's x86 builds replace the generic vec_dot_q4_K_q8_K with SIMD code:
 * the AVX2 form multiplies the unsigned 4-bit codes by the signed q8 codes
 * with vpmaddubsw (pairs of u8*s8 summed to s16; at most 2*15*128 = 3840, no
 * saturation), widens with vpmaddwd against the sub-block's 6-bit scale, and
 * sums in int32; with AVX-512 VNNI, vpdpbusd does the u8*s8 products and the
 * sum of four in one instruction.  The restatements below follow that
 * instruction mapping, compute the same exact int32 sums (sum_s sc*dot and
 * sum_s m*bsum) as orc_vec_dot_q4_K_q8_K, and combine them into the fp32
 * accumulator in the same order, so their results equal the scalar oracle's
 * bit for bit (the CPU tests check this).  They are only the CPU baseline;
 * the scalar function stays the checker. */
#if defined(__x86_64__)
#include <immintrin.h>

/* All eight 6-bit scales and mins at once, one byte each (the same values
 * q4K_scale_min gives, from three little-endian words of the packed bytes). */
static void q4K_unpack8(const uint8_t *s, int sc[8], int mn[8]) {
    uint32_t w0, w1, w2;
    memcpy(&w0, s, 4);
    memcpy(&w1, s + 4, 4);
    memcpy(&w2, s + 8, 4);
    const uint32_t sc03 = w0 & 0x3f3f3f3fu, mn03 = w1 & 0x3f3f3f3fu;
    const uint32_t sc47 = (w2 & 0x0f0f0f0fu) | ((w0 >> 2) & 0x30303030u);
    const uint32_t mn47 = ((w2 >> 4) & 0x0f0f0f0fu) | ((w1 >> 2) & 0x30303030u);
    for (int j = 0; j < 4; ++j) {
        sc[j] = (int)((sc03 >> (8 * j)) & 0xff);
        mn[j] = (int)((mn03 >> (8 * j)) & 0xff);
        sc[j + 4] = (int)((sc47 >> (8 * j)) & 0xff);
        mn[j + 4] = (int)((mn47 >> (8 * j)) & 0xff);
    }
}

/* fp16 -> fp32 with the F16C instruction (exact, as orc_fp16_to_fp32). */
__attribute__((target("f16c")))
static inline float h2f_f16c(uint16_t h) { return _cvtsh_ss(h); }

__attribute__((target("avx2,fma,f16c")))
static float dot_q4K_avx2(int64_t n, const orc_q4K *x, const orc_q8K *y) {
    const __m256i m4 = _mm256_set1_epi8(0x0f);
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int sc[8], mn[8];
        q4K_unpack8(x[b].scales, sc, mn);
        __m256i vs = _mm256_setzero_si256();
        for (int g = 0; g < 4; ++g) {
            const __m256i q = _mm256_loadu_si256((const __m256i *)(x[b].qs + 32 * g));
            const __m256i lo = _mm256_and_si256(q, m4);
            const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(q, 4), m4);
            const __m256i a0 = _mm256_loadu_si256((const __m256i *)(y[b].qs + 64 * g));
            const __m256i a1 = _mm256_loadu_si256((const __m256i *)(y[b].qs + 64 * g + 32));
            const __m256i p0 = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, a0), _mm256_set1_epi16((short)sc[2 * g]));
            const __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, a1), _mm256_set1_epi16((short)sc[2 * g + 1]));
            vs = _mm256_add_epi32(vs, _mm256_add_epi32(p0, p1));
        }
        __m128i h = _mm_add_epi32(_mm256_castsi256_si128(vs), _mm256_extracti128_si256(vs, 1));
        h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0x4e));
        h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0xb1));
        const int32_t isum = _mm_cvtsi128_si32(h);
        int32_t msum = 0;
        for (int s = 0; s < 8; ++s) msum += mn[s] * (y[b].bsums[2 * s] + y[b].bsums[2 * s + 1]);
        const float dx = y[b].d;
        acc += h2f_f16c(x[b].d) * dx * (float)isum;
        acc -= h2f_f16c(x[b].dmin) * dx * (float)msum;
    }
    return acc;
}

__attribute__((target("avx512f,avx512bw,avx512vl,avx512vnni,f16c")))
static float dot_q4K_vnni(int64_t n, const orc_q4K *x, const orc_q8K *y) {
    const __m256i m4 = _mm256_set1_epi8(0x0f);
    float acc = 0.0f;
    for (int64_t b = 0; b < n / QK; ++b) {
        int sc[8], mn[8];
        q4K_unpack8(x[b].scales, sc, mn);
        __m512i vs = _mm512_setzero_si512();
        for (int g = 0; g < 4; ++g) {
            /* sub-blocks 2g (low nibbles) and 2g+1 (high nibbles) against the
             * 64 contiguous q8 codes of those two sub-blocks */
            const __m256i q = _mm256_loadu_si256((const __m256i *)(x[b].qs + 32 * g));
            const __m512i codes = _mm512_inserti64x4(_mm512_castsi256_si512(_mm256_and_si256(q, m4)),
                                                     _mm256_and_si256(_mm256_srli_epi16(q, 4), m4), 1);
            const __m512i a = _mm512_loadu_si512((const void *)(y[b].qs + 64 * g));
            const __m512i dot = _mm512_dpbusd_epi32(_mm512_setzero_si512(), codes, a);
            const __m512i scv = _mm512_inserti64x4(_mm512_set1_epi32(sc[2 * g]), _mm256_set1_epi32(sc[2 * g + 1]), 1);
            vs = _mm512_add_epi32(vs, _mm512_mullo_epi32(dot, scv));
        }
        const int32_t isum = _mm512_reduce_add_epi32(vs);
        int32_t msum = 0;
        for (int s = 0; s < 8; ++s) msum += mn[s] * (y[b].bsums[2 * s] + y[b].bsums[2 * s + 1]);
        const float dx = y[b].d;
        acc += h2f_f16c(x[b].d) * dx * (float)isum;
        acc -= h2f_f16c(x[b].dmin) * dx * (float)msum;
    }
    return acc;
}
#endif

/* The instruction set orc_matvec_q4K_simd uses on this CPU: 2 = AVX-512
 * VNNI, 1 = AVX2, 0 = none (it then calls the scalar function). */
int orc_simd_level(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") &&
        __builtin_cpu_supports("avx512vl"))
        return 2;
    if (__builtin_cpu_supports("avx2")) return 1;
#endif
    return 0;
}

/* orc_matvec for q4_K weights with the vectorised dot product (level from
 * orc_simd_level(), or a lower one if `level` is smaller).  Returns the level
 * used. */
int orc_matvec_q4K_simd(const void *W, int64_t rows, int64_t k, const void *xq, int ntok, float *y, int nthreads,
                        int level) {
    int lv = orc_simd_level();
    if (level >= 0 && level < lv) lv = level;
    const size_t rb = row_bytes(ORC_Q4_K, k), xb = (size_t)(k / QK) * sizeof(orc_q8K);
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const orc_q4K *w = (const orc_q4K *)((const uint8_t *)W + (size_t)r * rb);
        for (int t = 0; t < ntok; ++t) {
            const orc_q8K *a = (const orc_q8K *)((const uint8_t *)xq + (size_t)t * xb);
            float v;
#if defined(__x86_64__)
            if (lv == 2) v = dot_q4K_vnni(k, w, a);
            else if (lv == 1) v = dot_q4K_avx2(k, w, a);
            else
#endif
                v = orc_vec_dot_q4_K_q8_K(k, w, a);
            y[(size_t)t * rows + r] = v;
        }
    }
    return lv;
}
