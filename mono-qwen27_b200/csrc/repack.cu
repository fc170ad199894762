// repack.cu — load-time planar repack of q6_K / q8_0 rows, and bit-exact
// row dequantization (the embedding gather).
//
// GGUF q6_K blocks are 210 bytes and q8_0 blocks 34 bytes, so their fields
// are only 2-byte aligned and cannot be streamed with 128-bit loads or TMA.
// The repack is a lossless rearrangement of each row:
//   q6_K: ceil(rb/4) tiles of 848 bytes, tile t holding blocks 4t..4t+3 as
//         ql[4][128] | qh[4][64] | scales[4][16] | d[4] (fp16 + 2 zero bytes);
//         blocks past the end of the row are zero (4240 vs 4200 bytes for a
//         K=5120 row, 14416 vs 14280 for K=17408);
//   q8_0: [qs rb*32 | d rb*2 | zero pad to 16] (0 extra bytes for rows of
//         32k values).
//
// Dequant follows ggml's dequantize_row_q4_K / q6_K / q8_0 (as restated in
// debug/official_dequant.c:47-65 and src/mono27b_executor.cu:1026-1048,
// :1233-1254) with explicitly rounded multiplies and subtractions, so the
// result is fl(fl(d*sc)*q) - fl(dmin*m) without fused multiply-adds: bit-exact
// against the CPU restatement compiled with -ffp-contract=off.
#include "m27b_device.cuh"
#include "m27b_launch.cuh"

namespace m27b {

size_t planar_row_bytes(int type, int rb) {
    if (type == M27B_TYPE_Q6_K) return (size_t)((rb + 3) / 4) * 848;
    if (type == M27B_TYPE_Q8_0) return (size_t)rb * 32 + (((size_t)rb * 2 + 15) & ~(size_t)15);
    return 0;
}

// grid (rb, rows), block 64: one block of one row per CTA (the output was
// zeroed first, so padding blocks and pad bytes stay zero).
__global__ void k_repack_q6K(const uint8_t *raw, uint8_t *out, int rb, size_t out_row) {
    const int b = blockIdx.x;
    const size_t r = blockIdx.y;
    const uint8_t *src = raw + (r * rb + b) * 210;
    uint8_t *tile = out + r * out_row + (size_t)(b >> 2) * 848;
    const int j = b & 3;
    for (int i = threadIdx.x; i < 210; i += blockDim.x) {
        const uint8_t v = src[i];
        if (i < 128) tile[j * 128 + i] = v;
        else if (i < 192) tile[512 + j * 64 + (i - 128)] = v;
        else if (i < 208) tile[768 + j * 16 + (i - 192)] = v;
        else tile[832 + j * 4 + (i - 208)] = v;
    }
}

__global__ void k_repack_q80(const uint8_t *raw, uint8_t *out, int rb, size_t out_row) {
    const int b = blockIdx.x;
    const size_t r = blockIdx.y;
    const uint8_t *src = raw + (r * rb + b) * 34;
    uint8_t *dst = out + r * out_row;
    for (int i = threadIdx.x; i < 34; i += blockDim.x) {
        const uint8_t v = src[i];
        if (i < 2) dst[(size_t)rb * 32 + (size_t)b * 2 + i] = v;
        else dst[(size_t)b * 32 + (i - 2)] = v;
    }
    if (b == rb - 1) {
        for (size_t i = (size_t)rb * 34 + threadIdx.x; i < out_row; i += blockDim.x) dst[i] = 0;
    }
}

cudaError_t launch_repack(int type, const void *raw, int rb, int rows, void *out, cudaStream_t st) {
    const size_t orow = planar_row_bytes(type, rb);
    if (type == M27B_TYPE_Q6_K) {
        cudaError_t e = cudaMemsetAsync(out, 0, orow * (size_t)rows, st);
        if (e != cudaSuccess) return e;
    }
    // grid.y is limited to 65535: walk the rows in slices.
    for (int r0 = 0; r0 < rows; r0 += 65535) {
        const int n = rows - r0 < 65535 ? rows - r0 : 65535;
        dim3 grid(rb, n);
        if (type == M27B_TYPE_Q6_K)
            k_repack_q6K<<<grid, 64, 0, st>>>((const uint8_t *)raw + (size_t)r0 * rb * 210, (uint8_t *)out + (size_t)r0 * orow,
                                              rb, orow);
        else
            k_repack_q80<<<grid, 64, 0, st>>>((const uint8_t *)raw + (size_t)r0 * rb * 34, (uint8_t *)out + (size_t)r0 * orow, rb,
                                              orow);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------------------
// Row dequantization.  grid (ceil(k/256), n), block 256: thread j of CTA bx
// writes value 256*bx + j of row rows[blockIdx.y].
struct DequantArgs {
    const uint8_t *w;
    const int32_t *rows;
    float *out;
    int ldo;
    int rb;
    int row_count;
    int k;
    int type;      // base ggml type
    bool planar;   // q6_K / q8_0 planar layout
    size_t row_stride;
};

M27B_DI float dq_q4K(const uint8_t *row, int e) {
    const m27b_block_q4_K *blk = (const m27b_block_q4_K *)row + (e >> 8);
    const int i = e & 255, g = i >> 6, within = i & 63, j = 2 * g + (within >> 5), l = within & 31;
    const uint8_t *s = blk->scales;
    int sc, mn;
    if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
    else { sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
    const uint8_t qb = blk->qs[32 * g + l];
    const int q = (within < 32) ? (qb & 15) : (qb >> 4);
    const float d = __half2float(__ushort_as_half(blk->d)), dmin = __half2float(__ushort_as_half(blk->dmin));
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
}

M27B_DI float dq_q6K(const uint8_t *row, int rb, int e, bool planar) {
    const int b = e >> 8, i = e & 255, half = i >> 7, r = (i & 127) >> 5, l = i & 31;
    const uint8_t *ql, *qh;
    int8_t sc;
    uint16_t dbits;
    if (planar) {
        const uint8_t *tile = row + (size_t)(b >> 2) * 848;
        const int j = b & 3;
        ql = tile + j * 128 + 64 * half;
        qh = tile + 512 + j * 64 + 32 * half;
        sc = (int8_t)tile[768 + j * 16 + (i >> 4)];
        dbits = (uint16_t)(tile[832 + j * 4] | (tile[832 + j * 4 + 1] << 8));
    } else {
        const uint8_t *blk = row + (size_t)b * 210;
        ql = blk + 64 * half;
        qh = blk + 128 + 32 * half;
        sc = (int8_t)blk[192 + (i >> 4)];
        dbits = (uint16_t)(blk[208] | (blk[209] << 8));
    }
    int lo = (r & 1) ? ql[l + 32] : ql[l];
    lo = (r & 2) ? (lo >> 4) : (lo & 15);
    const int q = (lo | (((qh[l] >> (2 * r)) & 3) << 4)) - 32;
    const float d = __half2float(__ushort_as_half(dbits));
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

M27B_DI float dq_q80(const uint8_t *row, int rb, int e, bool planar) {
    const int b = e >> 5, i = e & 31;
    int8_t q;
    uint16_t dbits;
    if (planar) {
        q = (int8_t)row[(size_t)b * 32 + i];
        dbits = (uint16_t)(row[(size_t)rb * 32 + 2 * b] | (row[(size_t)rb * 32 + 2 * b + 1] << 8));
    } else {
        const uint8_t *blk = row + (size_t)b * 34;
        q = (int8_t)blk[2 + i];
        dbits = (uint16_t)(blk[0] | (blk[1] << 8));
    }
    return __fmul_rn((float)q, __half2float(__ushort_as_half(dbits)));
}

__global__ void __launch_bounds__(256) k_dequant_rows(DequantArgs a) {
    const int e = blockIdx.x * 256 + threadIdx.x;
    if (e >= a.k) return;
    const int r = a.rows[blockIdx.y];
    float v = 0.0f;
    if (r >= 0 && r < a.row_count) {
        const uint8_t *row = a.w + (size_t)r * a.row_stride;
        if (a.type == M27B_TYPE_Q4_K) v = dq_q4K(row, e);
        else if (a.type == M27B_TYPE_Q6_K) v = dq_q6K(row, a.rb, e, a.planar);
        else v = dq_q80(row, a.rb, e, a.planar);
    }
    a.out[(size_t)blockIdx.y * a.ldo + e] = v;
}

cudaError_t launch_dequant_rows(int type, bool planar, const void *w, size_t row_stride, int rb, int row_count, int k,
                                const int32_t *rows, int n, float *out, int ldo, cudaStream_t st) {
    DequantArgs a;
    a.w = (const uint8_t *)w;
    a.rows = rows;
    a.out = out;
    a.ldo = ldo;
    a.rb = rb;
    a.row_count = row_count;
    a.k = k;
    a.type = type;
    a.planar = planar;
    a.row_stride = row_stride;
    for (int i0 = 0; i0 < n; i0 += 65535) {
        const int m = n - i0 < 65535 ? n - i0 : 65535;
        DequantArgs s = a;
        s.rows = rows + i0;
        s.out = out + (size_t)i0 * ldo;
        k_dequant_rows<<<dim3((k + 255) / 256, m), 256, 0, st>>>(s);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace m27b
