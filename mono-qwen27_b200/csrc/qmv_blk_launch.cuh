// qmv_blk_launch.cuh — launch the block-per-lane k-quant matvec (qmv_blk.cuh)
// for one block type: grid shape, shared memory, tensor maps.
#pragma once

#include "qmv_blk.cuh"
#include "m27b_launch.cuh"
#include "qmv_launch.cuh"

namespace m27b {

template <class BT, int NT, int EPI>
inline auto blk_kernel() {
    if constexpr (BT::BYTES == BlkQ4K::BYTES) return k_qmv_q4k_blk<NT, EPI>;
    else if constexpr (BT::BYTES == BlkQ5K::BYTES) return k_qmv_q5k_blk<NT, EPI>;
    else return k_qmv_iq4xs_blk<NT, EPI>;
}

template <class BT, int NT, int EPI>
cudaError_t run_blk(const QmvArgs &a, int sm_count, cudaStream_t st) {
    auto kern = blk_kernel<BT, NT, EPI>();
    const int nw = blk_warps(a.k, NT, BT::BYTES);
    if (nw < 1) return cudaErrorInvalidValue;
    const size_t smem = blk_smem_bytes(a.k, NT, BT::BYTES);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static size_t opted[64] = {0};
    if (smem > 48 * 1024 && (dev >= 64 || smem > opted[dev])) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) opted[dev] = smem;
    }
    // BLK_CTAS resident CTAs per SM by construction (shared memory <= BLK_SMEM_MAX each)
    const long groups = (a.rows + 7) / 8;
    const int P = (a.rb + 3) / 4;
    const long slots = (long)sm_count * BLK_CTAS;
    int split, nthreads, nst = BLK_STAGES;
    long grid;
    size_t smem_launch;
    // few row groups: one warp per group, every item of the group in flight
    // from the start (a stage per item), the warps spread over all SMs —
    // while that fits the shared memory the kernel is opted in for
    const int items = P * (EPI == EPI_SWIGLU ? 2 : 1);
    const long wpc = (groups + sm_count - 1) / sm_count;  // warps per CTA
    const bool all_in_flight = !(2 * groups >= slots * nw || P < 2) && groups >= 2L * sm_count &&
                               items <= BLK_MAX_STAGES && wpc <= nw &&
                               blk_smem_for((int)wpc, a.k, NT, BT::BYTES, items) <= smem;
    if (2 * groups >= slots * nw || P < 2) {
        // every warp streams whole row groups, one CTA per resident slot
        // (fewer only for a one-pass matrix with fewer groups than slots);
        // the kernel deals the groups warp-major, so the CTAs (and SMs)
        // differ by at most one group per warp index
        split = 1;
        grid = groups < slots ? groups : slots;
        nthreads = nw * 32;
        smem_launch = smem;
    } else if (all_in_flight) {
        split = 1;
        nst = items;
        grid = sm_count;
        nthreads = (int)wpc * 32;
        smem_launch = blk_smem_for((int)wpc, a.k, NT, BT::BYTES, nst);
    } else {
        // few row groups: the warps of a CTA split each group's passes
        split = P < nw ? P : nw;
        // one CTA per resident slot — two per SM while a CTA has at most 8
        // warps (registers and shared memory hold two); CTA c takes groups
        // c, c + grid, ...: the CTAs an SM holds then carry (nearly) the
        // same number of groups, and the SMs differ by at most one group
        const long split_slots = (long)sm_count * (split <= 8 ? 2 : 1);
        grid = groups < split_slots ? groups : split_slots;
        nthreads = split * 32;
        smem_launch = blk_smem_for(split, a.k, NT, BT::BYTES);
    }
    // box: 8 rows x 4 blocks (BT::BYTES uint32 words)
    CUtensorMap tm0, tm1;
    if (!encode_rows_u32(&tm0, a.w0, a.row_stride, a.rows, BT::BYTES)) return cudaErrorInvalidValue;
    if (EPI == EPI_SWIGLU) {
        if (!encode_rows_u32(&tm1, a.w1, a.row_stride, a.rows, BT::BYTES)) return cudaErrorInvalidValue;
    } else {
        tm1 = tm0;
    }
    return launch_pdl(kern, dim3((unsigned)grid), dim3(nthreads), smem_launch, st, a, tm0, tm1, split, nst);
}

template <class BT, int EPI>
cudaError_t run_blk_nt(int nt, const QmvArgs &a, int sm_count, cudaStream_t st) {
    switch (nt) {
    case 1: return run_blk<BT, 1, EPI>(a, sm_count, st);
    case 2: return run_blk<BT, 2, EPI>(a, sm_count, st);
    case 3: return run_blk<BT, 3, EPI>(a, sm_count, st);
    case 4: return run_blk<BT, 4, EPI>(a, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace m27b
