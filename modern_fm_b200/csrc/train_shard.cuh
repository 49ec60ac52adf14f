// train_shard.cuh — kernels of parameter-sharded multi-GPU FM training (the
// binary-FM row-table path over a data-parallel group).
//
// Rank r of N owns the keys i with i mod N = r (interleaved, so that a few
// keys present in every row, such as dense numeric features at the low ids,
// spread over the ranks): their parameters and optimizer state are stepped
// on that rank only. Every rank
// sees every row of every batch (the reference's mini-batch semantics,
// rust/src/fm.rs:373-411), but only its own keys' entries: the rank's CSR is
// the training CSR restricted to its key range. Per batch the forward writes
// each row's sums over the rank's keys, [S_r | lin_r - sq_r / 2]; one sum over
// the ranks gives S and the score s = w0 + sum_r (lin_r - sq_r / 2) + |S|^2 / 2
// (the same quantities as train_score_row, fm.rs:77-101, summed in a different
// order), from which every rank forms the same loss gradient g; stage 1 then
// steps the rank's own keys exactly as on one GPU. The only per-batch exchange
// is the row table (rows x (k + 1) values), whatever the number of touched
// keys: read from the other ranks' memory by the forward itself, block by
// block, or summed by one NCCL allreduce (the fallback).
#pragma once

#include "train_forward.cuh"
#include "train_tab.cuh"

namespace mfm {

// Per row: the number of its entries whose key i has i mod N = r. One warp
// per row. cnt[row] for row in [0, n_rows).
__global__ void __launch_bounds__(256)
    shard_count_kernel(const int64_t* __restrict__ indptr, const int32_t* __restrict__ indices,
                       int64_t n_rows, int N, int r, int64_t* __restrict__ cnt) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row], e = indptr[row + 1];
        int64_t n = 0;
        for (int64_t q = b + lane; q < e; q += 32) {
            n += (indices[q] % N == r) ? 1 : 0;
        }
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
        if (lane == 0) cnt[row] = n;
    }
}

// The rank's entries of each row, in the row's order, at sub_indptr[row].
template <class T>
__global__ void __launch_bounds__(256)
    shard_copy_kernel(const int64_t* __restrict__ indptr, const int32_t* __restrict__ indices,
                      const T* __restrict__ data, int64_t n_rows, int N, int r,
                      const int64_t* __restrict__ sub_indptr, int32_t* __restrict__ sub_indices,
                      T* __restrict__ sub_data) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row], e = indptr[row + 1];
        int64_t o = sub_indptr[row];
        for (int64_t q0 = b; q0 < e; q0 += 32) {
            const int64_t q = q0 + lane;
            const int32_t i = q < e ? indices[q] : -1;
            const bool mine = q < e && i % N == r;
            const unsigned m = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                const int64_t at = o + __popc(m & ((1u << lane) - 1u));
                sub_indices[at] = i;
                sub_data[at] = data[q];
            }
            o += __popc(m);
        }
    }
}

// Zeroes the keys this rank does not own in a (n_keys, width) array, so that
// one sum over the ranks gives every key its owner's values.
template <class T>
__global__ void shard_zero_unowned_kernel(T* __restrict__ a, int64_t n_keys, int64_t width,
                                          int N, int r) {
    const int64_t n = n_keys * width;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n;
         q += (int64_t)gridDim.x * blockDim.x)
        if ((q / width) % N != r) a[q] = T(0);
}

// After the cross-rank sum of the partial row table (stride PW >= k + 1):
// S to the stage-1 row table (stride k), the score and g = loss'(s) x
// sample_weight to grow (optimizer.rs:38-43). y and sw are in epoch order
// (pos0 = the batch's first epoch position). Thread 0 also records the
// batch in the group's progress word (the host's liveness view).
template <class T, int VEC, int NV>
__global__ void __launch_bounds__(256)
    fm_shard_finish_kernel(const T* __restrict__ part, int PW, T* __restrict__ tab,
                           T* __restrict__ grow, const T* __restrict__ y,
                           const T* __restrict__ sw, int64_t pos0, int64_t nrows,
                           const T* __restrict__ w0, int loss, unsigned* progress,
                           unsigned step) {
    constexpr int K = VEC * NV;
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j == 0 && progress) *(volatile unsigned*)progress = step;
    if (j >= nrows) return;
    const T* pr = part + j * PW;
    T ss = T(0);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const Vec<T, VEC> sv = *reinterpret_cast<const Vec<T, VEC>*>(pr + v * VEC);
        *reinterpret_cast<Vec<T, VEC>*>(tab + j * K + v * VEC) = sv;
#pragma unroll
        for (int u = 0; u < VEC; ++u) ss += sv.v[u] * sv.v[u];
    }
    const T s = w0[0] + (pr[K] + T(0.5) * ss);
    const T yy = y[pos0 + j];
    grow[j] = sw[pos0 + j] * (loss == MFM_LOSS_LOGISTIC ? sigmoid_t(s) - yy : s - yy);
}

// ------------------------------------------------- peer-memory exchange --

// Layout of each rank's exchange buffer: the failure word at byte 0, the
// forward's per-block flags (the exchange number each block has published)
// from kDpFlagsOffset, the two partial row tables from kDpDataOffset. The
// exchange itself runs at the end of the forward (shard_block_exchange).
constexpr size_t kDpFlagsOffset = 256;
constexpr int kDpMaxBlocks = 4096;
constexpr size_t kDpDataOffset = kDpFlagsOffset + 8 * (size_t)kDpMaxBlocks;

}  // namespace mfm
