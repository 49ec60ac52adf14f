// train_plan.cuh — per-epoch planning kernels of the training path: parameter
// layout moves, entry counts, expansion of rows into keyed entries, run and
// work-item tables, and the data-parallel run tables.
#pragma once

#include "train_opt.cuh"

namespace mfm {

// --------------------------------------------------------- layout moves --

// src (C, R, K) float64 row-major <-> dst (R, C, K) in T: the device keeps
// every key's classes contiguous (one gather per key); C = 1 is a plain copy.
template <class T>
__global__ void to_device_layout(const double* __restrict__ src, T* __restrict__ dst,
                                 int64_t C, int64_t R, int64_t K) {
    const int64_t total = C * R * K, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / (C * K), rem = i - r * C * K, c = rem / K, kk = rem - c * K;
        dst[i] = (T)src[(c * R + r) * K + kk];
    }
}
template <class T>
__global__ void from_device_layout(const T* __restrict__ src, double* __restrict__ dst,
                                   int64_t C, int64_t R, int64_t K) {
    const int64_t total = C * R * K, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / (C * K), rem = i - r * C * K, c = rem / K, kk = rem - c * K;
        dst[(c * R + r) * K + kk] = (double)src[i];
    }
}
template <class Tin, class Tout>
__global__ void convert_kernel(const Tin* __restrict__ src, Tout* __restrict__ dst, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = (Tout)src[i];
}

// ------------------------------------------------------- epoch planning --

__device__ __forceinline__ int64_t stream_count(int kind, int64_t z) {
    return kind == FEAT ? z : (kind == SLOT ? z * (z - 1) : z * (z - 1) / 2);
}

__global__ void count_kernel(int kind, const int32_t* __restrict__ order,
                             const int64_t* __restrict__ indptr, int64_t n_rows,
                             int64_t* __restrict__ cnt) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows) return;
    const int64_t row = order[i];
    cnt[i] = stream_count(kind, indptr[row + 1] - indptr[row]);
}

// y and sample weight in epoch order (row-table path: the forward reads rows
// by epoch position).
template <class T>
__global__ void permute_rows_kernel(const int32_t* __restrict__ order, const T* __restrict__ y,
                                    const T* __restrict__ sw, int64_t n_rows, T* __restrict__ py,
                                    T* __restrict__ psw) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows) return;
    const int64_t row = order[i];
    py[i] = y[row];
    psw[i] = sw[row];
}

__global__ void seg_lo_kernel(const int64_t* __restrict__ estart, int64_t n_rows, int64_t B,
                              int64_t nb, int64_t* __restrict__ seg_lo) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b > nb) return;
    const int64_t pos = b * B < n_rows ? b * B : n_rows;
    seg_lo[b] = estart[pos];
}

__device__ __forceinline__ void pair_step(int64_t& a, int64_t& b, int64_t z) {
    while (a < z - 1 && b >= z) {
        b = b - z + a + 2;
        ++a;
    }
}

// One warp per epoch position: writes the keys and batch-local entry ids of
// the row's entries, in the order the forward kernel writes their payloads.
// With erx set (FEAT only), instead of the ids (vals = nullptr: the sort
// generates them), each entry's value in epoch order (ex) and its (batch-local
// row, value) record (erx), for the row-table reduction.
template <class T>
__global__ void __launch_bounds__(256)
    expand_kernel(int kind, const int32_t* __restrict__ order, const int64_t* __restrict__ indptr,
                  const int32_t* __restrict__ indices, const int32_t* __restrict__ fid, int F,
                  int64_t pos_lo, int64_t pos_hi, int64_t B, const int64_t* __restrict__ estart,
                  const int64_t* __restrict__ seg_lo, uint32_t* __restrict__ keys,
                  uint32_t* __restrict__ vals, const T* __restrict__ data,
                  RowVal<T>* __restrict__ erx, T* __restrict__ ex) {
    // (FEAT with erx: keys[] is kept unsorted as the epoch-order CSR indices)
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t pos = pos_lo + (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
         pos < pos_hi; pos += nwarps) {
        const int64_t row = order[pos];
        const int64_t rb = indptr[row], z = indptr[row + 1] - rb;
        const int32_t* ix = indices + rb;
        const int64_t base = estart[pos];
        const int64_t local = base - seg_lo[pos / B];
        if (kind == FEAT) {
            const uint32_t rib = (uint32_t)(pos % B);
            for (int64_t a = lane; a < z; a += 32) {
                keys[base + a] = (uint32_t)ix[a];
                if (vals) vals[base + a] = (uint32_t)(local + a);
                if (erx) {
                    const T xv = data[rb + a];
                    erx[base + a] = RowVal<T>{rib, xv};
                    ex[base + a] = xv;
                }
            }
        } else if (kind == SLOT) {  // ordered pairs (a, b != a): key = i_a * F + f_b
            const int64_t tot = z * (z - 1);
            for (int64_t q = lane; q < tot; q += 32) {
                const int64_t a = q / (z - 1), bi = q - a * (z - 1), b = bi < a ? bi : bi + 1;
                keys[base + q] = (uint32_t)((int64_t)ix[a] * F + fid[ix[b]]);
                vals[base + q] = (uint32_t)(local + q);
            }
        } else {  // unordered pairs a < b: key = pair_slot(f_a, f_b)
            int64_t a = 0, b = 1 + lane, pi = lane;
            pair_step(a, b, z);
            while (a < z - 1) {
                const int fa = fid[ix[a]], fb = fid[ix[b]];
                keys[base + pi] = (uint32_t)(fa <= fb ? fa * F + fb : fb * F + fa);
                vals[base + pi] = (uint32_t)(local + pi);
                b += 32;
                pi += 32;
                pair_step(a, b, z);
            }
        }
    }
}

__global__ void head_kernel(const uint32_t* __restrict__ keys, int64_t n,
                            int32_t* __restrict__ head) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p < n) head[p] = (p == 0 || keys[p] != keys[p - 1]) ? 1 : 0;
}
__global__ void seg_head_kernel(const int64_t* __restrict__ seg_lo, int64_t nb,
                                int32_t* __restrict__ head) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b < nb && seg_lo[b] < seg_lo[b + 1]) head[seg_lo[b]] = 1;
}
__global__ void run_start_kernel(const int32_t* __restrict__ head,
                                 const int64_t* __restrict__ run_id, int64_t n,
                                 int64_t* __restrict__ run_start) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p < n && head[p]) run_start[run_id[p]] = p;
    if (p == 0) run_start[run_id[n]] = n;
}
__global__ void pieces_kernel(const int64_t* __restrict__ run_start, int64_t R,
                              int64_t* __restrict__ np, int64_t* __restrict__ longf) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int64_t c = ceil_div(run_start[r + 1] - run_start[r], kItem);
    np[r] = c;
    longf[r] = c > 1 ? 1 : 0;
}
__global__ void items_kernel(const int64_t* __restrict__ item_start,
                             const int64_t* __restrict__ long_scan, int64_t R,
                             int64_t* __restrict__ item_run, int64_t* __restrict__ long_list) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int64_t i0 = item_start[r], i1 = item_start[r + 1];
    for (int64_t i = i0; i < i1; ++i) item_run[i] = r;
    if (i1 - i0 > 1) long_list[long_scan[r]] = r;
}
// One 16-byte descriptor per work item: first sorted entry (epoch index),
// entry count (bit 31 set when the run has several items) and key.
struct ItemDesc {
    int64_t p0;
    uint32_t cnt;
    uint32_t key;
};
constexpr uint32_t kMultiItem = 0x80000000u;

__global__ void desc_kernel(const int64_t* __restrict__ item_run,
                            const int64_t* __restrict__ item_start,
                            const int64_t* __restrict__ run_start,
                            const uint32_t* __restrict__ keys, int64_t I,
                            ItemDesc* __restrict__ desc) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= I) return;
    const int64_t r = item_run[i], i0 = item_start[r], i1 = item_start[r + 1];
    const int64_t rs = run_start[r], re = run_start[r + 1];
    const int64_t p0 = rs + (i - i0) * kItem;
    const int64_t cnt = re - p0 < kItem ? re - p0 : kItem;
    ItemDesc d;
    d.p0 = p0;
    d.cnt = (uint32_t)cnt | (i1 - i0 > 1 ? kMultiItem : 0u);
    d.key = keys[rs];
    desc[i] = d;
}

// inv[seg_lo[b] + e] = sorted position (batch-local) of batch b's entry e.
__global__ void inverse_kernel(const int64_t* __restrict__ seg_lo,
                               const uint32_t* __restrict__ vals, uint32_t* __restrict__ inv) {
    const int64_t b = blockIdx.x, s0 = seg_lo[b], s1 = seg_lo[b + 1];
    for (int64_t p = s0 + threadIdx.x; p < s1; p += blockDim.x)
        inv[s0 + vals[p]] = (uint32_t)(p - s0);
}

__global__ void batch_tables_kernel(const int64_t* __restrict__ seg_lo, int64_t nb,
                                    const int64_t* __restrict__ run_id,
                                    const int64_t* __restrict__ item_start,
                                    const int64_t* __restrict__ long_scan,
                                    int64_t* __restrict__ bitem, int64_t* __restrict__ blong) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b > nb) return;
    const int64_t r = run_id[seg_lo[b]];
    bitem[b] = item_start[r];
    blong[b] = long_scan[r];
}

// Data-parallel plan: key of each run (distinct key per batch) and the runs
// before each batch.
__global__ void run_key_kernel(const uint32_t* __restrict__ keys, const int32_t* __restrict__ head,
                               const int64_t* __restrict__ runs, int64_t n,
                               uint32_t* __restrict__ rkey) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && head[i]) rkey[runs[i]] = keys[i];
}
__global__ void batch_runs_kernel(const int64_t* __restrict__ seg_lo, int64_t nb,
                                  const int64_t* __restrict__ runs, int64_t* __restrict__ brun) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b <= nb) brun[b] = runs[seg_lo[b]];
}

}  // namespace mfm
