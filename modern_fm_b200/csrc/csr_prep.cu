// csr_prep.cu — CSR canonicalisation on the device: the step before scoring
// and training.
//
// The reference canonicalises every CSR on the host before its native call:
// `X.tocsr().astype(np.float64); X.sum_duplicates()` and int64 / float64
// copies (python/modern_fm/_backend.py:44-52), then validates it
// (CsrView::new, rust/src/data.rs:14-44). mfm_csr_prep_device does the same on
// device memory and writes the engine's compute layout in one go: for a raw
// CSR in the boundary format (int64 indptr and indices, float64 values; rows
// in any column order, duplicate (row, column) entries allowed) it
//   * validates indptr (starts at 0, non-decreasing, ends at nnz) and every
//     column index against [0, n_features);
//   * sorts each row's entries by column and sums duplicates in float64, the
//     duplicates of one column added in their original order (explicit zeros
//     and zero sums are kept, as scipy keeps them);
//   * narrows to int32 columns and values in the compute dtype, so the result
//     feeds mfm_{fm,ffm,fwfm}_predict_device and mfm_fm_fit_device directly.
//
// Work split:
//   1. one streaming pass: csr_prep_rows_kernel (thread per row: indptr checks,
//      a bit per row start, the output indptr) and csr_prep_flat_kernel (four
//      coalesced entries per thread: range check, "greater than the previous
//      entry unless it starts a row", the narrowed copy). When every row is in
//      order, the common case, that copy is the result and nothing else runs.
//   2. otherwise csr_prep_sort_kernel (warp per row, rows grid-strided)
//      writes each row's distinct-column count: rows of up to kShortRow entries
//      that are out of order are sorted and merged once, into a scratch copy
//      at their input offsets; longer ones are listed for the sort. An
//      exclusive scan of the counts gives the output indptr.
//   3. long unsorted rows only: their narrowed columns are gathered into one
//      buffer and sorted stably within each row by the segmented radix sort
//      (segsort.cuh), so equal columns keep their original order.
//   4. csr_prep_place_kernel (in-order rows from the input, short sorted rows
//      from the scratch) and csr_prep_long_kernel (the long sorted rows): each
//      distinct column at its row's output offset plus its rank, with the
//      float64 sum of its duplicates, narrowed once.
// Every sum has a fixed order, so results are bitwise reproducible.
#include <algorithm>

#include "common.cuh"
#include "scan.cuh"
#include "segsort.cuh"

namespace mfm {
namespace {

constexpr int kShortRow = 256;  // longest row handled in shared memory
constexpr int kPrepWarps = 8;   // warps per block

enum : unsigned {
    kBadOrder = 1u,   // indptr decreases
    kBadEnds = 2u,    // indptr does not start at 0 / end at nnz, or leaves [0, nnz]
    kBadIndex = 4u,   // a column index outside [0, n_features)
    kUnsorted = 8u,   // some row is out of order or holds duplicates
};

// Pass 1, row part: one thread per row. Validates the row's bounds, marks
// each nonempty row's first entry in `starts` (one bit per entry) and writes
// the output indptr as a copy of the input's (final when every row turns out
// to be in order; rewritten by the scan otherwise).
__global__ void __launch_bounds__(256)
    csr_prep_rows_kernel(const int64_t* __restrict__ indptr, int64_t n_rows, int64_t nnz,
                         int64_t* __restrict__ indptr_out, unsigned* __restrict__ starts,
                         unsigned* flags) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    unsigned bad = 0;
    if (r < n_rows) {
        const int64_t lo = indptr[r], hi = indptr[r + 1];
        if (hi < lo)
            bad = kBadOrder;
        else if (lo < 0 || hi > nnz || (r == 0 && lo != 0) || (r == n_rows - 1 && hi != nnz))
            bad = kBadEnds;
        else if (lo < hi)
            atomicOr(starts + (lo >> 5), 1u << (lo & 31));
        indptr_out[r + 1] = hi;
        if (r == 0) indptr_out[0] = lo;
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    if (bad && (threadIdx.x & 31) == 0) atomicOr(flags, bad);
}

// Pass 1, entry part: kFlatItems entries per thread, strided by the block
// (entry q = tile + i * kFlatNT + tid) so every load and store is coalesced
// and a warp's 32 entries share one word of `starts`. Checks each column's
// range and that it exceeds its predecessor unless it starts a row, and writes
// the narrowed entry at the same position of the output.
constexpr int kFlatNT = 256, kFlatItems = 4;
template <class T>
__global__ void __launch_bounds__(kFlatNT)
    csr_prep_flat_kernel(const int64_t* __restrict__ indices, const double* __restrict__ data,
                         int64_t nnz, int64_t n_features, const unsigned* __restrict__ starts,
                         int32_t* __restrict__ ind_out, T* __restrict__ dat_out,
                         unsigned* flags) {
    const int64_t tile = (int64_t)blockIdx.x * (kFlatNT * kFlatItems);
    const int lane = threadIdx.x & 31;
    int64_t c[kFlatItems], pv[kFlatItems];
    double v[kFlatItems];
    unsigned sw[kFlatItems];
#pragma unroll
    for (int i = 0; i < kFlatItems; ++i) {  // every load issued before any use
        const int64_t q = tile + i * kFlatNT + threadIdx.x;
        const bool in = q < nnz;
        c[i] = in ? indices[q] : 0;
        v[i] = in ? data[q] : 0.0;
        pv[i] = (lane == 0 && in && q > 0) ? indices[q - 1] : 0;  // outside the warp's chunk
        sw[i] = in ? starts[q >> 5] : 0u;
    }
    unsigned bad = 0;
#pragma unroll
    for (int i = 0; i < kFlatItems; ++i) {
        const int64_t q = tile + i * kFlatNT + threadIdx.x;
        int64_t prev = __shfl_up_sync(0xffffffffu, c[i], 1);
        if (lane == 0) prev = pv[i];
        if (q < nnz) {
            const bool start = (sw[i] >> (q & 31)) & 1u;
            if (c[i] < 0 || c[i] >= n_features) bad |= kBadIndex;
            if (!start && !(c[i] > prev)) bad |= kUnsorted;
            ind_out[q] = (int32_t)c[i];
            dat_out[q] = (T)v[i];
        }
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    // flags only gain bits: once a bit is set, later warps skip the atomic on
    // the one shared word (on unsorted input nearly every warp finds disorder)
    if (bad && lane == 0 && (*(volatile unsigned*)flags & bad) != bad) atomicOr(flags, bad);
}

// Sorts a row's (column << 32 | position) pairs across one warp in registers:
// element e = r * 32 + lane lives in v[r]; a bitonic network over 32 R keys
// (the row's len keys, padded with the largest key), partners in other lanes
// exchanged by shuffles and partners in other registers compared in place —
// no shared-memory traffic. Equal columns keep their original order (the
// position breaks ties).
template <class K, int R>
__device__ __forceinline__ void warp_sort_regs(K (&v)[R], int lane) {
#pragma unroll
    for (int k = 2; k <= 32 * R; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {  // partner in register r ^ (j / 32) of the same lane
                const int jr = j >> 5;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (r & jr) continue;
                    const int e = r * 32 + lane;
                    const bool up = (e & k) == 0;
                    const K x = v[r], y = v[r | jr];
                    if ((x > y) == up) {
                        v[r] = y;
                        v[r | jr] = x;
                    }
                }
            } else {  // partner in lane ^ j, same register
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int e = r * 32 + lane;
                    const bool up = (e & k) == 0, lower = (lane & j) == 0;
                    const K o = __shfl_xor_sync(0xffffffffu, v[r], j);
                    const bool keep_min = lower == up;
                    v[r] = keep_min ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
                }
            }
        }
    }
}

// Sort keys: (column << 32) | position in 64 bits, or (column << 8) | position
// in 32 bits when every column fits in 24 bits (rows of at most 256 entries,
// so a position fits in 8): half the shuffles and compares per step.
template <class K>
struct SortKey;
template <>
struct SortKey<uint64_t> {
    static constexpr int kPosBits = 32;
    static constexpr uint64_t kPad = ~0ull;
};
template <>
struct SortKey<uint32_t> {
    static constexpr int kPosBits = 8;
    static constexpr uint32_t kPad = ~0u;
};
template <class K>
__device__ __forceinline__ K make_key(int64_t col, int pos) {
    return ((K)(uint32_t)col << SortKey<K>::kPosBits) | (K)(uint32_t)pos;
}
template <class K>
__device__ __forceinline__ uint32_t col_of(K key) { return (uint32_t)(key >> SortKey<K>::kPosBits); }
template <class K>
__device__ __forceinline__ uint32_t pos_of(K key) {
    return (uint32_t)(key & (((K)1 << SortKey<K>::kPosBits) - 1));
}

// Sorts the row staged in s[0, len) (len <= kShortRow) and writes it back
// sorted; registers per lane: 2 keys for rows of up to 64 entries, 8 otherwise.
template <class K>
__device__ __forceinline__ void warp_sort_row(K* s, int len, int lane) {
    if (len <= 64) {
        K v[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) v[r] = r * 32 + lane < len ? s[r * 32 + lane] : SortKey<K>::kPad;
        warp_sort_regs<K, 2>(v, lane);
#pragma unroll
        for (int r = 0; r < 2; ++r)
            if (r * 32 + lane < len) s[r * 32 + lane] = v[r];
    } else {
        K v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = r * 32 + lane < len ? s[r * 32 + lane] : SortKey<K>::kPad;
        warp_sort_regs<K, 8>(v, lane);
#pragma unroll
        for (int r = 0; r < 8; ++r)
            if (r * 32 + lane < len) s[r * 32 + lane] = v[r];
    }
    __syncwarp();
}

template <class K>
__device__ __forceinline__ uint32_t sorted_col(const K* s, int e) { return col_of(s[e]); }

// How each row reaches the output (row_kind).
enum : uint8_t {
    kRowInOrder = 0,  // strictly increasing: copied from the input as it is
    kRowSorted = 1,   // short and out of order: sorted, merged rows in the scratch
    kRowLong = 2,     // long and out of order: sorted by segmented_sort, written by
                      // csr_prep_long_kernel
};

// Pass 2 (some row is out of order), warp per row: each row's distinct-column
// count into cnt[row] and its kind. A short out-of-order row (up to kShortRow
// entries) is sorted once, here — keys (column, position) in a warp bitonic
// network in registers — and its distinct columns, ascending, each with the
// float64 sum of its duplicates in their original order narrowed once, are
// written to the scratch arrays at the row's input offset. Long out-of-order
// rows are listed for the segmented sort. Pass 1 has validated the structure
// and every column. flags[0] gets kUnsorted; flags[1] counts long rows. K:
// the sort key type (uint32_t when the columns fit in 24 bits).
template <class T, class K>
__global__ void __launch_bounds__(kPrepWarps * 32)
    csr_prep_sort_kernel(const int64_t* __restrict__ indptr, const int64_t* __restrict__ indices,
                         const double* __restrict__ data, int64_t n_rows,
                         int32_t* __restrict__ tmp_ind, T* __restrict__ tmp_dat,
                         int64_t* __restrict__ cnt, uint8_t* __restrict__ row_kind,
                         int64_t* __restrict__ long_row, int64_t max_long, unsigned* flags) {
    __shared__ K skey[kPrepWarps][kShortRow];
    __shared__ double sval[kPrepWarps][kShortRow];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t nwarps = (int64_t)gridDim.x * kPrepWarps;
    for (int64_t r = (int64_t)blockIdx.x * kPrepWarps + wib; r < n_rows; r += nwarps) {
        const int64_t lo = indptr[r], hi = indptr[r + 1];
        const int64_t len = hi - lo;
        const bool short_row = len <= kShortRow;
        bool unsorted = false;
        int64_t carry = -1;  // the previous chunk's last column
        for (int64_t base = lo; base < hi; base += 32) {
            const int64_t q = base + lane;
            const bool in = q < hi;
            const int64_t c = in ? indices[q] : 0;
            int64_t prev = __shfl_up_sync(0xffffffffu, c, 1);
            if (lane == 0) prev = carry;
            unsorted |= in && q > lo && !(c > prev);
            carry = __shfl_sync(0xffffffffu, c, 31);
            if (in && short_row) {
                skey[wib][q - lo] = make_key<K>(c, (int)(q - lo));
                sval[wib][q - lo] = data[q];
            }
        }
        unsorted = __any_sync(0xffffffffu, unsorted);
        int64_t count = len;
        uint8_t kind = kRowInOrder;
        if (unsorted && short_row) {
            kind = kRowSorted;
            __syncwarp();
            const K* sk = skey[wib];
            warp_sort_row(skey[wib], (int)len, lane);
            // heads of the sorted runs are the distinct columns in ascending
            // order; a head's rank is the number of heads before it, and its
            // sum adds the run's values in their original order
            int before = 0;
            for (int base = 0; base < (int)len; base += 32) {
                const int e = base + lane;
                const bool head =
                    e < (int)len && (e == 0 || sorted_col(sk, e) != sorted_col(sk, e - 1));
                const unsigned hm = __ballot_sync(0xffffffffu, head);
                if (head) {
                    const int rank = before + __popc(hm & ((1u << lane) - 1u));
                    const uint32_t key = sorted_col(sk, e);
                    double sum = sval[wib][pos_of(sk[e])];
                    for (int e2 = e + 1; e2 < (int)len && sorted_col(sk, e2) == key; ++e2)
                        sum += sval[wib][pos_of(sk[e2])];
                    tmp_ind[lo + rank] = (int32_t)key;
                    tmp_dat[lo + rank] = (T)sum;
                }
                before += __popc(hm);
            }
            count = before;
        } else if (unsorted) {
            kind = kRowLong;
            count = 0;  // counted after the sort
            // at most nnz / (kShortRow + 1) rows can be long in a valid CSR
            if (lane == 0) {
                const unsigned slot = atomicAdd(flags + 1, 1u);
                if (slot < max_long) long_row[slot] = r;
            }
        }
        if (unsorted && lane == 0 && !(*(volatile unsigned*)flags & kUnsorted))
            atomicOr(flags, kUnsorted);  // once set, later rows skip the atomic
        __syncwarp();  // the shared row is rewritten by the next row
        if (lane == 0) {
            cnt[r] = count;
            row_kind[r] = kind;
        }
    }
}

// Pass 3, warp per row: every row at its output offset — in-order rows from
// the input (narrowed), sorted rows from the scratch; long rows are left to
// csr_prep_long_kernel.
template <class T>
__global__ void __launch_bounds__(kPrepWarps * 32)
    csr_prep_place_kernel(const int64_t* __restrict__ indptr, const int64_t* __restrict__ indices,
                          const double* __restrict__ data, int64_t n_rows,
                          const int64_t* __restrict__ out_ptr,
                          const uint8_t* __restrict__ row_kind,
                          const int32_t* __restrict__ tmp_ind, const T* __restrict__ tmp_dat,
                          int32_t* __restrict__ ind_out, T* __restrict__ dat_out) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * kPrepWarps;
    for (int64_t r = (int64_t)blockIdx.x * kPrepWarps + (threadIdx.x >> 5); r < n_rows;
         r += nwarps) {
        const uint8_t kind = row_kind[r];
        if (kind == kRowLong) continue;
        const int64_t lo = indptr[r], o = out_ptr[r];
        if (kind == kRowInOrder) {
            const int64_t len = indptr[r + 1] - lo;
            for (int64_t t = lane; t < len; t += 32) {
                ind_out[o + t] = (int32_t)indices[lo + t];
                dat_out[o + t] = (T)data[lo + t];
            }
        } else {
            const int64_t n = out_ptr[r + 1] - o;
            for (int64_t t = lane; t < n; t += 32) {
                ind_out[o + t] = tmp_ind[lo + t];
                dat_out[o + t] = tmp_dat[lo + t];
            }
        }
    }
}

// Gathers the narrowed columns of the long unsorted rows into one buffer
// (segment j = long row j) with each entry's position within its row.
__global__ void __launch_bounds__(256)
    csr_prep_gather_long_kernel(const int64_t* __restrict__ indptr,
                                const int64_t* __restrict__ long_row, int64_t n_long,
                                const int64_t* __restrict__ seg_lo,
                                const int32_t* __restrict__ ind_narrow, uint32_t* __restrict__ key,
                                uint32_t* __restrict__ pos) {
    for (int64_t j = blockIdx.x; j < n_long; j += gridDim.x) {
        const int64_t lo = indptr[long_row[j]], s0 = seg_lo[j], len = seg_lo[j + 1] - s0;
        for (int64_t t = threadIdx.x; t < len; t += blockDim.x) {
            key[s0 + t] = (uint32_t)ind_narrow[lo + t];
            pos[s0 + t] = (uint32_t)t;
        }
    }
}

// Counts (write = false) or writes (write = true) the distinct columns of the
// sorted long rows: warp per row; a column's first sorted entry sums the run
// of its duplicates in original order (the sort is stable).
template <class T, bool WRITE>
__global__ void __launch_bounds__(kPrepWarps * 32)
    csr_prep_long_kernel(const int64_t* __restrict__ indptr, const double* __restrict__ data,
                         const int64_t* __restrict__ long_row, int64_t n_long,
                         const int64_t* __restrict__ seg_lo, const uint32_t* __restrict__ key,
                         const uint32_t* __restrict__ pos, int64_t* __restrict__ cnt_or_ptr,
                         int32_t* __restrict__ ind_out, T* __restrict__ dat_out) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * kPrepWarps;
    for (int64_t j = (int64_t)blockIdx.x * kPrepWarps + (threadIdx.x >> 5); j < n_long;
         j += nwarps) {
        const int64_t r = long_row[j], lo = indptr[r];
        const int64_t s0 = seg_lo[j], s1 = seg_lo[j + 1];
        int64_t o = WRITE ? cnt_or_ptr[r] : 0;
        int64_t heads = 0;
        for (int64_t base = s0; base < s1; base += 32) {
            const int64_t p = base + lane;
            const bool in = p < s1;
            const uint32_t kk = in ? key[p] : 0u;
            const bool head = in && (p == s0 || key[p - 1] != kk);
            const unsigned mask = __ballot_sync(0xffffffffu, head);
            if (WRITE && head) {
                double sum = data[lo + pos[p]];  // from the first occurrence
                for (int64_t p2 = p + 1; p2 < s1 && key[p2] == kk; ++p2) sum += data[lo + pos[p2]];
                const int64_t at = o + __popc(mask & ((1u << lane) - 1u));
                ind_out[at] = (int32_t)kk;
                dat_out[at] = (T)sum;
            }
            o += __popc(mask);
            heads += __popc(mask);
        }
        if (!WRITE && lane == 0) cnt_or_ptr[r] = heads;
    }
}

int key_bits_for(int64_t n_features) {
    int b = 1;
    while (b < 31 && (int64_t(1) << b) < n_features) ++b;
    return b;
}

template <class T>
int64_t csr_prep(int device, cudaStream_t s, int64_t n_rows, int64_t n_features, int64_t nnz,
                 const int64_t* indptr, const int64_t* indices, const double* data,
                 int64_t* indptr_out, int32_t* ind_out, T* dat_out) {
    if (n_rows == 0) {
        int64_t first = -1;
        d2h(&first, indptr, 1, s, "CSR prep indptr");
        MFM_CUDA(cudaStreamSynchronize(s), "CSR prep indptr");
        if (first != 0 || nnz != 0) fail(MFM_ERR_INVALID, "indptr must start at 0 and end at nnz");
        MFM_CUDA(cudaMemcpyAsync(indptr_out, indptr, sizeof(int64_t), cudaMemcpyDeviceToDevice, s),
                 "CSR prep indptr");
        MFM_CUDA(cudaStreamSynchronize(s), "CSR prep");
        return 0;
    }
    // pass 1 (streaming): validation, order check and the narrowed copy
    DevBuf<unsigned> flags(device, 2), starts(device, (size_t)(nnz / 32 + 1));
    MFM_CUDA(cudaMemsetAsync(flags.ptr, 0, 2 * sizeof(unsigned), s), "memset");
    MFM_CUDA(cudaMemsetAsync(starts.ptr, 0, starts.bytes(), s), "memset");
    csr_prep_rows_kernel<<<(unsigned)ceil_div(n_rows, 256), 256, 0, s>>>(
        indptr, n_rows, nnz, indptr_out, starts.ptr, flags.ptr);
    if (nnz > 0)
        csr_prep_flat_kernel<T><<<(unsigned)ceil_div(nnz, kFlatNT * kFlatItems), kFlatNT, 0, s>>>(
            indices, data, nnz, n_features, starts.ptr, ind_out, dat_out, flags.ptr);
    MFM_CHECK_LAUNCH("CSR prep check");
    unsigned h[2] = {0, 0};
    d2h(h, flags.ptr, 2, s, "CSR prep flags");
    MFM_CUDA(cudaStreamSynchronize(s), "CSR prep check");
    if (h[0] & kBadOrder) fail(MFM_ERR_INVALID, "indptr must be non-decreasing");
    if (h[0] & kBadEnds) fail(MFM_ERR_INVALID, "indptr must start at 0 and end at nnz");
    if (h[0] & kBadIndex)
        fail(MFM_ERR_INVALID, fmt("column index out of range [0, %lld)", (long long)n_features));
    if (!(h[0] & kUnsorted)) return nnz;  // canonical already: pass 1 wrote the result

    // some row is out of order: per-row distinct counts (and the long-row
    // list); counts go straight into indptr_out
    const int64_t max_long = std::min<int64_t>(n_rows, nnz / (kShortRow + 1) + 1);
    DevBuf<int64_t> long_row(device, (size_t)max_long);
    DevBuf<uint8_t> row_kind(device, (size_t)n_rows);
    DevBuf<int32_t> tmp_ind(device, (size_t)std::max<int64_t>(1, nnz));
    DevBuf<T> tmp_dat(device, (size_t)std::max<int64_t>(1, nnz));
    MFM_CUDA(cudaMemsetAsync(flags.ptr, 0, 2 * sizeof(unsigned), s), "memset");
    const unsigned grid = warp_grid(device, n_rows, kPrepWarps, 8);
    if (n_features <= ((int64_t)1 << 24))  // column and position in one 32-bit key
        csr_prep_sort_kernel<T, uint32_t><<<grid, kPrepWarps * 32, 0, s>>>(
            indptr, indices, data, n_rows, tmp_ind.ptr, tmp_dat.ptr, indptr_out, row_kind.ptr,
            long_row.ptr, max_long, flags.ptr);
    else
        csr_prep_sort_kernel<T, uint64_t><<<grid, kPrepWarps * 32, 0, s>>>(
            indptr, indices, data, n_rows, tmp_ind.ptr, tmp_dat.ptr, indptr_out, row_kind.ptr,
            long_row.ptr, max_long, flags.ptr);
    MFM_CHECK_LAUNCH("CSR prep sort");
    d2h(h, flags.ptr, 2, s, "CSR prep flags");
    MFM_CUDA(cudaStreamSynchronize(s), "CSR prep count");

    // long unsorted rows: stable segmented sort of their columns
    const int64_t n_long = h[1];  // <= max_long once the CSR is valid
    if (n_long > max_long) fail(MFM_ERR_INVALID, "indptr must be non-decreasing");
    DevBuf<int64_t> seg_lo;
    DevBuf<uint32_t> k0, v0, k1, v1;
    SortResult sorted{nullptr, nullptr};
    if (n_long > 0) {
        std::vector<int64_t> rows(n_long), bounds(n_rows + 1), lo(n_long + 1, 0);
        d2h(rows.data(), long_row.ptr, n_long, s, "CSR prep long rows");
        d2h(bounds.data(), indptr, n_rows + 1, s, "CSR prep indptr");
        MFM_CUDA(cudaStreamSynchronize(s), "CSR prep long rows");
        std::sort(rows.begin(), rows.end());  // a fixed buffer layout
        for (int64_t j = 0; j < n_long; ++j)
            lo[j + 1] = lo[j] + (bounds[rows[j] + 1] - bounds[rows[j]]);
        const int64_t total = lo[n_long];
        h2d(long_row.ptr, rows.data(), n_long, s, "CSR prep long rows");
        seg_lo.alloc(device, n_long + 1);
        h2d(seg_lo.ptr, lo.data(), n_long + 1, s, "CSR prep segments");
        k0.alloc(device, total);
        v0.alloc(device, total);
        k1.alloc(device, total);
        v1.alloc(device, total);
        csr_prep_gather_long_kernel<<<(unsigned)std::min<int64_t>(n_long, 65535), 256, 0, s>>>(
            indptr, long_row.ptr, n_long, seg_lo.ptr, ind_out, k0.ptr, v0.ptr);
        MFM_CHECK_LAUNCH("CSR prep gather");
        sorted = segmented_sort(device, s, k0.ptr, v0.ptr, k1.ptr, v1.ptr, seg_lo.ptr, n_long,
                                total, key_bits_for(n_features));
        const unsigned lg = warp_grid(device, n_long, kPrepWarps, 8);
        csr_prep_long_kernel<T, false><<<lg, kPrepWarps * 32, 0, s>>>(
            indptr, data, long_row.ptr, n_long, seg_lo.ptr, sorted.keys, sorted.vals, indptr_out,
            nullptr, nullptr);
        MFM_CHECK_LAUNCH("CSR prep long count");
    }
    exclusive_scan<int64_t, int64_t>(device, s, indptr_out, n_rows, indptr_out);
    csr_prep_place_kernel<T><<<grid, kPrepWarps * 32, 0, s>>>(
        indptr, indices, data, n_rows, indptr_out, row_kind.ptr, tmp_ind.ptr, tmp_dat.ptr,
        ind_out, dat_out);
    MFM_CHECK_LAUNCH("CSR prep place");
    if (n_long > 0) {
        const unsigned lg = warp_grid(device, n_long, kPrepWarps, 8);
        csr_prep_long_kernel<T, true><<<lg, kPrepWarps * 32, 0, s>>>(
            indptr, data, long_row.ptr, n_long, seg_lo.ptr, sorted.keys, sorted.vals, indptr_out,
            ind_out, dat_out);
        MFM_CHECK_LAUNCH("CSR prep long write");
    }
    int64_t nnz_out = 0;
    d2h(&nnz_out, indptr_out + n_rows, 1, s, "CSR prep nnz");
    MFM_CUDA(cudaStreamSynchronize(s), "CSR prep");
    return nnz_out;
}

}  // namespace
}  // namespace mfm

using namespace mfm;

extern "C" int mfm_csr_prep_device(int dtype, int device, int64_t n_rows, int64_t n_features,
                                   int64_t nnz, const int64_t* indptr, const int64_t* indices,
                                   const double* data, int64_t* indptr_out, int32_t* indices_out,
                                   void* data_out, int64_t* nnz_out, void* stream) {
    return guarded([&] {
        if (n_rows < 0 || nnz < 0 || n_features < 0) fail(MFM_ERR_INVALID, "negative CSR size");
        if (!indptr || !indptr_out || !nnz_out)
            fail(MFM_ERR_INVALID, "indptr, indptr_out and nnz_out must be provided");
        if (nnz > 0 && (!indices || !data || !indices_out || !data_out))
            fail(MFM_ERR_INVALID, "indices and data (in and out) must be provided when nnz > 0");
        if (n_features > INT32_MAX)
            fail(MFM_ERR_UNSUPPORTED, fmt("n_features %lld exceeds the engine's 2^31-1 limit",
                                          (long long)n_features));
        if (dtype != MFM_DTYPE_F32 && dtype != MFM_DTYPE_F64 && dtype != MFM_DTYPE_F32_F64)
            fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
        DeviceGuard g(device);
        // values keep float64 in both float64-arithmetic types
        cudaStream_t s = (cudaStream_t)stream;
        *nnz_out = dtype == MFM_DTYPE_F32
                       ? csr_prep<float>(device, s, n_rows, n_features, nnz, indptr, indices,
                                         data, indptr_out, indices_out, (float*)data_out)
                       : csr_prep<double>(device, s, n_rows, n_features, nnz, indptr, indices,
                                          data, indptr_out, indices_out, (double*)data_out);
    });
}
