// segsort.cuh — stable LSD radix sort of (key, value) uint32 pairs within
// independent segments (one segment per mini-batch).
//
// Each segment is cut into tiles of kSortTile entries. Per 8-bit digit pass:
//   1. seg_hist_kernel:    per-tile digit histogram (integer smem atomics);
//   2. seg_offsets_kernel: per segment, digit-major / tile-minor exclusive
//                          prefix -> the output offset of every (tile, digit);
//   3. seg_scatter_kernel: per tile, stable rank of each entry among equal
//                          digits (warp match + per-warp counts) and scatter.
// Stability makes the final order (key, original position) — deterministic,
// with no floating point involved. The last pass can replace each value by
// data gathered through it (RecGather): the sorted stream then carries what
// its consumer reads instead of an index into the unsorted one.
#pragma once

#include <type_traits>

#include "scan.cuh"

namespace mfm {

constexpr int kSortNT = 1024;
constexpr int kSortRounds = 4;
constexpr int kSortTile = kSortNT * kSortRounds;

__global__ void __launch_bounds__(256)
    seg_hist_kernel(const uint32_t* __restrict__ keys, const int64_t* __restrict__ tile_lo,
                    const int64_t* __restrict__ tile_hi, int shift,
                    uint32_t* __restrict__ hist) {
    __shared__ uint32_t h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int64_t lo = tile_lo[blockIdx.x], hi = tile_hi[blockIdx.x];
    for (int64_t p = lo + threadIdx.x; p < hi; p += 256) atomicAdd(&h[(keys[p] >> shift) & 255u], 1u);
    __syncthreads();
    hist[(int64_t)blockIdx.x * 256 + threadIdx.x] = h[threadIdx.x];
}

// One block (256 threads, thread = digit) per segment; converts the tiles'
// counts into absolute output offsets in place.
__global__ void __launch_bounds__(256)
    seg_offsets_kernel(const int64_t* __restrict__ seg_lo, const int64_t* __restrict__ seg_tile,
                       uint32_t* __restrict__ hist) {
    __shared__ uint32_t sm[8];
    const int b = blockIdx.x, d = threadIdx.x;
    const int64_t t0 = seg_tile[b], t1 = seg_tile[b + 1];
    uint32_t tot = 0;
    for (int64_t t = t0; t < t1; ++t) tot += hist[t * 256 + d];
    uint32_t all;
    const uint32_t before = block_exclusive_scan<uint32_t, 256>(tot, sm, all);
    // offsets are stored relative to the segment start (fits in 32 bits)
    uint32_t run = before;
    for (int64_t t = t0; t < t1; ++t) {
        const uint32_t c = hist[t * 256 + d];
        hist[t * 256 + d] = run;
        run += c;
    }
}

// Value writers of the scatter: plain (the value itself) or, on the last
// pass, two arrays gathered at segment start + value.
struct PlainValue {
    __device__ __forceinline__ void operator()(uint32_t* vout, int64_t dst, int64_t,
                                               uint32_t val) const {
        vout[dst] = val;
    }
};
template <class T>
struct RecGather {
    const uint32_t* a;  // -> vout
    const T* b;         // -> bout
    T* bout;
    __device__ __forceinline__ void operator()(uint32_t* vout, int64_t dst, int64_t seg0,
                                               uint32_t val) const {
        vout[dst] = a[seg0 + val];
        bout[dst] = b[seg0 + val];
    }
};

template <class Out>
__global__ void __launch_bounds__(kSortNT)
    seg_scatter_kernel(const uint32_t* __restrict__ kin, const uint32_t* __restrict__ vin,
                       uint32_t* __restrict__ kout, uint32_t* __restrict__ vout,
                       const int64_t* __restrict__ tile_lo, const int64_t* __restrict__ tile_hi,
                       const int64_t* __restrict__ tile_seg_lo, int shift,
                       const uint32_t* __restrict__ offs, Out out) {
    __shared__ uint32_t wh[kSortNT / 32][256];  // per-warp digit counts -> prefixes
    __shared__ uint32_t running[256];
    __shared__ uint32_t round_tot[256];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t lo = tile_lo[blockIdx.x], hi = tile_hi[blockIdx.x];
    const int64_t seg0 = tile_seg_lo[blockIdx.x];
    if (t < 256) running[t] = offs[(int64_t)blockIdx.x * 256 + t];
    const unsigned lt = (1u << lane) - 1u;
    for (int r = 0; r < kSortRounds; ++r) {
        const int64_t p = lo + (int64_t)r * kSortNT + t;
        const bool valid = p < hi;
        if (lo + (int64_t)r * kSortNT >= hi) break;  // uniform across the block
        uint32_t key = 0, val = 0;
        if (valid) {
            key = kin[p];
            val = vin[p];
        }
        const uint32_t d = valid ? (key >> shift) & 255u : 256u + (uint32_t)lane;
        for (int i = t; i < (kSortNT / 32) * 256; i += kSortNT) (&wh[0][0])[i] = 0;
        __syncthreads();
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int rank = __popc(peers & lt);
        if (valid && rank == 0) wh[warp][d] = (uint32_t)__popc(peers);
        __syncthreads();
        if (t < 256) {
            uint32_t acc = 0;
#pragma unroll 8
            for (int w = 0; w < kSortNT / 32; ++w) {
                const uint32_t c = wh[w][t];
                wh[w][t] = acc;
                acc += c;
            }
            round_tot[t] = acc;
        }
        __syncthreads();
        if (valid) {
            const int64_t dst = seg0 + running[d] + wh[warp][d] + rank;
            kout[dst] = key;
            out(vout, dst, seg0, val);
        }
        __syncthreads();
        if (t < 256) running[t] += round_tot[t];
        __syncthreads();
    }
}

// Builds the tile table: segment b = [seg_lo[b], seg_lo[b+1]) gets
// ceil(len/kSortTile) tiles numbered from seg_tile[b].
__global__ void seg_tiles_kernel(const int64_t* __restrict__ seg_lo, int64_t n_seg,
                                 const int64_t* __restrict__ seg_tile,
                                 int64_t* __restrict__ tile_lo, int64_t* __restrict__ tile_hi,
                                 int64_t* __restrict__ tile_seg_lo) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_seg) return;
    const int64_t s0 = seg_lo[b], s1 = seg_lo[b + 1];
    int64_t t = seg_tile[b];
    for (int64_t p = s0; p < s1; p += kSortTile, ++t) {
        tile_lo[t] = p;
        tile_hi[t] = p + kSortTile < s1 ? p + kSortTile : s1;
        tile_seg_lo[t] = s0;
    }
}

__global__ void seg_tile_count_kernel(const int64_t* __restrict__ seg_lo, int64_t n_seg,
                                      int64_t* __restrict__ cnt) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n_seg) cnt[b] = ceil_div(seg_lo[b + 1] - seg_lo[b], kSortTile);
}

// Sorts (keys, vals)[seg_lo[0], seg_lo[n_seg]) stably by key within each
// segment; only the low `key_bits` bits are examined. Segments must be
// shorter than 2^32 entries. Returns a pointer to whichever of the two
// buffers holds the result. With a RecGather `last`, the final pass writes
// last.a[seg start + value] as the value and last.b[...] into last.bout
// (at least one pass runs then, so the gather always happens). With kfirst
// set, the first pass reads its keys there instead of k0 (kfirst is never
// written; k0 only serves as scratch from the second pass on).
struct SortResult {
    uint32_t* keys;
    uint32_t* vals;
};

template <class Last = PlainValue>
SortResult segmented_sort(int device, cudaStream_t s, uint32_t* k0, uint32_t* v0, uint32_t* k1,
                          uint32_t* v1, const int64_t* d_seg_lo, int64_t n_seg, int64_t n_entries,
                          int key_bits, Last last = Last{}, const uint32_t* kfirst = nullptr) {
    SortResult res{k0, v0};
    constexpr bool gather = !std::is_same<Last, PlainValue>::value;
    if (gather && key_bits < 1) key_bits = 1;
    if (n_entries == 0 || key_bits <= 0 || n_seg == 0) return res;
    DevBuf<int64_t> seg_tile(device, n_seg + 1);
    seg_tile_count_kernel<<<(unsigned)ceil_div(n_seg, 256), 256, 0, s>>>(d_seg_lo, n_seg,
                                                                          seg_tile.ptr);
    exclusive_scan<int64_t, int64_t>(device, s, seg_tile.ptr, n_seg, seg_tile.ptr);
    int64_t n_tiles = 0;
    d2h(&n_tiles, seg_tile.ptr + n_seg, 1, s, "sort tile count");
    MFM_CUDA(cudaStreamSynchronize(s), "sort tile count");
    if (n_tiles == 0) return res;
    DevBuf<int64_t> tlo(device, n_tiles), thi(device, n_tiles), tseg(device, n_tiles);
    seg_tiles_kernel<<<(unsigned)ceil_div(n_seg, 256), 256, 0, s>>>(
        d_seg_lo, n_seg, seg_tile.ptr, tlo.ptr, thi.ptr, tseg.ptr);
    DevBuf<uint32_t> hist(device, (size_t)n_tiles * 256);
    const uint32_t* ki = kfirst ? kfirst : k0;
    uint32_t *vi = v0, *ko = k1, *vo = v1;
    for (int shift = 0; shift < key_bits; shift += 8) {
        seg_hist_kernel<<<(unsigned)n_tiles, 256, 0, s>>>(ki, tlo.ptr, thi.ptr, shift, hist.ptr);
        seg_offsets_kernel<<<(unsigned)n_seg, 256, 0, s>>>(d_seg_lo, seg_tile.ptr, hist.ptr);
        if (gather && shift + 8 >= key_bits)
            seg_scatter_kernel<Last><<<(unsigned)n_tiles, kSortNT, 0, s>>>(
                ki, vi, ko, vo, tlo.ptr, thi.ptr, tseg.ptr, shift, hist.ptr, last);
        else
            seg_scatter_kernel<PlainValue><<<(unsigned)n_tiles, kSortNT, 0, s>>>(
                ki, vi, ko, vo, tlo.ptr, thi.ptr, tseg.ptr, shift, hist.ptr, PlainValue{});
        MFM_CHECK_LAUNCH("segmented sort launch");
        // the next pass reads what this one wrote and writes the other pair
        uint32_t* nk = ko == k1 ? k0 : k1;
        uint32_t* nv = vo == v1 ? v0 : v1;
        ki = ko;
        vi = vo;
        ko = nk;
        vo = nv;
    }
    res.keys = const_cast<uint32_t*>(ki);
    res.vals = vi;
    return res;
}

}  // namespace mfm
