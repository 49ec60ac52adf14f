// segsort.cuh — stable LSD radix sort of (key, value) uint32 pairs within
// independent segments (one segment per mini-batch).
//
// Each segment is cut into tiles of kSortTile entries. Per 8-bit digit pass:
//   1. seg_hist_kernel:    per-tile digit histogram (integer smem atomics);
//   2. seg_offsets_kernel: per segment, digit-major / tile-minor exclusive
//                          prefix -> the output offset of every (tile, digit);
//   3. seg_scatter_kernel: per tile, stable rank of each entry among equal
//                          digits (warp match + per-warp counters, 16 keys per
//                          thread) and scatter.
// Stability makes the final order (key, original position) — deterministic,
// with no floating point involved. The last pass can replace each value by
// data gathered through it (RecGather): the sorted stream then carries what
// its consumer reads instead of an index into the unsorted one. When the
// values to sort are the entries' segment-relative positions, the first pass
// generates them (IOTA) instead of reading them.
#pragma once

#include <algorithm>
#include <type_traits>
#include <vector>

#include "scan.cuh"

namespace mfm {

constexpr int kSortNT = 256;    // threads per tile (= digits per pass)
constexpr int kSortItems = 16;  // keys per thread
constexpr int kSortTile = kSortNT * kSortItems;

// Blocks stride over the n_tiles tiles (a grid smaller than n_tiles leaves
// room on the device for other streams' kernels).
static __global__ void __launch_bounds__(256)
    seg_hist_kernel(const uint32_t* __restrict__ keys, const int64_t* __restrict__ tile_lo,
                    const int64_t* __restrict__ tile_hi, int64_t n_tiles, int shift,
                    uint32_t* __restrict__ hist) {
    __shared__ uint32_t h[256];
    for (int64_t tb = blockIdx.x; tb < n_tiles; tb += gridDim.x) {
        h[threadIdx.x] = 0;
        __syncthreads();
        const int64_t lo = tile_lo[tb], hi = tile_hi[tb];
        for (int64_t p = lo + threadIdx.x; p < hi; p += 256)
            atomicAdd(&h[(keys[p] >> shift) & 255u], 1u);
        __syncthreads();
        hist[tb * 256 + threadIdx.x] = h[threadIdx.x];
        __syncthreads();  // h is cleared for the next tile
    }
}

// One block (256 threads, thread = digit) per segment; converts the tiles'
// counts into absolute output offsets in place.
static __global__ void __launch_bounds__(256)
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
// pass, two arrays gathered at segment start + value. `load` is issued for all
// of a thread's values before any `store`, so the gathers overlap.
struct PlainValue {
    struct P {
        uint32_t v;
    };
    __device__ __forceinline__ P load(int64_t, uint32_t val) const { return P{val}; }
    __device__ __forceinline__ void store(uint32_t* vout, int64_t dst, const P& p) const {
        vout[dst] = p.v;
    }
};
// A (row, value) record, packed so one gather reads one sector: 8 bytes for
// float, 16 for double.
template <class T>
struct alignas(2 * sizeof(T)) RowVal {
    uint32_t row;
    T x;
};
template <class T>
struct RecGather {
    const RowVal<T>* a;  // row -> vout, value -> bout
    T* bout;
    struct P {
        uint32_t v;
        T x;
    };
    __device__ __forceinline__ P load(int64_t seg0, uint32_t val) const {
        const RowVal<T> r = a[seg0 + val];
        return P{r.row, r.x};
    }
    __device__ __forceinline__ void store(uint32_t* vout, int64_t dst, const P& p) const {
        vout[dst] = p.v;
        bout[dst] = p.x;
    }
};

// Per tile: 256 threads x 16 keys in a striped layout (item i of lane l in
// warp w sits at tile start + w*512 + i*32 + l, so a warp's items in item
// order are in position order). Each warp ranks its keys among equal digits
// with match_any and per-warp digit counters; a prefix over the warps per
// digit and over the digits gives each key its stable tile-local position.
// The tile is reordered by digit in shared memory, then written out: every
// digit's keys form one contiguous run of the output, so the stores coalesce.
template <class Out, bool IOTA = false>
__global__ void __launch_bounds__(kSortNT)
    seg_scatter_kernel(const uint32_t* __restrict__ kin, const uint32_t* __restrict__ vin,
                       uint32_t* __restrict__ kout, uint32_t* __restrict__ vout,
                       const int64_t* __restrict__ tile_lo, const int64_t* __restrict__ tile_hi,
                       const int64_t* __restrict__ tile_seg_lo, int64_t n_tiles, int shift,
                       const uint32_t* __restrict__ offs, Out out) {
    constexpr int NW = kSortNT / 32;
    __shared__ uint32_t cnt[NW][256];  // per-warp digit counts -> tile-local start per warp
    __shared__ uint32_t base[256];     // output offset (segment-relative) minus tile-local start
    __shared__ uint32_t scan_sm[NW];
    __shared__ uint2 skv[kSortTile];  // (key, value), one 8-byte store per entry
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int64_t tb = blockIdx.x; tb < n_tiles; tb += gridDim.x) {  // blocks stride over tiles
    const int64_t lo = tile_lo[tb], hi = tile_hi[tb];
    const int64_t seg0 = tile_seg_lo[tb];
    for (int i = t; i < NW * 256; i += kSortNT) (&cnt[0][0])[i] = 0;
    const uint32_t goff = offs[tb * 256 + t];
    const int n = (int)(hi - lo), q0 = warp * (32 * kSortItems) + lane;  // tile-local
    const uint32_t* kt = kin + lo;
    const uint32_t* vt = vin + lo;
    uint32_t key[kSortItems], val[kSortItems], rank[kSortItems];
#pragma unroll
    for (int i = 0; i < kSortItems; ++i) {
        const int q = q0 + i * 32;
        key[i] = q < n ? kt[q] : 0u;
        val[i] = IOTA ? (uint32_t)(lo - seg0) + (uint32_t)q : (q < n ? vt[q] : 0u);
    }
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < kSortItems; ++i) {
        const bool valid = q0 + i * 32 < n;
        const uint32_t d = valid ? (key[i] >> shift) & 255u : 256u + (uint32_t)lane;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int leader = __ffs(peers) - 1;
        uint32_t b = 0;
        if (valid && lane == leader) {
            b = cnt[warp][d];
            cnt[warp][d] = b + (uint32_t)__popc(peers);
        }
        b = __shfl_sync(0xffffffffu, b, leader);
        rank[i] = b + (uint32_t)__popc(peers & lt);
        __syncwarp();  // this item's counter update before the next item's read
    }
    __syncthreads();
    uint32_t tot = 0;  // thread t = digit t: prefix over the warps, then over the digits
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const uint32_t c = cnt[w][t];
        cnt[w][t] = tot;
        tot += c;
    }
    uint32_t all;
    const uint32_t dstart = block_exclusive_scan<uint32_t, kSortNT>(tot, scan_sm, all);
#pragma unroll
    for (int w = 0; w < NW; ++w) cnt[w][t] += dstart;
    base[t] = goff - dstart;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kSortItems; ++i)
        if (q0 + i * 32 < n) {
            const uint32_t d = (key[i] >> shift) & 255u;
            const uint32_t lp = cnt[warp][d] + rank[i];
            skv[lp] = make_uint2(key[i], val[i]);
        }
    __syncthreads();
    typename Out::P pay[kSortItems];
#pragma unroll
    for (int u = 0; u < kSortItems; ++u) {
        const int j = t + u * kSortNT;
        if (j < n) pay[u] = out.load(seg0, skv[j].y);
    }
#pragma unroll
    for (int u = 0; u < kSortItems; ++u) {
        const int j = t + u * kSortNT;
        if (j < n) {
            const uint32_t k = skv[j].x;
            const int64_t dst = seg0 + (int64_t)(base[(k >> shift) & 255u] + (uint32_t)j);
            kout[dst] = k;
            out.store(vout, dst, pay[u]);
        }
    }
    __syncthreads();  // shared memory is rewritten by the next tile
    }
}

// Builds the tile table: segment b = [seg_lo[b], seg_lo[b+1]) gets
// ceil(len/kSortTile) tiles numbered from seg_tile[b].
static __global__ void seg_tiles_kernel(const int64_t* __restrict__ seg_lo, int64_t n_seg,
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

static __global__ void seg_tile_count_kernel(const int64_t* __restrict__ seg_lo, int64_t n_seg,
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
        seg_hist_kernel<<<(unsigned)n_tiles, 256, 0, s>>>(ki, tlo.ptr, thi.ptr, n_tiles, shift,
                                                          hist.ptr);
        seg_offsets_kernel<<<(unsigned)n_seg, 256, 0, s>>>(d_seg_lo, seg_tile.ptr, hist.ptr);
        if (gather && shift + 8 >= key_bits)
            seg_scatter_kernel<Last><<<(unsigned)n_tiles, kSortNT, 0, s>>>(
                ki, vi, ko, vo, tlo.ptr, thi.ptr, tseg.ptr, n_tiles, shift, hist.ptr, last);
        else
            seg_scatter_kernel<PlainValue><<<(unsigned)n_tiles, kSortNT, 0, s>>>(
                ki, vi, ko, vo, tlo.ptr, thi.ptr, tseg.ptr, n_tiles, shift, hist.ptr,
                PlainValue{});
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

// The tile table of a whole epoch, built on the host from the segment
// bounds, so that sorting a range of segments needs no host round trip.
struct SortTiles {
    DevBuf<int64_t> seg_tile, tlo, thi, tseg;  // seg_tile: first tile of each segment (n_seg + 1)
    DevBuf<uint32_t> hist;                    // 256 counters / offsets per tile
    std::vector<int64_t> h_seg_tile;
    int64_t n_tiles = 0;
};

inline void build_sort_tiles(int device, cudaStream_t s, const std::vector<int64_t>& h_seg,
                             int64_t n_seg, SortTiles& T) {
    T.h_seg_tile.assign(n_seg + 1, 0);
    for (int64_t b = 0; b < n_seg; ++b)
        T.h_seg_tile[b + 1] = T.h_seg_tile[b] + ceil_div(h_seg[b + 1] - h_seg[b], kSortTile);
    T.n_tiles = T.h_seg_tile[n_seg];
    std::vector<int64_t> lo(T.n_tiles), hi(T.n_tiles), sg(T.n_tiles);
    for (int64_t b = 0; b < n_seg; ++b) {
        int64_t t = T.h_seg_tile[b];
        for (int64_t p = h_seg[b]; p < h_seg[b + 1]; p += kSortTile, ++t) {
            lo[t] = p;
            hi[t] = std::min<int64_t>(p + kSortTile, h_seg[b + 1]);
            sg[t] = h_seg[b];
        }
    }
    T.seg_tile.alloc(device, n_seg + 1);
    h2d(T.seg_tile.ptr, T.h_seg_tile.data(), n_seg + 1, s, "sort tiles");
    const int64_t nt = std::max<int64_t>(T.n_tiles, 1);
    T.tlo.alloc(device, nt);
    T.thi.alloc(device, nt);
    T.tseg.alloc(device, nt);
    T.hist.alloc(device, (size_t)nt * 256);
    if (T.n_tiles > 0) {
        h2d(T.tlo.ptr, lo.data(), T.n_tiles, s, "sort tiles");
        h2d(T.thi.ptr, hi.data(), T.n_tiles, s, "sort tiles");
        h2d(T.tseg.ptr, sg.data(), T.n_tiles, s, "sort tiles");
    }
    MFM_CUDA(cudaStreamSynchronize(s), "sort tiles");  // the host vectors go out of scope
}

// segmented_sort restricted to segments [b0, b1) with the epoch tile table T;
// no host synchronisation. Same buffer rules as segmented_sort. With iota,
// the values are each entry's position relative to its segment start: the
// first pass generates them and v0 is not read. max_grid > 0 caps the tile
// kernels' grids (their blocks then stride over the tiles), so that a sort
// running beside other work leaves room for it.
template <class Last = PlainValue>
SortResult segmented_sort_range(cudaStream_t s, const uint32_t* kfirst, uint32_t* k0, uint32_t* v0,
                                uint32_t* k1, uint32_t* v1, const int64_t* d_seg_lo, int64_t b0,
                                int64_t b1, SortTiles& T, int key_bits, Last last = Last{},
                                bool iota = false, unsigned max_grid = 0) {
    SortResult res{k0, v0};
    constexpr bool gather = !std::is_same<Last, PlainValue>::value;
    if (gather && key_bits < 1) key_bits = 1;
    const int64_t t0 = T.h_seg_tile[b0], t1 = T.h_seg_tile[b1];
    const uint32_t* ki = kfirst ? kfirst : k0;
    uint32_t *vi = v0, *ko = k1, *vo = v1;
    if (t1 > t0 && key_bits > 0) {
        const int64_t ntl = t1 - t0;
        const unsigned nt = (unsigned)(max_grid > 0 && ntl > (int64_t)max_grid ? max_grid : ntl),
                       ns = (unsigned)(b1 - b0);
        const int64_t* tlo = T.tlo.ptr + t0;
        const int64_t* thi = T.thi.ptr + t0;
        const int64_t* tsg = T.tseg.ptr + t0;
        uint32_t* hist = T.hist.ptr + t0 * 256;
        for (int shift = 0; shift < key_bits; shift += 8) {
            seg_hist_kernel<<<nt, 256, 0, s>>>(ki, tlo, thi, ntl, shift, hist);
            seg_offsets_kernel<<<ns, 256, 0, s>>>(d_seg_lo + b0, T.seg_tile.ptr + b0, T.hist.ptr);
            const bool gen = iota && shift == 0;
            if (gather && shift + 8 >= key_bits) {
                if (gen)
                    seg_scatter_kernel<Last, true><<<nt, kSortNT, 0, s>>>(
                        ki, vi, ko, vo, tlo, thi, tsg, ntl, shift, hist, last);
                else
                    seg_scatter_kernel<Last><<<nt, kSortNT, 0, s>>>(ki, vi, ko, vo, tlo, thi,
                                                                    tsg, ntl, shift, hist, last);
            } else if (gen) {
                seg_scatter_kernel<PlainValue, true><<<nt, kSortNT, 0, s>>>(
                    ki, vi, ko, vo, tlo, thi, tsg, ntl, shift, hist, PlainValue{});
            } else {
                seg_scatter_kernel<PlainValue><<<nt, kSortNT, 0, s>>>(
                    ki, vi, ko, vo, tlo, thi, tsg, ntl, shift, hist, PlainValue{});
            }
            MFM_CHECK_LAUNCH("segmented sort launch");
            uint32_t* nk = ko == k1 ? k0 : k1;
            uint32_t* nv = vo == v1 ? v0 : v1;
            ki = ko;
            vi = vo;
            ko = nk;
            vo = nv;
        }
    } else if (key_bits > 0) {  // no entries: report where a sort would have ended
        const int passes = (key_bits + 7) / 8;
        ki = passes % 2 ? k1 : k0;
        vi = passes % 2 ? v1 : v0;
    }
    res.keys = const_cast<uint32_t*>(ki);
    res.vals = vi;
    return res;
}

}  // namespace mfm
