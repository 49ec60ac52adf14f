// scan.cuh — device-wide exclusive prefix sum (reduce-then-scan, three
// launches, deterministic) and block-level scan helpers.
#pragma once

#include "common.cuh"

namespace mfm {

// Exclusive scan of one value per thread over a block of NT threads.
// `smem` holds NT/32 elements. Returns the prefix; `total` gets the sum.
template <class T, int NT>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem, T& total) {
    static_assert(NT % 32 == 0 && NT <= 1024, "block size");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem[warp] = x;
    __syncthreads();
    if (warp == 0) {
        T t = lane < NT / 32 ? smem[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            T y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < NT / 32) smem[lane] = t;
    }
    __syncthreads();
    const T before = warp > 0 ? smem[warp - 1] : T(0);
    total = smem[NT / 32 - 1];
    __syncthreads();
    return before + x - v;
}

constexpr int kScanNT = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanNT * kScanItems;

template <class Tin, class Tout>
__global__ void __launch_bounds__(kScanNT)
    scan_reduce_kernel(const Tin* __restrict__ in, int64_t n, Tout* __restrict__ sums) {
    __shared__ Tout sm[kScanNT / 32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    Tout s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i)
        if (base + i < n) s += (Tout)in[base + i];
    Tout total;
    block_exclusive_scan<Tout, kScanNT>(s, sm, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Exclusive scan of sums[0..nb) in place by one block; sums[nb] = total.
template <class T>
__global__ void __launch_bounds__(kScanNT) scan_sums_kernel(T* sums, int64_t nb) {
    __shared__ T sm[kScanNT / 32];
    T carry = 0;
    for (int64_t base = 0; base < nb; base += kScanNT) {
        const int64_t i = base + threadIdx.x;
        const T v = i < nb ? sums[i] : T(0);
        T total;
        const T ex = block_exclusive_scan<T, kScanNT>(v, sm, total);
        if (i < nb) sums[i] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) sums[nb] = carry;
}

template <class Tin, class Tout>
__global__ void __launch_bounds__(kScanNT)
    scan_apply_kernel(const Tin* __restrict__ in, int64_t n, const Tout* __restrict__ sums,
                      Tout* __restrict__ out) {
    __shared__ Tout sm[kScanNT / 32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    Tout v[kScanItems];
    Tout s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        v[i] = base + i < n ? (Tout)in[base + i] : Tout(0);
        s += v[i];
    }
    Tout total;
    Tout run = block_exclusive_scan<Tout, kScanNT>(s, sm, total) + sums[blockIdx.x];
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        if (base + i < n) out[base + i] = run;
        run += v[i];
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == kScanNT - 1) out[n] = run;
}

// out[0..n] = exclusive prefix sums of in[0..n), out[n] = total. `in` and
// `out` may alias only if Tin == Tout. Uses a scratch of ceil(n/4096)+1.
template <class Tin, class Tout>
void exclusive_scan(int device, cudaStream_t s, const Tin* in, int64_t n, Tout* out) {
    const int64_t nb = n > 0 ? ceil_div(n, kScanTile) : 1;
    DevBuf<Tout> sums(device, nb + 1);
    scan_reduce_kernel<Tin, Tout><<<(unsigned)nb, kScanNT, 0, s>>>(in, n, sums.ptr);
    scan_sums_kernel<Tout><<<1, kScanNT, 0, s>>>(sums.ptr, nb);
    scan_apply_kernel<Tin, Tout><<<(unsigned)nb, kScanNT, 0, s>>>(in, n, sums.ptr, out);
    MFM_CHECK_LAUNCH("scan launch");
}

}  // namespace mfm
