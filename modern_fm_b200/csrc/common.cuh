// common.cuh — shared runtime pieces of the B200 engine: error reporting,
// the per-device caching allocator and stream, warp helpers, vector types.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mfm_b200.h"

namespace mfm {

// ---------------------------------------------------------------- errors --

// Internal exception carrying an ABI return code; every extern "C" entry
// point catches it and stores the message for mfm_last_error().
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

std::string fmt(const char* f, ...);
[[noreturn]] void fail(int code, const std::string& msg);
void set_last_error(const std::string& msg);

#define MFM_CUDA(call, what)                                                        \
    do {                                                                            \
        cudaError_t e_ = (call);                                                    \
        if (e_ != cudaSuccess)                                                      \
            ::mfm::fail(MFM_ERR_CUDA, ::mfm::fmt("CUDA %s failed: %s", (what),      \
                                                 cudaGetErrorString(e_)));          \
    } while (0)

#define MFM_CHECK_LAUNCH(what) MFM_CUDA(cudaGetLastError(), what)

// Runs `body` and converts exceptions to an ABI return code.
template <class F>
int guarded(F&& body) {
    try {
        body();
        return MFM_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return MFM_ERR_CUDA;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return MFM_ERR_CUDA;
    }
}

// ------------------------------------------------------- device context --

// Selects `device` for the calling thread and restores the previous device
// on destruction.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int device);
    ~DeviceGuard();
};

// One non-blocking stream per device, shared by all calls on that device;
// calls on a device serialise on its mutex (the reference serialises on its
// cached context's default stream, rust/src/cuda/mod.rs:53-64).
cudaStream_t device_stream(int device);
std::mutex& device_mutex(int device);
int device_count();
int sm_count(int device);

// Per-device streams for work that runs beside the caller's stream: which = 0
// has the device's greatest priority, which = 1 its least.
cudaStream_t side_stream(int device, int which);

// Caching allocator: freed blocks are kept per device and reused for
// requests up to 2x smaller; on cudaMalloc failure the cache is released and
// the allocation retried once.
void* pool_alloc(int device, size_t bytes);
void pool_free(int device, void* p);
void pool_release_all();

template <class T>
struct DevBuf {
    T* ptr = nullptr;
    size_t n = 0;
    int dev = -1;
    DevBuf() = default;
    DevBuf(int device, size_t count) { alloc(device, count); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : ptr(o.ptr), n(o.n), dev(o.dev) { o.ptr = nullptr; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        reset();
        ptr = o.ptr;
        n = o.n;
        dev = o.dev;
        o.ptr = nullptr;
        return *this;
    }
    void alloc(int device, size_t count) {
        reset();
        dev = device;
        n = count;
        ptr = static_cast<T*>(pool_alloc(device, (count ? count : 1) * sizeof(T)));
    }
    void reset() {
        if (ptr) pool_free(dev, ptr);
        ptr = nullptr;
        n = 0;
    }
    ~DevBuf() { reset(); }
    size_t bytes() const { return n * sizeof(T); }
};

// Host->device / device->host copies on the device stream.
template <class T>
void h2d(T* dst, const T* src, size_t count, cudaStream_t s, const char* what) {
    if (count) MFM_CUDA(cudaMemcpyAsync(dst, src, count * sizeof(T), cudaMemcpyHostToDevice, s), what);
}
template <class T>
void d2h(T* dst, const T* src, size_t count, cudaStream_t s, const char* what) {
    if (count) MFM_CUDA(cudaMemcpyAsync(dst, src, count * sizeof(T), cudaMemcpyDeviceToHost, s), what);
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Grid size for a warp-per-item kernel: enough blocks to fill the GPU
// (a multiple of the SM count), never more than the work needs.
inline unsigned warp_grid(int device, int64_t items, int warps_per_block, int blocks_per_sm) {
    int64_t want = ceil_div(items, warps_per_block);
    int64_t cap = (int64_t)sm_count(device) * blocks_per_sm;
    if (want > cap) want = cap;
    return (unsigned)(want < 1 ? 1 : want);
}

// ---------------------------------------------------------- validation --

// CsrView::new (rust/src/data.rs:14-44), O(1) host part: lengths and the
// indptr end points. The O(nnz) part runs on the device (validate_csr_device).
void check_csr_host(const mfm_csr* x);
// check_field_ids (rust/src/data.rs:71-83).
void check_field_ids(const int64_t* field_ids, int64_t n_features, int64_t n_fields);
// Device-side O(nnz) CSR checks: indptr non-decreasing, every index in
// [0, n_features). Throws MFM_ERR_INVALID with the reference's messages.
void validate_csr_device(int device, cudaStream_t s, const int64_t* d_indptr, int64_t n_rows,
                         const int64_t* d_indices, int64_t nnz, int64_t n_features);

}  // namespace mfm

// ------------------------------------------------------------ device side --

namespace mfm {

template <class T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <class T, int N>
struct alignas(sizeof(T) * N) Vec {
    T v[N];
};

template <class T, int N>
__device__ __forceinline__ Vec<T, N> ldg_vec(const T* p) {
    return *reinterpret_cast<const Vec<T, N>*>(p);
}

}  // namespace mfm
