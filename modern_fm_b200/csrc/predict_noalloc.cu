// predict_noalloc.cu — FM scoring that allocates no device memory.
//
// Some callers cannot let a library allocate GPU memory: a host that owns the
// whole device budget through its own pool (a serving runtime or an embedding
// application that pre-reserves memory), or a latency-bound loop that cannot
// afford cudaMalloc / cudaFree, which may synchronise the device and stall
// every stream. mfm_fm_predict_csr_noalloc serves them: it computes exactly
// what mfm_fm_predict_csr computes, but stages the CSR, the parameters, the
// validation flags and the scores in one file-scope device array of
// kNoAllocScratchBytes (64 MiB) instead of allocating. Inputs that do not fit
// are rejected with MFM_ERR_UNSUPPORTED before any device work.
//
// The array is part of this file's device code module, which the CUDA runtime
// loads lazily (CUDA 12 loads modules on first use): the first call on each
// device loads it and so reserves the 64 MiB there, and every GPU that has
// made a call holds it until the process exits. A caller that reserves the
// rest of the device for its own pool makes its first call (any valid input)
// before reserving the pool, and before any stream capture. All calls share
// the array and it keeps the previous call's contents; the validation flags are
// cleared at the start of every call. Calls are serialised per device by the
// engine's device lock and run on the engine's stream for that device;
// calls that overlapped on the GPU would race on the shared array.
//
// MFM_DTYPE_F32_F64 scores with the float64 parameters it stages: the same
// float64 arithmetic on the caller's values.
#include "common.cuh"

namespace mfm {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// kernels and launchers defined in runtime.cu / predict.cu
__global__ void csr_check_kernel(const int64_t* __restrict__ indptr, int64_t n_rows,
                                 const int64_t* __restrict__ indices, int64_t nnz,
                                 int64_t n_features, unsigned int* flags);
__global__ void f64_to_f32_kernel(const double* __restrict__ src, float* __restrict__ dst,
                                  int64_t n);
void fm_launch_staged_f64(int device, cudaStream_t s, const int64_t* indptr,
                          const int64_t* indices, const double* data, int64_t n_rows,
                          double w0, const double* w, const double* v, int k, double* out);
void fm_launch_staged_f32(int device, cudaStream_t s, const int64_t* indptr,
                          const int64_t* indices, const double* data, int64_t n_rows,
                          double w0, const float* w, const float* v, int k, double* out);

namespace {

constexpr int kMaxDev = 64;
std::mutex g_setup_mu;
unsigned char* g_scratch_addr[kMaxDev];

// Device address of the static array on `device` (which must be current).
// Looked up once per device, on that device's first call.
unsigned char* scratch_address(int device) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        MFM_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "static scratch address lookup");
        g_scratch_addr[device] = static_cast<unsigned char*>(p);
    }
    return g_scratch_addr[device];
}

// Bump allocation of 256-byte aligned regions inside the static array.
struct Carve {
    unsigned char* base;
    size_t used = 0;
    template <class T>
    T* take(size_t count) {
        T* p = reinterpret_cast<T*>(base + used);
        used += (count * sizeof(T) + 255) / 256 * 256;
        return p;
    }
};

size_t region(size_t bytes) { return (bytes + 255) / 256 * 256; }

}  // namespace
}  // namespace mfm

using namespace mfm;

extern "C" int mfm_fm_predict_csr_noalloc(const mfm_csr* x, double w0, const double* w,
                                          const double* v, int64_t k, double* out,
                                          const mfm_exec* ex) {
    return guarded([&] {
        check_csr_host(x);
        if (x->n_rows == 0) return;
        if (k < 1 || k > 1024)
            fail(MFM_ERR_UNSUPPORTED,
                 fmt("CUDA FM prediction supports 1 <= k <= 1024, got %lld", (long long)k));
        const int dtype = ex ? ex->dtype : MFM_DTYPE_F64;
        const int device = ex ? ex->device : 0;
        if (dtype != MFM_DTYPE_F64 && dtype != MFM_DTYPE_F32 && dtype != MFM_DTYPE_F32_F64)
            fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
        const int64_t n = x->n_rows, nnz = x->nnz, nf = x->n_features;
        size_t need = region(sizeof(unsigned int)) + region((n + 1) * 8) + 2 * region(nnz * 8) +
                      region(nf * 8) + region(nf * k * 8) + region(n * 8);
        if (dtype == MFM_DTYPE_F32) need += region(nf * 4) + region(nf * k * 4);
        if (need > kNoAllocScratchBytes)
            fail(MFM_ERR_UNSUPPORTED,
                 fmt("input needs %zu bytes of device staging, more than the %zu-byte static "
                     "scratch of the allocation-free entry point; use mfm_fm_predict_csr",
                     need, kNoAllocScratchBytes));
        DeviceGuard guard(device);
        std::lock_guard<std::mutex> lk(device_mutex(device));
        // the engine's non-blocking stream for this device (created by the
        // engine's first call on the device; no device memory is allocated)
        cudaStream_t s = device_stream(device);
        Carve c{scratch_address(device)};
        unsigned int* flags = c.take<unsigned int>(1);
        int64_t* d_indptr = c.take<int64_t>(n + 1);
        int64_t* d_indices = c.take<int64_t>(nnz);
        double* d_data = c.take<double>(nnz);
        double* d_w = c.take<double>(nf);
        double* d_v = c.take<double>(nf * k);
        double* d_out = c.take<double>(n);
        MFM_CUDA(cudaMemsetAsync(flags, 0, sizeof(unsigned int), s), "flag clear");
        h2d(d_indptr, x->indptr, n + 1, s, "indptr upload");
        h2d(d_indices, x->indices, nnz, s, "indices upload");
        h2d(d_data, x->data, nnz, s, "data upload");
        h2d(d_w, w, nf, s, "w upload");
        h2d(d_v, v, nf * k, s, "V upload");
        const int64_t work = n > nnz ? n : nnz;
        const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(work, 256) + 1,
                                                          (int64_t)sm_count(device) * 8);
        csr_check_kernel<<<grid, 256, 0, s>>>(d_indptr, n, d_indices, nnz, nf, flags);
        MFM_CHECK_LAUNCH("CSR check launch");
        unsigned int h = 0;
        d2h(&h, flags, 1, s, "CSR check download");
        MFM_CUDA(cudaStreamSynchronize(s), "CSR check");
        if (h & 1u) fail(MFM_ERR_INVALID, "indptr must be non-decreasing");
        if (h & 2u)
            fail(MFM_ERR_INVALID, fmt("column index out of range [0, %lld)", (long long)nf));
        if (dtype != MFM_DTYPE_F32) {
            fm_launch_staged_f64(device, s, d_indptr, d_indices, d_data, n, w0, d_w, d_v, (int)k,
                                 d_out);
        } else {
            float* w32 = c.take<float>(nf);
            float* v32 = c.take<float>(nf * k);
            const unsigned g2 = (unsigned)std::min<int64_t>(ceil_div(nf * k, 256) + 1,
                                                            (int64_t)sm_count(device) * 8);
            f64_to_f32_kernel<<<g2, 256, 0, s>>>(d_w, w32, nf);
            f64_to_f32_kernel<<<g2, 256, 0, s>>>(d_v, v32, nf * k);
            MFM_CHECK_LAUNCH("parameter conversion");
            fm_launch_staged_f32(device, s, d_indptr, d_indices, d_data, n, w0, w32, v32, (int)k,
                                 d_out);
        }
        d2h(out, d_out, n, s, "output download");
        MFM_CUDA(cudaStreamSynchronize(s), "predict");
    });
}

extern "C" int64_t mfm_noalloc_scratch_bytes(void) { return (int64_t)kNoAllocScratchBytes; }
