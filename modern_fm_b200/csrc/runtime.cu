// runtime.cu — error state, device/stream management, caching allocator,
// input validation and the small utility entry points of the C ABI.
#include <map>
#include <unordered_map>

#include "common.cuh"

namespace mfm {

// ---------------------------------------------------------------- errors --

static thread_local std::string g_last_error;

std::string fmt(const char* f, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof(buf), f, ap);
    va_end(ap);
    return std::string(buf);
}

void fail(int code, const std::string& msg) { throw Error(code, msg); }
void set_last_error(const std::string& msg) { g_last_error = msg; }

// ------------------------------------------------------- device context --

static constexpr int kMaxDevices = 64;

DeviceGuard::DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    int n = device_count();
    if (n <= 0) fail(MFM_ERR_NO_DEVICE, "no CUDA device available");
    if (device < 0 || device >= n)
        fail(MFM_ERR_INVALID, fmt("device %d out of range [0, %d)", device, n));
    MFM_CUDA(cudaSetDevice(device), "set device");
}
DeviceGuard::~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
}

int device_count() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky "no device" status
        return 0;
    }
    return n;
}

static std::mutex g_dev_mu[kMaxDevices];
static cudaStream_t g_streams[kMaxDevices];
static int g_sms[kMaxDevices];
static std::mutex g_init_mu;

std::mutex& device_mutex(int device) { return g_dev_mu[device % kMaxDevices]; }

cudaStream_t device_stream(int device) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (!g_streams[device]) {
        cudaStream_t s;
        MFM_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
        g_streams[device] = s;
    }
    return g_streams[device];
}

cudaStream_t side_stream(int device, int which) {
    static cudaStream_t streams[kMaxDevices][2] = {};
    std::lock_guard<std::mutex> lk(g_init_mu);
    cudaStream_t& st = streams[device % kMaxDevices][which & 1];
    if (!st) {
        int least = 0, greatest = 0;
        MFM_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
        MFM_CUDA(cudaStreamCreateWithPriority(&st, cudaStreamNonBlocking,
                                              which == 0 ? greatest : least),
                 "stream create");
    }
    return st;
}

int sm_count(int device) {
    if (!g_sms[device]) {
        int v = 0;
        MFM_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device),
                 "device attribute");
        g_sms[device] = v;
    }
    return g_sms[device];
}

// ------------------------------------------------------ caching allocator --

namespace {
struct Pool {
    std::mutex mu;
    std::multimap<size_t, void*> free_blocks[kMaxDevices];
    std::unordered_map<void*, size_t> sizes[kMaxDevices];
};
Pool& pool() {
    static Pool* p = new Pool();  // never destroyed: outlives static teardown
    return *p;
}
size_t round_bytes(size_t b) {
    const size_t small = 512, big = size_t(2) << 20;
    return b >= big ? (b + big - 1) / big * big : (b + small - 1) / small * small;
}
}  // namespace

void* pool_alloc(int device, size_t bytes) {
    Pool& P = pool();
    size_t want = round_bytes(bytes);
    {
        std::lock_guard<std::mutex> lk(P.mu);
        auto& fb = P.free_blocks[device];
        auto it = fb.lower_bound(want);
        if (it != fb.end() && it->first <= 2 * want) {
            void* p = it->second;
            fb.erase(it);
            return p;
        }
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        // release this device's cache and retry once
        {
            std::lock_guard<std::mutex> lk(P.mu);
            for (auto& kv : P.free_blocks[device]) {
                cudaFree(kv.second);
                P.sizes[device].erase(kv.second);
            }
            P.free_blocks[device].clear();
        }
        e = cudaMalloc(&p, want);
        if (e != cudaSuccess) {
            cudaGetLastError();
            fail(MFM_ERR_CUDA, fmt("CUDA allocation of %zu bytes failed: %s", want,
                                   cudaGetErrorString(e)));
        }
    }
    std::lock_guard<std::mutex> lk(P.mu);
    P.sizes[device][p] = want;
    return p;
}

void pool_free(int device, void* p) {
    if (!p) return;
    Pool& P = pool();
    std::lock_guard<std::mutex> lk(P.mu);
    auto it = P.sizes[device].find(p);
    size_t sz = it == P.sizes[device].end() ? 0 : it->second;
    P.free_blocks[device].emplace(sz, p);
}

void pool_release_all() {
    Pool& P = pool();
    std::lock_guard<std::mutex> lk(P.mu);
    int prev = -1;
    cudaGetDevice(&prev);
    for (int d = 0; d < kMaxDevices; ++d) {
        if (P.free_blocks[d].empty()) continue;
        cudaSetDevice(d);
        cudaDeviceSynchronize();
        for (auto& kv : P.free_blocks[d]) {
            cudaFree(kv.second);
            P.sizes[d].erase(kv.second);
        }
        P.free_blocks[d].clear();
    }
    if (prev >= 0) cudaSetDevice(prev);
}

// ------------------------------------------------------------ validation --

void check_csr_host(const mfm_csr* x) {
    if (!x || !x->indptr) fail(MFM_ERR_INVALID, "indptr must have length n_rows + 1 (>= 1)");
    if (x->n_rows < 0) fail(MFM_ERR_INVALID, "indptr must have length n_rows + 1 (>= 1)");
    if (x->nnz < 0 || x->n_features < 0) fail(MFM_ERR_INVALID, "negative CSR size");
    if (x->indptr[x->n_rows] != x->nnz || x->indptr[0] != 0)
        fail(MFM_ERR_INVALID, "indptr must start at 0 and end at nnz");
    if (x->nnz > 0 && (!x->indices || !x->data))
        fail(MFM_ERR_INVALID, "indices and data must be provided when nnz > 0");
    if (x->n_features > INT32_MAX)
        fail(MFM_ERR_UNSUPPORTED, fmt("n_features %lld exceeds the engine's 2^31-1 limit",
                                      (long long)x->n_features));
}

void check_field_ids(const int64_t* field_ids, int64_t n_features, int64_t n_fields) {
    if (n_fields < 1 && n_features > 0) fail(MFM_ERR_INVALID, "field id out of range [0, 0)");
    for (int64_t i = 0; i < n_features; ++i)
        if (field_ids[i] < 0 || field_ids[i] >= n_fields)
            fail(MFM_ERR_INVALID, fmt("field id out of range [0, %lld)", (long long)n_fields));
}

__global__ void csr_check_kernel(const int64_t* __restrict__ indptr, int64_t n_rows,
                                 const int64_t* __restrict__ indices, int64_t nnz,
                                 int64_t n_features, unsigned int* flags) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    bool bad_order = false, bad_idx = false;
    for (int64_t r = t0; r < n_rows; r += stride) bad_order |= indptr[r + 1] < indptr[r];
    for (int64_t q = t0; q < nnz; q += stride) {
        int64_t i = indices[q];
        bad_idx |= (i < 0) | (i >= n_features);
    }
    if (__any_sync(0xffffffffu, bad_order) && (threadIdx.x & 31) == 0) atomicOr(flags, 1u);
    if (__any_sync(0xffffffffu, bad_idx) && (threadIdx.x & 31) == 0) atomicOr(flags, 2u);
}

void validate_csr_device(int device, cudaStream_t s, const int64_t* d_indptr, int64_t n_rows,
                         const int64_t* d_indices, int64_t nnz, int64_t n_features) {
    DevBuf<unsigned int> flags(device, 1);
    MFM_CUDA(cudaMemsetAsync(flags.ptr, 0, sizeof(unsigned int), s), "memset");
    int64_t work = n_rows > nnz ? n_rows : nnz;
    unsigned grid = (unsigned)std::min<int64_t>(ceil_div(work, 256) + 1,
                                                (int64_t)sm_count(device) * 8);
    csr_check_kernel<<<grid, 256, 0, s>>>(d_indptr, n_rows, d_indices, nnz, n_features,
                                          flags.ptr);
    MFM_CHECK_LAUNCH("CSR check launch");
    unsigned int h = 0;
    d2h(&h, flags.ptr, 1, s, "CSR check download");
    MFM_CUDA(cudaStreamSynchronize(s), "CSR check");
    if (h & 1u) fail(MFM_ERR_INVALID, "indptr must be non-decreasing");
    if (h & 2u)
        fail(MFM_ERR_INVALID, fmt("column index out of range [0, %lld)", (long long)n_features));
}

}  // namespace mfm

// ------------------------------------------------------------------ C ABI --

extern "C" int mfm_has_cuda(void) { return mfm::device_count() > 0 ? 1 : 0; }

extern "C" const char* mfm_last_error(void) { return mfm::g_last_error.c_str(); }

extern "C" int mfm_device_count(void) { return mfm::device_count(); }

extern "C" void mfm_release_cached_memory(void) { mfm::pool_release_all(); }
