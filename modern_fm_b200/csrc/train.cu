// train.cu — device-resident mini-batch training for FM, FFM and FwFM
// (binary and multiclass softmax) on sm_100a: the host side (Trainer: plan,
// batch loop, uploads and downloads, data-parallel groups) and the C ABI. It
// replaces the reference's cuda::{fm,ffm,fwfm}_train[_mc] host loops
// (rust/src/cuda/*_train*.rs), which accumulate with float atomics on the
// GPU and then download every batch's gradient for a CPU optimizer flush.
//
// Semantics follow the reference's CPU engine (rust/src/{fm,ffm,fwfm}.rs):
// every batch (a contiguous chunk of row_orders[e]) computes per-row gradients
// from the frozen batch-start parameters, sums them per touched coordinate,
// divides by the batch length and applies one optimizer step per touched
// coordinate (lazy L2; update sets: features for w and FM/FwFM V, (feature,
// field) slots hit by a pair for FFM V, hit field pairs for FwFM R; w0 always).
//
// Per epoch, for each entry stream (FEAT: one entry per nonzero keyed by
// feature; SLOT: one per ordered pair keyed by FFM slot; PAIR: one per
// unordered pair keyed by FwFM field pair): count -> scan -> expand ->
// segmented stable radix sort by key within each batch (segsort.cuh). Then,
// per batch, no float atomics anywhere (bitwise reproducible run to run):
//   binary FM, k = 1/2/4/8 16-byte vectors (train_tab.cuh): the forward writes
//     one row-table line per row (S) and the row's g; stage 1 recomputes each
//     sorted entry's gradient from them, reduces segments and steps the
//     optimizer; stage 2 folds runs that cross chunk boundaries and steps w0;
//   every other shape (train_payload.cuh): the forward writes each entry's
//     gradient payload to its sorted position; stage 1 sums work items of
//     <= kItem entries and steps single-item runs; stage 2 folds multi-item
//     runs and steps w0.
// Kernels: train_opt.cuh (optimizer, launch order), train_plan.cuh (plan),
// train_forward.cuh (forward), train_payload.cuh, train_tab.cuh (reductions).
#include <algorithm>
#include <chrono>
#include <thread>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <nccl.h>
#include <mutex>
#include <utility>
#include <cmath>

#include "train_tab.cuh"
#include "train_shard.cuh"
#include "scan.cuh"

// A data-parallel group: one NCCL communicator bound to a device.
struct mfm_dp {
    ncclComm_t comm;
    int world, rank, device;
    // mapped host words written by the device: [0] batches whose cross-rank
    // sum has completed (the host's liveness view of the group), [1] set when
    // a wait for a peer's flag gave up
    unsigned* prog_h;
    unsigned* prog_d;
    bool aborted;  // the communicator was aborted after a failure
    // Peer-memory exchange: one device buffer per rank, exported by CUDA IPC
    // and mapped by every other rank: a flag area (the rank's exchange count,
    // a failure word), then the exchange data. seq counts the group's
    // exchanges (the same on every rank; flags hold it, so they never reset).
    void* sym = nullptr;
    size_t sym_bytes = 0;
    std::vector<void*> peer;  // every rank's buffer as mapped here (own at [rank])
    unsigned long long seq = 0;
    int p2p = -1;  // -1 not set up, 0 unavailable (NCCL exchange), 1 mapped
};

namespace mfm {

// ----------------------------------------------------------------- host --

// Phase timing on the training stream, printed to stderr when the
// environment variable MFM_B200_TIMING is set (diagnostics only).
// Phase times of the calling thread's last fit (seconds): upload, plan,
// batches, download (mfm_fit_phase_seconds).
thread_local double g_phase_s[4] = {0.0, 0.0, 0.0, 0.0};

struct PhaseTimer {
    bool print = false;
    cudaStream_t s = nullptr;
    cudaEvent_t last = nullptr;
    std::string report;
    explicit PhaseTimer(cudaStream_t st) : s(st) {
        const char* e = getenv("MFM_B200_TIMING");
        print = e && *e && *e != '0';
        for (double& v : g_phase_s) v = 0.0;
        if (cudaEventCreate(&last) == cudaSuccess) cudaEventRecord(last, s);
    }
    // marks the end of a phase on stream s (the engine synchronises at every
    // phase boundary anyway: uploads, the plan's host round trips, the end of
    // an epoch's batches)
    void mark(const char* name) {
        if (!last) return;
        cudaEvent_t now;
        if (cudaEventCreate(&now) != cudaSuccess) return;
        cudaEventRecord(now, s);
        cudaEventSynchronize(now);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, last, now);
        cudaEventDestroy(last);
        last = now;
        const std::string n(name);
        const int slot = n == "upload" || n == "setup" ? 0 : n == "plan" ? 1
                         : n == "batches" ? 2 : n == "download" ? 3 : -1;
        if (slot >= 0) g_phase_s[slot] += ms * 1e-3;
        if (print) report += fmt(" %s=%.3fms", name, ms);
    }
    ~PhaseTimer() {
        if (last) cudaEventDestroy(last);
        if (print) fprintf(stderr, "mfm timing:%s\n", report.c_str());
    }
};

// Launch with programmatic stream serialization (see pdl_wait): the kernel may
// start while its predecessor in the stream drains. MFM_B200_PDL=0 turns the
// attribute off (plain stream order; the kernels' waits return at once).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("MFM_B200_PDL");
        return !(e && *e == '0');
    }();
    return on;
}

template <class... KArgs, class... Args>
void launch_pdl(void (*kern)(KArgs...), unsigned grid, unsigned block, cudaStream_t s,
                Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    MFM_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), "kernel launch");
}

unsigned blocks_for(int64_t n, int nt) { return (unsigned)std::max<int64_t>(1, ceil_div(n, nt)); }

int bits_for(int64_t n_keys) {
    int b = 0;
    while (b < 32 && ((int64_t)1 << b) < n_keys) ++b;
    return b;
}

// NCCL, loaded on first use (dlopen): a process that already holds a libnccl
// (e.g. PyTorch's) resolves to it, others to the system library; the engine
// never links NCCL, so single-GPU use does not depend on it.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                              ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
};
inline const NcclApi& nccl() {
    static const NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
        a.AllReduce = (decltype(a.AllReduce))dlsym(h, "ncclAllReduce");
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
        a.CommAbort = (decltype(a.CommAbort))dlsym(h, "ncclCommAbort");
        a.CommGetAsyncError = (decltype(a.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        a.GroupStart = (decltype(a.GroupStart))dlsym(h, "ncclGroupStart");
        a.GroupEnd = (decltype(a.GroupEnd))dlsym(h, "ncclGroupEnd");
        a.Broadcast = (decltype(a.Broadcast))dlsym(h, "ncclBroadcast");
        a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
        return a;
    }();
    if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.CommDestroy ||
        !api.CommAbort || !api.CommGetAsyncError || !api.GetErrorString || !api.GroupStart ||
        !api.GroupEnd || !api.Broadcast || !api.AllGather)
        fail(MFM_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    return api;
}
#define MFM_NCCL(call, what)                                                          \
    do {                                                                              \
        const ncclResult_t r_ = (call);                                               \
        if (r_ != ncclSuccess)                                                        \
            fail(MFM_ERR_CUDA, fmt("%s: %s", what, nccl().GetErrorString(r_)));       \
    } while (0)

// Data-parallel: batches the host may enqueue ahead of the device's progress.
constexpr uint32_t kDpAhead = 64;

// The group's liveness limit in seconds (MFM_B200_DP_TIMEOUT, default 300).
inline double dp_timeout_s() {
    static const double limit = [] {
        const char* e = getenv("MFM_B200_DP_TIMEOUT");
        const double v = e ? atof(e) : 0.0;
        return v > 0.0 ? v : 300.0;
    }();
    return limit;
}

// Waits for stream s under the group's liveness rules: a group error reported
// by NCCL, or no completion within the limit, aborts the communicator, lets
// the stream drain and fails the call.
inline void dp_sync(mfm_dp* dp, cudaStream_t s, const char* what) {
    const double limit = dp_timeout_s();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) return;
        if (q != cudaErrorNotReady) MFM_CUDA(q, what);
        ncclResult_t st = ncclSuccess;
        nccl().CommGetAsyncError(dp->comm, &st);
        const bool failed = st != ncclSuccess && st != ncclInProgress;
        if (failed ||
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit) {
            nccl().CommAbort(dp->comm);
            dp->aborted = true;
            cudaStreamSynchronize(s);  // the aborted collective lets the stream drain
            if (failed)
                fail(MFM_ERR_CUDA, fmt("data-parallel group failed in %s (NCCL: %s); the group "
                                       "was aborted",
                                       what, nccl().GetErrorString(st)));
            fail(MFM_ERR_CUDA, fmt("data-parallel group: %s did not complete in %.0f s (a peer "
                                   "is not answering); the group was aborted",
                                   what, limit));
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// One NCCL allreduce (min) of an int across the group.
inline int dp_all_min(mfm_dp* dp, int v, cudaStream_t s) {
    DevBuf<int> b(dp->device, 1);
    h2d(b.ptr, &v, 1, s, "group agreement");
    const ncclResult_t r = nccl().AllReduce(b.ptr, b.ptr, 1, ncclInt32, ncclMin, dp->comm, s);
    if (r != ncclSuccess) {
        nccl().CommAbort(dp->comm);
        dp->aborted = true;
        cudaStreamSynchronize(s);
        fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group was aborted",
                               nccl().GetErrorString(r)));
    }
    int out = 0;
    d2h(&out, b.ptr, 1, s, "group agreement");
    dp_sync(dp, s, "the group agreement");
    return out;
}

// Unmaps the peers' exchange buffers and frees this rank's, after every rank
// has unmapped (collective unless the group was aborted).
inline void dp_sym_release(mfm_dp* dp, cudaStream_t s) {
    if (!dp->sym) return;
    for (int p = 0; p < (int)dp->peer.size(); ++p)
        if (p != dp->rank && dp->peer[p]) cudaIpcCloseMemHandle(dp->peer[p]);
    dp->peer.clear();
    if (!dp->aborted) dp_all_min(dp, 1, s);
    cudaFree(dp->sym);
    dp->sym = nullptr;
    dp->sym_bytes = 0;
    dp->p2p = -1;
}

// Sets up (or grows) the peer-memory exchange: every rank allocates `need`
// bytes (zeroed), exports them by CUDA IPC and maps every other rank's.
// p2p = 1 when every rank mapped every peer; otherwise 0 and the exchange
// goes through NCCL. Opt-in: MFM_B200_DP_EXCHANGE=peer (the NCCL exchange
// is the default: on 2 B200s it measured faster, 108 against 113 ms per
// 10M-row epoch). Collective: every rank calls it with the same size.
inline void dp_sym_ensure(mfm_dp* dp, size_t need, cudaStream_t s) {
    if (dp->p2p == 0) return;
    if (dp->p2p == 1 && dp->sym_bytes >= need) return;
    const char* e = getenv("MFM_B200_DP_EXCHANGE");
    if (!(e && strcmp(e, "peer") == 0) || dp->world > kMaxDpRanks) {
        dp->p2p = 0;
        return;
    }
    dp_sym_release(dp, s);
    MFM_CUDA(cudaMalloc(&dp->sym, need), "exchange buffer");
    dp->sym_bytes = need;
    MFM_CUDA(cudaMemsetAsync(dp->sym, 0, need, s), "exchange buffer");
    struct Rec {
        cudaIpcMemHandle_t h;
        int dev, ok;
        char pad[56];
    };
    static_assert(sizeof(Rec) == 128, "exchange record");
    Rec mine;
    memset(&mine, 0, sizeof(mine));
    mine.ok = cudaIpcGetMemHandle(&mine.h, dp->sym) == cudaSuccess ? 1 : 0;
    cudaGetLastError();
    mine.dev = dp->device;
    const int W = dp->world;
    DevBuf<char> recs(dp->device, (int64_t)W * sizeof(Rec));
    h2d(recs.ptr + (size_t)dp->rank * sizeof(Rec), reinterpret_cast<const char*>(&mine),
        sizeof(Rec), s, "exchange handles");
    const ncclResult_t r = nccl().AllGather(recs.ptr + (size_t)dp->rank * sizeof(Rec), recs.ptr,
                                            sizeof(Rec), ncclChar, dp->comm, s);
    if (r != ncclSuccess) {
        nccl().CommAbort(dp->comm);
        dp->aborted = true;
        cudaStreamSynchronize(s);
        fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group was aborted",
                               nccl().GetErrorString(r)));
    }
    std::vector<Rec> all(W);
    d2h(reinterpret_cast<char*>(all.data()), recs.ptr, (size_t)W * sizeof(Rec), s,
        "exchange handles");
    dp_sync(dp, s, "the exchange set-up");
    dp->peer.assign(W, nullptr);
    dp->peer[dp->rank] = dp->sym;
    int ok = 1;
    for (int p = 0; p < W; ++p) ok &= all[p].ok;
    for (int p = 0; p < W && ok; ++p) {
        if (p == dp->rank) continue;
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, dp->device, all[p].dev) != cudaSuccess || !can ||
            cudaIpcOpenMemHandle(&dp->peer[p], all[p].h, cudaIpcMemLazyEnablePeerAccess) !=
                cudaSuccess) {
            cudaGetLastError();
            dp->peer[p] = nullptr;
            ok = 0;
        }
    }
    if (dp_all_min(dp, ok, s)) {
        dp->p2p = 1;
    } else {
        dp_sym_release(dp, s);
        dp->p2p = 0;
    }
}

struct Events {
    std::vector<cudaEvent_t> e;
    explicit Events(size_t n) : e(n, nullptr) {
        for (auto& x : e) MFM_CUDA(cudaEventCreateWithFlags(&x, cudaEventDisableTiming), "event");
    }
    ~Events() {
        for (auto x : e)
            if (x) cudaEventDestroy(x);
    }
    Events(const Events&) = delete;
    Events& operator=(const Events&) = delete;
};

// Batches per plan window of the row-table path (MFM_B200_PLAN_WINDOW).
inline int64_t plan_window() {
    static const int64_t w = [] {
        const char* e = getenv("MFM_B200_PLAN_WINDOW");
        const long long v = e ? atoll(e) : 0;
        return v > 0 ? (int64_t)v : (int64_t)128;
    }();
    return w;
}

// Blocks per SM the plan's kernels may take while batches run beside them
// (MFM_B200_PLAN_BLOCKS_PER_SM, default 4; 0 = uncapped).
inline int plan_blocks_per_sm() {
    static const int v = [] {
        const char* e = getenv("MFM_B200_PLAN_BLOCKS_PER_SM");
        return e ? atoi(e) : 4;
    }();
    return v;
}

template <class T>
struct Stream {
    int kind = FEAT;
    int64_t n_keys = 0;
    int W = 0, Wp = 0, cb1 = 0;  // used columns, padded row stride, first column of group 1
    DevBuf<ItemDesc> desc;
    DevBuf<uint32_t> inv;
    GroupDev<T> g0{}, g1{};
    // per-epoch plan
    DevBuf<int64_t> estart, seg_lo, run_start, item_start, item_run, long_list, bitem, blong;
    DevBuf<uint32_t> k0, v0, k1, v1;
    uint32_t *keys = nullptr, *vals = nullptr;
    std::vector<int64_t> h_seg, h_item, h_long;
    int64_t max_entries = 0, max_items = 0;
    DevBuf<T> pay, part;
    // binary FM row-table path: sorted (key, row, x) entries, the row table
    // and the chunk partials
    bool tab = false;
    int TW = 0;  // row stride of ph, pt and grad (k + 16 bytes)
    DevBuf<uint32_t> pidx;  // keys in epoch entry order (CSR indices by position)
    DevBuf<RowVal<T>> erx;  // (batch-local row, value) per entry in epoch order
    DevBuf<T> ex, rx, table, ph, pt, py, psw;
    uint32_t* rrow = nullptr;
    SortTiles tiles;
    // data-parallel: runs (distinct keys per batch) of the sorted stream
    DevBuf<int32_t> head;
    DevBuf<int64_t> runs;     // per entry: runs before it in the epoch (N + 1)
    DevBuf<uint32_t> rkey;    // key of each run
    DevBuf<int64_t> brun;     // runs before each batch (nb + 1)
    std::vector<int64_t> h_run;
    DevBuf<T> grad;           // (max runs per batch + 1, TW or Wp)
    std::vector<int64_t> h_estart;  // payload path, data-parallel: entry start per position
};

template <class T>
struct Trainer {
    int device;
    cudaStream_t s;
    Model model;
    int C;
    bool multiclass;
    int64_t n_rows, n_feat, F, k, B, nb, E;
    const mfm_train* tr;
    // device data
    DevBuf<int64_t> indptr;
    DevBuf<int32_t> indices, order_all, fid, ycls;
    DevBuf<T> data, y, sw, grow;
    // the device arrays every phase reads: the uploads above, or a caller's
    // device buffers (mfm_fm_fit_device)
    const int64_t* p_indptr = nullptr;
    const int32_t* p_indices = nullptr;
    const int32_t* p_order = nullptr;
    const int32_t* p_fid = nullptr;
    const T* p_data = nullptr;
    const T* p_y = nullptr;
    const T* p_sw = nullptr;
    // parameters + state per group: 0 = w0, 1 = w, 2 = V, 3 = R
    DevBuf<T> par[4], st[4][6];
    GroupDev<T> G[4] = {};
    OptDev opt;
    Stream<T> S[2];
    int n_streams = 1;
    DevBuf<GridBar> bar;
    bool coop = false;  // cooperative launches usable (persistent epoch loop)
    mfm_dp* dp = nullptr;  // data-parallel group (row-table path only)
    // parameter-sharded data-parallel training (binary FM row-table path):
    // this rank's keys (key mod world = rank), its restriction of the CSR, and the
    // partial row table that the group sums every batch (stride PW)
    bool shard = false;
    int64_t sh_rows = 0;
    DevBuf<int64_t> sh_indptr;
    DevBuf<int32_t> sh_indices;
    DevBuf<T> sh_data, part;
    DevBuf<ShardXchDev> sh_xch;  // the peer exchange's buffers, as the device sees them
    int PW = 0;

    void upload_group(int gi, const mfm_group* hg, int64_t R, int64_t K, int reg) {
        const int64_t n = (int64_t)C * R * K;
        auto up = [&](DevBuf<T>& dst, const double* src) {
            dst.alloc(device, n);
            if (!src) {
                MFM_CUDA(cudaMemsetAsync(dst.ptr, 0, n * sizeof(T), s), "state init");
                return;
            }
            DevBuf<double> tmp(device, n);
            h2d(tmp.ptr, src, n, s, "parameter upload");
            to_device_layout<T><<<blocks_for(n, 256), 256, 0, s>>>(tmp.ptr, dst.ptr, C, R, K);
            MFM_CHECK_LAUNCH("layout");
            MFM_CUDA(cudaStreamSynchronize(s), "parameter upload");
        };
        up(par[gi], hg->param);
        GroupDev<T>& g = G[gi];
        g = GroupDev<T>{par[gi].ptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                        (int64_t)C * K, reg};
        const int kind = tr->optimizer;
        if (kind == MFM_OPT_ADAGRAD) {
            up(st[gi][0], hg->acc);
            g.acc = st[gi][0].ptr;
        } else if (kind == MFM_OPT_ADAM) {
            up(st[gi][1], hg->m);
            up(st[gi][2], hg->s);
            up(st[gi][3], hg->t);
            g.m = st[gi][1].ptr;
            g.s = st[gi][2].ptr;
            g.t = st[gi][3].ptr;
        } else if (kind == MFM_OPT_FTRL) {
            up(st[gi][4], hg->z);
            up(st[gi][5], hg->n);
            g.z = st[gi][4].ptr;
            g.n = st[gi][5].ptr;
        }
    }

    void download_group(int gi, mfm_group* hg, int64_t R, int64_t K) {
        const int64_t n = (int64_t)C * R * K;
        auto down = [&](DevBuf<T>& src, double* dst) {
            if (!dst || !src.ptr) return;
            DevBuf<double> tmp(device, n);
            from_device_layout<T><<<blocks_for(n, 256), 256, 0, s>>>(src.ptr, tmp.ptr, C, R, K);
            MFM_CHECK_LAUNCH("layout");
            d2h(dst, tmp.ptr, n, s, "parameter download");
            MFM_CUDA(cudaStreamSynchronize(s), "parameter download");
        };
        down(par[gi], hg->param);
        const int kind = tr->optimizer;
        if (kind == MFM_OPT_ADAGRAD) down(st[gi][0], hg->acc);
        if (kind == MFM_OPT_ADAM) {
            down(st[gi][1], hg->m);
            down(st[gi][2], hg->s);
            down(st[gi][3], hg->t);
        }
        if (kind == MFM_OPT_FTRL) {
            down(st[gi][4], hg->z);
            down(st[gi][5], hg->n);
        }
    }

    // Row-table path, epoch-wide part (stream s): entry counts and starts,
    // batch bounds (host copy), epoch-order labels, buffers and the sort's
    // tile table. The per-window part (plan_tab_window) needs no host sync.
    void plan_tab_epoch(Stream<T>& st_, int e) {
        const int32_t* order = p_order + (int64_t)e * n_rows;
        {
            DevBuf<int64_t> cnt(device, n_rows);
            st_.estart.alloc(device, n_rows + 1);
            count_kernel<<<blocks_for(n_rows, 256), 256, 0, s>>>(FEAT, order, p_indptr, n_rows,
                                                               cnt.ptr);
            exclusive_scan<int64_t, int64_t>(device, s, cnt.ptr, n_rows, st_.estart.ptr);
            st_.seg_lo.alloc(device, nb + 1);
            seg_lo_kernel<<<blocks_for(nb + 1, 256), 256, 0, s>>>(st_.estart.ptr, n_rows, B, nb,
                                                                st_.seg_lo.ptr);
            st_.h_seg.resize(nb + 1);
            d2h(st_.h_seg.data(), st_.seg_lo.ptr, nb + 1, s, "plan download");
            MFM_CUDA(cudaStreamSynchronize(s), "plan");
        }
        const int64_t N = st_.h_seg[nb];
        st_.max_entries = 0;
        for (int64_t b = 0; b < nb; ++b) {
            const int64_t len = st_.h_seg[b + 1] - st_.h_seg[b];
            if (len >= ((int64_t)1 << 32))
                fail(MFM_ERR_UNSUPPORTED, "a batch has 2^32 or more gradient entries");
            st_.max_entries = std::max(st_.max_entries, len);
        }
        const int64_t N1 = std::max<int64_t>(N, 1);
        if (st_.k0.n < (size_t)N1 || !st_.k0.ptr) {
            st_.k0.alloc(device, N1);
            st_.v0.alloc(device, N1);
            st_.k1.alloc(device, N1);
            st_.v1.alloc(device, N1);
            st_.erx.alloc(device, N1);
            st_.pidx.alloc(device, N1);
            st_.ex.alloc(device, N1);
            st_.rx.alloc(device, N1);
        }
        if (st_.py.n < (size_t)n_rows || !st_.py.ptr) {
            st_.py.alloc(device, n_rows);
            st_.psw.alloc(device, n_rows);
        }
        permute_rows_kernel<T><<<blocks_for(n_rows, 256), 256, 0, s>>>(
            order, p_y, p_sw, n_rows, st_.py.ptr, st_.psw.ptr);
        MFM_CHECK_LAUNCH("plan");
        const int64_t mc = std::max<int64_t>(1, ceil_div(st_.max_entries, kChunk));
        if (st_.ph.n < (size_t)(mc * st_.TW) || !st_.ph.ptr) {
            st_.ph.alloc(device, mc * st_.TW);
            st_.pt.alloc(device, mc * st_.TW);
        }
        build_sort_tiles(device, s, st_.h_seg, nb, st_.tiles);  // synchronises s
    }

    // Row-table path, batches [b0, b1) of epoch e on stream ps: epoch-order
    // CSR entries (pidx, ex) and the sorted (key, row, x) stream.
    void plan_tab_window(Stream<T>& st_, int e, int64_t b0, int64_t b1, cudaStream_t ps,
                         int per_sm) {
        const int32_t* order = p_order + (int64_t)e * n_rows;
        const int64_t p0 = b0 * B, p1 = std::min(b1 * B, n_rows);
        if (p1 > p0)
            expand_kernel<T><<<warp_grid(device, p1 - p0, 8, per_sm > 0 ? per_sm : 8), 256, 0,
                               ps>>>(
                FEAT, order, p_indptr, p_indices, p_fid, (int)F, p0, p1, B, st_.estart.ptr,
                st_.seg_lo.ptr, st_.pidx.ptr, nullptr, p_data, st_.erx.ptr, st_.ex.ptr);
        MFM_CHECK_LAUNCH("expand");
        SortResult sr = segmented_sort_range(
            ps, st_.pidx.ptr, st_.k0.ptr, st_.v0.ptr, st_.k1.ptr, st_.v1.ptr, st_.seg_lo.ptr, b0,
            b1, st_.tiles, bits_for(st_.n_keys), RecGather<T>{st_.erx.ptr, st_.rx.ptr},
            /*iota=*/true, per_sm > 0 ? (unsigned)(per_sm * sm_count(device)) : 0u);
        st_.keys = sr.keys;  // the same buffers for every window
        st_.rrow = sr.vals;
    }

    // Data-parallel: runs of the sorted stream (every rank computes the same),
    // their keys, and the runs before each batch (host copy).
    void plan_tab_runs(Stream<T>& st_) {
        const int64_t N = st_.h_seg[nb];
        st_.head.alloc(device, std::max<int64_t>(N, 1));
        st_.runs.alloc(device, N + 1);
        if (N > 0) {
            head_kernel<<<blocks_for(N, 256), 256, 0, s>>>(st_.keys, N, st_.head.ptr);
            seg_head_kernel<<<blocks_for(nb, 256), 256, 0, s>>>(st_.seg_lo.ptr, nb, st_.head.ptr);
        }
        exclusive_scan<int32_t, int64_t>(device, s, st_.head.ptr, N, st_.runs.ptr);
        st_.brun.alloc(device, nb + 1);
        batch_runs_kernel<<<blocks_for(nb + 1, 256), 256, 0, s>>>(st_.seg_lo.ptr, nb,
                                                                st_.runs.ptr, st_.brun.ptr);
        st_.h_run.resize(nb + 1);
        d2h(st_.h_run.data(), st_.brun.ptr, nb + 1, s, "plan download");
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
        const int64_t R = st_.h_run[nb];
        st_.rkey.alloc(device, std::max<int64_t>(R, 1));
        if (N > 0)
            run_key_kernel<<<blocks_for(N, 256), 256, 0, s>>>(st_.keys, st_.head.ptr,
                                                            st_.runs.ptr, N, st_.rkey.ptr);
        int64_t mr = 0;
        for (int64_t b = 0; b < nb; ++b) mr = std::max(mr, st_.h_run[b + 1] - st_.h_run[b]);
        if (st_.grad.n < (size_t)((mr + 1) * st_.TW) || !st_.grad.ptr)
            st_.grad.alloc(device, (mr + 1) * st_.TW);
        MFM_CHECK_LAUNCH("plan");
    }

    // count -> scan -> expand -> segmented sort -> runs -> items, for epoch e
    void plan(Stream<T>& st_, int e) {
        const int32_t* order = p_order + (int64_t)e * n_rows;
        DevBuf<int64_t> cnt(device, n_rows);
        st_.estart.alloc(device, n_rows + 1);
        count_kernel<<<blocks_for(n_rows, 256), 256, 0, s>>>(st_.kind, order, p_indptr, n_rows,
                                                           cnt.ptr);
        exclusive_scan<int64_t, int64_t>(device, s, cnt.ptr, n_rows, st_.estart.ptr);
        st_.seg_lo.alloc(device, nb + 1);
        seg_lo_kernel<<<blocks_for(nb + 1, 256), 256, 0, s>>>(st_.estart.ptr, n_rows, B, nb,
                                                            st_.seg_lo.ptr);
        st_.h_seg.resize(nb + 1);
        d2h(st_.h_seg.data(), st_.seg_lo.ptr, nb + 1, s, "plan download");
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
        const int64_t N = st_.h_seg[nb];
        st_.max_entries = 0;
        for (int64_t b = 0; b < nb; ++b) {
            const int64_t len = st_.h_seg[b + 1] - st_.h_seg[b];
            if (len >= ((int64_t)1 << 32))
                fail(MFM_ERR_UNSUPPORTED, "a batch has 2^32 or more gradient entries");
            st_.max_entries = std::max(st_.max_entries, len);
        }
        if (st_.k0.n < (size_t)N || !st_.k0.ptr) {
            st_.k0.alloc(device, N);
            st_.v0.alloc(device, N);
            st_.k1.alloc(device, N);
            st_.v1.alloc(device, N);
        }
        expand_kernel<T><<<warp_grid(device, n_rows, 8, 8), 256, 0, s>>>(
            st_.kind, order, p_indptr, p_indices, p_fid, (int)F, 0, n_rows, B,
            st_.estart.ptr, st_.seg_lo.ptr, st_.k0.ptr, st_.v0.ptr, p_data,
            static_cast<RowVal<T>*>(nullptr), static_cast<T*>(nullptr));
        MFM_CHECK_LAUNCH("expand");
        SortResult sr = segmented_sort(device, s, st_.k0.ptr, st_.v0.ptr, st_.k1.ptr, st_.v1.ptr,
                                       st_.seg_lo.ptr, nb, N, bits_for(st_.n_keys));
        st_.keys = sr.keys;
        st_.vals = sr.vals;
        DevBuf<int32_t> head(device, N);
        DevBuf<int64_t> run_id(device, N + 1);
        if (N > 0) {
            head_kernel<<<blocks_for(N, 256), 256, 0, s>>>(st_.keys, N, head.ptr);
            seg_head_kernel<<<blocks_for(nb, 256), 256, 0, s>>>(st_.seg_lo.ptr, nb, head.ptr);
        }
        exclusive_scan<int32_t, int64_t>(device, s, head.ptr, N, run_id.ptr);
        int64_t Rn = 0;
        d2h(&Rn, run_id.ptr + N, 1, s, "plan download");
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
        st_.run_start.alloc(device, Rn + 1);
        run_start_kernel<<<blocks_for(std::max<int64_t>(N, 1), 256), 256, 0, s>>>(
            head.ptr, run_id.ptr, N, st_.run_start.ptr);
        DevBuf<int64_t> np(device, Rn), lf(device, Rn), lscan(device, Rn + 1);
        st_.item_start.alloc(device, Rn + 1);
        if (Rn > 0)
            pieces_kernel<<<blocks_for(Rn, 256), 256, 0, s>>>(st_.run_start.ptr, Rn, np.ptr,
                                                            lf.ptr);
        exclusive_scan<int64_t, int64_t>(device, s, np.ptr, Rn, st_.item_start.ptr);
        exclusive_scan<int64_t, int64_t>(device, s, lf.ptr, Rn, lscan.ptr);
        int64_t tot[2] = {0, 0};
        d2h(&tot[0], st_.item_start.ptr + Rn, 1, s, "plan download");
        d2h(&tot[1], lscan.ptr + Rn, 1, s, "plan download");
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
        st_.item_run.alloc(device, tot[0]);
        st_.long_list.alloc(device, tot[1]);
        if (Rn > 0)
            items_kernel<<<blocks_for(Rn, 256), 256, 0, s>>>(st_.item_start.ptr, lscan.ptr, Rn,
                                                           st_.item_run.ptr, st_.long_list.ptr);
        st_.desc.alloc(device, tot[0]);
        if (tot[0] > 0)
            desc_kernel<<<blocks_for(tot[0], 256), 256, 0, s>>>(
                st_.item_run.ptr, st_.item_start.ptr, st_.run_start.ptr, st_.keys, tot[0],
                st_.desc.ptr);
        if (st_.inv.n < (size_t)N || !st_.inv.ptr) st_.inv.alloc(device, N);
        if (N > 0) inverse_kernel<<<(unsigned)nb, 256, 0, s>>>(st_.seg_lo.ptr, st_.vals, st_.inv.ptr);
        st_.bitem.alloc(device, nb + 1);
        st_.blong.alloc(device, nb + 1);
        batch_tables_kernel<<<blocks_for(nb + 1, 256), 256, 0, s>>>(
            st_.seg_lo.ptr, nb, run_id.ptr, st_.item_start.ptr, lscan.ptr, st_.bitem.ptr,
            st_.blong.ptr);
        MFM_CHECK_LAUNCH("plan");
        st_.h_item.resize(nb + 1);
        st_.h_long.resize(nb + 1);
        d2h(st_.h_item.data(), st_.bitem.ptr, nb + 1, s, "plan download");
        d2h(st_.h_long.data(), st_.blong.ptr, nb + 1, s, "plan download");
        if (dp) {  // data-parallel: the runs of each batch index its cross-rank sums
            st_.brun.alloc(device, nb + 1);
            batch_runs_kernel<<<blocks_for(nb + 1, 256), 256, 0, s>>>(st_.seg_lo.ptr, nb,
                                                                    run_id.ptr, st_.brun.ptr);
            MFM_CHECK_LAUNCH("plan");
            st_.h_run.resize(nb + 1);
            d2h(st_.h_run.data(), st_.brun.ptr, nb + 1, s, "plan download");
        }
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
        if (dp) {
            int64_t mr = 0;
            for (int64_t b = 0; b < nb; ++b) mr = std::max(mr, st_.h_run[b + 1] - st_.h_run[b]);
            if (st_.grad.n < (size_t)((mr + 1) * st_.Wp) || !st_.grad.ptr)
                st_.grad.alloc(device, (mr + 1) * st_.Wp);
        }
        st_.max_items = 0;
        for (int64_t b = 0; b < nb; ++b)
            st_.max_items = std::max(st_.max_items, st_.h_item[b + 1] - st_.h_item[b]);
        if (st_.pay.n < (size_t)(st_.max_entries * st_.Wp) || !st_.pay.ptr)
            st_.pay.alloc(device, std::max<int64_t>(1, st_.max_entries * st_.Wp));
        if (st_.part.n < (size_t)(st_.max_items * st_.Wp) || !st_.part.ptr)
            st_.part.alloc(device, std::max<int64_t>(1, st_.max_items * st_.Wp));
    }

    RedArgs<T> red_args(Stream<T>& st_, int64_t b, T inv_bsz) {
        constexpr int VEC = 16 / (int)sizeof(T);
        RedArgs<T> R;
        R.desc = st_.desc.ptr;
        R.item_start = st_.item_start.ptr;
        R.long_list = st_.long_list.ptr;
        R.pay = st_.pay.ptr;
        R.part = st_.part.ptr;
        R.W = st_.W;
        R.Wp = st_.Wp;
        R.cb1 = st_.cb1;
        R.nv = st_.Wp / VEC;
        R.nvs = std::min(R.nv, 32);
        R.gpw = 32 / R.nvs;
        R.vec0 = st_.g0.width % VEC == 0 ? 1 : 0;
        R.seg = st_.h_seg[b];
        R.item0 = st_.h_item[b];
        R.g0 = st_.g0;
        R.g1 = st_.g1;
        R.opt = opt;
        R.inv_bsz = inv_bsz;
        R.grow = grow.ptr;
        R.C = C;
        R.gw0 = G[0];
        R.do_w0 = 0;
        R.nrows = 0;
        R.dp = 0;
        R.vals = nullptr;
        R.olo = R.ohi = 0;
        R.item_run = st_.item_run.ptr;
        R.run0 = R.nrun = 0;
        R.grad = nullptr;
        R.progress = nullptr;
        R.pstep = 0;
        return R;
    }

    // Optimizer configuration, entry streams and the forward arguments shared
    // by every batch. Payload columns are [V part | w part] so that the latent
    // columns start on a 16-byte boundary.
    FwdArgs<T> prepare(const mfm_train* c, const T* data, const T* yv, const int32_t* yc,
                       const T* swv) {
        opt = OptDev{c->optimizer, c->learning_rate, c->beta_1, c->beta_2, c->epsilon,
                     c->ftrl_beta, {c->l1_linear, c->l1_factors, 0.0},
                     {c->l2_linear, c->l2_factors, 0.0}};
        opt.lb1 = std::log2(c->beta_1);
        opt.lb2 = std::log2(c->beta_2);
        constexpr int VW = 16 / (int)sizeof(T);
        Stream<T>& s0 = S[0];
        s0.kind = FEAT;
        s0.n_keys = n_feat;
        if (model == M_FFM) {
            s0.W = C;  // w only
            s0.cb1 = C;
            s0.g0 = s0.g1 = G[1];
            Stream<T>& s1 = S[1];
            s1.kind = SLOT;
            s1.n_keys = n_feat * F;
            s1.W = (int)(C * k);
            s1.cb1 = s1.W;
            s1.g0 = s1.g1 = G[2];
            n_streams = 2;
        } else {
            s0.W = (int)(C * k + C);  // [V (C*k) | w (C)]
            s0.cb1 = (int)(C * k);
            s0.g0 = G[2];
            s0.g1 = G[1];
            if (model == M_FWFM) {
                Stream<T>& s1 = S[1];
                s1.kind = PAIR;
                s1.n_keys = F * F;
                s1.W = C;
                s1.cb1 = C;
                s1.g0 = s1.g1 = G[3];
                n_streams = 2;
            }
        }
        for (int si = 0; si < n_streams; ++si) S[si].Wp = (int)ceil_div(S[si].W, VW) * VW;
        // binary FM with k = NV * VW, NV in {1, 2, 4, 8}: row-table reduction
        const int64_t nvw = k / VW;
        if (model == M_FM && !multiclass && k % VW == 0 &&
            (nvw == 1 || nvw == 2 || nvw == 4 || nvw == 8)) {
            s0.tab = true;
            s0.TW = (int)k + VW;
            s0.table.alloc(device, std::max<int64_t>(1, std::min(B, n_rows)) * k);
        }
        int co = 0;
        MFM_CUDA(cudaDeviceGetAttribute(&co, cudaDevAttrCooperativeLaunch, device), "attribute");
        // The persistent epoch loop (one cooperative launch per epoch) is opt-in:
        // at 4096-row batches the per-batch launches are faster today.
        const char* pe = getenv("MFM_B200_EPOCH_KERNEL");
        coop = co != 0 && pe && *pe == '1';
        bar.alloc(device, 1);
        grow.alloc(device, std::max<int64_t>(1, std::min(B, n_rows)) * C);
        FwdArgs<T> A{};
        A.indptr = p_indptr;
        A.indices = p_indices;
        A.data = data;
        A.y = yv;
        A.ycls = yc;
        A.sw = swv;
        A.C = C;
        A.k = (int)k;
        A.F = (int)F;
        A.loss = c->loss;
        A.multiclass = multiclass ? 1 : 0;
        A.ls_on = (T)(1.0 - c->label_smoothing);
        A.ls_off = (T)(C > 1 ? c->label_smoothing / ((double)C - 1.0) : 0.0);
        A.w0 = G[0].p;
        A.w = G[1].p;
        A.v = G[2].p;
        A.r = G[3].p;
        A.fid = p_fid;
        A.grow = grow.ptr;
        A.tab = s0.table.ptr;
        A.TW = (int)k;  // row table: S only (g is in grow)
        p_data = data;
        p_y = yv;
        p_sw = swv;
        return A;
    }

    // Parameter group `gi` over caller-owned device arrays; missing state
    // arrays become zeroed buffers local to the call.
    void device_group(int gi, const mfm_dev_group* dg, int64_t len, int64_t width, int reg) {
        GroupDev<T>& g = G[gi];
        g = GroupDev<T>{(T*)dg->param, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                        width, reg};
        auto st_ptr = [&](int slot, void* ext) -> T* {
            if (ext) return (T*)ext;
            st[gi][slot].alloc(device, len);
            MFM_CUDA(cudaMemsetAsync(st[gi][slot].ptr, 0, len * sizeof(T), s), "state init");
            return st[gi][slot].ptr;
        };
        const int kind = tr->optimizer;
        if (kind == MFM_OPT_ADAGRAD) g.acc = st_ptr(0, dg->acc);
        if (kind == MFM_OPT_ADAM) {
            g.m = st_ptr(1, dg->m);
            g.s = st_ptr(2, dg->s);
            g.t = st_ptr(3, dg->t);
        }
        if (kind == MFM_OPT_FTRL) {
            g.z = st_ptr(4, dg->z);
            g.n = st_ptr(5, dg->n);
        }
    }

    // grid capped to the blocks that are resident at once (kernels whose
    // blocks wait on the same blocks of other ranks)
    template <class K>
    unsigned resident_cap(K kern, unsigned grid) {
        int per_sm = 0;
        MFM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0),
                 "occupancy");
        const int64_t cap = std::min<int64_t>((int64_t)per_sm * sm_count(device), kDpMaxBlocks);
        if (cap < 1) fail(MFM_ERR_CUDA, "the exchange kernel cannot be resident");
        return (unsigned)std::min<int64_t>(grid, cap);
    }
    void launch_forward(const FwdArgs<T>& A, int64_t nrows) {
        const unsigned grid = warp_grid(device, nrows, 8, 8);
        if (model == M_FM && !multiclass) {
            constexpr int VW = 16 / (int)sizeof(T);
            if (k % VW == 0 && k / VW <= 8) {
                const int nvec = (int)(k / VW);
                const unsigned g = (unsigned)sm_count(device) * 8;
#define MFM_FROWS(L_, LR_, CAP_)                                                            \
    {                                                                                       \
        const int64_t want = ceil_div(nrows * LR_, 256);                                    \
        const unsigned gr = (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, want));     \
        if (S[0].tab && shard)                                                              \
            launch_pdl(fm_forward_rows_kernel<T, VW, L_, LR_, CAP_, true, true>,              \
                       A.xch ? resident_cap(fm_forward_rows_kernel<T, VW, L_, LR_, CAP_, true, \
                                                                   true>, gr)                \
                             : gr,                                                          \
                       256, s, A);                                                          \
        else if (S[0].tab)                                                                  \
            launch_pdl(fm_forward_rows_kernel<T, VW, L_, LR_, CAP_, true>, gr, 256, s, A);  \
        else                                                                                \
            fm_forward_rows_kernel<T, VW, L_, LR_, CAP_><<<gr, 256, 0, s>>>(A);             \
        MFM_CHECK_LAUNCH("FM forward");                                                     \
        return;                                                                             \
    }
                if (nvec <= 1) MFM_FROWS(1, 16, 48)
                if (nvec <= 2) MFM_FROWS(2, 16, 48)
                if (nvec <= 4) MFM_FROWS(4, 16, 48)
                MFM_FROWS(8, 16, 32)
#undef MFM_FROWS
            }
        }
        if (model == M_FM) {
            const int D = C * (int)k;
            int Lc = 1, lgc = 0;
            while (Lc < D && Lc < 32) {
                Lc <<= 1;
                ++lgc;
            }
            if (D > 32 && D <= 128) {  // two nonzeros per warp step, up to 8 columns a lane
                Lc = 16;
                lgc = 4;
            }
            const int mcol = (D + Lc - 1) / Lc;
            const size_t sm = (size_t)8 * (D + 3 * C) * sizeof(T);
#define MFM_FWD(MC)                                                                   \
    if (mcol <= MC) {                                                                 \
        if (sm > 48 * 1024)                                                           \
            MFM_CUDA(cudaFuncSetAttribute(fm_forward_kernel<T, MC>,                   \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          (int)sm),                                   \
                     "forward smem attribute");                                       \
        fm_forward_kernel<T, MC><<<grid, 256, sm, s>>>(A, lgc);                       \
        MFM_CHECK_LAUNCH("FM forward");                                               \
        return;                                                                       \
    }
            MFM_FWD(1)
            MFM_FWD(2)
            MFM_FWD(4)
            MFM_FWD(8)
            MFM_FWD(16)
            MFM_FWD(32)
#undef MFM_FWD
            fail(MFM_ERR_UNSUPPORTED, "n_classes * k exceeds 1024");
        }
        const size_t sm = (size_t)8 * 2 * C * sizeof(T);
        constexpr int maxv = 16 / sizeof(T);
        const bool v4 = k % maxv == 0, v2 = k % 2 == 0;
        if (model == M_FFM) {
            // + per warp: staged values, indices and fields of a row
            const size_t smf = sm + (size_t)8 * kFfmStage * (sizeof(T) + 2 * sizeof(int32_t));
            if (v4)
                ffm_forward_kernel<T, maxv><<<grid, 256, smf, s>>>(A);
            else if (v2)
                ffm_forward_kernel<T, 2><<<grid, 256, smf, s>>>(A);
            else
                ffm_forward_kernel<T, 1><<<grid, 256, smf, s>>>(A);
        } else {
            const size_t smf = sm + (size_t)8 * kFfmStage * (sizeof(T) + 2 * sizeof(int32_t));
            if (v4)
                fwfm_forward_kernel<T, maxv><<<grid, 256, smf, s>>>(A);
            else if (v2)
                fwfm_forward_kernel<T, 2><<<grid, 256, smf, s>>>(A);
            else
                fwfm_forward_kernel<T, 1><<<grid, 256, smf, s>>>(A);
        }
        MFM_CHECK_LAUNCH("forward");
    }

    // Row-table reduction of batch b (binary FM): stage 1 per chunk, stage 2
    // per crossing run + w0.
    template <int NV>
    void launch_tab_t(const TabArgs<T>& TA, int64_t nchunks) {
        constexpr int VW = 16 / (int)sizeof(T);
        if (nchunks > 0) {
            const unsigned g = (unsigned)nchunks;
            switch (TA.opt.kind) {
            case MFM_OPT_SGD:
                launch_pdl(fm_tab_reduce_kernel<T, VW, NV, MFM_OPT_SGD>, g, kChunk, s, TA);
                break;
            case MFM_OPT_ADAGRAD:
                launch_pdl(fm_tab_reduce_kernel<T, VW, NV, MFM_OPT_ADAGRAD>, g, kChunk, s, TA);
                break;
            case MFM_OPT_ADAM:
                launch_pdl(fm_tab_reduce_kernel<T, VW, NV, MFM_OPT_ADAM>, g, kChunk, s, TA);
                break;
            default:
                launch_pdl(fm_tab_reduce_kernel<T, VW, NV, MFM_OPT_FTRL>, g, kChunk, s, TA);
            }
        }
        const int64_t warps = std::max<int64_t>(0, nchunks - 1);
        launch_pdl(fm_tab_fold_kernel<T, VW, NV>, (unsigned)(ceil_div(warps, 8) + 1), 256, s, TA,
                   nchunks);
        if (TA.dp) {  // cross-rank sum of the batch's run sums (+ w0), then the step
            MFM_CHECK_LAUNCH("row-table reduction");
            const size_t cnt = (size_t)(TA.nrun + 1) * TA.TW;
            const ncclResult_t r = nccl().AllReduce(
                TA.grad, TA.grad, cnt, sizeof(T) == 4 ? ncclFloat32 : ncclFloat64, ncclSum,
                dp->comm, s);
            if (r != ncclSuccess) {  // e.g. a peer process exited: abort, then drain
                nccl().CommAbort(dp->comm);
                dp->aborted = true;
                cudaStreamSynchronize(s);
                fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group was "
                                       "aborted", nccl().GetErrorString(r)));
            }
            launch_pdl(fm_tab_apply_kernel<T, VW, NV>,
                       (unsigned)std::max<int64_t>(
                           1, ceil_div(TA.nrun, 8 * tab_apply_runs_per_warp<NV>())),
                       256, s, TA);
        }
        MFM_CHECK_LAUNCH("row-table reduction");
    }
    void launch_tab(int64_t b, T inv_bsz, int64_t nrows, int64_t rlo, int64_t rhi,
                    uint32_t step) {
        constexpr int VW = 16 / (int)sizeof(T);
        Stream<T>& st_ = S[0];
        TabArgs<T> TA;
        TA.keys = st_.keys;
        TA.rrow = st_.rrow;
        TA.rx = st_.rx.ptr;
        TA.tab = st_.table.ptr;
        TA.ph = st_.ph.ptr;
        TA.pt = st_.pt.ptr;
        TA.TW = st_.TW;
        TA.seg = st_.h_seg[b];
        TA.n = st_.h_seg[b + 1] - st_.h_seg[b];
        TA.nrows = nrows;
        TA.grow = grow.ptr;
        TA.inv_bsz = inv_bsz;
        TA.gv = G[2];
        TA.gw = G[1];
        TA.gw0 = G[0];
        TA.opt = opt;
        const bool runs = dp && !shard;  // the run-sum exchange
        TA.dp = runs ? 1 : 0;
        TA.rlo = (uint32_t)rlo;
        TA.rhi = (uint32_t)rhi;
        TA.runs = st_.runs.ptr;
        TA.rkey = st_.rkey.ptr;
        TA.run0 = runs ? st_.h_run[b] : 0;
        TA.nrun = runs ? st_.h_run[b + 1] - st_.h_run[b] : 0;
        TA.grad = st_.grad.ptr;
        TA.progress = runs ? dp->prog_d : nullptr;
        TA.pstep = step;
        for (auto& r : TA.pre) r = L2Range{nullptr, 0};
        if (b + 1 < nb) {  // the next batch's epoch-order rows, pulled into L2 by stage 2
            const int64_t p1 = (b + 1) * B, n1 = std::min(B, n_rows - p1);
            const int64_t e0 = st_.h_seg[b + 1], ne = st_.h_seg[b + 2] - e0;
            TA.pre[0] = L2Range{st_.pidx.ptr + e0, ne * (int64_t)sizeof(uint32_t)};
            TA.pre[1] = L2Range{st_.ex.ptr + e0, ne * (int64_t)sizeof(T)};
            TA.pre[2] = L2Range{st_.estart.ptr + p1, (n1 + 1) * (int64_t)sizeof(int64_t)};
            TA.pre[3] = L2Range{st_.py.ptr + p1, n1 * (int64_t)sizeof(T)};
            TA.pre[4] = L2Range{st_.psw.ptr + p1, n1 * (int64_t)sizeof(T)};
        }
        const int64_t nchunks = ceil_div(TA.n, kChunk);
        switch (k / VW) {
        case 1: launch_tab_t<1>(TA, nchunks); break;
        case 2: launch_tab_t<2>(TA, nchunks); break;
        case 4: launch_tab_t<4>(TA, nchunks); break;
        default: launch_tab_t<8>(TA, nchunks); break;
        }
    }

    // Stage 1 and stage 2 of batch b on stream st_. Data-parallel: this
    // rank's rows are [rlo, rhi) of the batch (grow holds them from 0); the
    // sums land in st_.grad and reduce_apply_kernel steps them after the
    // cross-rank sum (launch_dp_apply).
    void launch_reduce(Stream<T>& st_, int64_t b, T inv_bsz, int64_t nrows, bool do_w0,
                       int64_t rlo = 0, int64_t rhi = 0) {
        constexpr int VEC = 16 / (int)sizeof(T);
        const int64_t i0 = st_.h_item[b], i1 = st_.h_item[b + 1];
        const int64_t l0 = st_.h_long[b], l1 = st_.h_long[b + 1];
        RedArgs<T> R = red_args(st_, b, inv_bsz);
        if (dp) {
            const int64_t pos0 = b * B;
            int64_t e[2] = {0, 0};
            d_entry_bounds(st_, pos0 + rlo, pos0 + rhi, e);
            R.dp = 1;
            R.vals = st_.vals + st_.h_seg[b];
            R.olo = (uint32_t)(e[0] - st_.h_seg[b]);
            R.ohi = (uint32_t)(e[1] - st_.h_seg[b]);
            R.run0 = st_.h_run[b];
            R.nrun = st_.h_run[b + 1] - st_.h_run[b];
            R.grad = st_.grad.ptr;
            nrows = rhi - rlo;  // the w0 sum covers this rank's rows
        }
        if (i1 > i0) {
            const int64_t warps = ceil_div(i1 - i0, R.gpw);
            reduce_items_kernel<T, VEC><<<blocks_for(warps, 8), 256, 0, s>>>(R, i1 - i0);
            MFM_CHECK_LAUNCH("reduce stage 1");
        }
        R.do_w0 = do_w0 ? 1 : 0;
        R.nrows = nrows;
        if (l1 > l0 || do_w0) {
            const unsigned blocks = (unsigned)(l1 - l0) + 1;
            reduce_runs_kernel<T, VEC><<<blocks, 256, 0, s>>>(R, l0, l1 - l0);
            MFM_CHECK_LAUNCH("reduce stage 2");
        }
    }

    // Cooperative launch of fm_epoch_kernel over all co-resident blocks.
    template <int FK, int P1, int P2, int P3>
    void launch_epoch_t(const FwdArgs<T>& base, int lgc, size_t fwd_smem) {
        constexpr int VEC = 16 / (int)sizeof(T);
        auto kern = fm_epoch_kernel<T, VEC, FK, P1, P2, P3>;
        const size_t smem = (256 + 8 * 32 * VEC) * sizeof(T) + fwd_smem;
        if (smem > 48 * 1024)
            MFM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem),
                     "epoch kernel smem attribute");
        int per_sm = 0;
        MFM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem),
                 "epoch kernel occupancy");
        if (per_sm < 1) fail(MFM_ERR_UNSUPPORTED, "epoch kernel does not fit on an SM");
        EpochArgs<T> EA;
        EA.fwd = base;
        EA.red = red_args(S[0], 0, T(1));
        EA.seg_lo = S[0].seg_lo.ptr;
        EA.bitem = S[0].bitem.ptr;
        EA.blong = S[0].blong.ptr;
        EA.nb = nb;
        EA.B = B;
        EA.n_rows = n_rows;
        EA.bar = bar.ptr;
        // MFM_B200_EPOCH_SPIN_LIMIT: polls (~100 ns each) before a barrier wait
        // gives up; MFM_B200_EPOCH_DROP_BLOCK: a block index that leaves at its
        // first barrier without arriving (failure-handling tests only)
        const char* sl = getenv("MFM_B200_EPOCH_SPIN_LIMIT");
        EA.spin_limit = sl && *sl ? strtoull(sl, nullptr, 10) : kBarrierSpinLimit;
        if (EA.spin_limit < 1 || EA.spin_limit > kBarrierSpinLimit)
            EA.spin_limit = kBarrierSpinLimit;
        const char* db = getenv("MFM_B200_EPOCH_DROP_BLOCK");
        EA.drop_block = db && *db ? atoi(db) : -1;
        MFM_CUDA(cudaMemsetAsync(bar.ptr, 0, sizeof(GridBar), s), "barrier init");
        void* args[] = {&EA, &lgc};
        MFM_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(per_sm * sm_count(device)),
                                             dim3(256), args, smem, s),
                 "epoch kernel launch");
        GridBar h{};
        d2h(&h, bar.ptr, 1, s, "barrier status");
        MFM_CUDA(cudaStreamSynchronize(s), "epoch kernel");
        if (h.err)
            fail(MFM_ERR_DEVICE_CHECK,
                 "a grid barrier wait gave up (a block did not arrive); the epoch stopped at "
                 "that barrier and the parameters are invalid");
    }

    // true when the whole epoch ran as one persistent launch
    bool launch_epoch(const FwdArgs<T>& base) {
        if (model != M_FM || n_streams != 1 || !coop || S[0].tab) return false;
        constexpr int VW = 16 / (int)sizeof(T);
        if (!multiclass && k % VW == 0 && k / VW <= 8) {
            const int nvec = (int)(k / VW);
            if (nvec <= 1) launch_epoch_t<0, 1, 16, 48>(base, 0, 0);
            else if (nvec <= 2) launch_epoch_t<0, 2, 16, 48>(base, 0, 0);
            else if (nvec <= 4) launch_epoch_t<0, 4, 16, 48>(base, 0, 0);
            else launch_epoch_t<0, 8, 32, 32>(base, 0, 0);
            return true;
        }
        const int D = C * (int)k;
        int Lc = 1, lgc = 0;
        while (Lc < D && Lc < 32) {
            Lc <<= 1;
            ++lgc;
        }
        const int mcol = (D + Lc - 1) / Lc;
        const size_t fs = (size_t)8 * (D + 3 * C) * sizeof(T);
        if (mcol <= 1) launch_epoch_t<1, 1, 0, 0>(base, lgc, fs);
        else if (mcol <= 2) launch_epoch_t<1, 2, 0, 0>(base, lgc, fs);
        else if (mcol <= 4) launch_epoch_t<1, 4, 0, 0>(base, lgc, fs);
        else if (mcol <= 8) launch_epoch_t<1, 8, 0, 0>(base, lgc, fs);
        else if (mcol <= 16) launch_epoch_t<1, 16, 0, 0>(base, lgc, fs);
        else launch_epoch_t<1, 32, 0, 0>(base, lgc, fs);
        return true;
    }

    // Data-parallel liveness: wait until `target` batches have completed their
    // cross-rank sum (the device advances dp->prog_h). A group error reported
    // by NCCL, or no progress for MFM_B200_DP_TIMEOUT seconds (default 300),
    // aborts the communicator, lets the stream drain and fails the call.
    void dp_wait(uint32_t target) {
        const double limit = dp_timeout_s();
        volatile unsigned* p = dp->prog_h;
        unsigned last = *p;
        auto t_last = std::chrono::steady_clock::now();
        while ((int32_t)(*p - target) < 0) {
            if (p[1]) {  // a peer-memory exchange gave up waiting for a peer
                nccl().CommAbort(dp->comm);
                dp->aborted = true;
                cudaStreamSynchronize(s);  // the exchange kernels return on their own
                fail(MFM_ERR_CUDA, fmt("data-parallel group: a peer did not publish its batch "
                                       "within %.0f s (a peer is not answering); the group was "
                                       "aborted",
                                       limit));
            }
            ncclResult_t st = ncclSuccess;
            nccl().CommGetAsyncError(dp->comm, &st);
            const unsigned cur = *p;
            const auto now = std::chrono::steady_clock::now();
            if (cur != last) {
                last = cur;
                t_last = now;
            }
            const bool stalled = std::chrono::duration<double>(now - t_last).count() > limit;
            if ((st != ncclSuccess && st != ncclInProgress) || stalled) {
                nccl().CommAbort(dp->comm);
                dp->aborted = true;
                cudaStreamSynchronize(s);  // the aborted collective lets the stream drain
                if (st != ncclSuccess && st != ncclInProgress)
                    fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group "
                                           "was aborted", nccl().GetErrorString(st)));
                fail(MFM_ERR_CUDA, fmt("data-parallel group: no batch completed for %.0f s (a "
                                       "peer is not answering); the group was aborted",
                                       limit));
            }
            std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
    }

    // Row-table path: each epoch's plan runs in windows of batches (one event
    // per window) on the plan stream, the batches on a high-priority stream
    // forked from and joined back to s.
    void run_tab(const FwdArgs<T>& base, PhaseTimer& pt) {
        const cudaStream_t caller = s;
        // The plan runs in windows of batches on a second, low-priority stream
        // beside the batches (the batch kernels are latency-bound and leave
        // most of the device idle); MFM_B200_PLAN_OVERLAP=0 runs it as one
        // window before the batches, on their stream.
        const char* ov = getenv("MFM_B200_PLAN_OVERLAP");
        const bool overlap = !(ov && *ov == '0') && !dp;
        const cudaStream_t hi = side_stream(device, 0);
        const cudaStream_t lo = overlap ? side_stream(device, 1) : hi;
        std::vector<std::pair<int64_t, int64_t>> win;
        for (int64_t b0 = 0, w = 0; b0 < nb; ++w) {  // 4, 8, 16, then plan_window() batches
            const int64_t len = !overlap ? nb
                                         : std::min<int64_t>(plan_window(),
                                                             (int64_t)4 << std::min<int64_t>(w, 20));
            const int64_t b1 = std::min(nb, b0 + len);
            win.emplace_back(b0, b1);
            b0 = b1;
        }
        Events ev(win.size() + 3);
        cudaEvent_t ev_fork = ev.e[win.size()], ev_ep = ev.e[win.size() + 1],
                    ev_join = ev.e[win.size() + 2];
        MFM_CUDA(cudaEventRecord(ev_fork, caller), "event");
        MFM_CUDA(cudaStreamWaitEvent(hi, ev_fork, 0), "event");
        s = hi;
        pt.s = hi;
        uint32_t gstep = 0;  // batches enqueued in this call
        if (dp) {
            if (dp->aborted)
                fail(MFM_ERR_INVALID, "the data-parallel group was aborted; create a new one");
            *(volatile unsigned*)dp->prog_h = 0u;
        }
        try {
            for (int64_t e = 0; e < E; ++e) {
                plan_tab_epoch(S[0], (int)e);
                pt.mark("plan");
                MFM_CUDA(cudaEventRecord(ev_ep, hi), "event");
                MFM_CUDA(cudaStreamWaitEvent(lo, ev_ep, 0), "event");
                for (size_t w = 0; w < win.size(); ++w) {
                    plan_tab_window(S[0], (int)e, win[w].first, win[w].second, lo,
                                    overlap ? plan_blocks_per_sm() : 0);
                    MFM_CUDA(cudaEventRecord(ev.e[w], lo), "event");
                }
                if (dp && !shard) plan_tab_runs(S[0]);
                for (size_t w = 0; w < win.size(); ++w) {
                    MFM_CUDA(cudaStreamWaitEvent(hi, ev.e[w], 0), "event");
                    for (int64_t b = win[w].first; b < win[w].second; ++b) {
                        // data-parallel: stay at most kDpAhead batches ahead of the
                        // device, so a stalled group is noticed here, never inside
                        // a launch blocked on a full queue
                        ++gstep;
                        if (dp && gstep > kDpAhead) dp_wait(gstep - kDpAhead);
                        const int64_t pos0 = b * B, nrows = std::min(B, n_rows - pos0);
                        const T inv_bsz = T(1) / (T)nrows;  // batch length (fm.rs:395-398)
                        // data-parallel (run sums): this rank scores rows [rlo, rhi)
                        // of the batch; sharded: every row, over the rank's keys
                        const bool slice = dp && !shard;
                        const int64_t rlo = slice ? nrows * dp->rank / dp->world : 0;
                        const int64_t rhi = slice ? nrows * (dp->rank + 1) / dp->world : nrows;
                        FwdArgs<T> A = base;
                        A.pos0 = pos0 + rlo;
                        A.nrows = rhi - rlo;
                        const unsigned long long seq = shard ? ++dp->seq : 0;
                        A.tab = shard ? shard_part(seq) : base.tab + rlo * base.TW;
                        if (shard && dp->p2p == 1) {  // the forward runs the exchange
                            A.xch = sh_xch.ptr;
                            A.seq = seq;
                            A.tab_out = S[0].table.ptr;
                            A.step = gstep;
                        }
                        A.TW = shard ? PW : base.TW;
                        A.grow = base.grow + rlo;
                        A.indptr = S[0].estart.ptr;  // rows by epoch position
                        A.indices = reinterpret_cast<const int32_t*>(S[0].pidx.ptr);
                        A.data = S[0].ex.ptr;
                        A.y = S[0].py.ptr;
                        A.sw = S[0].psw.ptr;
                        {  // stage 1's sorted stream of this batch, pulled into L2 by the forward
                            const int64_t sg = S[0].h_seg[b], ne = S[0].h_seg[b + 1] - sg;
                            A.pre[0] = L2Range{S[0].keys + sg, ne * (int64_t)sizeof(uint32_t)};
                            A.pre[1] = L2Range{S[0].rrow + sg, ne * (int64_t)sizeof(uint32_t)};
                            A.pre[2] = L2Range{S[0].rx.ptr + sg, ne * (int64_t)sizeof(T)};
                        }
                        launch_forward(A, rhi - rlo);
                        if (shard) shard_exchange(pos0, nrows, gstep);
                        launch_tab(b, inv_bsz, nrows, rlo, rhi, gstep);
                    }
                }
                if (dp) dp_wait(gstep);  // the epoch's last batch, before the next plan
                pt.mark("batches");
            }
        } catch (...) {
            cudaStreamSynchronize(lo);  // no kernel may outlive the buffers
            cudaStreamSynchronize(hi);
            s = caller;
            pt.s = caller;
            throw;
        }
        MFM_CUDA(cudaEventRecord(ev_join, hi), "event");
        MFM_CUDA(cudaStreamWaitEvent(caller, ev_join, 0), "event");
        s = caller;
        pt.s = caller;
        MFM_CUDA(cudaStreamSynchronize(s), "training");
    }

    // Epoch-order entry ids [e0, e1) of epoch positions [p0, p1) on stream
    // st_ (the plan's entry starts, host copy made per epoch).
    void d_entry_bounds(const Stream<T>& st_, int64_t p0, int64_t p1, int64_t* e) {
        e[0] = st_.h_estart[p0];
        e[1] = st_.h_estart[p1];
    }

    // Data-parallel: the cross-rank sum of every stream's batch sums (one NCCL
    // group), then the identical step on every rank.
    void launch_dp_apply(int64_t b, T inv_bsz, uint32_t step) {
        constexpr int VEC = 16 / (int)sizeof(T);
        MFM_CHECK_LAUNCH("reduce");
        ncclResult_t r = nccl().GroupStart();
        for (int si = 0; si < n_streams && r == ncclSuccess; ++si) {
            Stream<T>& st_ = S[si];
            const size_t cnt = (size_t)(st_.h_run[b + 1] - st_.h_run[b] + 1) * st_.Wp;
            r = nccl().AllReduce(st_.grad.ptr, st_.grad.ptr, cnt,
                                 sizeof(T) == 4 ? ncclFloat32 : ncclFloat64, ncclSum, dp->comm,
                                 s);
        }
        const ncclResult_t r2 = nccl().GroupEnd();
        if (r == ncclSuccess) r = r2;
        if (r != ncclSuccess) {  // e.g. a peer process exited: abort, then drain
            nccl().CommAbort(dp->comm);
            dp->aborted = true;
            cudaStreamSynchronize(s);
            fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group was "
                                   "aborted", nccl().GetErrorString(r)));
        }
        for (int si = 0; si < n_streams; ++si) {
            Stream<T>& st_ = S[si];
            RedArgs<T> R = red_args(st_, b, inv_bsz);
            R.dp = 1;
            R.run0 = st_.h_run[b];
            R.nrun = st_.h_run[b + 1] - st_.h_run[b];
            R.grad = st_.grad.ptr;
            R.do_w0 = si == n_streams - 1 ? 1 : 0;
            R.progress = R.do_w0 ? dp->prog_d : nullptr;
            R.pstep = step;
            const int64_t warps = std::max<int64_t>(1, ceil_div(R.nrun, R.gpw));
            reduce_apply_kernel<T, VEC><<<blocks_for(warps, 8), 256, 0, s>>>(R);
        }
        MFM_CHECK_LAUNCH("data-parallel apply");
    }

    // Parameter-sharded data parallelism (the row-table path's default;
    // MFM_B200_DP_MODE=runs selects the exchange of per-key run sums instead):
    // this rank's keys and its restriction of the CSR, which the plan and the
    // forward then see in place of the whole CSR.
    static bool shard_mode() {
        const char* m = getenv("MFM_B200_DP_MODE");
        return !(m && strcmp(m, "runs") == 0);
    }
    void shard_setup() {
        constexpr int VW = 16 / (int)sizeof(T);
        const int N = dp->world, r = dp->rank;
        DevBuf<int64_t> cnt(device, std::max<int64_t>(1, n_rows));
        const unsigned g = warp_grid(device, n_rows, 8, 8);
        shard_count_kernel<<<g, 256, 0, s>>>(p_indptr, p_indices, n_rows, N, r, cnt.ptr);
        sh_indptr.alloc(device, n_rows + 1);
        exclusive_scan<int64_t, int64_t>(device, s, cnt.ptr, n_rows, sh_indptr.ptr);
        int64_t nnz = 0;
        d2h(&nnz, sh_indptr.ptr + n_rows, 1, s, "shard plan");
        MFM_CUDA(cudaStreamSynchronize(s), "shard plan");
        sh_indices.alloc(device, std::max<int64_t>(1, nnz));
        sh_data.alloc(device, std::max<int64_t>(1, nnz));
        shard_copy_kernel<T><<<g, 256, 0, s>>>(p_indptr, p_indices, p_data, n_rows, N, r,
                                               sh_indptr.ptr, sh_indices.ptr, sh_data.ptr);
        MFM_CHECK_LAUNCH("shard plan");
        p_indptr = sh_indptr.ptr;
        p_indices = sh_indices.ptr;
        p_data = sh_data.ptr;
        PW = (int)k + VW;  // [S | lin - sq / 2], padded to a 16-byte row
        sh_rows = std::max<int64_t>(1, std::min(B, n_rows));
        // peer-memory exchange: two partial tables (alternating by batch)
        dp_sym_ensure(dp, kDpDataOffset + 2 * (size_t)sh_rows * PW * sizeof(T), s);
        if (dp->p2p == 1) {
            ShardXchDev X{};
            for (int p = 0; p < dp->world; ++p) {
                const char* base = static_cast<const char*>(dp->peer[p]);
                for (int par = 0; par < 2; ++par)
                    X.part[par][p] = base + kDpDataOffset + (size_t)par * sh_rows * PW * sizeof(T);
                X.flags[p] = reinterpret_cast<const unsigned long long*>(base + kDpFlagsOffset);
            }
            X.my_flags = reinterpret_cast<unsigned long long*>(static_cast<char*>(dp->sym) +
                                                               kDpFlagsOffset);
            X.fail = static_cast<unsigned*>(dp->sym);
            X.fail_h = dp->prog_d + 1;
            X.progress = dp->prog_d;
            X.spin = (unsigned long long)(dp_timeout_s() * 5e6);
            X.N = dp->world;
            X.rank = dp->rank;
            X.PW = PW;
            sh_xch.alloc(device, 1);
            h2d(sh_xch.ptr, &X, 1, s, "exchange set-up");
            MFM_CUDA(cudaStreamSynchronize(s), "exchange set-up");
        } else {
            part.alloc(device, sh_rows * PW);
        }
        shard = true;
    }
    // This rank's partial table for exchange number seq.
    T* shard_part(unsigned long long seq) {
        if (dp->p2p != 1) return part.ptr;
        return reinterpret_cast<T*>(static_cast<char*>(dp->sym) + kDpDataOffset) +
               (int64_t)(seq & 1) * sh_rows * PW;
    }
    // NCCL failure inside the fit: abort the communicator, let the stream
    // drain, fail the call.
    [[noreturn]] void dp_failed(ncclResult_t r) {
        nccl().CommAbort(dp->comm);
        dp->aborted = true;
        cudaStreamSynchronize(s);
        fail(MFM_ERR_CUDA, fmt("data-parallel group failed (NCCL: %s); the group was aborted",
                               nccl().GetErrorString(r)));
    }
    // Batch rows [pos0, pos0 + nrows) after the forward: the group's sum of
    // the partial row table, then S, the scores and g (identical on every rank).
    void shard_exchange(int64_t pos0, int64_t nrows, uint32_t step) {
        constexpr int VW = 16 / (int)sizeof(T);
        MFM_CHECK_LAUNCH("FM forward");
        if (dp->p2p == 1) return;  // the forward exchanged and finished its rows
        const ncclResult_t r =
            nccl().AllReduce(part.ptr, part.ptr, (size_t)(nrows * PW),
                             sizeof(T) == 4 ? ncclFloat32 : ncclFloat64, ncclSum, dp->comm, s);
        if (r != ncclSuccess) dp_failed(r);  // e.g. a peer process exited
        const unsigned g = (unsigned)std::max<int64_t>(1, ceil_div(nrows, 256));
#define MFM_FINISH(NV_)                                                                     \
    fm_shard_finish_kernel<T, VW, NV_><<<g, 256, 0, s>>>(                                   \
        part.ptr, PW, S[0].table.ptr, grow.ptr, S[0].py.ptr, S[0].psw.ptr, pos0, nrows, G[0].p, \
        tr->loss, dp->prog_d, step)
        switch (k / VW) {
        case 1: MFM_FINISH(1); break;
        case 2: MFM_FINISH(2); break;
        case 4: MFM_FINISH(4); break;
        default: MFM_FINISH(8); break;
        }
#undef MFM_FINISH
        MFM_CHECK_LAUNCH("shard exchange");
    }
    // After the fit: every rank zeroes the keys it does not own (parameters
    // and optimizer state) and one sum over the ranks gives every rank the
    // owners' values.
    void shard_gather() {
        for (int gi = 1; gi <= 2; ++gi) {
            const GroupDev<T>& g = G[gi];
            T* arrs[7] = {g.p, g.acc, g.m, g.s, g.t, g.z, g.n};
            for (T* a : arrs)
                if (a)
                    shard_zero_unowned_kernel<T><<<blocks_for(n_feat * g.width, 256), 256, 0,
                                                   s>>>(a, n_feat, g.width, dp->world,
                                                        dp->rank);
        }
        MFM_CHECK_LAUNCH("shard gather");
        ncclResult_t r = nccl().GroupStart();
        for (int gi = 1; gi <= 2 && r == ncclSuccess; ++gi) {
            const GroupDev<T>& g = G[gi];
            T* arrs[7] = {g.p, g.acc, g.m, g.s, g.t, g.z, g.n};
            for (T* a : arrs)
                if (a && r == ncclSuccess)
                    r = nccl().AllReduce(a, a, (size_t)(n_feat * g.width),
                                         sizeof(T) == 4 ? ncclFloat32 : ncclFloat64, ncclSum,
                                         dp->comm, s);
        }
        const ncclResult_t r2 = nccl().GroupEnd();
        if (r == ncclSuccess) r = r2;
        if (r != ncclSuccess) dp_failed(r);
        dp_sync(dp, s, "the final gather");
    }

    void run(const FwdArgs<T>& base, PhaseTimer& pt) {
        if (S[0].tab) {
            if (dp && shard_mode()) shard_setup();
            run_tab(base, pt);
            if (shard) shard_gather();
            return;
        }
        uint32_t gstep = 0;  // batches enqueued in this call (data-parallel liveness)
        if (dp) {
            if (dp->aborted)
                fail(MFM_ERR_INVALID, "the data-parallel group was aborted; create a new one");
            *(volatile unsigned*)dp->prog_h = 0u;
        }
        for (int64_t e = 0; e < E; ++e) {
            for (int si = 0; si < n_streams; ++si) {
                plan(S[si], (int)e);
                if (dp) {  // entry starts by position, for each rank's entry-id range
                    S[si].h_estart.resize(n_rows + 1);
                    d2h(S[si].h_estart.data(), S[si].estart.ptr, n_rows + 1, s,
                        "plan download");
                    MFM_CUDA(cudaStreamSynchronize(s), "plan");
                }
            }
            pt.mark("plan");
            if (!dp) {
                FwdArgs<T> A = base;
                A.order = p_order + e * n_rows;
                A.estart1 = S[0].estart.ptr;
                A.pay1 = S[0].pay.ptr;
                A.W1 = S[0].Wp;
                A.inv1 = S[0].inv.ptr;
                if (launch_epoch(A)) {
                    pt.mark("batches");
                    continue;
                }
            }
            for (int64_t b = 0; b < nb; ++b) {
                const int64_t pos0 = b * B, nrows = std::min(B, n_rows - pos0);
                const T inv_bsz = T(1) / (T)nrows;  // divide by batch length (fm.rs:395-398)
                // data-parallel: this rank scores rows [rlo, rhi) of the batch, and
                // stays at most kDpAhead batches ahead of the device
                const int64_t rlo = dp ? nrows * dp->rank / dp->world : 0;
                const int64_t rhi = dp ? nrows * (dp->rank + 1) / dp->world : nrows;
                ++gstep;
                if (dp && gstep > kDpAhead) dp_wait(gstep - kDpAhead);
                FwdArgs<T> A = base;
                A.order = p_order + e * n_rows;
                A.pos0 = pos0 + rlo;
                A.nrows = rhi - rlo;
                A.estart1 = S[0].estart.ptr;
                A.seg1 = S[0].h_seg[b];
                A.pay1 = S[0].pay.ptr;
                A.W1 = S[0].Wp;
                A.inv1 = S[0].inv.ptr;
                if (n_streams > 1) {
                    A.estart2 = S[1].estart.ptr;
                    A.seg2 = S[1].h_seg[b];
                    A.pay2 = S[1].pay.ptr;
                    A.W2 = S[1].Wp;
                    A.inv2 = S[1].inv.ptr;
                }
                launch_forward(A, rhi - rlo);
                for (int si = 0; si < n_streams; ++si)
                    launch_reduce(S[si], b, inv_bsz, nrows, si == n_streams - 1, rlo, rhi);
                if (dp) launch_dp_apply(b, inv_bsz, gstep);
            }
            if (dp) dp_wait(gstep);  // the epoch's last batch, before the next plan
            pt.mark("batches");
        }
        MFM_CUDA(cudaStreamSynchronize(s), "training");
    }
};

// ------------------------------------------------------------- entry point --

struct FitSpec {
    Model model;
    bool multiclass;
    int64_t C;
    const mfm_csr* x;
    const double* y;
    const int64_t* ycls;
    const double* sw;
    const int64_t* field_ids;
    int64_t F;
    const mfm_train* tr;
    int64_t k;
    mfm_group *w0, *w, *v, *r;
};

void validate_fit(const FitSpec& f) {
    check_csr_host(f.x);
    const mfm_train* tr = f.tr;
    if (!tr) fail(MFM_ERR_INVALID, "missing training configuration");
    if (tr->batch_size < 1) fail(MFM_ERR_INVALID, "batch_size must be >= 1");
    if (tr->optimizer < MFM_OPT_SGD || tr->optimizer > MFM_OPT_FTRL)
        fail(MFM_ERR_INVALID, fmt("unknown optimizer %d", tr->optimizer));
    if (!f.multiclass && tr->loss != MFM_LOSS_LOGISTIC && tr->loss != MFM_LOSS_SQUARED)
        fail(MFM_ERR_INVALID, fmt("unknown loss %d", tr->loss));
    if (f.k < 1 || f.k > 1024)
        fail(MFM_ERR_UNSUPPORTED,
             fmt("CUDA training supports 1 <= k <= 1024, got %lld", (long long)f.k));
    if (f.C < 1) fail(MFM_ERR_INVALID, "n_classes must be >= 1");
    if (f.multiclass && f.C > 32)
        fail(MFM_ERR_UNSUPPORTED,
             fmt("CUDA multiclass training supports up to 32 classes, got %lld", (long long)f.C));
    if (f.model == M_FM && f.C * f.k > 1024)
        fail(MFM_ERR_UNSUPPORTED, "n_classes * k must be <= 1024");
    if (f.model != M_FM) check_field_ids(f.field_ids, f.x->n_features, f.F);
    if (f.model == M_FFM && f.x->n_features * f.F >= ((int64_t)1 << 32))
        fail(MFM_ERR_UNSUPPORTED, "n_features * n_fields must be < 2^32");
    const int64_t n = f.x->n_rows;
    if (n >= ((int64_t)1 << 31)) fail(MFM_ERR_UNSUPPORTED, "n_rows must be < 2^31");
    if (tr->n_epochs < 0 || (tr->n_epochs > 0 && !tr->row_orders))
        fail(MFM_ERR_INVALID, "row_orders must be (n_epochs, n_rows)");
    for (int64_t i = 0; i < tr->n_epochs * n; ++i)
        if (tr->row_orders[i] < 0 || tr->row_orders[i] >= n)
            fail(MFM_ERR_INVALID, fmt("row_orders entry out of range [0, %lld)", (long long)n));
    if (f.multiclass)
        for (int64_t i = 0; i < n; ++i)
            if (f.ycls[i] < 0 || f.ycls[i] >= f.C)
                fail(MFM_ERR_INVALID,
                     fmt("class index out of range [0, %lld)", (long long)f.C));
    if (!f.w0 || !f.w || !f.v || !f.w0->param || !f.w->param || !f.v->param ||
        (f.model == M_FWFM && (!f.r || !f.r->param)))
        fail(MFM_ERR_INVALID, "parameter arrays must be provided");
}

template <class T>
void fit_impl(const FitSpec& f, int device, mfm_dp* dp = nullptr) {
    DeviceGuard guard(device);
    std::lock_guard<std::mutex> lk(device_mutex(device));
    Trainer<T> tr;
    tr.device = device;
    tr.dp = dp;
    tr.s = device_stream(device);
    cudaStream_t s = tr.s;
    PhaseTimer pt(s);
    tr.model = f.model;
    tr.C = (int)f.C;
    tr.multiclass = f.multiclass;
    tr.n_rows = f.x->n_rows;
    tr.n_feat = f.x->n_features;
    tr.F = f.model == M_FM ? 1 : f.F;
    tr.k = f.k;
    tr.B = f.tr->batch_size;
    tr.E = f.tr->n_epochs;
    tr.tr = f.tr;
    tr.nb = tr.n_rows > 0 ? ceil_div(tr.n_rows, tr.B) : 0;
    const int64_t n = tr.n_rows, nnz = f.x->nnz, nf = tr.n_feat;

    // data upload (indices narrowed to int32 and values to T on the device)
    tr.indptr.alloc(device, n + 1);
    h2d(tr.indptr.ptr, f.x->indptr, n + 1, s, "indptr upload");
    {
        DevBuf<int64_t> ix64(device, nnz);
        h2d(ix64.ptr, f.x->indices, nnz, s, "indices upload");
        validate_csr_device(device, s, tr.indptr.ptr, n, ix64.ptr, nnz, nf);
        tr.indices.alloc(device, nnz);
        convert_kernel<int64_t, int32_t><<<blocks_for(nnz, 256), 256, 0, s>>>(ix64.ptr,
                                                                            tr.indices.ptr, nnz);
        DevBuf<double> d64(device, nnz);
        h2d(d64.ptr, f.x->data, nnz, s, "data upload");
        tr.data.alloc(device, nnz);
        convert_kernel<double, T><<<blocks_for(nnz, 256), 256, 0, s>>>(d64.ptr, tr.data.ptr, nnz);
        DevBuf<double> sw64(device, n);
        h2d(sw64.ptr, f.sw, n, s, "sample_weight upload");
        tr.sw.alloc(device, n);
        convert_kernel<double, T><<<blocks_for(n, 256), 256, 0, s>>>(sw64.ptr, tr.sw.ptr, n);
        if (f.multiclass) {
            DevBuf<int64_t> y64(device, n);
            h2d(y64.ptr, f.ycls, n, s, "y upload");
            tr.ycls.alloc(device, n);
            convert_kernel<int64_t, int32_t><<<blocks_for(n, 256), 256, 0, s>>>(y64.ptr,
                                                                              tr.ycls.ptr, n);
        } else {
            DevBuf<double> y64(device, n);
            h2d(y64.ptr, f.y, n, s, "y upload");
            tr.y.alloc(device, n);
            convert_kernel<double, T><<<blocks_for(n, 256), 256, 0, s>>>(y64.ptr, tr.y.ptr, n);
        }
        const int64_t nro = tr.E * n;
        DevBuf<int64_t> ro64(device, nro);
        h2d(ro64.ptr, f.tr->row_orders, nro, s, "row_orders upload");
        tr.order_all.alloc(device, nro);
        convert_kernel<int64_t, int32_t><<<blocks_for(nro, 256), 256, 0, s>>>(
            ro64.ptr, tr.order_all.ptr, nro);
        MFM_CHECK_LAUNCH("upload conversion");
        MFM_CUDA(cudaStreamSynchronize(s), "upload");
    }
    if (f.model != M_FM) {
        std::vector<int32_t> f32(nf);
        for (int64_t i = 0; i < nf; ++i) f32[i] = (int32_t)f.field_ids[i];
        tr.fid.alloc(device, nf);
        h2d(tr.fid.ptr, f32.data(), nf, s, "field_ids upload");
        MFM_CUDA(cudaStreamSynchronize(s), "field_ids upload");
    }
    tr.p_indptr = tr.indptr.ptr;
    tr.p_indices = tr.indices.ptr;
    tr.p_order = tr.order_all.ptr;
    tr.p_fid = tr.fid.ptr;

    // parameters + optimizer state, device layout (key, class, k)
    const int64_t F = tr.F, k = tr.k;
    tr.upload_group(0, f.w0, 1, 1, 2);
    tr.upload_group(1, f.w, nf, 1, 0);
    if (f.model == M_FFM)
        tr.upload_group(2, f.v, nf * F, k, 1);
    else
        tr.upload_group(2, f.v, nf, k, 1);
    if (f.model == M_FWFM) tr.upload_group(3, f.r, F * F, 1, 1);

    FwdArgs<T> A = tr.prepare(f.tr, tr.data.ptr, tr.y.ptr, tr.ycls.ptr, tr.sw.ptr);
    pt.mark("upload");
    if (n > 0) tr.run(A, pt);
    (void)F;

    tr.download_group(0, f.w0, 1, 1);
    tr.download_group(1, f.w, nf, 1);
    if (f.model == M_FFM)
        tr.download_group(2, f.v, nf * F, k);
    else
        tr.download_group(2, f.v, nf, k);
    if (f.model == M_FWFM) tr.download_group(3, f.r, F * F, 1);
    pt.mark("download");
}

void fit_dispatch(const FitSpec& f, const mfm_exec* ex, mfm_dp* dp = nullptr) {
    validate_fit(f);
    const int dtype = ex ? ex->dtype : MFM_DTYPE_F64;
    const int device = dp ? dp->device : ex ? ex->device : 0;
    // float32 parameters with float64 arithmetic train as the reference does:
    // float64 parameters and state for the whole fit (_backend.py:116-130)
    if (dtype == MFM_DTYPE_F64 || dtype == MFM_DTYPE_F32_F64)
        fit_impl<double>(f, device, dp);
    else if (dtype == MFM_DTYPE_F32)
        fit_impl<float>(f, device, dp);
    else
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
}

}  // namespace mfm

using namespace mfm;

extern "C" int mfm_fm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                              const mfm_train* tr, int64_t k, mfm_group* w0, mfm_group* w,
                              mfm_group* v, const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FM, false, 1, x, y, nullptr, sample_weight, nullptr, 0, tr, k, w0, w, v,
                  nullptr};
        fit_dispatch(f, ex);
    });
}

extern "C" int mfm_fm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                                         const double* sample_weight, int64_t n_classes,
                                         const mfm_train* tr, int64_t k, mfm_group* w0,
                                         mfm_group* w, mfm_group* v, const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FM, true, n_classes, x, nullptr, y, sample_weight, nullptr, 0, tr, k,
                  w0, w, v, nullptr};
        fit_dispatch(f, ex);
    });
}

extern "C" int mfm_ffm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                               const int64_t* field_ids, int64_t n_fields, const mfm_train* tr,
                               int64_t k, mfm_group* w0, mfm_group* w, mfm_group* v,
                               const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FFM, false, 1, x, y, nullptr, sample_weight, field_ids, n_fields, tr, k,
                  w0, w, v, nullptr};
        fit_dispatch(f, ex);
    });
}

extern "C" int mfm_ffm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                                          const double* sample_weight, int64_t n_classes,
                                          const int64_t* field_ids, int64_t n_fields,
                                          const mfm_train* tr, int64_t k, mfm_group* w0,
                                          mfm_group* w, mfm_group* v, const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FFM, true, n_classes, x, nullptr, y, sample_weight, field_ids, n_fields,
                  tr, k, w0, w, v, nullptr};
        fit_dispatch(f, ex);
    });
}

extern "C" int mfm_fwfm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                                const int64_t* field_ids, int64_t n_fields, const mfm_train* tr,
                                int64_t k, mfm_group* w0, mfm_group* w, mfm_group* v,
                                mfm_group* r, const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FWFM, false, 1, x, y, nullptr, sample_weight, field_ids, n_fields, tr, k,
                  w0, w, v, r};
        fit_dispatch(f, ex);
    });
}

extern "C" int mfm_fwfm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                                           const double* sample_weight, int64_t n_classes,
                                           const int64_t* field_ids, int64_t n_fields,
                                           const mfm_train* tr, int64_t k, mfm_group* w0,
                                           mfm_group* w, mfm_group* v, mfm_group* r,
                                           const mfm_exec* ex) {
    return guarded([&] {
        FitSpec f{M_FWFM, true, n_classes, x, nullptr, y, sample_weight, field_ids, n_fields,
                  tr, k, w0, w, v, r};
        fit_dispatch(f, ex);
    });
}

// ---------------------------------------------------- device-resident fit --

namespace mfm {
template <class T>
void fm_fit_device_impl(int device, cudaStream_t s, const int64_t* indptr,
                        const int32_t* indices, const T* data, int64_t n_rows, int64_t n_features,
                        const T* y, const T* sw, const int32_t* d_order, const mfm_train* c,
                        int64_t k, const mfm_dev_group* w0, const mfm_dev_group* w,
                        const mfm_dev_group* v, mfm_dp* dp = nullptr) {
    DeviceGuard guard(device);
    std::lock_guard<std::mutex> lk(device_mutex(device));
    Trainer<T> tr;
    tr.device = device;
    tr.s = s;
    tr.dp = dp;
    PhaseTimer pt(s);
    tr.model = M_FM;
    tr.C = 1;
    tr.multiclass = false;
    tr.n_rows = n_rows;
    tr.n_feat = n_features;
    tr.F = 1;
    tr.k = k;
    tr.B = c->batch_size;
    tr.E = c->n_epochs;
    tr.tr = c;
    tr.nb = n_rows > 0 ? ceil_div(n_rows, tr.B) : 0;
    tr.p_indptr = indptr;
    tr.p_indices = indices;
    tr.p_order = d_order;
    tr.device_group(0, w0, 1, 1, 2);
    tr.device_group(1, w, n_features, 1, 0);
    tr.device_group(2, v, n_features * k, k, 1);
    FwdArgs<T> A = tr.prepare(c, data, y, nullptr, sw);
    pt.mark("setup");
    if (n_rows > 0) tr.run(A, pt);
}

void check_device_fit(const mfm_train* tr, int64_t k, int64_t n_rows, const mfm_dev_group* w0,
                      const mfm_dev_group* w, const mfm_dev_group* v) {
    if (!tr || tr->batch_size < 1) fail(MFM_ERR_INVALID, "batch_size must be >= 1");
    if (tr->optimizer < MFM_OPT_SGD || tr->optimizer > MFM_OPT_FTRL)
        fail(MFM_ERR_INVALID, fmt("unknown optimizer %d", tr->optimizer));
    if (tr->loss != MFM_LOSS_LOGISTIC && tr->loss != MFM_LOSS_SQUARED)
        fail(MFM_ERR_INVALID, fmt("unknown loss %d", tr->loss));
    if (k < 1 || k > 1024)
        fail(MFM_ERR_UNSUPPORTED,
             fmt("CUDA training supports 1 <= k <= 1024, got %lld", (long long)k));
    if (n_rows < 0 || n_rows >= ((int64_t)1 << 31))
        fail(MFM_ERR_UNSUPPORTED, "n_rows must be in [0, 2^31)");
    if (!w0 || !w || !v || !w0->param || !w->param || !v->param)
        fail(MFM_ERR_INVALID, "parameter arrays must be provided");
}

void fit_device_dispatch(int dtype, int device, const int64_t* indptr, const int32_t* indices,
                         const void* data, int64_t n_rows, int64_t n_features, const void* y,
                         const void* sample_weight, const int32_t* row_orders,
                         const mfm_train* tr, int64_t k, mfm_dev_group* w0, mfm_dev_group* w,
                         mfm_dev_group* v, void* stream, mfm_dp* dp) {
    check_device_fit(tr, k, n_rows, w0, w, v);
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == MFM_DTYPE_F32)
        fm_fit_device_impl<float>(device, s, indptr, indices, (const float*)data, n_rows,
                                  n_features, (const float*)y, (const float*)sample_weight,
                                  row_orders, tr, k, w0, w, v, dp);
    else if (dtype == MFM_DTYPE_F64)
        fm_fit_device_impl<double>(device, s, indptr, indices, (const double*)data, n_rows,
                                   n_features, (const double*)y, (const double*)sample_weight,
                                   row_orders, tr, k, w0, w, v, dp);
    else if (dtype == MFM_DTYPE_F32_F64)
        fail(MFM_ERR_INVALID,
             "device-resident training takes float64 (MFM_DTYPE_F64) or float32 arrays; "
             "float32 parameters with float64 arithmetic train in float64");
    else
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
}
}  // namespace mfm

extern "C" int mfm_fm_fit_device(int dtype, int device, const int64_t* indptr,
                                 const int32_t* indices, const void* data, int64_t n_rows,
                                 int64_t n_features, const void* y, const void* sample_weight,
                                 const int32_t* row_orders, const mfm_train* tr, int64_t k,
                                 mfm_dev_group* w0, mfm_dev_group* w, mfm_dev_group* v,
                                 void* stream) {
    return guarded([&] {
        fit_device_dispatch(dtype, device, indptr, indices, data, n_rows, n_features, y,
                            sample_weight, row_orders, tr, k, w0, w, v, stream, nullptr);
    });
}

// ----------------------------------------------------- data-parallel group --

extern "C" int mfm_dp_unique_id(unsigned char id[128]) {
    return guarded([&] {
        static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
        if (!id) fail(MFM_ERR_INVALID, "id must be provided");
        ncclUniqueId u;
        MFM_NCCL(nccl().GetUniqueId(&u), "ncclGetUniqueId");
        memcpy(id, &u, sizeof(u));
    });
}

extern "C" int mfm_dp_create(const unsigned char id[128], int world, int rank, int device,
                             mfm_dp** out) {
    return guarded([&] {
        if (!id || !out) fail(MFM_ERR_INVALID, "id and out must be provided");
        *out = nullptr;
        if (world < 1 || rank < 0 || rank >= world)
            fail(MFM_ERR_INVALID, fmt("rank %d outside [0, %d)", rank, world));
        DeviceGuard guard(device);
        ncclUniqueId u;
        memcpy(&u, id, sizeof(u));
        unsigned* h = nullptr;
        unsigned* dptr = nullptr;
        MFM_CUDA(cudaHostAlloc(&h, 2 * sizeof(unsigned), cudaHostAllocMapped), "progress word");
        h[0] = h[1] = 0u;
        if (cudaHostGetDevicePointer(&dptr, h, 0) != cudaSuccess) {
            cudaFreeHost(h);
            fail(MFM_ERR_CUDA, "mapped progress word unavailable");
        }
        ncclComm_t c = nullptr;
        const ncclResult_t r = nccl().CommInitRank(&c, world, u, rank);
        if (r != ncclSuccess) {
            cudaFreeHost(h);
            fail(MFM_ERR_CUDA, fmt("ncclCommInitRank: %s", nccl().GetErrorString(r)));
        }
        *out = new mfm_dp{c, world, rank, device, h, dptr, false};
    });
}

extern "C" int mfm_dp_destroy(mfm_dp* dp) {
    return guarded([&] {
        if (!dp) return;
        DeviceGuard guard(dp->device);
        try {  // collective unless aborted: no rank frees its buffer while another maps it
            dp_sym_release(dp, device_stream(dp->device));
        } catch (...) {
            cudaFree(dp->sym);  // the group was aborted meanwhile
        }
        const ncclComm_t c = dp->comm;
        const bool aborted = dp->aborted;  // an aborted communicator is already released
        cudaFreeHost(dp->prog_h);
        delete dp;
        if (!aborted) MFM_NCCL(nccl().CommDestroy(c), "ncclCommDestroy");
    });
}

extern "C" int mfm_fm_fit_device_dp(mfm_dp* dp, int dtype, const int64_t* indptr,
                                    const int32_t* indices, const void* data, int64_t n_rows,
                                    int64_t n_features, const void* y, const void* sample_weight,
                                    const int32_t* row_orders, const mfm_train* tr, int64_t k,
                                    mfm_dev_group* w0, mfm_dev_group* w, mfm_dev_group* v,
                                    void* stream) {
    return guarded([&] {
        if (!dp) fail(MFM_ERR_INVALID, "a data-parallel group must be provided");
        fit_device_dispatch(dtype, dp->device, indptr, indices, data, n_rows, n_features, y,
                            sample_weight, row_orders, tr, k, w0, w, v, stream, dp);
    });
}

extern "C" int mfm_fit_csr_dp(mfm_dp* dp, int dtype, int model, int64_t n_classes,
                              const mfm_csr* x, const double* y, const int64_t* ycls,
                              const double* sample_weight, const int64_t* field_ids,
                              int64_t n_fields, const mfm_train* tr, int64_t k, mfm_group* w0,
                              mfm_group* w, mfm_group* v, mfm_group* r) {
    return guarded([&] {
        if (!dp) fail(MFM_ERR_INVALID, "a data-parallel group must be provided");
        if (n_classes < 1) fail(MFM_ERR_INVALID, "n_classes must be >= 1");
        const Model m = model == MFM_MODEL_FM    ? M_FM
                        : model == MFM_MODEL_FFM ? M_FFM
                        : model == MFM_MODEL_FWFM
                            ? M_FWFM
                            : (fail(MFM_ERR_INVALID, fmt("unknown model kind %d", model)), M_FM);
        const bool mc = n_classes > 1;
        FitSpec f{m, mc, n_classes, x, mc ? nullptr : y, mc ? ycls : nullptr, sample_weight,
                  m == M_FM ? nullptr : field_ids, m == M_FM ? 0 : n_fields, tr, k, w0, w, v,
                  m == M_FWFM ? r : nullptr};
        const mfm_exec ex{dtype, dp->device, 1};
        fit_dispatch(f, &ex, dp);
    });
}

extern "C" void mfm_fit_phase_seconds(double out[4]) {
    for (int i = 0; i < 4; ++i) out[i] = mfm::g_phase_s[i];
}
