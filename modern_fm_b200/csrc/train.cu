// train.cu — device-resident mini-batch training for FM, FFM and FwFM
// (binary and multiclass softmax) on sm_100a, replacing the reference's
// cuda::{fm,ffm,fwfm}_train[_mc] host loops (rust/src/cuda/*_train*.rs), which
// accumulate with float atomics on the GPU and then download every batch's
// gradient for a CPU optimizer flush.
//
// Semantics follow the reference's CPU engine (rust/src/{fm,ffm,fwfm}.rs):
// every batch (a contiguous chunk of row_orders[e]) computes per-row gradients
// from the frozen batch-start parameters, sums them per touched coordinate,
// divides by the batch length and applies one optimizer step per touched
// coordinate (lazy L2; update sets: features for w and FM/FwFM V, (feature,
// field) slots hit by a pair for FFM V, hit field pairs for FwFM R; w0 always).
//
// Device pipeline (no float atomics, bitwise reproducible run to run):
//   per epoch, for each entry stream (FEAT: one entry per nonzero keyed by
//   feature; SLOT: one per ordered pair keyed by FFM slot; PAIR: one per
//   unordered pair keyed by FwFM field pair):
//     count -> scan -> expand (key, batch-local entry id) -> segmented stable
//     radix sort by key within each batch -> run detection -> work items of
//     <= kItem entries per run;
//     plus one 16-byte descriptor per work item and the inverse permutation
//     (entry -> sorted position);
//   per batch:
//     forward kernel (rows): scores, loss gradient, and each entry's gradient
//       payload (all classes) written straight to its sorted position, rows
//       padded to 16 bytes;
//     stage 1 (several work items per warp, 16-byte column vectors): sums the
//       contiguous payload rows of each item; single-item runs apply the
//       optimizer at once;
//     stage 2 (warp per multi-item run): combines the item partials in a
//       fixed order and applies; its last block steps w0 from the per-row
//       gradients.
#include <algorithm>
#include <cstring>
#include <dlfcn.h>
#include <nccl.h>
#include <mutex>
#include <utility>
#include <cmath>

#include "segsort.cuh"

// A data-parallel group: one NCCL communicator bound to a device.
struct mfm_dp {
    ncclComm_t comm;
    int world, rank, device;
};

namespace mfm {

constexpr int kItem = 32;  // entries per reduction work item (one warp)
enum StreamKind { FEAT = 0, SLOT = 1, PAIR = 2 };
enum Model { M_FM = 0, M_FFM = 1, M_FWFM = 2 };

// ------------------------------------------------------------ optimizer --

template <class T>
struct GroupDev {
    T *p, *acc, *m, *s, *t, *z, *n;
    int64_t width;  // parameters per key (per row of the device layout)
    int reg;        // 0 linear (l1/l2_linear), 1 factors, 2 none (w0)
};

struct OptDev {
    int kind;
    double lr, b1, b2, eps, fbeta;
    double l1[3], l2[3];
};

// Programmatic dependent launch (sm_90+): a kernel launched with the
// programmatic-serialization attribute may start while its predecessor in the
// stream drains. pdl_trigger lets the successor be scheduled once every block
// of this grid has started; pdl_wait blocks until the predecessor grid has
// completed and its writes are visible (immediately when launched normally).
// Every thread of a PDL kernel calls pdl_wait before its first write and
// before it exits, so this grid's completion implies its predecessor's.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One step of the reference's step_param / step_coord (rust/src/optimizer.rs:
// 48-167) for coordinate idx of group g with batch-mean data gradient dg.
template <class T>
__device__ __forceinline__ void opt_step(const GroupDev<T>& g, int64_t idx, T dg,
                                         const OptDev& o) {
    T th = g.p[idx];
    const T l1 = (T)o.l1[g.reg], l2 = (T)o.l2[g.reg], lr = (T)o.lr;
    switch (o.kind) {
    case MFM_OPT_SGD:  // apply_update, optimizer.rs:48-60
        th -= lr * (dg + l2 * th);
        break;
    case MFM_OPT_ADAGRAD: {
        const T gr = dg + l2 * th;
        const T a = g.acc[idx] + gr * gr;
        g.acc[idx] = a;
        th -= lr * gr / sqrt(a + (T)1e-10);
        break;
    }
    case MFM_OPT_ADAM: {  // adam_step, optimizer.rs:68-85 (lazy, per-coordinate t)
        const T gr = dg + l2 * th;
        const T b1 = (T)o.b1, b2 = (T)o.b2;
        const T t = g.t[idx] + T(1);
        const T m = b1 * g.m[idx] + (T(1) - b1) * gr;
        const T v = b2 * g.s[idx] + (T(1) - b2) * gr * gr;
        g.t[idx] = t;
        g.m[idx] = m;
        g.s[idx] = v;
        const T mh = m / (T(1) - pow(b1, t));
        const T vh = v / (T(1) - pow(b2, t));
        th -= lr * mh / (sqrt(vh) + (T)o.eps);
        break;
    }
    default: {  // FTRL-Proximal, ftrl_step, optimizer.rs:93-105 (pure data gradient)
        const T n = g.n[idx];
        const T nn = n + dg * dg;
        const T sigma = (sqrt(nn) - sqrt(n)) / lr;
        const T z = g.z[idx] + dg - sigma * th;
        g.z[idx] = z;
        g.n[idx] = nn;
        if (fabs(z) <= l1)
            th = T(0);
        else {
            const T sign = z < T(0) ? T(-1) : T(1);
            th = -(z - sign * l1) / (((T)o.fbeta + sqrt(nn)) / lr + l2);
        }
    }
    }
    g.p[idx] = th;
}

// opt_step on VEC consecutive coordinates [idx0, idx0 + VEC) of one group,
// with 16-byte loads and stores of the parameter and its state. The state is
// loaded before the gradients are known (`prefetch`) so the loads overlap the
// payload reduction; `commit` applies the step. OPT >= 0 fixes the optimizer
// at compile time (only its state vectors occupy registers).
template <class T, int VEC, int OPT = -1>
struct VecStep {
    Vec<T, VEC> p, a, b, c;  // param and up to three state vectors
    __device__ __forceinline__ void prefetch(const GroupDev<T>& g, int64_t idx0, int kind_rt) {
        const int kind = OPT >= 0 ? OPT : kind_rt;
        p = ldg_vec<T, VEC>(g.p + idx0);
        if (kind == MFM_OPT_ADAGRAD) {
            a = ldg_vec<T, VEC>(g.acc + idx0);
        } else if (kind == MFM_OPT_ADAM) {
            a = ldg_vec<T, VEC>(g.m + idx0);
            b = ldg_vec<T, VEC>(g.s + idx0);
            c = ldg_vec<T, VEC>(g.t + idx0);
        } else if (kind == MFM_OPT_FTRL) {
            a = ldg_vec<T, VEC>(g.z + idx0);
            b = ldg_vec<T, VEC>(g.n + idx0);
        }
    }
    // the state only (the caller already holds the parameter vector in p)
    __device__ __forceinline__ void prefetch_state(const GroupDev<T>& g, int64_t idx0,
                                                   int kind_rt) {
        const int kind = OPT >= 0 ? OPT : kind_rt;
        if (kind == MFM_OPT_ADAGRAD) {
            a = ldg_vec<T, VEC>(g.acc + idx0);
        } else if (kind == MFM_OPT_ADAM) {
            a = ldg_vec<T, VEC>(g.m + idx0);
            b = ldg_vec<T, VEC>(g.s + idx0);
            c = ldg_vec<T, VEC>(g.t + idx0);
        } else if (kind == MFM_OPT_FTRL) {
            a = ldg_vec<T, VEC>(g.z + idx0);
            b = ldg_vec<T, VEC>(g.n + idx0);
        }
    }
    __device__ __forceinline__ void commit(const GroupDev<T>& g, int64_t idx0, const T* dg,
                                           const OptDev& o) {
        const T l1 = (T)o.l1[g.reg], l2 = (T)o.l2[g.reg], lr = (T)o.lr;
        const int kind = OPT >= 0 ? OPT : o.kind;
#pragma unroll
        for (int u = 0; u < VEC; ++u) {
            T th = p.v[u];
            switch (kind) {
            case MFM_OPT_SGD:
                th -= lr * (dg[u] + l2 * th);
                break;
            case MFM_OPT_ADAGRAD: {
                const T gr = dg[u] + l2 * th;
                const T ac = a.v[u] + gr * gr;
                a.v[u] = ac;
                th -= lr * gr / sqrt(ac + (T)1e-10);
                break;
            }
            case MFM_OPT_ADAM: {
                const T gr = dg[u] + l2 * th;
                const T b1 = (T)o.b1, b2 = (T)o.b2;
                const T t = c.v[u] + T(1);
                const T m = b1 * a.v[u] + (T(1) - b1) * gr;
                const T v = b2 * b.v[u] + (T(1) - b2) * gr * gr;
                c.v[u] = t;
                a.v[u] = m;
                b.v[u] = v;
                const T mh = m / (T(1) - pow(b1, t));
                const T vh = v / (T(1) - pow(b2, t));
                th -= lr * mh / (sqrt(vh) + (T)o.eps);
                break;
            }
            default: {
                const T d = dg[u];
                const T n = b.v[u], nn = n + d * d;
                const T sigma = (sqrt(nn) - sqrt(n)) / lr;
                const T z = a.v[u] + d - sigma * th;
                a.v[u] = z;
                b.v[u] = nn;
                if (fabs(z) <= l1)
                    th = T(0);
                else {
                    const T sign = z < T(0) ? T(-1) : T(1);
                    th = -(z - sign * l1) / (((T)o.fbeta + sqrt(nn)) / lr + l2);
                }
            }
            }
            p.v[u] = th;
        }
        *reinterpret_cast<Vec<T, VEC>*>(g.p + idx0) = p;
        if (kind == MFM_OPT_ADAGRAD) {
            *reinterpret_cast<Vec<T, VEC>*>(g.acc + idx0) = a;
        } else if (kind == MFM_OPT_ADAM) {
            *reinterpret_cast<Vec<T, VEC>*>(g.m + idx0) = a;
            *reinterpret_cast<Vec<T, VEC>*>(g.s + idx0) = b;
            *reinterpret_cast<Vec<T, VEC>*>(g.t + idx0) = c;
        } else if (kind == MFM_OPT_FTRL) {
            *reinterpret_cast<Vec<T, VEC>*>(g.z + idx0) = a;
            *reinterpret_cast<Vec<T, VEC>*>(g.n + idx0) = b;
        }
    }
};

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
// With erow set (FEAT only), also each entry's batch-local row and value, for
// the row-table reduction.
template <class T>
__global__ void __launch_bounds__(256)
    expand_kernel(int kind, const int32_t* __restrict__ order, const int64_t* __restrict__ indptr,
                  const int32_t* __restrict__ indices, const int32_t* __restrict__ fid, int F,
                  int64_t pos_lo, int64_t pos_hi, int64_t B, const int64_t* __restrict__ estart,
                  const int64_t* __restrict__ seg_lo, uint32_t* __restrict__ keys,
                  uint32_t* __restrict__ vals, const T* __restrict__ data,
                  uint32_t* __restrict__ erow, T* __restrict__ ex) {
    // (FEAT with erow: keys[] is kept unsorted as the epoch-order CSR indices)
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
                vals[base + a] = (uint32_t)(local + a);
                if (erow) {
                    erow[base + a] = rib;
                    ex[base + a] = data[rb + a];
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

// ------------------------------------------------------ forward kernels --

template <class T>
struct FwdArgs {
    const int64_t* indptr;
    const int32_t* indices;
    const T* data;
    const int32_t* order;  // row_orders[e]
    int64_t pos0, nrows;   // this batch: epoch positions [pos0, pos0 + nrows)
    const int64_t* estart1;
    int64_t seg1;  // stream 1 (FEAT) entry start per position; batch start
    const int64_t* estart2;
    int64_t seg2;  // stream 2 (SLOT / PAIR)
    const T* y;
    const int32_t* ycls;
    const T* sw;
    int C, k, F, loss, multiclass;
    T ls_on, ls_off;  // softmax targets: 1 - eps for the true class, eps / (C - 1) otherwise
    const T *w0, *w, *v, *r;
    const int32_t* fid;
    const uint32_t* inv1;  // entry -> batch-local sorted position, stream 1
    const uint32_t* inv2;  // stream 2
    T* pay1;
    int W1;  // padded payload row stride (multiple of 16 bytes), stream 1
    T* pay2;
    int W2;
    T* grow;  // (nrows, C) per-row loss gradients, summed into the w0 gradient
    T* tab;   // row table (nrows, TW): [S (k) | g | pad] (binary FM row-table path)
    int TW;
};

template <class T>
__device__ __forceinline__ T sigmoid_t(T s) {  // optimizer.rs:28-35
    if (s >= T(0)) return T(1) / (T(1) + exp(-s));
    const T e = exp(s);
    return e / (T(1) + e);
}

// lane 0: per-class gradients of one row from its logits (sm_logit) into sm_g.
template <class T>
__device__ __forceinline__ void row_gradients(const FwdArgs<T>& A, int64_t row, const T* lg,
                                              T* g) {
    const T sw = A.sw[row];
    if (!A.multiclass) {  // loss_grad, optimizer.rs:38-43
        const T s = lg[0], y = A.y[row];
        g[0] = sw * (A.loss == MFM_LOSS_LOGISTIC ? sigmoid_t(s) - y : s - y);
        return;
    }
    // stable softmax with label smoothing, rust/src/fm.rs:357-393
    T mx = -INFINITY;
    for (int c = 0; c < A.C; ++c) mx = fmax(mx, lg[c]);
    T sum = T(0);
    for (int c = 0; c < A.C; ++c) {
        g[c] = exp(lg[c] - mx);
        sum += g[c];
    }
    const int yc = A.ycls[row];
    for (int c = 0; c < A.C; ++c) {
        const T p = g[c] / sum;
        g[c] = sw * (p - (c == yc ? A.ls_on : A.ls_off));
    }
}

// FM (binary and multiclass), any width: D = C*k latent columns per feature,
// split over Lc lanes (G = 32/Lc nonzeros per warp step), MCOL columns per
// lane. Payload per nonzero: [g_c (x cache_cf - v_cf x^2) (C*k) | g_c x (C)]
// (FmGradAccum::add_row, rust/src/fm.rs:133-146).
template <class T, int MCOL>
__device__ __forceinline__ void fm_forward_dev(const FwdArgs<T>& A, int lgc, unsigned char* smraw,
                                               int64_t warp0, int64_t nwarps) {
    const int C = A.C, k = A.k, D = C * k;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    T* sm = reinterpret_cast<T*>(smraw) + (size_t)wib * (D + 3 * C);
    T *colv = sm, *lins = sm + D, *logit = lins + C, *gs = logit + C;
    const int Lc = 1 << lgc, G = 32 >> lgc, grp = lane >> lgc, l = lane & (Lc - 1);
    for (int64_t j = warp0; j < A.nrows; j += nwarps) {
        const int64_t pos = A.pos0 + j, row = A.order[pos];
        const int64_t rb = A.indptr[row], z = A.indptr[row + 1] - rb;
        T cache[MCOL], sq[MCOL];
#pragma unroll
        for (int m = 0; m < MCOL; ++m) cache[m] = sq[m] = T(0);
        T lin = T(0);
        for (int64_t base = 0; base < z; base += 32) {
            const int nh = (int)min((int64_t)32, z - base);
            int32_t my_i = 0;
            T my_x = T(0);
            if (lane < nh) {
                my_i = A.indices[rb + base + lane];
                my_x = A.data[rb + base + lane];
            }
#pragma unroll 4  // four nonzeros' gathers in flight
            for (int t = 0; t < nh; t += G) {
                const int src = t + grp;
                const int32_t i = __shfl_sync(0xffffffffu, my_i, src);
                const T x = __shfl_sync(0xffffffffu, my_x, src);
                if (src < nh) {
                    const T* vi = A.v + (int64_t)i * D;
#pragma unroll
                    for (int m = 0; m < MCOL; ++m) {
                        const int jj = l + m * Lc;
                        if (jj < D) {
                            const T vx = vi[jj] * x;
                            cache[m] += vx;
                            sq[m] += vx * vx;
                        }
                    }
                    if (l < C) lin += A.w[(int64_t)i * C + l] * x;
                }
            }
        }
        for (int o = Lc; o < 32; o <<= 1) {
#pragma unroll
            for (int m = 0; m < MCOL; ++m) {
                cache[m] += __shfl_xor_sync(0xffffffffu, cache[m], o);
                sq[m] += __shfl_xor_sync(0xffffffffu, sq[m], o);
            }
            lin += __shfl_xor_sync(0xffffffffu, lin, o);
        }
        if (grp == 0) {
#pragma unroll
            for (int m = 0; m < MCOL; ++m) {
                const int jj = l + m * Lc;
                if (jj < D) colv[jj] = cache[m] * cache[m] - sq[m];
            }
            if (l < C) lins[l] = lin;
        }
        __syncwarp();
        for (int c = lane; c < C; c += 32) {
            T s = T(0);
            for (int t = 0; t < k; ++t) s += colv[c * k + t];
            logit[c] = A.w0[c] + lins[c] + T(0.5) * s;
        }
        __syncwarp();
        if (lane == 0) row_gradients(A, row, logit, gs);
        __syncwarp();
        for (int c = lane; c < C; c += 32) A.grow[j * C + c] = gs[c];
        // payload rows of this row's nonzeros (batch-local entry ids)
        const int64_t e0 = A.estart1[pos] - A.seg1;
        for (int64_t base = 0; base < z; base += 32) {
            const int nh = (int)min((int64_t)32, z - base);
            int32_t my_i = 0;
            T my_x = T(0);
            if (lane < nh) {
                my_i = A.indices[rb + base + lane];
                my_x = A.data[rb + base + lane];
            }
#pragma unroll 4  // four nonzeros' gathers in flight
            for (int t = 0; t < nh; t += G) {
                const int src = t + grp;
                const int32_t i = __shfl_sync(0xffffffffu, my_i, src);
                const T x = __shfl_sync(0xffffffffu, my_x, src);
                if (src < nh) {
                    const T* vi = A.v + (int64_t)i * D;
                    T* P = A.pay1 + (int64_t)A.inv1[A.seg1 + e0 + base + src] * A.W1;
                    if (l < C) P[D + l] = gs[l] * x;
#pragma unroll
                    for (int m = 0; m < MCOL; ++m) {
                        const int jj = l + m * Lc;
                        if (jj < D) P[jj] = gs[jj / k] * (x * cache[m] - vi[jj] * x * x);
                    }
                }
            }
        }
        __syncwarp();
    }
}

template <class T, int MCOL>
__global__ void __launch_bounds__(256) fm_forward_kernel(FwdArgs<T> A, int lgc) {
    extern __shared__ unsigned char smraw[];
    fm_forward_dev<T, MCOL>(A, lgc, smraw, ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5,
                            ((int64_t)gridDim.x * blockDim.x) >> 5);
}

// Binary FM, latent rows of up to 8 vectors (k <= 32 float32, k <= 16
// float64): LR lanes per row, L lanes per nonzero (VEC-wide loads), CAP
// nonzeros per iteration with every gather issued before use (as in the
// scoring kernel). Rows that fit one iteration keep their gathered latent rows
// in registers for the payload pass; longer rows gather again.
template <class T, int VEC, int L, int LR, int CAP>
struct RowsShape {
    static constexpr int G = LR / L, NC = CAP / LR, S = CAP / G;
};

template <class T, int VEC, int L, int LR, int CAP>
__device__ __forceinline__ void rows_gather(const FwdArgs<T>& A, int64_t rb, int64_t z,
                                            int64_t base, int rl, int grp, int l, bool act,
                                            int (&nh)[RowsShape<T, VEC, L, LR, CAP>::NC],
                                            Vec<T, VEC> (&q)[RowsShape<T, VEC, L, LR, CAP>::S],
                                            T (&xs)[RowsShape<T, VEC, L, LR, CAP>::S], T& lin,
                                            bool pdl = false) {
    using Sh = RowsShape<T, VEC, L, LR, CAP>;
    int32_t ii[Sh::NC];
    T xx[Sh::NC];
#pragma unroll
    for (int c = 0; c < Sh::NC; ++c) {
        const int64_t rem = z - base - LR * c;
        nh[c] = rem <= 0 ? 0 : (rem >= LR ? LR : (int)rem);
        ii[c] = 0;
        xx[c] = T(0);
        if (rl < nh[c]) {
            ii[c] = A.indices[rb + base + LR * c + rl];
            xx[c] = A.data[rb + base + LR * c + rl];
        }
    }
    if (pdl) pdl_wait();  // parameters below are the predecessor's output
#pragma unroll
    for (int c = 0; c < Sh::NC; ++c)
        if (rl < nh[c]) lin += A.w[ii[c]] * xx[c];
#pragma unroll
    for (int st = 0; st < Sh::S; ++st) {
        const int c = st / L, src = (st % L) * Sh::G + grp;
        const int32_t i = __shfl_sync(0xffffffffu, ii[c], src, LR);
        const T x = __shfl_sync(0xffffffffu, xx[c], src, LR);
        const bool ok = src < nh[c];
        xs[st] = ok ? x : T(0);
        if (ok && act) {
            q[st] = ldg_vec<T, VEC>(A.v + (int64_t)i * A.k + l * VEC);
        } else {
#pragma unroll
            for (int u = 0; u < VEC; ++u) q[st].v[u] = T(0);
        }
    }
}

template <class T, int VEC, int L, int LR, int CAP>
__device__ __forceinline__ void rows_payload(const FwdArgs<T>& A, int64_t e0, int64_t base,
                                             int grp, int l, bool act, T g, const T* cache,
                                             const int (&nh)[RowsShape<T, VEC, L, LR, CAP>::NC],
                                             const Vec<T, VEC> (&q)[RowsShape<T, VEC, L, LR, CAP>::S],
                                             const T (&xs)[RowsShape<T, VEC, L, LR, CAP>::S]) {
    using Sh = RowsShape<T, VEC, L, LR, CAP>;
#pragma unroll
    for (int st = 0; st < Sh::S; ++st) {
        const int c = st / L, src = (st % L) * Sh::G + grp;
        if (src >= nh[c]) continue;
        const int64_t a = base + LR * c + src;
        T* P = A.pay1 + (int64_t)A.inv1[A.seg1 + e0 + a] * A.W1;
        const T x = xs[st];
        if (act) {
            Vec<T, VEC> o;
#pragma unroll
            for (int u = 0; u < VEC; ++u) o.v[u] = g * (x * cache[u] - q[st].v[u] * x * x);
            *reinterpret_cast<Vec<T, VEC>*>(P + l * VEC) = o;
        }
        if (l == 0) P[A.k] = g * x;  // w column after the k latent columns
    }
}

// TAB: write the row table [S | g] instead of per-entry payloads.
template <class T, int VEC, int L, int LR, int CAP, bool TAB = false>
__device__ __forceinline__ void fm_forward_rows_dev(const FwdArgs<T>& A, int64_t slot0,
                                                    int64_t nslots) {
    using Sh = RowsShape<T, VEC, L, LR, CAP>;
    const int lane = threadIdx.x & 31, rl = lane & (LR - 1), grp = rl / L, l = rl % L;
    const bool act = l < A.k / VEC;
    if (TAB) pdl_trigger();
    for (int64_t j = slot0;; j += nslots) {
        const bool live = j < A.nrows;
        if (!__any_sync(0xffffffffu, live)) break;
        const int64_t pos = A.pos0 + j;
        // TAB: CSR, y and sample weight are already in epoch order
        const int64_t row = live ? (TAB ? pos : A.order[pos]) : 0;
        const int64_t rb = live ? A.indptr[row] : 0;
        const int64_t z = live ? A.indptr[row + 1] - rb : 0;
        // pass 1: score from the frozen parameters (train_score_row, fm.rs:77-101)
        T cache[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) cache[u] = T(0);
        T sq = T(0), lin = T(0);
        int nh[Sh::NC];
        Vec<T, VEC> q[Sh::S];
        T xs[Sh::S];
        int iters = 0;
        for (int64_t base = 0;; base += CAP, ++iters) {
            if (!__any_sync(0xffffffffu, base < z)) break;
            rows_gather<T, VEC, L, LR, CAP>(A, rb, z, base, rl, grp, l, act, nh, q, xs, lin, TAB);
#pragma unroll
            for (int st = 0; st < Sh::S; ++st)
#pragma unroll
                for (int u = 0; u < VEC; ++u) {
                    const T vx = q[st].v[u] * xs[st];
                    cache[u] += vx;
                    sq += vx * vx;
                }
        }
#pragma unroll
        for (int o = L; o < LR; o <<= 1)
#pragma unroll
            for (int u = 0; u < VEC; ++u) cache[u] += __shfl_xor_sync(0xffffffffu, cache[u], o);
        T pair = T(0);
        if (grp == 0 && act) {
#pragma unroll
            for (int u = 0; u < VEC; ++u) pair += cache[u] * cache[u];
        }
        T t = lin + T(0.5) * (pair - sq);
#pragma unroll
        for (int o = LR / 2; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        T g = T(0);
        if (TAB) pdl_wait();  // w0 and the writes below follow the predecessor
        if (live) {  // loss_grad x sample_weight, optimizer.rs:38-43
            const T s = A.w0[0] + t, y = A.y[row];
            g = A.sw[row] * (A.loss == MFM_LOSS_LOGISTIC ? sigmoid_t(s) - y : s - y);
            if (rl == 0) A.grow[j] = g;
        }
        if (TAB) {
            if (live) {
                T* tr = A.tab + j * A.TW;
                if (grp == 0 && act) {
                    Vec<T, VEC> o;
#pragma unroll
                    for (int u = 0; u < VEC; ++u) o.v[u] = cache[u];
                    *reinterpret_cast<Vec<T, VEC>*>(tr + l * VEC) = o;
                }
                if (rl == 0) tr[A.k] = g;
            }
            continue;
        }
        // pass 2: payload rows at their sorted positions
        const int64_t e0 = live ? A.estart1[pos] - A.seg1 : 0;
        if (iters == 1) {
            rows_payload<T, VEC, L, LR, CAP>(A, e0, 0, grp, l, act, g, cache, nh, q, xs);
        } else {
            for (int64_t base = 0;; base += CAP) {
                if (!__any_sync(0xffffffffu, base < z)) break;
                T dummy = T(0);
                rows_gather<T, VEC, L, LR, CAP>(A, rb, z, base, rl, grp, l, act, nh, q, xs, dummy);
                rows_payload<T, VEC, L, LR, CAP>(A, e0, base, grp, l, act, g, cache, nh, q, xs);
            }
        }
    }
    if (TAB) pdl_wait();
}

template <class T, int VEC, int L, int LR, int CAP, bool TAB = false>
__global__ void __launch_bounds__(256, 2) fm_forward_rows_kernel(FwdArgs<T> A) {
    fm_forward_rows_dev<T, VEC, L, LR, CAP, TAB>(
        A, ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LR,
        ((int64_t)gridDim.x * blockDim.x) / LR);
}

// FFM (binary and multiclass). Device V layout (n, F, C, k).
// Stream 1 (FEAT) payload: [g_c x_a] (w gradient);
// stream 2 (SLOT) payload per ordered pair (a, b != a), slot (i_a, f_b):
// [g_c x_a x_b V[i_b, f_a, c, :]] (FfmGradAccum::add_row, rust/src/ffm.rs:129-171).
// Rows of up to kFfmStage nonzeros are staged per warp in shared memory
// (index, value, field): pair decoding then needs no dependent global loads.
constexpr int kFfmStage = 64;

template <class T, int VEC>
__global__ void __launch_bounds__(256) ffm_forward_kernel(FwdArgs<T> A) {
    extern __shared__ unsigned char smraw[];
    const int C = A.C, k = A.k, F = A.F, CK = C * k;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    T* logit = reinterpret_cast<T*>(smraw) + (size_t)wib * 2 * C;
    T* gs = logit + C;
    T* s_x = reinterpret_cast<T*>(smraw) + (size_t)8 * 2 * C + (size_t)wib * kFfmStage;
    int32_t* s_ix = reinterpret_cast<int32_t*>(reinterpret_cast<T*>(smraw) + (size_t)8 * 2 * C +
                                               (size_t)8 * kFfmStage) +
                    (size_t)wib * 2 * kFfmStage;
    int32_t* s_f = s_ix + kFfmStage;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < A.nrows;
         j += nwarps) {
        const int64_t pos = A.pos0 + j, row = A.order[pos];
        const int64_t rb = A.indptr[row], z = A.indptr[row + 1] - rb;
        const int32_t* ix = A.indices + rb;
        const T* dv = A.data + rb;
        const bool staged = z <= kFfmStage;
        if (staged) {
            for (int q = lane; q < z; q += 32) {
                const int32_t i = ix[q];
                s_ix[q] = i;
                s_x[q] = dv[q];
                s_f[q] = A.fid[i];
            }
            __syncwarp();
        }
        for (int c = 0; c < C; ++c) {  // ffm_score_row, rust/src/ffm.rs:18-45
            T acc = T(0);
            if (staged) {
                for (int q = lane; q < z; q += 32) acc += A.w[(int64_t)s_ix[q] * C + c] * s_x[q];
                int64_t a = 0, b = 1 + lane;
                pair_step(a, b, z);
                while (a < z - 1) {  // two pairs per step, all four latent rows in flight
                    int64_t a2 = a, b2 = b + 32;
                    pair_step(a2, b2, z);
                    const bool two = a2 < z - 1;
                    const T* pa = A.v + (((int64_t)s_ix[a] * F + s_f[b]) * C + c) * k;
                    const T* pb = A.v + (((int64_t)s_ix[b] * F + s_f[a]) * C + c) * k;
                    const T* pc = two ? A.v + (((int64_t)s_ix[a2] * F + s_f[b2]) * C + c) * k : pa;
                    const T* pd = two ? A.v + (((int64_t)s_ix[b2] * F + s_f[a2]) * C + c) * k : pb;
                    T d1 = T(0), d2 = T(0);
                    for (int t = 0; t < k; t += VEC) {
                        const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
                        const Vec<T, VEC> qc = ldg_vec<T, VEC>(pc + t), qd = ldg_vec<T, VEC>(pd + t);
#pragma unroll
                        for (int u = 0; u < VEC; ++u) {
                            d1 += qa.v[u] * qb.v[u];
                            d2 += qc.v[u] * qd.v[u];
                        }
                    }
                    acc += d1 * s_x[a] * s_x[b];
                    if (!two) break;
                    acc += d2 * s_x[a2] * s_x[b2];
                    a = a2;
                    b = b2 + 32;
                    pair_step(a, b, z);
                }
            } else {
                for (int64_t q = lane; q < z; q += 32) acc += A.w[(int64_t)ix[q] * C + c] * dv[q];
                int64_t a = 0, b = 1 + lane;
                pair_step(a, b, z);
                while (a < z - 1) {
                    const int32_t ia = ix[a], ib = ix[b];
                    const int fa = A.fid[ia], fb = A.fid[ib];
                    const T* pa = A.v + (((int64_t)ia * F + fb) * C + c) * k;
                    const T* pb = A.v + (((int64_t)ib * F + fa) * C + c) * k;
                    T dot = T(0);
                    for (int t = 0; t < k; t += VEC) {
                        const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
#pragma unroll
                        for (int u = 0; u < VEC; ++u) dot += qa.v[u] * qb.v[u];
                    }
                    acc += dot * dv[a] * dv[b];
                    b += 32;
                    pair_step(a, b, z);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) logit[c] = A.w0[c] + acc;
        }
        __syncwarp();
        if (lane == 0) row_gradients(A, row, logit, gs);
        __syncwarp();
        for (int c = lane; c < C; c += 32) A.grow[j * C + c] = gs[c];
        const int64_t e1 = A.estart1[pos] - A.seg1;
        for (int64_t q = lane; q < z * C; q += 32) {
            const int64_t a = q / C;
            const int c = (int)(q - a * C);
            A.pay1[(int64_t)A.inv1[A.seg1 + e1 + a] * A.W1 + c] = gs[c] * dv[a];
        }
        const int64_t e2 = A.estart2[pos] - A.seg2;
        if (staged) {  // one ordered pair per lane step: k-wide vector gathers and stores
            for (int64_t pe = lane; pe < z * (z - 1); pe += 32) {
                const int64_t a = pe / (z - 1), bi = pe - a * (z - 1), b = bi < a ? bi : bi + 1;
                const T xa = s_x[a], xb = s_x[b];
                const T* src = A.v + ((int64_t)s_ix[b] * F + s_f[a]) * CK;
                T* P = A.pay2 + (int64_t)A.inv2[A.seg2 + e2 + pe] * A.W2;
                for (int c = 0; c < C; ++c)
                    for (int t = 0; t < k; t += VEC) {
                        const Vec<T, VEC> q = ldg_vec<T, VEC>(src + c * k + t);
                        Vec<T, VEC> o;
#pragma unroll
                        for (int u = 0; u < VEC; ++u) o.v[u] = gs[c] * xa * xb * q.v[u];
                        *reinterpret_cast<Vec<T, VEC>*>(P + c * k + t) = o;
                    }
            }
        } else {
            const int64_t tot = z * (z - 1) * CK;
            for (int64_t q = lane; q < tot; q += 32) {
                const int64_t pe = q / CK;
                const int col = (int)(q - pe * CK);
                const int64_t a = pe / (z - 1), bi = pe - a * (z - 1), b = bi < a ? bi : bi + 1;
                const int c = col / k, t = col - c * k;
                const int32_t ib = ix[b];
                const int fa = A.fid[ix[a]];
                A.pay2[(int64_t)A.inv2[A.seg2 + e2 + pe] * A.W2 + col] =
                    gs[c] * dv[a] * dv[b] * A.v[(((int64_t)ib * F + fa) * C + c) * k + t];
            }
        }
        __syncwarp();
    }
}

// FwFM (binary and multiclass). Device layouts: V (n, C, k), R (F*F, C).
// Stream 1 (FEAT) payload per nonzero a: [g_c x_a | g_c x_a sum_{b!=a}
// r_c(f_a,f_b) x_b v_{b,c,:}]; stream 2 (PAIR) payload per pair a < b:
// [g_c x_a x_b <v_a,c, v_b,c>] (FwfmGradAccum::add_row, rust/src/fwfm.rs:140-183).
template <class T, int VEC>
__global__ void __launch_bounds__(256) fwfm_forward_kernel(FwdArgs<T> A) {
    extern __shared__ unsigned char smraw[];
    const int C = A.C, k = A.k, F = A.F, W1 = A.W1, CK = C * k;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    T* logit = reinterpret_cast<T*>(smraw) + (size_t)wib * 2 * C;
    T* gs = logit + C;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < A.nrows;
         j += nwarps) {
        const int64_t pos = A.pos0 + j, row = A.order[pos];
        const int64_t rb = A.indptr[row], z = A.indptr[row + 1] - rb;
        const int32_t* ix = A.indices + rb;
        const T* dv = A.data + rb;
        for (int c = 0; c < C; ++c) {  // fwfm_score_row, rust/src/fwfm.rs:24-53
            T acc = T(0);
            for (int64_t q = lane; q < z; q += 32) acc += A.w[(int64_t)ix[q] * C + c] * dv[q];
            int64_t a = 0, b = 1 + lane;
            pair_step(a, b, z);
            while (a < z - 1) {
                const int32_t ia = ix[a], ib = ix[b];
                const int fa = A.fid[ia], fb = A.fid[ib];
                const T rw = A.r[(int64_t)(fa <= fb ? fa * F + fb : fb * F + fa) * C + c];
                const T* pa = A.v + ((int64_t)ia * C + c) * k;
                const T* pb = A.v + ((int64_t)ib * C + c) * k;
                T dot = T(0);
                for (int t = 0; t < k; t += VEC) {
                    const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
#pragma unroll
                    for (int u = 0; u < VEC; ++u) dot += qa.v[u] * qb.v[u];
                }
                acc += rw * dot * dv[a] * dv[b];
                b += 32;
                pair_step(a, b, z);
            }
            acc = warp_sum(acc);
            if (lane == 0) logit[c] = A.w0[c] + acc;
        }
        __syncwarp();
        if (lane == 0) row_gradients(A, row, logit, gs);
        __syncwarp();
        for (int c = lane; c < C; c += 32) A.grow[j * C + c] = gs[c];
        const int64_t e1 = A.estart1[pos] - A.seg1;
        const int W1u = CK + C;  // used columns: [v (C*k) | w (C)]
        for (int64_t q = lane; q < z * W1u; q += 32) {
            const int64_t a = q / W1u;
            const int col = (int)(q - a * W1u);
            T val;
            if (col >= CK) {
                val = gs[col - CK] * dv[a];
            } else {
                const int c = col / k, t = col - c * k;
                const int fa = A.fid[ix[a]];
                T s = T(0);
                for (int64_t b = 0; b < z; ++b) {
                    if (b == a) continue;
                    const int32_t ib = ix[b];
                    const int fb = A.fid[ib];
                    const T rw = A.r[(int64_t)(fa <= fb ? fa * F + fb : fb * F + fa) * C + c];
                    s += rw * dv[b] * A.v[((int64_t)ib * C + c) * k + t];
                }
                val = gs[c] * dv[a] * s;
            }
            A.pay1[(int64_t)A.inv1[A.seg1 + e1 + a] * W1 + col] = val;
        }
        const int64_t e2 = A.estart2[pos] - A.seg2;
        int64_t a = 0, b = 1 + lane, pi = lane;
        pair_step(a, b, z);
        while (a < z - 1) {
            const int32_t ia = ix[a], ib = ix[b];
            const T xab = dv[a] * dv[b];
            for (int c = 0; c < C; ++c) {
                const T* pa = A.v + ((int64_t)ia * C + c) * k;
                const T* pb = A.v + ((int64_t)ib * C + c) * k;
                T dot = T(0);
                for (int t = 0; t < k; ++t) dot += pa[t] * pb[t];
                A.pay2[(int64_t)A.inv2[A.seg2 + e2 + pi] * A.W2 + c] = gs[c] * xab * dot;
            }
            b += 32;
            pi += 32;
            pair_step(a, b, z);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------- reduce + optimizer --

template <class T>
struct RedArgs {
    const ItemDesc* desc;       // this batch's items start at desc[item0]
    const int64_t* item_start;  // per run
    const int64_t* long_list;   // runs with several items
    const T* pay;               // batch payload rows in sorted order, stride Wp
    T* part;                    // item partials (batch-local item index), stride Wp
    int W, Wp, cb1;             // used columns, row stride, first column of group 1
    int nv, nvs, gpw;           // vectors per row, vectors per lane group, groups per warp
    int vec0;                   // 1: vectors lying inside group 0 step with 16-byte accesses
    int64_t seg, item0;
    GroupDev<T> g0, g1;
    OptDev opt;
    T inv_bsz;
    // w0 step (last block of stage 2)
    const T* grow;
    int64_t nrows;
    int C, do_w0;
    GroupDev<T> gw0;
};

template <class T>
__device__ __forceinline__ void apply_col(const RedArgs<T>& R, uint32_t key, int col, T sum) {
    if (col < R.cb1)
        opt_step(R.g0, (int64_t)key * R.g0.width + col, sum * R.inv_bsz, R.opt);
    else
        opt_step(R.g1, (int64_t)key * R.g1.width + (col - R.cb1), sum * R.inv_bsz, R.opt);
}

// Applies one VEC-wide column vector `vv` of key `key`: 16-byte accesses when
// the vector lies inside group 0 (the latent columns), scalar steps otherwise.
template <class T, int VEC>
__device__ __forceinline__ bool vec_in_group0(const RedArgs<T>& R, int vv) {
    return R.vec0 && (vv + 1) * VEC <= R.cb1;
}

// Stage 1: lane groups of nvs lanes, gpw groups per warp, one work item per
// group; each lane sums VEC-wide column vectors over the item's contiguous
// payload rows. Items of single-item runs apply the optimizer directly.
template <class T, int VEC>
__device__ __forceinline__ void reduce_items_dev(const RedArgs<T>& R, int64_t n_items,
                                                 int64_t warp0, int64_t nwarps) {
    const int lane = threadIdx.x & 31, grp = lane / R.nvs, vl = lane % R.nvs;
    if (grp >= R.gpw) return;
    for (int64_t wi = warp0;; wi += nwarps) {
    const int64_t it = wi * R.gpw + grp;
    if (it >= n_items) return;
    const ItemDesc d = R.desc[R.item0 + it];
    const int cnt = (int)(d.cnt & ~kMultiItem);
    const bool multi = (d.cnt & kMultiItem) != 0;
    const T* rows = R.pay + (d.p0 - R.seg) * R.Wp;
    for (int vv = vl; vv < R.nv; vv += R.nvs) {
        const bool vec = !multi && vec_in_group0<T, VEC>(R, vv);
        const int64_t idx0 = (int64_t)d.key * R.g0.width + vv * VEC;
        VecStep<T, VEC> st;
        if (vec) st.prefetch(R.g0, idx0, R.opt.kind);  // overlaps the payload loads
        T acc[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) acc[c] = T(0);
#pragma unroll 4
        for (int q = 0; q < cnt; ++q) {
            const Vec<T, VEC> x = ldg_vec<T, VEC>(rows + (int64_t)q * R.Wp + vv * VEC);
#pragma unroll
            for (int c = 0; c < VEC; ++c) acc[c] += x.v[c];
        }
        if (multi) {
            Vec<T, VEC> o;
#pragma unroll
            for (int c = 0; c < VEC; ++c) o.v[c] = acc[c];
            *reinterpret_cast<Vec<T, VEC>*>(R.part + it * R.Wp + vv * VEC) = o;
        } else if (vec) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) acc[c] *= R.inv_bsz;
            st.commit(R.g0, idx0, acc, R.opt);
        } else {
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
                const int col = vv * VEC + c;
                if (col < R.W) apply_col(R, d.key, col, acc[c]);
            }
        }
    }
    }
}

template <class T, int VEC>
__global__ void __launch_bounds__(256) reduce_items_kernel(RedArgs<T> R, int64_t n_items) {
    reduce_items_dev<T, VEC>(R, n_items, ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5,
                             ((int64_t)gridDim.x * blockDim.x) >> 5);
}

// Stage 2: one block per multi-item run. 8 warps x gp lane groups take the
// run's item partials in a fixed stride, a shuffle tree folds the groups of a
// warp and shared memory folds the warps in order, then the run is applied.
// The last block steps w0 from the batch's per-row gradients (fixed tree).
// w0: the batch's per-row gradients summed in a fixed tree by one block,
// then one step per class (step_param with l1 = l2 = 0, optimizer.rs:114-135).
// Sum of grow[j * C + c] over j < nrows in a fixed tree (valid in thread 0);
// every thread of the block calls it.
template <class T>
__device__ __forceinline__ T block_sum_rows(const T* grow, int64_t nrows, int C, int c, T* sm) {
    T s = T(0);
    const int64_t bd = blockDim.x;
    int64_t j = threadIdx.x;
    for (; j + 7 * bd < nrows; j += 8 * bd) {  // eight loads in flight, same order
        T a[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = grow[(j + u * bd) * C + c];
#pragma unroll
        for (int u = 0; u < 8; ++u) s += a[u];
    }
    for (; j < nrows; j += bd) s += grow[j * C + c];
    sm[threadIdx.x] = s;
    __syncthreads();
    for (int h = blockDim.x / 2; h > 0; h >>= 1) {
        if (threadIdx.x < h) sm[threadIdx.x] += sm[threadIdx.x + h];
        __syncthreads();
    }
    const T r = sm[0];
    __syncthreads();
    return r;
}

template <class T>
__device__ __forceinline__ void w0_step_dev(const T* grow, int64_t nrows, int C, T inv_bsz,
                                            const GroupDev<T>& gw0, const OptDev& opt, T* sm) {
    for (int c = 0; c < C; ++c) {
        const T tot = block_sum_rows(grow, nrows, C, c, sm);
        if (threadIdx.x == 0) opt_step(gw0, c, tot * inv_bsz, opt);
    }
}

template <class T>
__device__ __forceinline__ void w0_dev(const RedArgs<T>& R, T* sm) {
    w0_step_dev(R.grow, R.nrows, R.C, R.inv_bsz, R.gw0, R.opt, sm);
}

template <class T, int VEC>
__device__ __forceinline__ void reduce_runs_dev(const RedArgs<T>& R, int64_t l0, int64_t n_long,
                                                int64_t blk0, int64_t nblk, T (*wsum)[32 * VEC]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int gp = 1;  // power-of-two group count per warp for the shuffle fold
    while (gp * 2 * R.nvs <= 32) gp *= 2;
    const int grp = lane / R.nvs, vl = lane % R.nvs;
    const bool in = grp < gp;
    const int stride = gp * 8, slot = warp * gp + grp;
    for (int64_t li = blk0; li < n_long; li += nblk) {  // uniform per block
        const int64_t r = R.long_list[l0 + li];
        const int64_t i0 = R.item_start[r] - R.item0, i1 = R.item_start[r + 1] - R.item0;
        const uint32_t key = R.desc[R.item0 + i0].key;
        for (int vb = 0; vb < R.nv; vb += R.nvs) {
            const int vv = vb + vl;
            T acc[VEC];
#pragma unroll
            for (int c = 0; c < VEC; ++c) acc[c] = T(0);
            if (in && vv < R.nv)
                for (int64_t it = i0 + slot; it < i1; it += stride) {
                    const Vec<T, VEC> x = ldg_vec<T, VEC>(R.part + it * R.Wp + vv * VEC);
#pragma unroll
                    for (int c = 0; c < VEC; ++c) acc[c] += x.v[c];
                }
            for (int o = gp / 2; o >= 1; o >>= 1)
#pragma unroll
                for (int c = 0; c < VEC; ++c) {
                    const T y = __shfl_down_sync(0xffffffffu, acc[c], o * R.nvs);
                    if (grp < o) acc[c] += y;
                }
            if (grp == 0)
#pragma unroll
                for (int c = 0; c < VEC; ++c) wsum[warp][vl * VEC + c] = acc[c];
            __syncthreads();
            if (warp == 0 && grp == 0 && vv < R.nv) {
                T tot[VEC];
#pragma unroll
                for (int c = 0; c < VEC; ++c) {
                    tot[c] = T(0);
                    for (int w = 0; w < 8; ++w) tot[c] += wsum[w][vl * VEC + c];
                }
                if (vec_in_group0<T, VEC>(R, vv)) {
                    const int64_t idx0 = (int64_t)key * R.g0.width + vv * VEC;
                    VecStep<T, VEC> st;
                    st.prefetch(R.g0, idx0, R.opt.kind);
#pragma unroll
                    for (int c = 0; c < VEC; ++c) tot[c] *= R.inv_bsz;
                    st.commit(R.g0, idx0, tot, R.opt);
                } else {
#pragma unroll
                    for (int c = 0; c < VEC; ++c) {
                        const int col = vv * VEC + c;
                        if (col < R.W) apply_col(R, key, col, tot[c]);
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Stage 2 as its own launch: one block per multi-item run; the last block
// steps w0.
template <class T, int VEC>
__global__ void __launch_bounds__(256) reduce_runs_kernel(RedArgs<T> R, int64_t l0, int64_t n_long) {
    __shared__ T sm[256];
    __shared__ __align__(16) T wsum[8][32 * VEC];
    if (blockIdx.x == gridDim.x - 1) {
        if (R.do_w0) w0_dev(R, sm);
        return;
    }
    reduce_runs_dev<T, VEC>(R, l0, n_long, blockIdx.x, gridDim.x - 1, wsum);
}

// ------------------------------------------ binary FM row-table reduction --
//
// Binary FM with k = NV * VEC (16-byte vectors, NV <= 8). The forward writes
// one table row per batch row, [S (k) | g | pad], S = sum_j V_j x_j the row's
// factor sum and g = dL/ds x sample weight. The reduction reads the batch's
// sorted entry stream (key, row, x) and recomputes each entry's gradient from
// the table exactly as FmGradAccum::add_row forms it (rust/src/fm.rs:136-146):
//   gv[t] = g (x S[t] - V[t] x x),   gw = g x,
// so no per-entry payload is ever written.
//
// Stage 1: one block per chunk of kChunk consecutive sorted entries, one
// entry per thread; a segmented shuffle reduction per warp, then the warps'
// pieces of a segment folded in warp order; the owner of a segment (its first
// entry) applies the optimizer. A segment continued from the previous chunk
// leaves its sum in ph[chunk]; the last segment, when it continues into the
// next chunk, leaves its sum in pt[chunk].
// Stage 2: one warp per chunk boundary that starts a crossing run folds
// pt[first chunk] + ph[...] in chunk order and applies; the last block steps
// w0. Every sum has a fixed shape, so results are bitwise reproducible.

constexpr int kChunk = 256;  // sorted entries per stage-1 block

template <class T>
struct TabArgs {
    const uint32_t* keys;  // sorted keys of the epoch's entry stream
    const uint32_t* rrow;  // batch-local row of each sorted entry
    const T* rx;           // value of each sorted entry
    const T* tab;          // (nrows, TW) [S | g | pad]
    T* ph;                 // (chunks, TW) sums continued from the previous chunk
    T* pt;                 // (chunks, TW) sums continued into the next chunk
    int TW;
    int64_t seg, n;        // this batch's entries: [seg, seg + n) of the sorted stream
    int64_t nrows;
    const T* grow;         // per-row g, for w0
    T inv_bsz;
    GroupDev<T> gv, gw, gw0;
    OptDev opt;
    // data-parallel batch (dp != 0): this rank scores rows [rlo, rhi) of the
    // batch; per-run sums go to grad (run - run0, stride TW; row nrun = w0)
    // instead of the optimizer, which fm_tab_apply_kernel runs after the
    // cross-rank sum
    int dp;
    uint32_t rlo, rhi;
    const int64_t* runs;   // per sorted entry: runs (distinct keys) before it in the epoch
    const uint32_t* rkey;  // key of each run of the epoch
    int64_t run0, nrun;    // this batch's runs: [run0, run0 + nrun)
    T* grad;
};

// float32 with k <= 16 under SGD / AdaGrad fits 4 blocks per SM (64 registers)
template <class T, int NV, int OPT>
constexpr int tab_min_blocks() {
    return (sizeof(T) == 4 && NV <= 4 && OPT <= MFM_OPT_ADAGRAD) ? 4 : 1;
}

template <class T, int VEC, int NV, int OPT>
__global__ void __launch_bounds__(kChunk, (tab_min_blocks<T, NV, OPT>())) fm_tab_reduce_kernel(TabArgs<T> A) {
    constexpr int K = VEC * NV, NVAL = K + 1, NW = kChunk / 32;
    __shared__ __align__(16) T wpart[NW][NVAL];
    __shared__ int wflag[NW];  // bit 0: lane 0 continues the previous warp; bit 1: one segment
    __shared__ uint32_t s_last;
    __shared__ int s_out;
    const unsigned FULL = 0xffffffffu;
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c0 = (int64_t)blockIdx.x * kChunk, i = c0 + tid;
    const int64_t cend = c0 + kChunk < A.n ? c0 + kChunk : A.n;
    const bool valid = i < A.n;
    const int64_t gi = A.seg + i;
    // prologue on the plan's arrays (not written by the predecessor)
    if (tid == 0) {
        const uint32_t lk = A.keys[A.seg + cend - 1];
        s_last = lk;
        s_out = cend < A.n && A.keys[A.seg + cend] == lk;
    }
    uint32_t key = 0, row = 0;
    T x = T(0);
    if (valid) {
        key = A.keys[gi];
        row = A.rrow[gi];
        x = A.rx[gi];
    }
    uint32_t kprev = __shfl_up_sync(FULL, key, 1);
    if (lane == 0) kprev = (valid && i > 0) ? A.keys[gi - 1] : ~key;
    const bool rhead = valid && (i == 0 || key != kprev);
    // warp segments start at real heads, at lane 0 and at every invalid lane
    const unsigned hm = __ballot_sync(FULL, rhead || lane == 0 || !valid);
    const unsigned after = hm & ~((2u << lane) - 1u);
    const int send = after ? __ffs(after) - 2 : 31;

    pdl_wait();  // the row table and the parameters are the predecessors' output
    T val[NVAL];
    // data-parallel: rows of other ranks' slices add nothing here
    const bool mine = valid && (!A.dp || (row >= A.rlo && row < A.rhi));
    if (mine) {
        const T* tr = A.tab + (int64_t)row * A.TW;
        const T* vp = A.gv.p + (int64_t)key * K;
        const T g = tr[K];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const Vec<T, VEC> sv = ldg_vec<T, VEC>(tr + v * VEC);
            const Vec<T, VEC> vk = ldg_vec<T, VEC>(vp + v * VEC);
#pragma unroll
            for (int u = 0; u < VEC; ++u) val[v * VEC + u] = g * (x * sv.v[u] - vk.v[u] * x * x);
        }
        val[K] = g * x;
    } else {
#pragma unroll
        for (int q = 0; q < NVAL; ++q) val[q] = T(0);
    }
    // segmented suffix sums: lane l ends with the sum over [l, send]; steps
    // beyond the warp's longest segment add nothing and are skipped
    const int seglen = (rhead || lane == 0) ? send - lane + 1 : 1;
    const int maxlen = (int)__reduce_max_sync(FULL, (unsigned)seglen);
    for (int o = 1; o < maxlen; o <<= 1) {
        const bool take = lane + o <= send;
#pragma unroll
        for (int q = 0; q < NVAL; ++q) {
            const T y = __shfl_down_sync(FULL, val[q], o);
            if (take) val[q] += y;
        }
    }
    if (lane == 0) {
        const bool cont = valid && !rhead && warp > 0;
        wflag[warp] = (cont ? 1 : 0) | (send == 31 ? 2 : 0);
        if (cont)
#pragma unroll
            for (int q = 0; q < NVAL; ++q) wpart[warp][q] = val[q];
    }
    __syncthreads();
    const bool owner = valid && (rhead || tid == 0);
    if (!owner) return;
    if (send == 31)
        for (int w2 = warp + 1; w2 < NW; ++w2) {
            const int f = wflag[w2];
            if (!(f & 1)) break;
#pragma unroll
            for (int q = 0; q < NVAL; ++q) val[q] += wpart[w2][q];
            if (!(f & 2)) break;
        }
    const int64_t cb = blockIdx.x;
    T* dst = nullptr;
    if (tid == 0 && !rhead)
        dst = A.ph + cb * A.TW;
    else if (s_out && key == s_last)
        dst = A.pt + cb * A.TW;
    if (dst) {
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            Vec<T, VEC> o;
#pragma unroll
            for (int u = 0; u < VEC; ++u) o.v[u] = val[v * VEC + u];
            *reinterpret_cast<Vec<T, VEC>*>(dst + v * VEC) = o;
        }
        dst[K] = val[K];
        return;
    }
    if (A.dp) {  // the run's sum for this rank, stepped after the cross-rank sum
        T* gd = A.grad + (A.runs[gi] - A.run0) * A.TW;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            Vec<T, VEC> o;
#pragma unroll
            for (int u = 0; u < VEC; ++u) o.v[u] = val[v * VEC + u];
            *reinterpret_cast<Vec<T, VEC>*>(gd + v * VEC) = o;
        }
        gd[K] = val[K];
        return;
    }
    // the whole run lies in this chunk: one optimizer step per coordinate
    VecStep<T, VEC, OPT> st[NV];
    VecStep<T, 1, OPT> sw1;
#pragma unroll
    for (int v = 0; v < NV; ++v) st[v].prefetch(A.gv, (int64_t)key * K + v * VEC, A.opt.kind);
    sw1.prefetch(A.gw, (int64_t)key, A.opt.kind);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        T dg[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) dg[u] = val[v * VEC + u] * A.inv_bsz;
        st[v].commit(A.gv, (int64_t)key * K + v * VEC, dg, A.opt);
    }
    const T dgw = val[K] * A.inv_bsz;
    sw1.commit(A.gw, (int64_t)key, &dgw, A.opt);
}

template <class T, int VEC, int NV>
__global__ void __launch_bounds__(256) fm_tab_fold_kernel(TabArgs<T> A, int64_t nchunks) {
    constexpr int K = VEC * NV;
    const unsigned FULL = 0xffffffffu;
    pdl_trigger();
    if (blockIdx.x == gridDim.x - 1) {
        __shared__ T sm[256];
        pdl_wait();
        if (!A.dp) {
            w0_step_dev(A.grow, A.nrows, 1, A.inv_bsz, A.gw0, A.opt, sm);
        } else {  // this rank's slice sum; stepped after the cross-rank sum
            const T tot = block_sum_rows(A.grow + A.rlo, (int64_t)(A.rhi - A.rlo), 1, 0, sm);
            if (threadIdx.x == 0) A.grad[A.nrun * A.TW] = tot;
        }
        return;
    }
    const int lane = threadIdx.x & 31;
    const int64_t c = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) + 1;
    if (c >= nchunks) {  // uniform per warp
        pdl_wait();
        return;
    }
    // prologue on the sorted keys: lane i reads the first key of chunk c + i;
    // lane 0 also the keys just before chunks c and c - 1
    const int64_t jl = c + lane;
    const uint32_t fk = jl < nchunks ? A.keys[A.seg + jl * kChunk] : 0u;
    uint32_t kb = 0, kq = 0;
    if (lane == 0) {
        kb = A.keys[A.seg + c * kChunk - 1];
        kq = c >= 2 ? A.keys[A.seg + (c - 1) * kChunk - 1] : 0u;
    }
    const uint32_t key = __shfl_sync(FULL, fk, 0);
    const int stop = lane == 0 ? (kb != key || (c >= 2 && kq == key)) : 0;
    // boundary c is not crossed, or is not the run's first crossed boundary
    if (__shfl_sync(FULL, stop, 0)) {
        pdl_wait();
        return;
    }
    int ones = __popc(__ballot_sync(FULL, jl < nchunks && fk == key));
    int64_t j1 = c + ones - 1;  // last chunk whose ph belongs to the run (keys are sorted)
    for (int64_t jb = c + 32; ones == 32; jb += 32) {
        const int64_t j = jb + lane;
        ones = __popc(__ballot_sync(FULL, j < nchunks && A.keys[A.seg + j * kChunk] == key));
        j1 = jb + ones - 1;
    }
    pdl_wait();  // the partials and the parameters are the predecessors' output
    // the run's partials: element 0 = pt[c - 1], element e >= 1 = ph[c + e - 1];
    // each lane loads one element, a butterfly folds every 32 of them (all
    // lanes end with the same bits), the groups of 32 are added in order
    const int64_t cnt = j1 - c + 2;
    const int own = lane < NV ? lane : NV;  // column vector this lane applies (NV = w)
    VecStep<T, VEC> st;
    VecStep<T, 1> s1;
    if (!A.dp) {
        if (lane < NV)
            st.prefetch(A.gv, (int64_t)key * K + lane * VEC, A.opt.kind);
        else if (lane == NV)
            s1.prefetch(A.gw, (int64_t)key, A.opt.kind);
    }
    T tot[K + 1];
#pragma unroll
    for (int q = 0; q <= K; ++q) tot[q] = T(0);
    for (int64_t e0 = 0; e0 < cnt; e0 += 32) {
        const int64_t e = e0 + lane;
        T part[K + 1];
        if (e < cnt) {
            const T* r = e == 0 ? A.pt + (c - 1) * A.TW : A.ph + (c + e - 1) * A.TW;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const Vec<T, VEC> x = ldg_vec<T, VEC>(r + v * VEC);
#pragma unroll
                for (int u = 0; u < VEC; ++u) part[v * VEC + u] = x.v[u];
            }
            part[K] = r[K];
        } else {
#pragma unroll
            for (int q = 0; q <= K; ++q) part[q] = T(0);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int q = 0; q <= K; ++q) part[q] += __shfl_xor_sync(FULL, part[q], o);
#pragma unroll
        for (int q = 0; q <= K; ++q) tot[q] += part[q];
    }
    if (A.dp) {  // the run's sum for this rank (its head entry lies before chunk c)
        T* gd = A.grad + (A.runs[A.seg + c * kChunk] - 1 - A.run0) * A.TW;
        if (lane < NV) {
            Vec<T, VEC> o;
#pragma unroll
            for (int u = 0; u < VEC; ++u) {
                T t = T(0);
#pragma unroll
                for (int v = 0; v < NV; ++v)
                    if (v == own) t = tot[v * VEC + u];
                o.v[u] = t;
            }
            *reinterpret_cast<Vec<T, VEC>*>(gd + lane * VEC) = o;
        } else if (lane == NV) {
            gd[K] = tot[K];
        }
        return;
    }
    if (lane < NV) {
        T dg[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) {
            T t = T(0);
#pragma unroll
            for (int v = 0; v < NV; ++v)
                if (v == own) t = tot[v * VEC + u];
            dg[u] = t * A.inv_bsz;
        }
        st.commit(A.gv, (int64_t)key * K + lane * VEC, dg, A.opt);
    } else if (lane == NV) {
        const T dg = tot[K] * A.inv_bsz;
        s1.commit(A.gw, (int64_t)key, &dg, A.opt);
    }
}

// Data-parallel step: after the cross-rank sum of grad, one warp per run of
// the batch applies the optimizer to its key (NV vector lanes + the w lane),
// identically on every rank; thread 0 of block 0 also steps w0.
template <class T, int VEC, int NV>
__global__ void __launch_bounds__(256) fm_tab_apply_kernel(TabArgs<T> A) {
    constexpr int K = VEC * NV;
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t key = j < A.nrun ? A.rkey[A.run0 + j] : 0u;  // plan data
    pdl_wait();  // grad is the cross-rank sum
    if (blockIdx.x == 0 && threadIdx.x == 0)
        opt_step(A.gw0, 0, A.grad[A.nrun * A.TW] * A.inv_bsz, A.opt);
    if (j >= A.nrun) return;
    const T* gd = A.grad + j * A.TW;
    if (lane < NV) {
        const int64_t idx0 = (int64_t)key * K + lane * VEC;
        VecStep<T, VEC> st;
        st.prefetch(A.gv, idx0, A.opt.kind);
        const Vec<T, VEC> g = ldg_vec<T, VEC>(gd + lane * VEC);
        T dg[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) dg[u] = g.v[u] * A.inv_bsz;
        st.commit(A.gv, idx0, dg, A.opt);
    } else if (lane == NV) {
        VecStep<T, 1> s1;
        s1.prefetch(A.gw, (int64_t)key, A.opt.kind);
        const T dg = gd[K] * A.inv_bsz;
        s1.commit(A.gw, (int64_t)key, &dg, A.opt);
    }
}

// --------------------------------------------------- persistent epoch loop --
//
// FM training runs a whole epoch's batch loop in one cooperative launch (all
// blocks co-resident): forward -> barrier -> stage 1 (+ w0 by block 0) ->
// [barrier -> stage 2, when the batch has multi-item runs] -> barrier. The
// grid barrier's wait is bounded: after kBarrierSpinLimit polls it records an
// error and moves on, so the launch always ends and the host reports
// MFM_ERR_DEVICE_CHECK instead of waiting forever.

struct GridBar {
    unsigned int count, gen, err, pad;
};
constexpr unsigned long long kBarrierSpinLimit = 1ull << 24;  // polls of ~100 ns

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void grid_barrier(GridBar* bar, unsigned int& gen) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int g = gen;
        __threadfence();  // release this block's writes
        const unsigned int arrived = atomicAdd(&bar->count, 1u);
        if (arrived == gridDim.x - 1) {
            atomicExch(&bar->count, 0u);
            __threadfence();
            atomicExch(&bar->gen, g + 1u);
        } else {
            unsigned long long polls = 0;
            while (ld_acquire_gpu(&bar->gen) == g) {
                if (++polls > kBarrierSpinLimit) {
                    atomicOr(&bar->err, 1u);
                    break;
                }
                __nanosleep(100);
            }
        }
        __threadfence();  // acquire the other blocks' writes
    }
    ++gen;
    __syncthreads();
}

template <class T>
struct EpochArgs {
    FwdArgs<T> fwd;  // per-batch fields are filled in the loop
    RedArgs<T> red;
    const int64_t* seg_lo;  // per-batch entry starts (nb + 1)
    const int64_t* bitem;   // per-batch first work item (nb + 1)
    const int64_t* blong;   // per-batch first multi-item run (nb + 1)
    int64_t nb, B, n_rows;
    GridBar* bar;
};

// FK = 0: row-group forward <L = P1, LR = P2, CAP = P3>; FK = 1: generic
// forward with MCOL = P1 (multiclass and other widths).
template <class T, int VEC, int FK, int P1, int P2, int P3>
__global__ void __launch_bounds__(256, 2) fm_epoch_kernel(EpochArgs<T> E, int lgc) {
    extern __shared__ __align__(16) unsigned char smraw[];
    T* sm = reinterpret_cast<T*>(smraw);
    T(*wsum)[32 * VEC] = reinterpret_cast<T(*)[32 * VEC]>(sm + 256);
    unsigned char* fwd_smem = reinterpret_cast<unsigned char*>(sm + 256 + 8 * 32 * VEC);
    unsigned int gen = 0;
    const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    for (int64_t b = 0; b < E.nb; ++b) {
        const int64_t pos0 = b * E.B;
        const int64_t nrows = E.n_rows - pos0 < E.B ? E.n_rows - pos0 : E.B;
        FwdArgs<T> A = E.fwd;
        A.pos0 = pos0;
        A.nrows = nrows;
        A.seg1 = E.seg_lo[b];
        if constexpr (FK == 0)
            fm_forward_rows_dev<T, VEC, P1, P2, P3>(A, gtid / P2, nthreads / P2);
        else
            fm_forward_dev<T, P1>(A, lgc, fwd_smem, gtid >> 5, nthreads >> 5);
        grid_barrier(E.bar, gen);
        RedArgs<T> R = E.red;
        R.seg = A.seg1;
        R.item0 = E.bitem[b];
        R.nrows = nrows;
        R.inv_bsz = T(1) / (T)nrows;
        const int64_t n_items = E.bitem[b + 1] - R.item0;
        const int64_t l0 = E.blong[b], nl = E.blong[b + 1] - l0;
        if (blockIdx.x == 0) w0_dev(R, sm);
        reduce_items_dev<T, VEC>(R, n_items, gtid >> 5, nthreads >> 5);
        if (nl > 0) {
            grid_barrier(E.bar, gen);
            reduce_runs_dev<T, VEC>(R, l0, nl, blockIdx.x, gridDim.x, wsum);
        }
        grid_barrier(E.bar, gen);
    }
}

// ----------------------------------------------------------------- host --

// Phase timing on the training stream, printed to stderr when the
// environment variable MFM_B200_TIMING is set (diagnostics only).
struct PhaseTimer {
    bool on = false;
    cudaStream_t s = nullptr;
    cudaEvent_t last = nullptr;
    std::string report;
    explicit PhaseTimer(cudaStream_t st) : s(st) {
        const char* e = getenv("MFM_B200_TIMING");
        on = e && *e && *e != '0';
        if (on) {
            cudaEventCreate(&last);
            cudaEventRecord(last, s);
        }
    }
    void mark(const char* name) {
        if (!on) return;
        cudaEvent_t now;
        cudaEventCreate(&now);
        cudaEventRecord(now, s);
        cudaEventSynchronize(now);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, last, now);
        cudaEventDestroy(last);
        last = now;
        report += fmt(" %s=%.3fms", name, ms);
    }
    ~PhaseTimer() {
        if (!on) return;
        if (last) cudaEventDestroy(last);
        fprintf(stderr, "mfm timing:%s\n", report.c_str());
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
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
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
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        return a;
    }();
    if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.CommDestroy ||
        !api.GetErrorString)
        fail(MFM_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    return api;
}
#define MFM_NCCL(call, what)                                                          \
    do {                                                                              \
        const ncclResult_t r_ = (call);                                               \
        if (r_ != ncclSuccess)                                                        \
            fail(MFM_ERR_CUDA, fmt("%s: %s", what, nccl().GetErrorString(r_)));       \
    } while (0)

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
        return v > 0 ? (int64_t)v : (int64_t)32;
    }();
    return w;
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
    int TW = 0;
    DevBuf<uint32_t> erow, pidx;  // pidx: keys in epoch entry order (CSR indices by position)
    DevBuf<T> ex, rx, table, ph, pt, py, psw;
    uint32_t* rrow = nullptr;
    SortTiles tiles;
    // data-parallel: runs (distinct keys per batch) of the sorted stream
    DevBuf<int32_t> head;
    DevBuf<int64_t> runs;     // per entry: runs before it in the epoch (N + 1)
    DevBuf<uint32_t> rkey;    // key of each run
    DevBuf<int64_t> brun;     // runs before each batch (nb + 1)
    std::vector<int64_t> h_run;
    DevBuf<T> grad;           // (max runs per batch + 1, TW)
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
            st_.erow.alloc(device, N1);
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
    void plan_tab_window(Stream<T>& st_, int e, int64_t b0, int64_t b1, cudaStream_t ps) {
        const int32_t* order = p_order + (int64_t)e * n_rows;
        const int64_t p0 = b0 * B, p1 = std::min(b1 * B, n_rows);
        if (p1 > p0)
            expand_kernel<T><<<warp_grid(device, p1 - p0, 8, 8), 256, 0, ps>>>(
                FEAT, order, p_indptr, p_indices, p_fid, (int)F, p0, p1, B, st_.estart.ptr,
                st_.seg_lo.ptr, st_.pidx.ptr, st_.v0.ptr, p_data, st_.erow.ptr, st_.ex.ptr);
        MFM_CHECK_LAUNCH("expand");
        SortResult sr = segmented_sort_range(
            ps, st_.pidx.ptr, st_.k0.ptr, st_.v0.ptr, st_.k1.ptr, st_.v1.ptr, st_.seg_lo.ptr, b0,
            b1, st_.tiles, bits_for(st_.n_keys),
            RecGather<T>{st_.erow.ptr, st_.ex.ptr, st_.rx.ptr});
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
            st_.estart.ptr, st_.seg_lo.ptr, st_.k0.ptr, st_.v0.ptr, p_data, nullptr,
            static_cast<T*>(nullptr));
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
        MFM_CUDA(cudaStreamSynchronize(s), "plan");
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
            s0.table.alloc(device, std::max<int64_t>(1, std::min(B, n_rows)) * s0.TW);
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
        A.TW = s0.TW;
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
        if (S[0].tab)                                                                       \
            launch_pdl(fm_forward_rows_kernel<T, VW, L_, LR_, CAP_, true>, gr, 256, s, A);  \
        else                                                                                \
            fm_forward_rows_kernel<T, VW, L_, LR_, CAP_><<<gr, 256, 0, s>>>(A);             \
        MFM_CHECK_LAUNCH("FM forward");                                                     \
        return;                                                                             \
    }
                if (nvec <= 1) MFM_FROWS(1, 16, 48)
                if (nvec <= 2) MFM_FROWS(2, 16, 48)
                if (nvec <= 4) MFM_FROWS(4, 16, 48)
                MFM_FROWS(8, 32, 32)
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
            if (v4)
                fwfm_forward_kernel<T, maxv><<<grid, 256, sm, s>>>(A);
            else if (v2)
                fwfm_forward_kernel<T, 2><<<grid, 256, sm, s>>>(A);
            else
                fwfm_forward_kernel<T, 1><<<grid, 256, sm, s>>>(A);
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
            MFM_NCCL(nccl().AllReduce(TA.grad, TA.grad, cnt,
                                      sizeof(T) == 4 ? ncclFloat32 : ncclFloat64, ncclSum,
                                      dp->comm, s),
                     "ncclAllReduce");
            launch_pdl(fm_tab_apply_kernel<T, VW, NV>,
                       (unsigned)std::max<int64_t>(1, ceil_div(TA.nrun, 8)), 256, s, TA);
        }
        MFM_CHECK_LAUNCH("row-table reduction");
    }
    void launch_tab(int64_t b, T inv_bsz, int64_t nrows, int64_t rlo, int64_t rhi) {
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
        TA.dp = dp ? 1 : 0;
        TA.rlo = (uint32_t)rlo;
        TA.rhi = (uint32_t)rhi;
        TA.runs = st_.runs.ptr;
        TA.rkey = st_.rkey.ptr;
        TA.run0 = dp ? st_.h_run[b] : 0;
        TA.nrun = dp ? st_.h_run[b + 1] - st_.h_run[b] : 0;
        TA.grad = st_.grad.ptr;
        const int64_t nchunks = ceil_div(TA.n, kChunk);
        switch (k / VW) {
        case 1: launch_tab_t<1>(TA, nchunks); break;
        case 2: launch_tab_t<2>(TA, nchunks); break;
        case 4: launch_tab_t<4>(TA, nchunks); break;
        default: launch_tab_t<8>(TA, nchunks); break;
        }
    }

    void launch_reduce(Stream<T>& st_, int64_t b, T inv_bsz, int64_t nrows, bool do_w0) {
        constexpr int VEC = 16 / (int)sizeof(T);
        const int64_t i0 = st_.h_item[b], i1 = st_.h_item[b + 1];
        const int64_t l0 = st_.h_long[b], l1 = st_.h_long[b + 1];
        RedArgs<T> R = red_args(st_, b, inv_bsz);
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
                 "a grid barrier wait gave up (blocks were not co-resident); results invalid");
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

    // Row-table path: each epoch's plan runs in windows of batches (one event
    // per window) on the plan stream, the batches on a high-priority stream
    // forked from and joined back to s.
    void run_tab(const FwdArgs<T>& base, PhaseTimer& pt) {
        const cudaStream_t caller = s;
        // MFM_B200_PLAN_OVERLAP=1 runs the plan in windows on a second stream
        // beside the batches; by default it is one window that precedes the
        // batches on one stream (the sort's blocks fill every SM, so
        // overlapping only delays the latency-bound batch kernels).
        const char* ov = getenv("MFM_B200_PLAN_OVERLAP");
        const bool overlap = ov && *ov == '1' && !dp;
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
        try {
            for (int64_t e = 0; e < E; ++e) {
                plan_tab_epoch(S[0], (int)e);
                pt.mark("plan");
                MFM_CUDA(cudaEventRecord(ev_ep, hi), "event");
                MFM_CUDA(cudaStreamWaitEvent(lo, ev_ep, 0), "event");
                for (size_t w = 0; w < win.size(); ++w) {
                    plan_tab_window(S[0], (int)e, win[w].first, win[w].second, lo);
                    MFM_CUDA(cudaEventRecord(ev.e[w], lo), "event");
                }
                if (dp) plan_tab_runs(S[0]);
                for (size_t w = 0; w < win.size(); ++w) {
                    MFM_CUDA(cudaStreamWaitEvent(hi, ev.e[w], 0), "event");
                    for (int64_t b = win[w].first; b < win[w].second; ++b) {
                        const int64_t pos0 = b * B, nrows = std::min(B, n_rows - pos0);
                        const T inv_bsz = T(1) / (T)nrows;  // batch length (fm.rs:395-398)
                        // data-parallel: this rank scores rows [rlo, rhi) of the batch
                        const int64_t rlo = dp ? nrows * dp->rank / dp->world : 0;
                        const int64_t rhi = dp ? nrows * (dp->rank + 1) / dp->world : nrows;
                        FwdArgs<T> A = base;
                        A.pos0 = pos0 + rlo;
                        A.nrows = rhi - rlo;
                        A.tab = base.tab + rlo * base.TW;
                        A.grow = base.grow + rlo;
                        A.indptr = S[0].estart.ptr;  // rows by epoch position
                        A.indices = reinterpret_cast<const int32_t*>(S[0].pidx.ptr);
                        A.data = S[0].ex.ptr;
                        A.y = S[0].py.ptr;
                        A.sw = S[0].psw.ptr;
                        launch_forward(A, rhi - rlo);
                        launch_tab(b, inv_bsz, nrows, rlo, rhi);
                    }
                }
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

    void run(const FwdArgs<T>& base, PhaseTimer& pt) {
        if (S[0].tab) {
            run_tab(base, pt);
            return;
        }
        for (int64_t e = 0; e < E; ++e) {
            for (int si = 0; si < n_streams; ++si) plan(S[si], (int)e);
            pt.mark("plan");
            {
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
                FwdArgs<T> A = base;
                A.order = p_order + e * n_rows;
                A.pos0 = pos0;
                A.nrows = nrows;
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
                launch_forward(A, nrows);
                for (int si = 0; si < n_streams; ++si)
                    launch_reduce(S[si], b, inv_bsz, nrows, si == n_streams - 1);
            }
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
void fit_impl(const FitSpec& f, int device) {
    DeviceGuard guard(device);
    std::lock_guard<std::mutex> lk(device_mutex(device));
    Trainer<T> tr;
    tr.device = device;
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

void fit_dispatch(const FitSpec& f, const mfm_exec* ex) {
    validate_fit(f);
    const int dtype = ex ? ex->dtype : MFM_DTYPE_F64;
    const int device = ex ? ex->device : 0;
    if (dtype == MFM_DTYPE_F64)
        fit_impl<double>(f, device);
    else if (dtype == MFM_DTYPE_F32)
        fit_impl<float>(f, device);
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
    if (dp && !tr.S[0].tab)
        fail(MFM_ERR_UNSUPPORTED,
             fmt("data-parallel training supports k = %d, %d, %d or %d in this dtype, got %lld",
                 16 / (int)sizeof(T), 32 / (int)sizeof(T), 64 / (int)sizeof(T),
                 128 / (int)sizeof(T), (long long)k));
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
        ncclComm_t c = nullptr;
        MFM_NCCL(nccl().CommInitRank(&c, world, u, rank), "ncclCommInitRank");
        *out = new mfm_dp{c, world, rank, device};
    });
}

extern "C" int mfm_dp_destroy(mfm_dp* dp) {
    return guarded([&] {
        if (!dp) return;
        DeviceGuard guard(dp->device);
        const ncclComm_t c = dp->comm;
        delete dp;
        MFM_NCCL(nccl().CommDestroy(c), "ncclCommDestroy");
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
