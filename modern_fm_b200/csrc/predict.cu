// predict.cu — sm_100a CSR scoring kernels for FM, FFM and FwFM, and the
// host entry points that replace the reference's cuda::{fm,ffm,fwfm}::predict_csr.
//
// Design (memory-bound sparse gather; no tensor-core work exists here):
//  * one warp per CSR row, grid sized to the SM count, rows strided by warp;
//  * the row's (index, value) slice is read once, 32 nonzeros per coalesced
//    load, and broadcast to the lanes that gather with warp shuffles;
//  * FM: a nonzero's latent row is split over L = 2^lg lanes with 16-byte
//    vector loads (k=16 float32: 4 lanes x float4 -> 8 nonzeros in flight per
//    warp step); lane groups are combined with xor shuffles and the
//    sum-of-squares identity finishes in registers: O(nnz k) per row;
//  * FFM / FwFM: the row's upper-triangle pair list (a < b, the reference's
//    pair order) is walked 32 pairs at a time, one pair per lane, each pair a
//    k-long dot of two vector-loaded latent rows: O(z^2 k) per row.
#include <algorithm>
#include <exception>
#include <thread>

#include "common.cuh"

namespace mfm {

constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------------ FM ----

template <class T, class IdxT, class ValT, class OutT, int VEC, int JMAX>
__global__ void __launch_bounds__(256)
    fm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                      const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base, T w0,
                      const T* __restrict__ w, const T* __restrict__ v, int k, int lg,
                      OutT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int L = 1 << lg;
    const int G = 32 >> lg;
    const int grp = lane >> lg;
    const int l = lane & (L - 1);
    const int nvec = k / VEC;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base, e = indptr[row + 1] - nnz_base;
        T acc[JMAX][VEC];
#pragma unroll
        for (int j = 0; j < JMAX; ++j)
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[j][q] = T(0);
        T sq = T(0), lin = T(0);
        for (int64_t base = b; base < e; base += 32) {
            const int nh = (int)min((int64_t)32, e - base);
            IdxT my_i = 0;
            T my_x = T(0);
            if (lane < nh) {
                my_i = indices[base + lane];
                my_x = (T)data[base + lane];
            }
#pragma unroll 2
            for (int t = 0; t < nh; t += G) {
                const int src = t + grp;
                const IdxT i = __shfl_sync(kFull, my_i, src);
                const T x = __shfl_sync(kFull, my_x, src);
                if (src < nh) {
                    const T* vi = v + (int64_t)i * k;
                    if (l == 0) lin += w[i] * x;
#pragma unroll
                    for (int j = 0; j < JMAX; ++j) {
                        const int vv = l + j * L;
                        if (vv < nvec) {
                            const Vec<T, VEC> q = ldg_vec<T, VEC>(vi + vv * VEC);
#pragma unroll
                            for (int c = 0; c < VEC; ++c) {
                                const T vx = q.v[c] * x;
                                acc[j][c] += vx;
                                sq += vx * vx;
                            }
                        }
                    }
                }
            }
        }
        // combine the G lane groups: afterwards every group holds the row's
        // factor sums sum_i v_if x_i for its lanes' factors
        for (int o = L; o < 32; o <<= 1)
#pragma unroll
            for (int j = 0; j < JMAX; ++j)
#pragma unroll
                for (int c = 0; c < VEC; ++c) acc[j][c] += __shfl_xor_sync(kFull, acc[j][c], o);
        T pair = T(0);
        if (grp == 0) {
#pragma unroll
            for (int j = 0; j < JMAX; ++j)
                if (l + j * L < nvec)
#pragma unroll
                    for (int c = 0; c < VEC; ++c) pair += acc[j][c] * acc[j][c];
        }
        // s = w0 + sum w_i x_i + 0.5 * (sum_f (sum_i v_if x_i)^2 - sum_if (v_if x_i)^2)
        const T total = warp_sum(lin + T(0.5) * (pair - sq));
        if (lane == 0) out[row] = (OutT)(w0 + total);
    }
}

// Row-group FM kernel for latent rows of up to 16 vectors: LR lanes score one
// row (32/LR rows per warp); a nonzero's latent row is spread over L lanes
// (VEC elements each, 16-byte loads), G = LR/L nonzeros per step. One
// iteration covers CAP nonzeros: their indices and values are loaded by the
// row's lanes at once, w is gathered lane-parallel, and all CAP/G latent-row
// gathers are issued before any of them is consumed, so a 39-nonzero row makes
// three dependent memory round trips (indptr, index slice, gathers).
template <class T, class IdxT, class ValT, class OutT, int VEC, int L, int LR, int CAP, int MINB>
__global__ void __launch_bounds__(256, MINB)
    fm_rows_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                   const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base, T w0,
                   const T* __restrict__ w, const T* __restrict__ v, int k,
                   OutT* __restrict__ out) {
    constexpr int G = LR / L;     // nonzeros per step
    constexpr int NC = CAP / LR;  // index chunks per iteration
    constexpr int S = CAP / G;    // hoisted gather steps per iteration
    static_assert(LR % L == 0 && CAP % LR == 0 && 32 % LR == 0, "row-group shape");
    const int lane = threadIdx.x & 31, rl = lane & (LR - 1), grp = rl / L, l = rl % L;
    const bool act = l < k / VEC;
    const int64_t nslots = ((int64_t)gridDim.x * blockDim.x) / LR;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LR;; row += nslots) {
        const bool live = row < n_rows;
        if (!__any_sync(kFull, live)) break;
        const int64_t b = live ? indptr[row] - nnz_base : 0;
        const int64_t e = live ? indptr[row + 1] - nnz_base : 0;
        T acc[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) acc[c] = T(0);
        T sq = T(0), lin = T(0);
        for (int64_t base = b;; base += CAP) {
            const bool more = base < e;
            if (!__any_sync(kFull, more)) break;
            int nh[NC];
            IdxT ii[NC];
            T xx[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int64_t rem = e - base - LR * c;
                nh[c] = !more || rem <= 0 ? 0 : (rem >= LR ? LR : (int)rem);
                ii[c] = 0;
                xx[c] = T(0);
                if (rl < nh[c]) {
                    ii[c] = indices[base + LR * c + rl];
                    xx[c] = (T)data[base + LR * c + rl];
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if (rl < nh[c]) lin += w[ii[c]] * xx[c];
            Vec<T, VEC> q[S];
            T xs[S];
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const int c = s / L, src = (s % L) * G + grp;
                const IdxT i = __shfl_sync(kFull, ii[c], src, LR);
                const T x = __shfl_sync(kFull, xx[c], src, LR);
                const bool ok = src < nh[c];
                xs[s] = ok ? x : T(0);
                if (ok && act) {
                    q[s] = ldg_vec<T, VEC>(v + (int64_t)i * k + l * VEC);
                } else {
#pragma unroll
                    for (int cc = 0; cc < VEC; ++cc) q[s].v[cc] = T(0);
                }
            }
#pragma unroll
            for (int s = 0; s < S; ++s)
#pragma unroll
                for (int cc = 0; cc < VEC; ++cc) {
                    const T vx = q[s].v[cc] * xs[s];
                    acc[cc] += vx;
                    sq += vx * vx;
                }
        }
#pragma unroll
        for (int o = L; o < LR; o <<= 1)
#pragma unroll
            for (int cc = 0; cc < VEC; ++cc) acc[cc] += __shfl_xor_sync(kFull, acc[cc], o);
        T pair = T(0);
        if (grp == 0 && act) {
#pragma unroll
            for (int cc = 0; cc < VEC; ++cc) pair += acc[cc] * acc[cc];
        }
        T t = lin + T(0.5) * (pair - sq);
#pragma unroll
        for (int o = LR / 2; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (rl == 0 && live) out[row] = (OutT)(w0 + t);
    }
}

// The row's upper-triangle pair list (a < b, a ascending then b ascending, the
// reference's order, rust/src/ffm.rs:32-43) is walked 32 entries at a time:
// each lane advances its (a, b) cursor by 32 positions.
__device__ __forceinline__ void pair_advance(int64_t& a, int64_t& b, int64_t z) {
    while (a < z - 1 && b >= z) {
        b = b - z + a + 2;
        ++a;
    }
}

// ----------------------------------------------------------------- FFM ----

template <class T, class IdxT, class ValT, class OutT, int VEC>
__global__ void __launch_bounds__(256)
    ffm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                       const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                       const int32_t* __restrict__ fid, int F, T w0, const T* __restrict__ w,
                       const T* __restrict__ v, int k, OutT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base, z = indptr[row + 1] - nnz_base - b;
        const IdxT* ix = indices + b;
        const ValT* dv = data + b;
        T acc = T(0);
        for (int64_t q = lane; q < z; q += 32) acc += w[ix[q]] * (T)dv[q];
        int64_t a = 0, bb = 1 + lane;
        pair_advance(a, bb, z);
        while (a < z - 1) {
            const IdxT ia = ix[a], ib = ix[bb];
            const T xa = (T)dv[a], xb = (T)dv[bb];
            const int fa = fid[ia], fb = fid[ib];
            const T* pa = v + ((int64_t)ia * F + fb) * k;  // V[i_a, f_b]
            const T* pb = v + ((int64_t)ib * F + fa) * k;  // V[i_b, f_a]
            T dot = T(0);
            for (int t = 0; t < k; t += VEC) {
                const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
#pragma unroll
                for (int c = 0; c < VEC; ++c) dot += qa.v[c] * qb.v[c];
            }
            acc += dot * xa * xb;
            bb += 32;
            pair_advance(a, bb, z);
        }
        acc = warp_sum(acc);
        if (lane == 0) out[row] = (OutT)(w0 + acc);
    }
}

// ---------------------------------------------------------------- FwFM ----

template <class T, class IdxT, class ValT, class OutT, int VEC>
__global__ void __launch_bounds__(256)
    fwfm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                        const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                        const int32_t* __restrict__ fid, int F, T w0, const T* __restrict__ w,
                        const T* __restrict__ v, const T* __restrict__ r, int k,
                        OutT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base, z = indptr[row + 1] - nnz_base - b;
        const IdxT* ix = indices + b;
        const ValT* dv = data + b;
        T acc = T(0);
        for (int64_t q = lane; q < z; q += 32) acc += w[ix[q]] * (T)dv[q];
        int64_t a = 0, bb = 1 + lane;
        pair_advance(a, bb, z);
        while (a < z - 1) {
            const IdxT ia = ix[a], ib = ix[bb];
            const T xa = (T)dv[a], xb = (T)dv[bb];
            const int fa = fid[ia], fb = fid[ib];
            const T rw = fa <= fb ? r[fa * F + fb] : r[fb * F + fa];  // pair_slot, fwfm.rs:17-21
            const T* pa = v + (int64_t)ia * k;
            const T* pb = v + (int64_t)ib * k;
            T dot = T(0);
            for (int t = 0; t < k; t += VEC) {
                const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
#pragma unroll
                for (int c = 0; c < VEC; ++c) dot += qa.v[c] * qb.v[c];
            }
            acc += rw * dot * xa * xb;
            bb += 32;
            pair_advance(a, bb, z);
        }
        acc = warp_sum(acc);
        if (lane == 0) out[row] = (OutT)(w0 + acc);
    }
}

// ------------------------------------------------------------- launchers --

template <class T>
int vec_width(int64_t k) {
    constexpr int maxv = 16 / (int)sizeof(T);
    if (k % maxv == 0) return maxv;
    if (maxv >= 2 && k % 2 == 0) return 2;
    return 1;
}

constexpr int kWarpsPerBlock = 8;
constexpr int kBlocksPerSm = 8;

template <class T, class IdxT, class ValT, class OutT, int VEC>
void fm_launch_vec(unsigned grid, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                   const ValT* data, int64_t n_rows, int64_t nnz_base, T w0, const T* w,
                   const T* v, int k, OutT* out) {
    const int nvec = k / VEC;
    int L = 1, lg = 0;
    while (L < nvec && L < 32) {
        L <<= 1;
        ++lg;
    }
    const int J = (nvec + L - 1) / L;
#define MFM_FM_CASE(JM)                                                                      \
    if (J <= JM) {                                                                           \
        fm_predict_kernel<T, IdxT, ValT, OutT, VEC, JM><<<grid, kWarpsPerBlock * 32, 0, s>>>( \
            indptr, indices, data, n_rows, nnz_base, w0, w, v, k, lg, out);                  \
        return;                                                                              \
    }
    MFM_FM_CASE(1)
    MFM_FM_CASE(2)
    MFM_FM_CASE(4)
    MFM_FM_CASE(8)
    MFM_FM_CASE(16)
    MFM_FM_CASE(32)
#undef MFM_FM_CASE
    fail(MFM_ERR_UNSUPPORTED, fmt("k=%d exceeds the FM kernel's register tiling", k));
}

// Row-group shapes (see fm_rows_kernel): returns false when k needs the
// generic kernel. Gathers hoisted per iteration stay at <= 48 registers.
template <class T, class IdxT, class ValT, class OutT>
bool fm_rows_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                    const ValT* data, int64_t n_rows, int64_t nnz_base, T w0, const T* w,
                    const T* v, int k, OutT* out) {
    constexpr int V = 16 / (int)sizeof(T);  // 4 floats or 2 doubles per 16-byte load
    if (k % V != 0) return false;
    const int nvec = k / V;
    const unsigned grid = (unsigned)sm_count(device) * 8;
#define MFM_ROWS(L_, LR_, CAP_, MB_)                                                       \
    {                                                                                      \
        const int64_t slots = (int64_t)grid * 256 / LR_;                                   \
        const unsigned g = (unsigned)std::max<int64_t>(                                    \
            1, std::min<int64_t>(grid, ceil_div(std::min(n_rows, slots) * LR_, 256)));     \
        fm_rows_kernel<T, IdxT, ValT, OutT, V, L_, LR_, CAP_, MB_><<<g, 256, 0, s>>>(       \
            indptr, indices, data, n_rows, nnz_base, w0, w, v, k, out);                    \
        return true;                                                                       \
    }
    if (nvec <= 2) MFM_ROWS(2, 16, 48, 4)
    if (nvec <= 4) MFM_ROWS(4, 16, 48, 4)
    if (nvec <= 8) MFM_ROWS(8, 32, 32, 4)
#undef MFM_ROWS
    return false;
}

template <class T, class IdxT, class ValT, class OutT>
void fm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
               const ValT* data, int64_t n_rows, int64_t nnz_base, double w0, const T* w,
               const T* v, int k, OutT* out) {
    if (n_rows <= 0) return;
    if (fm_rows_launch<T, IdxT, ValT, OutT>(device, s, indptr, indices, data, n_rows, nnz_base,
                                            (T)w0, w, v, k, out)) {
        MFM_CHECK_LAUNCH("FM predict launch");
        return;
    }
    const unsigned grid = warp_grid(device, n_rows, kWarpsPerBlock, kBlocksPerSm);
    switch (vec_width<T>(k)) {
    case 4:
        fm_launch_vec<T, IdxT, ValT, OutT, (16 / sizeof(T) >= 4 ? 4 : 1)>(
            grid, s, indptr, indices, data, n_rows, nnz_base, (T)w0, w, v, k, out);
        break;
    case 2:
        fm_launch_vec<T, IdxT, ValT, OutT, 2>(grid, s, indptr, indices, data, n_rows, nnz_base,
                                              (T)w0, w, v, k, out);
        break;
    default:
        fm_launch_vec<T, IdxT, ValT, OutT, 1>(grid, s, indptr, indices, data, n_rows, nnz_base,
                                              (T)w0, w, v, k, out);
    }
    MFM_CHECK_LAUNCH("FM predict launch");
}

template <class T, class IdxT, class ValT, class OutT>
void ffm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                const ValT* data, int64_t n_rows, int64_t nnz_base, const int32_t* fid, int F,
                double w0, const T* w, const T* v, int k, OutT* out) {
    if (n_rows <= 0) return;
    const unsigned grid = warp_grid(device, n_rows, kWarpsPerBlock, kBlocksPerSm);
    const int vw = vec_width<T>(k);
    if (vw == 4)
        ffm_predict_kernel<T, IdxT, ValT, OutT, (16 / sizeof(T) >= 4 ? 4 : 1)>
            <<<grid, kWarpsPerBlock * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, fid,
                                                  F, (T)w0, w, v, k, out);
    else if (vw == 2)
        ffm_predict_kernel<T, IdxT, ValT, OutT, 2><<<grid, kWarpsPerBlock * 32, 0, s>>>(
            indptr, indices, data, n_rows, nnz_base, fid, F, (T)w0, w, v, k, out);
    else
        ffm_predict_kernel<T, IdxT, ValT, OutT, 1><<<grid, kWarpsPerBlock * 32, 0, s>>>(
            indptr, indices, data, n_rows, nnz_base, fid, F, (T)w0, w, v, k, out);
    MFM_CHECK_LAUNCH("FFM predict launch");
}

template <class T, class IdxT, class ValT, class OutT>
void fwfm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                 const ValT* data, int64_t n_rows, int64_t nnz_base, const int32_t* fid, int F,
                 double w0, const T* w, const T* v, const T* r, int k, OutT* out) {
    if (n_rows <= 0) return;
    const unsigned grid = warp_grid(device, n_rows, kWarpsPerBlock, kBlocksPerSm);
    const int vw = vec_width<T>(k);
    if (vw == 4)
        fwfm_predict_kernel<T, IdxT, ValT, OutT, (16 / sizeof(T) >= 4 ? 4 : 1)>
            <<<grid, kWarpsPerBlock * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, fid,
                                                  F, (T)w0, w, v, r, k, out);
    else if (vw == 2)
        fwfm_predict_kernel<T, IdxT, ValT, OutT, 2><<<grid, kWarpsPerBlock * 32, 0, s>>>(
            indptr, indices, data, n_rows, nnz_base, fid, F, (T)w0, w, v, r, k, out);
    else
        fwfm_predict_kernel<T, IdxT, ValT, OutT, 1><<<grid, kWarpsPerBlock * 32, 0, s>>>(
            indptr, indices, data, n_rows, nnz_base, fid, F, (T)w0, w, v, r, k, out);
    MFM_CHECK_LAUNCH("FwFM predict launch");
}

// ------------------------------------------------- host-buffer predict --

__global__ void f64_to_f32_kernel(const double* __restrict__ src, float* __restrict__ dst,
                                  int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = (float)src[i];
}

// Parameters of one model, uploaded to one device in the compute dtype.
template <class T>
struct DevParams {
    DevBuf<T> w, v, r;
    DevBuf<int32_t> fid;
};

template <class T>
void upload_param(int device, cudaStream_t s, DevBuf<T>& dst, const double* src, size_t n,
                  const char* what) {
    dst.alloc(device, n);
    if (!n) return;
    if constexpr (sizeof(T) == sizeof(double)) {
        h2d(reinterpret_cast<double*>(dst.ptr), src, n, s, what);
    } else {
        DevBuf<double> tmp(device, n);
        h2d(tmp.ptr, src, n, s, what);
        unsigned grid = (unsigned)std::min<int64_t>(ceil_div((int64_t)n, 256),
                                                    (int64_t)sm_count(device) * 8);
        f64_to_f32_kernel<<<grid, 256, 0, s>>>(tmp.ptr, dst.ptr, (int64_t)n);
        MFM_CHECK_LAUNCH("parameter conversion");
        MFM_CUDA(cudaStreamSynchronize(s), "parameter conversion");
    }
}

enum class Model { FM, FFM, FWFM };

struct PredictArgs {
    Model model;
    const mfm_csr* x;
    const int64_t* field_ids;
    int64_t F;
    double w0;
    const double *w, *v, *r;
    int64_t k;
    double* out;
};

template <class T>
void predict_shard(const PredictArgs& A, int device, int64_t r0, int64_t r1) {
    DeviceGuard guard(device);
    std::lock_guard<std::mutex> lk(device_mutex(device));
    cudaStream_t s = device_stream(device);
    const mfm_csr* x = A.x;
    const int64_t nnz0 = x->indptr[r0], nnz1 = x->indptr[r1];
    const int64_t rows = r1 - r0, nnz = nnz1 - nnz0;
    DevBuf<int64_t> d_indptr(device, rows + 1), d_indices(device, nnz);
    DevBuf<double> d_data(device, nnz), d_out(device, rows);
    h2d(d_indptr.ptr, x->indptr + r0, rows + 1, s, "indptr upload");
    h2d(d_indices.ptr, x->indices + nnz0, nnz, s, "indices upload");
    h2d(d_data.ptr, x->data + nnz0, nnz, s, "data upload");
    // CsrView::new's O(nnz) checks (rust/src/data.rs:33-38), on the device
    validate_csr_device(device, s, d_indptr.ptr, rows, d_indices.ptr, nnz, x->n_features);
    DevParams<T> P;
    upload_param(device, s, P.w, A.w, x->n_features, "w upload");
    const int64_t vlen = A.model == Model::FFM ? x->n_features * A.F * A.k : x->n_features * A.k;
    upload_param(device, s, P.v, A.v, vlen, "V upload");
    if (A.model != Model::FM) {
        std::vector<int32_t> f32(x->n_features);
        for (int64_t i = 0; i < x->n_features; ++i) f32[i] = (int32_t)A.field_ids[i];
        P.fid.alloc(device, x->n_features);
        h2d(P.fid.ptr, f32.data(), f32.size(), s, "field_ids upload");
        MFM_CUDA(cudaStreamSynchronize(s), "field_ids upload");
    }
    if (A.model == Model::FWFM) upload_param(device, s, P.r, A.r, A.F * A.F, "R upload");
    if (A.model == Model::FM)
        fm_launch<T, int64_t, double, double>(device, s, d_indptr.ptr, d_indices.ptr, d_data.ptr,
                                              rows, nnz0, A.w0, P.w.ptr, P.v.ptr, (int)A.k,
                                              d_out.ptr);
    else if (A.model == Model::FFM)
        ffm_launch<T, int64_t, double, double>(device, s, d_indptr.ptr, d_indices.ptr,
                                               d_data.ptr, rows, nnz0, P.fid.ptr, (int)A.F,
                                               A.w0, P.w.ptr, P.v.ptr, (int)A.k, d_out.ptr);
    else
        fwfm_launch<T, int64_t, double, double>(device, s, d_indptr.ptr, d_indices.ptr,
                                                d_data.ptr, rows, nnz0, P.fid.ptr, (int)A.F,
                                                A.w0, P.w.ptr, P.v.ptr, P.r.ptr, (int)A.k,
                                                d_out.ptr);
    d2h(A.out + r0, d_out.ptr, rows, s, "output download");
    MFM_CUDA(cudaStreamSynchronize(s), "predict");
}

// Splits rows into n_devices contiguous shards of about equal nnz (rows are
// independent, so prediction needs no communication) and runs one host
// thread per device.
void predict_sharded(const PredictArgs& A, const mfm_exec* ex) {
    const int dtype = ex ? ex->dtype : MFM_DTYPE_F64;
    const int dev0 = ex ? ex->device : 0;
    int nd = ex && ex->n_devices > 0 ? ex->n_devices : 1;
    if (dtype != MFM_DTYPE_F64 && dtype != MFM_DTYPE_F32)
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
    const int avail = device_count();
    if (avail <= 0) fail(MFM_ERR_NO_DEVICE, "no CUDA device available");
    if (dev0 < 0 || dev0 + nd > avail)
        fail(MFM_ERR_INVALID, fmt("devices [%d, %d) out of range [0, %d)", dev0, dev0 + nd, avail));
    const mfm_csr* x = A.x;
    if (nd > x->n_rows) nd = (int)std::max<int64_t>(1, x->n_rows);
    std::vector<int64_t> cut(nd + 1, 0);
    cut[nd] = x->n_rows;
    for (int d = 1; d < nd; ++d) {
        const int64_t target = x->nnz / nd * d;
        cut[d] = std::lower_bound(x->indptr, x->indptr + x->n_rows + 1, target) - x->indptr;
        cut[d] = std::max(cut[d], cut[d - 1]);
    }
    auto run = [&](int d) {
        if (cut[d + 1] <= cut[d]) return;
        if (dtype == MFM_DTYPE_F64)
            predict_shard<double>(A, dev0 + d, cut[d], cut[d + 1]);
        else
            predict_shard<float>(A, dev0 + d, cut[d], cut[d + 1]);
    };
    if (nd == 1) {
        run(0);
        return;
    }
    std::vector<std::exception_ptr> errs(nd);
    std::vector<std::thread> th;
    for (int d = 0; d < nd; ++d)
        th.emplace_back([&, d] {
            try {
                run(d);
            } catch (...) {
                errs[d] = std::current_exception();
            }
        });
    for (auto& t : th) t.join();
    for (auto& e : errs)
        if (e) std::rethrow_exception(e);
}

void check_k(int64_t k, const char* model) {
    if (k < 1 || k > 1024)
        fail(MFM_ERR_UNSUPPORTED,
             fmt("CUDA %s prediction supports 1 <= k <= 1024, got %lld", model, (long long)k));
}

}  // namespace mfm

using namespace mfm;

extern "C" int mfm_fm_predict_csr(const mfm_csr* x, double w0, const double* w, const double* v,
                                  int64_t k, double* out, const mfm_exec* ex) {
    return guarded([&] {
        check_csr_host(x);
        if (x->n_rows == 0) return;
        check_k(k, "FM");
        PredictArgs A{Model::FM, x, nullptr, 0, w0, w, v, nullptr, k, out};
        predict_sharded(A, ex);
    });
}

extern "C" int mfm_ffm_predict_csr(const mfm_csr* x, const int64_t* field_ids, int64_t n_fields,
                                   double w0, const double* w, const double* v, int64_t k,
                                   double* out, const mfm_exec* ex) {
    return guarded([&] {
        check_field_ids(field_ids, x ? x->n_features : 0, n_fields);
        check_csr_host(x);
        if (x->n_rows == 0) return;
        check_k(k, "FFM");
        PredictArgs A{Model::FFM, x, field_ids, n_fields, w0, w, v, nullptr, k, out};
        predict_sharded(A, ex);
    });
}

extern "C" int mfm_fwfm_predict_csr(const mfm_csr* x, const int64_t* field_ids,
                                    int64_t n_fields, double w0, const double* w,
                                    const double* v, const double* r, int64_t k, double* out,
                                    const mfm_exec* ex) {
    return guarded([&] {
        check_field_ids(field_ids, x ? x->n_features : 0, n_fields);
        check_csr_host(x);
        if (x->n_rows == 0) return;
        check_k(k, "FwFM");
        PredictArgs A{Model::FWFM, x, field_ids, n_fields, w0, w, v, r, k, out};
        predict_sharded(A, ex);
    });
}

// ------------------------------------------------ device-resident predict --

extern "C" int mfm_fm_predict_device(int dtype, int device, const int64_t* indptr,
                                     const int32_t* indices, const void* data, int64_t n_rows,
                                     double w0, const void* w, const void* v, int64_t k,
                                     void* out, void* stream) {
    return guarded([&] {
        check_k(k, "FM");
        DeviceGuard g(device);
        cudaStream_t s = (cudaStream_t)stream;
        if (dtype == MFM_DTYPE_F32)
            fm_launch<float, int32_t, float, float>(device, s, indptr, indices, (const float*)data,
                                                    n_rows, 0, w0, (const float*)w,
                                                    (const float*)v, (int)k, (float*)out);
        else if (dtype == MFM_DTYPE_F64)
            fm_launch<double, int32_t, double, double>(
                device, s, indptr, indices, (const double*)data, n_rows, 0, w0,
                (const double*)w, (const double*)v, (int)k, (double*)out);
        else
            fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
    });
}

extern "C" int mfm_ffm_predict_device(int dtype, int device, const int64_t* indptr,
                                      const int32_t* indices, const void* data, int64_t n_rows,
                                      const int32_t* field_ids, int64_t n_fields, double w0,
                                      const void* w, const void* v, int64_t k, void* out,
                                      void* stream) {
    return guarded([&] {
        check_k(k, "FFM");
        DeviceGuard g(device);
        cudaStream_t s = (cudaStream_t)stream;
        if (dtype == MFM_DTYPE_F32)
            ffm_launch<float, int32_t, float, float>(device, s, indptr, indices,
                                                     (const float*)data, n_rows, 0, field_ids,
                                                     (int)n_fields, w0, (const float*)w,
                                                     (const float*)v, (int)k, (float*)out);
        else if (dtype == MFM_DTYPE_F64)
            ffm_launch<double, int32_t, double, double>(
                device, s, indptr, indices, (const double*)data, n_rows, 0, field_ids,
                (int)n_fields, w0, (const double*)w, (const double*)v, (int)k, (double*)out);
        else
            fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
    });
}

extern "C" int mfm_fwfm_predict_device(int dtype, int device, const int64_t* indptr,
                                       const int32_t* indices, const void* data, int64_t n_rows,
                                       const int32_t* field_ids, int64_t n_fields, double w0,
                                       const void* w, const void* v, const void* r, int64_t k,
                                       void* out, void* stream) {
    return guarded([&] {
        check_k(k, "FwFM");
        DeviceGuard g(device);
        cudaStream_t s = (cudaStream_t)stream;
        if (dtype == MFM_DTYPE_F32)
            fwfm_launch<float, int32_t, float, float>(
                device, s, indptr, indices, (const float*)data, n_rows, 0, field_ids,
                (int)n_fields, w0, (const float*)w, (const float*)v, (const float*)r, (int)k,
                (float*)out);
        else if (dtype == MFM_DTYPE_F64)
            fwfm_launch<double, int32_t, double, double>(
                device, s, indptr, indices, (const double*)data, n_rows, 0, field_ids,
                (int)n_fields, w0, (const double*)w, (const double*)v, (const double*)r, (int)k,
                (double*)out);
        else
            fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
    });
}

// ------------------------------------------- launchers for staged inputs --
// FM scoring over device copies in the boundary layout (int64 indices,
// float64 values), parameters in float64 or float32. Used by the
// allocation-free entry point (predict_noalloc.cu), which stages its inputs in
// its own static device buffer.
namespace mfm {
void fm_launch_staged_f64(int device, cudaStream_t s, const int64_t* indptr,
                          const int64_t* indices, const double* data, int64_t n_rows,
                          double w0, const double* w, const double* v, int k, double* out) {
    fm_launch<double, int64_t, double, double>(device, s, indptr, indices, data, n_rows, 0, w0,
                                               w, v, k, out);
}
void fm_launch_staged_f32(int device, cudaStream_t s, const int64_t* indptr,
                          const int64_t* indices, const double* data, int64_t n_rows,
                          double w0, const float* w, const float* v, int k, double* out) {
    fm_launch<float, int64_t, double, double>(device, s, indptr, indices, data, n_rows, 0, w0,
                                              w, v, k, out);
}
}  // namespace mfm
