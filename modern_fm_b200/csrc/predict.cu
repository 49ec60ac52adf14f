// predict.cu — sm_100a CSR scoring kernels for FM, FFM and FwFM (binary and
// multiclass), the host entry points that replace the reference's
// cuda::{fm,ffm,fwfm}::predict_csr, and the persistent model handle.
//
// Design (memory-bound sparse gather; no tensor-core work exists here):
//  * every kernel is generic over the arithmetic type T and the parameter
//    storage type P: (T, P) = (float, float), (double, double), or
//    (double, float) — float32 parameters read with 16-byte vector loads and
//    widened to float64 before any arithmetic, which is what the reference
//    computes for an estimator whose attributes are float32
//    (python/modern_fm/fm.py:655-658 stores them, _backend.py:36-41 widens them
//    to float64 before its float64 kernels, rust/src/fm.rs:16-40);
//  * FM: a row group of LR lanes per row, L lanes per nonzero, CAP nonzeros per
//    iteration whose latent-row gathers are all issued before any is consumed;
//    the sum-of-squares identity in registers: O(nnz k) per row;
//  * FFM / FwFM: one warp per row; the row's (index, value, field) slice is
//    staged once in shared memory (FwFM also stages the row's latent rows, each
//    reused by z-1 pairs); the upper-triangle pair list (a < b, the reference's
//    pair order) is walked 32 pairs at a time: O(z^2 k) per row;
//  * multiclass (C > 1): parameters are key-major — w (n, C), V (n, C, k)
//    (FFM: (n, F, C, k)), R (F*F, C) — so the C class slices of one key are
//    adjacent; the kernels take one pass per class over the row, each class
//    slice of each touched key read once. Scores are (n_rows, C).
#include <algorithm>
#include <atomic>
#include <cstring>
#include <exception>
#include <thread>

#include "common.cuh"

namespace mfm {

constexpr unsigned kFull = 0xffffffffu;

// Parameters of one model on the device, in the storage type P.
template <class P>
struct ScoreParams {
    const P* w;            // (n) or (n, C)
    const P* v;            // FM / FwFM (n, C, k); FFM (n, F, C, k)
    const P* r;            // FwFM (F, F) or (F*F, C)
    const int32_t* fid;    // FFM / FwFM field of each feature
    const double* w0c;     // multiclass intercepts (C), device
    double w0;             // binary intercept
    int k, F, C;
};

template <class T, bool MC, class P>
__device__ __forceinline__ T intercept(const ScoreParams<P>& M, int c) {
    if constexpr (MC)
        return (T)M.w0c[c];
    else
        return (T)M.w0;
}

// ------------------------------------------------------------------ FM ----

// Generic FM kernel (any k): one warp per row, a nonzero's latent row spread
// over L = 2^lg lanes with VEC-wide loads, JMAX vectors per lane.
template <class T, class P, class IdxT, class ValT, class OutT, int VEC, int JMAX, bool MC>
__global__ void __launch_bounds__(256)
    fm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                      const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                      ScoreParams<P> M, int lg, OutT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int L = 1 << lg;
    const int G = 32 >> lg;
    const int grp = lane >> lg;
    const int l = lane & (L - 1);
    const int k = M.k, nvec = k / VEC;
    const int C = MC ? M.C : 1;
    const int64_t ks = (int64_t)C * k;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base, e = indptr[row + 1] - nnz_base;
        for (int c = 0; c < C; ++c) {
            const P* vc = M.v + (int64_t)c * k;
            const P* wc = M.w + c;
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
                        const P* vi = vc + (int64_t)i * ks;
                        if (l == 0) lin += (T)wc[(int64_t)i * C] * x;
#pragma unroll
                        for (int j = 0; j < JMAX; ++j) {
                            const int vv = l + j * L;
                            if (vv < nvec) {
                                const Vec<P, VEC> q = ldg_vec<P, VEC>(vi + vv * VEC);
#pragma unroll
                                for (int u = 0; u < VEC; ++u) {
                                    const T vx = (T)q.v[u] * x;
                                    acc[j][u] += vx;
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
                    for (int u = 0; u < VEC; ++u)
                        acc[j][u] += __shfl_xor_sync(kFull, acc[j][u], o);
            T pair = T(0);
            if (grp == 0) {
#pragma unroll
                for (int j = 0; j < JMAX; ++j)
                    if (l + j * L < nvec)
#pragma unroll
                        for (int u = 0; u < VEC; ++u) pair += acc[j][u] * acc[j][u];
            }
            // s = w0 + sum w_i x_i + 0.5 (sum_f (sum_i v_if x_i)^2 - sum_if (v_if x_i)^2)
            const T total = warp_sum(lin + T(0.5) * (pair - sq));
            if (lane == 0) out[row * C + c] = (OutT)(intercept<T, MC>(M, c) + total);
        }
    }
}

// Row-group FM kernel for latent rows of up to 8 vectors: LR lanes score one
// row (32/LR rows per warp); a nonzero's latent row is spread over L lanes
// (VEC elements each, 16-byte loads), G = LR/L nonzeros per step. One
// iteration covers CAP nonzeros: their indices and values are loaded by the
// row's lanes at once, w is gathered lane-parallel, and all CAP/G latent-row
// gathers are issued before any of them is consumed, so a 39-nonzero row makes
// three dependent memory round trips (indptr, index slice, gathers). A value
// reaches the lanes that use it by shuffle only after the gathers are issued,
// so the in-flight gathers are the only per-step registers.
template <class T, class P, class IdxT, class ValT, class OutT, int VEC, int L, int LR, int CAP,
          int MINB, bool MC>
__global__ void __launch_bounds__(256, MINB)
    fm_rows_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                   const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                   ScoreParams<P> M, OutT* __restrict__ out) {
    constexpr int G = LR / L;     // nonzeros per step
    constexpr int NC = CAP / LR;  // index chunks per iteration
    constexpr int S = CAP / G;    // hoisted gather steps per iteration
    static_assert(LR % L == 0 && CAP % LR == 0 && 32 % LR == 0, "row-group shape");
    const int lane = threadIdx.x & 31, rl = lane & (LR - 1), grp = rl / L, l = rl % L;
    const int k = M.k;
    const bool act = l < k / VEC;
    const int C = MC ? M.C : 1;
    const int64_t ks = (int64_t)C * k;
    const int64_t nslots = ((int64_t)gridDim.x * blockDim.x) / LR;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LR;; row += nslots) {
        const bool live = row < n_rows;
        if (!__any_sync(kFull, live)) break;
        const int64_t b = live ? indptr[row] - nnz_base : 0;
        const int64_t e = live ? indptr[row + 1] - nnz_base : 0;
        for (int c = 0; c < C; ++c) {
            const P* vc = M.v + (int64_t)c * k + l * VEC;
            const P* wc = M.w + c;
            T acc[VEC];
#pragma unroll
            for (int u = 0; u < VEC; ++u) acc[u] = T(0);
            T sq = T(0), lin = T(0);
            for (int64_t base = b;; base += CAP) {
                const bool more = base < e;
                if (!__any_sync(kFull, more)) break;
                int nh[NC];
                IdxT ii[NC];
                ValT xx[NC];
#pragma unroll
                for (int cc = 0; cc < NC; ++cc) {
                    const int64_t rem = e - base - LR * cc;
                    nh[cc] = !more || rem <= 0 ? 0 : (rem >= LR ? LR : (int)rem);
                    ii[cc] = 0;
                    xx[cc] = ValT(0);
                    if (rl < nh[cc]) {
                        ii[cc] = indices[base + LR * cc + rl];
                        xx[cc] = data[base + LR * cc + rl];
                    }
                }
                P wv[NC];
#pragma unroll
                for (int cc = 0; cc < NC; ++cc)
                    wv[cc] = rl < nh[cc] ? wc[(int64_t)ii[cc] * C] : P(0);
                Vec<P, VEC> q[S];
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int cc = s / L, src = (s % L) * G + grp;
                    const IdxT i = __shfl_sync(kFull, ii[cc], src, LR);
                    if (src < nh[cc] && act) {
                        q[s] = ldg_vec<P, VEC>(vc + (int64_t)i * ks);
                    } else {
#pragma unroll
                        for (int u = 0; u < VEC; ++u) q[s].v[u] = P(0);
                    }
                }
#pragma unroll
                for (int cc = 0; cc < NC; ++cc) lin += (T)wv[cc] * (T)xx[cc];
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int cc = s / L, src = (s % L) * G + grp;
                    // lanes past the chunk's end hold value 0 (and q is 0 there)
                    const T x = (T)__shfl_sync(kFull, xx[cc], src, LR);
#pragma unroll
                    for (int u = 0; u < VEC; ++u) {
                        const T vx = (T)q[s].v[u] * x;
                        acc[u] += vx;
                        sq += vx * vx;
                    }
                }
            }
#pragma unroll
            for (int o = L; o < LR; o <<= 1)
#pragma unroll
                for (int u = 0; u < VEC; ++u) acc[u] += __shfl_xor_sync(kFull, acc[u], o);
            T pair = T(0);
            if (grp == 0 && act) {
#pragma unroll
                for (int u = 0; u < VEC; ++u) pair += acc[u] * acc[u];
            }
            T t = lin + T(0.5) * (pair - sq);
#pragma unroll
            for (int o = LR / 2; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
            if (rl == 0 && live) out[row * C + c] = (OutT)(intercept<T, MC>(M, c) + t);
        }
    }
}

// The row's upper-triangle pair list (a < b, a ascending then b ascending, the
// reference's order, rust/src/ffm.rs:32-43) is walked 32 entries at a time:
// each lane advances its (a, b) cursor by 32 positions.
__device__ __forceinline__ void pair_advance(int& a, int& b, int z) {
    while (a < z - 1 && b >= z) {
        b = b - z + a + 2;
        ++a;
    }
}

template <class T, class P, int VEC>
__device__ __forceinline__ T dot_global(const P* __restrict__ pa, const P* __restrict__ pb,
                                        int k) {
    T dot = T(0);
#pragma unroll 4
    for (int t = 0; t < k; t += VEC) {
        const Vec<P, VEC> qa = ldg_vec<P, VEC>(pa + t), qb = ldg_vec<P, VEC>(pb + t);
#pragma unroll
        for (int u = 0; u < VEC; ++u) dot += (T)qa.v[u] * (T)qb.v[u];
    }
    return dot;
}

// Rows whose entries fit the per-warp staging area are staged in shared
// memory; longer rows read their slice from global memory (L1-cached).
constexpr int kWarps = 8;
constexpr int kStageFfm = 128;        // entries per warp (FFM)
constexpr int kStageFwfm = 64;        // entries per warp (FwFM)
constexpr int kStageLatent = 4096;    // bytes of latent rows per warp (FwFM)

// ----------------------------------------------------------------- FFM ----

// score = w0 + sum_a w_a x_a + sum_{a<b} <V[i_a, f(i_b)], V[i_b, f(i_a)]> x_a x_b
// (rust/src/ffm.rs:18-45). One warp per row; one pass per class.
template <class T, class P, class IdxT, class ValT, class OutT, int VEC, bool MC>
__global__ void __launch_bounds__(256)
    ffm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                       const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                       ScoreParams<P> M, OutT* __restrict__ out) {
    __shared__ IdxT s_i[kWarps][kStageFfm];
    __shared__ int32_t s_f[kWarps][kStageFfm];
    __shared__ T s_x[kWarps][kStageFfm];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    IdxT* si = s_i[wib];
    int32_t* sf = s_f[wib];
    T* sx = s_x[wib];
    const int k = M.k, F = M.F;
    const int C = MC ? M.C : 1;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base;
        const int64_t z64 = indptr[row + 1] - nnz_base - b;
        const IdxT* ix = indices + b;
        const ValT* dv = data + b;
        const bool staged = z64 <= kStageFfm;
        if (staged) {
            for (int q = lane; q < (int)z64; q += 32) {
                const IdxT i = ix[q];
                si[q] = i;
                sx[q] = (T)dv[q];
                sf[q] = M.fid[i];
            }
            __syncwarp();
        }
        for (int c = 0; c < C; ++c) {
            T acc = T(0);
            if (staged) {
                const int z = (int)z64;
                for (int q = lane; q < z; q += 32) acc += (T)M.w[(int64_t)si[q] * C + c] * sx[q];
                int a = 0, bb = 1 + lane;
                pair_advance(a, bb, z);
                while (a < z - 1) {
                    const IdxT ia = si[a], ib = si[bb];
                    const int fa = sf[a], fb = sf[bb];
                    const P* pa = M.v + (((int64_t)ia * F + fb) * C + c) * k;  // V[i_a, f_b]
                    const P* pb = M.v + (((int64_t)ib * F + fa) * C + c) * k;  // V[i_b, f_a]
                    const T dot = dot_global<T, P, VEC>(pa, pb, k);
                    acc += dot * sx[a] * sx[bb];
                    bb += 32;
                    pair_advance(a, bb, z);
                }
            } else {
                for (int64_t q = lane; q < z64; q += 32)
                    acc += (T)M.w[(int64_t)ix[q] * C + c] * (T)dv[q];
                // rows longer than the staging area: int64 pair cursors
                int64_t a = 0, bb = 1 + lane;
                while (a < z64 - 1 && bb >= z64) {
                    bb = bb - z64 + a + 2;
                    ++a;
                }
                while (a < z64 - 1) {
                    const IdxT ia = ix[a], ib = ix[bb];
                    const int fa = M.fid[ia], fb = M.fid[ib];
                    const P* pa = M.v + (((int64_t)ia * F + fb) * C + c) * k;
                    const P* pb = M.v + (((int64_t)ib * F + fa) * C + c) * k;
                    const T dot = dot_global<T, P, VEC>(pa, pb, k);
                    acc += dot * (T)dv[a] * (T)dv[bb];
                    bb += 32;
                    while (a < z64 - 1 && bb >= z64) {
                        bb = bb - z64 + a + 2;
                        ++a;
                    }
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) out[row * C + c] = (OutT)(intercept<T, MC>(M, c) + acc);
        }
        __syncwarp();  // the staging area is rewritten by the next row
    }
}

// ---------------------------------------------------------------- FwFM ----

// One lane's share of a FwFM row read straight from global memory (L1-cached):
// the lane's entries of sum w_a x_a and its pairs (a, b), a < b, taken 32
// apart in row-major pair order with int64 cursors. The caller sums the warp.
template <class T, class P, class IdxT, class ValT, int VEC, bool MC>
__device__ __forceinline__ T fwfm_row_global(const IdxT* __restrict__ ix,
                                             const ValT* __restrict__ dv, int64_t z64,
                                             const ScoreParams<P>& M, int c, int lane) {
    const int k = M.k, F = M.F;
    const int C = MC ? M.C : 1;
    T acc = T(0);
    for (int64_t q = lane; q < z64; q += 32) acc += (T)M.w[(int64_t)ix[q] * C + c] * (T)dv[q];
    int64_t a = 0, bb = 1 + lane;
    while (a < z64 - 1 && bb >= z64) {
        bb = bb - z64 + a + 2;
        ++a;
    }
    while (a < z64 - 1) {
        const IdxT ia = ix[a], ib = ix[bb];
        const int fa = M.fid[ia], fb = M.fid[ib];
        const int slot = fa <= fb ? fa * F + fb : fb * F + fa;  // fwfm.rs:17-21
        const T rw = (T)M.r[(int64_t)slot * C + c];
        const T dot = dot_global<T, P, VEC>(M.v + ((int64_t)ia * C + c) * k,
                                            M.v + ((int64_t)ib * C + c) * k, k);
        acc += rw * dot * (T)dv[a] * (T)dv[bb];
        bb += 32;
        while (a < z64 - 1 && bb >= z64) {
            bb = bb - z64 + a + 2;
            ++a;
        }
    }
    return acc;
}

// score = w0 + sum_a w_a x_a + sum_{a<b} r[min f, max f] <v_a, v_b> x_a x_b
// (rust/src/fwfm.rs:24-53). One warp per row; the row's latent rows (class c
// slices) are staged in shared memory when they fit, so each is read from
// global memory once instead of once per pair.
template <class T, class P, class IdxT, class ValT, class OutT, int VEC, bool MC>
__global__ void __launch_bounds__(256)
    fwfm_predict_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                        const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                        ScoreParams<P> M, OutT* __restrict__ out) {
    constexpr int kLat = kStageLatent / (int)sizeof(P);
    __shared__ IdxT s_i[kWarps][kStageFwfm];
    __shared__ int32_t s_f[kWarps][kStageFwfm];
    __shared__ T s_x[kWarps][kStageFwfm];
    __shared__ __align__(16) P s_v[kWarps][kLat];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    IdxT* si = s_i[wib];
    int32_t* sf = s_f[wib];
    T* sx = s_x[wib];
    P* sv = s_v[wib];
    const int k = M.k, F = M.F, nv = k / VEC;
    const int C = MC ? M.C : 1;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
         row += nwarps) {
        const int64_t b = indptr[row] - nnz_base;
        const int64_t z64 = indptr[row + 1] - nnz_base - b;
        const IdxT* ix = indices + b;
        const ValT* dv = data + b;
        const bool staged = z64 <= kStageFwfm && z64 * k <= kLat;
        if (staged) {
            for (int q = lane; q < (int)z64; q += 32) {
                const IdxT i = ix[q];
                si[q] = i;
                sx[q] = (T)dv[q];
                sf[q] = M.fid[i];
            }
            __syncwarp();
        }
        for (int c = 0; c < C; ++c) {
            T acc = T(0);
            if (staged) {
                const int z = (int)z64;
                // the class-c latent slice of every entry, one VEC vector per lane step
                for (int t = lane; t < z * nv; t += 32) {
                    const int a = t / nv, u = t - a * nv;
                    *reinterpret_cast<Vec<P, VEC>*>(sv + a * k + u * VEC) =
                        ldg_vec<P, VEC>(M.v + ((int64_t)si[a] * C + c) * k + u * VEC);
                }
                for (int q = lane; q < z; q += 32) acc += (T)M.w[(int64_t)si[q] * C + c] * sx[q];
                __syncwarp();
                int a = 0, bb = 1 + lane;
                pair_advance(a, bb, z);
                while (a < z - 1) {
                    const int fa = sf[a], fb = sf[bb];
                    const int slot = fa <= fb ? fa * F + fb : fb * F + fa;  // fwfm.rs:17-21
                    const T rw = (T)M.r[(int64_t)slot * C + c];
                    const P* pa = sv + a * k;
                    const P* pb = sv + bb * k;
                    T dot = T(0);
                    for (int t = 0; t < k; t += VEC) {
                        const Vec<P, VEC> qa = *reinterpret_cast<const Vec<P, VEC>*>(pa + t);
                        const Vec<P, VEC> qb = *reinterpret_cast<const Vec<P, VEC>*>(pb + t);
#pragma unroll
                        for (int u = 0; u < VEC; ++u) dot += (T)qa.v[u] * (T)qb.v[u];
                    }
                    acc += rw * dot * sx[a] * sx[bb];
                    bb += 32;
                    pair_advance(a, bb, z);
                }
                __syncwarp();  // sv is rewritten by the next class
            } else {
                acc = fwfm_row_global<T, P, IdxT, ValT, VEC, MC>(ix, dv, z64, M, c, lane);
            }
            acc = warp_sum(acc);
            if (lane == 0) out[row * C + c] = (OutT)(intercept<T, MC>(M, c) + acc);
        }
        __syncwarp();
    }
}

// Rows of at most kGroupCap entries: one group of L lanes per row (L a power
// of two >= k), lane d owning latent dimension d. Each lane widens the row's
// a_q = x_q v_q[d] once into registers and sums r[f_a, f_b] a_a a_b over the
// row's pairs: one multiply-add per pair and lane, with r read from the
// block's symmetric copy already in the arithmetic type. Rows longer than
// kGroupCap are scored afterwards by the whole warp from global memory.
constexpr int kGroupCap = 16;
constexpr int kRTab = 2048;  // F * F * C entries of r held in shared memory

template <class T, class P, class IdxT, class ValT, class OutT, int L, int VEC, bool MC>
__global__ void __launch_bounds__(256, 4)  // 4 blocks per SM: 1.7x the 2-block speed
    fwfm_group_kernel(const int64_t* __restrict__ indptr, const IdxT* __restrict__ indices,
                      const ValT* __restrict__ data, int64_t n_rows, int64_t nnz_base,
                      ScoreParams<P> M, OutT* __restrict__ out) {
    constexpr int G = 32 / L;  // rows per warp pass
    const unsigned FULL = 0xffffffffu;
    __shared__ T s_r[kRTab];   // [c][fa][fb] = r[min, max] of class c
    const int F = M.F, k = M.k, C = MC ? M.C : 1, FF = F * F;
    for (int t = threadIdx.x; t < FF * C; t += blockDim.x) {
        const int c = t / FF, q = t - c * FF, fa = q / F, fb = q - fa * F;
        const int slot = fa <= fb ? fa * F + fb : fb * F + fa;  // fwfm.rs:17-21
        s_r[t] = (T)M.r[(int64_t)slot * C + c];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, d = lane & (L - 1), g = lane / L;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    for (int64_t base = warp0 * G; base < n_rows; base += nwarps * G) {
        const int64_t row = base + g;
        const bool live = row < n_rows;
        int64_t b = 0, z = 0;
        if (live) {
            b = indptr[row] - nnz_base;
            z = indptr[row + 1] - nnz_base - b;
        }
        const bool grp = live && z <= kGroupCap;
        for (int c = 0; c < C; ++c) {
            T acc = T(0);
            if (grp) {
                const IdxT* ix = indices + b;
                const ValT* dv = data + b;
                T a[kGroupCap];
                int f[kGroupCap];
#pragma unroll
                for (int q = 0; q < kGroupCap; ++q) {
                    a[q] = T(0);
                    f[q] = 0;
                    if (q < z) {
                        const IdxT i = ix[q];
                        const T x = (T)dv[q];
                        f[q] = M.fid[i];
                        if (d < k) a[q] = x * (T)M.v[((int64_t)i * C + c) * k + d];
                        if ((q & (L - 1)) == d) acc += (T)M.w[(int64_t)i * C + c] * x;
                    }
                }
                const T* rc = s_r + c * FF;
#pragma unroll
                for (int j = 1; j < kGroupCap; ++j) {
                    if (j < z) {
                        const T* rj = rc + f[j] * F;
                        T t = T(0);
#pragma unroll
                        for (int i = 0; i < j; ++i) t += rj[f[i]] * a[i];
                        acc += t * a[j];
                    }
                }
            }
#pragma unroll
            for (int o = L / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
            if (grp && d == 0) out[row * C + c] = (OutT)(intercept<T, MC>(M, c) + acc);
        }
        // the pass's long rows, one at a time by the whole warp
        unsigned longm = __ballot_sync(FULL, live && !grp && d == 0);
        while (longm) {
            const int64_t lrow = base + (__ffs(longm) - 1) / L;
            longm &= longm - 1;
            const int64_t lb = indptr[lrow] - nnz_base;
            const int64_t lz = indptr[lrow + 1] - nnz_base - lb;
            for (int c = 0; c < C; ++c) {
                T acc = fwfm_row_global<T, P, IdxT, ValT, VEC, MC>(indices + lb, data + lb, lz, M,
                                                                   c, lane);
                acc = warp_sum(acc);
                if (lane == 0) out[lrow * C + c] = (OutT)(intercept<T, MC>(M, c) + acc);
            }
        }
    }
}

// ------------------------------------------------------------- launchers --

// Widest vector (elements of P, at most 16 bytes) that divides k and whose
// loads stay aligned given the base pointers.
template <class P>
int vec_width(int64_t k, const void* a, const void* b = nullptr) {
    constexpr int maxv = 16 / (int)sizeof(P);
    auto fits = [&](int vw) {
        const uintptr_t al = (uintptr_t)vw * sizeof(P);
        return k % vw == 0 && (uintptr_t)a % al == 0 && (!b || (uintptr_t)b % al == 0);
    };
    if (fits(maxv)) return maxv;
    if (maxv >= 2 && fits(2)) return 2;
    return 1;
}

constexpr int kBlocksPerSm = 8;

template <class T, class P, class IdxT, class ValT, class OutT, int VEC, bool MC>
void fm_launch_vec(unsigned grid, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                   const ValT* data, int64_t n_rows, int64_t nnz_base, const ScoreParams<P>& M,
                   OutT* out) {
    const int nvec = M.k / VEC;
    int L = 1, lg = 0;
    while (L < nvec && L < 32) {
        L <<= 1;
        ++lg;
    }
    const int J = (nvec + L - 1) / L;
#define MFM_FM_CASE(JM)                                                                  \
    if (J <= JM) {                                                                       \
        fm_predict_kernel<T, P, IdxT, ValT, OutT, VEC, JM, MC>                           \
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, lg, out); \
        return;                                                                          \
    }
    MFM_FM_CASE(1)
    MFM_FM_CASE(2)
    MFM_FM_CASE(4)
    MFM_FM_CASE(8)
    MFM_FM_CASE(16)
    MFM_FM_CASE(32)
#undef MFM_FM_CASE
    fail(MFM_ERR_UNSUPPORTED, fmt("k=%d exceeds the FM kernel's register tiling", M.k));
}

// Row-group shapes (see fm_rows_kernel): returns false when k needs the
// generic kernel. (L, LR, CAP, blocks per SM) per number of 16-byte vectors in
// a latent row; float64 arithmetic on float32 parameters holds fewer gathers
// per iteration (its accumulators take twice the registers), and the
// multiclass variants (one more loop level live) run one block fewer per SM.
template <class T, class P, class IdxT, class ValT, class OutT, bool MC>
bool fm_rows_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                    const ValT* data, int64_t n_rows, int64_t nnz_base, const ScoreParams<P>& M,
                    OutT* out) {
    constexpr int V = 16 / (int)sizeof(P);  // 4 floats or 2 doubles per 16-byte load
    if (vec_width<P>(M.k, M.v) != V) return false;
    const int nvec = M.k / V;
    const unsigned grid = (unsigned)sm_count(device) * 8;
    constexpr bool wide = sizeof(T) > sizeof(P);
#define MFM_ROWS(L_, LR_, CAP_, MB_)                                                          \
    {                                                                                         \
        const int64_t slots = (int64_t)grid * 256 / LR_;                                      \
        const unsigned g = (unsigned)std::max<int64_t>(                                       \
            1, std::min<int64_t>(grid, ceil_div(std::min(n_rows, slots) * LR_, 256)));        \
        fm_rows_kernel<T, P, IdxT, ValT, OutT, V, L_, LR_, CAP_, (MC ? MB_ - 1 : MB_), MC>     \
            <<<g, 256, 0, s>>>(                                                               \
            indptr, indices, data, n_rows, nnz_base, M, out);                                 \
        return true;                                                                          \
    }
    if constexpr (wide) {
        if (nvec <= 2) MFM_ROWS(2, 16, 32, 4)
        if (nvec <= 4) MFM_ROWS(4, 16, 32, 4)
        if (nvec <= 8) MFM_ROWS(8, 32, 32, 3)
    } else {
        if (nvec <= 2) MFM_ROWS(2, 16, 48, 4)
        if (nvec <= 4) MFM_ROWS(4, 16, 48, 4)
        if (nvec <= 8) MFM_ROWS(8, 32, 32, 4)
    }
#undef MFM_ROWS
    return false;
}

template <class T, class P, class IdxT, class ValT, class OutT, bool MC>
void fm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
               const ValT* data, int64_t n_rows, int64_t nnz_base, const ScoreParams<P>& M,
               OutT* out) {
    if (n_rows <= 0) return;
    if (fm_rows_launch<T, P, IdxT, ValT, OutT, MC>(device, s, indptr, indices, data, n_rows,
                                                   nnz_base, M, out)) {
        MFM_CHECK_LAUNCH("FM predict launch");
        return;
    }
    const unsigned grid = warp_grid(device, n_rows, kWarps, kBlocksPerSm);
    switch (vec_width<P>(M.k, M.v)) {
    case 4:
        fm_launch_vec<T, P, IdxT, ValT, OutT, (16 / sizeof(P) >= 4 ? 4 : 1), MC>(
            grid, s, indptr, indices, data, n_rows, nnz_base, M, out);
        break;
    case 2:
        fm_launch_vec<T, P, IdxT, ValT, OutT, 2, MC>(grid, s, indptr, indices, data, n_rows,
                                                     nnz_base, M, out);
        break;
    default:
        fm_launch_vec<T, P, IdxT, ValT, OutT, 1, MC>(grid, s, indptr, indices, data, n_rows,
                                                     nnz_base, M, out);
    }
    MFM_CHECK_LAUNCH("FM predict launch");
}

template <class T, class P, class IdxT, class ValT, class OutT, bool MC>
void ffm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                const ValT* data, int64_t n_rows, int64_t nnz_base, const ScoreParams<P>& M,
                OutT* out) {
    if (n_rows <= 0) return;
    const unsigned grid = warp_grid(device, n_rows, kWarps, kBlocksPerSm);
    const int vw = vec_width<P>(M.k, M.v);
    if (vw == 4)
        ffm_predict_kernel<T, P, IdxT, ValT, OutT, (16 / sizeof(P) >= 4 ? 4 : 1), MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    else if (vw == 2)
        ffm_predict_kernel<T, P, IdxT, ValT, OutT, 2, MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    else
        ffm_predict_kernel<T, P, IdxT, ValT, OutT, 1, MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    MFM_CHECK_LAUNCH("FFM predict launch");
}

template <class T, class P, class IdxT, class ValT, class OutT, bool MC>
void fwfm_launch(int device, cudaStream_t s, const int64_t* indptr, const IdxT* indices,
                 const ValT* data, int64_t n_rows, int64_t nnz_base, const ScoreParams<P>& M,
                 OutT* out) {
    if (n_rows <= 0) return;
    const int vw = vec_width<P>(M.k, M.v);
    const int64_t rtab = (int64_t)M.F * M.F * (MC ? M.C : 1);
    if (M.k <= 32 && rtab <= kRTab) {
        const int L = M.k <= 4 ? 4 : M.k <= 8 ? 8 : M.k <= 16 ? 16 : 32;
        const unsigned grid = warp_grid(device, ceil_div(n_rows, (int64_t)(32 / L)), kWarps,
                                        kBlocksPerSm);
#define MFM_FWFM_GROUP(LL, VV)                                                                  \
    fwfm_group_kernel<T, P, IdxT, ValT, OutT, LL, VV, MC>                                      \
        <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out)
#define MFM_FWFM_L(LL)                                                                          \
    if (L == LL) {                                                                              \
        if (vw == 4)                                                                            \
            MFM_FWFM_GROUP(LL, (16 / sizeof(P) >= 4 ? 4 : 1));                                  \
        else if (vw == 2)                                                                       \
            MFM_FWFM_GROUP(LL, 2);                                                              \
        else                                                                                    \
            MFM_FWFM_GROUP(LL, 1);                                                              \
    }
        MFM_FWFM_L(4)
        MFM_FWFM_L(8)
        MFM_FWFM_L(16)
        MFM_FWFM_L(32)
#undef MFM_FWFM_L
#undef MFM_FWFM_GROUP
        MFM_CHECK_LAUNCH("FwFM predict launch");
        return;
    }
    const unsigned grid = warp_grid(device, n_rows, kWarps, kBlocksPerSm);
    if (vw == 4)
        fwfm_predict_kernel<T, P, IdxT, ValT, OutT, (16 / sizeof(P) >= 4 ? 4 : 1), MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    else if (vw == 2)
        fwfm_predict_kernel<T, P, IdxT, ValT, OutT, 2, MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    else
        fwfm_predict_kernel<T, P, IdxT, ValT, OutT, 1, MC>
            <<<grid, kWarps * 32, 0, s>>>(indptr, indices, data, n_rows, nnz_base, M, out);
    MFM_CHECK_LAUNCH("FwFM predict launch");
}

enum class Model { FM, FFM, FWFM };

// One scoring launch of `model` over a device CSR.
template <class T, class P, class IdxT, class ValT, class OutT>
void score_launch(Model model, bool mc, int device, cudaStream_t s, const int64_t* indptr,
                  const IdxT* indices, const ValT* data, int64_t n_rows, int64_t nnz_base,
                  const ScoreParams<P>& M, OutT* out) {
#define MFM_SCORE(fn)                                                                        \
    {                                                                                        \
        if (mc)                                                                              \
            fn<T, P, IdxT, ValT, OutT, true>(device, s, indptr, indices, data, n_rows, nnz_base, \
                                             M, out);                                        \
        else                                                                                 \
            fn<T, P, IdxT, ValT, OutT, false>(device, s, indptr, indices, data, n_rows,         \
                                              nnz_base, M, out);                             \
        return;                                                                              \
    }
    if (model == Model::FM) MFM_SCORE(fm_launch)
    if (model == Model::FFM) MFM_SCORE(ffm_launch)
    MFM_SCORE(fwfm_launch)
#undef MFM_SCORE
}

// ------------------------------------------------------ parameter upload --

// Narrows float64 to float32; sets *inexact when a value (other than NaN)
// changes, i.e. when the float32 copy is not the caller's value.
__global__ void narrow_f32_kernel(const double* __restrict__ src, float* __restrict__ dst,
                                  int64_t n, unsigned int* __restrict__ inexact) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double x = src[i];
        const float f = (float)x;
        dst[i] = f;
        bad |= ((double)f != x) && (x == x);
    }
    if (__any_sync(kFull, bad) && (threadIdx.x & 31) == 0 && inexact) atomicOr(inexact, 1u);
}

__global__ void f64_to_f32_kernel(const double* __restrict__ src, float* __restrict__ dst,
                                  int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = (float)src[i];
}

// Class-major (C, R, K) float64 -> key-major (R, C, K) float64 (multiclass
// parameters of the reference's layout into the scoring kernels').
__global__ void class_to_key_kernel(const double* __restrict__ src, double* __restrict__ dst,
                                    int64_t C, int64_t R, int64_t K) {
    const int64_t total = C * R * K, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / (C * K), rem = i - r * C * K, c = rem / K, kk = rem - c * K;
        dst[i] = src[(c * R + r) * K + kk];
    }
}

inline unsigned flat_grid(int device, int64_t n) {
    return (unsigned)std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(n, 256), (int64_t)sm_count(device) * 8));
}

// One model's parameters on one device: float64 copies (key-major), and
// float32 copies when the storage type is float32. `exact` tells whether the
// float32 copies equal the float64 values (decided on the device).
struct DevModel {
    Model model = Model::FM;
    int device = 0, C = 1, F = 1;
    int64_t n_features = 0, k = 0;
    double w0 = 0.0;
    DevBuf<double> w0c, w64, v64, r64;
    DevBuf<float> w32, v32, r32;
    DevBuf<int32_t> fid;
    bool have32 = false, exact = false;

    int64_t v_len() const {
        return model == Model::FFM ? n_features * F * (int64_t)C * k : n_features * (int64_t)C * k;
    }

    // Uploads parameters given in the reference's boundary layout: binary
    // w (n), V (n, k) / (n, F, k), R (F, F); multiclass class-major w0 (C),
    // w (C, n), V (C, n, k) / (C, n, F, k), R (C, F, F).
    void upload(cudaStream_t s, const double* w0p, const double* w, const double* v,
                const double* r, const int64_t* field_ids, bool narrow) {
        const int64_t nf = n_features;
        auto put = [&](DevBuf<double>& dst, const double* src, int64_t R, int64_t K) {
            const int64_t n = (int64_t)C * R * K;
            dst.alloc(device, n);
            if (!n) return;
            if (C == 1) {
                h2d(dst.ptr, src, n, s, "parameter upload");
                return;
            }
            DevBuf<double> tmp(device, n);
            h2d(tmp.ptr, src, n, s, "parameter upload");
            class_to_key_kernel<<<flat_grid(device, n), 256, 0, s>>>(tmp.ptr, dst.ptr, C, R, K);
            MFM_CHECK_LAUNCH("parameter layout");
            MFM_CUDA(cudaStreamSynchronize(s), "parameter upload");
        };
        if (C > 1) {
            w0c.alloc(device, C);
            h2d(w0c.ptr, w0p, C, s, "w0 upload");
        } else {
            w0 = *w0p;
        }
        put(w64, w, nf, 1);
        if (model == Model::FFM)
            put(v64, v, nf * F, k);
        else
            put(v64, v, nf, k);
        if (model == Model::FWFM) put(r64, r, (int64_t)F * F, 1);
        if (model != Model::FM) {
            std::vector<int32_t> f32(nf);
            for (int64_t i = 0; i < nf; ++i) f32[i] = (int32_t)field_ids[i];
            fid.alloc(device, nf);
            h2d(fid.ptr, f32.data(), f32.size(), s, "field_ids upload");
        }
        have32 = exact = false;
        if (narrow) {
            DevBuf<unsigned int> flag(device, 1);
            MFM_CUDA(cudaMemsetAsync(flag.ptr, 0, sizeof(unsigned int), s), "flag clear");
            auto nar = [&](DevBuf<double>& src, DevBuf<float>& dst) {
                dst.alloc(device, src.n);
                if (src.n)
                    narrow_f32_kernel<<<flat_grid(device, src.n), 256, 0, s>>>(
                        src.ptr, dst.ptr, (int64_t)src.n, flag.ptr);
            };
            nar(w64, w32);
            nar(v64, v32);
            if (model == Model::FWFM) nar(r64, r32);
            MFM_CHECK_LAUNCH("parameter narrowing");
            unsigned int h = 0;
            d2h(&h, flag.ptr, 1, s, "narrowing check");
            MFM_CUDA(cudaStreamSynchronize(s), "parameter narrowing");
            have32 = true;
            exact = h == 0;
        } else {
            MFM_CUDA(cudaStreamSynchronize(s), "parameter upload");
        }
    }

    template <class P>
    ScoreParams<P> view() const {
        ScoreParams<P> M{};
        if constexpr (sizeof(P) == sizeof(double)) {
            M.w = w64.ptr;
            M.v = v64.ptr;
            M.r = r64.ptr;
        } else {
            M.w = w32.ptr;
            M.v = v32.ptr;
            M.r = r32.ptr;
        }
        M.fid = fid.ptr;
        M.w0c = w0c.ptr;
        M.w0 = w0;
        M.k = (int)k;
        M.F = F;
        M.C = C;
        return M;
    }
};

// The storage / arithmetic pair a dtype selects for a model whose float64
// parameters are resident: float64; float32 (both); float32 storage with
// float64 arithmetic when the float32 copies are exact, else float64.
enum class Mode { F64, F32, F32_F64 };

inline Mode mode_of(int dtype, const DevModel& m) {
    if (dtype == MFM_DTYPE_F32) return Mode::F32;
    if (dtype == MFM_DTYPE_F32_F64 && m.have32 && m.exact) return Mode::F32_F64;
    return Mode::F64;
}

// Scores a device CSR in the boundary format (int64 indices, float64 values)
// into float64 scores.
void score_boundary(const DevModel& m, int dtype, cudaStream_t s, const int64_t* indptr,
                    const int64_t* indices, const double* data, int64_t n_rows, double* out) {
    const bool mc = m.C > 1;
    switch (mode_of(dtype, m)) {
    case Mode::F32:
        score_launch<float, float, int64_t, double, double>(m.model, mc, m.device, s, indptr,
                                                            indices, data, n_rows, 0,
                                                            m.view<float>(), out);
        break;
    case Mode::F32_F64:
        score_launch<double, float, int64_t, double, double>(m.model, mc, m.device, s, indptr,
                                                             indices, data, n_rows, 0,
                                                             m.view<float>(), out);
        break;
    default:
        score_launch<double, double, int64_t, double, double>(m.model, mc, m.device, s, indptr,
                                                              indices, data, n_rows, 0,
                                                              m.view<double>(), out);
    }
}

void check_dtype(int dtype) {
    if (dtype != MFM_DTYPE_F64 && dtype != MFM_DTYPE_F32 && dtype != MFM_DTYPE_F32_F64)
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
}

// ------------------------------------------------- host-buffer predict --

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

void predict_shard(const PredictArgs& A, int dtype, int device, int64_t r0, int64_t r1) {
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
    DevModel m;
    m.model = A.model;
    m.device = device;
    m.F = A.model == Model::FM ? 1 : (int)A.F;
    m.n_features = x->n_features;
    m.k = A.k;
    m.upload(s, &A.w0, A.w, A.v, A.r, A.field_ids, dtype != MFM_DTYPE_F64);
    // the CSR's indptr keeps its absolute offsets: the kernels subtract nnz0
    const bool mc = false;
    switch (mode_of(dtype, m)) {
    case Mode::F32:
        score_launch<float, float, int64_t, double, double>(m.model, mc, device, s,
                                                            d_indptr.ptr, d_indices.ptr,
                                                            d_data.ptr, rows, nnz0,
                                                            m.view<float>(), d_out.ptr);
        break;
    case Mode::F32_F64:
        score_launch<double, float, int64_t, double, double>(m.model, mc, device, s,
                                                             d_indptr.ptr, d_indices.ptr,
                                                             d_data.ptr, rows, nnz0,
                                                             m.view<float>(), d_out.ptr);
        break;
    default:
        score_launch<double, double, int64_t, double, double>(m.model, mc, device, s,
                                                              d_indptr.ptr, d_indices.ptr,
                                                              d_data.ptr, rows, nnz0,
                                                              m.view<double>(), d_out.ptr);
    }
    d2h(A.out + r0, d_out.ptr, rows, s, "output download");
    MFM_CUDA(cudaStreamSynchronize(s), "predict");
}

// Contiguous row shards of about equal nnz, one per device.
std::vector<int64_t> shard_cuts(const mfm_csr* x, int nd) {
    std::vector<int64_t> cut(nd + 1, 0);
    cut[nd] = x->n_rows;
    for (int d = 1; d < nd; ++d) {
        const int64_t target = x->nnz / nd * d;
        cut[d] = std::lower_bound(x->indptr, x->indptr + x->n_rows + 1, target) - x->indptr;
        cut[d] = std::max(cut[d], cut[d - 1]);
    }
    return cut;
}

// Runs run(d) for d in [0, nd) on one host thread per device; rethrows the
// first failure.
template <class F>
void per_device(int nd, F&& run) {
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

// Splits rows into n_devices contiguous shards of about equal nnz (rows are
// independent, so prediction needs no communication) and runs one host
// thread per device.
void predict_sharded(const PredictArgs& A, const mfm_exec* ex) {
    const int dtype = ex ? ex->dtype : MFM_DTYPE_F64;
    const int dev0 = ex ? ex->device : 0;
    int nd = ex && ex->n_devices > 0 ? ex->n_devices : 1;
    check_dtype(dtype);
    const int avail = device_count();
    if (avail <= 0) fail(MFM_ERR_NO_DEVICE, "no CUDA device available");
    if (dev0 < 0 || dev0 + nd > avail)
        fail(MFM_ERR_INVALID, fmt("devices [%d, %d) out of range [0, %d)", dev0, dev0 + nd, avail));
    const mfm_csr* x = A.x;
    if (nd > x->n_rows) nd = (int)std::max<int64_t>(1, x->n_rows);
    const std::vector<int64_t> cut = shard_cuts(x, nd);
    per_device(nd, [&](int d) {
        if (cut[d + 1] > cut[d]) predict_shard(A, dtype, dev0 + d, cut[d], cut[d + 1]);
    });
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

namespace mfm {

// Device-resident scoring in the compute layout: indices int32; data, params
// and scores per dtype (float32: all float; float64: all double;
// float32-float64: params float, data and scores double).
void device_score(Model model, int dtype, int device, const int64_t* indptr,
                  const int32_t* indices, const void* data, int64_t n_rows,
                  const ScoreParams<float>& Mf, const ScoreParams<double>& Md, bool mc, void* out,
                  cudaStream_t s) {
    if (dtype == MFM_DTYPE_F32)
        score_launch<float, float, int32_t, float, float>(model, mc, device, s, indptr, indices,
                                                          (const float*)data, n_rows, 0, Mf,
                                                          (float*)out);
    else if (dtype == MFM_DTYPE_F64)
        score_launch<double, double, int32_t, double, double>(model, mc, device, s, indptr,
                                                              indices, (const double*)data,
                                                              n_rows, 0, Md, (double*)out);
    else if (dtype == MFM_DTYPE_F32_F64)
        score_launch<double, float, int32_t, double, double>(model, mc, device, s, indptr,
                                                             indices, (const double*)data,
                                                             n_rows, 0, Mf, (double*)out);
    else
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
}

template <class P>
ScoreParams<P> raw_params(double w0, const void* w, const void* v, const void* r,
                          const int32_t* fid, int64_t k, int64_t F) {
    ScoreParams<P> M{};
    M.w = (const P*)w;
    M.v = (const P*)v;
    M.r = (const P*)r;
    M.fid = fid;
    M.w0 = w0;
    M.k = (int)k;
    M.F = (int)F;
    M.C = 1;
    return M;
}

}  // namespace mfm

extern "C" int mfm_fm_predict_device(int dtype, int device, const int64_t* indptr,
                                     const int32_t* indices, const void* data, int64_t n_rows,
                                     double w0, const void* w, const void* v, int64_t k,
                                     void* out, void* stream) {
    return guarded([&] {
        check_k(k, "FM");
        DeviceGuard g(device);
        device_score(Model::FM, dtype, device, indptr, indices, data, n_rows,
                     raw_params<float>(w0, w, v, nullptr, nullptr, k, 1),
                     raw_params<double>(w0, w, v, nullptr, nullptr, k, 1), false, out,
                     (cudaStream_t)stream);
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
        device_score(Model::FFM, dtype, device, indptr, indices, data, n_rows,
                     raw_params<float>(w0, w, v, nullptr, field_ids, k, n_fields),
                     raw_params<double>(w0, w, v, nullptr, field_ids, k, n_fields), false, out,
                     (cudaStream_t)stream);
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
        device_score(Model::FWFM, dtype, device, indptr, indices, data, n_rows,
                     raw_params<float>(w0, w, v, r, field_ids, k, n_fields),
                     raw_params<double>(w0, w, v, r, field_ids, k, n_fields), false, out,
                     (cudaStream_t)stream);
    });
}

// ------------------------------------------------------------ model handle --
//
// A model resident on the device across calls. The reference uploads the
// parameters on every CUDA predict call (rust/src/cuda/mod.rs:9-12,
// rust/src/cuda/fm.rs:61-109) and scores a multiclass model with one binary
// call per class, each re-uploading X (python/modern_fm/fm.py:666-674); a
// handle uploads the parameters once and scores all classes in one call.

struct mfm_model {
    mfm::DevModel m;
    int dtype = MFM_DTYPE_F64;
    bool ready = false;
};

namespace mfm {
namespace {
Model model_kind(int kind) {
    if (kind == MFM_MODEL_FM) return Model::FM;
    if (kind == MFM_MODEL_FFM) return Model::FFM;
    if (kind == MFM_MODEL_FWFM) return Model::FWFM;
    fail(MFM_ERR_INVALID, fmt("unknown model kind %d", kind));
}
}  // namespace
}  // namespace mfm

extern "C" int mfm_model_create(int kind, int dtype, int device, int64_t n_features,
                                int64_t n_fields, int64_t k, int64_t n_classes,
                                mfm_model** out) {
    return guarded([&] {
        if (!out) fail(MFM_ERR_INVALID, "out must be provided");
        *out = nullptr;
        const Model model = model_kind(kind);
        check_dtype(dtype);
        check_k(k, model == Model::FM ? "FM" : model == Model::FFM ? "FFM" : "FwFM");
        if (n_features < 0 || n_features >= ((int64_t)1 << 31))
            fail(MFM_ERR_UNSUPPORTED, "n_features must be in [0, 2^31)");
        if (n_classes < 1 || n_classes > 1024) fail(MFM_ERR_INVALID, "n_classes must be in [1, 1024]");
        if (model != Model::FM && (n_fields < 1 || n_fields > 4096))
            fail(MFM_ERR_INVALID, "n_fields must be in [1, 4096]");
        const int avail = device_count();
        if (avail <= 0) fail(MFM_ERR_NO_DEVICE, "no CUDA device available");
        if (device < 0 || device >= avail)
            fail(MFM_ERR_INVALID, fmt("device %d out of range [0, %d)", device, avail));
        auto* h = new mfm_model();
        h->m.model = model;
        h->m.device = device;
        h->m.n_features = n_features;
        h->m.F = model == Model::FM ? 1 : (int)n_fields;
        h->m.k = k;
        h->m.C = (int)n_classes;
        h->dtype = dtype;
        *out = h;
    });
}

extern "C" int mfm_model_set_params(mfm_model* h, const double* w0, const double* w,
                                    const double* v, const double* r,
                                    const int64_t* field_ids) {
    return guarded([&] {
        if (!h) fail(MFM_ERR_INVALID, "null model handle");
        DevModel& m = h->m;
        if (!w0 || (m.n_features > 0 && (!w || !v)) || (m.model == Model::FWFM && !r))
            fail(MFM_ERR_INVALID, "parameter arrays must be provided");
        if (m.model != Model::FM) check_field_ids(field_ids, m.n_features, m.F);
        DeviceGuard guard(m.device);
        std::lock_guard<std::mutex> lk(device_mutex(m.device));
        h->ready = false;
        m.upload(device_stream(m.device), w0, w, v, r, field_ids, h->dtype != MFM_DTYPE_F64);
        h->ready = true;
    });
}

extern "C" int mfm_model_info(const mfm_model* h, int* dtype_used) {
    return guarded([&] {
        if (!h || !dtype_used) fail(MFM_ERR_INVALID, "null argument");
        if (!h->ready) fail(MFM_ERR_INVALID, "model parameters are not set");
        const Mode md = mode_of(h->dtype, h->m);
        *dtype_used = md == Mode::F32 ? MFM_DTYPE_F32
                      : md == Mode::F32_F64 ? MFM_DTYPE_F32_F64
                                            : MFM_DTYPE_F64;
    });
}

extern "C" int mfm_model_predict_csr(mfm_model* h, const mfm_csr* x, double* out) {
    return guarded([&] {
        if (!h) fail(MFM_ERR_INVALID, "null model handle");
        if (!h->ready) fail(MFM_ERR_INVALID, "model parameters are not set");
        check_csr_host(x);
        DevModel& m = h->m;
        if (x->n_features != m.n_features)
            fail(MFM_ERR_INVALID, fmt("X has %lld features, the model %lld",
                                      (long long)x->n_features, (long long)m.n_features));
        if (x->n_rows == 0) return;
        const int device = m.device;
        DeviceGuard guard(device);
        std::lock_guard<std::mutex> lk(device_mutex(device));
        cudaStream_t s = device_stream(device);
        const int64_t n = x->n_rows, nnz = x->nnz;
        DevBuf<int64_t> d_indptr(device, n + 1), d_indices(device, nnz);
        DevBuf<double> d_data(device, nnz), d_out(device, n * m.C);
        h2d(d_indptr.ptr, x->indptr, n + 1, s, "indptr upload");
        h2d(d_indices.ptr, x->indices, nnz, s, "indices upload");
        h2d(d_data.ptr, x->data, nnz, s, "data upload");
        validate_csr_device(device, s, d_indptr.ptr, n, d_indices.ptr, nnz, x->n_features);
        score_boundary(m, h->dtype, s, d_indptr.ptr, d_indices.ptr, d_data.ptr, n, d_out.ptr);
        d2h(out, d_out.ptr, n * m.C, s, "output download");
        MFM_CUDA(cudaStreamSynchronize(s), "predict");
    });
}

extern "C" int mfm_model_predict_device(mfm_model* h, const int64_t* indptr,
                                        const int32_t* indices, const void* data, int64_t n_rows,
                                        void* out, void* stream) {
    return guarded([&] {
        if (!h) fail(MFM_ERR_INVALID, "null model handle");
        if (!h->ready) fail(MFM_ERR_INVALID, "model parameters are not set");
        if (n_rows < 0) fail(MFM_ERR_INVALID, "negative CSR size");
        if (n_rows == 0) return;
        DevModel& m = h->m;
        DeviceGuard guard(m.device);
        cudaStream_t s = (cudaStream_t)stream;
        const bool mc = m.C > 1;
        // data and scores: float32 in float32 mode, float64 otherwise
        if (h->dtype == MFM_DTYPE_F32)
            score_launch<float, float, int32_t, float, float>(m.model, mc, m.device, s, indptr,
                                                              indices, (const float*)data,
                                                              n_rows, 0, m.view<float>(),
                                                              (float*)out);
        else if (mode_of(h->dtype, m) == Mode::F32_F64)
            score_launch<double, float, int32_t, double, double>(
                m.model, mc, m.device, s, indptr, indices, (const double*)data, n_rows, 0,
                m.view<float>(), (double*)out);
        else
            score_launch<double, double, int32_t, double, double>(
                m.model, mc, m.device, s, indptr, indices, (const double*)data, n_rows, 0,
                m.view<double>(), (double*)out);
    });
}

extern "C" void mfm_model_free(mfm_model* h) {
    if (!h) return;
    DeviceGuard guard(h->m.device);
    std::lock_guard<std::mutex> lk(device_mutex(h->m.device));
    delete h;
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
    fm_launch<double, double, int64_t, double, double, false>(
        device, s, indptr, indices, data, n_rows, 0,
        raw_params<double>(w0, w, v, nullptr, nullptr, k, 1), out);
}
void fm_launch_staged_f32(int device, cudaStream_t s, const int64_t* indptr,
                          const int64_t* indices, const double* data, int64_t n_rows,
                          double w0, const float* w, const float* v, int k, double* out) {
    fm_launch<float, float, int64_t, double, double, false>(
        device, s, indptr, indices, data, n_rows, 0,
        raw_params<float>(w0, w, v, nullptr, nullptr, k, 1), out);
}
}  // namespace mfm
