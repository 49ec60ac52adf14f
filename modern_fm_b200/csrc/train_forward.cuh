// train_forward.cuh — training forward kernels: scores from the frozen
// batch-start parameters, the loss gradient, and per model either gradient
// payloads (FFM, FwFM, multiclass FM) or the row table (binary FM).
#pragma once

#include "train_plan.cuh"

namespace mfm {

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
    L2Range pre[3];  // row-table path: stage 1's sorted (key, row, x) of this batch
    T* tab;   // row table (nrows, TW = k): S per row (binary FM row-table path; g in grow)
    int TW;
    // parameter-sharded training with the exchange over peer memory (PART):
    // the group's buffers (device memory), this batch's exchange number (its
    // parity picks the buffer), the stage-1 row table to fill (stride k) and
    // the progress step
    const struct ShardXchDev* xch;
    unsigned long long seq;
    T* tab_out;
    unsigned step;
};

constexpr int kMaxDpRanks = 16;
// Every rank's exchange buffers as this rank addresses them: the partial row
// tables (two, alternating by the parity of the exchange number) and the
// per-block flag arrays, with this rank's own flags, failure words and
// liveness word.
struct ShardXchDev {
    const void* part[2][kMaxDpRanks];
    const unsigned long long* flags[kMaxDpRanks];
    unsigned long long* my_flags;
    unsigned* fail;    // this rank's failure word (device memory)
    unsigned* fail_h;  // the group's mapped host failure word
    unsigned* progress;
    unsigned long long spin;  // polls of about 0.2 us before a wait gives up
    int N, rank, PW;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

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

// Parameter-sharded training, exchange over peer memory: after this block
// has written its rows' partial sums [S_r | lin_r - sq_r / 2], it raises its
// flag to the batch's exchange number, waits until the same block of every
// other rank has done so (bounded: a wait that gives up sets the failure
// words, and later exchanges skip at once), sums its rows over the ranks in
// rank order (the other ranks' rows read over NVLink) and finishes them: S to
// the stage-1 row table, g = loss'(w0 + sum (lin - sq/2) + |S|^2 / 2) x sw to
// grow (optimizer.rs:38-43). Every block of the forward's grid is resident at
// once on every rank (the launch caps the grid), so no wait depends on a block
// that cannot run. A rank rewrites a table two batches later, after its whole
// previous forward saw every other rank's flags of that batch, by which time
// each has finished reading it.
template <class T, int VEC, int LR>
__device__ __forceinline__ void shard_block_exchange(const FwdArgs<T>& A, int64_t slot0,
                                                  int64_t nslots) {
    __shared__ int s_ok;
    __shared__ __align__(16) T s_row[(256 / 16) * (32 + 4)];  // slots x PW, PW <= k + VEC
    constexpr int SPB = 256 / LR;  // row slots per block
    const ShardXchDev& X = *A.xch;
    const int K = A.k, PW = X.PW, tid = threadIdx.x;
    __syncthreads();  // the block's rows are written
    if (tid == 0) {
        int ok = *(volatile unsigned*)X.fail == 0u;
        st_release_sys_u64(X.my_flags + blockIdx.x, A.seq);
        for (int p = 0; p < X.N && ok; ++p) {
            if (p == X.rank) continue;
            unsigned long long it = 0;
            while (ld_acquire_sys_u64(X.flags[p] + blockIdx.x) < A.seq) {
                if (++it > X.spin) {
                    ok = 0;
                    break;
                }
                __nanosleep(200);
            }
        }
        if (!ok) {
            *(volatile unsigned*)X.fail = 1u;
            *(volatile unsigned*)X.fail_h = 1u;
        } else if (blockIdx.x == 0 && X.progress) {
            *(volatile unsigned*)X.progress = A.step;
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const int par = (int)(A.seq & 1);
    // this block's row slots: SPB consecutive slots, then every nslots
    for (int64_t j0 = (slot0 / SPB) * SPB; j0 < A.nrows; j0 += nslots) {
        const int nr = (int)(A.nrows - j0 < SPB ? A.nrows - j0 : SPB);
        const int nvec = nr * PW / VEC;
        for (int f = tid; f < nvec; f += blockDim.x) {  // rows j0.. as 16-byte vectors
            Vec<T, VEC> acc;
            for (int p0 = 0; p0 < X.N; p0 += 4) {  // four ranks' loads in flight, then added
                Vec<T, VEC> v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (p0 + q < X.N) {
                        const T* src = static_cast<const T*>(X.part[par][p0 + q]) + j0 * PW +
                                       (int64_t)f * VEC;
                        if constexpr (sizeof(T) == 8) {
                            const double2 w = __ldcv(reinterpret_cast<const double2*>(src));
                            v[q].v[0] = w.x;
                            v[q].v[1] = w.y;
                        } else {
                            const float4 w = __ldcv(reinterpret_cast<const float4*>(src));
                            v[q].v[0] = w.x;
                            v[q].v[1] = w.y;
                            v[q].v[2] = w.z;
                            v[q].v[3] = w.w;
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (p0 + q < X.N)
#pragma unroll
                        for (int u = 0; u < VEC; ++u)
                            acc.v[u] = (p0 + q == 0) ? v[q].v[u] : acc.v[u] + v[q].v[u];
            }
            *reinterpret_cast<Vec<T, VEC>*>(s_row + f * VEC) = acc;
        }
        __syncthreads();
        if (tid < nr) {
            const int64_t j = j0 + tid;
            const T* pr = s_row + tid * PW;
            T ss = T(0);
            for (int c = 0; c < K; c += VEC) {
                Vec<T, VEC> sv;
#pragma unroll
                for (int u = 0; u < VEC; ++u) {
                    sv.v[u] = pr[c + u];
                    ss += sv.v[u] * sv.v[u];
                }
                *reinterpret_cast<Vec<T, VEC>*>(A.tab_out + j * K + c) = sv;
            }
            const int64_t pos = A.pos0 + j;
            const T sc = A.w0[0] + (pr[K] + T(0.5) * ss), y = A.y[pos];
            A.grow[j] = A.sw[pos] * (A.loss == MFM_LOSS_LOGISTIC ? sigmoid_t(sc) - y : sc - y);
        }
        __syncthreads();  // s_row is rewritten by the next slots
    }
}

// TAB: write the row table (S) and g instead of per-entry payloads.
// PART (with TAB; parameter-sharded training): the row's sums over this
// rank's keys only, [S | lin - sq / 2] at stride A.TW; no score, no g (both
// follow from the cross-rank sum of these rows).
template <class T, int VEC, int L, int LR, int CAP, bool TAB = false, bool PART = false>
__device__ __forceinline__ void fm_forward_rows_dev(const FwdArgs<T>& A, int64_t slot0,
                                                    int64_t nslots) {
    using Sh = RowsShape<T, VEC, L, LR, CAP>;
    const int lane = threadIdx.x & 31, rl = lane & (LR - 1), grp = rl / L, l = rl % L;
    const bool act = l < A.k / VEC;
    if (TAB) {
        pdl_trigger();
        if (threadIdx.x == 0)
            for (int r = 0; r < 3; ++r) prefetch_slice(A.pre[r], blockIdx.x, gridDim.x);
    }
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
        T t = PART ? lin - T(0.5) * sq : lin + T(0.5) * (pair - sq);
#pragma unroll
        for (int o = LR / 2; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        T g = T(0);
        if (TAB) pdl_wait();  // w0 and the writes below follow the predecessor
        if (live && !PART) {  // loss_grad x sample_weight, optimizer.rs:38-43
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
                if (PART && rl == 0) tr[A.k] = t;
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
    if (PART && A.xch) shard_block_exchange<T, VEC, LR>(A, slot0, nslots);
}

template <class T, int VEC, int L, int LR, int CAP, bool TAB = false, bool PART = false>
__global__ void __launch_bounds__(256, 2) fm_forward_rows_kernel(FwdArgs<T> A) {
    fm_forward_rows_dev<T, VEC, L, LR, CAP, TAB, PART>(
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
    // rows of up to kFfmStage nonzeros: index, value and field staged per warp
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
        for (int c = 0; c < C; ++c) {  // fwfm_score_row, rust/src/fwfm.rs:24-53
            T acc = T(0);
            for (int64_t q = lane; q < z; q += 32)
                acc += A.w[(int64_t)(staged ? s_ix[q] : ix[q]) * C + c] * (staged ? s_x[q] : dv[q]);
            int64_t a = 0, b = 1 + lane;
            pair_step(a, b, z);
            while (a < z - 1) {
                const int32_t ia = staged ? s_ix[a] : ix[a], ib = staged ? s_ix[b] : ix[b];
                const int fa = staged ? s_f[a] : A.fid[ia], fb = staged ? s_f[b] : A.fid[ib];
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
        if (staged) {  // lane per entry a: sum over partners b with k-wide vectors
            for (int a = lane; a < z; a += 32) {
                const T xa = s_x[a];
                const int fa = s_f[a];
                T* P = A.pay1 + (int64_t)A.inv1[A.seg1 + e1 + a] * W1;
                for (int c = 0; c < C; ++c) {
                    for (int t = 0; t < k; t += VEC) {
                        T sum[VEC];
#pragma unroll
                        for (int u = 0; u < VEC; ++u) sum[u] = T(0);
                        for (int b = 0; b < z; ++b) {
                            if (b == a) continue;
                            const int fb = s_f[b];
                            const T rw =
                                A.r[(int64_t)(fa <= fb ? fa * F + fb : fb * F + fa) * C + c];
                            const Vec<T, VEC> q =
                                ldg_vec<T, VEC>(A.v + ((int64_t)s_ix[b] * C + c) * k + t);
#pragma unroll
                            for (int u = 0; u < VEC; ++u) sum[u] += rw * s_x[b] * q.v[u];
                        }
                        Vec<T, VEC> o;
#pragma unroll
                        for (int u = 0; u < VEC; ++u) o.v[u] = gs[c] * xa * sum[u];
                        *reinterpret_cast<Vec<T, VEC>*>(P + c * k + t) = o;
                    }
                    P[CK + c] = gs[c] * xa;
                }
            }
        } else {
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
        }
        const int64_t e2 = A.estart2[pos] - A.seg2;
        int64_t a = 0, b = 1 + lane, pi = lane;
        pair_step(a, b, z);
        while (a < z - 1) {
            const int32_t ia = staged ? s_ix[a] : ix[a], ib = staged ? s_ix[b] : ix[b];
            const T xab = dv[a] * dv[b];
            for (int c = 0; c < C; ++c) {
                const T* pa = A.v + ((int64_t)ia * C + c) * k;
                const T* pb = A.v + ((int64_t)ib * C + c) * k;
                T dot = T(0);
                for (int t = 0; t < k; t += VEC) {
                    const Vec<T, VEC> qa = ldg_vec<T, VEC>(pa + t), qb = ldg_vec<T, VEC>(pb + t);
#pragma unroll
                    for (int u = 0; u < VEC; ++u) dot += qa.v[u] * qb.v[u];
                }
                A.pay2[(int64_t)A.inv2[A.seg2 + e2 + pi] * A.W2 + c] = gs[c] * xab * dot;
            }
            b += 32;
            pi += 32;
            pair_step(a, b, z);
        }
        __syncwarp();
    }
}

}  // namespace mfm
