// train_payload.cuh — reduction of per-entry gradient payloads in sorted
// order (stage 1: work items; stage 2: multi-item runs; w0) and the opt-in
// persistent epoch kernel of that path.
#pragma once

#include "train_forward.cuh"

namespace mfm {

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
    // data-parallel batch (dp != 0): only this rank's entries, those whose
    // batch-local entry id vals[p] lies in [olo, ohi), are summed; the run sums
    // go to grad (batch-local run index, stride Wp; row nrun: the w0 sum per
    // class over this rank's rows, grow[0, nrows)) instead of the optimizer,
    // which reduce_apply_kernel runs after the cross-rank sum
    int dp;
    const uint32_t* vals;       // batch-local entry id per batch-local sorted position
    uint32_t olo, ohi;
    const int64_t* item_run;    // epoch run of each item
    int64_t run0, nrun;         // this batch's runs: [run0, run0 + nrun)
    T* grad;
    unsigned* progress;         // mapped host word, set to pstep by the apply
    unsigned pstep;
};

template <class T, int VEC>
__device__ __forceinline__ void store_vec(T* dst, const T* v) {
    Vec<T, VEC> o;
#pragma unroll
    for (int c = 0; c < VEC; ++c) o.v[c] = v[c];
    *reinterpret_cast<Vec<T, VEC>*>(dst) = o;
}

// Steps the scalar columns [vv*VEC, vv*VEC + VEC) of key `key` (those below
// W) with column sums `sum`: every column's loads are issued before the first
// step, so the columns cost one memory round trip, not one each.
template <class T, int VEC>
__device__ __forceinline__ void apply_cols(const RedArgs<T>& R, uint32_t key, int vv,
                                           const T* sum) {
    CoordStep<T> cs[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
        const int col = vv * VEC + c;
        if (col >= R.W) continue;
        if (col < R.cb1)
            cs[c].load(R.g0, (int64_t)key * R.g0.width + col, R.opt.kind);
        else
            cs[c].load(R.g1, (int64_t)key * R.g1.width + (col - R.cb1), R.opt.kind);
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
        const int col = vv * VEC + c;
        if (col >= R.W) continue;
        if (col < R.cb1)
            cs[c].apply(R.g0, (int64_t)key * R.g0.width + col, sum[c] * R.inv_bsz, R.opt);
        else
            cs[c].apply(R.g1, (int64_t)key * R.g1.width + (col - R.cb1), sum[c] * R.inv_bsz,
                        R.opt);
    }
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
        const bool vec = !R.dp && !multi && vec_in_group0<T, VEC>(R, vv);
        const int64_t idx0 = (int64_t)d.key * R.g0.width + vv * VEC;
        VecStep<T, VEC> st;
        if (vec) st.prefetch(R.g0, idx0, R.opt.kind);  // overlaps the payload loads
        T acc[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) acc[c] = T(0);
        if (!R.dp) {
#pragma unroll 4
            for (int q = 0; q < cnt; ++q) {
                const Vec<T, VEC> x = ldg_vec<T, VEC>(rows + (int64_t)q * R.Wp + vv * VEC);
#pragma unroll
                for (int c = 0; c < VEC; ++c) acc[c] += x.v[c];
            }
        } else {  // this rank's entries only (other ranks' payload rows are stale)
            const uint32_t* ids = R.vals + (d.p0 - R.seg);
#pragma unroll 4
            for (int q = 0; q < cnt; ++q) {
                const uint32_t id = ids[q];
                if (id < R.olo || id >= R.ohi) continue;
                const Vec<T, VEC> x = ldg_vec<T, VEC>(rows + (int64_t)q * R.Wp + vv * VEC);
#pragma unroll
                for (int c = 0; c < VEC; ++c) acc[c] += x.v[c];
            }
        }
        if (R.dp && !multi) {  // the run's sum for this rank, stepped after the cross-rank sum
            store_vec<T, VEC>(R.grad + (R.item_run[R.item0 + it] - R.run0) * R.Wp + vv * VEC,
                              acc);
        } else if (multi) {
            Vec<T, VEC> o;
#pragma unroll
            for (int c = 0; c < VEC; ++c) o.v[c] = acc[c];
            *reinterpret_cast<Vec<T, VEC>*>(R.part + it * R.Wp + vv * VEC) = o;
        } else if (vec) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) acc[c] *= R.inv_bsz;
            st.commit(R.g0, idx0, acc, R.opt);
        } else {
            apply_cols<T, VEC>(R, d.key, vv, acc);
        }
    }
    }
}

template <class T, int VEC>
__global__ void __launch_bounds__(256, 4) reduce_items_kernel(RedArgs<T> R, int64_t n_items) {
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
    if (!R.dp) {
        w0_step_dev(R.grow, R.nrows, R.C, R.inv_bsz, R.gw0, R.opt, sm);
        return;
    }
    for (int c = 0; c < R.C; ++c) {  // this rank's sums, stepped after the cross-rank sum
        const T tot = block_sum_rows(R.grow, R.nrows, R.C, c, sm);
        if (threadIdx.x == 0) R.grad[R.nrun * R.Wp + c] = tot;
    }
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
                if (R.dp) {  // stepped after the cross-rank sum
                    store_vec<T, VEC>(R.grad + (r - R.run0) * R.Wp + vv * VEC, tot);
                } else if (vec_in_group0<T, VEC>(R, vv)) {
                    const int64_t idx0 = (int64_t)key * R.g0.width + vv * VEC;
                    VecStep<T, VEC> st;
                    st.prefetch(R.g0, idx0, R.opt.kind);
#pragma unroll
                    for (int c = 0; c < VEC; ++c) tot[c] *= R.inv_bsz;
                    st.commit(R.g0, idx0, tot, R.opt);
                } else {
                    apply_cols<T, VEC>(R, key, vv, tot);
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

// Data-parallel step (after the cross-rank sum of grad): lane groups of nvs
// lanes, one run per group, the run's column sums stepped as stage 1 steps a
// single-item run; w0 by thread 0 of block 0 when do_w0, which also records
// the step in the progress word.
template <class T, int VEC>
__global__ void __launch_bounds__(256, 4) reduce_apply_kernel(RedArgs<T> R) {
    const int lane = threadIdx.x & 31, grp = lane / R.nvs, vl = lane % R.nvs;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (R.do_w0)
            for (int c = 0; c < R.C; ++c)
                opt_step(R.gw0, c, R.grad[R.nrun * R.Wp + c] * R.inv_bsz, R.opt);
        if (R.progress) *(volatile unsigned*)R.progress = R.pstep;
    }
    if (grp >= R.gpw) return;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t wi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;; wi += nwarps) {
        const int64_t j = wi * R.gpw + grp;
        if (j >= R.nrun) return;
        const uint32_t key = R.desc[R.item_start[R.run0 + j]].key;
        const T* g = R.grad + j * R.Wp;
        for (int vv = vl; vv < R.nv; vv += R.nvs) {
            T acc[VEC];
            const Vec<T, VEC> x = ldg_vec<T, VEC>(g + vv * VEC);
#pragma unroll
            for (int c = 0; c < VEC; ++c) acc[c] = x.v[c];
            if (vec_in_group0<T, VEC>(R, vv)) {
                const int64_t idx0 = (int64_t)key * R.g0.width + vv * VEC;
                VecStep<T, VEC> st;
                st.prefetch(R.g0, idx0, R.opt.kind);
#pragma unroll
                for (int c = 0; c < VEC; ++c) acc[c] *= R.inv_bsz;
                st.commit(R.g0, idx0, acc, R.opt);
            } else {
                apply_cols<T, VEC>(R, key, vv, acc);
            }
        }
    }
}

// --------------------------------------------------- persistent epoch loop --
//
// FM training runs a whole epoch's batch loop in one cooperative launch (all
// blocks co-resident): forward -> barrier -> stage 1 (+ w0 by block 0) ->
// [barrier -> stage 2, when the batch has multi-item runs] -> barrier. The
// grid barrier's wait is bounded: after `limit` polls a block records an error
// flag; a block that sees the flag (while waiting, or after any barrier)
// returns at once, so after the first timeout the whole launch ends within one
// more wait and the host reports MFM_ERR_DEVICE_CHECK, with no further batch
// applied.

struct GridBar {
    unsigned int count, gen, err, pad;
};
constexpr unsigned long long kBarrierSpinLimit = 1ull << 24;  // polls of ~100 ns

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Returns false when the barrier failed (a wait gave up, here or in another
// block): the caller returns. `drop` makes this block leave without arriving
// (a block lost before the barrier, for the failure-handling test).
__device__ __forceinline__ bool grid_barrier(GridBar* bar, unsigned int& gen,
                                             unsigned long long limit, bool drop) {
    __shared__ unsigned int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int ok = 0;
        if (!drop) {
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
                    if (ld_acquire_gpu(&bar->err)) break;  // another block gave up
                    if (++polls > limit) {
                        atomicOr(&bar->err, 1u);
                        break;
                    }
                    __nanosleep(100);
                }
            }
            __threadfence();  // acquire the other blocks' writes
            ok = ld_acquire_gpu(&bar->err) == 0u;
        }
        s_ok = ok;
    }
    ++gen;
    __syncthreads();
    return s_ok != 0u;
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
    unsigned long long spin_limit;  // polls before a barrier wait gives up
    int drop_block;                 // block that leaves at its first barrier (-1: none)
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
    const bool drop = (int)blockIdx.x == E.drop_block;
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
        if (!grid_barrier(E.bar, gen, E.spin_limit, drop)) return;
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
            if (!grid_barrier(E.bar, gen, E.spin_limit, drop)) return;
            reduce_runs_dev<T, VEC>(R, l0, nl, blockIdx.x, gridDim.x, wsum);
        }
        if (!grid_barrier(E.bar, gen, E.spin_limit, drop)) return;
    }
}

}  // namespace mfm
