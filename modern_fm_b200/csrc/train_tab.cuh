// train_tab.cuh — binary FM row-table reduction: per-entry gradients
// recomputed from the row table in sorted order, segment sums, optimizer
// steps, crossing-run folds and the data-parallel apply.
#pragma once

#include "train_payload.cuh"

namespace mfm {

// ------------------------------------------ binary FM row-table reduction --
//
// Binary FM with k = NV * VEC (16-byte vectors, NV <= 8). The forward writes
// one table row per batch row, S (k) = sum_j V_j x_j the row's factor sum
// (rows of k elements: whole 32-byte sectors), and the row's
// g = dL/ds x sample weight into grow (4096 values, held in L1). The reduction reads the batch's
// sorted entry stream (key, row, x). Each entry's gradient is the one
// FmGradAccum::add_row forms (rust/src/fm.rs:136-146),
//   gv[t] = g (x S[t] - V[t] x x),   gw = g x,
// and V is the same row for every entry of a key's run, so the run's sum is
//   sum gv[t] = sum (g x S[t]) - V[t] sum (g x x):
// the reduction sums [g x S (k) | g x | g x x] from the table alone (no
// per-entry latent-row load, no per-entry payload written) and the step that
// owns the run subtracts V times the last column.
//
// Stage 1: one block per chunk of kChunk consecutive sorted entries, one
// entry per thread; a segmented shuffle reduction per warp, then the warps'
// pieces of a segment folded in warp order at the segment's owner (its first
// entry). The owners of the runs that end in the chunk hand their sums to
// shared memory and the whole block applies the optimizer to (run, vector)
// items. A segment continued from the previous chunk leaves its sum in
// ph[chunk]; the last segment, when it continues into the next chunk, leaves
// its sum in pt[chunk].
// Stage 2: one warp per chunk boundary that starts a crossing run folds
// pt[first chunk] + ph[...] in chunk order and applies; the last block steps
// w0. Every sum has a fixed shape, so results are bitwise reproducible.

constexpr int kChunk = 256;  // sorted entries per stage-1 block

template <class T>
struct TabArgs {
    const uint32_t* keys;  // sorted keys of the epoch's entry stream
    const uint32_t* rrow;  // batch-local row of each sorted entry
    const T* rx;           // value of each sorted entry
    const T* tab;          // (nrows, k) S per row
    T* ph;                 // (chunks, TW) sums continued from the previous chunk
    T* pt;                 // (chunks, TW) sums continued into the next chunk
    int TW;
    int64_t seg, n;        // this batch's entries: [seg, seg + n) of the sorted stream
    int64_t nrows;
    const T* grow;         // per-row g (the entries' g, and w0's)
    T inv_bsz;
    GroupDev<T> gv, gw, gw0;
    OptDev opt;
    // data-parallel batch (dp != 0): this rank scores rows [rlo, rhi) of the
    // batch; per-run sums [g x S | g x | g x x] go to grad (run - run0,
    // stride TW; row nrun = w0) instead of the optimizer, which
    // fm_tab_apply_kernel runs after the cross-rank sum
    int dp;
    uint32_t rlo, rhi;
    const int64_t* runs;   // per sorted entry: runs (distinct keys) before it in the epoch
    const uint32_t* rkey;  // key of each run of the epoch
    int64_t run0, nrun;    // this batch's runs: [run0, run0 + nrun)
    T* grad;
    L2Range pre[5];        // the next batch's epoch-order rows, for its forward
    unsigned* progress;    // data-parallel: mapped host word, set to pstep by the apply
    unsigned pstep;
};

// Blocks per SM the stage-1 kernel is held to: the per-entry column sums are
// its largest live state (the owners' steps hold one vector at a time)
template <class T, int NV, int OPT>
constexpr int tab_min_blocks() {
    return sizeof(T) == 4 ? (NV <= 4 ? 4 : 3) : (OPT == MFM_OPT_ADAM ? 2 : 3);
}

template <class T, int VEC, int NV, int OPT>
__global__ void __launch_bounds__(kChunk, (tab_min_blocks<T, NV, OPT>())) fm_tab_reduce_kernel(TabArgs<T> A) {
    constexpr int K = VEC * NV, NVAL = K + 2, NW = kChunk / 32;
    __shared__ __align__(16) T wpart[NW][NVAL];
    __shared__ int wflag[NW];  // bit 0: lane 0 continues the previous warp; bit 1: one segment
    __shared__ uint32_t s_last;
    __shared__ int s_out;
    __shared__ T s_sum[kChunk][NVAL];  // sums of the runs stepped in this block
    __shared__ uint32_t s_key[kChunk];
    __shared__ int s_wcnt[NW];
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
    if (mine) {  // [g x S | g x | g x x]
        const T* tr = A.tab + (int64_t)row * K;
        const T gx = __ldg(A.grow + row) * x;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const Vec<T, VEC> sv = ldg_vec<T, VEC>(tr + v * VEC);
#pragma unroll
            for (int u = 0; u < VEC; ++u) val[v * VEC + u] = gx * sv.v[u];
        }
        val[K] = gx;
        val[K + 1] = gx * x;
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
    // mode 1: written out (a run crossing the chunk's edge leaves its partial
    // in ph / pt; in data-parallel mode every run leaves the rank's sum in
    // grad); 3: stepped in this block
    int mode = 0;
    if (owner) {
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
        if (!dst && A.dp) dst = A.grad + (A.runs[gi] - A.run0) * A.TW;
        if (dst) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                Vec<T, VEC> o;
#pragma unroll
                for (int u = 0; u < VEC; ++u) o.v[u] = val[v * VEC + u];
                *reinterpret_cast<Vec<T, VEC>*>(dst + v * VEC) = o;
            }
            dst[K] = val[K];
            dst[K + 1] = val[K + 1];
            mode = 1;
        } else {
            mode = 3;
        }
    }
    // the runs stepped here hand their sums to the whole block: the owners
    // write them to shared memory in thread order, then every thread steps
    // (run, vector) items — 16-byte parameter and state accesses of one key
    // are taken by consecutive threads, and each thread holds one vector's
    // state at a time
    const unsigned m3 = __ballot_sync(FULL, mode == 3);
    if (lane == 0) s_wcnt[warp] = __popc(m3);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w2 = 0; w2 < NW; ++w2) {
        before += w2 < warp ? s_wcnt[w2] : 0;
        total += s_wcnt[w2];
    }
    if (mode == 3) {
        const int slot = before + __popc(m3 & ((1u << lane) - 1u));
#pragma unroll
        for (int q = 0; q < NVAL; ++q) s_sum[slot][q] = val[q];
        s_key[slot] = key;
    }
    __syncthreads();
    // w of run tid; V items (run, vector) four per thread at a time, all
    // loads of a group issued before the first step
    const bool hw = tid < total;
    VecStep<T, 1, OPT> sw1;
    if (hw) sw1.prefetch(A.gw, (int64_t)s_key[tid], A.opt.kind);
    const int nvi = total * NV;
    constexpr int G = OPT == MFM_OPT_ADAM ? 1 : OPT == MFM_OPT_FTRL ? 2 : 4;  // no spills
    for (int base = tid; base < nvi; base += G * kChunk) {
        VecStep<T, VEC, OPT> st[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int it = base + j * kChunk;
            if (it < nvi)
                st[j].prefetch(A.gv, (int64_t)s_key[it / NV] * K + (it % NV) * VEC, A.opt.kind);
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int it = base + j * kChunk;
            if (it < nvi) {  // sum gv = sum (g x S) - V sum (g x x)
                const int slot = it / NV, v = it % NV;
                const T* sv = s_sum[slot];
                T dg[VEC];
#pragma unroll
                for (int u = 0; u < VEC; ++u)
                    dg[u] = (sv[v * VEC + u] - st[j].p.v[u] * sv[K + 1]) * A.inv_bsz;
                st[j].commit(A.gv, (int64_t)s_key[slot] * K + v * VEC, dg, A.opt);
            }
        }
    }
    if (hw) {
        const T dgw = s_sum[tid][K] * A.inv_bsz;
        sw1.commit(A.gw, (int64_t)s_key[tid], &dgw, A.opt);
    }
}

template <class T, int VEC, int NV>
__global__ void __launch_bounds__(256) fm_tab_fold_kernel(TabArgs<T> A, int64_t nchunks) {
    constexpr int K = VEC * NV;
    const unsigned FULL = 0xffffffffu;
    pdl_trigger();
    if (threadIdx.x == 0)
        for (int r = 0; r < 5; ++r) prefetch_slice(A.pre[r], blockIdx.x, gridDim.x);
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
    T tot[K + 2];
#pragma unroll
    for (int q = 0; q < K + 2; ++q) tot[q] = T(0);
    for (int64_t e0 = 0; e0 < cnt; e0 += 32) {
        const int64_t e = e0 + lane;
        T part[K + 2];
        if (e < cnt) {
            const T* r = e == 0 ? A.pt + (c - 1) * A.TW : A.ph + (c + e - 1) * A.TW;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const Vec<T, VEC> x = ldg_vec<T, VEC>(r + v * VEC);
#pragma unroll
                for (int u = 0; u < VEC; ++u) part[v * VEC + u] = x.v[u];
            }
            part[K] = r[K];
            part[K + 1] = r[K + 1];
        } else {
#pragma unroll
            for (int q = 0; q < K + 2; ++q) part[q] = T(0);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int q = 0; q < K + 2; ++q) part[q] += __shfl_xor_sync(FULL, part[q], o);
#pragma unroll
        for (int q = 0; q < K + 2; ++q) tot[q] += part[q];
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
            gd[K + 1] = tot[K + 1];
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
            dg[u] = (t - st.p.v[u] * tot[K + 1]) * A.inv_bsz;
        }
        st.commit(A.gv, (int64_t)key * K + lane * VEC, dg, A.opt);
    } else if (lane == NV) {
        const T dg = tot[K] * A.inv_bsz;
        s1.commit(A.gw, (int64_t)key, &dg, A.opt);
    }
}

// Data-parallel step: after the cross-rank sum of grad, a group of NV + 1
// lanes per run of the batch (NV vector lanes + the w lane; 32 / (NV + 1) runs
// per warp) applies the optimizer to its key, identically on every rank;
// thread 0 of block 0 also steps w0.
template <int NV>
constexpr int tab_apply_runs_per_warp() {
    return 32 / (NV + 1);
}
template <class T, int VEC, int NV>
__global__ void __launch_bounds__(256) fm_tab_apply_kernel(TabArgs<T> A) {
    constexpr int K = VEC * NV, RPW = tab_apply_runs_per_warp<NV>();
    pdl_trigger();
    const int wl = threadIdx.x & 31;
    const int lane = wl % (NV + 1);  // lane within the run's group
    const bool spare = wl >= RPW * (NV + 1);  // lanes beyond the warp's last group
    const int64_t j =
        (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * RPW + (spare ? 0 : wl / (NV + 1));
    const uint32_t key = j < A.nrun ? A.rkey[A.run0 + j] : 0u;  // plan data
    pdl_wait();  // grad is the cross-rank sum
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        opt_step(A.gw0, 0, A.grad[A.nrun * A.TW] * A.inv_bsz, A.opt);
        if (A.progress) *(volatile unsigned*)A.progress = A.pstep;  // the sum has arrived
    }
    if (spare || j >= A.nrun) return;
    const T* gd = A.grad + j * A.TW;
    if (lane < NV) {
        const int64_t idx0 = (int64_t)key * K + lane * VEC;
        VecStep<T, VEC> st;
        st.prefetch(A.gv, idx0, A.opt.kind);
        const Vec<T, VEC> g = ldg_vec<T, VEC>(gd + lane * VEC);
        const T gxx = gd[K + 1];
        T dg[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) dg[u] = (g.v[u] - st.p.v[u] * gxx) * A.inv_bsz;
        st.commit(A.gv, idx0, dg, A.opt);
    } else if (lane == NV) {
        VecStep<T, 1> s1;
        s1.prefetch(A.gw, (int64_t)key, A.opt.kind);
        const T dg = gd[K] * A.inv_bsz;
        s1.commit(A.gw, (int64_t)key, &dg, A.opt);
    }
}

}  // namespace mfm
