// train_opt.cuh — training constants, parameter groups, the optimizer steps
// (rust/src/optimizer.rs) and the launch-order helpers (programmatic
// dependent launch) every training kernel uses.
#pragma once

#include "segsort.cuh"

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
    double lb1, lb2;  // log2(b1), log2(b2): Adam's b^t as exp2(t log2 b)
};

// Programmatic dependent launch (sm_90+): a kernel launched with the
// programmatic-serialization attribute may start while its predecessor in the
// stream drains. pdl_trigger lets the successor be scheduled once every block
// of this grid has started; pdl_wait blocks until the predecessor grid has
// completed and its writes are visible (immediately when launched normally).
// Every thread of a PDL kernel calls pdl_wait before its first write and
// before it exits, so this grid's completion implies its predecessor's.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// A contiguous byte range to pull into L2 ahead of the kernel that reads it.
struct L2Range {
    const void* p;
    int64_t bytes;
};
// Slice `part` of `nparts` of r, trimmed to 16-byte boundaries, requested with
// one bulk L2 prefetch (no registers, no wait; a hint the hardware may drop).
__device__ __forceinline__ void prefetch_slice(const L2Range& r, int64_t part, int64_t nparts) {
    if (!r.p || r.bytes <= 0) return;
    const int64_t per = (r.bytes + nparts - 1) / nparts;
    const uintptr_t base = (uintptr_t)r.p;
    uintptr_t lo = base + (uintptr_t)(per * part), hi = lo + (uintptr_t)per;
    const uintptr_t end = base + (uintptr_t)r.bytes;
    if (hi > end) hi = end;
    lo = (lo + 15) & ~(uintptr_t)15;
    hi &= ~(uintptr_t)15;
    if (hi <= lo) return;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)(hi - lo))
                 : "memory");
}

__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// gr / sqrt(a) for AdaGrad: float32 through the hardware reciprocal square
// root (rsqrtf, at most 2 ulp from the correctly rounded value, one
// instruction instead of a rounded square root and a rounded division);
// float64 correctly rounded.
__device__ __forceinline__ float adagrad_scale(float gr, float a) { return gr * rsqrtf(a); }
__device__ __forceinline__ double adagrad_scale(double gr, double a) { return gr / sqrt(a); }

// One step of the reference's step_param / step_coord (rust/src/optimizer.rs:
// 48-167) for coordinate idx of group g with batch-mean data gradient dg.
// Split in two so that a caller stepping several scalar coordinates issues
// every coordinate's parameter and state loads before the first step.
template <class T>
struct CoordStep {
    T p, a, b, c;  // param and up to three state values
    __device__ __forceinline__ void load(const GroupDev<T>& g, int64_t idx, int kind) {
        p = g.p[idx];
        if (kind == MFM_OPT_ADAGRAD) {
            a = g.acc[idx];
        } else if (kind == MFM_OPT_ADAM) {
            a = g.m[idx];
            b = g.s[idx];
            c = g.t[idx];
        } else if (kind == MFM_OPT_FTRL) {
            a = g.z[idx];
            b = g.n[idx];
        }
    }
    __device__ __forceinline__ void apply(const GroupDev<T>& g, int64_t idx, T dg,
                                          const OptDev& o) {
        T th = p;
        const T l1 = (T)o.l1[g.reg], l2 = (T)o.l2[g.reg], lr = (T)o.lr;
        switch (o.kind) {
        case MFM_OPT_SGD:  // apply_update, optimizer.rs:48-60
            th -= lr * (dg + l2 * th);
            break;
        case MFM_OPT_ADAGRAD: {
            const T gr = dg + l2 * th;
            const T ac = a + gr * gr;
            g.acc[idx] = ac;
            th -= lr * adagrad_scale(gr, ac + (T)1e-10);
            break;
        }
        case MFM_OPT_ADAM: {  // adam_step, optimizer.rs:68-85 (lazy, per-coordinate t)
            const T gr = dg + l2 * th;
            const T b1 = (T)o.b1, b2 = (T)o.b2;
            const T t = c + T(1);
            const T m = b1 * a + (T(1) - b1) * gr;
            const T v = b2 * b + (T(1) - b2) * gr * gr;
            g.t[idx] = t;
            g.m[idx] = m;
            g.s[idx] = v;
            const T mh = m / (T(1) - exp2(t * (T)o.lb1));  // b1^t
            const T vh = v / (T(1) - exp2(t * (T)o.lb2));  // b2^t
            th -= lr * mh / (sqrt(vh) + (T)o.eps);
            break;
        }
        default: {  // FTRL-Proximal, ftrl_step, optimizer.rs:93-105 (pure data gradient)
            const T n = b;
            const T nn = n + dg * dg;
            const T sigma = (sqrt(nn) - sqrt(n)) / lr;
            const T z = a + dg - sigma * th;
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
};

template <class T>
__device__ __forceinline__ void opt_step(const GroupDev<T>& g, int64_t idx, T dg,
                                         const OptDev& o) {
    CoordStep<T> cs;
    cs.load(g, idx, o.kind);
    cs.apply(g, idx, dg, o);
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
        // Adam's bias corrections 1 - b^t, computed once per distinct step
        // count in the vector (a key's coordinates are stepped together, so
        // their counts normally agree) and reused: the same values either way
        T t_prev = T(0), bc1 = T(1), bc2 = T(1);
        bool have_bc = false;
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
                th -= lr * adagrad_scale(gr, ac + (T)1e-10);
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
                if (!have_bc || t != t_prev) {
                    bc1 = T(1) - exp2(t * (T)o.lb1);  // b1^t
                    bc2 = T(1) - exp2(t * (T)o.lb2);  // b2^t
                    t_prev = t;
                    have_bc = true;
                }
                const T mh = m / bc1;
                const T vh = v / bc2;
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

}  // namespace mfm
