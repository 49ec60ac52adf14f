/*
 * mfm_oracle.c — CPU oracle (TEST INFRASTRUCTURE ONLY; see mfm_oracle.h).
 *
 * Restates modern_fm v1.1.1's Rust CPU engine operation for operation. Every
 * function cites the reference file:line it follows (paths relative to the
 * reference project root). Built with -ffp-contract=off so that a*b+c is
 * never fused, like the reference's Rust and NumPy code.
 */
#include "mfm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ADAGRAD_EPS 1e-10 /* rust/src/optimizer.rs:25 */

/* ------------------------------------------------------------------------ */
/* validation                                                               */
/* ------------------------------------------------------------------------ */

/* CsrView::new — rust/src/data.rs:14-44 */
int orc_check_csr(const int64_t* indptr, int64_t indptr_len, const int64_t* indices,
                  int64_t indices_len, int64_t data_len, int64_t n_cols, char* err,
                  int errlen) {
    if (indptr_len < 1) {
        snprintf(err, errlen, "indptr must have length n_rows + 1 (>= 1)");
        return -1;
    }
    if (indices_len != data_len) {
        snprintf(err, errlen, "indices and data length mismatch: %lld vs %lld",
                 (long long)indices_len, (long long)data_len);
        return -1;
    }
    if (indptr[indptr_len - 1] != data_len || indptr[0] != 0) {
        snprintf(err, errlen, "indptr must start at 0 and end at nnz");
        return -1;
    }
    for (int64_t r = 0; r + 1 < indptr_len; ++r) {
        if (indptr[r + 1] < indptr[r]) {
            snprintf(err, errlen, "indptr must be non-decreasing");
            return -1;
        }
    }
    for (int64_t q = 0; q < indices_len; ++q) {
        if (indices[q] < 0 || indices[q] >= n_cols) {
            snprintf(err, errlen, "column index out of range [0, %lld)", (long long)n_cols);
            return -1;
        }
    }
    return 0;
}

/* check_field_ids — rust/src/data.rs:71-83 */
int orc_check_field_ids(const int64_t* field_ids, int64_t len, int64_t n_features,
                        int64_t n_fields, char* err, int errlen) {
    if (len != n_features) {
        snprintf(err, errlen, "field_ids length %lld does not match n_features %lld",
                 (long long)len, (long long)n_features);
        return -1;
    }
    for (int64_t i = 0; i < len; ++i) {
        if (field_ids[i] < 0 || field_ids[i] >= n_fields) {
            snprintf(err, errlen, "field id out of range [0, %lld)", (long long)n_fields);
            return -1;
        }
    }
    return 0;
}

/* _prep_csr — python/modern_fm/_backend.py:44-52: `X.astype(np.float64);
 * X.sum_duplicates()`. scipy sorts each row by column and then adds each
 * column's duplicates left to right (explicit zeros are kept). Restated with a
 * stable sort, so a column's duplicates are added in their original order; the
 * result equals scipy's whenever scipy's order of equal columns is that order
 * (rows it does not reorder, at most two duplicates of a column) and differs
 * from it by rounding otherwise. The input must pass orc_check_csr. Writes
 * indptr_out (n_rows+1), indices_out / data_out (up to nnz); returns the
 * canonical entry count. */
int64_t orc_prep_csr(int64_t n_rows, const int64_t* indptr, const int64_t* indices,
                     const double* data, int64_t* indptr_out, int64_t* indices_out,
                     double* data_out) {
    int64_t o = 0, cap = 0;
    int64_t* perm = NULL;
    indptr_out[0] = 0;
    for (int64_t r = 0; r < n_rows; ++r) {
        const int64_t lo = indptr[r], len = indptr[r + 1] - lo;
        if (len > cap) {
            cap = len;
            perm = (int64_t*)realloc(perm, (size_t)cap * sizeof(int64_t));
        }
        /* stable insertion sort of the row's positions by column */
        for (int64_t t = 0; t < len; ++t) {
            int64_t u = t;
            while (u > 0 && indices[lo + perm[u - 1]] > indices[lo + t]) {
                perm[u] = perm[u - 1];
                --u;
            }
            perm[u] = t;
        }
        for (int64_t t = 0; t < len;) {
            const int64_t col = indices[lo + perm[t]];
            double x = data[lo + perm[t]];
            for (++t; t < len && indices[lo + perm[t]] == col; ++t) x += data[lo + perm[t]];
            indices_out[o] = col;
            data_out[o] = x;
            ++o;
        }
        indptr_out[r + 1] = o;
    }
    free(perm);
    return o;
}

/* ------------------------------------------------------------------------ */
/* optimizer primitives — rust/src/optimizer.rs                             */
/* ------------------------------------------------------------------------ */

/* sigmoid — optimizer.rs:28-35 (stable branch form) */
double orc_sigmoid(double s) {
    if (s >= 0.0) return 1.0 / (1.0 + exp(-s));
    double e = exp(s);
    return e / (1.0 + e);
}

/* loss_grad — optimizer.rs:38-43 */
static double loss_grad(int loss, double s, double y) {
    return loss == ORC_LOSS_LOGISTIC ? orc_sigmoid(s) - y : s - y;
}

/* apply_update (SGD / AdaGrad) — optimizer.rs:48-60 */
static void apply_update(double* theta, double grad, double* acc, double lr, int kind) {
    if (kind == ORC_OPT_SGD) {
        *theta -= lr * grad;
    } else {
        *acc += grad * grad;
        *theta -= lr * grad / sqrt(*acc + ADAGRAD_EPS);
    }
}

/* adam_step — optimizer.rs:68-85 */
void orc_adam_step(double* theta, double grad, double* m, double* v, double* t, double lr,
                   double b1, double b2, double eps) {
    *t += 1.0;
    *m = b1 * *m + (1.0 - b1) * grad;
    *v = b2 * *v + (1.0 - b2) * grad * grad;
    double m_hat = *m / (1.0 - pow(b1, *t));
    double v_hat = *v / (1.0 - pow(b2, *t));
    *theta -= lr * m_hat / (sqrt(v_hat) + eps);
}

/* ftrl_step — optimizer.rs:93-105 */
void orc_ftrl_step(double* theta, double g, double* z, double* n, double alpha, double beta,
                   double l1, double l2) {
    double n_new = *n + g * g;
    double sigma = (sqrt(n_new) - sqrt(*n)) / alpha;
    *z += g - sigma * *theta;
    *n = n_new;
    double zi = *z;
    if (fabs(zi) <= l1) {
        *theta = 0.0;
    } else {
        double sign = zi < 0.0 ? -1.0 : 1.0;
        *theta = -(zi - sign * l1) / ((beta + sqrt(n_new)) / alpha + l2);
    }
}

/* step_param / step_coord — optimizer.rs:114-167. `st` arrays are indexed at
 * idx only on the path that uses them. */
static void step_coord(double* theta, double data_grad, double l1, double l2, orc_state st,
                       int64_t idx, const orc_opt* o) {
    switch (o->kind) {
    case ORC_OPT_FTRL:
        orc_ftrl_step(theta, data_grad, &st.z[idx], &st.n[idx], o->lr, o->ftrl_beta, l1, l2);
        break;
    case ORC_OPT_ADAM:
        orc_adam_step(theta, data_grad + l2 * *theta, &st.m[idx], &st.s[idx], &st.t[idx],
                      o->lr, o->beta1, o->beta2, o->eps);
        break;
    default:
        apply_update(theta, data_grad + l2 * *theta, st.acc ? &st.acc[idx] : NULL, o->lr,
                     o->kind);
    }
}

/* Offset a state view by `off` elements (McState::class_views,
 * optimizer.rs:428-458; class_slice :290-296). */
static orc_state state_at(orc_state st, int64_t off) {
    orc_state r;
    r.acc = st.acc ? st.acc + off : NULL;
    r.m = st.m ? st.m + off : NULL;
    r.s = st.s ? st.s + off : NULL;
    r.t = st.t ? st.t + off : NULL;
    r.z = st.z ? st.z + off : NULL;
    r.n = st.n ? st.n + off : NULL;
    return r;
}

/* ------------------------------------------------------------------------ */
/* row scoring                                                              */
/* ------------------------------------------------------------------------ */

/* fm_score_row — rust/src/fm.rs:16-40 */
static double fm_score_row(const int64_t* idx, const double* val, int64_t z, double w0,
                           const double* w, const double* v, int64_t k, double* sum,
                           double* sum_sq) {
    double s = w0;
    for (int64_t f = 0; f < k; ++f) sum[f] = sum_sq[f] = 0.0;
    for (int64_t a = 0; a < z; ++a) {
        int64_t i = idx[a];
        double x = val[a];
        s += w[i] * x;
        const double* vi = v + i * k;
        for (int64_t f = 0; f < k; ++f) {
            double vx = vi[f] * x;
            sum[f] += vx;
            sum_sq[f] += vx * vx;
        }
    }
    double pairwise = 0.0;
    for (int64_t f = 0; f < k; ++f) pairwise += sum[f] * sum[f] - sum_sq[f];
    return s + 0.5 * pairwise;
}

/* train_score_row — rust/src/fm.rs:77-101 ((dot - sq) order, fills cache) */
static double train_score_row(const int64_t* idx, const double* val, int64_t z, double w0,
                              const double* w, const double* v, int64_t k, double* cache) {
    for (int64_t f = 0; f < k; ++f) cache[f] = 0.0;
    double s = w0, sq = 0.0;
    for (int64_t a = 0; a < z; ++a) {
        int64_t i = idx[a];
        double x = val[a];
        s += w[i] * x;
        const double* vi = v + i * k;
        for (int64_t f = 0; f < k; ++f) {
            double vx = vi[f] * x;
            cache[f] += vx;
            sq += vx * vx;
        }
    }
    double dot = 0.0;
    for (int64_t f = 0; f < k; ++f) dot += cache[f] * cache[f];
    return s + 0.5 * (dot - sq);
}

/* ffm_score_row — rust/src/ffm.rs:18-45 */
static double ffm_score_row(const int64_t* idx, const double* val, int64_t z,
                            const int64_t* field_ids, double w0, const double* w,
                            const double* v, int64_t F, int64_t k) {
    double s = w0;
    for (int64_t a = 0; a < z; ++a) s += w[idx[a]] * val[a];
    for (int64_t a = 0; a < z; ++a) {
        int64_t i = idx[a];
        double xi = val[a];
        int64_t fi = field_ids[i];
        for (int64_t b = a + 1; b < z; ++b) {
            int64_t j = idx[b];
            double xj = val[b];
            int64_t fj = field_ids[j];
            const double* vi = v + (i * F + fj) * k;
            const double* vj = v + (j * F + fi) * k;
            double dot = 0.0;
            for (int64_t t = 0; t < k; ++t) dot += vi[t] * vj[t];
            s += dot * xi * xj;
        }
    }
    return s;
}

/* pair_slot — rust/src/fwfm.rs:17-21 */
static inline int64_t pair_slot(int64_t fa, int64_t fb, int64_t F) {
    return fa <= fb ? fa * F + fb : fb * F + fa;
}

/* fwfm_score_row — rust/src/fwfm.rs:24-53 */
static double fwfm_score_row(const int64_t* idx, const double* val, int64_t z,
                             const int64_t* field_ids, double w0, const double* w,
                             const double* v, const double* r, int64_t F, int64_t k) {
    double s = w0;
    for (int64_t a = 0; a < z; ++a) s += w[idx[a]] * val[a];
    for (int64_t a = 0; a < z; ++a) {
        int64_t i = idx[a];
        double xi = val[a];
        int64_t fi = field_ids[i];
        for (int64_t b = a + 1; b < z; ++b) {
            int64_t j = idx[b];
            double xj = val[b];
            int64_t fj = field_ids[j];
            const double* vi = v + i * k;
            const double* vj = v + j * k;
            double dot = 0.0;
            for (int64_t t = 0; t < k; ++t) dot += vi[t] * vj[t];
            s += r[pair_slot(fi, fj, F)] * dot * xi * xj;
        }
    }
    return s;
}

/* ------------------------------------------------------------------------ */
/* prediction                                                               */
/* ------------------------------------------------------------------------ */

typedef struct {
    int model; /* 0 FM, 1 FFM, 2 FwFM */
    const int64_t *indptr, *indices, *field_ids;
    const double *data, *w, *v, *r;
    double w0;
    int64_t n_rows, F, k;
    double* out;
    int n_threads;
} predict_job;

typedef struct {
    predict_job* job;
    int tid;
} predict_arg;

static void* predict_worker(void* p) {
    predict_arg* a = (predict_arg*)p;
    predict_job* j = a->job;
    int64_t per = (j->n_rows + j->n_threads - 1) / j->n_threads;
    int64_t lo = per * a->tid, hi = lo + per < j->n_rows ? lo + per : j->n_rows;
    double* sum = (double*)malloc(sizeof(double) * (size_t)(j->k > 0 ? j->k : 1));
    double* sq = (double*)malloc(sizeof(double) * (size_t)(j->k > 0 ? j->k : 1));
    for (int64_t row = lo; row < hi; ++row) {
        int64_t b = j->indptr[row], e = j->indptr[row + 1];
        const int64_t* idx = j->indices + b;
        const double* val = j->data + b;
        if (j->model == 0)
            j->out[row] = fm_score_row(idx, val, e - b, j->w0, j->w, j->v, j->k, sum, sq);
        else if (j->model == 1)
            j->out[row] = ffm_score_row(idx, val, e - b, j->field_ids, j->w0, j->w, j->v,
                                        j->F, j->k);
        else
            j->out[row] = fwfm_score_row(idx, val, e - b, j->field_ids, j->w0, j->w, j->v,
                                         j->r, j->F, j->k);
    }
    free(sum);
    free(sq);
    return NULL;
}

/* Rows are independent, so splitting them across threads gives results
 * identical to the reference's serial loops (fm.rs:58-70, ffm.rs:73-91,
 * fwfm.rs:82-101). */
static void run_predict(predict_job* job) {
    int nt = job->n_threads < 1 ? 1 : job->n_threads;
    if (job->n_rows < nt) nt = job->n_rows < 1 ? 1 : (int)job->n_rows;
    job->n_threads = nt;
    predict_arg args[256];
    pthread_t th[256];
    if (nt > 256) nt = job->n_threads = 256;
    for (int t = 0; t < nt; ++t) {
        args[t].job = job;
        args[t].tid = t;
    }
    for (int t = 1; t < nt; ++t) pthread_create(&th[t], NULL, predict_worker, &args[t]);
    predict_worker(&args[0]);
    for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

void orc_fm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                        int64_t n_rows, double w0, const double* w, const double* v,
                        int64_t k, double* out, int n_threads) {
    predict_job j = {0, indptr, indices, NULL, data, w, v, NULL, w0, n_rows, 0, k, out,
                     n_threads};
    run_predict(&j);
}

void orc_ffm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                         int64_t n_rows, const int64_t* field_ids, double w0,
                         const double* w, const double* v, int64_t n_fields, int64_t k,
                         double* out, int n_threads) {
    predict_job j = {1, indptr, indices, field_ids, data, w, v, NULL, w0, n_rows,
                     n_fields, k, out, n_threads};
    run_predict(&j);
}

void orc_fwfm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                          int64_t n_rows, const int64_t* field_ids, double w0,
                          const double* w, const double* v, const double* r,
                          int64_t n_fields, int64_t k, double* out, int n_threads) {
    predict_job j = {2, indptr, indices, field_ids, data, w, v, r, w0, n_rows,
                     n_fields, k, out, n_threads};
    run_predict(&j);
}

/* dense_row_nonzeros — rust/src/data.rs:60-69 (exact zeros skipped) */
static int64_t dense_row_nonzeros(const double* row, int64_t n, int64_t* idx, double* val) {
    int64_t z = 0;
    for (int64_t i = 0; i < n; ++i)
        if (row[i] != 0.0) {
            idx[z] = i;
            val[z++] = row[i];
        }
    return z;
}

/* predict_dense — fm.rs:42-55, ffm.rs:48-69, fwfm.rs:56-78 */
static void predict_dense(int model, const double* x, int64_t n_rows, int64_t n_features,
                          const int64_t* field_ids, double w0, const double* w,
                          const double* v, const double* r, int64_t F, int64_t k,
                          double* out) {
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n_features + 1));
    double* val = (double*)malloc(sizeof(double) * (size_t)(n_features + 1));
    double* sum = (double*)malloc(sizeof(double) * (size_t)(k + 1));
    double* sq = (double*)malloc(sizeof(double) * (size_t)(k + 1));
    for (int64_t row = 0; row < n_rows; ++row) {
        int64_t z = dense_row_nonzeros(x + row * n_features, n_features, idx, val);
        if (model == 0)
            out[row] = fm_score_row(idx, val, z, w0, w, v, k, sum, sq);
        else if (model == 1)
            out[row] = ffm_score_row(idx, val, z, field_ids, w0, w, v, F, k);
        else
            out[row] = fwfm_score_row(idx, val, z, field_ids, w0, w, v, r, F, k);
    }
    free(idx);
    free(val);
    free(sum);
    free(sq);
}

void orc_fm_predict_dense(const double* x, int64_t n_rows, int64_t n_features, double w0,
                          const double* w, const double* v, int64_t k, double* out) {
    predict_dense(0, x, n_rows, n_features, NULL, w0, w, v, NULL, 0, k, out);
}
void orc_ffm_predict_dense(const double* x, int64_t n_rows, int64_t n_features,
                           const int64_t* field_ids, double w0, const double* w,
                           const double* v, int64_t n_fields, int64_t k, double* out) {
    predict_dense(1, x, n_rows, n_features, field_ids, w0, w, v, NULL, n_fields, k, out);
}
void orc_fwfm_predict_dense(const double* x, int64_t n_rows, int64_t n_features,
                            const int64_t* field_ids, double w0, const double* w,
                            const double* v, const double* r, int64_t n_fields, int64_t k,
                            double* out) {
    predict_dense(2, x, n_rows, n_features, field_ids, w0, w, v, r, n_fields, k, out);
}

/* ------------------------------------------------------------------------ */
/* gradient accumulators                                                    */
/* ------------------------------------------------------------------------ */

/* One batch accumulator: FmGradAccum (fm.rs:115-221), FfmGradAccum
 * (ffm.rs:103-252) and FwfmGradAccum (fwfm.rs:112-242) share this shape:
 * features (gw, touched, seen), a second key space of "slots" (FFM
 * (feature, field) slots with k-wide gv, FwFM upper-triangle field pairs with
 * scalar gr), and FM/FwFM per-feature k-wide gv. */
typedef struct {
    double g_w0;
    double* gw;
    double* gv;
    int64_t* touched;
    int64_t n_touched;
    unsigned char* seen;
    int64_t* tslot;
    int64_t n_tslot;
    unsigned char* seen_slot;
    double* gr;
} accum;

static int accum_init(accum* a, int64_t n, int64_t gv_len, int64_t n_slots, int64_t gr_len) {
    memset(a, 0, sizeof(*a));
    a->gw = (double*)calloc((size_t)(n > 0 ? n : 1), sizeof(double));
    a->gv = (double*)calloc((size_t)(gv_len > 0 ? gv_len : 1), sizeof(double));
    a->touched = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    a->seen = (unsigned char*)calloc((size_t)(n > 0 ? n : 1), 1);
    a->tslot = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n_slots > 0 ? n_slots : 1));
    a->seen_slot = (unsigned char*)calloc((size_t)(n_slots > 0 ? n_slots : 1), 1);
    a->gr = (double*)calloc((size_t)(gr_len > 0 ? gr_len : 1), sizeof(double));
    return (a->gw && a->gv && a->touched && a->seen && a->tslot && a->seen_slot && a->gr)
               ? 0
               : -1;
}

static void accum_free(accum* a) {
    free(a->gw);
    free(a->gv);
    free(a->touched);
    free(a->seen);
    free(a->tslot);
    free(a->seen_slot);
    free(a->gr);
}

static inline void touch(accum* a, int64_t i) {
    if (!a->seen[i]) {
        a->seen[i] = 1;
        a->touched[a->n_touched++] = i;
    }
}
static inline void touch_slot(accum* a, int64_t s) {
    if (!a->seen_slot[s]) {
        a->seen_slot[s] = 1;
        a->tslot[a->n_tslot++] = s;
    }
}

/* FmGradAccum::add_row — fm.rs:133-146 */
static void fm_add_row(accum* a, const int64_t* idx, const double* val, int64_t z, double g,
                       const double* cache, const double* v, int64_t k) {
    a->g_w0 += g;
    for (int64_t p = 0; p < z; ++p) {
        int64_t i = idx[p];
        double x = val[p];
        touch(a, i);
        a->gw[i] += g * x;
        int64_t base = i * k;
        for (int64_t f = 0; f < k; ++f)
            a->gv[base + f] += g * (x * cache[f] - v[base + f] * x * x);
    }
}

/* FmGradAccum::merge_from — fm.rs:151-169 (other is cleared) */
static void fm_merge_from(accum* self, accum* other, int64_t k) {
    self->g_w0 += other->g_w0;
    other->g_w0 = 0.0;
    for (int64_t q = 0; q < other->n_touched; ++q) {
        int64_t i = other->touched[q];
        touch(self, i);
        self->gw[i] += other->gw[i];
        other->gw[i] = 0.0;
        int64_t base = i * k;
        for (int64_t f = 0; f < k; ++f) {
            self->gv[base + f] += other->gv[base + f];
            other->gv[base + f] = 0.0;
        }
        other->seen[i] = 0;
    }
    other->n_touched = 0;
}

/* FmGradAccum::flush — fm.rs:174-220 (update order w0 -> w -> V) */
static void fm_flush(accum* a, double bsz, double* w0, double* w, double* v, orc_state st_w0,
                     orc_state st_w, orc_state st_v, int64_t k, const orc_opt* o) {
    step_coord(w0, a->g_w0 / bsz, 0.0, 0.0, st_w0, 0, o);
    a->g_w0 = 0.0;
    for (int64_t q = 0; q < a->n_touched; ++q) {
        int64_t i = a->touched[q];
        step_coord(&w[i], a->gw[i] / bsz, o->l1_linear, o->l2_linear, st_w, i, o);
        a->gw[i] = 0.0;
        int64_t base = i * k;
        for (int64_t f = 0; f < k; ++f) {
            int64_t vi = base + f;
            step_coord(&v[vi], a->gv[vi] / bsz, o->l1_factors, o->l2_factors, st_v, vi, o);
            a->gv[vi] = 0.0;
        }
        a->seen[i] = 0;
    }
    a->n_touched = 0;
}

/* FfmGradAccum::add_row — ffm.rs:129-171 */
static void ffm_add_row(accum* a, const int64_t* idx, const double* val, int64_t z,
                        const int64_t* field_ids, double g, const double* v, int64_t F,
                        int64_t k) {
    a->g_w0 += g;
    for (int64_t p = 0; p < z; ++p) {
        touch(a, idx[p]);
        a->gw[idx[p]] += g * val[p];
    }
    for (int64_t p = 0; p < z; ++p) {
        int64_t i = idx[p];
        double xi = val[p];
        int64_t fi = field_ids[i];
        for (int64_t b = p + 1; b < z; ++b) {
            int64_t j = idx[b];
            double xj = val[b];
            int64_t fj = field_ids[j];
            double coef = g * xi * xj;
            int64_t slot_a = i * F + fj, slot_b = j * F + fi;
            int64_t va = slot_a * k, vb = slot_b * k;
            for (int64_t t = 0; t < k; ++t) {
                a->gv[va + t] += coef * v[vb + t];
                a->gv[vb + t] += coef * v[va + t];
            }
            touch_slot(a, slot_a);
            touch_slot(a, slot_b);
        }
    }
}

/* FfmGradAccum::merge_from — ffm.rs:174-200 */
static void ffm_merge_from(accum* self, accum* other, int64_t k) {
    self->g_w0 += other->g_w0;
    other->g_w0 = 0.0;
    for (int64_t q = 0; q < other->n_touched; ++q) {
        int64_t i = other->touched[q];
        touch(self, i);
        self->gw[i] += other->gw[i];
        other->gw[i] = 0.0;
        other->seen[i] = 0;
    }
    other->n_touched = 0;
    for (int64_t q = 0; q < other->n_tslot; ++q) {
        int64_t s = other->tslot[q];
        touch_slot(self, s);
        int64_t base = s * k;
        for (int64_t t = 0; t < k; ++t) {
            self->gv[base + t] += other->gv[base + t];
            other->gv[base + t] = 0.0;
        }
        other->seen_slot[s] = 0;
    }
    other->n_tslot = 0;
}

/* FfmGradAccum::flush — ffm.rs:205-251 (w0, then w, then V slots) */
static void ffm_flush(accum* a, double bsz, double* w0, double* w, double* v,
                      orc_state st_w0, orc_state st_w, orc_state st_v, int64_t k,
                      const orc_opt* o) {
    step_coord(w0, a->g_w0 / bsz, 0.0, 0.0, st_w0, 0, o);
    a->g_w0 = 0.0;
    for (int64_t q = 0; q < a->n_touched; ++q) {
        int64_t i = a->touched[q];
        step_coord(&w[i], a->gw[i] / bsz, o->l1_linear, o->l2_linear, st_w, i, o);
        a->gw[i] = 0.0;
        a->seen[i] = 0;
    }
    a->n_touched = 0;
    for (int64_t q = 0; q < a->n_tslot; ++q) {
        int64_t s = a->tslot[q];
        int64_t base = s * k;
        for (int64_t t = 0; t < k; ++t) {
            int64_t vi = base + t;
            step_coord(&v[vi], a->gv[vi] / bsz, o->l1_factors, o->l2_factors, st_v, vi, o);
            a->gv[vi] = 0.0;
        }
        a->seen_slot[s] = 0;
    }
    a->n_tslot = 0;
}

/* FwfmGradAccum::add_row — fwfm.rs:140-183 */
static void fwfm_add_row(accum* a, const int64_t* idx, const double* val, int64_t z,
                         const int64_t* field_ids, double g, const double* v, const double* r,
                         int64_t F, int64_t k) {
    a->g_w0 += g;
    for (int64_t p = 0; p < z; ++p) {
        touch(a, idx[p]);
        a->gw[idx[p]] += g * val[p];
    }
    for (int64_t p = 0; p < z; ++p) {
        int64_t i = idx[p];
        double xi = val[p];
        int64_t fi = field_ids[i];
        for (int64_t b = p + 1; b < z; ++b) {
            int64_t j = idx[b];
            double xj = val[b];
            int64_t fj = field_ids[j];
            int64_t slot = pair_slot(fi, fj, F);
            double coef = g * xi * xj;
            double rw = r[slot];
            int64_t vi = i * k, vj = j * k;
            double dot = 0.0;
            for (int64_t t = 0; t < k; ++t) {
                dot += v[vi + t] * v[vj + t];
                a->gv[vi + t] += coef * rw * v[vj + t];
                a->gv[vj + t] += coef * rw * v[vi + t];
            }
            a->gr[slot] += coef * dot;
            touch_slot(a, slot);
        }
    }
}

/* FwfmGradAccum::flush — fwfm.rs:188-241 (w0, then w+V per feature, then R) */
static void fwfm_flush(accum* a, double bsz, double* w0, double* w, double* v, double* r,
                       orc_state st_w0, orc_state st_w, orc_state st_v, orc_state st_r,
                       int64_t k, const orc_opt* o) {
    step_coord(w0, a->g_w0 / bsz, 0.0, 0.0, st_w0, 0, o);
    a->g_w0 = 0.0;
    for (int64_t q = 0; q < a->n_touched; ++q) {
        int64_t i = a->touched[q];
        step_coord(&w[i], a->gw[i] / bsz, o->l1_linear, o->l2_linear, st_w, i, o);
        a->gw[i] = 0.0;
        int64_t base = i * k;
        for (int64_t f = 0; f < k; ++f) {
            int64_t vi = base + f;
            step_coord(&v[vi], a->gv[vi] / bsz, o->l1_factors, o->l2_factors, st_v, vi, o);
            a->gv[vi] = 0.0;
        }
        a->seen[i] = 0;
    }
    a->n_touched = 0;
    for (int64_t q = 0; q < a->n_tslot; ++q) {
        int64_t s = a->tslot[q];
        step_coord(&r[s], a->gr[s] / bsz, o->l1_factors, o->l2_factors, st_r, s, o);
        a->gr[s] = 0.0;
        a->seen_slot[s] = 0;
    }
    a->n_tslot = 0;
}

/* ------------------------------------------------------------------------ */
/* persistent worker pool for the n_jobs>1 batch fill (rayon stand-in)      */
/* ------------------------------------------------------------------------ */

typedef struct {
    int n;
    pthread_t* th;
    pthread_barrier_t start, done;
    void (*fn)(void*, int);
    void* arg;
    int quit;
} pool_t;

typedef struct {
    pool_t* p;
    int tid;
} pool_arg;

static void* pool_main(void* raw) {
    pool_arg* a = (pool_arg*)raw;
    for (;;) {
        pthread_barrier_wait(&a->p->start);
        if (a->p->quit) break;
        a->p->fn(a->p->arg, a->tid);
        pthread_barrier_wait(&a->p->done);
    }
    free(a);
    return NULL;
}

static void pool_init(pool_t* p, int n) {
    p->n = n;
    p->quit = 0;
    p->th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n);
    pthread_barrier_init(&p->start, NULL, (unsigned)n);
    pthread_barrier_init(&p->done, NULL, (unsigned)n);
    for (int t = 1; t < n; ++t) {
        pool_arg* a = (pool_arg*)malloc(sizeof(pool_arg));
        a->p = p;
        a->tid = t;
        pthread_create(&p->th[t], NULL, pool_main, a);
    }
}

static void pool_run(pool_t* p, void (*fn)(void*, int), void* arg) {
    p->fn = fn;
    p->arg = arg;
    pthread_barrier_wait(&p->start);
    fn(arg, 0);
    pthread_barrier_wait(&p->done);
}

static void pool_destroy(pool_t* p) {
    p->quit = 1;
    pthread_barrier_wait(&p->start);
    for (int t = 1; t < p->n; ++t) pthread_join(p->th[t], NULL);
    pthread_barrier_destroy(&p->start);
    pthread_barrier_destroy(&p->done);
    free(p->th);
}

/* ------------------------------------------------------------------------ */
/* binary FM / FFM training with the n_jobs contiguous-chunk split           */
/* ------------------------------------------------------------------------ */

typedef struct {
    int model; /* 0 FM, 1 FFM */
    const int64_t *indptr, *indices, *field_ids;
    const double *data, *y, *sw, *w, *v;
    double w0;
    int64_t F, k;
    int loss;
    accum* accs;
    double** caches;
    const int64_t* batch;
    int64_t batch_len, chunk_len;
} fill_job;

/* accumulate_chunk — fm.rs:227-246 / ffm.rs:257-280 */
static void fill_chunk(void* raw, int tid) {
    fill_job* j = (fill_job*)raw;
    int64_t lo = (int64_t)tid * j->chunk_len;
    if (lo >= j->batch_len) return; /* zip() stops at the shorter side */
    int64_t hi = lo + j->chunk_len < j->batch_len ? lo + j->chunk_len : j->batch_len;
    accum* a = &j->accs[tid];
    for (int64_t q = lo; q < hi; ++q) {
        int64_t row = j->batch[q];
        int64_t b = j->indptr[row], e = j->indptr[row + 1];
        const int64_t* idx = j->indices + b;
        const double* val = j->data + b;
        if (j->model == 0) {
            double s = train_score_row(idx, val, e - b, j->w0, j->w, j->v, j->k,
                                       j->caches[tid]);
            double g = j->sw[row] * loss_grad(j->loss, s, j->y[row]);
            fm_add_row(a, idx, val, e - b, g, j->caches[tid], j->v, j->k);
        } else {
            double s = ffm_score_row(idx, val, e - b, j->field_ids, j->w0, j->w, j->v, j->F,
                                     j->k);
            double g = j->sw[row] * loss_grad(j->loss, s, j->y[row]);
            ffm_add_row(a, idx, val, e - b, j->field_ids, g, j->v, j->F, j->k);
        }
    }
}

/* fm::fit_csr — fm.rs:265-318; ffm::fit_csr — ffm.rs:296-356 */
static int fit_binary(int model, const int64_t* indptr, const int64_t* indices,
                      const double* data, int64_t n_rows, int64_t n_features, const double* y,
                      const double* sw, const int64_t* field_ids, int64_t F, double* w0,
                      double* w, double* v, int64_t k, orc_state st_w0, orc_state st_w,
                      orc_state st_v, int loss, const orc_opt* o, const int64_t* row_orders,
                      int64_t n_epochs, int64_t batch_size, int n_jobs) {
    int nt = n_jobs < 1 ? 1 : n_jobs;
    int64_t n = n_features;
    int64_t gv_len = model == 0 ? n * k : n * F * k;
    int64_t n_slots = model == 0 ? 0 : n * F;
    accum* accs = (accum*)calloc((size_t)nt, sizeof(accum));
    double** caches = (double**)calloc((size_t)nt, sizeof(double*));
    int rc = 0;
    for (int t = 0; t < nt; ++t) {
        if (accum_init(&accs[t], n, gv_len, n_slots, 0)) rc = -1;
        caches[t] = (double*)calloc((size_t)(k > 0 ? k : 1), sizeof(double));
    }
    pool_t pool;
    if (!rc && nt > 1) pool_init(&pool, nt);
    fill_job job;
    memset(&job, 0, sizeof(job));
    job.model = model;
    job.indptr = indptr;
    job.indices = indices;
    job.field_ids = field_ids;
    job.data = data;
    job.y = y;
    job.sw = sw;
    job.w = w;
    job.v = v;
    job.F = F;
    job.k = k;
    job.loss = loss;
    job.accs = accs;
    job.caches = caches;
    for (int64_t e = 0; !rc && e < n_epochs; ++e) {
        const int64_t* order = row_orders + e * n_rows;
        for (int64_t start = 0; start < n_rows; start += batch_size) {
            int64_t len = n_rows - start < batch_size ? n_rows - start : batch_size;
            job.batch = order + start;
            job.batch_len = len;
            job.w0 = *w0;
            if (nt == 1) {
                job.chunk_len = len;
                fill_chunk(&job, 0);
            } else {
                job.chunk_len = (len + nt - 1) / nt; /* div_ceil */
                pool_run(&pool, fill_chunk, &job);
                for (int t = 1; t < nt; ++t) {
                    if (model == 0)
                        fm_merge_from(&accs[0], &accs[t], k);
                    else
                        ffm_merge_from(&accs[0], &accs[t], k);
                }
            }
            if (model == 0)
                fm_flush(&accs[0], (double)len, w0, w, v, st_w0, st_w, st_v, k, o);
            else
                ffm_flush(&accs[0], (double)len, w0, w, v, st_w0, st_w, st_v, k, o);
        }
    }
    if (!rc && nt > 1) pool_destroy(&pool);
    for (int t = 0; t < nt; ++t) {
        accum_free(&accs[t]);
        free(caches[t]);
    }
    free(accs);
    free(caches);
    return rc;
}

int orc_fm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                   int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                   double* w0, double* w, double* v, int64_t k, orc_state st_w0,
                   orc_state st_w, orc_state st_v, int loss, const orc_opt* opt,
                   const int64_t* row_orders, int64_t n_epochs, int64_t batch_size,
                   int n_jobs) {
    return fit_binary(0, indptr, indices, data, n_rows, n_features, y, sw, NULL, 0, w0, w, v,
                      k, st_w0, st_w, st_v, loss, opt, row_orders, n_epochs, batch_size,
                      n_jobs);
}

int orc_ffm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                    int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                    const int64_t* field_ids, int64_t n_fields, double* w0, double* w,
                    double* v, int64_t k, orc_state st_w0, orc_state st_w, orc_state st_v,
                    int loss, const orc_opt* opt, const int64_t* row_orders,
                    int64_t n_epochs, int64_t batch_size, int n_jobs) {
    return fit_binary(1, indptr, indices, data, n_rows, n_features, y, sw, field_ids,
                      n_fields, w0, w, v, k, st_w0, st_w, st_v, loss, opt, row_orders,
                      n_epochs, batch_size, n_jobs);
}

/* fwfm::fit_csr — fwfm.rs:252-300 (serial) */
int orc_fwfm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                     int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                     const int64_t* field_ids, int64_t F, double* w0, double* w, double* v,
                     double* r, int64_t k, orc_state st_w0, orc_state st_w, orc_state st_v,
                     orc_state st_r, int loss, const orc_opt* o, const int64_t* row_orders,
                     int64_t n_epochs, int64_t batch_size) {
    accum a;
    if (accum_init(&a, n_features, n_features * k, F * F, F * F)) {
        accum_free(&a);
        return -1;
    }
    for (int64_t e = 0; e < n_epochs; ++e) {
        const int64_t* order = row_orders + e * n_rows;
        for (int64_t start = 0; start < n_rows; start += batch_size) {
            int64_t len = n_rows - start < batch_size ? n_rows - start : batch_size;
            for (int64_t q = 0; q < len; ++q) {
                int64_t row = order[start + q];
                int64_t b = indptr[row], e2 = indptr[row + 1];
                double s = fwfm_score_row(indices + b, data + b, e2 - b, field_ids, *w0, w, v,
                                          r, F, k);
                double g = sw[row] * loss_grad(loss, s, y[row]);
                fwfm_add_row(&a, indices + b, data + b, e2 - b, field_ids, g, v, r, F, k);
            }
            fwfm_flush(&a, (double)len, w0, w, v, r, st_w0, st_w, st_v, st_r, k, o);
        }
    }
    accum_free(&a);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* multiclass (softmax) training — fm.rs:333-409, ffm.rs:371-447,            */
/* fwfm.rs:307-394                                                          */
/* ------------------------------------------------------------------------ */

static int fit_multiclass(int model, const int64_t* indptr, const int64_t* indices,
                          const double* data, int64_t n_rows, int64_t n, const int64_t* y,
                          const double* sw, int64_t C, const int64_t* field_ids, int64_t F,
                          double* w0, double* w, double* v, double* r, int64_t k,
                          orc_state st_w0, orc_state st_w, orc_state st_v, orc_state st_r,
                          const orc_opt* o, double ls, const int64_t* row_orders,
                          int64_t n_epochs, int64_t batch_size) {
    int64_t vc = model == 1 ? n * F * k : n * k; /* V entries per class */
    int64_t rc = F * F;                           /* R entries per class */
    int64_t n_slots = model == 0 ? 0 : (model == 1 ? n * F : F * F);
    accum* acc = (accum*)calloc((size_t)C, sizeof(accum));
    int bad = 0;
    for (int64_t c = 0; c < C; ++c)
        if (accum_init(&acc[c], n, vc, n_slots, model == 2 ? rc : 0)) bad = 1;
    double off = C > 1 ? ls / ((double)C - 1.0) : 0.0;
    double* probs = (double*)calloc((size_t)C, sizeof(double));
    double* caches = (double*)calloc((size_t)(C * (k > 0 ? k : 1)), sizeof(double));
    for (int64_t e = 0; !bad && e < n_epochs; ++e) {
        const int64_t* order = row_orders + e * n_rows;
        for (int64_t start = 0; start < n_rows; start += batch_size) {
            int64_t len = n_rows - start < batch_size ? n_rows - start : batch_size;
            for (int64_t q = 0; q < len; ++q) {
                int64_t row = order[start + q];
                int64_t b = indptr[row], e2 = indptr[row + 1], z = e2 - b;
                const int64_t* idx = indices + b;
                const double* val = data + b;
                int64_t yc = y[row];
                double s_w = sw[row];
                /* pass 1: per-class logits from the frozen parameters */
                for (int64_t c = 0; c < C; ++c) {
                    if (model == 0)
                        probs[c] = train_score_row(idx, val, z, w0[c], w + c * n, v + c * vc,
                                                   k, caches + c * k);
                    else if (model == 1)
                        probs[c] = ffm_score_row(idx, val, z, field_ids, w0[c], w + c * n,
                                                 v + c * vc, F, k);
                    else
                        probs[c] = fwfm_score_row(idx, val, z, field_ids, w0[c], w + c * n,
                                                  v + c * vc, r + c * rc, F, k);
                }
                /* stable softmax: subtract max, sum exp in class order */
                double maxl = -INFINITY;
                for (int64_t c = 0; c < C; ++c) maxl = fmax(maxl, probs[c]);
                double sum_ex = 0.0;
                for (int64_t c = 0; c < C; ++c) {
                    probs[c] = exp(probs[c] - maxl);
                    sum_ex += probs[c];
                }
                for (int64_t c = 0; c < C; ++c) {
                    double p = probs[c] / sum_ex;
                    double target = c == yc ? 1.0 - ls : off;
                    double g = s_w * (p - target);
                    if (model == 0)
                        fm_add_row(&acc[c], idx, val, z, g, caches + c * k, v + c * vc, k);
                    else if (model == 1)
                        ffm_add_row(&acc[c], idx, val, z, field_ids, g, v + c * vc, F, k);
                    else
                        fwfm_add_row(&acc[c], idx, val, z, field_ids, g, v + c * vc,
                                     r + c * rc, F, k);
                }
            }
            double bsz = (double)len;
            for (int64_t c = 0; c < C; ++c) {
                orc_state s0 = state_at(st_w0, c), sw_ = state_at(st_w, c * n),
                          sv = state_at(st_v, c * vc);
                if (model == 0)
                    fm_flush(&acc[c], bsz, &w0[c], w + c * n, v + c * vc, s0, sw_, sv, k, o);
                else if (model == 1)
                    ffm_flush(&acc[c], bsz, &w0[c], w + c * n, v + c * vc, s0, sw_, sv, k, o);
                else
                    fwfm_flush(&acc[c], bsz, &w0[c], w + c * n, v + c * vc, r + c * rc, s0,
                               sw_, sv, state_at(st_r, c * rc), k, o);
            }
        }
    }
    for (int64_t c = 0; c < C; ++c) accum_free(&acc[c]);
    free(acc);
    free(probs);
    free(caches);
    return bad ? -1 : 0;
}

int orc_fm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                              const double* data, int64_t n_rows, int64_t n_features,
                              const int64_t* y, const double* sw, int64_t n_classes,
                              double* w0, double* w, double* v, int64_t k, orc_state st_w0,
                              orc_state st_w, orc_state st_v, const orc_opt* opt,
                              double label_smoothing, const int64_t* row_orders,
                              int64_t n_epochs, int64_t batch_size) {
    orc_state none;
    memset(&none, 0, sizeof(none));
    return fit_multiclass(0, indptr, indices, data, n_rows, n_features, y, sw, n_classes,
                          NULL, 0, w0, w, v, NULL, k, st_w0, st_w, st_v, none, opt,
                          label_smoothing, row_orders, n_epochs, batch_size);
}

int orc_ffm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                               const double* data, int64_t n_rows, int64_t n_features,
                               const int64_t* y, const double* sw, int64_t n_classes,
                               const int64_t* field_ids, int64_t n_fields, double* w0,
                               double* w, double* v, int64_t k, orc_state st_w0,
                               orc_state st_w, orc_state st_v, const orc_opt* opt,
                               double label_smoothing, const int64_t* row_orders,
                               int64_t n_epochs, int64_t batch_size) {
    orc_state none;
    memset(&none, 0, sizeof(none));
    return fit_multiclass(1, indptr, indices, data, n_rows, n_features, y, sw, n_classes,
                          field_ids, n_fields, w0, w, v, NULL, k, st_w0, st_w, st_v, none,
                          opt, label_smoothing, row_orders, n_epochs, batch_size);
}

int orc_fwfm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                                const double* data, int64_t n_rows, int64_t n_features,
                                const int64_t* y, const double* sw, int64_t n_classes,
                                const int64_t* field_ids, int64_t n_fields, double* w0,
                                double* w, double* v, double* r, int64_t k,
                                orc_state st_w0, orc_state st_w, orc_state st_v,
                                orc_state st_r, const orc_opt* opt, double label_smoothing,
                                const int64_t* row_orders, int64_t n_epochs,
                                int64_t batch_size) {
    return fit_multiclass(2, indptr, indices, data, n_rows, n_features, y, sw, n_classes,
                          field_ids, n_fields, w0, w, v, r, k, st_w0, st_w, st_v, st_r, opt,
                          label_smoothing, row_orders, n_epochs, batch_size);
}
