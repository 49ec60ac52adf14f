/*
 * mfm_oracle.h — CPU oracle for the modern_fm sparse-CSR FM / FFM / FwFM path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference's
 * Rust CPU engine (modern_fm v1.1.1, rust/src/{data,fm,ffm,fwfm,optimizer}.rs),
 * operation for operation, used as the checker for the CUDA path and as the
 * timed CPU baseline. Nothing in the product library (modern_fm_b200/) links,
 * loads or calls it; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg do.
 *
 * Pinned against: the reference's own known-answer vectors (FM 4.25, FFM 9.5,
 * FwFM 10.25, hand-computed SGD / Adam / multiclass steps, optimizer first
 * steps) and against fixtures produced by the reference's NumPy ground truth
 * (python/modern_fm/_reference.py, _reference_train.py), which the reference
 * specifies as bit-for-bit with its Rust engine at n_jobs=1.
 *
 * Conventions (all arrays float64 / int64, C-contiguous, as at the reference's
 * PyO3 boundary, rust/src/lib.rs:1-7):
 *   CSR: indptr[n_rows+1], indices[nnz], data[nnz]
 *   FM   V: (n_features, k)            FFM V: (n_features, n_fields, k)
 *   FwFM V: (n_features, k), R: (n_fields, n_fields) (upper triangle read)
 *   multiclass: w0 (C), w (C, n), V (C, n, ...), R (C, F, F)
 *   row_orders: (n_epochs, n_rows)
 * Optional state pointers are NULL when the owning optimizer is off.
 */
#ifndef MFM_ORACLE_H
#define MFM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_LOSS_LOGISTIC = 0, ORC_LOSS_SQUARED = 1 };
enum { ORC_OPT_SGD = 0, ORC_OPT_ADAGRAD = 1, ORC_OPT_ADAM = 2, ORC_OPT_FTRL = 3 };

/* Optimizer + hyperparameters (rust/src/optimizer.rs:6-17). */
typedef struct {
    int kind;          /* ORC_OPT_* */
    double lr;         /* learning_rate (FTRL: alpha) */
    double beta1, beta2, eps; /* Adam */
    double ftrl_beta;  /* FTRL stabilizer */
    double l1_linear, l2_linear, l1_factors, l2_factors;
} orc_opt;

/* State of one parameter group (theta array of length len):
 * acc = AdaGrad accumulator, (m, s, t) = Adam, (z, n) = FTRL.
 * Mirrors AdamStateMut / FtrlStateMut / GroupStateMut (optimizer.rs:177-320). */
typedef struct {
    double *acc, *m, *s, *t, *z, *n;
} orc_state;

/* ---- validation (rust/src/data.rs:14-44, 71-83) ---- */
/* Returns 0 on success, -1 with a message in err (size errlen) otherwise. */
int orc_check_csr(const int64_t* indptr, int64_t indptr_len, const int64_t* indices,
                  int64_t indices_len, int64_t data_len, int64_t n_cols, char* err,
                  int errlen);
int orc_check_field_ids(const int64_t* field_ids, int64_t len, int64_t n_features,
                        int64_t n_fields, char* err, int errlen);
/* _prep_csr (python/modern_fm/_backend.py:44-52): sort each row by column and
 * sum duplicate columns, stable order. Returns the canonical entry count. */
int64_t orc_prep_csr(int64_t n_rows, const int64_t* indptr, const int64_t* indices,
                     const double* data, int64_t* indptr_out, int64_t* indices_out,
                     double* data_out);

/* ---- prediction (serial per row in the reference; n_threads splits rows) ---- */
void orc_fm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                        int64_t n_rows, double w0, const double* w, const double* v,
                        int64_t k, double* out, int n_threads);
void orc_fm_predict_dense(const double* x, int64_t n_rows, int64_t n_features, double w0,
                          const double* w, const double* v, int64_t k, double* out);
void orc_ffm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                         int64_t n_rows, const int64_t* field_ids, double w0,
                         const double* w, const double* v, int64_t n_fields, int64_t k,
                         double* out, int n_threads);
void orc_ffm_predict_dense(const double* x, int64_t n_rows, int64_t n_features,
                           const int64_t* field_ids, double w0, const double* w,
                           const double* v, int64_t n_fields, int64_t k, double* out);
void orc_fwfm_predict_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                          int64_t n_rows, const int64_t* field_ids, double w0,
                          const double* w, const double* v, const double* r,
                          int64_t n_fields, int64_t k, double* out, int n_threads);
void orc_fwfm_predict_dense(const double* x, int64_t n_rows, int64_t n_features,
                            const int64_t* field_ids, double w0, const double* w,
                            const double* v, const double* r, int64_t n_fields, int64_t k,
                            double* out);

/* ---- training. Binary w0 + its state are scalars passed by pointer. ----
 * st_w0 / st_w / st_v / st_r: state for each parameter group (fields NULL
 * when unused). Returns 0, or -1 on allocation failure. */
int orc_fm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                   int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                   double* w0, double* w, double* v, int64_t k, orc_state st_w0,
                   orc_state st_w, orc_state st_v, int loss, const orc_opt* opt,
                   const int64_t* row_orders, int64_t n_epochs, int64_t batch_size,
                   int n_jobs);
int orc_ffm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                    int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                    const int64_t* field_ids, int64_t n_fields, double* w0, double* w,
                    double* v, int64_t k, orc_state st_w0, orc_state st_w, orc_state st_v,
                    int loss, const orc_opt* opt, const int64_t* row_orders,
                    int64_t n_epochs, int64_t batch_size, int n_jobs);
int orc_fwfm_fit_csr(const int64_t* indptr, const int64_t* indices, const double* data,
                     int64_t n_rows, int64_t n_features, const double* y, const double* sw,
                     const int64_t* field_ids, int64_t n_fields, double* w0, double* w,
                     double* v, double* r, int64_t k, orc_state st_w0, orc_state st_w,
                     orc_state st_v, orc_state st_r, int loss, const orc_opt* opt,
                     const int64_t* row_orders, int64_t n_epochs, int64_t batch_size);

/* Multiclass (softmax): all state arrays are (C, ...) row-major, y is int64. */
int orc_fm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                              const double* data, int64_t n_rows, int64_t n_features,
                              const int64_t* y, const double* sw, int64_t n_classes,
                              double* w0, double* w, double* v, int64_t k, orc_state st_w0,
                              orc_state st_w, orc_state st_v, const orc_opt* opt,
                              double label_smoothing, const int64_t* row_orders,
                              int64_t n_epochs, int64_t batch_size);
int orc_ffm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                               const double* data, int64_t n_rows, int64_t n_features,
                               const int64_t* y, const double* sw, int64_t n_classes,
                               const int64_t* field_ids, int64_t n_fields, double* w0,
                               double* w, double* v, int64_t k, orc_state st_w0,
                               orc_state st_w, orc_state st_v, const orc_opt* opt,
                               double label_smoothing, const int64_t* row_orders,
                               int64_t n_epochs, int64_t batch_size);
int orc_fwfm_fit_multiclass_csr(const int64_t* indptr, const int64_t* indices,
                                const double* data, int64_t n_rows, int64_t n_features,
                                const int64_t* y, const double* sw, int64_t n_classes,
                                const int64_t* field_ids, int64_t n_fields, double* w0,
                                double* w, double* v, double* r, int64_t k,
                                orc_state st_w0, orc_state st_w, orc_state st_v,
                                orc_state st_r, const orc_opt* opt, double label_smoothing,
                                const int64_t* row_orders, int64_t n_epochs,
                                int64_t batch_size);

/* Scalar optimizer primitives, exported for known-answer tests
 * (optimizer.rs:28-105). */
double orc_sigmoid(double s);
void orc_adam_step(double* theta, double g, double* m, double* v, double* t, double lr,
                   double b1, double b2, double eps);
void orc_ftrl_step(double* theta, double g, double* z, double* n, double alpha, double beta,
                   double l1, double l2);

#ifdef __cplusplus
}
#endif
#endif
