/*
 * mfm_b200.h — C ABI of the B200-native (sm_100a) modern_fm engine:
 * sparse-CSR FM / FFM / FwFM scoring and mini-batch training (binary and
 * multiclass softmax) on NVIDIA B200.
 *
 * This ABI replaces the reference's CUDA backend entry points (modern_fm
 * v1.1.1, Rust crate `modern-fm`). Each function names the reference
 * interface it stands in for. Plain pointers and sizes only: every array is a
 * HOST array in the reference's boundary format (float64 values, int64
 * indices, C-contiguous; rust/src/lib.rs:1-7) unless the name says `_device`.
 *
 * Return codes: 0 = success; < 0 = invalid input (the reference raises
 * ValueError, rust/src/lib.rs:30-32); > 0 = CUDA / device failure (the
 * reference raises RuntimeError from predict, lib.rs:1510-1512, and ValueError
 * from fit, lib.rs:437). The message is in mfm_last_error() (thread-local).
 * No entry point falls back to a CPU path.
 */
#ifndef MFM_B200_H
#define MFM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MFM_OK 0
#define MFM_ERR_INVALID (-1)     /* bad shapes / CSR / ids / hyperparameters */
#define MFM_ERR_UNSUPPORTED (-2) /* valid but outside this engine's limits (e.g. k > 1024) */
#define MFM_ERR_CUDA 1           /* a CUDA runtime call failed */
#define MFM_ERR_NO_DEVICE 2      /* no usable CUDA device */
#define MFM_ERR_DEVICE_CHECK 3   /* a kernel's own bounds / status check fired */

/* Compute types. MFM_DTYPE_F64: float64 parameters, values, arithmetic and
 * scores (the reference's own arithmetic, rust/src/lib.rs:1-7). MFM_DTYPE_F32:
 * float32 throughout (half the bytes of every gather). MFM_DTYPE_F32_F64:
 * float32 parameters, float64 values, arithmetic and scores — what the
 * reference computes for an estimator whose learned attributes are float32
 * (its default, python/modern_fm/fm.py:655-658: the attributes are widened to
 * float64 before its float64 kernels). Where parameters arrive as float64
 * host arrays, F32_F64 stores them as float32 only when every value is exactly
 * a float32 (checked on the device) and otherwise keeps float64, so its
 * result is always the float64 arithmetic on the caller's values. Training
 * keeps float64 parameters for the whole fit in F32_F64, as the reference
 * does (python/modern_fm/_backend.py:116-130). */
enum { MFM_DTYPE_F64 = 0, MFM_DTYPE_F32 = 1, MFM_DTYPE_F32_F64 = 2 };
enum { MFM_MODEL_FM = 0, MFM_MODEL_FFM = 1, MFM_MODEL_FWFM = 2 };
enum { MFM_LOSS_LOGISTIC = 0, MFM_LOSS_SQUARED = 1 };
enum { MFM_OPT_SGD = 0, MFM_OPT_ADAGRAD = 1, MFM_OPT_ADAM = 2, MFM_OPT_FTRL = 3 };

/* CSR matrix (scipy indptr/indices/data), host memory.
 * Stands in for CsrView (rust/src/data.rs:7-11). */
typedef struct {
    const int64_t* indptr;  /* n_rows + 1 */
    const int64_t* indices; /* nnz */
    const double* data;     /* nnz */
    int64_t n_rows;
    int64_t nnz;
    int64_t n_features;
} mfm_csr;

/* Execution options. dtype (MFM_DTYPE_*) selects the device storage and
 * arithmetic types of parameters, sums and optimizer state. device is the
 * first CUDA ordinal; predict shards rows over n_devices devices. */
typedef struct {
    int dtype;
    int device;
    int n_devices;
} mfm_exec;

/* Training configuration: the scalar arguments of the reference's fit entry
 * points (rust/src/lib.rs:283-322) plus row_orders (n_epochs, n_rows). */
typedef struct {
    int loss;      /* MFM_LOSS_* (binary only) */
    int optimizer; /* MFM_OPT_* */
    double learning_rate, l1_linear, l2_linear, l1_factors, l2_factors;
    double beta_1, beta_2, epsilon, ftrl_beta, label_smoothing;
    const int64_t* row_orders;
    int64_t n_epochs;
    int64_t batch_size;
} mfm_train;

/* One parameter group (w0, w, V or R) and its optimizer state, all read and
 * written in place. acc = AdaGrad accumulator; (m, s, t) = Adam; (z, n) =
 * FTRL. A NULL state pointer means "not provided": the engine keeps a zeroed
 * device-side state for the duration of the call, exactly as the reference
 * does with its local_state (rust/src/lib.rs:79-87). For binary models the w0
 * group points at scalars. */
typedef struct {
    double* param;
    double* acc;
    double* m;
    double* s;
    double* t;
    double* z;
    double* n;
} mfm_group;

/* Replaces cuda::available() / has_cuda (rust/src/cuda/mod.rs:38-44,
 * rust/src/lib.rs:1471-1482): 1 when a CUDA device is usable. */
int mfm_has_cuda(void);

/* Thread-local message for the last non-zero return code. */
const char* mfm_last_error(void);

/* Number of CUDA devices visible to the process (0 when none). */
int mfm_device_count(void);

/* ---- prediction (transfer-inclusive, like the reference) ---------------- */

/* Replaces fm_predict_cuda_csr -> cuda::fm::predict_csr
 * (rust/src/lib.rs:1488-1513, rust/src/cuda/fm.rs:61-109).
 * w: (n_features), v: (n_features, k), out: (n_rows). */
int mfm_fm_predict_csr(const mfm_csr* x, double w0, const double* w, const double* v,
                       int64_t k, double* out, const mfm_exec* ex);

/* Replaces ffm_predict_cuda_csr -> cuda::ffm::predict_csr
 * (rust/src/lib.rs:1519-1548, rust/src/cuda/ffm.rs:81-136).
 * field_ids: (n_features), v: (n_features, n_fields, k). */
int mfm_ffm_predict_csr(const mfm_csr* x, const int64_t* field_ids, int64_t n_fields,
                        double w0, const double* w, const double* v, int64_t k, double* out,
                        const mfm_exec* ex);

/* Replaces fwfm_predict_cuda_csr -> cuda::fwfm::predict_csr
 * (rust/src/lib.rs:1554-1590, rust/src/cuda/fwfm.rs:77-135).
 * v: (n_features, k), r: (n_fields, n_fields), upper triangle read. */
int mfm_fwfm_predict_csr(const mfm_csr* x, const int64_t* field_ids, int64_t n_fields,
                         double w0, const double* w, const double* v, const double* r,
                         int64_t k, double* out, const mfm_exec* ex);

/* ---- training (whole fit call device-resident) --------------------------- */

/* Replaces fm_fit_csr(use_cuda=True) -> cuda::fm_train::fit_csr
 * (rust/src/lib.rs:283-439, rust/src/cuda/fm_train.rs:175-444).
 * Groups: w0 (scalar), w (n_features), v (n_features, k). */
int mfm_fm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                   const mfm_train* tr, int64_t k, mfm_group* w0, mfm_group* w, mfm_group* v,
                   const mfm_exec* ex);

/* Replaces fm_fit_multiclass_csr(use_cuda=True) -> cuda::fm_train_mc
 * (rust/src/lib.rs:449-630, rust/src/cuda/fm_train_mc.rs:163-472).
 * y: class ids (n_rows). Groups: w0 (C), w (C, n_features), v (C, n_features, k). */
int mfm_fm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                              const double* sample_weight, int64_t n_classes,
                              const mfm_train* tr, int64_t k, mfm_group* w0, mfm_group* w,
                              mfm_group* v, const mfm_exec* ex);

/* Replaces ffm_fit_csr(use_cuda=True) -> cuda::ffm_train::fit_csr
 * (rust/src/lib.rs:635-793, rust/src/cuda/ffm_train.rs:197-436).
 * v: (n_features, n_fields, k). */
int mfm_ffm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                    const int64_t* field_ids, int64_t n_fields, const mfm_train* tr,
                    int64_t k, mfm_group* w0, mfm_group* w, mfm_group* v,
                    const mfm_exec* ex);

/* Replaces ffm_fit_multiclass_csr(use_cuda=True) -> cuda::ffm_train_mc
 * (rust/src/lib.rs:800-978, rust/src/cuda/ffm_train_mc.rs:198-515).
 * v: (C, n_features, n_fields, k). */
int mfm_ffm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                               const double* sample_weight, int64_t n_classes,
                               const int64_t* field_ids, int64_t n_fields,
                               const mfm_train* tr, int64_t k, mfm_group* w0, mfm_group* w,
                               mfm_group* v, const mfm_exec* ex);

/* Replaces fwfm_fit_csr(use_cuda=True) -> cuda::fwfm_train::fit_csr
 * (rust/src/lib.rs:1049-1242, rust/src/cuda/fwfm_train.rs:314-610).
 * v: (n_features, k), r: (n_fields, n_fields). */
int mfm_fwfm_fit_csr(const mfm_csr* x, const double* y, const double* sample_weight,
                     const int64_t* field_ids, int64_t n_fields, const mfm_train* tr,
                     int64_t k, mfm_group* w0, mfm_group* w, mfm_group* v, mfm_group* r,
                     const mfm_exec* ex);

/* Replaces fwfm_fit_multiclass_csr(use_cuda=True) -> cuda::fwfm_train
 * (rust/src/lib.rs:1249-1466, rust/src/cuda/fwfm_train.rs:615-955).
 * v: (C, n_features, k), r: (C, n_fields, n_fields). */
int mfm_fwfm_fit_multiclass_csr(const mfm_csr* x, const int64_t* y,
                                const double* sample_weight, int64_t n_classes,
                                const int64_t* field_ids, int64_t n_fields,
                                const mfm_train* tr, int64_t k, mfm_group* w0, mfm_group* w,
                                mfm_group* v, mfm_group* r, const mfm_exec* ex);

/* ---- device-resident prediction (no reference counterpart) -------------
 * Every pointer is DEVICE memory on `device`, already in the compute layout:
 * indptr int64 (n_rows+1), indices int32, data/w/v/r/out in `dtype`
 * (MFM_DTYPE_F32: all float; MFM_DTYPE_F64: all double; MFM_DTYPE_F32_F64:
 * w/v/r float, data and out double). `stream` is a cudaStream_t (NULL = legacy default).
 * No host<->device copies, no allocation, no validation beyond sizes: the
 * caller guarantees the CSR is canonical and in range. Used for
 * device-resident throughput and by callers that keep data on the GPU. */
int mfm_fm_predict_device(int dtype, int device, const int64_t* indptr,
                          const int32_t* indices, const void* data, int64_t n_rows,
                          double w0, const void* w, const void* v, int64_t k, void* out,
                          void* stream);
int mfm_ffm_predict_device(int dtype, int device, const int64_t* indptr,
                           const int32_t* indices, const void* data, int64_t n_rows,
                           const int32_t* field_ids, int64_t n_fields, double w0,
                           const void* w, const void* v, int64_t k, void* out, void* stream);
int mfm_fwfm_predict_device(int dtype, int device, const int64_t* indptr,
                            const int32_t* indices, const void* data, int64_t n_rows,
                            const int32_t* field_ids, int64_t n_fields, double w0,
                            const void* w, const void* v, const void* r, int64_t k, void* out,
                            void* stream);

/* ---- device-side CSR canonicalisation ------------------------------------
 * Replaces the host canonicalisation the reference runs before every native
 * call, `_prep_csr` (python/modern_fm/_backend.py:44-52: float64 cast, scipy
 * sum_duplicates, int64 / float64 copies), and the O(nnz) part of its CSR
 * validation (CsrView::new, rust/src/data.rs:14-44). Input: a DEVICE CSR on
 * `device` in the boundary format (indptr int64 (n_rows+1), indices int64,
 * data float64), rows in any column order, duplicate (row, column) entries
 * allowed. Output (caller-owned DEVICE buffers of n_rows+1 / nnz / nnz
 * entries): the canonical CSR in the compute layout the *_device entry points
 * take: columns sorted within each row, duplicates summed in float64 in their
 * original order (explicit zeros kept), indices int32, data in `dtype`
 * (float64 for MFM_DTYPE_F32_F64).
 * *nnz_out (host) receives the canonical entry count. Invalid CSR structure or
 * a column outside [0, n_features) returns MFM_ERR_INVALID with the
 * reference's message. Runs on `stream` (a cudaStream_t) and synchronises it. */
int mfm_csr_prep_device(int dtype, int device, int64_t n_rows, int64_t n_features, int64_t nnz,
                        const int64_t* indptr, const int64_t* indices, const double* data,
                        int64_t* indptr_out, int32_t* indices_out, void* data_out,
                        int64_t* nnz_out, void* stream);

/* ---- libffm text reader ---------------------------------------------------
 * Replaces the reading half of the reference's load_libffm
 * (python/modern_fm/libffm.py:31-83): parses a libffm file
 * (`<label> <field>:<feature>:<value> ...` per line) on the host with
 * n_threads threads (<= 0: every core) into a raw CSR in the boundary format:
 * rows in file order, entries in token order, duplicates kept (the reference
 * sums them when it builds its CSR; mfm_csr_prep_device does that on the
 * device), float64 labels, and an int64 field id per feature (n_features =
 * largest feature + 1; features never seen get field 0, as in the reference).
 * Values are correctly rounded, as Python's float() reads them. Errors return
 * MFM_ERR_INVALID with the reference's messages and line numbers ("path:line:
 * bad token ...; expected field:feature:value", "negative field/feature in",
 * "feature F maps to fields A and B", "could not convert string to float");
 * features beyond 2^31-1 return MFM_ERR_UNSUPPORTED. The arrays belong to the
 * handle: mfm_libffm_arrays gives pointers valid until mfm_libffm_free. */
typedef struct mfm_libffm mfm_libffm;
int mfm_libffm_read(const char* path, int n_threads, mfm_libffm** out);
int mfm_libffm_info(const mfm_libffm* f, int64_t* n_rows, int64_t* nnz, int64_t* n_features);
int mfm_libffm_arrays(const mfm_libffm* f, const int64_t** indptr, const int64_t** indices,
                      const double** data, const double** y, const int64_t** field_ids);
void mfm_libffm_free(mfm_libffm* f);

/* ---- early-stopping evaluation on the device -----------------------------
 * Replaces the host evaluation the reference's early-stopped FM fits run after
 * every epoch, `metric(y_val, fm_predict_fast(X_val, w0, w, V))`
 * (python/modern_fm/fm.py:321-322) with logistic_loss (label smoothing
 * applied to the target) or squared_loss (python/modern_fm/losses.py:25-42,
 * 64-68). The validation CSR and the parameters are DEVICE arrays in the
 * compute layout of mfm_fm_predict_device; y and sample_weight are float64
 * DEVICE arrays (sample_weight NULL = unweighted mean). The loss is reduced in
 * float64 on the device in a fixed order (bitwise reproducible) and written to
 * *loss_out (host); n_rows = 0 gives NaN, as NumPy's mean of nothing. */
int mfm_fm_eval_device(int dtype, int device, const int64_t* indptr, const int32_t* indices,
                       const void* data, int64_t n_rows, double w0, const void* w, const void* v,
                       int64_t k, const double* y, const double* sample_weight, int loss,
                       double label_smoothing, double* loss_out, void* stream);

/* The same evaluation for the FFM and FwFM estimators' early-stopped fits,
 * which score the validation set with ffm_predict / fwfm_predict on the host
 * every epoch (python/modern_fm/ffm.py:210-212, python/modern_fm/fwfm.py:157-161).
 * Parameters and field ids as in mfm_ffm_predict_device /
 * mfm_fwfm_predict_device. */
int mfm_ffm_eval_device(int dtype, int device, const int64_t* indptr, const int32_t* indices,
                        const void* data, int64_t n_rows, const int32_t* field_ids,
                        int64_t n_fields, double w0, const void* w, const void* v, int64_t k,
                        const double* y, const double* sample_weight, int loss,
                        double label_smoothing, double* loss_out, void* stream);
int mfm_fwfm_eval_device(int dtype, int device, const int64_t* indptr, const int32_t* indices,
                         const void* data, int64_t n_rows, const int32_t* field_ids,
                         int64_t n_fields, double w0, const void* w, const void* v,
                         const void* r, int64_t k, const double* y,
                         const double* sample_weight, int loss, double label_smoothing,
                         double* loss_out, void* stream);

/* ---- persistent model handle ----------------------------------------------
 * The reference uploads the parameters on every CUDA predict call
 * (rust/src/cuda/mod.rs:9-12, rust/src/cuda/fm.rs:61-109) and scores a
 * multiclass model with one binary call per class, each re-uploading X
 * (python/modern_fm/fm.py:666-674, `decision_function`). A handle keeps one
 * model's parameters resident on `device` across calls and scores every class
 * of a row in one pass.
 *   mfm_model_create: kind MFM_MODEL_*, dtype MFM_DTYPE_*, n_fields (FFM /
 *     FwFM), k, n_classes (1 = binary: one score per row; C >= 2: C logits per
 *     row, each the binary score with class c's parameters).
 *   mfm_model_set_params: parameters in the reference's boundary layout,
 *     float64 host arrays: binary w0 (scalar), w (n), V (n, k) or FFM
 *     (n, F, k), R (F, F); multiclass class-major w0 (C), w (C, n),
 *     V (C, n, k) or FFM (C, n, F, k), R (C, F, F); field_ids int64 (n) for
 *     FFM / FwFM (NULL for FM). Uploaded once (key-major on the device).
 *   mfm_model_info: the compute type the handle scores in (F32_F64 falls back
 *     to F64 when the parameters are not exactly float32).
 *   mfm_model_predict_csr: host CSR in the boundary format, validated as
 *     mfm_fm_predict_csr does; out (n_rows) or (n_rows, C) float64.
 *   mfm_model_predict_device: DEVICE CSR in the compute layout (indptr int64,
 *     indices int32, canonical and in range); data and out float32 for
 *     MFM_DTYPE_F32, float64 otherwise; on `stream` (a cudaStream_t), no
 *     allocation, no synchronisation.
 *   mfm_model_free: releases the device copies. */
typedef struct mfm_model mfm_model;
int mfm_model_create(int kind, int dtype, int device, int64_t n_features, int64_t n_fields,
                     int64_t k, int64_t n_classes, mfm_model** out);
int mfm_model_set_params(mfm_model* m, const double* w0, const double* w, const double* v,
                         const double* r, const int64_t* field_ids);
int mfm_model_info(const mfm_model* m, int* dtype_used);
int mfm_model_predict_csr(mfm_model* m, const mfm_csr* x, double* out);
int mfm_model_predict_device(mfm_model* m, const int64_t* indptr, const int32_t* indices,
                             const void* data, int64_t n_rows, void* out, void* stream);
void mfm_model_free(mfm_model* m);

/* ---- allocation-free FM scoring --------------------------------------------
 * No counterpart in the reference: an addition for callers that cannot let
 * the library allocate GPU memory, such as a host that owns the whole device
 * budget through its own pool, or a latency-bound serving loop that cannot
 * afford cudaMalloc / cudaFree (they may synchronise the device and stall
 * every stream). Same arguments, results and errors as mfm_fm_predict_csr on
 * ex->device (n_devices is ignored), but the CSR, parameters, validation flags
 * and scores are staged in one static device array of
 * mfm_noalloc_scratch_bytes() bytes (64 MiB) that every GPU loading this
 * library holds until the process exits; no cudaMalloc, cudaFree or other
 * allocating routine is called. Inputs whose staging does not fit return
 * MFM_ERR_UNSUPPORTED before any device work. The first call on a device
 * loads the array's code module (the CUDA runtime loads modules lazily), which
 * reserves the 64 MiB on that device, and looks up the array's device address
 * (cudaGetSymbolAddress): make that first call before reserving the rest of
 * the device for a pool, and before any stream capture. Calls run on the
 * engine's own non-blocking stream for the device and synchronise it. Calls
 * share the array: each call clears the flags it needs, and calls that overlap
 * on the GPU race on the array (the engine serialises calls on one device
 * within a process). MFM_DTYPE_F32_F64 computes as MFM_DTYPE_F64 here. */
int mfm_fm_predict_csr_noalloc(const mfm_csr* x, double w0, const double* w, const double* v,
                               int64_t k, double* out, const mfm_exec* ex);

/* Size in bytes of the static array behind mfm_fm_predict_csr_noalloc. */
int64_t mfm_noalloc_scratch_bytes(void);

/* ---- device-resident training (no reference counterpart) -----------------
 * Binary FM training over caller-owned DEVICE arrays on `device`: indptr
 * int64 (n_rows+1), indices int32, data / y / sample_weight / parameters /
 * state in `dtype`; row_orders int32 (tr->n_epochs, n_rows) on the device
 * (tr->row_orders is ignored). Hyperparameters, n_epochs and batch_size come
 * from *tr. Parameters and state are updated in place on the device; a NULL
 * state pointer means a zeroed state local to the call. The caller guarantees
 * a canonical, in-range CSR. Runs on `stream` (a cudaStream_t). */
typedef struct {
    void* param;
    void* acc;
    void* m;
    void* s;
    void* t;
    void* z;
    void* n;
} mfm_dev_group;

int mfm_fm_fit_device(int dtype, int device, const int64_t* indptr, const int32_t* indices,
                      const void* data, int64_t n_rows, int64_t n_features, const void* y,
                      const void* sample_weight, const int32_t* row_orders,
                      const mfm_train* tr, int64_t k, mfm_dev_group* w0, mfm_dev_group* w,
                      mfm_dev_group* v, void* stream);

/* ---- data-parallel training (no reference counterpart) -------------------
 * Synchronous multi-GPU training with the one-GPU mini-batch semantics (the
 * same row_orders chunking, every batch's step equal to a one-GPU step up to
 * summation order); every rank holds the whole training set. Two exchanges:
 *   binary FM with k = 2, 4, 8, 16 (float64) or 4, 8, 16, 32 (float32), the
 *     row-table path: parameter-sharded by key. Rank r owns the keys with
 *     key mod world = r (parameters and optimizer state stepped there only)
 *     and scores every row of each batch over its own keys; the ranks sum
 *     the batch's row table (rows x (k + 1) values) with one ncclAllReduce
 *     (or, with MFM_B200_DP_EXCHANGE=peer, the forward kernel reads the other
 *     ranks' rows over NVLink through CUDA IPC mappings, with bounded flag
 *     waits; every rank must run the same GPU model); after the fit one sum
 *     over the ranks gives every rank every key. MFM_B200_DP_MODE=runs selects
 *     the second exchange instead;
 *   every other shape (FFM, FwFM, multiclass, other k): parameters
 *     replicated; each global batch is cut into `world` contiguous row
 *     slices, rank r scores slice r, the per-key gradient sums over the
 *     batch's sorted union of touched keys are summed with one
 *     ncclAllReduce, and every rank applies the identical optimizer step.
 * NCCL is loaded on first use (dlopen "libnccl.so.2"). A rank that stops
 * answering ends the other ranks' fits with an error after
 * MFM_B200_DP_TIMEOUT seconds (default 300); the group must then be recreated.
 *   mfm_dp_unique_id: rank 0 makes the group id (128 bytes) and the caller
 *     hands it to every rank;
 *   mfm_dp_create: every rank, concurrently; binds the group to `device`;
 *   mfm_dp_destroy: after the last fit. */
typedef struct mfm_dp mfm_dp;
int mfm_dp_unique_id(unsigned char id[128]);
int mfm_dp_create(const unsigned char id[128], int world, int rank, int device, mfm_dp** out);
int mfm_dp_destroy(mfm_dp* dp);

/* mfm_fm_fit_device across the group (same arguments; the device is the
 * group's). Every rank must call it with the same data, row orders, initial
 * parameters and hyperparameters; results are identical on every rank. */
int mfm_fm_fit_device_dp(mfm_dp* dp, int dtype, const int64_t* indptr, const int32_t* indices,
                         const void* data, int64_t n_rows, int64_t n_features, const void* y,
                         const void* sample_weight, const int32_t* row_orders,
                         const mfm_train* tr, int64_t k, mfm_dev_group* w0, mfm_dev_group* w,
                         mfm_dev_group* v, void* stream);

/* Any fit of the host-buffer entry points above — FM, FFM or FwFM
 * (model = MFM_MODEL_*), binary (n_classes = 1: y, float64 labels) or
 * multiclass softmax (n_classes = C >= 2: ycls, class ids) — run as one
 * data-parallel fit across the group: the same arguments, layouts, in-place
 * updates and results as mfm_fm_fit_csr / mfm_fm_fit_multiclass_csr /
 * mfm_ffm_fit_csr / mfm_ffm_fit_multiclass_csr / mfm_fwfm_fit_csr /
 * mfm_fwfm_fit_multiclass_csr on the group's device (field_ids / n_fields for
 * FFM and FwFM, r for FwFM; NULL otherwise). Every rank calls it with the
 * same data, row orders, initial parameters and hyperparameters (either
 * exchange above, by shape), so every rank ends with the same parameters,
 * equal to a one-GPU fit up to summation order. No reference counterpart (the
 * reference trains on one device). */
int mfm_fit_csr_dp(mfm_dp* dp, int dtype, int model, int64_t n_classes, const mfm_csr* x,
                   const double* y, const int64_t* ycls, const double* sample_weight,
                   const int64_t* field_ids, int64_t n_fields, const mfm_train* tr, int64_t k,
                   mfm_group* w0, mfm_group* w, mfm_group* v, mfm_group* r);

/* Device time (seconds, CUDA events) of the calling thread's last fit, by
 * phase: out[0] uploads and setup, out[1] the epochs' plans (sorts), out[2]
 * the epochs' batches, out[3] the download of parameters and state. No
 * reference counterpart (diagnostics). */
void mfm_fit_phase_seconds(double out[4]);

/* Release the engine's cached device memory on every device. */
void mfm_release_cached_memory(void);

#ifdef __cplusplus
}
#endif
#endif
