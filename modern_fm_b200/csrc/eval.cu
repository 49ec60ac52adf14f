// eval.cu — early-stopping evaluation on the device.
//
// The reference's estimators evaluate the validation set after every epoch
// of an early-stopped fit on the host: `metric(y_val, fm_predict_fast(X_val,
// w0, w, V))` (python/modern_fm/fm.py:321-322) with metric = logistic_loss or
// squared_loss (python/modern_fm/losses.py:25-42, 64-68), which needs the
// whole parameter set on the host each epoch; the FFM and FwFM estimators do
// the same with ffm_predict / fwfm_predict (python/modern_fm/ffm.py:210-212,
// python/modern_fm/fwfm.py:157-161). mfm_{fm,ffm,fwfm}_eval_device score a
// device-resident validation CSR with device-resident parameters and reduce
// the loss on the device; only the scalar comes back.
//
// The loss is accumulated in float64 in a fixed shape (kEvalBlocks x kEvalNT
// strided partial sums, a fixed xor tree per warp, warps and blocks added in
// index order), so the value is bitwise reproducible on any device. It equals
// NumPy's mean up to the order of the additions.
#include "common.cuh"

#include <algorithm>

namespace mfm {
namespace {

constexpr int kEvalBlocks = 592;  // fixed, not SM-derived: the summation shape
constexpr int kEvalNT = 256;

// Per-block partial sums of (per-sample loss x weight, weight).
template <class T>
__global__ void __launch_bounds__(kEvalNT)
    eval_loss_kernel(const T* __restrict__ score, const double* __restrict__ y,
                     const double* __restrict__ sw, int64_t n, int loss, double eps,
                     double* __restrict__ part) {
    __shared__ double sa[kEvalNT / 32], sb[kEvalNT / 32];
    double a = 0.0, b = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * kEvalNT + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * kEvalNT) {
        const double s = (double)score[i];
        double t = y[i], per;
        if (loss == MFM_LOSS_LOGISTIC) {
            // losses.py:39-41: smoothed target, stable binary cross-entropy
            if (eps != 0.0) t = t * (1.0 - eps) + 0.5 * eps;
            per = fmax(s, 0.0) - s * t + log1p(exp(-fabs(s)));
        } else {
            const double d = s - t;  // losses.py:68
            per = 0.5 * (d * d);
        }
        const double wt = sw ? sw[i] : 1.0;
        a += per * wt;
        b += wt;
    }
    a = warp_sum(a);
    b = warp_sum(b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sa[warp] = a;
        sb[warp] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double ta = 0.0, tb = 0.0;
        for (int i = 0; i < kEvalNT / 32; ++i) {
            ta += sa[i];
            tb += sb[i];
        }
        part[2 * blockIdx.x] = ta;
        part[2 * blockIdx.x + 1] = tb;
    }
}

// One thread adds the block partials in block order: sum(loss x w) / sum(w)
// (losses.py:25-28; without weights sum(w) is the row count, NumPy's mean).
__global__ void eval_final_kernel(const double* __restrict__ part, int nb,
                                  double* __restrict__ out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double a = 0.0, b = 0.0;
    for (int i = 0; i < nb; ++i) {
        a += part[2 * i];
        b += part[2 * i + 1];
    }
    out[0] = a / b;
}

// Scores the validation rows with `score` (a call of one of the
// mfm_*_predict_device entry points into the buffer it is given), then reduces
// the loss in the fixed shape above.
template <class T, class Score>
double eval_scores(int device, cudaStream_t s, int64_t n_rows, const double* y, const double* sw,
                   int loss, double eps, Score&& score) {
    DevBuf<T> buf(device, (size_t)n_rows);
    const int rc = score(buf.ptr);
    if (rc != MFM_OK) fail(rc, mfm_last_error());
    const int nb = (int)std::min<int64_t>(kEvalBlocks, ceil_div(n_rows, kEvalNT));
    DevBuf<double> part(device, 2 * (size_t)nb), res(device, 1);
    eval_loss_kernel<T><<<nb, kEvalNT, 0, s>>>(buf.ptr, y, sw, n_rows, loss, eps, part.ptr);
    eval_final_kernel<<<1, 32, 0, s>>>(part.ptr, nb, res.ptr);
    MFM_CHECK_LAUNCH("evaluation");
    double h = 0.0;
    d2h(&h, res.ptr, 1, s, "evaluation result");
    MFM_CUDA(cudaStreamSynchronize(s), "evaluation");
    return h;
}

// Shared argument checks and the float32 / float64 score-buffer choice.
template <class Score>
void eval_entry(int dtype, int device, const int64_t* indptr, int64_t n_rows, const double* y,
                const double* sample_weight, int loss, double label_smoothing, double* loss_out,
                void* stream, Score&& score) {
    if (!loss_out) fail(MFM_ERR_INVALID, "loss_out must be provided");
    if (loss != MFM_LOSS_LOGISTIC && loss != MFM_LOSS_SQUARED)
        fail(MFM_ERR_INVALID, fmt("unknown loss %d", loss));
    if (n_rows < 0) fail(MFM_ERR_INVALID, "negative CSR size");
    if (n_rows > 0 && (!indptr || !y)) fail(MFM_ERR_INVALID, "indptr and y must be provided");
    if (dtype != MFM_DTYPE_F32 && dtype != MFM_DTYPE_F64 && dtype != MFM_DTYPE_F32_F64)
        fail(MFM_ERR_INVALID, fmt("unknown dtype %d", dtype));
    if (n_rows == 0) {  // NumPy: the mean of no values is nan
        *loss_out = __builtin_nan("");
        return;
    }
    DeviceGuard g(device);
    cudaStream_t s = (cudaStream_t)stream;
    *loss_out = dtype == MFM_DTYPE_F32
                    ? eval_scores<float>(device, s, n_rows, y, sample_weight, loss,
                                         label_smoothing, score)
                    : eval_scores<double>(device, s, n_rows, y, sample_weight, loss,
                                          label_smoothing, score);
}

}  // namespace
}  // namespace mfm

using namespace mfm;

extern "C" int mfm_fm_eval_device(int dtype, int device, const int64_t* indptr,
                                  const int32_t* indices, const void* data, int64_t n_rows,
                                  double w0, const void* w, const void* v, int64_t k,
                                  const double* y, const double* sample_weight, int loss,
                                  double label_smoothing, double* loss_out, void* stream) {
    return guarded([&] {
        eval_entry(dtype, device, indptr, n_rows, y, sample_weight, loss, label_smoothing,
                   loss_out, stream, [&](void* out) {
                       return mfm_fm_predict_device(dtype, device, indptr, indices, data, n_rows,
                                                    w0, w, v, k, out, stream);
                   });
    });
}

extern "C" int mfm_ffm_eval_device(int dtype, int device, const int64_t* indptr,
                                   const int32_t* indices, const void* data, int64_t n_rows,
                                   const int32_t* field_ids, int64_t n_fields, double w0,
                                   const void* w, const void* v, int64_t k, const double* y,
                                   const double* sample_weight, int loss,
                                   double label_smoothing, double* loss_out, void* stream) {
    return guarded([&] {
        eval_entry(dtype, device, indptr, n_rows, y, sample_weight, loss, label_smoothing,
                   loss_out, stream, [&](void* out) {
                       return mfm_ffm_predict_device(dtype, device, indptr, indices, data,
                                                     n_rows, field_ids, n_fields, w0, w, v, k,
                                                     out, stream);
                   });
    });
}

extern "C" int mfm_fwfm_eval_device(int dtype, int device, const int64_t* indptr,
                                    const int32_t* indices, const void* data, int64_t n_rows,
                                    const int32_t* field_ids, int64_t n_fields, double w0,
                                    const void* w, const void* v, const void* r, int64_t k,
                                    const double* y, const double* sample_weight, int loss,
                                    double label_smoothing, double* loss_out, void* stream) {
    return guarded([&] {
        eval_entry(dtype, device, indptr, n_rows, y, sample_weight, loss, label_smoothing,
                   loss_out, stream, [&](void* out) {
                       return mfm_fwfm_predict_device(dtype, device, indptr, indices, data,
                                                      n_rows, field_ids, n_fields, w0, w, v, r,
                                                      k, out, stream);
                   });
    });
}
