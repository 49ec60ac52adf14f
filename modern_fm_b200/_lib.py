"""ctypes binding of libmfm_b200.so (the C ABI declared in include/mfm_b200.h).

Loading fails loudly: there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes as ct
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmfm_b200.so")

MFM_OK = 0
MFM_ERR_INVALID, MFM_ERR_UNSUPPORTED = -1, -2
MFM_DTYPE_F64, MFM_DTYPE_F32, MFM_DTYPE_F32_F64 = 0, 1, 2
MFM_MODEL_FM, MFM_MODEL_FFM, MFM_MODEL_FWFM = 0, 1, 2
DTYPES = {"float64": MFM_DTYPE_F64, "f64": MFM_DTYPE_F64, "float32": MFM_DTYPE_F32,
          "f32": MFM_DTYPE_F32, "float32-float64": MFM_DTYPE_F32_F64,
          "f32-f64": MFM_DTYPE_F32_F64, "f32_f64": MFM_DTYPE_F32_F64}
LOSSES = {"logistic": 0, "squared": 1}
OPTIMIZERS = {"sgd": 0, "adagrad": 1, "adam": 2, "ftrl": 3}

i64p = ct.POINTER(ct.c_int64)
i32p = ct.POINTER(ct.c_int32)
f64p = ct.POINTER(ct.c_double)


class Csr(ct.Structure):
    _fields_ = [("indptr", i64p), ("indices", i64p), ("data", f64p), ("n_rows", ct.c_int64),
                ("nnz", ct.c_int64), ("n_features", ct.c_int64)]


class Exec(ct.Structure):
    _fields_ = [("dtype", ct.c_int), ("device", ct.c_int), ("n_devices", ct.c_int)]


class Train(ct.Structure):
    _fields_ = [("loss", ct.c_int), ("optimizer", ct.c_int), ("learning_rate", ct.c_double),
                ("l1_linear", ct.c_double), ("l2_linear", ct.c_double),
                ("l1_factors", ct.c_double), ("l2_factors", ct.c_double),
                ("beta_1", ct.c_double), ("beta_2", ct.c_double), ("epsilon", ct.c_double),
                ("ftrl_beta", ct.c_double), ("label_smoothing", ct.c_double),
                ("row_orders", i64p), ("n_epochs", ct.c_int64), ("batch_size", ct.c_int64)]


class Group(ct.Structure):
    _fields_ = [(n, f64p) for n in ("param", "acc", "m", "s", "t", "z", "n")]


class DevGroup(ct.Structure):
    """mfm_dev_group: device pointers (integers) in the compute dtype."""
    _fields_ = [(n, ct.c_void_p) for n in ("param", "acc", "m", "s", "t", "z", "n")]


_SIGNATURES = {
    "mfm_has_cuda": (ct.c_int, []),
    "mfm_last_error": (ct.c_char_p, []),
    "mfm_device_count": (ct.c_int, []),
    "mfm_release_cached_memory": (None, []),
    "mfm_fm_predict_csr": (ct.c_int, [ct.POINTER(Csr), ct.c_double, f64p, f64p, ct.c_int64,
                                      f64p, ct.POINTER(Exec)]),
    "mfm_ffm_predict_csr": (ct.c_int, [ct.POINTER(Csr), i64p, ct.c_int64, ct.c_double, f64p,
                                       f64p, ct.c_int64, f64p, ct.POINTER(Exec)]),
    "mfm_fwfm_predict_csr": (ct.c_int, [ct.POINTER(Csr), i64p, ct.c_int64, ct.c_double, f64p,
                                        f64p, f64p, ct.c_int64, f64p, ct.POINTER(Exec)]),
    "mfm_fm_fit_csr": (ct.c_int, [ct.POINTER(Csr), f64p, f64p, ct.POINTER(Train), ct.c_int64]
                       + [ct.POINTER(Group)] * 3 + [ct.POINTER(Exec)]),
    "mfm_fm_fit_multiclass_csr": (ct.c_int, [ct.POINTER(Csr), i64p, f64p, ct.c_int64,
                                             ct.POINTER(Train), ct.c_int64]
                                  + [ct.POINTER(Group)] * 3 + [ct.POINTER(Exec)]),
    "mfm_ffm_fit_csr": (ct.c_int, [ct.POINTER(Csr), f64p, f64p, i64p, ct.c_int64,
                                   ct.POINTER(Train), ct.c_int64]
                        + [ct.POINTER(Group)] * 3 + [ct.POINTER(Exec)]),
    "mfm_ffm_fit_multiclass_csr": (ct.c_int, [ct.POINTER(Csr), i64p, f64p, ct.c_int64, i64p,
                                              ct.c_int64, ct.POINTER(Train), ct.c_int64]
                                   + [ct.POINTER(Group)] * 3 + [ct.POINTER(Exec)]),
    "mfm_fwfm_fit_csr": (ct.c_int, [ct.POINTER(Csr), f64p, f64p, i64p, ct.c_int64,
                                    ct.POINTER(Train), ct.c_int64]
                         + [ct.POINTER(Group)] * 4 + [ct.POINTER(Exec)]),
    "mfm_fwfm_fit_multiclass_csr": (ct.c_int, [ct.POINTER(Csr), i64p, f64p, ct.c_int64, i64p,
                                               ct.c_int64, ct.POINTER(Train), ct.c_int64]
                                    + [ct.POINTER(Group)] * 4 + [ct.POINTER(Exec)]),
    "mfm_fm_fit_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                     ct.c_int64, ct.c_int64, ct.c_void_p, ct.c_void_p,
                                     ct.c_void_p, ct.POINTER(Train), ct.c_int64]
                          + [ct.POINTER(DevGroup)] * 3 + [ct.c_void_p]),
    "mfm_dp_unique_id": (ct.c_int, [ct.c_char_p]),
    "mfm_dp_create": (ct.c_int, [ct.c_char_p, ct.c_int, ct.c_int, ct.c_int,
                                 ct.POINTER(ct.c_void_p)]),
    "mfm_dp_destroy": (ct.c_int, [ct.c_void_p]),
    "mfm_fm_fit_device_dp": (ct.c_int, [ct.c_void_p, ct.c_int, ct.c_void_p, ct.c_void_p,
                                        ct.c_void_p, ct.c_int64, ct.c_int64, ct.c_void_p,
                                        ct.c_void_p, ct.c_void_p, ct.POINTER(Train), ct.c_int64]
                             + [ct.POINTER(DevGroup)] * 3 + [ct.c_void_p]),
    "mfm_fit_csr_dp": (ct.c_int, [ct.c_void_p, ct.c_int, ct.c_int, ct.c_int64, ct.POINTER(Csr),
                                  f64p, i64p, f64p, i64p, ct.c_int64, ct.POINTER(Train),
                                  ct.c_int64] + [ct.POINTER(Group)] * 4),
    "mfm_fit_phase_seconds": (None, [ct.POINTER(ct.c_double)]),
    "mfm_csr_prep_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_int64, ct.c_int64, ct.c_int64,
                                       ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                       ct.c_void_p, ct.c_void_p, i64p, ct.c_void_p]),
    "mfm_fm_eval_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                      ct.c_int64, ct.c_double, ct.c_void_p, ct.c_void_p,
                                      ct.c_int64, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_double,
                                      f64p, ct.c_void_p]),
    "mfm_ffm_eval_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p,
                                       ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_int64,
                                       ct.c_double, ct.c_void_p, ct.c_void_p, ct.c_int64,
                                       ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_double, f64p,
                                       ct.c_void_p]),
    "mfm_fwfm_eval_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p,
                                        ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_int64,
                                        ct.c_double, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                        ct.c_int64, ct.c_void_p, ct.c_void_p, ct.c_int,
                                        ct.c_double, f64p, ct.c_void_p]),
    "mfm_model_create": (ct.c_int, [ct.c_int, ct.c_int, ct.c_int, ct.c_int64, ct.c_int64,
                                    ct.c_int64, ct.c_int64, ct.POINTER(ct.c_void_p)]),
    "mfm_model_set_params": (ct.c_int, [ct.c_void_p, f64p, f64p, f64p, f64p, i64p]),
    "mfm_model_info": (ct.c_int, [ct.c_void_p, ct.POINTER(ct.c_int)]),
    "mfm_model_predict_csr": (ct.c_int, [ct.c_void_p, ct.POINTER(Csr), f64p]),
    "mfm_model_predict_device": (ct.c_int, [ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                            ct.c_int64, ct.c_void_p, ct.c_void_p]),
    "mfm_model_free": (None, [ct.c_void_p]),
    "mfm_libffm_read": (ct.c_int, [ct.c_char_p, ct.c_int, ct.POINTER(ct.c_void_p)]),
    "mfm_libffm_info": (ct.c_int, [ct.c_void_p, i64p, i64p, i64p]),
    "mfm_libffm_arrays": (ct.c_int, [ct.c_void_p] + [ct.POINTER(ct.c_void_p)] * 5),
    "mfm_libffm_free": (None, [ct.c_void_p]),
    "mfm_fm_predict_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p,
                                         ct.c_void_p, ct.c_int64, ct.c_double, ct.c_void_p,
                                         ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_void_p]),
    "mfm_ffm_predict_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p,
                                          ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_int64,
                                          ct.c_double, ct.c_void_p, ct.c_void_p, ct.c_int64,
                                          ct.c_void_p, ct.c_void_p]),
    "mfm_fwfm_predict_device": (ct.c_int, [ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p,
                                           ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_int64,
                                           ct.c_double, ct.c_void_p, ct.c_void_p, ct.c_void_p,
                                           ct.c_int64, ct.c_void_p, ct.c_void_p]),
}

_lib = None


def lib():
    """The loaded engine library. Raises if it was not built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA engine with "
                "`python -m modern_fm_b200.build` (there is no CPU fallback)")
        L = ct.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().mfm_last_error()
    return msg.decode() if msg else ""


def ptr(a, kind=f64p):
    return None if a is None else a.ctypes.data_as(kind)


def make_csr(indptr, indices, data, n_features, exc=ValueError):
    """(Csr struct, keepalive) for int64/float64 C-contiguous CSR arrays.
    `exc` is the exception type for a malformed CSR (the reference raises
    RuntimeError from predict and ValueError from fit)."""
    indptr = np.ascontiguousarray(indptr, dtype=np.int64)
    indices = np.ascontiguousarray(indices, dtype=np.int64)
    data = np.ascontiguousarray(data, dtype=np.float64)
    if indptr.size == 0:
        raise exc("indptr must have length n_rows + 1 (>= 1)")
    if indices.size != data.size:
        raise exc(
            f"indices and data length mismatch: {indices.size} vs {data.size}")
    c = Csr(ptr(indptr, i64p), ptr(indices, i64p), ptr(data), indptr.size - 1, data.size,
            int(n_features))
    return c, (indptr, indices, data)


def dtype_code(dt):
    """MFM_DTYPE_* code of a compute-type name (float64, float32,
    float32-float64) or code."""
    if isinstance(dt, int):
        if dt in (MFM_DTYPE_F64, MFM_DTYPE_F32, MFM_DTYPE_F32_F64):
            return dt
    else:
        code = DTYPES.get(str(dt))
        if code is not None:
            return code
    raise ValueError(
        f"unknown compute dtype {dt!r} (expected float64, float32 or float32-float64)")


def exec_options(dtype=None, device=None, n_devices=None):
    """Execution options from arguments or the environment:
    MFM_B200_DTYPE (float32-float64 | float64 | float32, default
    float32-float64: float64 arithmetic, parameters stored as float32 whenever
    every value is exactly a float32), MFM_B200_DEVICE (default 0),
    MFM_B200_NUM_GPUS (default 1)."""
    code = dtype_code(dtype or os.environ.get("MFM_B200_DTYPE", "float32-float64"))
    dev = int(device if device is not None else os.environ.get("MFM_B200_DEVICE", "0"))
    nd = int(n_devices if n_devices is not None else os.environ.get("MFM_B200_NUM_GPUS", "1"))
    return Exec(code, dev, max(1, nd))


def fit_phase_seconds() -> dict:
    """Device seconds of the calling thread's last fit by phase (upload,
    plan, batches, download)."""
    out = (ct.c_double * 4)()
    lib().mfm_fit_phase_seconds(out)
    return dict(zip(("upload", "plan", "batches", "download"), list(out)))
