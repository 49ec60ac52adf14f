"""CPU-side checks of the C ABI and its Python mirror: the library loads,
exports every entry point include/mfm_b200.h declares, reports no device here,
and host-side validation raises the reference's exception types before any
device work."""

import ctypes as ct
import os
import re

import numpy as np
import pytest

from modern_fm_b200 import _lib, _rust

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "mfm_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mfm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for name in ("mfm_fm_predict_csr", "mfm_ffm_predict_csr", "mfm_fwfm_predict_csr",
                 "mfm_fm_fit_csr", "mfm_fm_fit_multiclass_csr", "mfm_ffm_fit_csr",
                 "mfm_ffm_fit_multiclass_csr", "mfm_fwfm_fit_csr", "mfm_fwfm_fit_multiclass_csr",
                 "mfm_has_cuda", "mfm_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = ct.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    _lib.lib()  # the typed binding loads too


def test_mirror_exposes_the_reference_cuda_entry_points():
    # rust/src/lib.rs:1592-1614 registers these names
    for name in _rust.CUDA_FUNCTIONS:
        assert callable(getattr(_rust, name))


@pytest.mark.skipif(_rust.has_cuda(), reason="checks the no-device behaviour")
def test_no_device_is_reported_not_hidden():
    assert _rust.has_cuda() is False
    assert _lib.lib().mfm_device_count() == 0
    with pytest.raises(RuntimeError, match="no CUDA device"):
        _rust.fm_predict_cuda_csr(np.array([0, 1]), np.array([0]), np.array([1.0]), 2, 0.0,
                                  np.zeros(2), np.zeros((2, 4)))


def _fit_args(**over):
    n, d, k = 4, 3, 2
    a = dict(indptr=np.array([0, 1, 2, 3, 4]), indices=np.array([0, 1, 2, 0]),
             data=np.ones(4), n_features=d, y=np.array([0.0, 1.0, 0.0, 1.0]),
             sample_weight=np.ones(n), w0=0.0, acc_w0=0.0, w=np.zeros(d), v=np.zeros((d, k)),
             acc_w=np.zeros(d), acc_v=np.zeros((d, k)), loss="logistic", optimizer="adagrad",
             learning_rate=0.1, l2_linear=0.0, l2_factors=0.0, beta_1=0.9, beta_2=0.999,
             epsilon=1e-8, row_orders=np.arange(n)[None, :], batch_size=2, n_jobs=1,
             l1_linear=0.0, l1_factors=0.0, ftrl_beta=1.0, use_cuda=True)
    a.update(over)
    return a


@pytest.mark.parametrize("over,msg", [
    (dict(loss="hinge"), "unknown loss"),
    (dict(optimizer="rmsprop"), "unknown optimizer"),
    (dict(batch_size=0), "batch_size must be >= 1"),
    (dict(w=np.zeros(5)), "shape mismatch"),
    (dict(acc_v=np.zeros((3, 3))), "accumulator shapes must match w and V"),
    (dict(y=np.zeros(3)), "y length 3 != n_rows 4"),
    (dict(sample_weight=np.ones(2)), "sample_weight length 2 != n_rows 4"),
    (dict(row_orders=np.array([[0, 1, 2, 7]])), r"row_orders entry out of range \[0, 4\)"),
    (dict(row_orders=np.array([[0, 1, 2]])), "row_orders second dimension 3 != n_rows 4"),
    (dict(indptr=np.array([0, 1, 2, 3, 5])), "indptr must start at 0 and end at nnz"),
    (dict(adam_state=(0.0, 0.0, 0.0)), "adam_state is only valid for optimizer='adam'"),
])
def test_fit_validation_is_value_error(over, msg):
    with pytest.raises(ValueError, match=msg):
        _rust.fm_fit_csr(**_fit_args(**over))


def test_fit_use_cuda_false_is_not_served_by_the_engine():
    with pytest.raises(ValueError, match="CUDA engine"):
        _rust.fm_fit_csr(**_fit_args(use_cuda=False))


def test_readwrite_arrays_must_be_float64_contiguous():
    with pytest.raises(TypeError):
        _rust.fm_fit_csr(**_fit_args(w=np.zeros(3, dtype=np.float32)))


def test_multiclass_class_index_range():
    a = _fit_args()
    with pytest.raises(ValueError, match=r"class index out of range \[0, 2\)"):
        _rust.fm_fit_multiclass_csr(
            a["indptr"], a["indices"], a["data"], 3, np.array([0, 1, 2, 0]), np.ones(4),
            np.zeros(2), np.zeros((2, 3)), np.zeros((2, 3, 2)), "sgd", 0.1, 0.0, 0.0, 0.0, 0.9,
            0.999, 1e-8, np.arange(4)[None, :], 2, 0.0, 0.0, 1.0, use_cuda=True)


def test_exec_options_from_environment(monkeypatch):
    monkeypatch.setenv("MFM_B200_DTYPE", "float32")
    monkeypatch.setenv("MFM_B200_NUM_GPUS", "4")
    ex = _lib.exec_options()
    assert ex.dtype == _lib.MFM_DTYPE_F32 and ex.n_devices == 4 and ex.device == 0
    monkeypatch.setenv("MFM_B200_DTYPE", "float16")
    with pytest.raises(ValueError, match="unknown compute dtype"):
        _lib.exec_options()


def _prep_call(dtype=_lib.MFM_DTYPE_F32, n_rows=2, n_features=4, nnz=2, null=False):
    """mfm_csr_prep_device with dummy (never dereferenced) pointers: every case
    below fails in the host checks, before any device work."""
    p = None if null else 16
    out = ct.c_int64(-1)
    return _lib.lib().mfm_csr_prep_device(dtype, 0, n_rows, n_features, nnz, p, p, p, p, p, p,
                                          ct.byref(out), None)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(n_rows=-1), _lib.MFM_ERR_INVALID, "negative CSR size"),
    (dict(nnz=-3), _lib.MFM_ERR_INVALID, "negative CSR size"),
    (dict(null=True), _lib.MFM_ERR_INVALID, "must be provided"),
    (dict(n_features=2**31), _lib.MFM_ERR_UNSUPPORTED, "2^31-1 limit"),
    (dict(dtype=9), _lib.MFM_ERR_INVALID, "unknown dtype 9"),
])
def test_csr_prep_host_checks(kw, code, msg):
    assert _prep_call(**kw) == code
    assert msg in _lib.last_error()


def test_eval_host_checks_and_empty_input():
    L = _lib.lib()
    out = ct.c_double(0.0)
    rc = L.mfm_fm_eval_device(_lib.MFM_DTYPE_F64, 0, 16, 16, 16, 3, 0.0, 16, 16, 4, 16, None, 7,
                              0.0, ct.byref(out), None)
    assert rc == _lib.MFM_ERR_INVALID and "unknown loss 7" in _lib.last_error()
    rc = L.mfm_fm_eval_device(5, 0, 16, 16, 16, 3, 0.0, 16, 16, 4, 16, None, 0, 0.0,
                              ct.byref(out), None)
    assert rc == _lib.MFM_ERR_INVALID and "unknown dtype 5" in _lib.last_error()
    # no rows: NumPy's mean of nothing (nan), answered before any device work
    rc = L.mfm_fm_eval_device(_lib.MFM_DTYPE_F64, 0, None, None, None, 0, 0.0, None, None, 4,
                              None, None, 0, 0.0, ct.byref(out), None)
    assert rc == _lib.MFM_OK and np.isnan(out.value)
