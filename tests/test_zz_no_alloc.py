"""The allocation-free FM scoring entry point, mfm_fm_predict_csr_noalloc.

It exists for callers that cannot let the library allocate GPU memory (a host
that owns the device budget through its own pool, or a serving loop that
cannot afford the device-wide synchronisation of cudaMalloc / cudaFree). It
must return what mfm_fm_predict_csr returns, call after call, while staging
everything in its static device array. This file is collected last so that a
run stopping at the first failure has already run every other test.
"""

import ctypes as ct

import numpy as np
import pytest
import scipy.sparse as sp

from modern_fm_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-10  # the float64 scoring tolerance of the other GPU tests


def _noalloc():
    L = _lib.lib()
    fn = L.mfm_fm_predict_csr_noalloc
    fn.restype = ct.c_int
    fn.argtypes = [ct.POINTER(_lib.Csr), ct.c_double, _lib.f64p, _lib.f64p, ct.c_int64,
                   _lib.f64p, ct.POINTER(_lib.Exec)]
    L.mfm_noalloc_scratch_bytes.restype = ct.c_int64
    return L, fn


def _problem(seed, n, d, k, density):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, d))
    X[rng.random(size=X.shape) > density] = 0.0
    M = sp.csr_matrix(X)
    return (M.indptr.astype(np.int64), M.indices.astype(np.int64), M.data,
            float(rng.normal()), rng.normal(size=d), rng.normal(size=(d, k)))


def _both(fn, L, prob, dtype):
    ip, ix, dv, w0, w, V = prob
    csr, keep = _lib.make_csr(ip, ix, dv, len(w))
    ex = _lib.Exec(dtype, 0, 1)
    ref = np.full(len(ip) - 1, np.nan)
    got = np.full(len(ip) - 1, np.nan)
    rc = L.mfm_fm_predict_csr(csr, w0, _lib.ptr(w), _lib.ptr(V), V.shape[1], _lib.ptr(ref), ex)
    assert rc == 0, _lib.last_error()
    rc = fn(csr, w0, _lib.ptr(w), _lib.ptr(V), V.shape[1], _lib.ptr(got), ex)
    assert rc == 0, _lib.last_error()
    return got, ref


@pytest.mark.parametrize("dtype", [_lib.MFM_DTYPE_F64, _lib.MFM_DTYPE_F32])
def test_noalloc_matches_the_allocating_entry_point_on_consecutive_calls(dtype):
    L, fn = _noalloc()
    # the second problem is smaller, so stale contents of the shared array
    # from the first call would show up as wrong scores
    for prob in (_problem(0, 3000, 400, 16, 0.05), _problem(1, 700, 90, 8, 0.2)):
        got, ref = _both(fn, L, prob, dtype)
        np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)


def test_noalloc_allocates_no_device_memory():
    import torch

    L, fn = _noalloc()
    prob = _problem(2, 2000, 300, 16, 0.05)
    ip, ix, dv, w0, w, V = prob
    csr, keep = _lib.make_csr(ip, ix, dv, len(w))
    ex = _lib.Exec(_lib.MFM_DTYPE_F64, 0, 1)
    out = np.empty(len(ip) - 1)
    assert fn(csr, w0, _lib.ptr(w), _lib.ptr(V), 16, _lib.ptr(out), ex) == 0
    free_before = torch.cuda.mem_get_info(0)[0]
    for _ in range(2):
        assert fn(csr, w0, _lib.ptr(w), _lib.ptr(V), 16, _lib.ptr(out), ex) == 0
    assert torch.cuda.mem_get_info(0)[0] == free_before


def test_noalloc_rejects_inputs_beyond_its_static_array():
    L, fn = _noalloc()
    limit = L.mfm_noalloc_scratch_bytes()
    d, k = 1 << 20, 16  # V alone is 128 MiB in float64
    assert d * k * 8 > limit
    ip, ix, dv = np.array([0, 1], np.int64), np.array([3], np.int64), np.array([1.0])
    w, V = np.zeros(d), np.zeros((d, k))
    csr, keep = _lib.make_csr(ip, ix, dv, d)
    out = np.empty(1)
    rc = fn(csr, 0.0, _lib.ptr(w), _lib.ptr(V), k, _lib.ptr(out), _lib.Exec(0, 0, 1))
    assert rc == -2
    assert "static scratch" in _lib.last_error()
