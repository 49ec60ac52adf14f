"""GPU parity of the persistent model handle (mfm_model_*) and of multiclass
scoring, through the C ABI, against the oracle.

The reference scores a multiclass model one class at a time with the binary
kernels (python/modern_fm/fm.py:666-674); the oracle does the same with each
class's parameters, and the handle's (n_rows, C) logits must match every
column. Tolerances: float64 arithmetic rtol = atol = 1e-10 (the reference's
CUDA bar, tests/test_cuda_parity.py:30-31); float32 arithmetic 1e-5 relative
with an absolute floor of 1e-5 times the row's sum of |terms|.
"""

import zlib

import numpy as np
import pytest
import scipy.sparse as sp

from modern_fm_b200.model import DeviceModel
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL64 = ATOL64 = 1e-10


def _csr(rng, n, d, density, ragged=True):
    X = sp.random(n, d, density=density, format="csr", random_state=int(rng.integers(1 << 30)),
                  data_rvs=lambda m: rng.lognormal(0.0, 0.5, size=m))
    if ragged:  # a few long rows and some empty ones
        X = sp.vstack([X, sp.random(3, d, density=min(1.0, 40 * density), format="csr",
                                    random_state=1), sp.csr_matrix((2, d))]).tocsr()
    return X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data.astype(np.float64)


def _oracle(kind, ip, ix, dv, d, fid, w0, w, V, R):
    if kind == "fm":
        return O.fm_predict_fast_csr(ip, ix, dv, d, w0, w, V)
    if kind == "ffm":
        return O.ffm_predict_csr(ip, ix, dv, d, fid, w0, w, V)
    return O.fwfm_predict_csr(ip, ix, dv, d, fid, w0, w, V, R)


def _params(rng, kind, C, d, F, k, f32):
    lead = (C,) if C > 1 else ()
    w0 = rng.normal(size=C) if C > 1 else float(rng.normal())
    w = rng.normal(size=lead + (d,)) * 0.3
    V = rng.normal(size=lead + ((d, F, k) if kind == "ffm" else (d, k))) * 0.3
    R = rng.uniform(size=lead + (F, F)) if kind == "fwfm" else None
    if f32:
        w, V = (a.astype(np.float32).astype(np.float64) for a in (w, V))
        if R is not None:
            R = R.astype(np.float32).astype(np.float64)
    return w0, w, V, R


@pytest.mark.parametrize("kind", ["fm", "ffm", "fwfm"])
@pytest.mark.parametrize("C", [1, 3, 10])
@pytest.mark.parametrize("dtype", ["float64", "float32-float64", "float32"])
def test_model_matches_oracle(kind, C, dtype):
    rng = np.random.default_rng(zlib.crc32(f"{kind}/{C}/{dtype}".encode()))
    d, F, k = 400, 5, 8
    ip, ix, dv = _csr(rng, 600, d, 0.03)
    fid = rng.integers(0, F, size=d)
    w0, w, V, R = _params(rng, kind, C, d, F, k, f32=dtype != "float64")
    with DeviceModel(kind, d, k, n_fields=F, n_classes=C, dtype=dtype) as m:
        m.set_params(w0, w, V, R, None if kind == "fm" else fid)
        assert m.dtype_used == dtype
        got = m.predict_csr(ip, ix, dv)
        assert got.shape == ((len(ip) - 1,) if C == 1 else (len(ip) - 1, C))
        got = got.reshape(len(ip) - 1, C)
        for c in range(C):
            pc = (lambda a: a[c]) if C > 1 else (lambda a: a)
            want = _oracle(kind, ip, ix, dv, d, fid, pc(w0) if C > 1 else w0, pc(w), pc(V),
                           None if R is None else pc(R))
            if dtype == "float32":
                scale = _oracle(kind, ip, ix, np.abs(dv), d, fid,
                                abs(pc(w0) if C > 1 else w0), np.abs(pc(w)), np.abs(pc(V)),
                                None if R is None else np.abs(pc(R))) + 1.0
                assert np.all(np.abs(got[:, c] - want) <= 1e-5 * np.abs(want) + 1e-5 * scale)
            else:
                np.testing.assert_allclose(got[:, c], want, rtol=RTOL64, atol=ATOL64)


def test_model_reused_across_calls_and_inexact_fallback():
    """Parameters upload once; repeated calls are bitwise equal; float64
    parameters that are not float32 values make float32-float64 score in
    float64 (bitwise the float64 handle's result)."""
    rng = np.random.default_rng(5)
    d, k = 300, 16
    ip, ix, dv = _csr(rng, 1000, d, 0.05)
    w0, w, V, _ = _params(rng, "fm", 1, d, 1, k, f32=False)
    with DeviceModel("fm", d, k, dtype="float32-float64") as a, \
            DeviceModel("fm", d, k, dtype="float64") as b:
        a.set_params(w0, w, V)
        b.set_params(w0, w, V)
        assert a.dtype_used == "float64"
        s1 = a.predict_csr(ip, ix, dv)
        s2 = a.predict_csr(ip, ix, dv)
        np.testing.assert_array_equal(s1, s2)
        np.testing.assert_array_equal(s1, b.predict_csr(ip, ix, dv))


def test_model_predict_device_matches_host_path():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    d, k, C = 500, 8, 4
    ip, ix, dv = _csr(rng, 2000, d, 0.02, ragged=False)
    w0, w, V, _ = _params(rng, "fm", C, d, 1, k, f32=True)
    with DeviceModel("fm", d, k, n_classes=C, dtype="float32-float64") as m:
        m.set_params(w0, w, V)
        host = m.predict_csr(ip, ix, dv)
        t = lambda a, dt: torch.from_numpy(a).to("cuda", dt)  # noqa: E731
        out = torch.empty((len(ip) - 1, C), dtype=torch.float64, device="cuda")
        m.predict_device(t(ip, torch.int64), t(ix, torch.int32), t(dv, torch.float64), out)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), host, rtol=1e-13, atol=1e-13)


def test_model_errors():
    import ctypes as ct

    from modern_fm_b200 import _lib

    with pytest.raises(ValueError, match="kind"):
        DeviceModel("xfm", 10, 4)
    m = DeviceModel("fm", 10, 4)
    with pytest.raises(ValueError, match="not set"):
        m.predict_csr(np.array([0, 1]), np.array([0]), np.ones(1))
    m.set_params(0.0, np.zeros(10), np.zeros((10, 4)))
    # a CSR whose width differs from the model's
    csr, keep = _lib.make_csr(np.array([0, 1]), np.array([0]), np.ones(1), 11)
    out = np.zeros(1)
    assert _lib.lib().mfm_model_predict_csr(m._h, ct.byref(csr), _lib.ptr(out)) == \
        _lib.MFM_ERR_INVALID
    assert "features" in _lib.last_error()
    with pytest.raises(ValueError, match="column index out of range"):
        m.predict_csr(np.array([0, 1]), np.array([12]), np.ones(1))
    m.close()
