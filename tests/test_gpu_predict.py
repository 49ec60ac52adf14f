"""GPU parity of the CSR scoring kernels (FM / FFM / FwFM), through the C ABI,
against the C oracle and the reference's NumPy golden outputs.

Tolerances: float64 arithmetic (MFM_DTYPE_F64, and MFM_DTYPE_F32_F64 on
float32-valued parameters) uses the reference's own CUDA bar, rtol = atol =
1e-10 (tests/test_cuda_parity.py:30-31); float32 arithmetic uses the target
bar of 1e-5 relative, with an absolute floor of 1e-5 times the row's
magnitude scale (the sum of the absolute values of the score's terms) so that
scores near zero are judged on their scale.
"""

import numpy as np
import pytest
import scipy.sparse as sp

import golden_io
import run_cases
from modern_fm_b200 import _rust
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL64 = ATOL64 = 1e-10
RTOL32 = 1e-5


@pytest.fixture
def f32(monkeypatch):
    monkeypatch.setenv("MFM_B200_DTYPE", "float32")


@pytest.fixture
def f64(monkeypatch):
    monkeypatch.setenv("MFM_B200_DTYPE", "float64")


def _abs_scale(case):
    """Per-row sum of |terms| of the score: the oracle's score of the same
    row with every value, parameter and weight replaced by its magnitude."""
    a = case.a
    n, m = case["n_features"], case["model"]
    ip, ix, dv = a["indptr"], a["indices"], np.abs(a["data"])
    if m == "fm":
        return _scale_fm(ip, ix, a["data"], case["w0"], a["w"], a["V"])
    if m == "ffm":
        return O.ffm_predict_csr(ip, ix, dv, n, a["field_ids"], abs(case["w0"]),
                                 np.abs(a["w"]), np.abs(a["V"])) + 1.0
    return O.fwfm_predict_csr(ip, ix, dv, n, a["field_ids"], abs(case["w0"]), np.abs(a["w"]),
                              np.abs(a["V"]), np.abs(a["r"])) + 1.0


def _round32(case):
    """The case with every parameter rounded to float32 (as a float32
    estimator's attributes are), values kept float64."""
    a = dict(case.a)
    for key in ("w", "V", "r"):
        if key in a:
            a[key] = a[key].astype(np.float32).astype(np.float64)
    return golden_io.Case(dict(case), a)


def _scale_fm(ip, ix, dv, w0, w, V):
    """Per-row sum of the absolute terms of the FM score (for float32 atol)."""
    n = len(ip) - 1
    X = sp.csr_matrix((np.abs(dv), ix, ip), shape=(n, len(w)))
    aV = np.abs(V)
    return abs(w0) + X @ np.abs(w) + 0.5 * ((X @ aV) ** 2).sum(axis=1) + 1.0


def _random_csr(rng, n, d, density):
    X = rng.normal(size=(n, d))
    X[rng.random(size=X.shape) > density] = 0.0
    Xc = sp.csr_matrix(X)
    return Xc.indptr.astype(np.int64), Xc.indices.astype(np.int64), Xc.data


@pytest.mark.parametrize("case", golden_io.load("predict.npz"), ids=lambda c: c.name)
def test_predict_golden_f64(case, f64):
    got = run_cases.predict_case(_rust, case, cuda=True)
    np.testing.assert_allclose(got, case.a["out"], rtol=RTOL64, atol=ATOL64)
    np.testing.assert_allclose(got, run_cases.predict_case(O, case, cuda=False), rtol=RTOL64,
                               atol=ATOL64)


@pytest.mark.parametrize("case", golden_io.load("predict.npz"), ids=lambda c: c.name)
def test_predict_golden_f32(case, f32):
    got = run_cases.predict_case(_rust, case, cuda=True)
    want = case.a["out"]
    scale = _abs_scale(case)
    assert np.all(np.abs(got - want) <= RTOL32 * np.abs(want) + 1e-5 * scale)


@pytest.mark.parametrize("case", golden_io.load("predict.npz"), ids=lambda c: c.name)
def test_predict_golden_f32_f64(case, monkeypatch):
    """float32 parameters, float64 values and arithmetic: the reference's
    computation for a float32 estimator. Against the oracle on the same
    float32-rounded parameters at the float64 bar."""
    monkeypatch.setenv("MFM_B200_DTYPE", "float32-float64")
    c = _round32(case)
    got = run_cases.predict_case(_rust, c, cuda=True)
    want = run_cases.predict_case(O, c, cuda=False)
    np.testing.assert_allclose(got, want, rtol=RTOL64, atol=ATOL64)


def test_f32_f64_inexact_parameters_fall_back_to_f64(monkeypatch):
    """Parameters that are not float32 values are scored in float64: the
    result is bitwise that of MFM_DTYPE_F64."""
    rng = np.random.default_rng(11)
    ip, ix, dv = _random_csr(rng, 500, 300, 0.05)
    w0, w, V = 0.3, rng.normal(size=300), rng.normal(size=(300, 16)) * 0.2
    monkeypatch.setenv("MFM_B200_DTYPE", "float64")
    a = _rust.fm_predict_cuda_csr(ip, ix, dv, 300, w0, w, V)
    monkeypatch.setenv("MFM_B200_DTYPE", "float32-float64")
    b = _rust.fm_predict_cuda_csr(ip, ix, dv, 300, w0, w, V)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 8, 12, 16, 17, 24, 32, 64, 130, 1024])
@pytest.mark.parametrize("dtype", ["float64", "float32", "float32-float64"])
def test_fm_predict_k_range(k, dtype, monkeypatch):
    """Every latent width reaches a kernel shape (row-group or generic); rows
    of 0 to 150 nonzeros cover one and several gather iterations."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    rng = np.random.default_rng(k)
    ip, ix, dv = _random_csr(rng, 300, 200, 0.2)
    ip2, ix2, dv2 = _random_csr(rng, 20, 200, 0.75)  # ~150 nonzeros per row
    ip = np.concatenate([ip, ip2[1:] + ip[-1]])
    ix, dv = np.concatenate([ix, ix2]), np.concatenate([dv, dv2])
    w0, w, V = rng.normal(), rng.normal(size=200), rng.normal(size=(200, k)) * 0.3
    if dtype == "float32-float64":
        w, V = w.astype(np.float32).astype(np.float64), V.astype(np.float32).astype(np.float64)
    want = O.fm_predict_fast_csr(ip, ix, dv, 200, w0, w, V)
    got = _rust.fm_predict_cuda_csr(ip, ix, dv, 200, w0, w, V)
    if dtype != "float32":
        np.testing.assert_allclose(got, want, rtol=RTOL64, atol=1e-9 * max(1.0, k / 16))
    else:
        scale = _scale_fm(ip, ix, dv, w0, w, V)
        assert np.all(np.abs(got - want) <= RTOL32 * np.abs(want) + 1e-5 * scale)


def test_empty_rows_and_single_nonzero():
    # tests/test_cuda_parity.py:51-64
    X = sp.csr_matrix((4, 6))
    out = _rust.fm_predict_cuda_csr(X.indptr, X.indices, X.data, 6, 1.5, np.zeros(6),
                                    np.ones((6, 3)))
    np.testing.assert_allclose(out, np.full(4, 1.5), rtol=RTOL64, atol=ATOL64)
    Xd = np.zeros((3, 5))
    Xd[1, 2] = -2.0
    Xc = sp.csr_matrix(Xd)
    w = np.arange(5.0)
    out = _rust.fm_predict_cuda_csr(Xc.indptr, Xc.indices, Xc.data, 5, 0.5, w,
                                    np.ones((5, 4)))
    np.testing.assert_allclose(out, [0.5, 0.5 + w[2] * -2.0, 0.5], rtol=RTOL64, atol=ATOL64)
    fid = np.array([0, 1, 2, 0, 1])
    out = _rust.ffm_predict_cuda_csr(Xc.indptr, Xc.indices, Xc.data, 5, fid, 0.5, w,
                                     np.ones((5, 3, 4)))
    np.testing.assert_allclose(out, [0.5, 0.5 + w[2] * -2.0, 0.5], rtol=RTOL64, atol=ATOL64)
    out = _rust.fwfm_predict_cuda_csr(Xc.indptr, Xc.indices, Xc.data, 5, fid, 0.5, w,
                                      np.ones((5, 4)), np.ones((3, 3)))
    np.testing.assert_allclose(out, [0.5, 0.5 + w[2] * -2.0, 0.5], rtol=RTOL64, atol=ATOL64)


def test_zero_row_matrix():
    out = _rust.fm_predict_cuda_csr(np.array([0]), np.array([], dtype=np.int64), np.array([]),
                                    3, 1.0, np.zeros(3), np.zeros((3, 2)))
    assert out.shape == (0,)


def test_known_answers():
    # FM 4.25 (rust/src/fm.rs:433-441), FFM 9.5 (ffm.rs:454-474), FwFM 10.25 (fwfm.rs:411-420)
    ip, ix, dv = np.array([0, 2]), np.array([0, 1]), np.array([2.0, 3.0])
    V = np.array([[1.0, 0.0], [1.0, 1.0]])
    out = _rust.fm_predict_cuda_csr(ip, ix, dv, 2, 0.25, np.array([0.5, -1.0]), V)
    assert abs(out[0] - 4.25) < 1e-12
    r = np.ones((2, 2))
    r[0, 1] = 2.0
    out = _rust.fwfm_predict_cuda_csr(ip, ix, dv, 2, np.array([0, 1]), 0.25,
                                      np.array([0.5, -1.0]), V, r)
    assert abs(out[0] - 10.25) < 1e-12
    V3 = np.zeros((3, 2, 2))
    V3[0, 0], V3[0, 1] = [1.0, 0.0], [0.0, 1.0]
    V3[1, 0], V3[1, 1] = [1.0, 1.0], [2.0, 0.0]
    V3[2, 0], V3[2, 1] = [0.5, 0.5], [1.0, -1.0]
    out = _rust.ffm_predict_cuda_csr(np.array([0, 3]), np.array([0, 1, 2]),
                                     np.array([1.0, 2.0, 3.0]), 3, np.array([0, 0, 1]), 0.0,
                                     np.zeros(3), V3)
    assert abs(out[0] - 9.5) < 1e-12


@pytest.mark.parametrize("k", [1, 3, 4, 5, 8, 16, 17, 32, 33])
@pytest.mark.parametrize("F", [3, 9, 46])
@pytest.mark.parametrize("dtype", ["float64", "float32"])
def test_fwfm_row_lengths_latent_widths_and_field_counts(k, F, dtype, monkeypatch):
    """FwFM rows of every length 0..40 in one call (the register-staged rows
    of at most 16 entries and the longer ones scored by a whole warp), latent
    widths on both sides of each lane-group size, and a field count whose
    F x F table is too large for the block's shared copy (46 x 46)."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    rng = np.random.default_rng(1000 * k + F)
    d = 300
    lens = np.tile(np.arange(41), 3)
    rng.shuffle(lens)
    ip = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ix = np.concatenate([np.sort(rng.choice(d, size=n, replace=False)) for n in lens])
    ix = ix.astype(np.int64)
    dv = rng.uniform(-1.0, 1.0, size=len(ix))
    fid = rng.integers(0, F, size=d)
    w0, w = 0.25, rng.normal(size=d) * 0.3
    V, r = rng.normal(size=(d, k)) * 0.3, rng.uniform(size=(F, F))
    if dtype == "float32":
        w, V, r = (a.astype(np.float32).astype(np.float64) for a in (w, V, r))
    got = _rust.fwfm_predict_cuda_csr(ip, ix, dv, d, fid, w0, w, V, r)
    want = O.fwfm_predict_csr(ip, ix, dv, d, fid, w0, w, V, r)
    if dtype == "float64":
        np.testing.assert_allclose(got, want, rtol=RTOL64, atol=ATOL64)
    else:
        scale = O.fwfm_predict_csr(ip, ix, np.abs(dv), d, fid, w0, np.abs(w), np.abs(V),
                                   r) + 1.0
        assert np.all(np.abs(got - want) <= RTOL32 * np.abs(want) + 1e-5 * scale)


def test_ffm_large_row(f64):
    # a single row with z = 2048 nonzeros (tests/test_cuda_parity.py:126-136)
    rng = np.random.default_rng(0)
    d = 2048
    X = sp.csr_matrix(rng.normal(size=(1, d)))
    w0, w = float(rng.normal()), rng.normal(size=d)
    V = rng.normal(size=(d, 4, 4))
    fid = rng.integers(0, 4, size=d)
    want = O.ffm_predict_csr(X.indptr, X.indices, X.data, d, fid, w0, w, V)
    got = _rust.ffm_predict_cuda_csr(X.indptr, X.indices, X.data, d, fid, w0, w, V)
    np.testing.assert_allclose(got, want, rtol=RTOL64, atol=ATOL64)
    Vf = rng.normal(size=(d, 4))
    r = rng.uniform(size=(4, 4))
    want = O.fwfm_predict_csr(X.indptr, X.indices, X.data, d, fid, w0, w, Vf, r)
    got = _rust.fwfm_predict_cuda_csr(X.indptr, X.indices, X.data, d, fid, w0, w, Vf, r)
    np.testing.assert_allclose(got, want, rtol=RTOL64, atol=1e-9)


def test_predict_validation_on_device():
    # the reference raises RuntimeError for everything inside the CUDA predict
    # call, CSR checks included (rust/src/lib.rs:1506-1512), and ValueError for
    # the field-id check that precedes it (lib.rs:1536-1537)
    ip, ix, dv = np.array([0, 1, 2]), np.array([0, 5]), np.ones(2)
    with pytest.raises(RuntimeError, match=r"column index out of range \[0, 3\)"):
        _rust.fm_predict_cuda_csr(ip, ix, dv, 3, 0.0, np.zeros(3), np.zeros((3, 2)))
    with pytest.raises(RuntimeError, match="indptr must be non-decreasing"):
        _rust.fm_predict_cuda_csr(np.array([0, 2, 1, 2]), np.array([0, 1]), np.ones(2), 3, 0.0,
                                  np.zeros(3), np.zeros((3, 2)))
    with pytest.raises(ValueError, match=r"field id out of range \[0, 2\)"):
        _rust.ffm_predict_cuda_csr(np.array([0, 1]), np.array([0]), np.ones(1), 2,
                                   np.array([0, 2]), 0.0, np.zeros(2), np.zeros((2, 2, 2)))
    with pytest.raises(RuntimeError, match="1 <= k <= 1024"):
        _rust.fm_predict_cuda_csr(np.array([0, 1]), np.array([0]), np.ones(1), 2, 0.0,
                                  np.zeros(2), np.zeros((2, 1025)))


def test_ctr_shaped_f32_f64_against_oracle(monkeypatch):
    """The CTR-shaped FM workload (39 fields, Zipf ids, k=16) with float32
    parameters and float64 arithmetic, at the float64 bar."""
    from modern_fm_b200 import workloads

    monkeypatch.setenv("MFM_B200_DTYPE", "float32-float64")
    X, _ = workloads.ctr_fm(n_rows=20000, seed=6)
    rng = np.random.default_rng(2)
    d = X.n_features
    w = rng.normal(0, 0.1, d).astype(np.float32).astype(np.float64)
    V = rng.normal(0, 0.1, (d, 16)).astype(np.float32).astype(np.float64)
    want = O.fm_predict_fast_csr(X.indptr, X.indices, X.data, d, -3.0, w, V, n_threads=4)
    got = _rust.fm_predict_cuda_csr(X.indptr, X.indices, X.data, d, -3.0, w, V)
    np.testing.assert_allclose(got, want, rtol=RTOL64, atol=ATOL64)


def test_ctr_shaped_f32_against_oracle(f32):
    """A CTR-shaped FM workload (39 fields, Zipf ids, k=16) in float32."""
    from modern_fm_b200 import workloads

    X, _ = workloads.ctr_fm(n_rows=20000, seed=5)
    rng = np.random.default_rng(1)
    d = X.n_features
    w0, w, V = -3.0, rng.normal(0, 0.1, d), rng.normal(0, 0.1, (d, 16))
    want = O.fm_predict_fast_csr(X.indptr, X.indices, X.data, d, w0, w, V, n_threads=4)
    got = _rust.fm_predict_cuda_csr(X.indptr, X.indices, X.data, d, w0, w, V)
    scale = _scale_fm(X.indptr, X.indices, X.data, w0, w, V)
    assert np.all(np.abs(got - want) <= RTOL32 * np.abs(want) + 1e-6 * scale)


def test_multi_device_sharding_matches_single(monkeypatch):
    if _rust.has_cuda() and __import__("modern_fm_b200._lib", fromlist=["x"]).lib(
    ).mfm_device_count() < 2:
        pytest.skip("needs 2 GPUs")
    rng = np.random.default_rng(3)
    ip, ix, dv = _random_csr(rng, 5000, 100, 0.1)
    w0, w, V = rng.normal(), rng.normal(size=100), rng.normal(size=(100, 8))
    one = _rust.fm_predict_cuda_csr(ip, ix, dv, 100, w0, w, V)
    monkeypatch.setenv("MFM_B200_NUM_GPUS", "2")
    two = _rust.fm_predict_cuda_csr(ip, ix, dv, 100, w0, w, V)
    np.testing.assert_array_equal(one, two)
