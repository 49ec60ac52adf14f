"""GPU parity of the device early-stopping evaluation (mfm_{fm,ffm,fwfm}_eval_device)
against the oracle: the reference's `metric(y_val, fm_predict_fast(X_val,
...))` (python/modern_fm/fm.py:321-322), and its FFM / FwFM counterparts
(python/modern_fm/ffm.py:210-212, python/modern_fm/fwfm.py:157-161), restated
on the CPU.

Tolerances: float64 compute 1e-9 relative (scores within the reference's CUDA
bar of 1e-10, the mean in another addition order); float32 compute 1e-4
relative (scores within 1e-5). Repeated calls are bitwise equal.
"""

import math

import numpy as np
import pytest
import scipy.sparse as sp

import golden_io
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(seed, n=5000, d=3000, k=16, density=0.01):
    rng = np.random.default_rng(seed)
    X = sp.random(n, d, density=density, format="csr", random_state=seed,
                  data_rvs=lambda m: rng.lognormal(0.0, 1.0, size=m))
    ip, ix, dv = X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data
    w0, w, V = -0.2, rng.normal(size=d) * 0.3, rng.normal(size=(d, k)) * 0.2
    y = (rng.random(n) < 0.3).astype(np.float64)
    sw = rng.uniform(0.5, 2.0, size=n)
    return ip, ix, dv, w0, w, V, y, sw


def _run(case, dtype, loss, eps, weighted):
    from modern_fm_b200.evaluate import fm_eval_device

    ip, ix, dv, w0, w, V, y, sw = case
    tdt = torch.float32 if dtype == "float32" else torch.float64
    pdt = torch.float64 if dtype == "float64" else torch.float32
    c = lambda a, t: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", t)  # noqa: E731
    return fm_eval_device(c(ip, torch.int64), c(ix, torch.int32), c(dv, tdt), w0, c(w, pdt),
                          c(V, pdt), c(y, torch.float64),
                          c(sw, torch.float64) if weighted else None, loss=loss,
                          label_smoothing=eps)


def _want(case, loss, eps, weighted):
    ip, ix, dv, w0, w, V, y, sw = case
    s = O.fm_predict_fast_csr(ip, ix, dv, len(w), w0, w, V)
    if loss == "logistic":
        return O.logistic_loss(y, s, label_smoothing=eps, sample_weight=sw if weighted else None)
    return O.squared_loss(y, s, sample_weight=sw if weighted else None)


@pytest.mark.parametrize("dtype,rtol", [("float64", 1e-9), ("float32", 1e-4),
                                        ("float32-float64", 1e-9)])
@pytest.mark.parametrize("loss,eps,weighted", [("logistic", 0.0, False),
                                               ("logistic", 0.1, True),
                                               ("squared", 0.0, False),
                                               ("squared", 0.0, True)])
def test_eval_matches_oracle(dtype, rtol, loss, eps, weighted):
    case = _case(1)
    if dtype == "float32-float64":  # float32 parameters, float64 values and arithmetic
        ip, ix, dv, w0, w, V, y, sw = case
        case = (ip, ix, dv, w0, w.astype(np.float32).astype(np.float64),
                V.astype(np.float32).astype(np.float64), y, sw)
    got = _run(case, dtype, loss, eps, weighted)
    want = _want(case, loss, eps, weighted)
    assert got == pytest.approx(want, rel=rtol)


def test_eval_is_bitwise_reproducible():
    case = _case(2, n=200_000, d=20_000, density=0.0005)
    a = _run(case, "float64", "logistic", 0.0, True)
    b = _run(case, "float64", "logistic", 0.0, True)
    assert a == b and math.isfinite(a)


def test_eval_empty_and_invalid():
    case = _case(3, n=10)
    ip, ix, dv, w0, w, V, y, sw = case
    empty = (np.zeros(1, np.int64), np.zeros(0, np.int64), np.zeros(0), w0, w, V,
             np.zeros(0), np.zeros(0))
    assert math.isnan(_run(empty, "float64", "squared", 0.0, False))
    with pytest.raises(ValueError):
        _run(case, "float64", "hinge", 0.0, False)


@pytest.mark.parametrize("case", golden_io.load("losses.npz"), ids=lambda c: c.name)
@pytest.mark.parametrize("dtype,rtol", [("float64", 1e-12), ("float32", 1e-5)])
def test_device_eval_matches_reference_golden(case, dtype, rtol):
    """Against the reference's own losses.py values: one nonzero per row (its
    own feature, value 1) with w = the fixture's raw scores, w0 = 0 and V = 0,
    so each device score is the raw score (float64 exactly; float32 rounded
    once)."""
    raw = case.a["raw"]
    n, k = len(raw), 4
    c = (np.arange(n + 1, dtype=np.int64), np.arange(n, dtype=np.int64), np.ones(n), 0.0, raw,
         np.zeros((n, k)), case.a["y"], case.a["sample_weight"])
    got = _run(c, dtype, case["loss"], case["label_smoothing"], case["weighted"])
    assert got == pytest.approx(case.a["value"][0], rel=rtol)


@pytest.mark.parametrize("model", ["ffm", "fwfm"])
@pytest.mark.parametrize("dtype,rtol", [("float64", 1e-9), ("float32", 1e-4),
                                        ("float32-float64", 1e-9)])
@pytest.mark.parametrize("loss,eps,weighted", [("logistic", 0.1, True), ("squared", 0.0, False)])
def test_field_aware_eval_matches_oracle(model, dtype, rtol, loss, eps, weighted):
    from modern_fm_b200.evaluate import ffm_eval_device, fwfm_eval_device

    rng = np.random.default_rng(17)
    n, d, F, k = 3000, 600, 6, 4
    X = sp.random(n, d, density=0.01, format="csr", random_state=17,
                  data_rvs=lambda m: rng.lognormal(0.0, 0.5, size=m))
    ip, ix, dv = X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data
    fid = rng.integers(0, F, size=d)
    w0, w = 0.1, rng.normal(size=d) * 0.3
    V = rng.normal(size=(d, F, k) if model == "ffm" else (d, k)) * 0.3
    R = rng.uniform(size=(F, F))
    if dtype != "float64":
        w, V, R = (a.astype(np.float32).astype(np.float64) for a in (w, V, R))
    y = (rng.random(n) < 0.3).astype(np.float64)
    sw = rng.uniform(0.5, 2.0, size=n)
    if model == "ffm":
        s = O.ffm_predict_csr(ip, ix, dv, d, fid, w0, w, V)
    else:
        s = O.fwfm_predict_csr(ip, ix, dv, d, fid, w0, w, V, R)
    swa = sw if weighted else None
    want = (O.logistic_loss(y, s, label_smoothing=eps, sample_weight=swa) if loss == "logistic"
            else O.squared_loss(y, s, sample_weight=swa))
    tdt = torch.float32 if dtype == "float32" else torch.float64
    pdt = torch.float64 if dtype == "float64" else torch.float32
    c = lambda a, t: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", t)  # noqa: E731
    args = (c(ip, torch.int64), c(ix, torch.int32), c(dv, tdt), c(fid, torch.int32), w0,
            c(w, pdt), c(V, pdt))
    kw = dict(sample_weight=c(sw, torch.float64) if weighted else None, loss=loss,
              label_smoothing=eps)
    if model == "ffm":
        got = ffm_eval_device(*args, c(y, torch.float64), **kw)
    else:
        got = fwfm_eval_device(*args, c(R, pdt), c(y, torch.float64), **kw)
    assert got == pytest.approx(want, rel=rtol)
