"""GPU parity of the device early-stopping evaluation (mfm_fm_eval_device)
against the oracle: the reference's `metric(y_val, fm_predict_fast(X_val,
...))` (python/modern_fm/fm.py:321-322) restated on the CPU.

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
    c = lambda a, t: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", t)  # noqa: E731
    return fm_eval_device(c(ip, torch.int64), c(ix, torch.int32), c(dv, tdt), w0, c(w, tdt),
                          c(V, tdt), c(y, torch.float64),
                          c(sw, torch.float64) if weighted else None, loss=loss,
                          label_smoothing=eps)


def _want(case, loss, eps, weighted):
    ip, ix, dv, w0, w, V, y, sw = case
    s = O.fm_predict_fast_csr(ip, ix, dv, len(w), w0, w, V)
    if loss == "logistic":
        return O.logistic_loss(y, s, label_smoothing=eps, sample_weight=sw if weighted else None)
    return O.squared_loss(y, s, sample_weight=sw if weighted else None)


@pytest.mark.parametrize("dtype,rtol", [("float64", 1e-9), ("float32", 1e-4)])
@pytest.mark.parametrize("loss,eps,weighted", [("logistic", 0.0, False),
                                               ("logistic", 0.1, True),
                                               ("squared", 0.0, False),
                                               ("squared", 0.0, True)])
def test_eval_matches_oracle(dtype, rtol, loss, eps, weighted):
    case = _case(1)
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
