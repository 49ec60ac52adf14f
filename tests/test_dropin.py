"""The engine composed beneath the reference's unchanged Python package.

Runs where the reference's python/ tree is available: set MFM_REFERENCE_PYTHON
to that directory; without it the tests that need the package are skipped. CPU only: the CPU
entry points are served by the C oracle standing in for the reference's Rust
engine, and the CUDA entry points report no device here.
"""

import importlib
import os
import sys

import numpy as np
import pytest

from modern_fm_b200 import dropin
from oracle import oracle as O

REF = os.environ.get("MFM_REFERENCE_PYTHON", "")


def test_composed_module_has_the_reference_surface():
    mod = dropin.make_rust_module(O)
    # rust/src/lib.rs:1592-1614
    for n in ("has_cuda", "fm_predict_cuda_csr", "ffm_predict_cuda_csr", "fwfm_predict_cuda_csr",
              "fm_predict_fast_dense", "fm_predict_fast_csr", "ffm_predict_dense",
              "ffm_predict_csr", "fwfm_predict_dense", "fwfm_predict_csr", "fm_fit_csr",
              "fm_fit_multiclass_csr", "ffm_fit_csr", "ffm_fit_multiclass_csr", "fwfm_fit_csr",
              "fwfm_fit_multiclass_csr"):
        assert callable(getattr(mod, n)), n


@pytest.fixture
def reference_pkg():
    if not REF or not os.path.isdir(os.path.join(REF, "modern_fm")):
        pytest.skip("reference python package not available (set MFM_REFERENCE_PYTHON)")
    saved = {k: v for k, v in sys.modules.items() if k == "modern_fm" or k.startswith("modern_fm.")}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, REF)
    try:
        dropin.install(cpu_backend=O)
        pkg = importlib.import_module("modern_fm")
        yield pkg
    finally:
        sys.path.remove(REF)
        for k in [k for k in sys.modules if k == "modern_fm" or k.startswith("modern_fm.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_reference_estimators_run_through_the_composed_module(reference_pkg):
    from modern_fm import FMClassifier, _backend, _reference_train

    assert _backend.has_rust()
    rng = np.random.default_rng(0)
    X = rng.normal(size=(120, 10))
    X[rng.random(size=X.shape) > 0.4] = 0.0
    y = (X @ rng.normal(size=10) > 0).astype(int)
    common = dict(n_factors=4, max_iter=3, random_state=0, batch_size=8, dtype="float64")
    m = FMClassifier(**common).fit(X, y)
    got = m.decision_function(X)
    # the same fit through the reference's NumPy trainer (its _rust-less path)
    composed = _backend._rust
    _backend._rust = None
    try:
        want = FMClassifier(**common).fit(X, y).decision_function(X)
    finally:
        _backend._rust = composed
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-12)
    assert _reference_train is not None


def test_backend_cuda_without_a_device_is_a_runtime_error(reference_pkg):
    from modern_fm import FMClassifier, _backend

    if _backend.has_cuda():
        pytest.skip("a CUDA device is present")
    X = np.eye(4)
    with pytest.raises(RuntimeError, match="cuda"):
        FMClassifier(backend="cuda").fit(X, np.array([0, 1, 0, 1]))
