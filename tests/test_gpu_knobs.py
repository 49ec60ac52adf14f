"""The engine's execution switches change scheduling, not arithmetic: a fit
under each must equal the default fit bit for bit. The switches are read once
per process, so every variant runs in its own subprocess.

  MFM_B200_PDL=0                 plain stream order instead of programmatic launch
  MFM_B200_PLAN_OVERLAP=0        the plan as one window before the batches, on
                                 their stream (default: windows on a second stream)
  MFM_B200_PLAN_WINDOW=2         two-batch plan windows (default 128)
  MFM_B200_PLAN_BLOCKS_PER_SM=0  uncapped sort grids beside the batches (default 4)
  MFM_B200_EPOCH_KERNEL=1        one cooperative launch per epoch (payload path)
"""

import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import sys, numpy as np
sys.path.insert(0, {root!r})
from modern_fm_b200 import _rust, workloads
kind, out = sys.argv[1], sys.argv[2]
if kind == "binary":      # row-table path: binary FM, k = 16
    X, _ = workloads.ctr_fm(n_rows=3000, seed=7, space=2**15, vocab=2**10)
    rng = np.random.default_rng(1)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    d = X.n_features
    w, V = np.zeros(d), rng.normal(0, 0.05, (d, 16))
    ro = workloads.row_orders(X.n_rows, 2, seed=2)
    res = _rust.fm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), 0.0, 0.0, w, V,
                           np.zeros(d), np.zeros_like(V), "logistic", "adagrad", 0.05, 1e-5, 1e-5,
                           0.9, 0.999, 1e-8, ro, 256, 1, 0.0, 0.0, 1.0, use_cuda=True)
    np.savez(out, w0=res[0], w=w, V=V)
elif kind == "barrier":   # epoch kernel with a block that never arrives, then a clean fit
    import os, time
    X, yc, sw = workloads.softmax_ctr(2000, 9, n_features=5000, n_classes=4, mean_nnz=12)
    rng = np.random.default_rng(3)
    C, k, d = 4, 8, X.n_features
    ro = workloads.row_orders(X.n_rows, 1, seed=4)
    def fit():
        w0, w, V = np.zeros(C), np.zeros((C, d)), rng.normal(0, 0.05, (C, d, k))
        _rust.fm_fit_multiclass_csr(X.indptr, X.indices, X.data, d, yc, sw, w0, w, V, "adagrad",
                                    0.05, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, ro, 128, 0.0, 0.0,
                                    1.0, use_cuda=True)
        return V
    t = time.perf_counter()
    try:
        fit()
        msg = "no error"
    except ValueError as e:
        msg = str(e)
    dt = time.perf_counter() - t
    del os.environ["MFM_B200_EPOCH_DROP_BLOCK"]
    V = fit()
    np.savez(out, failed_s=dt, ok=np.isfinite(V).all(), msg=np.array(msg))
else:                     # payload path: softmax FM, 4 classes
    X, yc, sw = workloads.softmax_ctr(2000, 9, n_features=5000, n_classes=4, mean_nnz=12)
    rng = np.random.default_rng(3)
    C, k, d = 4, 8, X.n_features
    w0, w, V = np.zeros(C), np.zeros((C, d)), rng.normal(0, 0.05, (C, d, k))
    ro = workloads.row_orders(X.n_rows, 2, seed=4)
    _rust.fm_fit_multiclass_csr(X.indptr, X.indices, X.data, d, yc, sw, w0, w, V, "adagrad",
                                0.05, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, ro, 128, 0.0, 0.0, 1.0,
                                use_cuda=True)
    np.savez(out, w0=w0, w=w, V=V)
"""


def _run(kind, env_extra, d):
    out = os.path.join(d, f"{kind}_{'_'.join(sorted(env_extra)) or 'default'}.npz")
    env = dict(os.environ)
    for key in ("MFM_B200_PDL", "MFM_B200_PLAN_OVERLAP", "MFM_B200_PLAN_WINDOW",
                "MFM_B200_PLAN_BLOCKS_PER_SM", "MFM_B200_EPOCH_KERNEL",
                "MFM_B200_EPOCH_SPIN_LIMIT", "MFM_B200_EPOCH_DROP_BLOCK"):
        env.pop(key, None)
    env.update(env_extra)
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(root=ROOT), kind, out], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return dict(np.load(out))


@pytest.mark.parametrize("kind,env_extra", [
    ("binary", {"MFM_B200_PDL": "0"}),
    ("binary", {"MFM_B200_PLAN_OVERLAP": "0"}),
    ("binary", {"MFM_B200_PLAN_WINDOW": "2", "MFM_B200_PLAN_BLOCKS_PER_SM": "1"}),
    ("binary", {"MFM_B200_PLAN_BLOCKS_PER_SM": "0"}),
    ("multiclass", {"MFM_B200_EPOCH_KERNEL": "1"}),
])
def test_switch_is_bitwise_neutral(kind, env_extra):
    with tempfile.TemporaryDirectory() as d:
        base = _run(kind, {}, d)
        other = _run(kind, env_extra, d)
    for key in base:
        np.testing.assert_array_equal(base[key], other[key], err_msg=key)


def test_epoch_barrier_timeout_ends_the_launch():
    """A block that never arrives at the persistent epoch kernel's grid
    barrier (a lost block, made on the host through MFM_B200_EPOCH_DROP_BLOCK)
    makes the other blocks' bounded waits give up after
    MFM_B200_EPOCH_SPIN_LIMIT polls; every block then leaves the launch, the
    fit returns MFM_ERR_DEVICE_CHECK within seconds, and the process's next fit
    on the same GPU succeeds."""
    with tempfile.TemporaryDirectory() as d:
        r = _run("barrier", {"MFM_B200_EPOCH_KERNEL": "1", "MFM_B200_EPOCH_SPIN_LIMIT": "20000",
                             "MFM_B200_EPOCH_DROP_BLOCK": "0"}, d)
    assert "grid barrier" in str(r["msg"])
    assert float(r["failed_s"]) < 30.0
    assert bool(r["ok"])
