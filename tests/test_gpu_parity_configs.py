"""Parity at the benchmark configurations' shapes, through the reference-facing
`_rust` mirror (C ABI, host buffers), against the oracle fitted on the same
inputs from the same initial parameters.

Bars (the hot path's stated targets): final test AUC within 1e-3; weights
after an epoch within 1e-4 relative (absolute floor 1e-4 x the array's largest
magnitude) in float32 arithmetic, and at the float64 training bar (1e-7
relative, 1e-9 absolute) in float64; FTRL exact-zero patterns identical.
Every fit runs in float32 (the narrow mode, where these bars bite) and in the
default arithmetic (float64 training, the reference's).

Data: the seeded synthetic stand-ins of `modern_fm_b200.workloads` with the
configurations' shapes (one-hot 16 x 16 CTR for FM / FFM, 9 Zipf one-hot
fields for FwFM FTRL, ragged softmax rows for the multiclass FM, scaled down
so the oracle finishes in seconds).
"""

import numpy as np
import pytest
from sklearn.metrics import roc_auc_score

from modern_fm_b200 import _rust, workloads
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = ["float32", "float32-float64"]


def _check_weights(got, ref, dtype, keys, atol32=None):
    for g, r, key in zip(got, ref, keys):
        g, r = np.asarray(g, dtype=np.float64), np.asarray(r, dtype=np.float64)
        if dtype == "float32":
            scale = max(float(np.max(np.abs(r))), 1e-12)
            atol = 1e-4 * scale if atol32 is None else atol32
            np.testing.assert_allclose(g, r, rtol=1e-4, atol=atol, err_msg=key)
        else:
            np.testing.assert_allclose(g, r, rtol=1e-7, atol=1e-9, err_msg=key)


# --------------------------------------------------------- C0 / C1: one-hot --

def _onehot():
    """40k training and 20k test rows of one draw (the same planted field-pair
    tables), as configuration 0 describes."""
    X, y, fid = workloads.onehot_ctr(60000, 0)
    return X.rows(0, 40000), y[:40000], X.rows(40000, 60000), y[40000:], fid


def _fit_fm(mod, cuda, Xtr, ytr, V0, epochs, ro):
    d = Xtr.n_features
    w, V = np.zeros(d), V0.copy()
    res = mod.fm_fit_csr(Xtr.indptr, Xtr.indices, Xtr.data, d, ytr, np.ones(Xtr.n_rows), 0.0,
                         0.0, w, V, np.zeros(d), np.zeros_like(V), "logistic", "adagrad", 0.05,
                         1e-5, 1e-5, 0.9, 0.999, 1e-8, ro[:epochs], 512, 4, 0.0, 0.0, 1.0,
                         use_cuda=cuda)
    return res[0], w, V


def _fit_ffm(mod, cuda, Xtr, ytr, fid, V0, epochs, ro):
    d = Xtr.n_features
    w, V = np.zeros(d), V0.copy()
    res = mod.ffm_fit_csr(Xtr.indptr, Xtr.indices, Xtr.data, d, ytr, np.ones(Xtr.n_rows), fid,
                          0.0, 0.0, w, V, np.zeros(d), np.zeros_like(V), "logistic", "adagrad",
                          0.05, 1e-5, 1e-5, 0.9, 0.999, 1e-8, ro[:epochs], 512, 4, 0.0, 0.0, 1.0,
                          use_cuda=cuda)
    return res[0], w, V


@pytest.mark.parametrize("dtype", DTYPES)
def test_c0_fm_auc_and_weights(dtype, monkeypatch):
    """Config 0: FM k=16, AdaGrad 0.05, batch 512, 10 epochs, L2 1e-5."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    Xtr, ytr, Xte, yte, _ = _onehot()
    V0 = np.random.default_rng(0).normal(0, 0.01, (256, 16))
    ro = workloads.row_orders(Xtr.n_rows, 10, 1)
    # one epoch: weights
    _check_weights(_fit_fm(_rust, True, Xtr, ytr, V0, 1, ro),
                   _fit_fm(O, False, Xtr, ytr, V0, 1, ro), dtype, ("w0", "w", "V"))
    # ten epochs: test AUC
    g = _fit_fm(_rust, True, Xtr, ytr, V0, 10, ro)
    r = _fit_fm(O, False, Xtr, ytr, V0, 10, ro)
    sg = O.fm_predict_fast_csr(Xte.indptr, Xte.indices, Xte.data, 256, *g)
    sr = O.fm_predict_fast_csr(Xte.indptr, Xte.indices, Xte.data, 256, *r)
    a_g, a_r = roc_auc_score(yte, sg), roc_auc_score(yte, sr)
    assert abs(a_g - a_r) <= 1e-3, (a_g, a_r)
    assert a_r > 0.7  # the planted interactions are learnt


@pytest.mark.parametrize("dtype", DTYPES)
def test_c1_ffm_auc_and_weights(dtype, monkeypatch):
    """Config 1: FFM k=8 on the same data, field = feature // 16, AdaGrad
    0.05, batch 512, 10 epochs."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    Xtr, ytr, Xte, yte, fid = _onehot()
    V0 = np.random.default_rng(1).uniform(0, 0.1, (256, 16, 8))
    ro = workloads.row_orders(Xtr.n_rows, 10, 1)
    _check_weights(_fit_ffm(_rust, True, Xtr, ytr, fid, V0, 1, ro),
                   _fit_ffm(O, False, Xtr, ytr, fid, V0, 1, ro), dtype, ("w0", "w", "V"))
    g = _fit_ffm(_rust, True, Xtr, ytr, fid, V0, 10, ro)
    r = _fit_ffm(O, False, Xtr, ytr, fid, V0, 10, ro)
    sg = O.ffm_predict_csr(Xte.indptr, Xte.indices, Xte.data, 256, fid, *g)
    sr = O.ffm_predict_csr(Xte.indptr, Xte.indices, Xte.data, 256, fid, *r)
    a_g, a_r = roc_auc_score(yte, sg), roc_auc_score(yte, sr)
    assert abs(a_g - a_r) <= 1e-3, (a_g, a_r)
    assert a_r > 0.7


# ----------------------------------------------------------- C3: FwFM FTRL --

def _fit_fwfm(mod, cuda, X, y, fid, V0, ro):
    d, F, k = X.n_features, 9, 8
    w, V, r = np.zeros(d), V0.copy(), np.ones((F, F))
    res = mod.fwfm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), fid, 0.0, 0.0,
                           w, V, r, np.zeros(d), np.zeros((d, k)), np.zeros((F, F)), "logistic",
                           "ftrl", 0.05, 0.0, 0.0, 0.9, 0.999, 1e-8, ro, 1024, 1.0, 0.1, 1.0,
                           use_cuda=cuda)
    return res[0], w, V, r


@pytest.mark.parametrize("dtype", DTYPES)
def test_c3_fwfm_ftrl_zero_pattern_weights_and_auc(dtype, monkeypatch):
    """Config 3: FwFM k=8, FTRL-Proximal (alpha 0.05, beta 1, l1 1.0 / 0.1),
    batch 1024, 9 one-hot Zipf fields; 160k training rows, 40k test rows."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    X, y, fid = workloads.fwfm_ctr(200000, seed=3)
    n_tr = 160000
    Xtr, ytr = X.rows(0, n_tr), y[:n_tr]
    Xte, yte = X.rows(n_tr, X.n_rows), y[n_tr:]
    V0 = np.random.default_rng(3).normal(0, 0.01, (X.n_features, 8))
    ro = workloads.row_orders(n_tr, 1, seed=5)
    g = _fit_fwfm(_rust, True, Xtr, ytr, fid, V0, ro)
    r = _fit_fwfm(O, False, Xtr, ytr, fid, V0, ro)
    for key, a, b in (("w", g[1], r[1]), ("V", g[2], r[2])):
        np.testing.assert_array_equal(a == 0.0, b == 0.0, err_msg=f"{key} zero pattern")
    assert np.sum(r[1] == 0.0) > 0 and np.sum(r[2] == 0.0) > 0
    _check_weights(g, r, dtype, ("w0", "w", "V", "r"))
    d = X.n_features
    sg = O.fwfm_predict_csr(Xte.indptr, Xte.indices, Xte.data, d, fid, *g)
    sr = O.fwfm_predict_csr(Xte.indptr, Xte.indices, Xte.data, d, fid, *r)
    a_g, a_r = roc_auc_score(yte, sg), roc_auc_score(yte, sr)
    assert abs(a_g - a_r) <= 1e-3, (a_g, a_r)


# ------------------------------------------------ C4: softmax multiclass FM --

@pytest.mark.parametrize("dtype", DTYPES)
def test_c4_softmax_fm_adam_weights(dtype, monkeypatch):
    """Config 4 scaled down: softmax FM C=10, k=8, Adam 1e-3, batch 2048,
    ragged rows (Poisson(30)+1), LogNormal values, sample weights U(0.5, 2),
    label smoothing 0.1; 60k rows over 200k features, one epoch.

    In float32 the absolute floor is 0.1 x the learning rate: Adam's step is
    lr m / (sqrt(s) + eps), about +-lr whatever the gradient's size, so a
    coordinate whose few gradients are near zero (a handful among 16M) can
    move by up to lr on a float32 rounding of those gradients."""
    monkeypatch.setenv("MFM_B200_DTYPE", dtype)
    X, yc, sw = workloads.softmax_ctr(60000, 4, n_features=200_000)
    C, k, d = 10, 8, X.n_features
    V0 = np.random.default_rng(4).normal(0, 0.01, (C, d, k))
    ro = workloads.row_orders(X.n_rows, 1, 6)
    outs = []
    for mod, cuda in ((_rust, True), (O, False)):
        w0, w, V = np.zeros(C), np.zeros((C, d)), V0.copy()
        mod.fm_fit_multiclass_csr(X.indptr, X.indices, X.data, d, yc, sw, w0, w, V, "adam",
                                  1e-3, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, ro, 2048, 0.0, 0.0,
                                  1.0, use_cuda=cuda)
        outs.append((w0, w, V))
    _check_weights(outs[0], outs[1], dtype, ("w0", "w", "V"), atol32=0.1 * 1e-3)
