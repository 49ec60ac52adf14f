"""GPU parity of device-resident training (FM / FFM / FwFM, binary and
multiclass softmax, SGD / AdaGrad / Adam / FTRL) through the C ABI, against
the C oracle and the reference's NumPy golden outputs.

Tolerances: float64 compute is held to 1e-7 relative / 1e-9 absolute on every
parameter and optimizer-state array (the reference's CUDA training bar is
1e-7 / 1e-8 on final predictions, tests/test_cuda_parity.py:167-168);
float32 compute to 1e-4 relative on weights after an epoch, with an absolute
floor of 1e-4 times the array's scale; FTRL zero patterns must be identical.
"""

import numpy as np
import pytest

import golden_io
import run_cases
from modern_fm_b200 import _rust, workloads
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-7, 1e-9


def _close(got, want, key, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol, err_msg=key)


@pytest.mark.parametrize("case", golden_io.load("train_binary.npz"), ids=lambda c: c.name)
def test_train_binary_golden(case):
    got = run_cases.train_binary_case(_rust, case, use_cuda=True)
    ref = run_cases.train_binary_case(O, case, use_cuda=False)
    a = case.a
    for key in ("w0", "w", "V", "r"):
        if key in a:
            _close(got[key], a[key], key)
            _close(got[key], ref[key], key)
    if case["optimizer"] == "adagrad":
        for key in ("acc_w0", "acc_w", "acc_V"):
            _close(got[key], ref[key], key)
    for key in ("adam", "ftrl"):
        if key in ref:
            for i, (g, r) in enumerate(zip(got[key], ref[key])):
                _close(g, r, f"{key}_{i}")
    if case["optimizer"] == "ftrl":
        np.testing.assert_array_equal(got["w"] == 0.0, ref["w"] == 0.0)
        np.testing.assert_array_equal(got["V"] == 0.0, ref["V"] == 0.0)


@pytest.mark.parametrize("case", golden_io.load("train_multiclass.npz"), ids=lambda c: c.name)
def test_train_multiclass_golden(case):
    got = run_cases.train_multiclass_case(_rust, case, use_cuda=True)
    ref = run_cases.train_multiclass_case(O, case, use_cuda=False)
    for key in ("w0", "w", "V", "r"):
        if key in case.a:
            _close(got[key], case.a[key], key)
            _close(got[key], ref[key], key)


def _fm_fit(mod, X, y, sw, params, ro, bs, cuda, optimizer="adagrad", **kw):
    w0, w, V = params
    w, V = np.array(w, dtype=np.float64), np.array(V, dtype=np.float64)
    aw, av = np.zeros_like(w), np.zeros_like(V)
    hp = dict(learning_rate=0.05, l2_linear=1e-5, l2_factors=1e-5, l1_linear=0.0,
              l1_factors=0.0)
    hp.update(kw)
    res = mod.fm_fit_csr(X.indptr, X.indices, X.data, X.n_features, y, sw, w0, 0.0, w, V, aw,
                         av, "logistic", optimizer, hp["learning_rate"], hp["l2_linear"],
                         hp["l2_factors"], 0.9, 0.999, 1e-8, ro, bs, 1, hp["l1_linear"],
                         hp["l1_factors"], 1.0, use_cuda=cuda)
    return res[0], w, V, aw, av


def test_hot_features_long_runs_f64():
    """CTR-shaped rows: 13 numeric features occur in every row, so a batch of
    1000 rows has runs of 1000 entries (multi-item reduction path)."""
    X, _ = workloads.ctr_fm(n_rows=3000, seed=11, space=2**16, vocab=2**12)
    rng = np.random.default_rng(0)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    params = (0.0, np.zeros(X.n_features), rng.normal(0, 0.05, (X.n_features, 16)))
    ro = workloads.row_orders(X.n_rows, 2, seed=1)
    sw = np.ones(X.n_rows)
    got = _fm_fit(_rust, X, y, sw, params, ro, 1000, True)
    ref = _fm_fit(O, X, y, sw, params, ro, 1000, False)
    for g, r, key in zip(got, ref, ("w0", "w", "V", "acc_w", "acc_V")):
        _close(g, r, key)


def test_training_is_bitwise_deterministic():
    X, y, fid = workloads.onehot_ctr(4000, seed=0)
    rng = np.random.default_rng(0)
    params = (0.0, np.zeros(256), rng.normal(0, 0.05, (256, 16)))
    ro = workloads.row_orders(X.n_rows, 2, seed=3)
    a = _fm_fit(_rust, X, y, np.ones(X.n_rows), params, ro, 512, True)
    b = _fm_fit(_rust, X, y, np.ones(X.n_rows), params, ro, 512, True)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)


def test_epoch_by_epoch_state_handoff_equals_one_call():
    """Early-stopping drives one epoch per call, round-tripping the optimizer
    state (rust/src/lib.rs:34-77); the result equals one multi-epoch call."""
    X, y, _ = workloads.onehot_ctr(1500, seed=2)
    rng = np.random.default_rng(1)
    w_init, V_init = np.zeros(256), rng.normal(0, 0.05, (256, 8))
    ro = workloads.row_orders(X.n_rows, 3, seed=4)
    for opt in ("adagrad", "adam", "ftrl"):
        kw = dict(l1_linear=0.01, l1_factors=0.001) if opt == "ftrl" else {}
        one = _fm_fit(_rust, X, y, np.ones(X.n_rows), (0.0, w_init, V_init), ro, 64, True,
                      optimizer=opt, **kw)
        w, V = w_init.copy(), V_init.copy()
        aw, av, w0, acc0 = np.zeros(256), np.zeros((256, 8)), 0.0, 0.0
        ad = (0.0, 0.0, 0.0) + tuple(np.zeros_like(a) for a in (w, w, w, V, V, V))
        ft = (0.0, 0.0) + tuple(np.zeros_like(a) for a in (w, w, V, V))
        for e in range(3):
            res = _rust.fm_fit_csr(
                X.indptr, X.indices, X.data, 256, y, np.ones(X.n_rows), w0, acc0, w, V, aw, av,
                "logistic", opt, 0.05, 1e-5, 1e-5, 0.9, 0.999, 1e-8, ro[e:e + 1], 64, 1,
                kw.get("l1_linear", 0.0), kw.get("l1_factors", 0.0), 1.0,
                adam_state=ad if opt == "adam" else None,
                ftrl_state=ft if opt == "ftrl" else None, use_cuda=True)
            w0, acc0 = res[0], res[1]
            if opt == "adam":
                ad = tuple(res[2]) + ad[3:]
            if opt == "ftrl":
                ft = tuple(res[3]) + ft[2:]
        np.testing.assert_array_equal(w0, one[0])
        np.testing.assert_array_equal(w, one[1])
        np.testing.assert_array_equal(V, one[2])


def test_f32_fm_onehot_against_oracle(monkeypatch):
    """Config-0 shape (16 x 16 one-hot, k=16, AdaGrad 0.05, batch 512) in
    float32: weights after one epoch within 1e-4 relative of the float64
    oracle, scores within 1e-5."""
    monkeypatch.setenv("MFM_B200_DTYPE", "float32")
    X, y, _ = workloads.onehot_ctr(40000, seed=0)
    rng = np.random.default_rng(0)
    params = (0.0, np.zeros(256), rng.normal(0, 0.01, (256, 16)))
    ro = workloads.row_orders(X.n_rows, 1, seed=0)
    got = _fm_fit(_rust, X, y, np.ones(X.n_rows), params, ro, 512, True)
    ref = _fm_fit(O, X, y, np.ones(X.n_rows), params, ro, 512, False)
    for g, r, key in zip(got[:3], ref[:3], ("w0", "w", "V")):
        scale = np.max(np.abs(r))
        np.testing.assert_allclose(g, r, rtol=1e-4, atol=1e-4 * scale, err_msg=key)


def test_f32_ftrl_fwfm_zero_pattern(monkeypatch):
    """Config-3 shape (9 one-hot Zipf fields, FwFM k=8, FTRL with L1) in
    float32: the exact-zero pattern of w matches the float64 oracle."""
    monkeypatch.setenv("MFM_B200_DTYPE", "float32")
    X, y, fid = workloads.fwfm_ctr(20000, seed=3)
    rng = np.random.default_rng(3)
    d, F, k = X.n_features, 9, 8
    w, V, r = np.zeros(d), rng.normal(0, 0.01, (d, k)), np.ones((F, F))
    outs = []
    for mod, cuda in ((_rust, True), (O, False)):
        wv, Vv, rv = w.copy(), V.copy(), r.copy()
        mod.fwfm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), fid, 0.0, 0.0,
                         wv, Vv, rv, np.zeros(d), np.zeros((d, k)), np.zeros((F, F)),
                         "logistic", "ftrl", 0.05, 0.0, 0.0, 0.9, 0.999, 1e-8,
                         workloads.row_orders(X.n_rows, 1, seed=5), 1024, 1.0, 0.1, 1.0,
                         use_cuda=cuda)
        outs.append((wv, Vv, rv))
    np.testing.assert_array_equal(outs[0][0] == 0.0, outs[1][0] == 0.0)
    assert np.sum(outs[0][0] == 0.0) > 0


@pytest.mark.parametrize("dtype,opt", [("float32", "adagrad"), ("float64", "adam"),
                                       ("float32", "ftrl")])
def test_device_resident_fit_matches_host_fit(dtype, opt):
    """mfm_fm_fit_device on caller-owned device arrays gives exactly what the
    host-buffer entry point gives (same kernels, same order)."""
    import torch

    from modern_fm_b200 import _lib

    X, y, _ = workloads.onehot_ctr(3000, seed=6)
    rng = np.random.default_rng(2)
    d, k = X.n_features, 16
    w_init, V_init = rng.normal(0, 0.01, d), rng.normal(0, 0.01, (d, k))
    ro = workloads.row_orders(X.n_rows, 2, seed=8)
    kw = dict(l1_linear=0.01, l1_factors=0.001) if opt == "ftrl" else {}
    import os

    os.environ["MFM_B200_DTYPE"] = dtype
    try:
        host = _fm_fit(_rust, X, y, np.ones(X.n_rows), (0.1, w_init, V_init), ro, 256, True,
                       optimizer=opt, **kw)
    finally:
        del os.environ["MFM_B200_DTYPE"]
    tdt = torch.float32 if dtype == "float32" else torch.float64
    dev = torch.device("cuda", 0)
    t = lambda a, dt=tdt: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device=dev)  # noqa
    ip, ix, dv = t(X.indptr, torch.int64), t(X.indices, torch.int32), t(X.data)
    yy, sw, rot = t(y), t(np.ones(X.n_rows)), t(ro, torch.int32)
    w0, w, V = t([0.1]), t(w_init), t(V_init)
    hp = dict(learning_rate=0.05, l2_linear=1e-5, l2_factors=1e-5)
    tr = _lib.Train(_lib.LOSSES["logistic"], _lib.OPTIMIZERS[opt], hp["learning_rate"],
                    kw.get("l1_linear", 0.0), hp["l2_linear"], kw.get("l1_factors", 0.0),
                    hp["l2_factors"], 0.9, 0.999, 1e-8, 1.0, 0.0, None, ro.shape[0], 256)
    g = [_lib.DevGroup(a.data_ptr(), None, None, None, None, None, None) for a in (w0, w, V)]
    code = _lib.MFM_DTYPE_F32 if dtype == "float32" else _lib.MFM_DTYPE_F64
    stream = torch.cuda.current_stream(dev)
    rc = _lib.lib().mfm_fm_fit_device(code, 0, ip.data_ptr(), ix.data_ptr(), dv.data_ptr(),
                                      X.n_rows, d, yy.data_ptr(), sw.data_ptr(), rot.data_ptr(),
                                      tr, k, g[0], g[1], g[2], stream.cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert float(w0.item()) == float(np.float64(host[0]).astype(np.float32 if dtype == "float32"
                                                             else np.float64))
    np.testing.assert_array_equal(w.cpu().numpy().astype(np.float64),
                                  host[1].astype(tdt == torch.float32 and np.float32
                                                 or np.float64).astype(np.float64))
    np.testing.assert_array_equal(V.cpu().numpy().astype(np.float64),
                                  host[2].astype(tdt == torch.float32 and np.float32
                                                 or np.float64).astype(np.float64))


@pytest.mark.parametrize("opt", ["sgd", "adagrad", "adam", "ftrl"])
def test_runs_across_many_chunks_f64(opt):
    """Batches of 10,000 CTR-shaped rows: the 13 numeric features occur in
    every row, so each of their runs spans 40 chunks of 256 sorted entries
    (more chunk partials than one warp folds at once)."""
    X, _ = workloads.ctr_fm(n_rows=20000, seed=5, space=2**16, vocab=2**12)
    rng = np.random.default_rng(4)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    sw = rng.uniform(0.5, 1.5, X.n_rows)
    params = (0.0, np.zeros(X.n_features), rng.normal(0, 0.05, (X.n_features, 8)))
    ro = workloads.row_orders(X.n_rows, 1, seed=2)
    kw = dict(l1_linear=0.01, l1_factors=0.001) if opt == "ftrl" else {}
    got = _fm_fit(_rust, X, y, sw, params, ro, 10000, True, optimizer=opt, **kw)
    ref = _fm_fit(O, X, y, sw, params, ro, 10000, False, optimizer=opt, **kw)
    keys = ("w0", "w", "V", "acc_w", "acc_V") if opt == "adagrad" else ("w0", "w", "V")
    for g, r, key in zip(got, ref, keys):
        _close(g, r, key)
    if opt == "ftrl":
        np.testing.assert_array_equal(got[1] == 0.0, ref[1] == 0.0)


@pytest.mark.parametrize("opt", ["sgd", "adagrad"])
def test_runs_across_many_chunks_f32(monkeypatch, opt):
    """The 40-chunk runs in float32 (k=16, the row-table shape of the CTR
    benchmark): weights within 1e-4 relative of the float64 oracle. (Adam is
    held to the float64 bar above: its normalised first steps are +-lr for
    any nonzero gradient, so float32 rounding of a near-zero gradient moves a
    weight by up to lr.)"""
    monkeypatch.setenv("MFM_B200_DTYPE", "float32")
    X, _ = workloads.ctr_fm(n_rows=20000, seed=6, space=2**16, vocab=2**12)
    rng = np.random.default_rng(5)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    params = (0.0, np.zeros(X.n_features), rng.normal(0, 0.05, (X.n_features, 16)))
    ro = workloads.row_orders(X.n_rows, 2, seed=3)
    got = _fm_fit(_rust, X, y, np.ones(X.n_rows), params, ro, 10000, True, optimizer=opt)
    ref = _fm_fit(O, X, y, np.ones(X.n_rows), params, ro, 10000, False, optimizer=opt)
    for g, r, key in zip(got[:3], ref[:3], ("w0", "w", "V")):
        scale = np.max(np.abs(r))
        np.testing.assert_allclose(g, r, rtol=1e-4, atol=1e-4 * scale, err_msg=key)


@pytest.mark.parametrize("k", [4, 8, 16])
def test_single_feature_and_empty_batches(k):
    """One feature (a single sort key, zero key bits), rows without nonzeros
    and a batch made only of empty rows: w0 still steps every batch."""
    n = 60
    rng = np.random.default_rng(k)
    nz = np.ones(n, dtype=np.int64)
    nz[:10] = 0          # epoch 0, batch 0: all empty
    nz[25:30] = 0
    indptr = np.concatenate([[0], np.cumsum(nz)])
    X = workloads.Csr(indptr, np.zeros(int(indptr[-1]), dtype=np.int64),
                      rng.uniform(0.5, 2.0, int(indptr[-1])), 1)
    y = (rng.random(n) < 0.5).astype(np.float64)
    params = (0.2, np.array([0.1]), rng.normal(0, 0.1, (1, k)))
    ro = np.stack([np.arange(n), rng.permutation(n)])
    for opt in ("sgd", "adagrad", "adam", "ftrl"):
        got = _fm_fit(_rust, X, y, np.ones(n), params, ro, 10, True, optimizer=opt)
        ref = _fm_fit(O, X, y, np.ones(n), params, ro, 10, False, optimizer=opt)
        for g, r, key in zip(got[:3], ref[:3], ("w0", "w", "V")):
            _close(g, r, f"{opt} {key}")
