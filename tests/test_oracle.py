"""Pin the C oracle: the reference's own known-answer vectors and the golden
fixtures made from its NumPy ground truth. CPU only."""

import numpy as np
import pytest

import golden_io
import run_cases
from oracle import oracle as O

PRED_RTOL = 1e-12  # rust<->numpy predict tolerance, tests/test_rust_parity.py:19-20
TRAIN_RTOL = 1e-9  # rust<->numpy train tolerance, tests/test_rust_train_parity.py:29-30


def _csr1(x):
    x = np.asarray(x, dtype=np.float64)[None, :]
    idx = np.nonzero(x[0])[0]
    return np.array([0, len(idx)], np.int64), idx.astype(np.int64), x[0, idx]


# ---- known answers: rust/src/{fm,ffm,fwfm,optimizer}.rs tests; tests/test_*_correctness.py


def test_fm_known_answer_4_25():
    # rust/src/fm.rs:433-441; tests/test_fm_correctness.py:38-45
    w0, w, V = 0.25, np.array([0.5, -1.0]), np.array([[1.0, 0.0], [1.0, 1.0]])
    out = O.fm_predict_fast_dense(np.array([[2.0, 3.0]]), w0, w, V)
    assert abs(out[0] - 4.25) < 1e-12
    out = O.fm_predict_fast_csr(*_csr1([2.0, 3.0]), 2, w0, w, V)
    assert abs(out[0] - 4.25) < 1e-12


def test_fm_zero_row_is_bias():
    # rust/src/fm.rs:444-447
    out = O.fm_predict_fast_dense(np.zeros((1, 3)), 1.5, np.ones(3), np.ones((3, 2)))
    assert out[0] == 1.5


def test_ffm_known_answer_9_5():
    # rust/src/ffm.rs:454-474; tests/test_ffm_correctness.py:6-23
    V = np.zeros((3, 2, 2))
    V[0, 0], V[0, 1] = [1.0, 0.0], [0.0, 1.0]
    V[1, 0], V[1, 1] = [1.0, 1.0], [2.0, 0.0]
    V[2, 0], V[2, 1] = [0.5, 0.5], [1.0, -1.0]
    fid = np.array([0, 0, 1])
    out = O.ffm_predict_dense(np.array([[1.0, 2.0, 3.0]]), fid, 0.0, np.zeros(3), V)
    assert abs(out[0] - 9.5) < 1e-12
    out = O.ffm_predict_csr(*_csr1([1.0, 2.0, 3.0]), 3, fid, 0.0, np.zeros(3), V)
    assert abs(out[0] - 9.5) < 1e-12


def test_ffm_single_nonzero_has_no_pairwise():
    # rust/src/ffm.rs:476-483
    out = O.ffm_predict_dense(np.array([[0.0, -1.5, 0.0]]), np.array([0, 1, 1]), 0.5,
                              np.array([0.0, 2.0, 0.0]), np.full((3, 2, 2), 7.0))
    assert abs(out[0] - (0.5 + 2.0 * -1.5)) < 1e-12


def test_fwfm_known_answers():
    # rust/src/fwfm.rs:401-420; tests/test_fwfm.py:44-51
    w0, w, V = 0.25, np.array([0.5, -1.0]), np.array([[1.0, 0.0], [1.0, 1.0]])
    r = np.ones((2, 2))
    out = O.fwfm_predict_dense(np.array([[2.0, 3.0]]), np.array([0, 1]), w0, w, V, r)
    assert abs(out[0] - 4.25) < 1e-12
    r[0, 1] = 2.0
    out = O.fwfm_predict_dense(np.array([[2.0, 3.0]]), np.array([0, 1]), w0, w, V, r)
    assert abs(out[0] - 10.25) < 1e-12


def _fit1(optimizer, lr=1.0):
    w, v, aw, av = np.zeros(1), np.zeros((1, 1)), np.zeros(1), np.zeros((1, 1))
    ad = (0.0, 0.0, 0.0, np.zeros(1), np.zeros(1), np.zeros(1), np.zeros((1, 1)),
          np.zeros((1, 1)), np.zeros((1, 1))) if optimizer == "adam" else None
    res = O.fm_fit_csr(np.array([0, 1]), np.array([0]), np.array([1.0]), 1, np.array([1.0]),
                       np.array([1.0]), 0.0, 0.0, w, v, aw, av, "logistic", optimizer, lr, 0.0,
                       0.0, 0.9, 0.999, 1e-8, np.array([[0]]), 1, 1, 0.0, 0.0, 1.0,
                       adam_state=ad)
    return res, w, v


def test_one_sgd_step_hand_computed():
    # rust/src/fm.rs:450-468: s=0, g=-0.5 -> w0 = w = 0.5, V stays 0
    res, w, v = _fit1("sgd")
    assert abs(res[0] - 0.5) < 1e-15 and abs(w[0] - 0.5) < 1e-15 and v[0, 0] == 0.0


def test_adam_one_step_hand_computed():
    # rust/src/fm.rs:471-491: w0, w ~= +1, V stays 0, t = 1
    res, w, v = _fit1("adam")
    assert abs(res[0] - 1.0) < 1e-6 and abs(w[0] - 1.0) < 1e-6 and v[0, 0] == 0.0
    assert res[2][2] == 1.0


def test_multiclass_one_sgd_step_hand_computed():
    # rust/src/fm.rs:494-516
    w0, w, v = np.zeros(2), np.zeros((2, 1)), np.zeros((2, 1, 1))
    O.fm_fit_multiclass_csr(np.array([0, 1]), np.array([0]), np.array([1.0]), 1, np.array([0]),
                            np.array([1.0]), w0, w, v, "sgd", 1.0, 0.0, 0.0, 0.0, 0.9, 0.999,
                            1e-8, np.array([[0]]), 1, 0.0, 0.0, 1.0)
    np.testing.assert_allclose(w0, [0.5, -0.5], atol=1e-15)
    np.testing.assert_allclose(w[:, 0], [0.5, -0.5], atol=1e-15)
    assert np.all(v == 0.0)


def test_optimizer_primitives():
    # rust/src/optimizer.rs:466-509
    assert abs(O.sigmoid(0.0) - 0.5) < 1e-15
    assert O.sigmoid(40.0) > 0.999999 and O.sigmoid(-40.0) < 1e-6
    import ctypes as ct

    th, z, n = ct.c_double(0.0), ct.c_double(0.0), ct.c_double(0.0)
    O.lib().orc_ftrl_step(ct.byref(th), ct.c_double(2.0), ct.byref(z), ct.byref(n),
                          ct.c_double(1.0), ct.c_double(1.0), ct.c_double(0.0), ct.c_double(0.0))
    assert abs(th.value + 2.0 / 3.0) < 1e-12 and n.value == 4.0 and abs(z.value - 2.0) < 1e-12
    th, z, n = ct.c_double(0.0), ct.c_double(0.0), ct.c_double(0.0)
    O.lib().orc_ftrl_step(ct.byref(th), ct.c_double(0.5), ct.byref(z), ct.byref(n),
                          ct.c_double(1.0), ct.c_double(1.0), ct.c_double(1.0), ct.c_double(0.0))
    assert th.value == 0.0
    th, m, v, t = (ct.c_double(0.0) for _ in range(4))
    O.lib().orc_adam_step(ct.byref(th), ct.c_double(2.0), ct.byref(m), ct.byref(v),
                          ct.byref(t), ct.c_double(0.1), ct.c_double(0.9), ct.c_double(0.999),
                          ct.c_double(1e-8))
    assert abs(th.value + 0.1) < 1e-6 and t.value == 1.0


def test_full_batch_is_one_averaged_sgd_step():
    # tests/test_training_reference.py:122-140
    rng = np.random.default_rng(0)
    n, d, lr = 50, 6, 0.05
    X = rng.normal(size=(n, d))
    y = (rng.normal(size=n) > 0).astype(np.float64)
    w, V = np.zeros(d), rng.normal(0.0, 0.02, size=(d, 3))
    w_init, V_init = w.copy(), V.copy()
    ip = np.arange(0, n * d + 1, d, dtype=np.int64)
    ix = np.tile(np.arange(d), n).astype(np.int64)
    res = O.fm_fit_csr(ip, ix, X.ravel(), d, y, np.ones(n), 0.0, 0.0, w, V, np.zeros(d),
                       np.zeros_like(V), "logistic", "sgd", lr, 0.0, 0.0, 0.9, 0.999, 1e-8,
                       np.arange(n)[None, :], n, 1, 0.0, 0.0, 1.0)
    s = O.fm_predict_fast_dense(X, 0.0, w_init, V_init)
    g = 1.0 / (1.0 + np.exp(-s)) - y
    assert np.isclose(res[0], -lr * g.mean())
    np.testing.assert_allclose(w, -lr * (g[:, None] * X).mean(axis=0))


# ---- golden fixtures from the NumPy reference


@pytest.mark.parametrize("case", golden_io.load("predict.npz"), ids=lambda c: c.name)
def test_oracle_predict_golden(case):
    got = run_cases.predict_case(O, case, cuda=False)
    np.testing.assert_allclose(got, case.a["out"], rtol=PRED_RTOL, atol=PRED_RTOL)
    X = case.dense()
    a = case.a
    if case["model"] == "fm":
        dense = O.fm_predict_fast_dense(X, case["w0"], a["w"], a["V"])
        np.testing.assert_allclose(got, a["out_naive"], rtol=1e-10, atol=1e-10)
    elif case["model"] == "ffm":
        dense = O.ffm_predict_dense(X, a["field_ids"], case["w0"], a["w"], a["V"])
    else:
        dense = O.fwfm_predict_dense(X, a["field_ids"], case["w0"], a["w"], a["V"], a["r"])
    np.testing.assert_array_equal(dense, got)


@pytest.mark.parametrize("case", golden_io.load("train_binary.npz"), ids=lambda c: c.name)
def test_oracle_train_binary_golden(case):
    got = run_cases.train_binary_case(O, case, use_cuda=False)
    a = case.a
    for key in ("w0", "w", "V", "r"):
        if key in a:
            np.testing.assert_allclose(got[key], a[key], rtol=TRAIN_RTOL, atol=1e-12,
                                       err_msg=key)
    if "acc_w" in a and case["optimizer"] == "adagrad":
        np.testing.assert_allclose(got["acc_w0"], a["acc_w0"], rtol=TRAIN_RTOL)
        np.testing.assert_allclose(got["acc_w"], a["acc_w"], rtol=TRAIN_RTOL, atol=1e-15)
        np.testing.assert_allclose(got["acc_V"], a["acc_V"], rtol=TRAIN_RTOL, atol=1e-15)
    if "adam_0" in a:
        for i in range(9):
            np.testing.assert_allclose(got["adam"][i], a[f"adam_{i}"], rtol=TRAIN_RTOL,
                                       atol=1e-15, err_msg=f"adam_{i}")
    if "ftrl_0" in a:
        for i in range(6):
            np.testing.assert_allclose(got["ftrl"][i], a[f"ftrl_{i}"], rtol=TRAIN_RTOL,
                                       atol=1e-15, err_msg=f"ftrl_{i}")
        # FTRL exact-zero pattern is identical (tests/test_cuda_parity.py:266-276)
        np.testing.assert_array_equal(got["w"] == 0.0, a["w"] == 0.0)


@pytest.mark.parametrize("case", golden_io.load("train_multiclass.npz"), ids=lambda c: c.name)
def test_oracle_train_multiclass_golden(case):
    got = run_cases.train_multiclass_case(O, case, use_cuda=False)
    for key in ("w0", "w", "V", "r"):
        if key in case.a:
            np.testing.assert_allclose(got[key], case.a[key], rtol=TRAIN_RTOL, atol=1e-12,
                                       err_msg=key)


@pytest.mark.parametrize("model", ["fm", "ffm"])
def test_oracle_n_jobs_chunked_is_reproducible_and_close(model):
    """n_jobs>1 splits each batch into contiguous chunks merged in chunk order
    (rust/src/fm.rs:286-311): reproducible for a fixed n_jobs, and equal to the
    serial path up to float summation order."""
    case = next(c for c in golden_io.load("train_binary.npz")
                if c["model"] == model and c["optimizer"] == "adagrad"
                and c["batch_size"] > 1 and c.get("loss") == "logistic")
    serial = run_cases.train_binary_case(O, case, use_cuda=False, n_jobs=1)
    par1 = run_cases.train_binary_case(O, case, use_cuda=False, n_jobs=3)
    par2 = run_cases.train_binary_case(O, case, use_cuda=False, n_jobs=3)
    np.testing.assert_array_equal(par1["V"], par2["V"])
    np.testing.assert_allclose(par1["V"], serial["V"], rtol=1e-9, atol=1e-12)


def test_oracle_validation_errors():
    with pytest.raises(ValueError, match="indptr must start at 0 and end at nnz"):
        O.fm_predict_fast_csr(np.array([0, 2]), np.array([0]), np.array([1.0]), 2, 0.0,
                              np.zeros(2), np.zeros((2, 2)))
    with pytest.raises(ValueError, match="column index out of range"):
        O.fm_predict_fast_csr(np.array([0, 1]), np.array([5]), np.array([1.0]), 2, 0.0,
                              np.zeros(2), np.zeros((2, 2)))
    with pytest.raises(ValueError, match="field id out of range"):
        O.ffm_predict_csr(np.array([0, 1]), np.array([1]), np.array([1.0]), 2, np.array([0, 9]),
                          0.0, np.zeros(2), np.zeros((2, 2, 2)))
