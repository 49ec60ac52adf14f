"""Small workloads of each kernel family for profiling runs (ncu).

    python -m modern_fm_b200.profile_cases CASE [--rows N] [--dtype D] [--reps R]

Each case builds one seeded synthetic input with the shape of a benchmark
configuration, runs the engine once to warm up and then R more times, and
prints one JSON line with the mean wall time per repetition (host clock, for
orientation only: profiles take kernel durations from ncu). Cases:

  score-fm        FM scoring, CTR-shaped 39 fields, 2^22 features, k=16
  score-ffm       FFM scoring, 16 one-hot fields x 16, k=8
  score-fwfm      FwFM scoring, 9 Zipf one-hot fields (~373k features), k=8
  score-softmax   softmax FM scoring, C=10, k=8, ragged rows over 1M features
  train-fm        binary FM AdaGrad epoch, CTR-shaped, batch 4096, k=16
  train-ffm       FFM AdaGrad epoch, one-hot 16 x 16, batch 512, k=8
  train-fwfm      FwFM FTRL epoch, 9 Zipf fields, batch 1024, k=8
  train-softmax   softmax FM Adam epoch, C=10, k=8, batch 2048
  eval            FM validation loss on the device (logistic, weighted)
  prep            device CSR canonicalisation, canonical and unsorted input

Scoring and eval run in float32 parameters with float64 arithmetic unless
--dtype says otherwise; training runs in float64 unless --dtype float32.
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np


def _t(a, dt, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)


def _r32(a):
    return np.asarray(a, dtype=np.float32).astype(np.float64)


def _score_case(kind, rows, dtype, reps, dev):
    import torch

    from . import workloads as WL
    from .model import DeviceModel

    rng = np.random.default_rng(0)
    C, F, fid, R = 1, 0, None, None
    if kind == "fm":
        X, _ = WL.ctr_fm(rows, 2)
        k = 16
    elif kind == "ffm":
        X, _, fid = WL.onehot_ctr(rows, 7)
        F, k = 16, 8
    elif kind == "fwfm":
        X, _, fid = WL.fwfm_ctr(rows, 13, labels=False)
        F, k = 9, 8
        R = _r32(rng.uniform(size=(F, F)))
    else:
        X, _, _ = WL.softmax_ctr(rows, 4, score_fn=lambda Xs, *a: np.zeros(Xs.n_rows))
        C, k = 10, 8
    d = X.n_features
    lead = (C,) if C > 1 else ()
    w0 = rng.normal(size=C) if C > 1 else -0.5
    w = _r32(rng.normal(0, 0.1, lead + (d,)))
    V = _r32(rng.normal(0, 0.1, lead + ((d, F, k) if kind == "ffm" else (d, k))))
    m = DeviceModel(kind if kind != "softmax" else "fm", d, k, n_fields=F, n_classes=C,
                    dtype=dtype, device=dev.index or 0)
    m.set_params(w0, w, V, R, fid)
    vdt = torch.float32 if dtype == "float32" else torch.float64
    ip, ix, dv = _t(X.indptr, torch.int64, dev), _t(X.indices, torch.int32, dev), _t(
        X.data, vdt, dev)
    out = torch.empty((X.n_rows, C) if C > 1 else (X.n_rows,), dtype=vdt, device=dev)
    m.predict_device(ip, ix, dv, out)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        m.predict_device(ip, ix, dv, out)
    torch.cuda.synchronize()
    return {"rows": X.n_rows, "nnz": X.nnz, "dtype_used": m.dtype_used,
            "s_per_rep": (time.perf_counter() - t) / reps}


def _train_case(kind, rows, dtype, reps):
    import os

    from . import _rust
    from . import workloads as WL

    os.environ["MFM_B200_DTYPE"] = "float32" if dtype == "float32" else "float64"
    rng = np.random.default_rng(0)
    if kind == "fm":
        X, y = WL.ctr_fm(rows, 2, labels=True)
        d, k, B = X.n_features, 16, 4096
        ro = WL.row_orders(X.n_rows, 1, 1)

        def fit():
            w, V = np.zeros(d), rng.normal(0, 0.01, (d, k))
            _rust.fm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), 0.0, 0.0, w,
                             V, np.zeros(d), np.zeros_like(V), "logistic", "adagrad", 0.05, 1e-5,
                             1e-5, 0.9, 0.999, 1e-8, ro, B, 1, 0.0, 0.0, 1.0, use_cuda=True)
    elif kind == "ffm":
        X, y, fid = WL.onehot_ctr(rows, 0)
        d, F, k = 256, 16, 8
        ro = WL.row_orders(X.n_rows, 1, 1)

        def fit():
            w, V = np.zeros(d), rng.uniform(0, 0.1, (d, F, k))
            _rust.ffm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), fid, 0.0,
                              0.0, w, V, np.zeros(d), np.zeros_like(V), "logistic", "adagrad",
                              0.05, 1e-5, 1e-5, 0.9, 0.999, 1e-8, ro, 512, 1, 0.0, 0.0, 1.0,
                              use_cuda=True)
    elif kind == "fwfm":
        X, y, fid = WL.fwfm_ctr(rows, 3)
        d, F, k = X.n_features, 9, 8
        ro = WL.row_orders(X.n_rows, 1, 5)

        def fit():
            w, V, R = np.zeros(d), rng.normal(0, 0.01, (d, k)), np.ones((F, F))
            _rust.fwfm_fit_csr(X.indptr, X.indices, X.data, d, y, np.ones(X.n_rows), fid, 0.0,
                               0.0, w, V, R, np.zeros(d), np.zeros((d, k)), np.zeros((F, F)),
                               "logistic", "ftrl", 0.05, 0.0, 0.0, 0.9, 0.999, 1e-8, ro, 1024,
                               1.0, 0.1, 1.0, use_cuda=True)
    else:
        X, y, sw = WL.softmax_ctr(rows, 4, n_features=200_000)
        C, k, d = 10, 8, X.n_features
        ro = WL.row_orders(X.n_rows, 1, 6)

        def fit():
            w0, w, V = np.zeros(C), np.zeros((C, d)), rng.normal(0, 0.01, (C, d, k))
            _rust.fm_fit_multiclass_csr(X.indptr, X.indices, X.data, d, y, sw, w0, w, V, "adam",
                                        1e-3, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, ro, 2048, 0.0,
                                        0.0, 1.0, use_cuda=True)
    fit()
    t = time.perf_counter()
    for _ in range(reps):
        fit()
    return {"rows": X.n_rows, "nnz": X.nnz, "s_per_rep": (time.perf_counter() - t) / reps}


def _eval_case(rows, dtype, reps, dev):
    import torch

    from . import workloads as WL
    from .evaluate import fm_eval_device

    X, y = WL.ctr_fm(rows, 2, labels=True)
    rng = np.random.default_rng(0)
    d, k = X.n_features, 16
    pdt = torch.float64 if dtype == "float64" else torch.float32
    vdt = torch.float32 if dtype == "float32" else torch.float64
    args = (_t(X.indptr, torch.int64, dev), _t(X.indices, torch.int32, dev),
            _t(X.data, vdt, dev), -0.5, _t(rng.normal(0, 0.1, d), pdt, dev),
            _t(rng.normal(0, 0.1, (d, k)), pdt, dev), _t(y, torch.float64, dev),
            _t(rng.uniform(0.5, 2.0, X.n_rows), torch.float64, dev))
    fm_eval_device(*args)
    t = time.perf_counter()
    for _ in range(reps):
        fm_eval_device(*args)
    return {"rows": X.n_rows, "s_per_rep": (time.perf_counter() - t) / reps}


def _prep_case(rows, dtype, reps, dev):
    import torch

    from . import workloads as WL
    from .prep import prep_csr_device

    X, _ = WL.ctr_fm(rows, 2)
    ip = _t(X.indptr, torch.int64, dev)
    ix = _t(X.indices, torch.int64, dev)
    dv = _t(X.data, torch.float64, dev)
    # every row reversed, its middle entry's column set to its first entry's
    lens = ip[1:] - ip[:-1]
    row = torch.repeat_interleave(torch.arange(X.n_rows, device=dev), lens)
    q = torch.arange(X.nnz, device=dev)
    rev = ip[row] + ip[row + 1] - 1 - q
    ixr, dvr = ix[rev].clone(), dv[rev].clone()
    mid = ip[:-1] + lens // 2
    has = lens > 2
    ixr[mid[has]] = ixr[ip[:-1][has]]
    out = dtype if dtype in ("float32", "float64") else "float64"
    for a, b in ((ix, dv), (ixr, dvr)):
        prep_csr_device(ip, a, b, X.n_features, dtype=out)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        for a, b in ((ix, dv), (ixr, dvr)):
            prep_csr_device(ip, a, b, X.n_features, dtype=out)
    torch.cuda.synchronize()
    return {"rows": X.n_rows, "s_per_rep": (time.perf_counter() - t) / reps}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["score-fm", "score-ffm", "score-fwfm", "score-softmax",
                                     "train-fm", "train-ffm", "train-fwfm", "train-softmax",
                                     "eval", "prep"])
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--dtype", default=None, choices=["float32-float64", "float64", "float32"])
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    kind = a.case.split("-", 1)[-1]
    if a.case.startswith("score"):
        rows = a.rows or 1_000_000
        r = _score_case(kind, rows, a.dtype or "float32-float64", a.reps, dev)
    elif a.case.startswith("train"):
        rows = a.rows or {"fm": 400_000, "ffm": 40_000, "fwfm": 200_000, "softmax": 100_000}[kind]
        r = _train_case(kind, rows, a.dtype or "float64", a.reps)
    elif a.case == "eval":
        r = _eval_case(a.rows or 1_000_000, a.dtype or "float32-float64", a.reps, dev)
    else:
        r = _prep_case(a.rows or 1_000_000, a.dtype or "float64", a.reps, dev)
    r["case"] = a.case
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
