"""Generate the golden fixtures in tests/golden/ from the reference's NumPy
ground truth (modern_fm v1.1.1, python/modern_fm/_reference.py and
_reference_train.py).

Run in a container where the reference source tree is present:

    python tests/golden/make_golden.py --reference /path/to/reference/python

The reference specifies these NumPy trainers as bit-for-bit with its Rust CPU
engine at n_jobs=1 (_reference_train.py:8-18), so the fixtures pin both the C
oracle and the CUDA path. Inputs are seeded and small; every case stores its
inputs, hyperparameters and the reference's outputs.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import scipy.sparse as sp

HERE = os.path.dirname(os.path.abspath(__file__))


def sparse_dense_X(rng, n, d, density):
    """Dense X with exact zeros (the reference's tests/conftest.py fixture shape)."""
    X = rng.normal(size=(n, d))
    X[rng.random(size=X.shape) > density] = 0.0
    return X


def csr_arrays(X):
    Xc = sp.csr_matrix(X)
    Xc.sum_duplicates()
    return (Xc.indptr.astype(np.int64), Xc.indices.astype(np.int64),
            Xc.data.astype(np.float64))


class Writer:
    def __init__(self):
        self.arrays = {}
        self.cases = []

    def add(self, name, meta, **arrays):
        self.cases.append(dict(name=name, **meta))
        for k, v in arrays.items():
            self.arrays[f"{name}/{k}"] = np.asarray(v)

    def save(self, fname):
        self.arrays["__cases__"] = np.frombuffer(json.dumps(self.cases).encode(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, fname), **self.arrays)
        print(f"wrote {fname}: {len(self.cases)} cases")


def make_predict(R):
    w = Writer()
    for seed in (0, 1, 2):
        rng = np.random.default_rng(seed)
        for k in (1, 4, 16, 64):
            X = sparse_dense_X(rng, 40, 30, 0.25)
            X[0] = 0.0  # empty row -> bias
            X[1] = 0.0
            X[1, 3] = -2.0  # single nonzero -> no pairwise term
            w0, wl, V = float(rng.normal()), rng.normal(size=30), rng.normal(size=(30, k))
            ip, ix, dv = csr_arrays(X)
            w.add(f"fm_s{seed}_k{k}", dict(model="fm", n_features=30, w0=w0),
                  indptr=ip, indices=ix, data=dv, w=wl, V=V,
                  out=R.fm_predict_fast(X, w0, wl, V),
                  out_naive=R.fm_predict_naive(X, w0, wl, V))
        for F in (1, 4, 8):
            for k in (1, 4):
                X = sparse_dense_X(rng, 30, 20, 0.3)
                X[0] = 0.0
                w0, wl = float(rng.normal()), rng.normal(size=20)
                V = rng.normal(size=(20, F, k))
                fid = rng.integers(0, F, size=20)
                ip, ix, dv = csr_arrays(X)
                w.add(f"ffm_s{seed}_F{F}_k{k}", dict(model="ffm", n_features=20, w0=w0),
                      indptr=ip, indices=ix, data=dv, w=wl, V=V, field_ids=fid,
                      out=R.ffm_predict(X, fid, w0, wl, V))
        for F in (1, 3, 5):
            k = 4
            X = sparse_dense_X(rng, 30, 20, 0.3)
            X[0] = 0.0
            w0, wl = float(rng.normal()), rng.normal(size=20)
            V = rng.normal(size=(20, k))
            r = rng.uniform(0.0, 2.0, size=(F, F))
            fid = rng.integers(0, F, size=20)
            ip, ix, dv = csr_arrays(X)
            w.add(f"fwfm_s{seed}_F{F}", dict(model="fwfm", n_features=20, w0=w0),
                  indptr=ip, indices=ix, data=dv, w=wl, V=V, r=r, field_ids=fid,
                  out=R.fwfm_predict(X, fid, w0, wl, V, r))
    w.save("predict.npz")


HP = dict(learning_rate=0.1, l2_linear=1e-4, l2_factors=1e-4)


def _hp(optimizer):
    hp = dict(HP)
    if optimizer == "ftrl":
        hp.update(l1_linear=0.01, l1_factors=0.001, learning_rate=0.5)
    return hp


def make_train_binary(T):
    w = Writer()
    # FM: every optimizer x loss x batch size (the reference's CUDA parity grid,
    # tests/test_cuda_parity.py:170-194, at a smaller size)
    rng = np.random.default_rng(10)
    n, d, k, E = 48, 16, 4, 2
    X = sparse_dense_X(rng, n, d, 0.3)
    margin = X @ rng.normal(size=d)
    params = (0.0, rng.normal(size=d) * 0.01, rng.normal(size=(d, k)) * 0.01)
    ro = np.vstack([rng.permutation(n) for _ in range(E)]).astype(np.int64)
    sw = rng.uniform(0.5, 2.0, size=n)
    ip, ix, dv = csr_arrays(X)
    for opt in ("sgd", "adagrad", "adam", "ftrl"):
        for loss in ("logistic", "squared"):
            y = (margin > 0).astype(np.float64) if loss == "logistic" else margin
            for bs in (1, 7, n):
                hp = _hp(opt)
                st = [0.0, np.zeros(d), np.zeros((d, k))]
                ad = T.new_adam_state(0.0, params[1], params[2]) if opt == "adam" else None
                ft = T.new_ftrl_state(0.0, params[1], params[2]) if opt == "ftrl" else None
                use_sw = bs == 7
                out = T.fm_fit_reference(X, y, params, loss=loss, optimizer=opt, row_orders=ro,
                                         batch_size=bs, sample_weight=sw if use_sw else None,
                                         state=st, adam_state=ad, ftrl_state=ft, **hp)
                extra = {}
                if ad is not None:
                    extra.update({f"adam_{i}": np.asarray(a, dtype=np.float64)
                                  for i, a in enumerate(ad)})
                if ft is not None:
                    extra.update({f"ftrl_{i}": np.asarray(a, dtype=np.float64)
                                  for i, a in enumerate(ft)})
                w.add(f"fm_{opt}_{loss}_b{bs}",
                      dict(model="fm", loss=loss, optimizer=opt, batch_size=bs, n_features=d,
                           use_sw=use_sw, hp=hp, w0_init=params[0]),
                      indptr=ip, indices=ix, data=dv, y=y, sw=sw if use_sw else np.ones(n),
                      w_init=params[1], V_init=params[2], row_orders=ro,
                      w0=np.float64(out[0]), w=out[1], V=out[2],
                      acc_w0=np.float64(st[0]), acc_w=st[1], acc_V=st[2], **extra)
    # FFM and FwFM: every optimizer, logistic, batch 1 and 5
    rng = np.random.default_rng(11)
    n, d, F, k, E = 30, 12, 3, 3, 2
    X = sparse_dense_X(rng, n, d, 0.35)
    y = (X @ rng.normal(size=d) > 0).astype(np.float64)
    fid = rng.integers(0, F, size=d)
    ffm_params = (0.0, rng.normal(size=d) * 0.01, rng.uniform(0.0, 0.3, size=(d, F, k)))
    fwfm_params = (0.0, rng.normal(size=d) * 0.01, rng.normal(size=(d, k)) * 0.1,
                   np.ones((F, F)))
    ro = np.vstack([rng.permutation(n) for _ in range(E)]).astype(np.int64)
    ip, ix, dv = csr_arrays(X)
    for opt in ("sgd", "adagrad", "adam", "ftrl"):
        for bs in (1, 5):
            hp = _hp(opt)
            st = [0.0, np.zeros(d), np.zeros((d, F, k))]
            out = T.ffm_fit_reference(X, y, fid, ffm_params, loss="logistic", optimizer=opt,
                                      row_orders=ro, batch_size=bs, state=st, **hp)
            w.add(f"ffm_{opt}_b{bs}",
                  dict(model="ffm", loss="logistic", optimizer=opt, batch_size=bs,
                       n_features=d, hp=hp, w0_init=0.0),
                  indptr=ip, indices=ix, data=dv, y=y, sw=np.ones(n), field_ids=fid,
                  w_init=ffm_params[1], V_init=ffm_params[2], row_orders=ro,
                  w0=np.float64(out[0]), w=out[1], V=out[2])
            out = T.fwfm_fit_reference(X, y, fid, fwfm_params, loss="logistic", optimizer=opt,
                                       row_orders=ro, batch_size=bs, **hp)
            w.add(f"fwfm_{opt}_b{bs}",
                  dict(model="fwfm", loss="logistic", optimizer=opt, batch_size=bs,
                       n_features=d, hp=hp, w0_init=0.0),
                  indptr=ip, indices=ix, data=dv, y=y, sw=np.ones(n), field_ids=fid,
                  w_init=fwfm_params[1], V_init=fwfm_params[2], r_init=fwfm_params[3],
                  row_orders=ro, w0=np.float64(out[0]), w=out[1], V=out[2], r=out[3])
    w.save("train_binary.npz")


def make_train_multiclass(T):
    w = Writer()
    rng = np.random.default_rng(12)
    n, d, F, k, C, E = 30, 12, 3, 3, 3, 2
    X = sparse_dense_X(rng, n, d, 0.35)
    margin = X @ rng.normal(size=d)
    y = np.digitize(margin, np.quantile(margin, [1 / 3, 2 / 3])).astype(np.int64)
    fid = rng.integers(0, F, size=d)
    sw = rng.uniform(0.5, 2.0, size=n)
    ro = np.vstack([rng.permutation(n) for _ in range(E)]).astype(np.int64)
    fm_p = (np.zeros(C), rng.normal(size=(C, d)) * 0.01, rng.normal(size=(C, d, k)) * 0.05)
    ffm_p = (np.zeros(C), rng.normal(size=(C, d)) * 0.01,
             rng.uniform(0.0, 0.3, size=(C, d, F, k)))
    fwfm_p = (np.zeros(C), rng.normal(size=(C, d)) * 0.01, rng.normal(size=(C, d, k)) * 0.1,
              np.ones((C, F, F)))
    ip, ix, dv = csr_arrays(X)
    for opt in ("sgd", "adagrad", "adam", "ftrl"):
        for bs in (1, 6):
            hp = _hp(opt)
            meta = dict(optimizer=opt, batch_size=bs, n_features=d, hp=hp, label_smoothing=0.1,
                        n_classes=C)
            common = dict(indptr=ip, indices=ix, data=dv, y=y, sw=sw, row_orders=ro)
            out = T.fm_fit_multiclass_reference(X, y, fm_p, optimizer=opt, row_orders=ro,
                                                batch_size=bs, label_smoothing=0.1,
                                                sample_weight=sw, **hp)
            w.add(f"fm_mc_{opt}_b{bs}", dict(model="fm", **meta), **common,
                  w0_init=fm_p[0], w_init=fm_p[1], V_init=fm_p[2],
                  w0=out[0], w=out[1], V=out[2])
            out = T.ffm_fit_multiclass_reference(X, y, fid, ffm_p, optimizer=opt, row_orders=ro,
                                                 batch_size=bs, label_smoothing=0.1,
                                                 sample_weight=sw, **hp)
            w.add(f"ffm_mc_{opt}_b{bs}", dict(model="ffm", **meta), **common, field_ids=fid,
                  w0_init=ffm_p[0], w_init=ffm_p[1], V_init=ffm_p[2],
                  w0=out[0], w=out[1], V=out[2])
            out = T.fwfm_fit_multiclass_reference(X, y, fid, fwfm_p, optimizer=opt,
                                                  row_orders=ro, batch_size=bs,
                                                  label_smoothing=0.1, sample_weight=sw, **hp)
            w.add(f"fwfm_mc_{opt}_b{bs}", dict(model="fwfm", **meta), **common, field_ids=fid,
                  w0_init=fwfm_p[0], w_init=fwfm_p[1], V_init=fwfm_p[2], r_init=fwfm_p[3],
                  w0=out[0], w=out[1], V=out[2], r=out[3])
    w.save("train_multiclass.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference/python",
                    help="path to the reference's python/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from modern_fm import _reference as R  # noqa: E402
    from modern_fm import _reference_train as T  # noqa: E402

    make_predict(R)
    make_train_binary(T)
    make_train_multiclass(T)


if __name__ == "__main__":
    main()
