"""Generate the golden fixtures in tests/golden/ from the reference's NumPy
ground truth (modern_fm v1.1.1, python/modern_fm/_reference.py and
_reference_train.py), its CSR preparation (_backend._prep_csr), its validation metrics
(losses.py) and its libffm reader (libffm.py).

Run in a container where the reference source tree is present:

    python tests/golden/make_golden.py --reference /path/to/reference/python [--only prep losses]

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


def _raw_csr(rng, n_rows, n_features, lens, dup_pool=None, sort_rows=False):
    """Rows of the given lengths; columns drawn with repeats from `dup_pool`
    columns per row (None: any column), in draw order unless sorted; values
    N(0, 1) with some explicit zeros and negative zeros."""
    ip, ix, dv = [0], [], []
    for r in range(n_rows):
        L = int(lens[r % len(lens)])
        if dup_pool is None:
            c = rng.integers(0, n_features, size=L)
        else:
            base = rng.choice(n_features, size=min(dup_pool, n_features), replace=False)
            c = base[rng.integers(0, len(base), size=L)]
        if sort_rows:
            c = np.sort(c, kind="stable")
        v = rng.normal(size=L)
        v[rng.random(L) < 0.05] = 0.0
        v[rng.random(L) < 0.02] = -0.0
        ix.extend(c.tolist())
        dv.extend(v.tolist())
        ip.append(len(ix))
    return (np.array(ip, dtype=np.int64), np.array(ix, dtype=np.int64),
            np.array(dv, dtype=np.float64))


def make_prep(B):
    """The reference's `_prep_csr` (python/modern_fm/_backend.py:44-52) on raw
    CSR inputs. `exact` marks cases where the duplicate-summation order is
    the original one (canonical input, rows already in order, at most two
    duplicates of a column), so the values are pinned bitwise."""
    w = Writer()
    rng = np.random.default_rng(7)
    cases = [
        ("canonical", dict(n_rows=200, n_features=300, lens=[0, 3, 12, 40]), True),
        ("sorted_dups", dict(n_rows=100, n_features=64, lens=[0, 1, 5, 39, 300], dup_pool=8,
                             sort_rows=True), True),
        ("unsorted_pairs", dict(n_rows=80, n_features=1 << 22, lens=[2, 17, 39, 400]), True),
        ("unsorted_short_many", dict(n_rows=400, n_features=40, lens=[0, 3, 9, 16], dup_pool=4),
         False),
        ("unsorted_long_many", dict(n_rows=16, n_features=5000,
                                    lens=[257, 3, 300, 0, 1000, 39, 4096, 4097], dup_pool=40),
         False),
    ]
    for name, kw, exact in cases:
        ip, ix, dv = _raw_csr(rng, **kw)
        if name == "canonical":  # strictly increasing rows, no duplicates
            X = sp.csr_matrix((dv, ix, ip), shape=(len(ip) - 1, kw["n_features"]))
            X.sum_duplicates()
            ip, ix, dv = X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data
        X = sp.csr_matrix((dv.copy(), ix.copy(), ip.copy()), shape=(len(ip) - 1, kw["n_features"]))
        oip, oix, odv, nf = B._prep_csr(X)
        w.add(name, dict(n_features=int(nf), exact=exact), indptr=ip, indices=ix, data=dv,
              out_indptr=oip, out_indices=oix, out_data=odv)
    w.save("prep.npz")


def make_losses(L):
    """The reference's validation metrics (python/modern_fm/losses.py:25-68)
    on seeded raw scores: logistic (with and without label smoothing and
    sample weights) and squared."""
    w = Writer()
    rng = np.random.default_rng(8)
    for i, (loss, eps, weighted) in enumerate([("logistic", 0.0, False), ("logistic", 0.1, True),
                                               ("logistic", 0.0, True), ("squared", 0.0, False),
                                               ("squared", 0.0, True)]):
        n = 1000
        raw = rng.normal(size=n) * 3.0
        raw[:5] = [0.0, 40.0, -40.0, 700.0, -700.0]  # the stable form's edge cases
        y = (rng.random(n) < 0.3).astype(np.float64) if loss == "logistic" else rng.normal(size=n)
        sw = rng.uniform(0.5, 2.0, size=n)
        if loss == "logistic":
            val = L.logistic_loss(y, raw, label_smoothing=eps, sample_weight=sw if weighted else None)
        else:
            val = L.squared_loss(y, raw, sample_weight=sw if weighted else None)
        w.add(f"{loss}_{i}", dict(loss=loss, label_smoothing=eps, weighted=weighted),
              raw=raw, y=y, sample_weight=sw, value=np.array([val]))
    w.save("losses.npz")


def make_libffm(LF):
    """The reference's load_libffm (python/modern_fm/libffm.py:31-83) on seeded
    libffm texts: its canonical X, y and field_ids, or the message of the
    ValueError it raises (the file path replaced by "{path}")."""
    import tempfile

    w = Writer()
    rng = np.random.default_rng(9)

    def random_text(n, m, nl, sep, dups):
        fields = rng.integers(0, 7, size=m)
        lines = []
        for _ in range(n):
            L = int(rng.integers(0, 12))
            toks = [repr(float(rng.integers(0, 2)))]
            js = rng.integers(0, m, size=L)
            if dups and L > 2:
                js[-1] = js[0]  # one duplicate: exact sums
            for j in js:
                v = rng.normal()
                sv = repr(float(v)) if rng.random() < 0.7 else "%.3e" % v
                toks.append(f"{fields[j]}:{j}:{sv}")
            lines.append(sep.join(toks))
        return nl.join(lines) + nl

    texts = {
        "known": "1 0:0:1 1:2:0.5\n0 0:1:1 1:2:2\n",  # tests/test_libffm.py:9-17
        "random_lf": random_text(400, 300, "\n", " ", False),
        "random_crlf_blank": "\r\n" + random_text(300, 200, "\r\n", "\t", False) + "\r\n",
        "random_cr": random_text(300, 200, "\r", "  ", False),
        "dups": random_text(300, 50, "\n", " ", True),
        "specials": "1 0:0:nan 1:1:-inf 2:2:1e400 3:3:.5 4:4:5. 5:1_0:2_5.0_1e-0_3\n0 6:6:+7\n",
        "err_token": "1 0:0:1 not_a_triple\n",  # tests/test_libffm.py:58-62
        "err_conflict": "1 0:0:1\n\n0 1:0:2\n",
        "err_negative": "1 0:-1:1\n",
        "err_label": "abc 0:0:1\n",
        "err_four_parts": "1 0:0:1:2\n",
        "err_int": "1 0:0:1 0:x:1\n",
        "err_underscores": "1 0:0:1__0\n",
        "err_hex": "1 0:0:0x10\n",
        "err_conflict_before_token": "1 0:0:1 1:0:1 bad\n",
    }
    d = tempfile.mkdtemp()
    for name, text in texts.items():
        path = os.path.join(d, name + ".ffm")
        with open(path, "w", newline="") as fh:
            fh.write(text)
        raw = np.frombuffer(text.encode(), dtype=np.uint8)
        try:
            X, y, f = LF.load_libffm(path)
        except ValueError as e:
            w.add(name, dict(error=str(e).replace(path, "{path}")), text=raw)
            continue
        w.add(name, dict(error=None, n_features=int(X.shape[1])), text=raw,
              indptr=X.indptr.astype(np.int64), indices=X.indices.astype(np.int64), data=X.data,
              y=y, field_ids=f)
    w.save("libffm.npz")


MAKERS = ("predict", "train_binary", "train_multiclass", "prep", "losses", "libffm")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MFM_REFERENCE_PYTHON"),
                    help="path to the reference's python/ directory (default: "
                         "$MFM_REFERENCE_PYTHON)")
    ap.add_argument("--only", nargs="*", choices=MAKERS, default=list(MAKERS),
                    help="fixture files to (re)generate")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MFM_REFERENCE_PYTHON")
    sys.path.insert(0, args.reference)
    from modern_fm import _backend as B  # noqa: E402
    from modern_fm import _reference as R  # noqa: E402
    from modern_fm import _reference_train as T  # noqa: E402
    from modern_fm import libffm as LF  # noqa: E402
    from modern_fm import losses as L  # noqa: E402

    if "predict" in args.only:
        make_predict(R)
    if "train_binary" in args.only:
        make_train_binary(T)
    if "train_multiclass" in args.only:
        make_train_multiclass(T)
    if "prep" in args.only:
        make_prep(B)
    if "losses" in args.only:
        make_losses(L)
    if "libffm" in args.only:
        make_libffm(LF)


if __name__ == "__main__":
    main()
