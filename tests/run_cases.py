"""Drive golden cases through any module with the reference's `_rust`
signatures (rust/src/lib.rs): the C oracle (oracle/oracle.py, use_cuda=False)
or the product mirror (modern_fm_b200._rust, use_cuda=True)."""

import numpy as np


def predict_case(mod, case, cuda):
    a = case.a
    n = case["n_features"]
    m = case["model"]
    if m == "fm":
        fn = mod.fm_predict_cuda_csr if cuda else mod.fm_predict_fast_csr
        return fn(a["indptr"], a["indices"], a["data"], n, case["w0"], a["w"], a["V"])
    if m == "ffm":
        fn = mod.ffm_predict_cuda_csr if cuda else mod.ffm_predict_csr
        return fn(a["indptr"], a["indices"], a["data"], n, a["field_ids"], case["w0"], a["w"],
                  a["V"])
    fn = mod.fwfm_predict_cuda_csr if cuda else mod.fwfm_predict_csr
    return fn(a["indptr"], a["indices"], a["data"], n, a["field_ids"], case["w0"], a["w"],
              a["V"], a["r"])


def _hp(case):
    hp = dict(l1_linear=0.0, l1_factors=0.0)
    hp.update(case["hp"])
    return hp


def train_binary_case(mod, case, use_cuda, n_jobs=1):
    """Returns dict(w0, w, V[, r], acc_w0, acc_w, acc_V[, adam..., ftrl...])."""
    a = case.a
    hp = _hp(case)
    m = case["model"]
    w = np.array(a["w_init"], dtype=np.float64)
    V = np.array(a["V_init"], dtype=np.float64)
    acc_w, acc_V = np.zeros_like(w), np.zeros_like(V)
    opt = case["optimizer"]
    common = dict(loss=case["loss"], optimizer=opt, learning_rate=hp["learning_rate"],
                  l2_linear=hp["l2_linear"], l2_factors=hp["l2_factors"], beta_1=0.9,
                  beta_2=0.999, epsilon=1e-8, row_orders=a["row_orders"],
                  batch_size=case["batch_size"], l1_linear=hp["l1_linear"],
                  l1_factors=hp["l1_factors"], ftrl_beta=1.0)
    out = dict(w=w, V=V, acc_w=acc_w, acc_V=acc_V)
    if m == "fwfm":
        r = np.array(a["r_init"], dtype=np.float64)
        acc_r = np.zeros_like(r)
        out.update(r=r, acc_r=acc_r)
        ad = ((0.0, 0.0, 0.0) + tuple(np.zeros_like(x) for x in (w, w, w, V, V, V, r, r, r))
              if opt == "adam" else None)
        ft = ((0.0, 0.0) + tuple(np.zeros_like(x) for x in (w, w, V, V, r, r))
              if opt == "ftrl" else None)
        res = mod.fwfm_fit_csr(a["indptr"], a["indices"], a["data"], case["n_features"], a["y"],
                               a["sw"], a["field_ids"], case["w0_init"], 0.0, w, V, r, acc_w,
                               acc_V, acc_r, adam_state=ad, ftrl_state=ft, use_cuda=use_cuda,
                               **common)
    else:
        ad = ((0.0, 0.0, 0.0) + tuple(np.zeros_like(x) for x in (w, w, w, V, V, V))
              if opt == "adam" else None)
        ft = ((0.0, 0.0) + tuple(np.zeros_like(x) for x in (w, w, V, V))
              if opt == "ftrl" else None)
        if m == "fm":
            res = mod.fm_fit_csr(a["indptr"], a["indices"], a["data"], case["n_features"],
                                 a["y"], a["sw"], case["w0_init"], 0.0, w, V, acc_w, acc_V,
                                 n_jobs=n_jobs, adam_state=ad, ftrl_state=ft,
                                 use_cuda=use_cuda, **common)
        else:
            res = mod.ffm_fit_csr(a["indptr"], a["indices"], a["data"], case["n_features"],
                                  a["y"], a["sw"], a["field_ids"], case["w0_init"], 0.0, w, V,
                                  acc_w, acc_V, n_jobs=n_jobs, adam_state=ad, ftrl_state=ft,
                                  use_cuda=use_cuda, **common)
    out["w0"], out["acc_w0"] = res[0], res[1]
    if ad is not None:
        out["adam"] = tuple(res[2]) + tuple(ad[3:])
    if ft is not None:
        out["ftrl"] = tuple(res[3]) + tuple(ft[2:])
    return out


def train_multiclass_case(mod, case, use_cuda):
    a = case.a
    hp = _hp(case)
    m = case["model"]
    opt = case["optimizer"]
    w0 = np.array(a["w0_init"], dtype=np.float64)
    w = np.array(a["w_init"], dtype=np.float64)
    V = np.array(a["V_init"], dtype=np.float64)
    common = dict(optimizer=opt, learning_rate=hp["learning_rate"], l2_linear=hp["l2_linear"],
                  l2_factors=hp["l2_factors"], label_smoothing=case["label_smoothing"],
                  beta_1=0.9, beta_2=0.999, epsilon=1e-8, row_orders=a["row_orders"],
                  batch_size=case["batch_size"], l1_linear=hp["l1_linear"],
                  l1_factors=hp["l1_factors"], ftrl_beta=1.0, use_cuda=use_cuda)
    out = dict(w0=w0, w=w, V=V)
    if m == "fm":
        mod.fm_fit_multiclass_csr(a["indptr"], a["indices"], a["data"], case["n_features"],
                                  a["y"], a["sw"], w0, w, V, **common)
    elif m == "ffm":
        mod.ffm_fit_multiclass_csr(a["indptr"], a["indices"], a["data"], case["n_features"],
                                   a["y"], a["sw"], a["field_ids"], w0, w, V, **common)
    else:
        r = np.array(a["r_init"], dtype=np.float64)
        out["r"] = r
        mod.fwfm_fit_multiclass_csr(a["indptr"], a["indices"], a["data"], case["n_features"],
                                    a["y"], a["sw"], a["field_ids"], w0, w, V, r, **common)
    return out
