"""Host-side mirror of the reference's `modern_fm._rust` module for the CUDA path.

The reference's PyO3 module (modern_fm v1.1.1, rust/src/lib.rs:1592-1614) is
the Python->native boundary that `python/modern_fm/_backend.py` calls. This
module re-implements, with the same names, argument order, in-place mutation,
return tuples and exception types, every entry point that reaches CUDA:

    has_cuda, fm_predict_cuda_csr, ffm_predict_cuda_csr, fwfm_predict_cuda_csr,
    fm_fit_csr / fm_fit_multiclass_csr / ffm_fit_csr / ffm_fit_multiclass_csr /
    fwfm_fit_csr / fwfm_fit_multiclass_csr with use_cuda=True

over the C ABI of libmfm_b200.so (include/mfm_b200.h). Shape checks mirror
lib.rs; CSR/field-id/row-order validation runs inside the library. The
CPU-engine entry points of the reference (use_cuda=False and the
*_predict_fast_* / *_predict_{csr,dense} functions) are not part of this
engine: `modern_fm_b200.dropin` composes this module with a CPU backend.

Compute dtype / devices come from MFM_B200_DTYPE (default float32-float64: the
reference's own arithmetic), MFM_B200_DEVICE and MFM_B200_NUM_GPUS.
"""

from __future__ import annotations

import numpy as np

from . import _lib as L

_CPU_MSG = ("modern_fm_b200 is the CUDA engine: use_cuda=False calls belong to the "
            "reference's CPU engine (see modern_fm_b200.dropin)")


def has_cuda() -> bool:
    """rust/src/lib.rs:1471-1482: True when a CUDA device is usable."""
    try:
        return bool(L.lib().mfm_has_cuda())
    except OSError:
        return False


def _raise(rc, fit):
    """Error types of the reference boundary: every error raised inside a CUDA
    predict call (CSR structure, k range, device) is a RuntimeError
    (rust/src/lib.rs:1506-1512); every fit error is a ValueError (lib.rs:437).
    Shape and field-id checks run before the call and raise ValueError."""
    msg = L.last_error()
    if fit:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _check_field_ids(field_ids, n_features, n_fields):
    # check_field_ids, rust/src/data.rs:71-83 (ValueError, before the device call)
    if field_ids.size != n_features:
        raise ValueError(
            f"field_ids length {field_ids.size} does not match n_features {n_features}")
    if field_ids.size and (field_ids.min() < 0 or field_ids.max() >= n_fields):
        raise ValueError(f"field id out of range [0, {n_fields})")


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _rw(a, name):
    """A PyReadwriteArray<f64>: must be a C-contiguous float64 ndarray."""
    if not isinstance(a, np.ndarray) or a.dtype != np.float64 or not a.flags.c_contiguous \
            or not a.flags.writeable:
        raise TypeError(f"{name} must be a writeable C-contiguous float64 ndarray")
    return a


def _check_w_v(n_features, w, v_rows):
    # check_w_v_fm, rust/src/lib.rs:174-183
    if w.size != n_features or v_rows != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, V rows={v_rows}")


# ------------------------------------------------------------------ predict


def fm_predict_cuda_csr(indptr, indices, data, n_features, w0, w, v):
    """rust/src/lib.rs:1488-1513."""
    w, v = _f64(w), _f64(v)
    if v.ndim != 2:
        raise ValueError(f"V must be 2-D (n_features, k), got shape {v.shape}")
    _check_w_v(n_features, w, v.shape[0])
    csr, keep = L.make_csr(indptr, indices, data, n_features, exc=RuntimeError)
    out = np.empty(csr.n_rows, dtype=np.float64)
    ex = L.exec_options()
    rc = L.lib().mfm_fm_predict_csr(csr, float(w0), L.ptr(w), L.ptr(v), v.shape[1], L.ptr(out),
                                    ex)
    if rc:
        _raise(rc, fit=False)
    return out


def ffm_predict_cuda_csr(indptr, indices, data, n_features, field_ids, w0, w, v):
    """rust/src/lib.rs:1519-1548."""
    w, v, field_ids = _f64(w), _f64(v), _i64(field_ids)
    if v.ndim != 3:
        raise ValueError(f"V must be 3-D (n_features, n_fields, k), got shape {v.shape}")
    _check_w_v(n_features, w, v.shape[0])
    _check_field_ids(field_ids, n_features, v.shape[1])
    csr, keep = L.make_csr(indptr, indices, data, n_features, exc=RuntimeError)
    out = np.empty(csr.n_rows, dtype=np.float64)
    rc = L.lib().mfm_ffm_predict_csr(csr, L.ptr(field_ids, L.i64p), v.shape[1], float(w0),
                                     L.ptr(w), L.ptr(v), v.shape[2], L.ptr(out),
                                     L.exec_options())
    if rc:
        _raise(rc, fit=False)
    return out


def fwfm_predict_cuda_csr(indptr, indices, data, n_features, field_ids, w0, w, v, r):
    """rust/src/lib.rs:1554-1590."""
    w, v, r, field_ids = _f64(w), _f64(v), _f64(r), _i64(field_ids)
    if r.ndim != 2 or r.shape[0] != r.shape[1]:
        raise ValueError(f"R must be square, got {list(r.shape)}")
    if v.ndim != 2:
        raise ValueError(f"V must be 2-D (n_features, k), got shape {v.shape}")
    _check_w_v(n_features, w, v.shape[0])
    _check_field_ids(field_ids, n_features, r.shape[0])
    csr, keep = L.make_csr(indptr, indices, data, n_features, exc=RuntimeError)
    out = np.empty(csr.n_rows, dtype=np.float64)
    rc = L.lib().mfm_fwfm_predict_csr(csr, L.ptr(field_ids, L.i64p), r.shape[0], float(w0),
                                      L.ptr(w), L.ptr(v), L.ptr(r), v.shape[1], L.ptr(out),
                                      L.exec_options())
    if rc:
        _raise(rc, fit=False)
    return out


# --------------------------------------------------------------------- fit


def _parse(loss, optimizer):
    # parse_loss / parse_optimizer, rust/src/lib.rs:89-115
    if loss is not None and loss not in L.LOSSES:
        raise ValueError(f"unknown loss {loss!r}")
    if optimizer not in L.OPTIMIZERS:
        raise ValueError(f"unknown optimizer {optimizer!r}")


def _train(loss, optimizer, lr, l1l, l2l, l1f, l2f, b1, b2, eps, fb, ls, row_orders, bs):
    if bs == 0:
        raise ValueError("batch_size must be >= 1")
    ro = _i64(row_orders)
    if ro.ndim != 2:
        raise ValueError("row_orders must be 2-D (n_epochs, n_rows)")
    t = L.Train(L.LOSSES.get(loss, 0), L.OPTIMIZERS[optimizer], lr, l1l, l2l, l1f, l2f, b1, b2,
                eps, fb, ls, L.ptr(ro, L.i64p), ro.shape[0], int(bs))
    return t, ro


def _check_sw_ro(n_rows, y, sw, ro):
    # check_fit_args / check_sw_ro, rust/src/lib.rs:117-160
    if y.size != n_rows:
        raise ValueError(f"y length {y.size} != n_rows {n_rows}")
    if sw.size != n_rows:
        raise ValueError(f"sample_weight length {sw.size} != n_rows {n_rows}")
    if ro.shape[1] != n_rows:
        raise ValueError(f"row_orders second dimension {ro.shape[1]} != n_rows {n_rows}")


def _group(param, acc=None, **state):
    g = L.Group(L.ptr(param), L.ptr(acc), None, None, None, None, None)
    for k, a in state.items():
        setattr(g, k, L.ptr(a))
    return g


def _binary_state(optimizer, adam_state, ftrl_state, shapes, names):
    """Binary state tuples (rust/src/lib.rs:39-72): the scalar w0 moments ride
    by value (returned), the arrays are mutated in place. Returns
    (w0-state dict of 1-element arrays, per-group state dicts)."""
    if adam_state is not None and optimizer != "adam":
        raise ValueError("adam_state is only valid for optimizer='adam'")
    if ftrl_state is not None and optimizer != "ftrl":
        raise ValueError("ftrl_state is only valid for optimizer='ftrl'")
    s0, groups = {}, [dict() for _ in shapes]
    # the w0-level scalars are always live for the active optimizer and are
    # returned even when no state tuple was passed (lib.rs:337-340, 438)
    if optimizer == "adam":
        s0 = dict(m=np.zeros(1), s=np.zeros(1), t=np.zeros(1))
    elif optimizer == "ftrl":
        s0 = dict(z=np.zeros(1), n=np.zeros(1))
    what = " and ".join([", ".join(names[:-1]), names[-1]]) if len(names) > 2 else \
        " and ".join(names)
    if adam_state is not None:
        s0 = dict(m=np.array([float(adam_state[0])]), s=np.array([float(adam_state[1])]),
                  t=np.array([float(adam_state[2])]))
        arrs = list(adam_state[3:])
        if len(arrs) != 3 * len(shapes):
            raise ValueError(f"adam_state shapes must match {what}")
        for i, sz in enumerate(shapes):
            for j, key in enumerate(("m", "s", "t")):
                a = _rw(arrs[3 * i + j], "adam_state")
                if a.size != sz:
                    raise ValueError(f"adam_state shapes must match {what}")
                groups[i][key] = a
    if ftrl_state is not None:
        s0 = dict(z=np.array([float(ftrl_state[0])]), n=np.array([float(ftrl_state[1])]))
        arrs = list(ftrl_state[2:])
        if len(arrs) != 2 * len(shapes):
            raise ValueError(f"ftrl_state shapes must match {what}")
        for i, sz in enumerate(shapes):
            for j, key in enumerate(("z", "n")):
                a = _rw(arrs[2 * i + j], "ftrl_state")
                if a.size != sz:
                    raise ValueError(f"ftrl_state shapes must match {what}")
                groups[i][key] = a
    return s0, groups


def _scalars(w0a, acc0, s0):
    # FitScalars, rust/src/lib.rs:74-77
    adam = (float(s0["m"][0]), float(s0["s"][0]), float(s0["t"][0])) if "m" in s0 else \
        (0.0, 0.0, 0.0)
    ftrl = (float(s0["z"][0]), float(s0["n"][0])) if "z" in s0 else (0.0, 0.0)
    return float(w0a[0]), float(acc0[0]), adam, ftrl


def fm_fit_csr(indptr, indices, data, n_features, y, sample_weight, w0, acc_w0, w, v, acc_w,
               acc_v, loss, optimizer, learning_rate, l2_linear, l2_factors, beta_1, beta_2,
               epsilon, row_orders, batch_size, n_jobs, l1_linear, l1_factors, ftrl_beta,
               adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:283-439 with use_cuda=True (n_jobs is ignored on the GPU,
    as in the reference's CUDA path)."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(loss, optimizer)
    tr, ro = _train(loss, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, 0.0, row_orders, batch_size)
    w, v = _rw(w, "w"), _rw(v, "v")
    acc_w, acc_v = _rw(acc_w, "acc_w"), _rw(acc_v, "acc_v")
    if v.ndim != 2:
        raise ValueError(f"V must be 2-D (n_features, k), got shape {v.shape}")
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, "
                         f"V rows={v.shape[0]}")
    if acc_w.size != w.size or acc_v.size != v.size:
        raise ValueError("accumulator shapes must match w and V")
    s0, (gw, gv) = _binary_state(optimizer, adam_state, ftrl_state, [w.size, v.size],
                                 ["w", "V"])
    y, sw = _f64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    w0a, acc0 = np.array([float(w0)]), np.array([float(acc_w0)])
    g0 = _group(w0a, acc0, **s0)
    g1, g2 = _group(w, acc_w, **gw), _group(v, acc_v, **gv)
    rc = L.lib().mfm_fm_fit_csr(csr, L.ptr(y), L.ptr(sw), tr, v.shape[1], g0, g1, g2,
                                L.exec_options())
    if rc:
        _raise(rc, fit=True)
    return _scalars(w0a, acc0, s0)


def ffm_fit_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0, acc_w0, w,
                v, acc_w, acc_v, loss, optimizer, learning_rate, l2_linear, l2_factors, beta_1,
                beta_2, epsilon, row_orders, batch_size, n_jobs, l1_linear, l1_factors,
                ftrl_beta, adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:635-793 with use_cuda=True."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(loss, optimizer)
    tr, ro = _train(loss, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, 0.0, row_orders, batch_size)
    w, v = _rw(w, "w"), _rw(v, "v")
    acc_w, acc_v = _rw(acc_w, "acc_w"), _rw(acc_v, "acc_v")
    if v.ndim != 3:
        raise ValueError(f"V must be 3-D (n_features, n_fields, k), got shape {v.shape}")
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, "
                         f"V rows={v.shape[0]}")
    field_ids = _i64(field_ids)
    if field_ids.size != n_features:
        raise ValueError(
            f"field_ids length {field_ids.size} does not match n_features {n_features}")
    if acc_w.size != w.size or acc_v.size != v.size:
        raise ValueError("accumulator shapes must match w and V")
    s0, (gw, gv) = _binary_state(optimizer, adam_state, ftrl_state, [w.size, v.size],
                                 ["w", "V"])
    y, sw = _f64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    w0a, acc0 = np.array([float(w0)]), np.array([float(acc_w0)])
    g0 = _group(w0a, acc0, **s0)
    g1, g2 = _group(w, acc_w, **gw), _group(v, acc_v, **gv)
    rc = L.lib().mfm_ffm_fit_csr(csr, L.ptr(y), L.ptr(sw), L.ptr(field_ids, L.i64p), v.shape[1],
                                 tr, v.shape[2], g0, g1, g2, L.exec_options())
    if rc:
        _raise(rc, fit=True)
    return _scalars(w0a, acc0, s0)


def fwfm_fit_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0, acc_w0, w,
                 v, r, acc_w, acc_v, acc_r, loss, optimizer, learning_rate, l2_linear,
                 l2_factors, beta_1, beta_2, epsilon, row_orders, batch_size, l1_linear,
                 l1_factors, ftrl_beta, adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:1049-1242 with use_cuda=True."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(loss, optimizer)
    tr, ro = _train(loss, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, 0.0, row_orders, batch_size)
    w, v, r = _rw(w, "w"), _rw(v, "v"), _rw(r, "r")
    acc_w, acc_v, acc_r = _rw(acc_w, "acc_w"), _rw(acc_v, "acc_v"), _rw(acc_r, "acc_r")
    if r.ndim != 2 or r.shape[0] != r.shape[1]:
        raise ValueError(f"R must be square, got {list(r.shape)}")
    if v.ndim != 2:
        raise ValueError(f"V must be 2-D (n_features, k), got shape {v.shape}")
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, "
                         f"V rows={v.shape[0]}")
    field_ids = _i64(field_ids)
    if field_ids.size != n_features:
        raise ValueError(
            f"field_ids length {field_ids.size} does not match n_features {n_features}")
    if acc_w.size != w.size or acc_v.size != v.size or acc_r.size != r.size:
        raise ValueError("accumulator shapes must match w, V and R")
    s0, (gw, gv, gr) = _binary_state(optimizer, adam_state, ftrl_state,
                                     [w.size, v.size, r.size], ["w", "V", "R"])
    y, sw = _f64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    w0a, acc0 = np.array([float(w0)]), np.array([float(acc_w0)])
    g0 = _group(w0a, acc0, **s0)
    g1, g2, g3 = _group(w, acc_w, **gw), _group(v, acc_v, **gv), _group(r, acc_r, **gr)
    rc = L.lib().mfm_fwfm_fit_csr(csr, L.ptr(y), L.ptr(sw), L.ptr(field_ids, L.i64p),
                                  r.shape[0], tr, v.shape[1], g0, g1, g2, g3, L.exec_options())
    if rc:
        _raise(rc, fit=True)
    return _scalars(w0a, acc0, s0)


def _mc_state(optimizer, state, adam_state, ftrl_state, params, names):
    """Multiclass state (rust/src/lib.rs:45-72): all (C, ...) arrays, in place."""
    if adam_state is not None and optimizer != "adam":
        raise ValueError("adam_state is only valid for optimizer='adam'")
    if ftrl_state is not None and optimizer != "ftrl":
        raise ValueError("ftrl_state is only valid for optimizer='ftrl'")
    what = "(" + ", ".join(names) + ")"
    groups = [dict() for _ in params]
    if state is not None:
        if len(state) != len(params):
            raise ValueError(f"state shapes must match {what}")
        for g, a, p in zip(groups, state, params):
            a = _rw(a, "state")
            if a.size != p.size:
                raise ValueError(f"state shapes must match {what}")
            g["acc"] = a
    for tup, keys, label in ((adam_state, ("m", "s", "t"), "adam_state"),
                             (ftrl_state, ("z", "n"), "ftrl_state")):
        if tup is None:
            continue
        if len(tup) != len(keys) * len(params):
            raise ValueError(f"{label} shapes must match {what}")
        for i, p in enumerate(params):
            for j, key in enumerate(keys):
                a = _rw(tup[len(keys) * i + j], label)
                if a.size != p.size:
                    raise ValueError(f"{label} shapes must match {what}")
                groups[i][key] = a
    return groups


def _check_y_mc(y, n_classes):
    if y.size and (y.min() < 0 or y.max() >= n_classes):
        raise ValueError(f"class index out of range [0, {n_classes})")


def fm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, w0, w, v,
                          optimizer, learning_rate, l2_linear, l2_factors, label_smoothing,
                          beta_1, beta_2, epsilon, row_orders, batch_size, l1_linear,
                          l1_factors, ftrl_beta, state=None, adam_state=None, ftrl_state=None,
                          use_cuda=False):
    """rust/src/lib.rs:449-630 with use_cuda=True."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(None, optimizer)
    tr, ro = _train(None, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, label_smoothing, row_orders,
                    batch_size)
    w0, w, v = _rw(w0, "w0"), _rw(w, "w"), _rw(v, "v")
    if v.ndim != 3 or w.ndim != 2:
        raise ValueError("w must be (C, n_features) and V (C, n_features, k)")
    C, k = v.shape[0], v.shape[2]
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}, "
                         f"w0={w0.size}, w={list(w.shape)}, V dims={list(v.shape)}")
    gs = _mc_state(optimizer, state, adam_state, ftrl_state, [w0, w, v], ["w0", "w", "V"])
    y, sw = _i64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    _check_y_mc(y, C)
    g0, g1, g2 = (_group(p, **g) for p, g in zip((w0, w, v), gs))
    rc = L.lib().mfm_fm_fit_multiclass_csr(csr, L.ptr(y, L.i64p), L.ptr(sw), C, tr, k, g0, g1,
                                           g2, L.exec_options())
    if rc:
        _raise(rc, fit=True)


def ffm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0,
                           w, v, optimizer, learning_rate, l2_linear, l2_factors,
                           label_smoothing, beta_1, beta_2, epsilon, row_orders, batch_size,
                           l1_linear, l1_factors, ftrl_beta, state=None, adam_state=None,
                           ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:800-978 with use_cuda=True."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(None, optimizer)
    tr, ro = _train(None, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, label_smoothing, row_orders,
                    batch_size)
    w0, w, v = _rw(w0, "w0"), _rw(w, "w"), _rw(v, "v")
    if v.ndim != 4 or w.ndim != 2:
        raise ValueError("w must be (C, n_features) and V (C, n_features, n_fields, k)")
    C, F, k = v.shape[0], v.shape[2], v.shape[3]
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}, "
                         f"w0={w0.size}, w={list(w.shape)}, V dims={list(v.shape)}")
    field_ids = _i64(field_ids)
    if field_ids.size != n_features:
        raise ValueError(
            f"field_ids length {field_ids.size} does not match n_features {n_features}")
    gs = _mc_state(optimizer, state, adam_state, ftrl_state, [w0, w, v], ["w0", "w", "V"])
    y, sw = _i64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    _check_y_mc(y, C)
    g0, g1, g2 = (_group(p, **g) for p, g in zip((w0, w, v), gs))
    rc = L.lib().mfm_ffm_fit_multiclass_csr(csr, L.ptr(y, L.i64p), L.ptr(sw), C,
                                            L.ptr(field_ids, L.i64p), F, tr, k, g0, g1, g2,
                                            L.exec_options())
    if rc:
        _raise(rc, fit=True)


def fwfm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0,
                            w, v, r, optimizer, learning_rate, l2_linear, l2_factors,
                            label_smoothing, beta_1, beta_2, epsilon, row_orders, batch_size,
                            l1_linear, l1_factors, ftrl_beta, state=None, adam_state=None,
                            ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:1249-1466 with use_cuda=True."""
    if not use_cuda:
        raise ValueError(_CPU_MSG)
    _parse(None, optimizer)
    tr, ro = _train(None, optimizer, learning_rate, l1_linear, l2_linear, l1_factors,
                    l2_factors, beta_1, beta_2, epsilon, ftrl_beta, label_smoothing, row_orders,
                    batch_size)
    w0, w, v, r = _rw(w0, "w0"), _rw(w, "w"), _rw(v, "v"), _rw(r, "r")
    if v.ndim != 3 or w.ndim != 2 or r.ndim != 3:
        raise ValueError("w must be (C, n), V (C, n, k) and R (C, F, F)")
    C, k, F = v.shape[0], v.shape[2], r.shape[1]
    if r.shape[0] != C or r.shape[2] != F:
        raise ValueError(f"R must be (n_classes, n_fields, n_fields), got {list(r.shape)}")
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}, "
                         f"w0={w0.size}, w={list(w.shape)}, V dims={list(v.shape)}")
    field_ids = _i64(field_ids)
    if field_ids.size != n_features:
        raise ValueError(
            f"field_ids length {field_ids.size} does not match n_features {n_features}")
    gs = _mc_state(optimizer, state, adam_state, ftrl_state, [w0, w, v, r],
                   ["w0", "w", "V", "R"])
    y, sw = _i64(y), _f64(sample_weight)
    csr, keep = L.make_csr(indptr, indices, data, n_features)
    _check_sw_ro(csr.n_rows, y, sw, ro)
    _check_y_mc(y, C)
    g0, g1, g2, g3 = (_group(p, **g) for p, g in zip((w0, w, v, r), gs))
    rc = L.lib().mfm_fwfm_fit_multiclass_csr(csr, L.ptr(y, L.i64p), L.ptr(sw), C,
                                             L.ptr(field_ids, L.i64p), F, tr, k, g0, g1, g2,
                                             g3, L.exec_options())
    if rc:
        _raise(rc, fit=True)


CUDA_FUNCTIONS = (
    "has_cuda", "fm_predict_cuda_csr", "ffm_predict_cuda_csr", "fwfm_predict_cuda_csr",
    "fm_fit_csr", "fm_fit_multiclass_csr", "ffm_fit_csr", "ffm_fit_multiclass_csr",
    "fwfm_fit_csr", "fwfm_fit_multiclass_csr",
)
