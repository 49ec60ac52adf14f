"""CPU oracle bindings (TEST INFRASTRUCTURE ONLY).

Python face of ``oracle/mfm_oracle.c``, the C restatement of modern_fm's Rust
CPU engine. It exposes the CPU half of the reference's ``modern_fm._rust``
PyO3 module (rust/src/lib.rs:185-275, 283-1242: ``fm_predict_fast_*``,
``ffm_predict_*``, ``fwfm_predict_*`` and the ``*_fit_*csr`` functions with
``use_cuda=False``), with the same argument order, in-place mutation and
return tuples. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg import this module; the product package never does.
"""

from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libmfm_oracle.so")

LOSSES = {"logistic": 0, "squared": 1}
OPTIMIZERS = {"sgd": 0, "adagrad": 1, "adam": 2, "ftrl": 3}

_i64p = ct.POINTER(ct.c_int64)
_f64p = ct.POINTER(ct.c_double)


class _Opt(ct.Structure):
    _fields_ = [
        ("kind", ct.c_int),
        ("lr", ct.c_double),
        ("beta1", ct.c_double),
        ("beta2", ct.c_double),
        ("eps", ct.c_double),
        ("ftrl_beta", ct.c_double),
        ("l1_linear", ct.c_double),
        ("l2_linear", ct.c_double),
        ("l1_factors", ct.c_double),
        ("l2_factors", ct.c_double),
    ]


class _State(ct.Structure):
    _fields_ = [(n, _f64p) for n in ("acc", "m", "s", "t", "z", "n")]


def build() -> str:
    """Compile the oracle (make -C oracle) if the shared object is missing."""
    if not os.path.exists(_SO):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ct.CDLL(build())
        L.orc_check_csr.restype = ct.c_int
        L.orc_check_csr.argtypes = [_i64p, ct.c_int64, _i64p, ct.c_int64, ct.c_int64,
                                    ct.c_int64, ct.c_char_p, ct.c_int]
        L.orc_check_field_ids.restype = ct.c_int
        L.orc_check_field_ids.argtypes = [_i64p, ct.c_int64, ct.c_int64, ct.c_int64,
                                          ct.c_char_p, ct.c_int]
        L.orc_prep_csr.restype = ct.c_int64
        L.orc_prep_csr.argtypes = [ct.c_int64, _i64p, _i64p, _f64p, _i64p, _i64p, _f64p]
        L.orc_sigmoid.restype = ct.c_double
        L.orc_sigmoid.argtypes = [ct.c_double]
        for name in ("orc_fm_fit_csr", "orc_ffm_fit_csr", "orc_fwfm_fit_csr",
                     "orc_fm_fit_multiclass_csr", "orc_ffm_fit_multiclass_csr",
                     "orc_fwfm_fit_multiclass_csr"):
            getattr(L, name).restype = ct.c_int
        _lib = L
    return _lib


def _p(a, kind=_f64p):
    return None if a is None else a.ctypes.data_as(kind)


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _check_csr(indptr, indices, data, n_cols):
    err = ct.create_string_buffer(256)
    rc = lib().orc_check_csr(_p(indptr, _i64p), len(indptr), _p(indices, _i64p), len(indices),
                             len(data), n_cols, err, 256)
    if rc:
        raise ValueError(err.value.decode())


def _check_field_ids(field_ids, n_features, n_fields):
    err = ct.create_string_buffer(256)
    rc = lib().orc_check_field_ids(_p(field_ids, _i64p), len(field_ids), n_features, n_fields,
                                   err, 256)
    if rc:
        raise ValueError(err.value.decode())


def _nthreads(n_threads):
    return max(1, int(n_threads))


# --------------------------------------------------------------------------
# CSR canonicalisation (python/modern_fm/_backend.py:44-52)
# --------------------------------------------------------------------------

def prep_csr(indptr, indices, data, n_features):
    """`_prep_csr` restated: validate, sort each row by column and sum
    duplicate columns in float64 in their original order. Returns
    (indptr, indices, data) as int64 / int64 / float64 arrays."""
    indptr, indices, data = _i64(indptr), _i64(indices), _f64(data)
    _check_csr(indptr, indices, data, n_features)
    n_rows = len(indptr) - 1
    ip = np.empty(n_rows + 1, dtype=np.int64)
    ix = np.empty(max(len(indices), 1), dtype=np.int64)
    dv = np.empty(max(len(indices), 1))
    m = lib().orc_prep_csr(n_rows, _p(indptr, _i64p), _p(indices, _i64p), _p(data),
                           _p(ip, _i64p), _p(ix, _i64p), _p(dv))
    return ip, ix[:m].copy(), dv[:m].copy()


# --------------------------------------------------------------------------
# validation metrics (python/modern_fm/losses.py)
# --------------------------------------------------------------------------

def _weighted_mean(values, sample_weight):
    """losses.py:25-28."""
    if sample_weight is None:
        return values.mean()
    sample_weight = np.asarray(sample_weight, dtype=np.float64)
    return (values * sample_weight).sum() / sample_weight.sum()


def logistic_loss(y, raw, label_smoothing=0.0, sample_weight=None):
    """losses.py:31-42: max(s, 0) - s*y + log1p(exp(-|s|)), smoothed target."""
    y = np.asarray(y, dtype=np.float64)
    s = np.asarray(raw, dtype=np.float64)
    if label_smoothing:
        y = y * (1.0 - label_smoothing) + 0.5 * label_smoothing
    return _weighted_mean(np.maximum(s, 0.0) - s * y + np.log1p(np.exp(-np.abs(s))),
                          sample_weight)


def squared_loss(y, raw, sample_weight=None):
    """losses.py:64-68: 0.5 (s - y)^2."""
    y = np.asarray(y, dtype=np.float64)
    s = np.asarray(raw, dtype=np.float64)
    return _weighted_mean(0.5 * (s - y) ** 2, sample_weight)


# --------------------------------------------------------------------------
# prediction
# --------------------------------------------------------------------------

def fm_predict_fast_csr(indptr, indices, data, n_features, w0, w, v, n_threads=1):
    indptr, indices, data, w, v = _i64(indptr), _i64(indices), _f64(data), _f64(w), _f64(v)
    _check_csr(indptr, indices, data, n_features)
    out = np.empty(len(indptr) - 1)
    lib().orc_fm_predict_csr(_p(indptr, _i64p), _p(indices, _i64p), _p(data),
                             ct.c_int64(len(out)), ct.c_double(w0), _p(w), _p(v),
                             ct.c_int64(v.shape[1]), _p(out), ct.c_int(_nthreads(n_threads)))
    return out


def fm_predict_fast_dense(x, w0, w, v):
    x, w, v = _f64(x), _f64(w), _f64(v)
    out = np.empty(x.shape[0])
    lib().orc_fm_predict_dense(_p(x), ct.c_int64(x.shape[0]), ct.c_int64(x.shape[1]),
                               ct.c_double(w0), _p(w), _p(v), ct.c_int64(v.shape[1]), _p(out))
    return out


def ffm_predict_csr(indptr, indices, data, n_features, field_ids, w0, w, v, n_threads=1):
    indptr, indices, data = _i64(indptr), _i64(indices), _f64(data)
    field_ids, w, v = _i64(field_ids), _f64(w), _f64(v)
    _check_field_ids(field_ids, n_features, v.shape[1])
    _check_csr(indptr, indices, data, n_features)
    out = np.empty(len(indptr) - 1)
    lib().orc_ffm_predict_csr(_p(indptr, _i64p), _p(indices, _i64p), _p(data),
                              ct.c_int64(len(out)), _p(field_ids, _i64p), ct.c_double(w0),
                              _p(w), _p(v), ct.c_int64(v.shape[1]), ct.c_int64(v.shape[2]),
                              _p(out), ct.c_int(_nthreads(n_threads)))
    return out


def ffm_predict_dense(x, field_ids, w0, w, v):
    x, field_ids, w, v = _f64(x), _i64(field_ids), _f64(w), _f64(v)
    _check_field_ids(field_ids, x.shape[1], v.shape[1])
    out = np.empty(x.shape[0])
    lib().orc_ffm_predict_dense(_p(x), ct.c_int64(x.shape[0]), ct.c_int64(x.shape[1]),
                                _p(field_ids, _i64p), ct.c_double(w0), _p(w), _p(v),
                                ct.c_int64(v.shape[1]), ct.c_int64(v.shape[2]), _p(out))
    return out


def fwfm_predict_csr(indptr, indices, data, n_features, field_ids, w0, w, v, r, n_threads=1):
    indptr, indices, data = _i64(indptr), _i64(indices), _f64(data)
    field_ids, w, v, r = _i64(field_ids), _f64(w), _f64(v), _f64(r)
    if r.ndim != 2 or r.shape[0] != r.shape[1]:
        raise ValueError(f"R must be square, got {list(r.shape)}")
    _check_field_ids(field_ids, n_features, r.shape[0])
    _check_csr(indptr, indices, data, n_features)
    out = np.empty(len(indptr) - 1)
    lib().orc_fwfm_predict_csr(_p(indptr, _i64p), _p(indices, _i64p), _p(data),
                               ct.c_int64(len(out)), _p(field_ids, _i64p), ct.c_double(w0),
                               _p(w), _p(v), _p(r), ct.c_int64(r.shape[0]),
                               ct.c_int64(v.shape[1]), _p(out), ct.c_int(_nthreads(n_threads)))
    return out


def fwfm_predict_dense(x, field_ids, w0, w, v, r):
    x, field_ids, w, v, r = _f64(x), _i64(field_ids), _f64(w), _f64(v), _f64(r)
    if r.ndim != 2 or r.shape[0] != r.shape[1]:
        raise ValueError(f"R must be square, got {list(r.shape)}")
    _check_field_ids(field_ids, x.shape[1], r.shape[0])
    out = np.empty(x.shape[0])
    lib().orc_fwfm_predict_dense(_p(x), ct.c_int64(x.shape[0]), ct.c_int64(x.shape[1]),
                                 _p(field_ids, _i64p), ct.c_double(w0), _p(w), _p(v), _p(r),
                                 ct.c_int64(r.shape[0]), ct.c_int64(v.shape[1]), _p(out))
    return out


# --------------------------------------------------------------------------
# training
# --------------------------------------------------------------------------

def _opt(optimizer, lr, beta_1, beta_2, epsilon, ftrl_beta, l1_linear, l2_linear,
         l1_factors, l2_factors):
    if optimizer not in OPTIMIZERS:
        raise ValueError(f"unknown optimizer {optimizer!r}")
    return _Opt(OPTIMIZERS[optimizer], lr, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
                l2_linear, l1_factors, l2_factors)


def _state(**arrs):
    st = _State()
    for name, a in arrs.items():
        setattr(st, name, _p(a))
    return st


def _rw(a, shape_like=None):
    """In-place float64 C-contiguous array required (PyReadwriteArray)."""
    if not isinstance(a, np.ndarray) or a.dtype != np.float64 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float64 ndarray")
    return a


def _ro(indptr, indices, data, y, sw, row_orders, y_dtype=np.float64):
    return (_i64(indptr), _i64(indices), _f64(data),
            np.ascontiguousarray(y, dtype=y_dtype), _f64(sw), _i64(row_orders))


def _check_fit(indptr, indices, data, n_features, y, sw, ro, n_classes=None):
    _check_csr(indptr, indices, data, n_features)
    n_rows = len(indptr) - 1
    if len(y) != n_rows:
        raise ValueError(f"y length {len(y)} != n_rows {n_rows}")
    if n_classes is not None and np.any((y < 0) | (y >= n_classes)):
        raise ValueError(f"class index out of range [0, {n_classes})")
    if len(sw) != n_rows:
        raise ValueError(f"sample_weight length {len(sw)} != n_rows {n_rows}")
    if ro.ndim != 2 or ro.shape[1] != n_rows:
        raise ValueError(f"row_orders second dimension {ro.shape[-1]} != n_rows {n_rows}")
    if ro.size and (ro.min() < 0 or ro.max() >= n_rows):
        raise ValueError(f"row_orders entry out of range [0, {n_rows})")


def _binary_states(optimizer, adam_state, ftrl_state, shapes, acc_w0):
    """Unpack the binary (scalar-w0) state tuples of rust/src/lib.rs:39-72.

    Returns (scalars, states-per-group, keepalive). Groups: w0, then one per
    array in `shapes` (w, V[, R]). The scalar w0 state lives in 1-element
    arrays that are read back into the returned tuple."""
    if adam_state is not None and optimizer != "adam":
        raise ValueError("adam_state is only valid for optimizer='adam'")
    if ftrl_state is not None and optimizer != "ftrl":
        raise ValueError("ftrl_state is only valid for optimizer='ftrl'")
    g = len(shapes)
    s0 = {"acc": np.array([acc_w0], dtype=np.float64)}
    if optimizer == "adam":
        sc = adam_state[:3] if adam_state is not None else (0.0, 0.0, 0.0)
        s0.update(m=np.array([sc[0]]), s=np.array([sc[1]]), t=np.array([sc[2]]))
        arrs = (list(adam_state[3:]) if adam_state is not None
                else [np.zeros(sh) for sh in shapes for _ in range(3)])
        groups = [dict(m=_rw(arrs[3 * i]), s=_rw(arrs[3 * i + 1]), t=_rw(arrs[3 * i + 2]))
                  for i in range(g)]
        for i, sh in enumerate(shapes):
            for kk in ("m", "s", "t"):
                if groups[i][kk].size != int(np.prod(sh)):
                    raise ValueError("adam_state shapes must match w and V")
    elif optimizer == "ftrl":
        sc = ftrl_state[:2] if ftrl_state is not None else (0.0, 0.0)
        s0.update(z=np.array([sc[0]]), n=np.array([sc[1]]))
        arrs = (list(ftrl_state[2:]) if ftrl_state is not None
                else [np.zeros(sh) for sh in shapes for _ in range(2)])
        groups = [dict(z=_rw(arrs[2 * i]), n=_rw(arrs[2 * i + 1])) for i in range(g)]
        for i, sh in enumerate(shapes):
            for kk in ("z", "n"):
                if groups[i][kk].size != int(np.prod(sh)):
                    raise ValueError("ftrl_state shapes must match w and V")
    else:
        groups = [dict() for _ in range(g)]
    return s0, groups


def _binary_return(w0, s0):
    m = (float(s0["m"][0]), float(s0["s"][0]), float(s0["t"][0])) if "m" in s0 else (0.0, 0.0, 0.0)
    z = (float(s0["z"][0]), float(s0["n"][0])) if "z" in s0 else (0.0, 0.0)
    return float(w0[0]), float(s0["acc"][0]), m, z


def fm_fit_csr(indptr, indices, data, n_features, y, sample_weight, w0, acc_w0, w, v, acc_w,
               acc_v, loss, optimizer, learning_rate, l2_linear, l2_factors, beta_1, beta_2,
               epsilon, row_orders, batch_size, n_jobs, l1_linear, l1_factors, ftrl_beta,
               adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:283-439 (CPU branch -> fm::fit_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    if loss not in LOSSES:
        raise ValueError(f"unknown loss {loss!r}")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders)
    w, v, acc_w, acc_v = _rw(w), _rw(v), _rw(acc_w), _rw(acc_v)
    k = v.shape[1]
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, V rows={v.shape[0]}")
    if acc_w.size != w.size or acc_v.size != v.size:
        raise ValueError("accumulator shapes must match w and V")
    s0, (gw, gv) = _binary_states(optimizer, adam_state, ftrl_state, [w.shape, v.shape], acc_w0)
    _check_fit(indptr, indices, data, n_features, y, sw, ro)
    w0a = np.array([w0], dtype=np.float64)
    rc = lib().orc_fm_fit_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y), _p(sw), _p(w0a), _p(w), _p(v), ct.c_int64(k),
        _state(**s0), _state(acc=acc_w, **gw), _state(acc=acc_v, **gv), ct.c_int(LOSSES[loss]),
        ct.byref(opt), _p(ro, _i64p), ct.c_int64(ro.shape[0]), ct.c_int64(batch_size),
        ct.c_int(max(1, int(n_jobs))))
    if rc:
        raise MemoryError("oracle allocation failed")
    return _binary_return(w0a, s0)


def ffm_fit_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0, acc_w0, w,
                v, acc_w, acc_v, loss, optimizer, learning_rate, l2_linear, l2_factors, beta_1,
                beta_2, epsilon, row_orders, batch_size, n_jobs, l1_linear, l1_factors,
                ftrl_beta, adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:635-793 (CPU branch -> ffm::fit_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    if loss not in LOSSES:
        raise ValueError(f"unknown loss {loss!r}")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders)
    field_ids = _i64(field_ids)
    w, v, acc_w, acc_v = _rw(w), _rw(v), _rw(acc_w), _rw(acc_v)
    n_fields, k = v.shape[1], v.shape[2]
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, V rows={v.shape[0]}")
    _check_field_ids(field_ids, n_features, n_fields)
    if acc_w.size != w.size or acc_v.size != v.size:
        raise ValueError("accumulator shapes must match w and V")
    s0, (gw, gv) = _binary_states(optimizer, adam_state, ftrl_state, [w.shape, v.shape], acc_w0)
    _check_fit(indptr, indices, data, n_features, y, sw, ro)
    w0a = np.array([w0], dtype=np.float64)
    rc = lib().orc_ffm_fit_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y), _p(sw), _p(field_ids, _i64p), ct.c_int64(n_fields),
        _p(w0a), _p(w), _p(v), ct.c_int64(k), _state(**s0), _state(acc=acc_w, **gw),
        _state(acc=acc_v, **gv), ct.c_int(LOSSES[loss]), ct.byref(opt), _p(ro, _i64p),
        ct.c_int64(ro.shape[0]), ct.c_int64(batch_size), ct.c_int(max(1, int(n_jobs))))
    if rc:
        raise MemoryError("oracle allocation failed")
    return _binary_return(w0a, s0)


def fwfm_fit_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0, acc_w0, w,
                 v, r, acc_w, acc_v, acc_r, loss, optimizer, learning_rate, l2_linear,
                 l2_factors, beta_1, beta_2, epsilon, row_orders, batch_size, l1_linear,
                 l1_factors, ftrl_beta, adam_state=None, ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:1049-1242 (CPU branch -> fwfm::fit_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    if loss not in LOSSES:
        raise ValueError(f"unknown loss {loss!r}")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders)
    field_ids = _i64(field_ids)
    w, v, r, acc_w, acc_v, acc_r = _rw(w), _rw(v), _rw(r), _rw(acc_w), _rw(acc_v), _rw(acc_r)
    k, n_fields = v.shape[1], r.shape[0]
    if r.shape[1] != n_fields:
        raise ValueError(f"R must be square, got {list(r.shape)}")
    if w.size != n_features or v.shape[0] != n_features:
        raise ValueError(f"shape mismatch: n_features={n_features}, w={w.size}, V rows={v.shape[0]}")
    _check_field_ids(field_ids, n_features, n_fields)
    if acc_w.size != w.size or acc_v.size != v.size or acc_r.size != r.size:
        raise ValueError("accumulator shapes must match w, V and R")
    s0, (gw, gv, gr) = _binary_states(optimizer, adam_state, ftrl_state,
                                      [w.shape, v.shape, r.shape], acc_w0)
    _check_fit(indptr, indices, data, n_features, y, sw, ro)
    w0a = np.array([w0], dtype=np.float64)
    rc = lib().orc_fwfm_fit_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y), _p(sw), _p(field_ids, _i64p), ct.c_int64(n_fields),
        _p(w0a), _p(w), _p(v), _p(r), ct.c_int64(k), _state(**s0), _state(acc=acc_w, **gw),
        _state(acc=acc_v, **gv), _state(acc=acc_r, **gr), ct.c_int(LOSSES[loss]),
        ct.byref(opt), _p(ro, _i64p), ct.c_int64(ro.shape[0]), ct.c_int64(batch_size))
    if rc:
        raise MemoryError("oracle allocation failed")
    return _binary_return(w0a, s0)


def _mc_states(optimizer, state, adam_state, ftrl_state, shapes):
    """Multiclass state tuples (rust/src/lib.rs:45-72): every array (C, ...)
    mutated in place; zero-filled locals when None."""
    if adam_state is not None and optimizer != "adam":
        raise ValueError("adam_state is only valid for optimizer='adam'")
    if ftrl_state is not None and optimizer != "ftrl":
        raise ValueError("ftrl_state is only valid for optimizer='ftrl'")
    g = len(shapes)
    accs = [_rw(a) for a in state] if state is not None else [np.zeros(sh) for sh in shapes]
    if len(accs) != g or any(a.size != int(np.prod(sh)) for a, sh in zip(accs, shapes)):
        raise ValueError("state shapes must match (w0, w, V)")
    groups = [dict(acc=accs[i]) for i in range(g)]
    if optimizer == "adam":
        arrs = ([_rw(a) for a in adam_state] if adam_state is not None
                else [np.zeros(sh) for sh in shapes for _ in range(3)])
        for i, sh in enumerate(shapes):
            for j, kk in enumerate(("m", "s", "t")):
                a = arrs[3 * i + j]
                if a.size != int(np.prod(sh)):
                    raise ValueError("adam_state shapes must match (w0, w, V)")
                groups[i][kk] = a
    elif optimizer == "ftrl":
        arrs = ([_rw(a) for a in ftrl_state] if ftrl_state is not None
                else [np.zeros(sh) for sh in shapes for _ in range(2)])
        for i, sh in enumerate(shapes):
            for j, kk in enumerate(("z", "n")):
                a = arrs[2 * i + j]
                if a.size != int(np.prod(sh)):
                    raise ValueError("ftrl_state shapes must match (w0, w, V)")
                groups[i][kk] = a
    return groups


def fm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, w0, w, v,
                          optimizer, learning_rate, l2_linear, l2_factors, label_smoothing,
                          beta_1, beta_2, epsilon, row_orders, batch_size, l1_linear,
                          l1_factors, ftrl_beta, state=None, adam_state=None, ftrl_state=None,
                          use_cuda=False):
    """rust/src/lib.rs:449-630 (CPU branch -> fm::fit_multiclass_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders,
                                           y_dtype=np.int64)
    w0, w, v = _rw(w0), _rw(w), _rw(v)
    C, k = v.shape[0], v.shape[2]
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}")
    g0, gw, gv = _mc_states(optimizer, state, adam_state, ftrl_state,
                            [w0.shape, w.shape, v.shape])
    _check_fit(indptr, indices, data, n_features, y, sw, ro, n_classes=C)
    rc = lib().orc_fm_fit_multiclass_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y, _i64p), _p(sw), ct.c_int64(C), _p(w0), _p(w), _p(v),
        ct.c_int64(k), _state(**g0), _state(**gw), _state(**gv), ct.byref(opt),
        ct.c_double(label_smoothing), _p(ro, _i64p), ct.c_int64(ro.shape[0]),
        ct.c_int64(batch_size))
    if rc:
        raise MemoryError("oracle allocation failed")


def ffm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0,
                           w, v, optimizer, learning_rate, l2_linear, l2_factors,
                           label_smoothing, beta_1, beta_2, epsilon, row_orders, batch_size,
                           l1_linear, l1_factors, ftrl_beta, state=None, adam_state=None,
                           ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:800-978 (CPU branch -> ffm::fit_multiclass_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders,
                                           y_dtype=np.int64)
    field_ids = _i64(field_ids)
    w0, w, v = _rw(w0), _rw(w), _rw(v)
    C, n_fields, k = v.shape[0], v.shape[2], v.shape[3]
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}")
    _check_field_ids(field_ids, n_features, n_fields)
    g0, gw, gv = _mc_states(optimizer, state, adam_state, ftrl_state,
                            [w0.shape, w.shape, v.shape])
    _check_fit(indptr, indices, data, n_features, y, sw, ro, n_classes=C)
    rc = lib().orc_ffm_fit_multiclass_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y, _i64p), _p(sw), ct.c_int64(C), _p(field_ids, _i64p),
        ct.c_int64(n_fields), _p(w0), _p(w), _p(v), ct.c_int64(k), _state(**g0), _state(**gw),
        _state(**gv), ct.byref(opt), ct.c_double(label_smoothing), _p(ro, _i64p),
        ct.c_int64(ro.shape[0]), ct.c_int64(batch_size))
    if rc:
        raise MemoryError("oracle allocation failed")


def fwfm_fit_multiclass_csr(indptr, indices, data, n_features, y, sample_weight, field_ids, w0,
                            w, v, r, optimizer, learning_rate, l2_linear, l2_factors,
                            label_smoothing, beta_1, beta_2, epsilon, row_orders, batch_size,
                            l1_linear, l1_factors, ftrl_beta, state=None, adam_state=None,
                            ftrl_state=None, use_cuda=False):
    """rust/src/lib.rs:1249-1466 (CPU branch -> fwfm::fit_multiclass_csr)."""
    if use_cuda:
        raise ValueError("the oracle is the CPU engine; use_cuda=True is not served here")
    opt = _opt(optimizer, learning_rate, beta_1, beta_2, epsilon, ftrl_beta, l1_linear,
               l2_linear, l1_factors, l2_factors)
    if batch_size == 0:
        raise ValueError("batch_size must be >= 1")
    indptr, indices, data, y, sw, ro = _ro(indptr, indices, data, y, sample_weight, row_orders,
                                           y_dtype=np.int64)
    field_ids = _i64(field_ids)
    w0, w, v, r = _rw(w0), _rw(w), _rw(v), _rw(r)
    C, k, n_fields = v.shape[0], v.shape[2], r.shape[1]
    if r.shape[0] != C or r.shape[2] != n_fields:
        raise ValueError(f"R must be (n_classes, n_fields, n_fields), got {list(r.shape)}")
    if w0.size != C or w.shape != (C, n_features) or v.shape[1] != n_features:
        raise ValueError(f"shape mismatch: n_classes={C}, n_features={n_features}")
    _check_field_ids(field_ids, n_features, n_fields)
    g0, gw, gv, gr = _mc_states(optimizer, state, adam_state, ftrl_state,
                                [w0.shape, w.shape, v.shape, r.shape])
    _check_fit(indptr, indices, data, n_features, y, sw, ro, n_classes=C)
    rc = lib().orc_fwfm_fit_multiclass_csr(
        _p(indptr, _i64p), _p(indices, _i64p), _p(data), ct.c_int64(len(indptr) - 1),
        ct.c_int64(n_features), _p(y, _i64p), _p(sw), ct.c_int64(C), _p(field_ids, _i64p),
        ct.c_int64(n_fields), _p(w0), _p(w), _p(v), _p(r), ct.c_int64(k), _state(**g0),
        _state(**gw), _state(**gv), _state(**gr), ct.byref(opt), ct.c_double(label_smoothing),
        _p(ro, _i64p), ct.c_int64(ro.shape[0]), ct.c_int64(batch_size))
    if rc:
        raise MemoryError("oracle allocation failed")


def sigmoid(s: float) -> float:
    return lib().orc_sigmoid(ct.c_double(s))


CPU_FUNCTIONS = (
    "fm_predict_fast_dense", "fm_predict_fast_csr", "ffm_predict_dense", "ffm_predict_csr",
    "fwfm_predict_dense", "fwfm_predict_csr", "fm_fit_csr", "fm_fit_multiclass_csr",
    "ffm_fit_csr", "ffm_fit_multiclass_csr", "fwfm_fit_csr", "fwfm_fit_multiclass_csr",
)
