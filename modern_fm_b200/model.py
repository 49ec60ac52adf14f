"""A model resident on the GPU across scoring calls (mfm_model_* in the C ABI).

The reference uploads every parameter on each CUDA predict call
(rust/src/cuda/mod.rs:9-12) and scores a multiclass model with one binary call
per class, re-uploading X each time (python/modern_fm/fm.py:666-674).
``DeviceModel`` uploads the parameters once and scores every class of a row in
one pass; each call moves only the CSR (and the scores back).
"""

from __future__ import annotations

import ctypes as ct

import numpy as np

from . import _lib

_KINDS = {"fm": _lib.MFM_MODEL_FM, "ffm": _lib.MFM_MODEL_FFM, "fwfm": _lib.MFM_MODEL_FWFM}
_NAMES = {v: k for k, v in _lib.DTYPES.items() if "-" in k or k in ("float64", "float32")}


def _check(rc):
    if rc < 0:
        raise ValueError(_lib.last_error())
    if rc != 0:
        raise RuntimeError(_lib.last_error())


class DeviceModel:
    """FM / FFM / FwFM parameters on one GPU.

    ``kind`` is "fm", "ffm" or "fwfm"; ``n_classes`` 1 gives one score per
    row, C >= 2 gives C logits per row (class c scored with class c's
    parameters, as the reference's per-class calls do). ``dtype`` is
    "float32-float64" (float64 arithmetic; parameters stored as float32 when
    every value is exactly a float32, else float64), "float64" or "float32".
    """

    def __init__(self, kind: str, n_features: int, k: int, n_fields: int = 0,
                 n_classes: int = 1, dtype: str = "float32-float64", device: int = 0):
        if kind not in _KINDS:
            raise ValueError(f"kind must be one of {sorted(_KINDS)}")
        self.kind, self.n_features, self.k = kind, int(n_features), int(k)
        self.n_fields, self.n_classes, self.device = int(n_fields), int(n_classes), int(device)
        self._dtype = _lib.dtype_code(dtype)
        h = ct.c_void_p()
        _check(_lib.lib().mfm_model_create(_KINDS[kind], self._dtype, self.device,
                                           self.n_features, self.n_fields, self.k,
                                           self.n_classes, ct.byref(h)))
        self._h = h

    def set_params(self, w0, w, V, R=None, field_ids=None):
        """Uploads parameters in the reference's layout (float64 arrays;
        multiclass class-major: w0 (C,), w (C, n), V (C, n, k) or FFM
        (C, n, F, k), R (C, F, F))."""
        C, n, k, F = self.n_classes, self.n_features, self.k, self.n_fields
        w0a = np.ascontiguousarray(np.atleast_1d(np.asarray(w0, dtype=np.float64)))
        w = np.ascontiguousarray(w, dtype=np.float64)
        V = np.ascontiguousarray(V, dtype=np.float64)
        lead = (C,) if C > 1 else ()
        vshape = lead + ((n, F, k) if self.kind == "ffm" else (n, k))
        if w0a.size != C or w.shape != lead + (n,) or V.shape != vshape:
            raise ValueError(f"shape mismatch: w0 {w0a.shape}, w {w.shape}, V {V.shape} for "
                             f"n_classes={C}, n_features={n}, k={k}")
        Ra = None
        if self.kind == "fwfm":
            if R is None:
                raise ValueError("R is required for fwfm")
            Ra = np.ascontiguousarray(R, dtype=np.float64)
            if Ra.shape != lead + (F, F):
                raise ValueError(f"R must have shape {lead + (F, F)}")
        fid = None
        if self.kind != "fm":
            if field_ids is None:
                raise ValueError("field_ids is required for ffm / fwfm")
            fid = np.ascontiguousarray(field_ids, dtype=np.int64)
        self._keep = (w0a, w, V, Ra, fid)
        _check(_lib.lib().mfm_model_set_params(self._h, _lib.ptr(w0a), _lib.ptr(w), _lib.ptr(V),
                                               _lib.ptr(Ra), _lib.ptr(fid, _lib.i64p)))
        self._keep = None

    @property
    def dtype_used(self) -> str:
        """The compute type scoring runs in (float32-float64 becomes float64
        when the parameters are not exactly float32)."""
        d = ct.c_int(0)
        _check(_lib.lib().mfm_model_info(self._h, ct.byref(d)))
        return {_lib.MFM_DTYPE_F64: "float64", _lib.MFM_DTYPE_F32: "float32",
                _lib.MFM_DTYPE_F32_F64: "float32-float64"}[d.value]

    def predict_csr(self, indptr, indices, data, out=None):
        """Scores a host CSR (int64 / float64, the reference's boundary
        format); returns float64 scores (n_rows,) or (n_rows, C)."""
        csr, keep = _lib.make_csr(indptr, indices, data, self.n_features)
        n = csr.n_rows
        shape = (n,) if self.n_classes == 1 else (n, self.n_classes)
        if out is None:
            out = np.empty(shape, dtype=np.float64)
        elif out.shape != shape or out.dtype != np.float64 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float64 array of shape {shape}")
        _check(_lib.lib().mfm_model_predict_csr(self._h, ct.byref(csr), _lib.ptr(out)))
        return out

    def predict_device(self, indptr, indices, data, out, stream=None):
        """Scores a canonical device CSR (torch tensors: int64 indptr, int32
        indices; data float32 for dtype float32, float64 otherwise) into
        ``out`` on ``stream`` (default: the current torch stream)."""
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(indptr.device)
        _check(_lib.lib().mfm_model_predict_device(self._h, indptr.data_ptr(),
                                                   indices.data_ptr(), data.data_ptr(),
                                                   indptr.numel() - 1, out.data_ptr(),
                                                   s.cuda_stream))
        return out

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().mfm_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
