"""Early-stopping evaluation on the device (mfm_fm_eval_device).

The reference evaluates the validation set on the host after every epoch of
an early-stopped fit: ``metric(y_val, fm_predict_fast(X_val, w0, w, V))``
(python/modern_fm/fm.py:321-322, metric from python/modern_fm/losses.py).
``fm_eval_device`` computes the same value from a device-resident validation
CSR and device-resident parameters; only the scalar loss leaves the GPU.
"""

from __future__ import annotations

import ctypes as ct

from . import _lib

_DTYPES = {"float32": _lib.MFM_DTYPE_F32, "float64": _lib.MFM_DTYPE_F64}


def fm_eval_device(indptr, indices, data, w0: float, w, v, y, sample_weight=None,
                   loss: str = "logistic", label_smoothing: float = 0.0, stream=None) -> float:
    """Mean validation loss of an FM on CUDA tensors.

    ``indptr`` int64 (n_rows + 1), ``indices`` int32, ``data`` / ``w`` /
    ``v`` (n_features, k) in one compute dtype (float32 or float64), as
    produced by ``prep.prep_csr_device``; ``y`` and ``sample_weight`` float64.
    ``loss`` is "logistic" (binary cross-entropy from raw scores, with the
    reference's label smoothing of the target) or "squared" (0.5 (s - y)^2).
    Raises ValueError for invalid arguments, RuntimeError for CUDA failures.
    """
    import torch

    if loss not in _lib.LOSSES:
        raise ValueError(f"loss must be one of {sorted(_lib.LOSSES)}")
    dt = {torch.float32: "float32", torch.float64: "float64"}.get(data.dtype)
    if dt is None or w.dtype != data.dtype or v.dtype != data.dtype:
        raise ValueError("data, w and v must share one dtype: float32 or float64")
    if indptr.dtype != torch.int64 or indices.dtype != torch.int32:
        raise ValueError("indptr must be int64 and indices int32")
    if y.dtype != torch.float64 or (sample_weight is not None
                                    and sample_weight.dtype != torch.float64):
        raise ValueError("y and sample_weight must be float64")
    ts = [indptr, indices, data, w, v, y] + ([sample_weight] if sample_weight is not None else [])
    if not all(t.is_cuda and t.is_contiguous() for t in ts):
        raise ValueError("every array must be a contiguous CUDA tensor")
    n_rows = indptr.numel() - 1
    if y.numel() != n_rows or (sample_weight is not None and sample_weight.numel() != n_rows):
        raise ValueError("y and sample_weight must have one entry per row")
    if v.dim() != 2 or v.shape[0] != w.numel():
        raise ValueError("v must have shape (n_features, k)")
    dev = indptr.device
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    out = ct.c_double(0.0)
    rc = _lib.lib().mfm_fm_eval_device(
        _DTYPES[dt], dev.index if dev.index is not None else torch.cuda.current_device(),
        indptr.data_ptr(), indices.data_ptr(), data.data_ptr(), n_rows, float(w0),
        w.data_ptr(), v.data_ptr(), int(v.shape[1]), y.data_ptr(),
        sample_weight.data_ptr() if sample_weight is not None else None,
        _lib.LOSSES[loss], float(label_smoothing), ct.byref(out), s.cuda_stream)
    if rc < 0:
        raise ValueError(_lib.last_error())
    if rc != 0:
        raise RuntimeError(_lib.last_error())
    return out.value
