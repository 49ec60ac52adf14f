"""Early-stopping evaluation on the device (mfm_{fm,ffm,fwfm}_eval_device).

The reference evaluates the validation set on the host after every epoch of
an early-stopped fit: ``metric(y_val, fm_predict_fast(X_val, w0, w, V))``
(python/modern_fm/fm.py:321-322), and ffm_predict / fwfm_predict for the FFM
and FwFM estimators (python/modern_fm/ffm.py:210-212,
python/modern_fm/fwfm.py:157-161), metric from python/modern_fm/losses.py.
``fm_eval_device`` / ``ffm_eval_device`` / ``fwfm_eval_device`` compute the
same value from a device-resident validation CSR and device-resident
parameters; only the scalar loss leaves the GPU.
"""

from __future__ import annotations

import ctypes as ct

from . import _lib


def _dtype_code(data, params):
    """Compute type from the tensors: all float32, all float64, or float64
    data with float32 parameters (float64 arithmetic)."""
    import torch

    pd = {p.dtype for p in params}
    if len(pd) != 1:
        raise ValueError("w, v (and r) must share one dtype")
    pd = pd.pop()
    if data.dtype == torch.float32 and pd == torch.float32:
        return _lib.MFM_DTYPE_F32
    if data.dtype == torch.float64 and pd == torch.float64:
        return _lib.MFM_DTYPE_F64
    if data.dtype == torch.float64 and pd == torch.float32:
        return _lib.MFM_DTYPE_F32_F64
    raise ValueError("data and parameters must be float32 / float32, float64 / float64 or "
                     "float64 data with float32 parameters")


def _common(indptr, indices, data, params, y, sample_weight, loss):
    import torch

    if loss not in _lib.LOSSES:
        raise ValueError(f"loss must be one of {sorted(_lib.LOSSES)}")
    code = _dtype_code(data, params)
    if indptr.dtype != torch.int64 or indices.dtype != torch.int32:
        raise ValueError("indptr must be int64 and indices int32")
    if y.dtype != torch.float64 or (sample_weight is not None
                                    and sample_weight.dtype != torch.float64):
        raise ValueError("y and sample_weight must be float64")
    ts = [indptr, indices, data, y] + list(params) + (
        [sample_weight] if sample_weight is not None else [])
    if not all(t.is_cuda and t.is_contiguous() for t in ts):
        raise ValueError("every array must be a contiguous CUDA tensor")
    n_rows = indptr.numel() - 1
    if y.numel() != n_rows or (sample_weight is not None and sample_weight.numel() != n_rows):
        raise ValueError("y and sample_weight must have one entry per row")
    dev = indptr.device
    return code, n_rows, dev, dev.index if dev.index is not None else torch.cuda.current_device()


def _finish(rc, out):
    if rc < 0:
        raise ValueError(_lib.last_error())
    if rc != 0:
        raise RuntimeError(_lib.last_error())
    return out.value


def _stream(stream, dev):
    import torch

    return (stream if stream is not None else torch.cuda.current_stream(dev)).cuda_stream


def fm_eval_device(indptr, indices, data, w0: float, w, v, y, sample_weight=None,
                   loss: str = "logistic", label_smoothing: float = 0.0, stream=None) -> float:
    """Mean validation loss of an FM on CUDA tensors.

    ``indptr`` int64 (n_rows + 1), ``indices`` int32, ``data``, ``w`` and
    ``v`` (n_features, k) all float32, all float64, or float64 data with
    float32 parameters (float64 arithmetic), as produced by
    ``prep.prep_csr_device``; ``y`` and ``sample_weight`` float64. ``loss`` is
    "logistic" (binary cross-entropy from raw scores, with the reference's
    label smoothing of the target) or "squared" (0.5 (s - y)^2). Raises
    ValueError for invalid arguments, RuntimeError for CUDA failures.
    """
    code, n_rows, dev, di = _common(indptr, indices, data, (w, v), y, sample_weight, loss)
    if v.dim() != 2 or v.shape[0] != w.numel():
        raise ValueError("v must have shape (n_features, k)")
    out = ct.c_double(0.0)
    rc = _lib.lib().mfm_fm_eval_device(
        code, di, indptr.data_ptr(), indices.data_ptr(), data.data_ptr(), n_rows, float(w0),
        w.data_ptr(), v.data_ptr(), int(v.shape[1]), y.data_ptr(),
        sample_weight.data_ptr() if sample_weight is not None else None,
        _lib.LOSSES[loss], float(label_smoothing), ct.byref(out), _stream(stream, dev))
    return _finish(rc, out)


def ffm_eval_device(indptr, indices, data, field_ids, w0: float, w, v, y, sample_weight=None,
                    loss: str = "logistic", label_smoothing: float = 0.0, stream=None) -> float:
    """Mean validation loss of an FFM: ``v`` (n_features, n_fields, k),
    ``field_ids`` int32 CUDA tensor (n_features); otherwise as
    ``fm_eval_device``."""
    import torch

    code, n_rows, dev, di = _common(indptr, indices, data, (w, v), y, sample_weight, loss)
    if v.dim() != 3 or v.shape[0] != w.numel():
        raise ValueError("v must have shape (n_features, n_fields, k)")
    if field_ids.dtype != torch.int32 or field_ids.numel() != w.numel() or not field_ids.is_cuda:
        raise ValueError("field_ids must be an int32 CUDA tensor with one entry per feature")
    out = ct.c_double(0.0)
    rc = _lib.lib().mfm_ffm_eval_device(
        code, di, indptr.data_ptr(), indices.data_ptr(), data.data_ptr(), n_rows,
        field_ids.data_ptr(), int(v.shape[1]), float(w0), w.data_ptr(), v.data_ptr(),
        int(v.shape[2]), y.data_ptr(),
        sample_weight.data_ptr() if sample_weight is not None else None,
        _lib.LOSSES[loss], float(label_smoothing), ct.byref(out), _stream(stream, dev))
    return _finish(rc, out)


def fwfm_eval_device(indptr, indices, data, field_ids, w0: float, w, v, r, y,
                     sample_weight=None, loss: str = "logistic", label_smoothing: float = 0.0,
                     stream=None) -> float:
    """Mean validation loss of a FwFM: ``v`` (n_features, k), ``r``
    (n_fields, n_fields), ``field_ids`` int32 CUDA tensor (n_features);
    otherwise as ``fm_eval_device``."""
    import torch

    code, n_rows, dev, di = _common(indptr, indices, data, (w, v, r), y, sample_weight, loss)
    if v.dim() != 2 or v.shape[0] != w.numel() or r.dim() != 2 or r.shape[0] != r.shape[1]:
        raise ValueError("v must have shape (n_features, k) and r (n_fields, n_fields)")
    if field_ids.dtype != torch.int32 or field_ids.numel() != w.numel() or not field_ids.is_cuda:
        raise ValueError("field_ids must be an int32 CUDA tensor with one entry per feature")
    out = ct.c_double(0.0)
    rc = _lib.lib().mfm_fwfm_eval_device(
        code, di, indptr.data_ptr(), indices.data_ptr(), data.data_ptr(), n_rows,
        field_ids.data_ptr(), int(r.shape[0]), float(w0), w.data_ptr(), v.data_ptr(),
        r.data_ptr(), int(v.shape[1]), y.data_ptr(),
        sample_weight.data_ptr() if sample_weight is not None else None,
        _lib.LOSSES[loss], float(label_smoothing), ct.byref(out), _stream(stream, dev))
    return _finish(rc, out)
