"""Device-side CSR canonicalisation (mfm_csr_prep_device).

The reference canonicalises every CSR on the host before each native call:
``X.tocsr().astype(np.float64); X.sum_duplicates()`` and int64 / float64 copies
(python/modern_fm/_backend.py:44-52). ``prep_csr_device`` does that work on
data already in GPU memory and returns the canonical CSR in the layout the
engine's ``*_device`` entry points take (int32 columns, values in the compute
dtype), so a raw CSR uploaded once never goes back through the host.
"""

from __future__ import annotations

import ctypes as ct

from . import _lib

_DTYPES = {"float32": _lib.MFM_DTYPE_F32, "float64": _lib.MFM_DTYPE_F64}


def prep_csr_device(indptr, indices, data, n_features: int, dtype: str = "float32",
                    stream=None):
    """Canonicalise a device CSR: validate it, sort each row by column, sum
    duplicate (row, column) entries in float64 (in their original order) and
    narrow to int32 columns and ``dtype`` values.

    ``indptr`` (int64, n_rows + 1), ``indices`` (int64) and ``data`` (float64)
    are CUDA tensors on one device. Returns ``(indptr, indices, data)`` CUDA
    tensors (int64, int32, ``dtype``) holding the canonical entries only.
    Raises ValueError for an invalid CSR (the reference's CsrView messages,
    rust/src/data.rs:14-44) and RuntimeError for a CUDA failure; there is no
    CPU path. ``stream`` is a torch.cuda.Stream (default: the current one).
    """
    import torch

    if dtype not in _DTYPES:
        raise ValueError(f"dtype must be one of {sorted(_DTYPES)}")
    for name, t, want in (("indptr", indptr, torch.int64), ("indices", indices, torch.int64),
                          ("data", data, torch.float64)):
        if not t.is_cuda or t.dtype != want or not t.is_contiguous() or t.dim() != 1:
            raise ValueError(f"{name} must be a contiguous 1-D CUDA {want} tensor")
    if indices.numel() != data.numel():
        raise ValueError("indices and data must have the same length")
    if indptr.numel() < 1:
        raise ValueError("indptr must have length n_rows + 1 (>= 1)")
    dev = indptr.device
    if indices.device != dev or data.device != dev:
        raise ValueError("indptr, indices and data must be on one device")
    n_rows, nnz = indptr.numel() - 1, indices.numel()
    tdt = torch.float32 if dtype == "float32" else torch.float64
    ip_out = torch.empty(n_rows + 1, dtype=torch.int64, device=dev)
    ix_out = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    dv_out = torch.empty(max(nnz, 1), dtype=tdt, device=dev)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    nnz_out = ct.c_int64(0)
    rc = _lib.lib().mfm_csr_prep_device(
        _DTYPES[dtype], dev.index if dev.index is not None else torch.cuda.current_device(),
        n_rows, int(n_features), nnz, indptr.data_ptr(), indices.data_ptr(), data.data_ptr(),
        ip_out.data_ptr(), ix_out.data_ptr(), dv_out.data_ptr(), ct.byref(nnz_out),
        s.cuda_stream)
    if rc < 0:
        raise ValueError(_lib.last_error())
    if rc != 0:
        raise RuntimeError(_lib.last_error())
    m = nnz_out.value
    return ip_out, ix_out[:m], dv_out[:m]
