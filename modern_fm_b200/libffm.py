"""libffm files into the engine: the reference's load_libffm
(python/modern_fm/libffm.py:31-83) as a native multi-threaded reader
(mfm_libffm_read) followed by device canonicalisation (mfm_csr_prep_device).
"""

from __future__ import annotations

import ctypes as ct
import os

import numpy as np

from . import _lib


def read_libffm_raw(path, n_threads: int = 0):
    """Parse a libffm file on the host with the native reader.

    Returns ``(indptr, indices, data, y, field_ids, n_features)`` as NumPy
    arrays in the boundary format: rows in file order, entries in token order
    with duplicates kept (not yet canonical), float64 labels, int64 field id
    per feature. Raises ValueError with the reference's messages.
    """
    L = _lib.lib()
    h = ct.c_void_p()
    rc = L.mfm_libffm_read(os.fsencode(os.fspath(path)), int(n_threads), ct.byref(h))
    if rc != 0:
        raise ValueError(_lib.last_error())
    try:
        n_rows, nnz, nf = ct.c_int64(), ct.c_int64(), ct.c_int64()
        L.mfm_libffm_info(h, ct.byref(n_rows), ct.byref(nnz), ct.byref(nf))
        ptrs = [ct.c_void_p() for _ in range(5)]
        L.mfm_libffm_arrays(h, *[ct.byref(p) for p in ptrs])

        def copy(p, n, dt):
            if n == 0:
                return np.zeros(0, dtype=dt)
            return np.ctypeslib.as_array(ct.cast(p, ct.POINTER(np.ctypeslib.as_ctypes_type(dt))),
                                         shape=(n,)).copy()

        indptr = copy(ptrs[0], n_rows.value + 1, np.int64)
        indices = copy(ptrs[1], nnz.value, np.int64)
        data = copy(ptrs[2], nnz.value, np.float64)
        y = copy(ptrs[3], n_rows.value, np.float64)
        field_ids = copy(ptrs[4], nf.value, np.int64)
    finally:
        L.mfm_libffm_free(h)
    return indptr, indices, data, y, field_ids, nf.value


def load_libffm_device(path, dtype: str = "float32", n_threads: int = 0, device=None):
    """load_libffm onto the GPU: read on the host, upload the raw CSR, and
    canonicalise it on the device (sorted rows, duplicates summed in float64,
    int32 columns, ``dtype`` values).

    Returns ``(indptr, indices, data, y, field_ids, n_features)``: the first
    four are CUDA tensors (y float64), field_ids a NumPy int64 array (the
    argument the reference's FFM / FwFM estimators take).
    """
    import torch

    from .prep import prep_csr_device

    ip, ix, dv, y, field_ids, nf = read_libffm_raw(path, n_threads)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else int(device))
    up = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    ip_d, ix_d, dv_d = prep_csr_device(up(ip), up(ix), up(dv), nf, dtype=dtype)
    return ip_d, ix_d, dv_d, up(y), field_ids, nf
