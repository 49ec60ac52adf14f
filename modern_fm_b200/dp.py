"""Synchronous data-parallel FM / FFM / FwFM training over NCCL (one process per GPU).

Every rank holds the whole training set, the parameters and the optimizer
state. Each global mini-batch (the same row_orders chunking as one GPU) is cut
into `world` contiguous row slices; rank r scores slice r, the per-key gradient
sums over the batch's sorted union of touched keys are summed across ranks
with one ncclAllReduce, and every rank applies the identical optimizer step:
the mini-batch math of a one-GPU fit, up to summation order. The reference has
no multi-GPU training; the single-GPU semantics it defines are
rust/src/fm.rs:373-411 (batch loop) and rust/src/optimizer.rs:48-167 (steps).

    import torch.distributed as dist
    dist.init_process_group("gloo")            # any backend: it carries the group id and
    group = DataParallelGroup(device=local_rank)  # the peer check before each fit
    group.fm_fit_device(...)                    # binary FM on device arrays, or
    group.fit_csr(...)                          # any model, host buffers (every rank, same
    group.close()                               # arguments)

A rank that has left is found by the bounded barrier before each fit; a rank
lost during a fit stops the device's progress, and the engine aborts the NCCL
communicator after MFM_B200_DP_TIMEOUT seconds (the call returns an error and
the group must be recreated).
"""

from __future__ import annotations

import ctypes as ct

from . import _lib

ID_BYTES = 128


def slice_rows(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of a batch of n_rows that rank `rank` of `world` scores
    (the engine's split: floor(n*r/G), floor(n*(r+1)/G))."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    return n_rows * rank // world, n_rows * (rank + 1) // world


def broadcast_unique_id(id_bytes: bytes | None, group=None) -> bytes:
    """The NCCL group id made on rank 0, delivered to every rank through
    torch.distributed (a 128-byte CPU tensor: works on gloo and on nccl)."""
    import torch
    import torch.distributed as dist

    buf = torch.zeros(ID_BYTES, dtype=torch.uint8)
    if dist.get_rank(group) == 0:
        if id_bytes is None or len(id_bytes) != ID_BYTES:
            raise ValueError("rank 0 must supply the 128-byte group id")
        buf[:] = torch.frombuffer(bytearray(id_bytes), dtype=torch.uint8)
    if dist.get_backend(group) == "nccl":
        dev = torch.device("cuda", torch.cuda.current_device())
        t = buf.to(dev)
        dist.broadcast(t, src=0, group=group)
        buf = t.cpu()
    else:
        dist.broadcast(buf, src=0, group=group)
    return bytes(buf.numpy().tobytes())


def check_peers(timeout_s: float = 60.0, group=None) -> None:
    """Every rank of the torch.distributed group is still there: a bounded
    barrier (gloo: monitored_barrier, which names the missing ranks; other
    backends: barrier under the group's own timeout). Raises RuntimeError
    instead of letting the next NCCL collective wait for a rank that left."""
    import datetime

    import torch.distributed as dist

    try:
        if dist.get_backend(group) == "gloo":
            dist.monitored_barrier(group, timeout=datetime.timedelta(seconds=timeout_s))
        else:
            dist.barrier(group)
    except Exception as exc:  # the backends raise several types
        raise RuntimeError(f"data-parallel group: a peer is missing ({exc})") from exc


def new_unique_id() -> bytes:
    out = ct.create_string_buffer(ID_BYTES)
    if _lib.lib().mfm_dp_unique_id(out) != 0:
        raise RuntimeError(_lib.last_error())
    return out.raw


class DataParallelGroup:
    """One NCCL communicator over the torch.distributed world, bound to
    `device` (default: LOCAL_RANK of the current process)."""

    def __init__(self, device: int | None = None, group=None):
        import os

        import torch.distributed as dist

        self._group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = int(os.environ.get("LOCAL_RANK", "0")) if device is None else int(device)
        uid = broadcast_unique_id(new_unique_id() if self.rank == 0 else None, group)
        h = ct.c_void_p()
        if _lib.lib().mfm_dp_create(uid, self.world, self.rank, self.device, ct.byref(h)) != 0:
            raise RuntimeError(_lib.last_error())
        self._h = h

    @property
    def handle(self):
        return self._h

    def fm_fit_device(self, dtype, indptr, indices, data, n_rows, n_features, y, sample_weight,
                      row_orders, train, k, w0, w, v, stream, check_peers_s: float | None = 60.0):
        """mfm_fm_fit_device_dp: device pointers (ints) in the compute dtype,
        `train` an _lib.Train, w0/w/v _lib.DevGroup; raises RuntimeError with
        the engine's message on failure. First checks that every rank is still
        present (check_peers, skipped with check_peers_s=None); during the fit
        the engine aborts the group if no batch completes for
        MFM_B200_DP_TIMEOUT seconds."""
        if check_peers_s is not None:
            check_peers(check_peers_s, self._group)
        rc = _lib.lib().mfm_fm_fit_device_dp(self._h, dtype, indptr, indices, data, n_rows,
                                             n_features, y, sample_weight, row_orders, train, k,
                                             w0, w, v, stream)
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def fit_csr(self, model: str, x, n_features: int, y, sample_weight, params, train, k: int,
                n_classes: int = 1, field_ids=None, n_fields: int | None = None,
                dtype: str = "float64", check_peers_s: float | None = 60.0):
        """mfm_fit_csr_dp: one fit of the reference's host-buffer layout across
        the group. `model` is "fm", "ffm" or "fwfm"; x = (indptr, indices,
        data) (int64 / int64 / float64); y float64 labels (binary,
        n_classes = 1) or int64 class ids (multiclass); `params` a list of
        _lib.Group for w0, w, V (and R for fwfm) over float64 arrays updated
        in place; `train` an _lib.Train with row_orders set. Every rank calls
        it with the same arguments; raises RuntimeError with the engine's
        message on failure."""
        import numpy as np

        if check_peers_s is not None:
            check_peers(check_peers_s, self._group)
        kind = {"fm": _lib.MFM_MODEL_FM, "ffm": _lib.MFM_MODEL_FFM, "fwfm": _lib.MFM_MODEL_FWFM}
        if model not in kind:
            raise ValueError(f"model must be one of {sorted(kind)}")
        csr, keep = _lib.make_csr(x[0], x[1], x[2], n_features)
        mc = n_classes > 1
        yv = np.ascontiguousarray(y, dtype=np.int64 if mc else np.float64)
        sw = np.ascontiguousarray(sample_weight, dtype=np.float64)
        fid = None if field_ids is None else np.ascontiguousarray(field_ids, dtype=np.int64)
        if n_fields is None:
            n_fields = 0 if fid is None or not fid.size else int(fid.max()) + 1
        groups = list(params) + [None] * (4 - len(params))
        rc = _lib.lib().mfm_fit_csr_dp(
            self._h, _lib.dtype_code(dtype), kind[model], int(n_classes), ct.byref(csr),
            None if mc else _lib.ptr(yv), _lib.ptr(yv, _lib.i64p) if mc else None,
            _lib.ptr(sw), _lib.ptr(fid, _lib.i64p), n_fields, ct.byref(train), int(k),
            *[ct.byref(g) if g is not None else None for g in groups])
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def close(self):
        if self._h:
            _lib.lib().mfm_dp_destroy(self._h)
            self._h = None
