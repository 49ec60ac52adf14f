"""Host logic of data-parallel training on CPU: the row-slice rule, the group
id hand-off over a 2-rank gloo world, and argument checks that precede any
NCCL or device work."""

import ctypes as ct
import os
import socket
import tempfile

import numpy as np
import pytest

from modern_fm_b200 import _lib, dp


@pytest.mark.parametrize("n,world", [(0, 1), (1, 2), (7, 3), (4096, 8), (4097, 8), (5, 8)])
def test_slices_partition_the_batch(n, world):
    cuts = [dp.slice_rows(n, world, r) for r in range(world)]
    assert cuts[0][0] == 0 and cuts[-1][1] == n
    for (a, b), (c, d) in zip(cuts, cuts[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in cuts]
    assert max(sizes) - min(sizes) <= 1


def test_slice_rejects_bad_rank():
    with pytest.raises(ValueError):
        dp.slice_rows(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _id_worker(rank, world, port, payload, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = dp.broadcast_unique_id(payload if rank == 0 else None)
        with open(os.path.join(out_dir, f"r{rank}.bin"), "wb") as f:
            f.write(got)
    finally:
        dist.destroy_process_group()


def test_group_id_reaches_every_rank_over_gloo():
    import torch.multiprocessing as mp

    payload = bytes(np.random.default_rng(0).integers(0, 256, 128, dtype=np.uint8))
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_id_worker, args=(2, _free_port(), payload, d), nprocs=2, join=True)
        for r in range(2):
            with open(os.path.join(d, f"r{r}.bin"), "rb") as f:
                assert f.read() == payload


def test_group_arguments_are_checked_before_nccl():
    L = _lib.lib()
    h = ct.c_void_p()
    uid = bytes(128)
    assert L.mfm_dp_create(uid, 2, 2, 0, ct.byref(h)) == _lib.MFM_ERR_INVALID
    assert "rank" in _lib.last_error()
    assert L.mfm_dp_create(uid, 0, 0, 0, ct.byref(h)) == _lib.MFM_ERR_INVALID
    assert h.value is None
    tr = _lib.Train(0, 1, 0.05, 0, 0, 0, 0, 0.9, 0.999, 1e-8, 1, 0, None, 1, 16)
    g = _lib.DevGroup(None, None, None, None, None, None, None)
    rc = L.mfm_fm_fit_device_dp(None, _lib.MFM_DTYPE_F32, None, None, None, 0, 1, None, None,
                                None, tr, 4, g, g, g, None)
    assert rc == _lib.MFM_ERR_INVALID and "group" in _lib.last_error()
    assert L.mfm_dp_destroy(None) == 0


def _peer_worker(rank, world, port, leave, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    if leave and rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        dp.check_peers(timeout_s=3.0)
        res = "ok"
    except RuntimeError as exc:
        res = "error: " + str(exc)
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(res)
    os._exit(0)


@pytest.mark.parametrize("leave", [False, True])
def test_missing_peer_is_found_before_the_next_collective(leave):
    """The bounded barrier before each data-parallel fit passes with every rank
    present and raises (naming the group failure) when rank 1 has left."""
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_peer_worker, args=(2, _free_port(), leave, d), nprocs=2, join=False)
        for _ in range(4):  # join() returns after each process; bounded overall
            if ctx.join(30):
                break
        with open(os.path.join(d, "r0.txt")) as f:
            got = f.read()
    if leave:
        assert got.startswith("error: data-parallel group: a peer is missing"), got
    else:
        assert got == "ok"
