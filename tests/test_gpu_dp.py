"""Data-parallel training on 2 GPUs: binary FM on device arrays
(mfm_fm_fit_device_dp, the row-table path, parameter-sharded by key) and FFM /
FwFM / multiclass softmax FM / binary FM of other widths from host buffers
(mfm_fit_csr_dp, the payload path). Every rank ends bitwise equal to the others, and equal to a one-GPU fit
of the same inputs within the float64 training tolerance (1e-7 relative /
1e-9 absolute: only the summation order differs — per-rank partial sums, then
the cross-rank sum)."""

import os
import socket
import tempfile

import numpy as np
import pytest

from modern_fm_b200 import workloads

pytestmark = pytest.mark.gpu

K, BATCH, EPOCHS = 8, 512, 2


def _data():
    X, _ = workloads.ctr_fm(n_rows=6000, seed=21, space=2**14, vocab=2**11)
    rng = np.random.default_rng(3)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    sw = rng.uniform(0.5, 1.5, X.n_rows)
    V = rng.normal(0, 0.05, (X.n_features, K))
    ro = workloads.row_orders(X.n_rows, EPOCHS, seed=5).astype(np.int32)
    return X, y, sw, V, ro


def _fit(opt, device, group=None, **fit_kw):
    import torch

    from modern_fm_b200 import _lib

    X, y, sw, V0, ro = _data()
    dev = torch.device("cuda", device)
    t = lambda a, dt=torch.float64: torch.as_tensor(np.ascontiguousarray(a), dtype=dt,  # noqa
                                                    device=dev)
    ip, ix, dv = t(X.indptr, torch.int64), t(X.indices, torch.int32), t(X.data)
    yy, ss, rot = t(y), t(sw), t(ro, torch.int32)
    w0, w, V = t([0.0]), t(np.zeros(X.n_features)), t(V0)
    state = [t(np.zeros(1)), t(np.zeros(X.n_features)), t(np.zeros_like(V0))]
    tr = _lib.Train(_lib.LOSSES["logistic"], _lib.OPTIMIZERS[opt], 0.05, 0.0, 1e-5, 0.0, 1e-5,
                    0.9, 0.999, 1e-8, 1.0, 0.0, None, EPOCHS, BATCH)
    g = [_lib.DevGroup(p.data_ptr(), a.data_ptr() if opt == "adagrad" else None, None, None,
                       None, None, None) for p, a in zip((w0, w, V), state)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    args = (_lib.MFM_DTYPE_F64, ip.data_ptr(), ix.data_ptr(), dv.data_ptr(), X.n_rows,
            X.n_features, yy.data_ptr(), ss.data_ptr(), rot.data_ptr(), tr, K, g[0], g[1], g[2],
            stream)
    if group is None:
        rc = _lib.lib().mfm_fm_fit_device(args[0], device, *args[1:])
        assert rc == 0, _lib.last_error()
    else:
        group.fm_fit_device(*args, **fit_kw)
    torch.cuda.synchronize(dev)
    return {n: a.cpu().numpy() for n, a in (("w0", w0), ("w", w), ("V", V),
                                            ("acc_w", state[1]), ("acc_V", state[2]))}


def _worker(rank, world, port, opt, out_dir, mode="shard"):
    import torch
    import torch.distributed as dist

    from modern_fm_b200 import dp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      MFM_B200_DP_MODE="runs" if mode == "runs" else "shard",
                      MFM_B200_DP_EXCHANGE="peer" if mode == "shard_peer" else "nccl")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    group = None
    try:
        group = dp.DataParallelGroup(device=rank)
        res = _fit(opt, rank, group)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), **res)
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["shard", "shard_peer", "runs"])
@pytest.mark.parametrize("opt", ["adagrad", "adam"])
def test_two_gpu_data_parallel_fit(opt, mode):
    """shard: each rank owns half the keys and the ranks sum the row table
    with an NCCL allreduce (shard_peer: the forward kernel reads the other
    rank's rows over NVLink); runs: every rank holds every key and the ranks
    sum the per-key run sums with NCCL."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _free_port(), opt, d, mode), nprocs=2, join=True)
        ranks = [dict(np.load(os.path.join(d, f"r{r}.npz"))) for r in range(2)]
    for key in ranks[0]:
        np.testing.assert_array_equal(ranks[0][key], ranks[1][key], err_msg=key)
    one = _fit(opt, 0)
    keys = ("w0", "w", "V", "acc_w", "acc_V") if opt == "adagrad" else ("w0", "w", "V")
    for key in keys:
        np.testing.assert_allclose(ranks[0][key], one[key], rtol=1e-7, atol=1e-9, err_msg=key)
    assert np.abs(ranks[0]["V"] - _data()[3]).max() > 1e-4  # training moved the factors


@pytest.mark.parametrize("mode", ["shard", "shard_peer", "runs"])
def test_one_rank_group_fit(mode):
    """A group of one rank runs the whole multi-GPU pipeline on one GPU (the
    restricted CSR, the partial forward, the exchange — an NCCL allreduce over
    one rank or the forward's own flag and buffer — the finish step and the
    final gather) and must give the one-GPU fit within the float64 training
    tolerance."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(1, _free_port(), "adagrad", d, mode), nprocs=1, join=True)
        got = dict(np.load(os.path.join(d, "r0.npz")))
    one = _fit("adagrad", 0)
    for key in ("w0", "w", "V", "acc_w", "acc_V"):
        np.testing.assert_allclose(got[key], one[key], rtol=1e-7, atol=1e-9, err_msg=key)
    assert np.abs(got["V"] - _data()[3]).max() > 1e-4


def _lost_peer_worker(rank, world, port, out_dir):
    import time

    import torch
    import torch.distributed as dist

    from modern_fm_b200 import dp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      MFM_B200_DP_TIMEOUT="5")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    group = dp.DataParallelGroup(device=rank)
    if rank == 1:
        os._exit(0)  # leaves between steps: none of its kernels or collectives in flight
    t0 = time.time()
    try:  # no host-side peer check: the engine's own progress timeout must end the fit
        _fit("adagrad", rank, group, check_peers_s=None)
        res = "no error"
    except RuntimeError as exc:
        res = "error: " + str(exc)
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(f"{res} | {time.time() - t0:.1f}")
    group.close()
    os._exit(0)


def test_lost_peer_aborts_the_group_with_an_error():
    """A rank that leaves between steps stops the group's progress; the other
    rank's fit aborts the communicator after MFM_B200_DP_TIMEOUT (5 s) and
    raises instead of waiting forever."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_lost_peer_worker, args=(2, _free_port(), d), nprocs=2, join=False)
        for _ in range(6):
            if ctx.join(30):
                break
        with open(os.path.join(d, "r0.txt")) as f:
            res, secs = f.read().rsplit(" | ", 1)
    assert res.startswith("error: data-parallel group"), res
    assert float(secs) < 120


# ------------------------------------------------ payload path, host buffers --

def _payload_case(name):
    """(model, n_classes, X, y, sw, field_ids, n_fields, params, hp) of a small
    case of each payload-path shape; params are fresh float64 arrays."""
    rng = np.random.default_rng(17)
    if name == "ffm":
        X, y, fid = workloads.onehot_ctr(3000, 4, n_fields=6, n_cats=8)
        d, F, k = X.n_features, 6, 4
        params = [np.zeros(1), np.zeros(d), rng.uniform(0, 0.1, (d, F, k))]
        return "ffm", 1, X, y, np.ones(X.n_rows), fid, F, params, ("adagrad", 0.05, 0.0, 0.0)
    if name == "fwfm":
        X, y, fid = workloads.fwfm_ctr(3000, 8, vocabs=(300, 200, 100, 50))
        d, F, k = X.n_features, 4, 4
        params = [np.zeros(1), np.zeros(d), rng.normal(0, 0.05, (d, k)), np.ones((F, F))]
        return "fwfm", 1, X, y, np.ones(X.n_rows), fid, F, params, ("ftrl", 0.05, 0.01, 0.001)
    if name == "softmax":
        X, yc, sw = workloads.softmax_ctr(3000, 9, n_features=4000, n_classes=4, mean_nnz=12)
        C, d, k = 4, X.n_features, 4
        params = [np.zeros(C), np.zeros((C, d)), rng.normal(0, 0.05, (C, d, k))]
        return "fm", C, X, yc, sw, None, 0, params, ("adam", 0.01, 0.0, 0.0)
    X, _ = workloads.ctr_fm(n_rows=3000, seed=23, space=2**13, vocab=2**10)
    y = (rng.random(X.n_rows) < 0.3).astype(np.float64)
    d, k = X.n_features, 3  # a width outside the row-table path
    params = [np.zeros(1), np.zeros(d), rng.normal(0, 0.05, (d, k))]
    return "fm", 1, X, y, rng.uniform(0.5, 1.5, X.n_rows), None, 0, params, ("adagrad", 0.05, 0, 0)


def _payload_fit(name, group=None):
    """Fit the case through the data-parallel group (group given) or through
    the one-GPU entry points on device 0; returns the parameter arrays."""
    from modern_fm_b200 import _lib

    model, C, X, y, sw, fid, F, params, (opt, lr, l1w, l1v) = _payload_case(name)
    ro = workloads.row_orders(X.n_rows, 2, seed=6)
    groups, keep = [], []
    for p in params:
        acc = np.zeros_like(p) if opt == "adagrad" else None
        if opt == "adam":
            st = [np.zeros_like(p) for _ in range(3)]
            g = _lib.Group(_lib.ptr(p), None, *[_lib.ptr(a) for a in st], None, None)
        elif opt == "ftrl":
            st = [np.zeros_like(p) for _ in range(2)]
            g = _lib.Group(_lib.ptr(p), None, None, None, None, *[_lib.ptr(a) for a in st])
        else:
            st = [acc]
            g = _lib.Group(_lib.ptr(p), _lib.ptr(acc), None, None, None, None, None)
        groups.append(g)
        keep.append(st)
    tr = _lib.Train(_lib.LOSSES["logistic"], _lib.OPTIMIZERS[opt], lr, l1w, 1e-5, l1v, 1e-5,
                    0.9, 0.999, 1e-8, 1.0, 0.1 if C > 1 else 0.0,
                    _lib.ptr(ro, _lib.i64p), ro.shape[0], 256)
    k = params[2].shape[-1]
    if group is not None:
        group.fit_csr(model, (X.indptr, X.indices, X.data), X.n_features, y, sw, groups, tr, k,
                      n_classes=C, field_ids=fid, n_fields=F or None)
    else:
        import ctypes as ct

        L = _lib.lib()
        csr, kp = _lib.make_csr(X.indptr, X.indices, X.data, X.n_features)
        ex = _lib.Exec(_lib.MFM_DTYPE_F64, 0, 1)
        g = [ct.byref(x) for x in groups]
        fidp = _lib.ptr(np.ascontiguousarray(fid, np.int64), _lib.i64p) if fid is not None \
            else None
        if model == "fm" and C > 1:
            rc = L.mfm_fm_fit_multiclass_csr(csr, _lib.ptr(y, _lib.i64p), _lib.ptr(sw), C, tr, k,
                                             *g, ex)
        elif model == "fm":
            rc = L.mfm_fm_fit_csr(csr, _lib.ptr(y), _lib.ptr(sw), tr, k, *g, ex)
        elif model == "ffm":
            rc = L.mfm_ffm_fit_csr(csr, _lib.ptr(y), _lib.ptr(sw), fidp, F, tr, k, *g, ex)
        else:
            rc = L.mfm_fwfm_fit_csr(csr, _lib.ptr(y), _lib.ptr(sw), fidp, F, tr, k, *g, ex)
        assert rc == 0, _lib.last_error()
    return {f"p{i}": p for i, p in enumerate(params)}


def _payload_worker(rank, world, port, name, out_dir):
    import torch
    import torch.distributed as dist

    from modern_fm_b200 import dp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    group = None
    try:
        group = dp.DataParallelGroup(device=rank)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), **_payload_fit(name, group))
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["ffm", "fwfm", "softmax", "fm_k3"])
def test_two_gpu_data_parallel_payload_fit(name):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_payload_worker, args=(2, _free_port(), name, d), nprocs=2, join=True)
        ranks = [dict(np.load(os.path.join(d, f"r{r}.npz"))) for r in range(2)]
    for key in ranks[0]:
        np.testing.assert_array_equal(ranks[0][key], ranks[1][key], err_msg=key)
    one = _payload_fit(name)
    for key in one:
        np.testing.assert_allclose(ranks[0][key], one[key], rtol=1e-7, atol=1e-9, err_msg=key)
