"""The arithmetic of parameter-sharded multi-GPU FM training, on the CPU.

Rank r of N owns the keys with key mod N = r and, for every row of a batch,
forms the row's sums over its own keys only: S_r = sum_j V_j x_j and
u_r = sum_j w_j x_j - 1/2 sum_j |V_j x_j|^2. The engine sums these partial row
tables across the ranks and scores each row as
    s = w0 + sum_r u_r + 1/2 |sum_r S_r|^2,
which is FM's score (rust/src/fm.rs:77-101) with its sums taken in another
order. These tests check that decomposition against the oracle for several
rank counts, and run the exchange itself as an allreduce between two gloo
ranks, as the engine's NCCL exchange does between GPUs.
"""

import os
import socket
import tempfile

import numpy as np
import pytest
import scipy.sparse as sp

from oracle import oracle as O


def _problem(seed, n=300, d=500, k=8, density=0.03):
    rng = np.random.default_rng(seed)
    X = sp.random(n, d, density=density, format="csr", random_state=seed,
                  data_rvs=lambda m: rng.normal(size=m))
    return (X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data,
            float(rng.normal()), rng.normal(size=d) * 0.3, rng.normal(size=(d, k)) * 0.3)


def _partial_table(ip, ix, dv, w, V, world, rank):
    """Rank `rank`'s partial row table: [S_r (k) | u_r] per row."""
    n, k = len(ip) - 1, V.shape[1]
    out = np.zeros((n, k + 1))
    for r in range(n):
        for q in range(ip[r], ip[r + 1]):
            j, x = ix[q], dv[q]
            if j % world != rank:
                continue
            vx = V[j] * x
            out[r, :k] += vx
            out[r, k] += w[j] * x - 0.5 * vx @ vx
    return out


def _scores(table, w0):
    k = table.shape[1] - 1
    S = table[:, :k]
    return w0 + table[:, k] + 0.5 * np.einsum("ij,ij->i", S, S)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partial_row_tables_sum_to_the_fm_score(world):
    ip, ix, dv, w0, w, V = _problem(world)
    total = sum(_partial_table(ip, ix, dv, w, V, world, r) for r in range(world))
    want = O.fm_predict_fast_csr(ip, ix, dv, len(w), w0, w, V)
    np.testing.assert_allclose(_scores(total, w0), want, rtol=1e-12, atol=1e-12)


def _gloo_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ip, ix, dv, w0, w, V = _problem(11)
        t = torch.from_numpy(_partial_table(ip, ix, dv, w, V, world, rank))
        dist.all_reduce(t)  # the batch's exchange: one sum of the row tables
        np.save(os.path.join(out_dir, f"r{rank}.npy"), _scores(t.numpy(), w0))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_table_exchange_between_two_gloo_ranks():
    """Two ranks, each with half the keys, exchange their partial tables with
    one allreduce; both end with the same scores, the oracle's."""
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_gloo_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        got = [np.load(os.path.join(d, f"r{r}.npy")) for r in range(2)]
    np.testing.assert_array_equal(got[0], got[1])
    ip, ix, dv, w0, w, V = _problem(11)
    want = O.fm_predict_fast_csr(ip, ix, dv, len(w), w0, w, V)
    np.testing.assert_allclose(got[0], want, rtol=1e-12, atol=1e-12)
