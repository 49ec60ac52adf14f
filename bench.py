"""Benchmark: FM CSR scoring rows/s on B200 (the large CTR-shaped FM config:
39 fields, 2^22 features, k=16), with the HBM roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one scoring pass over one 2,000,000-row test batch per GPU (weak
scaling: every rank scores its own seeded shard; rows are independent so no
collective exists on this path). The arithmetic is the reference's: float64
values, sums and scores on float32 parameters, as its default float32
estimator computes (attributes stored float32, widened to float64 before its
float64 kernels). `value` is device-resident throughput (CSR, parameters and
output already in HBM, CUDA events on the launch stream, max over ranks);
`e2e` is the same metric through the C ABI with pinned HOST buffers in the
boundary format (int64 indices, float64 values): the model handle
(mfm_model_predict_csr, parameters resident) as the headline and the
reference-shaped stateless call (mfm_fm_predict_csr, parameters uploaded every
call) beside it — host->device copies, validation and the device->host read of
the scores all inside the timed region. `f32` is the float32-arithmetic figure.
`--impl reference` times the reference's CPU engine (its C restatement, rows
split over every host core) on the same configuration. The line also carries
`train` (one 10M-row FM AdaGrad epoch in float64, float32 beside it, parity of
a float64 fit against the oracle; `train_dp` across ranks for N > 1) and
`prep` (device CSR canonicalisation of the scoring batch in the boundary
format, canonical and unsorted with duplicates) and, at N = 1, `libffm` (the
native libffm reader on a CTR-shaped file, and loading it onto the GPU).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ROWS = 2_000_000          # test rows per GPU
N_FEATURES = 2 ** 22
K = 16
NNZ_PER_ROW = 39
SEED = 2
# algorithmic bytes per row, float32 parameters with float64 values and
# scores: indptr 8 + nnz*(idx 4 + val 8) + nnz*(k+1)*4 (w and V gathers) + score 8
BYTES_PER_ROW = 8 + NNZ_PER_ROW * 12 + NNZ_PER_ROW * (K + 1) * 4 + 8
# float32 throughout: values 4 B, score 4 B
BYTES_PER_ROW_F32 = 8 + NNZ_PER_ROW * 8 + NNZ_PER_ROW * (K + 1) * 4 + 4
CONFIG = {
    "workload": "FM predict, CTR-shaped: 39 fields (13 numeric + 26 Zipf(1.1) hashed "
                "categorical), 2^22 features, k=16, float32 parameters, float64 values and "
                "arithmetic, 2,000,000 rows per GPU",
    "rows_per_gpu": N_ROWS, "n_features": N_FEATURES, "k": K, "nnz_per_row": NNZ_PER_ROW,
    "l2_policy": "inputs larger than L2 (CSR 624 MB + V 268 MB per GPU; L2 126 MB)",
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic():
    """DRAM bytes per launch of the scoring kernel from the committed ncu
    summary (profiles/fm_predict_ctr39.json), scaled to N_ROWS."""
    p = os.path.join(ROOT, "profiles", "fm_predict_ctr39.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_row"]) * N_ROWS
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        if self.idx < 0:  # sampling off
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "50"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def cpu_baseline(X, w0, w, V, n_sample, threads):
    """The reference's CPU scoring (its C restatement, rows split over
    `threads` host threads) on the first n_sample rows of the same input."""
    from oracle import oracle as O

    sub = X.rows(0, n_sample)
    warm = X.rows(0, min(1000, n_sample))
    O.fm_predict_fast_csr(warm.indptr, warm.indices, warm.data, N_FEATURES, w0, w, V,
                          n_threads=threads)
    t = time.perf_counter()
    out = O.fm_predict_fast_csr(sub.indptr, sub.indices, sub.data, N_FEATURES, w0, w, V,
                                n_threads=threads)
    dt = time.perf_counter() - t
    return n_sample / dt, out


def host_inputs(dev):
    """Boundary-format host copies (pinned) of the device workload."""
    import torch

    from modern_fm_b200.workloads import Csr

    ip = dev["indptr"].cpu().pin_memory()
    ix = dev["indices"].to(torch.int64).cpu().pin_memory()
    dv = dev["data"].to(torch.float64).cpu().pin_memory()
    return Csr(ip.numpy(), ix.numpy(), dv.numpy(), dev["n_features"]), (ip, ix, dv)


def make_params(local, dev_t):
    import torch

    g = torch.Generator(device=dev_t)
    g.manual_seed(1234)
    w = torch.randn(N_FEATURES, generator=g, device=dev_t, dtype=torch.float64) * 0.1
    V = torch.randn(N_FEATURES, K, generator=g, device=dev_t, dtype=torch.float64) * 0.1
    return -3.0, w, V


TRAIN_ROWS = 10_000_000
TRAIN_BATCH = 4096


def train_inputs(n, seed, dev_t, L, _lib):
    """The training workload on the device: CTR-shaped CSR (float64 values),
    labels drawn from a planted FM with N(0, 0.1) parameters at ~3 %
    positives, unit sample weights, one shuffled row order, and the initial
    latent factors N(0, 0.01) (float64)."""
    import torch

    from modern_fm_b200 import workloads as WL

    X = WL.ctr_fm_torch(n, seed, device=dev_t, value_dtype=torch.float64)
    g = torch.Generator(device=dev_t)
    g.manual_seed(seed + 4219)
    wp = (torch.randn(N_FEATURES, generator=g, device=dev_t) * 0.1).contiguous()
    Vp = (torch.randn(N_FEATURES, K, generator=g, device=dev_t) * 0.1).contiguous()
    sc = torch.empty(n, dtype=torch.float64, device=dev_t)
    stream = torch.cuda.current_stream(dev_t)
    rc = L.mfm_fm_predict_device(_lib.MFM_DTYPE_F32_F64, dev_t.index, X["indptr"].data_ptr(),
                                 X["indices"].data_ptr(), X["data"].data_ptr(), n, 0.0,
                                 wp.data_ptr(), Vp.data_ptr(), K, sc.data_ptr(), stream.cuda_stream)
    if rc:
        raise RuntimeError(_lib.last_error())
    lo, hi = -50.0, 50.0
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if float(torch.sigmoid(sc + mid).mean()) > 0.03:
            hi = mid
        else:
            lo = mid
    y = (torch.rand(n, generator=g, device=dev_t, dtype=torch.float64)
         < torch.sigmoid(sc + 0.5 * (lo + hi))).double()
    sw = torch.ones(n, device=dev_t, dtype=torch.float64)
    order = torch.randperm(n, generator=g, device=dev_t).to(torch.int32).contiguous()
    V0 = (torch.randn(N_FEATURES, K, generator=g, device=dev_t, dtype=torch.float64)
          * 0.01).contiguous()
    return X, y, sw, order, V0


def _tr_adagrad(_lib, row_orders=None, n_epochs=1):
    return _lib.Train(_lib.LOSSES["logistic"], _lib.OPTIMIZERS["adagrad"], 0.05, 0.0, 1e-5, 0.0,
                      1e-5, 0.9, 0.999, 1e-8, 1.0, 0.0, row_orders, n_epochs, TRAIN_BATCH)


def _device_fit(L, _lib, dtype, local, X, y, sw, order, n, V0, stream):
    """One epoch per call of mfm_fm_fit_device on fresh zero-initialised
    w / state and the given V (all in `dtype`). Returns (epoch, w0, w, V)."""
    import torch

    tdt = torch.float32 if dtype == _lib.MFM_DTYPE_F32 else torch.float64
    data = X["data"].to(tdt)
    yt, swt = y.to(tdt), sw.to(tdt)
    w0 = torch.zeros(1, device=V0.device, dtype=tdt)
    w = torch.zeros(N_FEATURES, device=V0.device, dtype=tdt)
    V = V0.to(tdt).clone()
    acc0, accw, accV = torch.zeros_like(w0), torch.zeros_like(w), torch.zeros_like(V)
    tr = _tr_adagrad(_lib)
    grp = [_lib.DevGroup(p.data_ptr(), a.data_ptr(), None, None, None, None, None)
           for p, a in ((w0, acc0), (w, accw), (V, accV))]

    def epoch():
        rc = L.mfm_fm_fit_device(dtype, local, X["indptr"].data_ptr(), X["indices"].data_ptr(),
                                 data.data_ptr(), n, N_FEATURES, yt.data_ptr(), swt.data_ptr(),
                                 order.data_ptr(), tr, K, grp[0], grp[1], grp[2],
                                 stream.cuda_stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    return epoch, w0, w, V, (data, yt, swt, acc0, accw, accV, tr, grp)


def train_measure(args, rank, world, local, dev_t, L, _lib):
    """FM AdaGrad training on the large CTR config: 10M rows, batch 4096,
    k=16, one epoch per step, in float64 (the reference's training
    arithmetic: float64 parameters and state for the whole fit,
    python/modern_fm/_backend.py:116-130), with float32 as a secondary figure.
    Returns the `train` object of the JSON line (rank 0) or None."""
    import torch

    n = args.train_rows
    X, y, sw, order, V0 = train_inputs(n, SEED + 100 + rank, dev_t, L, _lib)
    stream = torch.cuda.current_stream(dev_t)
    # algorithmic bytes of one epoch (s = bytes per parameter / value): per row
    # indptr 8, per entry index 4 + value s + (w, V) gathers (k+1) s, label and
    # sample weight 2 s; per (batch, touched feature) parameter and AdaGrad
    # state read and written: 4 (k+1) s
    rows_of = torch.repeat_interleave(
        torch.arange(n, device=dev_t), X["indptr"][1:] - X["indptr"][:-1])
    pos_of = torch.empty(n, dtype=torch.int64, device=dev_t)
    pos_of[order.long()] = torch.arange(n, device=dev_t)
    keys = (pos_of[rows_of] // TRAIN_BATCH) * N_FEATURES + X["indices"].long()
    touched = int(torch.unique(keys).numel())
    del rows_of, pos_of, keys
    nnz = int(X["indices"].numel())

    def bytes_epoch(sz):
        return n * 8 + nnz * (4 + sz + (K + 1) * sz) + n * 2 * sz + touched * (K + 1) * sz * 4

    def run(dtype, steps):
        epoch, w0, w, V, keep = _device_fit(L, _lib, dtype, local, X, y, sw, order, n, V0,
                                            stream)
        epoch()  # warm-up: allocator and module load
        torch.cuda.synchronize()
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            epoch()
        t1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
        if not np.isfinite(float(V.abs().max())):
            raise RuntimeError("training diverged")
        return ms

    ms = run(_lib.MFM_DTYPE_F64, args.train_steps)
    ms32 = run(_lib.MFM_DTYPE_F32, args.train_steps)
    peak, _ = peaks()
    b64, b32 = bytes_epoch(8), bytes_epoch(4)
    out = {
        "metric": "FM AdaGrad training rows/s (CTR-shaped 39 fields, 2^22 features, k=16, "
                  "batch 4096, 1 epoch per step)",
        "value": world * n / (ms / 1e3), "unit": "rows/s", "rows_per_gpu": n, "dtype": "f64",
        "steps": args.train_steps, "ms_per_step": ms, "scaling": "weak (independent fits)",
        "roofline": {"bound": "hbm", "achieved": b64 / (ms / 1e3) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": b64 / (ms / 1e3) / 1e9 / peak,
                     "bytes_per_epoch": b64, "touched_per_epoch": touched},
        "f32": {"value": world * n / (ms32 / 1e3), "unit": "rows/s", "ms_per_step": ms32,
                "dtype": "f32", "roofline": {"achieved": b32 / (ms32 / 1e3) / 1e9,
                                             "frac": b32 / (ms32 / 1e3) / 1e9 / peak,
                                             "bytes_per_epoch": b32}},
    }
    if args.train_e2e_rows <= 0:
        return out if rank == 0 else None

    # e2e: the reference-facing fit entry point with pinned host buffers in
    # the boundary format (int64 indices, float64 values / parameters / state)
    n_e = min(n, args.train_e2e_rows)
    ip = X["indptr"][: n_e + 1].cpu().pin_memory()
    ix = X["indices"][: int(ip[-1])].to(torch.int64).cpu().pin_memory()
    dv = X["data"][: int(ip[-1])].cpu().pin_memory()
    yh = y[:n_e].cpu().pin_memory()
    swh = torch.ones(n_e, dtype=torch.float64).pin_memory()
    roh = torch.arange(n_e, dtype=torch.int64).reshape(1, -1).pin_memory()
    wh = torch.zeros(N_FEATURES, dtype=torch.float64).pin_memory()
    Vh = V0.cpu().pin_memory()
    awh, aVh = torch.zeros_like(wh).pin_memory(), torch.zeros_like(Vh).pin_memory()
    csr, keep = _lib.make_csr(ip.numpy(), ix.numpy(), dv.numpy(), N_FEATURES)
    tr_h = _tr_adagrad(_lib, _lib.ptr(roh.numpy(), _lib.i64p), 1)
    w0a, a0a = np.zeros(1), np.zeros(1)
    gh = [_lib.Group(_lib.ptr(p), _lib.ptr(a), None, None, None, None, None)
          for p, a in ((w0a, a0a), (wh.numpy(), awh.numpy()), (Vh.numpy(), aVh.numpy()))]
    ex = _lib.Exec(_lib.MFM_DTYPE_F64, local, 1)

    def e2e_fit():
        rc = L.mfm_fm_fit_csr(csr, _lib.ptr(yh.numpy()), _lib.ptr(swh.numpy()), tr_h, K, gh[0],
                              gh[1], gh[2], ex)
        if rc:
            raise RuntimeError(_lib.last_error())

    e2e_fit()
    barrier(world)
    t = time.perf_counter()
    e2e_fit()
    e2e_s = max_over_ranks(time.perf_counter() - t, world)
    h2d = sum(a.numpy().nbytes for a in (ip, ix, dv, yh, swh, roh, wh, Vh, awh, aVh)) + 16
    d2h = sum(a.numpy().nbytes for a in (wh, Vh, awh, aVh)) + 16

    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O

        # the oracle's fit (n_jobs = every host thread) of the first n_c rows,
        # one epoch in row order, and the engine's float64 fit of the same rows
        n_c = args.train_cpu_rows
        ipc = ip.numpy()[: n_c + 1]
        nzc = int(ipc[-1])
        threads = os.cpu_count() or 1
        wc, Vc = np.zeros(N_FEATURES), V0.cpu().numpy().copy()
        awc, aVc = np.zeros(N_FEATURES), np.zeros_like(Vc)
        t = time.perf_counter()
        r0 = O.fm_fit_csr(ipc, ix.numpy()[:nzc], dv.numpy()[:nzc], N_FEATURES, yh.numpy()[:n_c],
                          np.ones(n_c), 0.0, 0.0, wc, Vc, awc, aVc, "logistic", "adagrad", 0.05,
                          1e-5, 1e-5, 0.9, 0.999, 1e-8, np.arange(n_c)[None, :], TRAIN_BATCH,
                          threads, 0.0, 0.0, 1.0)
        cpu = {"value": n_c / (time.perf_counter() - t), "unit": "rows/s", "cores": threads,
               "kind": "port", "sample": f"first {n_c} rows, one epoch, n_jobs={threads} "
                                         "(contiguous-chunk split, rust/src/fm.rs:286-311)"}
        Xc = dict(indptr=X["indptr"][: n_c + 1].contiguous(), indices=X["indices"][:nzc],
                  data=X["data"][:nzc])
        oc = torch.arange(n_c, dtype=torch.int32, device=dev_t)
        epoch, w0g, wg, Vg, keep_c = _device_fit(L, _lib, _lib.MFM_DTYPE_F64, local, Xc,
                                                 y[:n_c], sw[:n_c], oc, n_c, V0, stream)
        epoch()
        torch.cuda.synchronize()
        wg, Vg = wg.cpu().numpy(), Vg.cpu().numpy()
        ok_w = np.allclose(wg, wc, rtol=1e-7, atol=1e-9)
        ok_v = np.allclose(Vg, Vc, rtol=1e-7, atol=1e-9)
        ok_w0 = abs(float(w0g.item()) - r0[0]) <= 1e-7 * abs(r0[0]) + 1e-9
        parity = {"ok": bool(ok_w and ok_v and ok_w0), "rows": n_c,
                  "max_abs_dw": float(np.abs(wg - wc).max()),
                  "max_abs_dV": float(np.abs(Vg - Vc).max()),
                  "tolerance": "float64 fit of the first rows against the oracle's fit: "
                               "rtol 1e-7, atol 1e-9 on w0, w and V"}
    if rank != 0:
        return None
    out["e2e"] = {"value": world * n_e / e2e_s, "unit": "rows/s", "rows": n_e, "dtype": "f64",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    if cpu:
        out["cpu_baseline"] = cpu
    if parity:
        out["parity"] = parity
    return out


def train_dp_measure(args, rank, world, local, dev_t, L, _lib):
    """One data-parallel fit across all ranks (N > 1): the same 10M-row epoch
    and global batches of 4096 rows, in float64, parameter-sharded by key
    (each rank owns 1/N of the keys and their optimizer state, scores every
    row over its own keys, and the ranks sum the batch's row table, 4096 x
    (k + 2) values, with one NCCL allreduce per batch; the engine's default).
    Parity: rank 0 also fits the same epochs on its own GPU alone and
    compares."""
    import torch

    from modern_fm_b200 import dp as DP

    n = args.train_rows
    X, y, sw, order, V0 = train_inputs(n, SEED + 100, dev_t, L, _lib)  # same data on every rank
    stream = torch.cuda.current_stream(dev_t)
    dt = _lib.MFM_DTYPE_F64
    w0, w, V = (torch.zeros(1, device=dev_t, dtype=torch.float64),
                torch.zeros(N_FEATURES, device=dev_t, dtype=torch.float64), V0.clone())
    acc0, accw, accV = torch.zeros_like(w0), torch.zeros_like(w), torch.zeros_like(V)
    tr = _tr_adagrad(_lib)
    grp = [_lib.DevGroup(p.data_ptr(), a.data_ptr(), None, None, None, None, None)
           for p, a in ((w0, acc0), (w, accw), (V, accV))]
    group = DP.DataParallelGroup(device=local)
    try:
        def epoch():
            group.fm_fit_device(dt, X["indptr"].data_ptr(), X["indices"].data_ptr(),
                                X["data"].data_ptr(), n, N_FEATURES, y.data_ptr(),
                                sw.data_ptr(), order.data_ptr(), tr, K, grp[0], grp[1], grp[2],
                                stream.cuda_stream)

        epoch()
        torch.cuda.synchronize()
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.train_steps):
            epoch()
        t1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(t0.elapsed_time(t1) / args.train_steps, world)
        batches_ms = max_over_ranks(_lib.fit_phase_seconds()["batches"] * 1e3, world)
    finally:
        group.close()
    parity = None
    if rank == 0:
        one, w0s, ws, Vs, keep = _device_fit(L, _lib, dt, local, X, y, sw, order, n, V0, stream)
        for _ in range(1 + args.train_steps):
            one()
        torch.cuda.synchronize()
        dv_ = float((V - Vs).abs().max())
        ok = bool(torch.allclose(V, Vs, rtol=1e-7, atol=1e-9)
                  and torch.allclose(w, ws, rtol=1e-7, atol=1e-9)
                  and torch.allclose(w0, w0s, rtol=1e-7, atol=1e-9))
        parity = {"ok": ok, "max_abs_dV": dv_,
                  "tolerance": "rank 0's parameters after the data-parallel epochs against a "
                               "one-GPU fit of the same epochs: rtol 1e-7, atol 1e-9 (float64, "
                               "sums in another order)"}
    barrier(world)
    if rank != 0:
        return None
    return {"metric": "FM AdaGrad data-parallel training rows/s (one fit, global batch 4096, "
                      "parameters sharded by key, NCCL allreduce of the row table per batch)",
            "value": n / (ms / 1e3), "unit": "rows/s", "n_gpus": world, "rows": n,
            "dtype": "f64", "steps": args.train_steps, "ms_per_step": ms, "scaling": "strong",
            "batches_ms_per_epoch": batches_ms, "parity": parity}


def softmax_dp_measure(args, rank, world, local, dev_t, L, _lib):
    """C4 (softmax FM C=10, k=8, Adam 1e-3, batch 2048, 3 epochs, sample
    weights, label smoothing 0.1, ragged rows over 1M features) as ONE
    data-parallel fit across all ranks (N > 1; mfm_fit_csr_dp, host float64
    buffers): each global batch of 2048 rows split over the ranks, the batch's
    touched-key gradient sums (C x (k + 1) per key) summed with NCCL, the
    identical step on every rank. Strong scaling of one fit: rows/s = 3 epochs
    x rows / time, max over ranks; the device time of the epochs' batches
    (plans and transfers excluded) beside the wall time. Parity: rank 0 fits
    the same problem on its GPU alone (float64, 1e-7 relative / 1e-9
    absolute)."""
    from modern_fm_b200 import _rust
    from modern_fm_b200 import dp as DP
    from modern_fm_b200 import workloads as WL
    from modern_fm_b200.model import DeviceModel

    n4 = args.softmax_rows

    def gpu_scores(Xg, w0g, wg, Vg):
        with DeviceModel("fm", Xg.n_features, Vg.shape[1], dtype="float64", device=local) as mg:
            mg.set_params(w0g, wg, Vg)
            return mg.predict_csr(Xg.indptr, Xg.indices, Xg.data)
    X, yc, sw = WL.softmax_ctr(n4, 4, score_fn=gpu_scores)
    C, k, d = 10, 8, X.n_features
    V0 = np.random.default_rng(0).normal(0, 0.01, (C, d, k))
    ro = WL.row_orders(n4, 3, 6)

    def fresh():
        w0, w, V = np.zeros(C), np.zeros((C, d)), V0.copy()
        st = [[np.zeros_like(p) for _ in range(3)] for p in (w0, w, V)]
        groups = [_lib.Group(_lib.ptr(p), None, *[_lib.ptr(a) for a in s3], None, None)
                  for p, s3 in zip((w0, w, V), st)]
        return (w0, w, V), st, groups

    def train(rows_order):
        return _lib.Train(0, _lib.OPTIMIZERS["adam"], 1e-3, 0.0, 1e-5, 0.0, 1e-5, 0.9, 0.999,
                          1e-8, 1.0, 0.1, _lib.ptr(rows_order, _lib.i64p), rows_order.shape[0],
                          2048)
    group = DP.DataParallelGroup(device=local)
    try:
        ro1 = np.ascontiguousarray(ro[:1])
        p, st, g = fresh()
        group.fit_csr("fm", (X.indptr, X.indices, X.data), d, yc, sw, g, train(ro1), k,
                      n_classes=C)  # warm-up: one epoch
        p, st, g = fresh()
        barrier(world)
        t = time.perf_counter()
        group.fit_csr("fm", (X.indptr, X.indices, X.data), d, yc, sw, g, train(ro), k,
                      n_classes=C)
        wall = max_over_ranks(time.perf_counter() - t, world)
        ph = _lib.fit_phase_seconds()
        batches = max_over_ranks(ph["batches"], world)
    finally:
        group.close()
    parity = None
    if rank == 0:
        w0s, ws, Vs = np.zeros(C), np.zeros((C, d)), V0.copy()
        t = time.perf_counter()
        _rust.fm_fit_multiclass_csr(X.indptr, X.indices, X.data, d, yc, sw, w0s, ws, Vs, "adam",
                                    1e-3, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, ro, 2048, 0.0, 0.0,
                                    1.0, use_cuda=True)
        one_wall = time.perf_counter() - t
        one_batches = _lib.fit_phase_seconds()["batches"]
        ok = all(np.allclose(a, b, rtol=1e-7, atol=1e-9) for a, b in zip(p, (w0s, ws, Vs)))
        parity = {"ok": bool(ok), "max_abs_dV": float(np.abs(p[2] - Vs).max()),
                  "one_gpu_fit_s": one_wall, "one_gpu_batches_s": one_batches,
                  "tolerance": "rank 0's parameters against a one-GPU fit of the same epochs: "
                               "rtol 1e-7, atol 1e-9 (float64, sums in another order)"}
    barrier(world)
    if rank != 0:
        return None
    return {"metric": "softmax FM (C=10, k=8, Adam) data-parallel training rows/s (one fit, "
                      "global batch 2048 split over the ranks, NCCL allreduce of the batch's "
                      "touched-key sums)",
            "value": 3 * n4 / wall, "unit": "rows/s", "n_gpus": world, "rows": n4,
            "epochs": 3, "dtype": "f64", "fit_s": wall, "batches_s": batches,
            "batches_rows_per_s": 3 * n4 / batches, "scaling": "strong", "parity": parity,
            "path": "mfm_fit_csr_dp (host float64 buffers, transfers included in fit_s)"}


PREP_BYTES_PER_ENTRY = 8 + 8 + 4 + 8  # int64 + float64 read, int32 + float64 written
PREP_BYTES_PER_ROW = 8 + 8            # indptr read and written


def prep_measure(args, local, dev_t, L, _lib, X):
    """Device CSR canonicalisation (mfm_csr_prep_device, the reference's
    `_prep_csr`, python/modern_fm/_backend.py:44-52) on the scoring batch in the
    boundary format (int64 indices, float64 values), twice: as generated
    (already canonical: the one-pass path) and with every row reversed and its
    middle entry's column set to its first entry's (unsorted with one duplicate
    per row: the full path). Timed per call with CUDA events (each call ends
    with a stream synchronisation, inside the timing); parity of the first
    2,000 rows against the oracle."""
    import ctypes as ct

    import torch

    n = X["indptr"].numel() - 1
    ip = X["indptr"]
    ix = X["indices"].long()
    dv = X["data"].double()
    nnz = ix.numel()
    lens = ip[1:] - ip[:-1]
    row = torch.repeat_interleave(torch.arange(n, device=dev_t), lens)
    q = torch.arange(nnz, device=dev_t)
    rev = ip[row] + ip[row + 1] - 1 - q
    ix_raw, dv_raw = ix[rev].clone(), dv[rev].clone()
    mid = ip[:-1] + lens // 2
    has = lens > 2
    ix_raw[mid[has]] = ix_raw[ip[:-1][has]]
    ip_out = torch.empty(n + 1, dtype=torch.int64, device=dev_t)
    ix_out = torch.empty(nnz, dtype=torch.int32, device=dev_t)
    dv_out = torch.empty(nnz, dtype=torch.float64, device=dev_t)
    stream = torch.cuda.current_stream(dev_t)
    res = {}
    for name, (a, b) in (("canonical", (ix, dv)), ("unsorted_dup", (ix_raw, dv_raw))):
        m = ct.c_int64(0)

        def call():
            rc = L.mfm_csr_prep_device(_lib.MFM_DTYPE_F32_F64, local, n, N_FEATURES, nnz,
                                       ip.data_ptr(), a.data_ptr(), b.data_ptr(),
                                       ip_out.data_ptr(), ix_out.data_ptr(), dv_out.data_ptr(),
                                       ct.byref(m), stream.cuda_stream)
            if rc:
                raise RuntimeError(_lib.last_error())

        for _ in range(3):
            call()
        steps = 10
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record(stream)
        for _ in range(steps):
            call()
        ev[1].record(stream)
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / steps
        algo = n * PREP_BYTES_PER_ROW + nnz * (8 + 8) + m.value * (4 + 8)
        from oracle import oracle as O

        rows = 2000
        e = int(ip[rows].item())
        want = O.prep_csr(ip[:rows + 1].cpu().numpy(), a[:e].cpu().numpy(), b[:e].cpu().numpy(),
                          N_FEATURES)
        got_ip = ip_out[:rows + 1].cpu().numpy()
        mm = int(got_ip[-1])
        parity = bool(np.array_equal(got_ip, want[0])
                      and np.array_equal(ix_out[:mm].cpu().numpy().astype(np.int64), want[1])
                      and np.array_equal(dv_out[:mm].cpu().numpy(), want[2]))
        res[name] = {"rows_per_s": n / (ms / 1e3), "ms_per_call": ms, "nnz_in": nnz,
                     "nnz_out": m.value, "achieved_gbs": algo / (ms / 1e3) / 1e9,
                     "algorithmic_bytes": algo, "parity": parity}
    peak, kind = peaks()
    for v in res.values():
        v["frac"] = v["achieved_gbs"] / peak
    res["peak_gbs"], res["peak_kind"] = peak, kind
    res["bytes"] = ("indptr 8 read + 8 written per row; per input entry int64 column + float64 "
                    "value read; per output entry int32 column + float64 value written")
    res["workload"] = ("the 2,000,000-row scoring batch in the boundary format (int64 / "
                       "float64), canonical and with rows reversed plus one duplicate per row")
    return res


def libffm_measure(local, dev_t):
    """The native libffm reader (mfm_libffm_read; the reference's load_libffm,
    python/modern_fm/libffm.py:31-83, is pure Python) on a CTR-shaped file:
    20,000 seeded rows of 39 `field:feature:value` tokens (13 numeric values
    in %g form, 26 one-hot), written ten times over (200,000 rows). Times the
    host read with every host thread and the full load onto the GPU (read,
    upload, device canonicalisation); parity of the raw read against the
    values written (Python's float() of each literal). Any failure is
    reported in the line instead of the figures."""
    import tempfile

    import torch

    from modern_fm_b200.libffm import load_libffm_device, read_libffm_raw

    try:
        rng = np.random.default_rng(SEED)
        n0, z, reps = 20_000, NNZ_PER_ROW, 10
        feat = np.sort(rng.integers(0, N_FEATURES, size=(n0, z)), axis=1)
        fld = feat % z  # one field per feature, as the format requires
        vals = np.where(np.arange(z)[None, :] < 13, np.round(rng.lognormal(0, 2, (n0, z)), 6), 1.0)
        lab = (rng.random(n0) < 0.03).astype(np.int64)
        vtxt = np.char.mod("%g", vals)
        tok = np.char.add(np.char.add(np.char.add(np.char.add(fld.astype(str), ":"),
                                                  feat.astype(str)), ":"), vtxt)
        block = "".join(f"{lab[i]} " + " ".join(tok[i]) + "\n" for i in range(n0))
        d = tempfile.mkdtemp()
        path = os.path.join(d, "ctr.ffm")
        with open(path, "w") as fh:
            fh.write(block * reps)
        size = os.path.getsize(path)
        threads = os.cpu_count() or 1
        host = []
        for _ in range(3):
            t = time.perf_counter()
            ip, ix, dv, y, f, nf = read_libffm_raw(path, threads)
            host.append(time.perf_counter() - t)
        want_v = np.array([float(v) for v in vtxt.ravel()])
        parity = bool(np.array_equal(ix[:n0 * z], feat.ravel())
                      and np.array_equal(dv[:n0 * z].view(np.int64), want_v.view(np.int64))
                      and np.array_equal(y[:n0], lab.astype(np.float64))
                      and len(y) == n0 * reps and np.array_equal(ip[:n0 + 1], np.arange(n0 + 1) * z))
        dev = []
        for _ in range(3):
            torch.cuda.synchronize()
            t = time.perf_counter()
            out = load_libffm_device(path, dtype="float32", n_threads=threads, device=local)
            torch.cuda.synchronize()
            dev.append(time.perf_counter() - t)
            del out
        os.remove(path)
        os.rmdir(d)
        n = n0 * reps
        h, g = statistics.median(host), statistics.median(dev)
        return {"rows": n, "bytes": size, "threads": threads,
                "host_read": {"s": h, "rows_per_s": n / h, "mb_per_s": size / h / 1e6},
                "load_to_device": {"s": g, "rows_per_s": n / g, "mb_per_s": size / g / 1e6},
                "parity": parity,
                "workload": "20,000 seeded CTR-shaped rows (39 tokens: 13 numeric %g values, 26 "
                            "one-hot) written ten times; host read with every host thread; load = "
                            "read + upload + device canonicalisation (float32)"}
    except Exception as exc:  # a failure here must not cost the rest of the line
        return {"error": f"{type(exc).__name__}: {exc}"}


def _device_rate(fn, steps, stream):
    """Mean ms per call of `fn` (CUDA events on the launch stream, 3 warm-up
    calls)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def _roof(bytes_per_row, rows, ms):
    peak, kind = peaks()
    ach = bytes_per_row * rows / (ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "peak_kind": kind, "bytes_per_row": bytes_per_row}


def _check(rc, _lib):
    if rc:
        raise RuntimeError(_lib.last_error())


def configs_measure(args, local, dev_t, L, _lib):
    """The other configurations, at N = 1, in the reference's arithmetic
    (float32 parameters with float64 values and math for scoring, float64
    training). Per configuration: device-resident scoring rows/s over a
    2,000,000-row batch of its generator with the roofline of its algorithmic
    bytes, parity of those scores against the oracle on a row sample (1e-10),
    e2e scoring through the model handle (host CSR in, scores out), one fit
    through the reference-facing C ABI (host float64 buffers, transfers
    included) at the configuration's hyperparameters, and the oracle's fit and
    scoring of a bounded sample on the host cores as cpu_baseline.
      ffm      C1: FFM k=8, 16 one-hot fields x 16, AdaGrad 0.05, batch 512,
               10 epochs over 40,000 rows;
      fwfm     C3: FwFM k=8, 9 Zipf one-hot fields (~373k features), FTRL
               (alpha 0.05, beta 1, l1 1.0 / 0.1), batch 1024, 1 epoch over
               200,000 rows;
      softmax  C4: softmax FM C=10, k=8, ragged Poisson(30)+1 rows over 1M
               features, Adam 1e-3, batch 2048, sample weights, label
               smoothing 0.1, 3 epochs over --softmax-rows rows."""
    import torch

    from modern_fm_b200 import _rust
    from modern_fm_b200 import workloads as WL
    from modern_fm_b200.model import DeviceModel
    from oracle import oracle as O

    os.environ["MFM_B200_DTYPE"] = "float32-float64"
    stream = torch.cuda.current_stream(dev_t)
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    res = {}
    T = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev_t, dt)  # noqa: E731

    def r32(a):
        return np.asarray(a, dtype=np.float32).astype(np.float64)

    def scoring(kind, X, fid, F, k, w0, w, V, R, bytes_per_row, C=1):
        """Device-resident scoring (model handle, float32-float64), parity,
        e2e through the handle."""
        n = X.n_rows
        m = DeviceModel(kind, X.n_features, k, n_fields=F, n_classes=C, device=local)
        m.set_params(w0, w, V, R, fid)
        ip, ix, dv = T(X.indptr, torch.int64), T(X.indices, torch.int32), T(X.data, torch.float64)
        out = torch.empty((n, C) if C > 1 else (n,), dtype=torch.float64, device=dev_t)
        ms = _device_rate(lambda: m.predict_device(ip, ix, dv, out, stream), 10, stream)
        samp = X.rows(0, 2000)
        got = out[:2000].cpu().numpy().reshape(2000, C)
        ok = True
        for c in range(C):
            pc = (lambda a: a[c]) if C > 1 else (lambda a: a)
            if kind == "fm":
                want = O.fm_predict_fast_csr(samp.indptr, samp.indices, samp.data, X.n_features,
                                             pc(w0), pc(w), pc(V))
            elif kind == "ffm":
                want = O.ffm_predict_csr(samp.indptr, samp.indices, samp.data, X.n_features, fid,
                                         pc(w0), pc(w), pc(V))
            else:
                want = O.fwfm_predict_csr(samp.indptr, samp.indices, samp.data, X.n_features,
                                          fid, pc(w0), pc(w), pc(V), pc(R))
            ok &= bool(np.allclose(got[:, c], want, rtol=1e-10, atol=1e-10))
        hbuf = np.empty((n, C) if C > 1 else (n,))
        m.predict_csr(X.indptr, X.indices, X.data, out=hbuf)
        t = time.perf_counter()
        for _ in range(3):
            m.predict_csr(X.indptr, X.indices, X.data, out=hbuf)
        e2e = (time.perf_counter() - t) / 3
        mdt = m.dtype_used
        m.close()
        return {"rows": n, "rows_per_s": n / (ms / 1e3), "ms_per_launch": ms,
                "dtype": "f64", "param_storage": "f32" if mdt == "float32-float64" else "f64",
                "roofline": _roof(bytes_per_row, n, ms), "parity": ok,
                "e2e": {"rows_per_s": n / e2e, "h2d_bytes_per_step": X.indptr.nbytes +
                        X.indices.nbytes + X.data.nbytes, "d2h_bytes_per_step": hbuf.nbytes,
                        "path": "mfm_model_predict_csr"}}

    # ---- C1: FFM ----
    try:
        Xs, ys, fid = WL.onehot_ctr(2_000_000, 7)
        Xall, yall, _ = WL.onehot_ctr(60000, 0)
        Xtr, ytr, Xte = Xall.rows(0, 40000), yall[:40000], Xall.rows(40000, 60000)
        d, F, k = 256, 16, 8
        V0 = rng.uniform(0, 0.1, (d, F, k))
        ro = WL.row_orders(Xtr.n_rows, 10, 1)

        def fit(mod, cuda, epochs, n_jobs=1):
            w, V = np.zeros(d), V0.copy()
            r = mod.ffm_fit_csr(Xtr.indptr, Xtr.indices, Xtr.data, d, ytr, np.ones(Xtr.n_rows),
                                fid, 0.0, 0.0, w, V, np.zeros(d), np.zeros_like(V), "logistic",
                                "adagrad", 0.05, 1e-5, 1e-5, 0.9, 0.999, 1e-8, ro[:epochs], 512,
                                n_jobs, 0.0, 0.0, 1.0, use_cuda=cuda)
            return r[0], w, V
        fit(_rust, True, 10)
        t = time.perf_counter()
        w0, w, V = fit(_rust, True, 10)
        fit_s = time.perf_counter() - t
        t = time.perf_counter()
        fit(O, False, 1, threads)
        cpu_fit = Xtr.n_rows / (time.perf_counter() - t)
        t = time.perf_counter()
        O.ffm_predict_csr(Xte.indptr, Xte.indices, Xte.data, d, fid, w0, w, V, n_threads=threads)
        cpu_pred = Xte.n_rows / (time.perf_counter() - t)
        # predict bytes per row (float32 parameters, float64 values and scores):
        # indptr 8 + z (index 4 + value 8) + z w 4 + z (z-1) pair slots k 4 + score 8
        z = 16
        res["ffm"] = {
            "workload": "C1: FFM k=8, 16 one-hot fields x 16 categories (256 features), "
                        "field = feature // 16",
            "predict": scoring("ffm", Xs, fid, F, k, w0, r32(w), r32(V), None,
                               8 + z * 12 + z * 4 + z * (z - 1) * k * 4 + 8),
            "train": {"fit_s": fit_s, "rows_per_s": Xtr.n_rows * 10 / fit_s, "dtype": "f64",
                      "path": "mfm_ffm_fit_csr (host float64 buffers, transfers included)",
                      "config": "AdaGrad 0.05, batch 512, 10 epochs, 40,000 rows"},
            "cpu_baseline": {"value": cpu_fit, "unit": "train rows/s", "predict_rows_per_s":
                             cpu_pred, "cores": threads, "kind": "port",
                             "sample": "one epoch of the 40,000 training rows (n_jobs = every "
                                       "host thread) and scoring of the 20,000 test rows"}}
    except Exception as exc:
        res["ffm"] = {"error": f"{type(exc).__name__}: {exc}"}

    # ---- C3: FwFM FTRL ----
    try:
        X, y, fid = WL.fwfm_ctr(200000, 3)
        Xs, _, _ = WL.fwfm_ctr(2_000_000, 13, labels=False)
        d, F, k = X.n_features, 9, 8
        V0 = rng.normal(0, 0.01, (d, k))
        ro = WL.row_orders(X.n_rows, 1, 5)

        def fitw(mod, cuda, Xf, yf, rof):
            w, V, R = np.zeros(d), V0.copy(), np.ones((F, F))
            r = mod.fwfm_fit_csr(Xf.indptr, Xf.indices, Xf.data, d, yf, np.ones(Xf.n_rows), fid,
                                 0.0, 0.0, w, V, R, np.zeros(d), np.zeros((d, k)),
                                 np.zeros((F, F)), "logistic", "ftrl", 0.05, 0.0, 0.0, 0.9,
                                 0.999, 1e-8, rof, 1024, 1.0, 0.1, 1.0, use_cuda=cuda)
            return r[0], w, V, R
        fitw(_rust, True, X, y, ro)
        t = time.perf_counter()
        w0, w, V, R = fitw(_rust, True, X, y, ro)
        fit_s = time.perf_counter() - t
        n_c = 40000
        Xc = X.rows(0, n_c)
        t = time.perf_counter()
        fitw(O, False, Xc, y[:n_c], np.arange(n_c)[None, :])
        cpu_fit = n_c / (time.perf_counter() - t)
        t = time.perf_counter()
        O.fwfm_predict_csr(X.indptr, X.indices, X.data, d, fid, w0, w, V, R, n_threads=threads)
        cpu_pred = X.n_rows / (time.perf_counter() - t)
        z = 9  # indptr 8 + z (4 + 8) + z (k + 1) 4 (w, V) + score 8; R read from cache
        res["fwfm"] = {
            "workload": "C3: FwFM k=8, 9 one-hot Zipf(1.05) fields, ~373k features",
            "predict": scoring("fwfm", Xs, fid, F, k, w0, r32(w), r32(V), r32(R),
                               8 + z * 12 + z * (k + 1) * 4 + 8),
            "train": {"fit_s": fit_s, "rows_per_s": X.n_rows / fit_s, "dtype": "f64",
                      "path": "mfm_fwfm_fit_csr (host float64 buffers, transfers included)",
                      "config": "FTRL alpha 0.05, beta 1, l1 1.0 / 0.1, batch 1024, 1 epoch, "
                                "200,000 rows"},
            "cpu_baseline": {"value": cpu_fit, "unit": "train rows/s", "predict_rows_per_s":
                             cpu_pred, "cores": 1, "kind": "port",
                             "sample": f"one epoch of {n_c} rows (the reference's FwFM "
                                       "training is serial, rust/src/fwfm.rs:1-9) and scoring "
                                       "of the 200,000 rows on every host thread"}}
    except Exception as exc:
        res["fwfm"] = {"error": f"{type(exc).__name__}: {exc}"}

    # ---- C4: softmax FM ----
    try:
        n4 = args.softmax_rows

        def gpu_scores(Xg, w0g, wg, Vg):  # the planted per-class FMs, scored on the GPU
            with DeviceModel("fm", Xg.n_features, Vg.shape[1], dtype="float64",
                             device=local) as mg:
                mg.set_params(w0g, wg, Vg)
                return mg.predict_csr(Xg.indptr, Xg.indices, Xg.data)
        X, yc, sw = WL.softmax_ctr(n4, 4, score_fn=gpu_scores)
        C, k, d = 10, 8, X.n_features
        V0 = rng.normal(0, 0.01, (C, d, k))
        ro = WL.row_orders(n4, 3, 6)

        def fitm(mod, cuda, Xf, yf, swf, rof):
            w0, w, V = np.zeros(C), np.zeros((C, d)), V0.copy()
            mod.fm_fit_multiclass_csr(Xf.indptr, Xf.indices, Xf.data, d, yf, swf, w0, w, V,
                                      "adam", 1e-3, 1e-5, 1e-5, 0.1, 0.9, 0.999, 1e-8, rof,
                                      2048, 0.0, 0.0, 1.0, use_cuda=cuda)
            return w0, w, V
        fitm(_rust, True, X, yc, sw, ro)
        t = time.perf_counter()
        w0, w, V = fitm(_rust, True, X, yc, sw, ro)
        fit_s = time.perf_counter() - t
        n_c = 20000
        Xc = X.rows(0, n_c)
        t = time.perf_counter()
        fitm(O, False, Xc, yc[:n_c], sw[:n_c], np.arange(n_c)[None, :])
        cpu_fit = n_c / (time.perf_counter() - t)
        zm = X.nnz / X.n_rows  # mean nonzeros per row
        bpr = 8 + zm * 12 + zm * C * (k + 1) * 4 + C * 8
        res["softmax"] = {
            "workload": f"C4: softmax FM C=10, k=8, ragged Poisson(30)+1 rows (mean "
                        f"{zm:.1f} nonzeros), 1M features, {n4} rows",
            "predict": scoring("fm", X, None, 0, k, w0, r32(w), r32(V), None, bpr, C=C),
            "train": {"fit_s": fit_s, "rows_per_s": n4 * 3 / fit_s, "dtype": "f64",
                      "path": "mfm_fm_fit_multiclass_csr (host float64 buffers, transfers "
                              "included)",
                      "config": "Adam 1e-3, batch 2048, 3 epochs, sample weights U(0.5, 2), "
                                "label smoothing 0.1"},
            "cpu_baseline": {"value": cpu_fit, "unit": "train rows/s", "cores": 1,
                             "kind": "port",
                             "sample": f"one epoch of {n_c} rows (the reference's multiclass "
                                       "training is serial, rust/src/lib.rs:446-448)"}}
    except Exception as exc:
        res["softmax"] = {"error": f"{type(exc).__name__}: {exc}"}
    return res


def run_ours(args):
    import torch

    from modern_fm_b200 import _lib
    from modern_fm_b200 import workloads as WL

    global N_ROWS
    N_ROWS = args.rows
    rank, world, local = dist_setup(args.gpus)
    dev_t = torch.device("cuda", local)
    torch.cuda.set_device(dev_t)
    L = _lib.lib()
    if args.dp_only:  # data-parallel measurements only (N > 1)
        out = {"n_gpus": world,
               "train_dp": train_dp_measure(args, rank, world, local, dev_t, L, _lib),
               "softmax_dp": softmax_dp_measure(args, rank, world, local, dev_t, L, _lib)}
        if rank == 0:
            print(json.dumps(out), flush=True)
        import torch.distributed as dist

        dist.destroy_process_group()
        return
    if args.train_only:
        train = train_measure(args, rank, world, local, dev_t, L, _lib)
        train_dp = train_dp_measure(args, rank, world, local, dev_t, L, _lib) if world > 1 else None
        if train:
            train["n_gpus"] = world
            if train_dp:
                train["train_dp"] = train_dp
            print(json.dumps(train), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    X = WL.ctr_fm_torch(N_ROWS, SEED + rank, device=dev_t, value_dtype=torch.float64)
    X32 = dict(X, data=X["data"].float())
    w0, w64, V64 = make_params(local, dev_t)
    # float32 parameters (a float32 estimator's attributes), float64 values
    w32, V32 = w64.float().contiguous(), V64.float().contiguous()
    out = torch.empty(N_ROWS, dtype=torch.float64, device=dev_t)
    out32 = torch.empty(N_ROWS, dtype=torch.float32, device=dev_t)
    stream = torch.cuda.current_stream(dev_t)

    def step(dtype=_lib.MFM_DTYPE_F32_F64):
        # each compute type with arrays of its own element types: float32 data /
        # parameters / scores; float64 data with float32 parameters; float64
        src, o = (X32, out32) if dtype == _lib.MFM_DTYPE_F32 else (X, out)
        pw, pv = (w64, V64) if dtype == _lib.MFM_DTYPE_F64 else (w32, V32)
        assert pv.element_size() == (8 if dtype == _lib.MFM_DTYPE_F64 else 4)
        assert src["data"].element_size() == (4 if dtype == _lib.MFM_DTYPE_F32 else 8)
        rc = L.mfm_fm_predict_device(dtype, local, src["indptr"].data_ptr(),
                                     src["indices"].data_ptr(), src["data"].data_ptr(), N_ROWS,
                                     w0, pw.data_ptr(), pv.data_ptr(), K, o.data_ptr(),
                                     stream.cuda_stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    def timed(dtype, steps, clocks=False):
        """(total ms, mean launch ms, clock summary) of `steps` device steps."""
        for _ in range(max(3, args.warmup)):
            step(dtype)
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local if clocks else -1) as clk:
            if clocks:
                time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for i in range(steps):
                starts[i].record(stream)
                step(dtype)
                ends[i].record(stream)
            t1.record(stream)
            torch.cuda.synchronize()
        barrier(world)
        total = max_over_ranks(t0.elapsed_time(t1), world)
        launch = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends)),
                                world)
        return total, launch, clk.summary() if clocks else None

    if args.kernel_only:  # profiling runs: one scoring kernel, no other measurement
        kd = _lib.dtype_code(args.kernel_dtype)
        total_ms, launch_ms, _ = timed(kd, args.steps)
        if rank == 0:
            print(json.dumps({"kernel_only": True, "dtype": args.kernel_dtype, "rows": N_ROWS,
                              "launch_ms": launch_ms, "ms_per_step": total_ms / args.steps}),
                  flush=True)
        return
    total_ms, launch_ms, clocks = timed(_lib.MFM_DTYPE_F32_F64, args.steps, clocks=True)
    f32_total, f32_launch, _ = timed(_lib.MFM_DTYPE_F32, max(10, args.steps // 5))

    # e2e through the C ABI with pinned host buffers in the boundary format:
    # the model handle (parameters resident, uploaded once) and the
    # reference-shaped stateless call (parameters uploaded every call)
    from modern_fm_b200.model import DeviceModel

    Xh, keep = host_inputs(X)
    w_h = w32.double().cpu().pin_memory()
    V_h = V32.double().cpu().pin_memory()
    out_h = torch.empty(N_ROWS, dtype=torch.float64).pin_memory()
    out_h2 = torch.empty(N_ROWS, dtype=torch.float64).pin_memory()
    csr, keep2 = _lib.make_csr(Xh.indptr, Xh.indices, Xh.data, N_FEATURES)
    model = DeviceModel("fm", N_FEATURES, K, dtype="float32-float64", device=local)
    model.set_params(w0, w_h.numpy(), V_h.numpy())
    model_dtype = model.dtype_used
    ex = _lib.Exec(_lib.MFM_DTYPE_F32_F64, local, 1)

    def e2e_step():
        rc = L.mfm_model_predict_csr(model._h, csr, _lib.ptr(out_h.numpy()))
        if rc:
            raise RuntimeError(_lib.last_error())

    def e2e_stateless():
        rc = L.mfm_fm_predict_csr(csr, w0, _lib.ptr(w_h.numpy()), _lib.ptr(V_h.numpy()), K,
                                  _lib.ptr(out_h2.numpy()), ex)
        if rc:
            raise RuntimeError(_lib.last_error())

    def wall(fn, steps):
        for _ in range(2):
            fn()
        barrier(world)
        t = time.perf_counter()
        for _ in range(steps):
            fn()
        return max_over_ranks((time.perf_counter() - t) / steps, world)

    e2e_steps = max(2, min(args.steps, 5))
    e2e_s = wall(e2e_step, e2e_steps)
    e2e_sl_s = wall(e2e_stateless, e2e_steps)
    model.close()
    h2d = Xh.indptr.nbytes + Xh.indices.nbytes + Xh.data.nbytes
    h2d_sl = h2d + w_h.numpy().nbytes + V_h.numpy().nbytes

    # parity of the timed kernel's output on a row sample against the oracle
    # (the same float32-valued parameters, float64 arithmetic): 1e-10
    from oracle import oracle as O

    samp = Xh.rows(0, 4000)
    want = O.fm_predict_fast_csr(samp.indptr, samp.indices, samp.data, N_FEATURES, w0,
                                 w_h.numpy(), V_h.numpy(), n_threads=8)
    got = out[:4000].cpu().numpy()
    parity = bool(np.allclose(got, want, rtol=1e-10, atol=1e-10))
    e2e_par = bool(np.allclose(out_h.numpy()[:4000], want, rtol=1e-10, atol=1e-10)
                   and np.allclose(out_h2.numpy()[:4000], want, rtol=1e-10, atol=1e-10))
    got32 = out32[:4000].double().cpu().numpy()
    par32 = bool(np.all(np.abs(got32 - want) <= 1e-5 * np.abs(want) + 1e-5))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        n_s = 300_000
        rate, _ = cpu_baseline(Xh, w0, w_h.numpy(), V_h.numpy(), n_s, threads)
        cpu = {"value": rate, "unit": "rows/s", "cores": threads, "kind": "port",
               "sample": f"first {n_s} rows of the rank-0 test batch, float64 arithmetic, rows "
                         f"split over {threads} host threads (the reference's own CPU predict "
                         "is single-threaded, rust/src/fm.rs:58-70)"}

    prep = None if args.no_prep else prep_measure(args, local, dev_t, L, _lib, X)
    libffm = (libffm_measure(local, dev_t)
              if rank == 0 and world == 1 and not args.no_libffm else None)
    configs = (configs_measure(args, local, dev_t, L, _lib)
               if rank == 0 and world == 1 and not args.no_configs else None)
    train = None if args.no_train else train_measure(args, rank, world, local, dev_t, L, _lib)
    train_dp = (train_dp_measure(args, rank, world, local, dev_t, L, _lib)
                if world > 1 and not args.no_train else None)
    softmax_dp = (softmax_dp_measure(args, rank, world, local, dev_t, L, _lib)
                  if world > 1 and not args.no_train and not args.no_configs else None)

    if rank == 0:
        rows_total = N_ROWS * world
        ms_per_step = total_ms / args.steps
        value = rows_total / (ms_per_step / 1e3)
        peak, peak_kind = peaks()
        achieved = BYTES_PER_ROW * N_ROWS / (launch_ms / 1e3) / 1e9
        traffic = ncu_traffic()
        f32_ms = f32_total / max(10, args.steps // 5)
        a32 = BYTES_PER_ROW_F32 * N_ROWS / (f32_launch / 1e3) / 1e9
        line = {
            "metric": "FM CSR predict rows/s (CTR-shaped 39 fields, 2^22 features, k=16)",
            "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "param_storage": "f32",
            "arithmetic": "float64 values, sums and scores on float32 parameters: the "
                          "reference's computation for its default float32 estimator "
                          "(python/modern_fm/fm.py:655-658, _backend.py:36-41)",
            "data": "synthetic (seeded, generated on the GPU)", "config": CONFIG,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "bytes_per_row": BYTES_PER_ROW},
            "e2e": {"value": rows_total / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": N_ROWS * 8, "parity": e2e_par,
                    "path": "mfm_model_predict_csr (parameters resident in a model handle, "
                            f"{model_dtype}); host CSR int64 / float64 up, float64 scores down",
                    "stateless": {"value": rows_total / e2e_sl_s, "unit": "rows/s",
                                  "h2d_bytes_per_step": h2d_sl,
                                  "path": "mfm_fm_predict_csr (float64 parameters uploaded "
                                          "every call, as the reference's CUDA predict)"}},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "parity": parity,
            "parity_tolerance": "rtol = atol = 1e-10 against the oracle on 4,000 rows",
            "f32": {"value": rows_total / (f32_ms / 1e3), "unit": "rows/s", "ms_per_step": f32_ms,
                    "dtype": "f32", "parity": par32,
                    "roofline": {"achieved": a32, "frac": a32 / peak,
                                 "bytes_per_row": BYTES_PER_ROW_F32},
                    "note": "float32 arithmetic throughout (secondary: narrower than the "
                            "reference's float64)"},
        }
        if cpu:
            line["cpu_baseline"] = cpu
        if prep:
            line["prep"] = prep
        if libffm:
            line["libffm"] = libffm
        if train:
            line["train"] = train
        if configs:
            line.update(configs)
        if train_dp:
            line["train_dp"] = train_dp
        if softmax_dp:
            line["softmax_dp"] = softmax_dp
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU path on the same configuration (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from modern_fm_b200 import workloads as WL

    n_s = 200_000
    X, _ = WL.ctr_fm(n_s, SEED)
    rng = np.random.default_rng(1234)
    w = rng.normal(0, 0.1, N_FEATURES)
    V = rng.normal(0, 0.1, (N_FEATURES, K))
    threads = os.cpu_count() or 1
    from oracle import oracle as O

    for _ in range(max(1, min(args.warmup, 2))):
        O.fm_predict_fast_csr(X.indptr, X.indices, X.data, N_FEATURES, -3.0, w, V,
                              n_threads=threads)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        O.fm_predict_fast_csr(X.indptr, X.indices, X.data, N_FEATURES, -3.0, w, V,
                              n_threads=threads)
        times.append(time.perf_counter() - t)
    ms = statistics.mean(times) * 1e3
    value = n_s / (ms / 1e3)
    line = {
        "impl": "reference",
        "metric": "FM CSR predict rows/s (CTR-shaped 39 fields, 2^22 features, k=16)",
        "value": value, "unit": "rows/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded)", "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{n_s} rows per step (bounded sample of the workload), "
                                   f"rows split over {threads} host threads"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--rows", type=int, default=N_ROWS,
                    help="rows per GPU (smaller cases for profiling runs)")
    ap.add_argument("--no-train", action="store_true", help="skip the training measurement")
    ap.add_argument("--train-only", action="store_true",
                    help="only the training measurement (profiling runs)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-libffm", action="store_true",
                    help="skip the libffm reader measurement")
    ap.add_argument("--dp-only", action="store_true",
                    help="only the data-parallel training measurements (N > 1)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the other configurations (ffm, fwfm, softmax keys)")
    ap.add_argument("--softmax-rows", type=int, default=2_000_000,
                    help="rows of the softmax configuration")
    ap.add_argument("--no-prep", action="store_true",
                    help="skip the device CSR canonicalisation measurement")
    ap.add_argument("--train-rows", type=int, default=TRAIN_ROWS)
    ap.add_argument("--train-steps", type=int, default=2)
    ap.add_argument("--train-e2e-rows", type=int, default=2_000_000)
    ap.add_argument("--train-cpu-rows", type=int, default=200_000)
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the device-resident kernel (profiling runs)")
    ap.add_argument("--kernel-dtype", default="float32-float64",
                    choices=["float32-float64", "float32", "float64"],
                    help="compute type of the --kernel-only scoring kernel")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
