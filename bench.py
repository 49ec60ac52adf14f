"""Benchmark: FM CSR scoring rows/s on B200 (the large CTR-shaped FM config:
39 fields, 2^22 features, k=16, float32), with the HBM roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one scoring pass over one 2,000,000-row test batch per GPU (weak
scaling: every rank scores its own seeded shard; rows are independent so no
collective exists on this path). `value` is device-resident throughput (CSR,
parameters and output already in HBM, CUDA events on the launch stream, max
over ranks); `e2e` is the same metric through the reference-facing C ABI
(mfm_fm_predict_csr) with pinned HOST buffers in the boundary format (int64
indices, float64 values and parameters) — host->device copies, validation,
conversion and the device->host read of the scores all inside the timed region.
`--impl reference` times the reference's CPU engine (its C restatement, rows
split over every host core) on the same configuration.
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
# algorithmic bytes per row, float32 compute: indptr 8 + nnz*(idx 4 + val 4)
# + nnz*(k+1)*4 (w and V gathers) + score 4
BYTES_PER_ROW = 8 + NNZ_PER_ROW * 8 + NNZ_PER_ROW * (K + 1) * 4 + 4
CONFIG = {
    "workload": "FM predict, CTR-shaped: 39 fields (13 numeric + 26 Zipf(1.1) hashed "
                "categorical), 2^22 features, k=16, float32, 2,000,000 rows per GPU",
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
    X = WL.ctr_fm_torch(N_ROWS, SEED + rank, device=dev_t)
    w0, w64, V64 = make_params(local, dev_t)
    w32, V32 = w64.float().contiguous(), V64.float().contiguous()
    out = torch.empty(N_ROWS, dtype=torch.float32, device=dev_t)
    stream = torch.cuda.current_stream(dev_t)

    def step():
        rc = L.mfm_fm_predict_device(_lib.MFM_DTYPE_F32, local, X["indptr"].data_ptr(),
                                     X["indices"].data_ptr(), X["data"].data_ptr(), N_ROWS, w0,
                                     w32.data_ptr(), V32.data_ptr(), K, out.data_ptr(),
                                     stream.cuda_stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = max_over_ranks(t0.elapsed_time(t1), world)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    launch_ms = max_over_ranks(launch_ms, world)
    clocks = clk.summary()
    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"kernel_only": True, "rows": N_ROWS, "launch_ms": launch_ms,
                              "ms_per_step": total_ms / args.steps}), flush=True)
        return

    # e2e through the C ABI with pinned host buffers in the boundary format
    Xh, keep = host_inputs(X)
    w_h = w64.cpu().pin_memory()
    V_h = V64.cpu().pin_memory()
    out_h = torch.empty(N_ROWS, dtype=torch.float64).pin_memory()
    csr, keep2 = _lib.make_csr(Xh.indptr, Xh.indices, Xh.data, N_FEATURES)
    ex = _lib.Exec(_lib.MFM_DTYPE_F32, local, 1)

    def e2e_step():
        rc = L.mfm_fm_predict_csr(csr, w0, _lib.ptr(w_h.numpy()), _lib.ptr(V_h.numpy()), K,
                                  _lib.ptr(out_h.numpy()), ex)
        if rc:
            raise RuntimeError(_lib.last_error())

    for _ in range(2):
        e2e_step()
    e2e_steps = max(2, min(args.steps, 5))
    barrier(world)
    t = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks((time.perf_counter() - t) / e2e_steps, world)
    h2d = (Xh.indptr.nbytes + Xh.indices.nbytes + Xh.data.nbytes + w_h.numpy().nbytes
           + V_h.numpy().nbytes)

    # parity of the timed kernel's output on a row sample against the oracle
    from oracle import oracle as O

    samp = Xh.rows(0, 4000)
    want = O.fm_predict_fast_csr(samp.indptr, samp.indices, samp.data, N_FEATURES, w0,
                                 w_h.numpy(), V_h.numpy(), n_threads=8)
    got = out[:4000].double().cpu().numpy()
    parity = bool(np.all(np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-5))
    e2e_par = bool(np.allclose(out_h.numpy()[:4000], want, rtol=1e-5, atol=1e-5))

    cpu = None
    if rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        n_s = 300_000
        rate, _ = cpu_baseline(Xh, w0, w_h.numpy(), V_h.numpy(), n_s, threads)
        cpu = {"value": rate, "unit": "rows/s", "cores": threads, "kind": "port",
               "sample": f"first {n_s} rows of the rank-0 test batch, rows split over "
                         f"{threads} host threads (the reference's own CPU predict is "
                         "single-threaded, rust/src/fm.rs:58-70)"}

    if rank == 0:
        rows_total = N_ROWS * world
        ms_per_step = total_ms / args.steps
        value = rows_total / (ms_per_step / 1e3)
        peak, peak_kind = peaks()
        achieved = BYTES_PER_ROW * N_ROWS / (launch_ms / 1e3) / 1e9
        traffic = ncu_traffic()
        line = {
            "metric": "FM CSR predict rows/s (CTR-shaped 39 fields, 2^22 features, k=16)",
            "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, generated on the GPU)", "config": CONFIG,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "bytes_per_row": BYTES_PER_ROW},
            "e2e": {"value": rows_total / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": N_ROWS * 8, "parity": e2e_par},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "parity": parity,
        }
        if cpu:
            line["cpu_baseline"] = cpu
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
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the device-resident kernel (profiling runs)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
