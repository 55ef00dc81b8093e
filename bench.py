"""Benchmark of the memory-bound layer path on B200.

Workload (the configuration the headline metric is quoted
on): LayerNorm (affine, eps 1e-5) followed by the reference's tanh-GELU,
forward + backward, fp32, x [16384, 4096] ~ N(0,1), weight ~ U(0.5,1.5),
bias ~ N(0,0.1), upstream grad ~ N(0,1).  One step = the fused forward kernel
+ the fused VJP kernel (+ its dweight/dbias finisher); with N GPUs each rank
owns its own 16384 rows (weak scaling, row sharding) and the step ends with
the data-parallel exchange of the [4096] dweight/dbias partials (NCCL
all-reduce).  Inputs are larger than L2 (268 MB per tensor vs 126 MB), so no
flush is needed between steps.

`value` is whole-job algorithmic GB/s: sum over ranks of the bytes each
kernel must move (each input read once, each output written once) divided by
the max over ranks of the device-timed step time.  `e2e` is the same metric
through the C ABI with host buffers: pinned host -> device copies of x and dy
and device -> host copies of y, dx, dweight and dbias inside the timed region.

`--impl reference` times the reference algorithm on the host cores instead:
the oracle port of oxitorch's CPU path (the Rust reference cannot be built on
this image), on a bounded row sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, COLS = 16384, 4096
EPS = 1e-5
F32 = 4
# Algorithmic bytes per row: fwd reads x, writes y (+ mean, rstd);
# VJP reads x, dy (+ mean, rstd), writes dx.  Parameters: w, b read by both,
# dw, db written by the VJP.
FWD_BYTES_ROW = 2 * COLS * F32 + 2 * F32
BWD_BYTES_ROW = 3 * COLS * F32 + 2 * F32
PARAM_BYTES_FWD = 2 * COLS * F32
PARAM_BYTES_BWD = 4 * COLS * F32
METRIC = "HBM GB/s & % of B200 peak, norm/softmax/CE/embed fwd+bwd at 1/2/4/8 GPUs"


def algorithmic_bytes(rows):
    fwd = rows * FWD_BYTES_ROW + PARAM_BYTES_FWD
    bwd = rows * BWD_BYTES_ROW + PARAM_BYTES_BWD
    return fwd, bwd


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---- clocks -------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi sampled every 50 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        self.tmp.seek(0)
        sm, smax, reasons, n = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.tmp.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            n += 1
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.tmp.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": n}


# ---- CPU reference (oracle port) -------------------------------------------------------

def _oracle_step(rows, seed):
    """One fwd+bwd of the composed reference path on `rows` rows; returns seconds."""
    import numpy as np
    from oracle import oxiref as R
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, COLS), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, COLS).astype(np.float32)
    b = (rng.standard_normal(COLS, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    dy = rng.standard_normal((rows, COLS), dtype=np.float32)
    t0 = time.perf_counter()
    xt, wt, bt = R.from_numpy(x, True), R.from_numpy(w, True), R.from_numpy(b, True)
    y = R.gelu(R.layer_norm(xt, wt, bt, EPS))
    y.backward(dy)
    return time.perf_counter() - t0


def cpu_baseline(budget_s=10.0, rows=128):
    """Single-threaded oracle port on repeated `rows`-row samples for ~budget_s."""
    _oracle_step(8, 0)  # build/load the C oracle, warm caches
    total, reps = 0.0, 0
    while total < budget_s or reps < 1:
        total += _oracle_step(rows, 2 + reps)
        reps += 1
    fwd, bwd = algorithmic_bytes(rows)
    gbs = (fwd + bwd) * reps / total / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{reps} x {rows} rows of [16384, 4096] (oracle port, single thread), "
                      f"{total:.1f} s"}


def _pool_worker(args):
    rows, seed = args
    return _oracle_step(rows, seed)


def run_reference(args, rank, world):
    """--impl reference: the oracle port on all host cores, row-sharded across a
    spawn-started process pool; each step is a bounded row sample."""
    if rank != 0:
        return
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    rows_per_worker = 64
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        pool.map(_pool_worker, [(8, 0)] * cores)
        times = []
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            pool.map(_pool_worker, [(rows_per_worker, 1000 * step + i) for i in range(cores)])
            if step >= args.warmup:
                times.append(time.perf_counter() - t0)
    rows = rows_per_worker * cores
    fwd, bwd = algorithmic_bytes(rows)
    per_step = sum(times) / len(times)
    gbs = (fwd + bwd) / per_step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) / U(0.5,1.5) / N(0,0.1) inputs of config 2's distributions)",
        "config": {"workload": "layer_norm+gelu fwd+bwd, fp32, x [16384, 4096] (BASELINE config 2)",
                   "rows_per_step_sample": rows, "cols": COLS},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{rows_per_worker} rows per process x {cores} processes per step "
                                   "(oracle port of the reference CPU path; Rust reference not "
                                   "buildable: no cargo)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- GPU arm -----------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    global ROWS
    ROWS = args.rows
    import torch
    import torch.distributed as dist
    from oxitorch_b200 import _native as N

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L = N.load()
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream

    g = torch.Generator(device=dev)
    g.manual_seed(2 + 1000 * rank)
    x = torch.randn(ROWS, COLS, device=dev, generator=g)
    dy = torch.randn(ROWS, COLS, device=dev, generator=g)
    w = torch.rand(COLS, device=dev, generator=g) + 0.5
    b = torch.randn(COLS, device=dev, generator=g) * 0.1
    y = torch.empty_like(x)
    dx = torch.empty_like(x)
    mean = torch.empty(ROWS, device=dev)
    rstd = torch.empty(ROWS, device=dev)
    dw = torch.empty(COLS, device=dev)
    db = torch.empty(COLS, device=dev)
    ws_bytes = L.oxc_layer_norm_bwd_workspace_size(ROWS, COLS)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    dwdb = torch.empty(2 * COLS, device=dev)

    def fwd(xp, yp):
        N.check(L.oxc_layer_norm_fwd(xp, w.data_ptr(), b.data_ptr(), yp, mean.data_ptr(),
                                     rstd.data_ptr(), ROWS, COLS, EPS, N.ACT_GELU_TANH, s))

    def bwd(xp, dyp, dxp):
        N.check(L.oxc_layer_norm_bwd(xp, w.data_ptr(), b.data_ptr(), mean.data_ptr(),
                                     rstd.data_ptr(), dyp, dxp, dwdb.data_ptr(),
                                     dwdb.data_ptr() + COLS * F32, ROWS, COLS, N.ACT_GELU_TANH,
                                     N.GRAD_REF, ws.data_ptr(), ws_bytes, s))

    def exchange():
        if world > 1:
            dist.all_reduce(dwdb)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        fwd(x.data_ptr(), y.data_ptr())
        if ev is not None:
            ev[1].record(stream)
        bwd(x.data_ptr(), dy.data_ptr(), dx.data_ptr())
        if ev is not None:
            ev[2].record(stream)
        exchange()

    launches_per_step = 4  # fwd, VJP, 2 x column-sum finisher

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(args.steps):
        step(events[i])
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in events)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in events)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps

    fwd_bytes, bwd_bytes = algorithmic_bytes(ROWS)
    value = world * (fwd_bytes + bwd_bytes) / (ms_per_step * 1e-3) / 1e9
    peak, peak_kind = measured_peak()

    # ---- e2e: host buffers through the C ABI --------------------------------------------
    e2e_steps = 0 if args.skip_e2e else max(1, min(args.steps, 5))
    hx = torch.empty(ROWS, COLS, pin_memory=True)
    hdy = torch.empty(ROWS, COLS, pin_memory=True)
    hx.copy_(x)
    hdy.copy_(dy)
    hy = torch.empty(ROWS, COLS, pin_memory=True)
    hdx = torch.empty(ROWS, COLS, pin_memory=True)
    hdwdb = torch.empty(2 * COLS, pin_memory=True)
    xs = torch.empty_like(x)
    dys = torch.empty_like(dy)

    def e2e_step():
        xs.copy_(hx, non_blocking=True)
        dys.copy_(hdy, non_blocking=True)
        fwd(xs.data_ptr(), y.data_ptr())
        bwd(xs.data_ptr(), dys.data_ptr(), dx.data_ptr())
        exchange()
        hy.copy_(y, non_blocking=True)
        hdx.copy_(dx, non_blocking=True)
        hdwdb.copy_(dwdb, non_blocking=True)

    if e2e_steps:
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = (world * (fwd_bytes + bwd_bytes) / (e2e_ms / e2e_steps * 1e-3) / 1e9
                 if e2e_steps else None)
    h2d = 2 * ROWS * COLS * F32
    d2h = 2 * ROWS * COLS * F32 + 2 * COLS * F32

    if rank != 0:
        return
    cpu = cpu_baseline() if (world == 1 and not args.no_cpu_baseline) else None
    achieved = bwd_bytes / (bwd_ms * 1e-3) / 1e9
    traffic = _profiled_traffic()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded torch N(0,1) x/dy, U(0.5,1.5) weight, N(0,0.1) bias; no dataset)",
        "config": {
            "workload": "layer_norm(affine)+gelu(tanh) fwd+bwd, fp32, x [16384, 4096] per GPU "
                        "(BASELINE config 2)",
            "rows_per_gpu": ROWS, "cols": COLS, "eps": EPS,
            "parallelism": f"row-sharded data parallel x{world}, dweight/dbias all-reduce",
            "grad_mode": "ref (reference graph: rsqrt detached)",
            "l2": "no flush: every input (268 MB) is larger than the 126 MB L2",
            "algorithmic_bytes_per_gpu_step": fwd_bytes + bwd_bytes,
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "ln_bwd_kernel (layer_norm+gelu VJP, incl. dweight/dbias finisher)",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs: torch copy read+write)",
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "fwd_kernel_gbs": fwd_bytes / (fwd_ms * 1e-3) / 1e9,
            "fwd_kernel_frac": fwd_bytes / (fwd_ms * 1e-3) / 1e9 / peak,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        },
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / e2e_steps if e2e_steps else None,
                "path": "pinned host -> oxc_layer_norm_fwd/bwd (C ABI) -> pinned host"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def _profiled_traffic():
    """DRAM bytes per launch of the VJP kernel from the committed ncu summary
    (profiles/ln_gelu_bwd_16384x4096.json), or None if absent."""
    path = os.path.join(ROOT, "profiles", "ln_gelu_bwd_16384x4096.json")
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="rows per GPU (default: config 2's 16384; smaller only for profiling)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs: no host-buffer leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
