"""Benchmark of the memory-bound layer path on B200.

Default run: the headline workload (LayerNorm (affine,
eps 1e-5) followed by the reference's tanh-GELU, forward + backward, fp32,
x [16384, 4096]) timed for exactly --steps steps, then every other BASELINE
config timed the same way and reported under `per_workload`:

  rms        config 1: RMSNorm fwd+VJP, x [4096, 4096] (fits L2: 3 rotating input sets)
  ce         config 3: cross-entropy fwd+VJP, logits [32768, 32000]
  embedding  config 4: gather + duplicate-id VJP, table [32000, 4096],
             ids [64, 2048] Zipf(1.1) clipped
  mlp_block  config 5: RMSNorm + SwiGLU (transposed gate view) + dim-1
             sum/max/argmax + whole-tensor L2 of {dx, dg, du}, 65536 tokens

`--workload` runs one of them (or `registry`: config 5 through the generic
elementwise registry; `optim`: the optimizer step; `loader`: the device data
path) as the headline instead.

Inputs are the seeded numpy arrays of each config (`config_inputs`: numpy
Generator(PCG64(k)) for config k, drawn in a fixed order), generated once on
the host of rank 0, uploaded outside the timed region and broadcast to the
other ranks.  The parity tests draw the same arrays from the same function,
so the benchmarked inputs are the tested inputs.

`value` is whole-job algorithmic GB/s: sum over ranks of the bytes each kernel
must move (each input read once, each output written once) divided by the max
over ranks of the device-timed duration of the K steps.  With N GPUs every
rank owns a full config (weak scaling); `strong_scaling` also times the global
config split N ways against the same config on one GPU.  The data-parallel
exchange of a step (an all-reduce of weight-gradient partials) runs on NCCL's
stream and overlaps the next step's forward; the timed region ends after the
last exchange.  `e2e` is the same metric through the C ABI with host buffers:
pinned host -> device copies of the step's inputs and device -> host copies of
its outputs inside the timed region.

`--impl reference` times the reference algorithm on the host cores instead:
the oracle port of oxitorch's CPU path (the Rust reference cannot be built on
this image), on bounded row slices of the same workloads.
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

F32 = 4
METRIC = "HBM GB/s & % of B200 peak, norm/softmax/CE/embed fwd+bwd at 1/2/4/8 GPUs"
PER_WORKLOAD = ("rms", "ce", "embedding", "mlp_block")


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def log(*a):
    print("[bench]", *a, file=sys.stderr, flush=True)


# ---- seeded inputs of the BASELINE configs ----------------------------------------------

def config_spec(k, rows=0):
    """(name, shape, dtype) of config k's inputs, in drawing order.  `rows`
    (profiling only) replaces the row (token, id) count."""
    f, i = "float32", "int64"
    if k == 1:
        m = rows or 4096
        return [("x", (m, 4096), f), ("w", (4096,), f), ("dy", (m, 4096), f)]
    if k == 2:
        m = rows or 16384
        return [("x", (m, 4096), f), ("w", (4096,), f), ("b", (4096,), f), ("dy", (m, 4096), f)]
    if k == 3:
        m = rows or 32768
        return [("logits", (m, 32000), f), ("targets", (m,), i)]
    if k == 4:
        n = rows or 64 * 2048
        return [("table", (32000, 4096), f), ("ids", (n,), i), ("dout", (n, 4096), f)]
    if k == 5:
        m = rows or 65536
        return [("x", (m, 4096), f), ("w", (1, 4096), f), ("gate_buf", (11008, m), f),
                ("up", (m, 11008), f), ("dy", (m, 4096), f), ("dh", (m, 11008), f)]
    raise ValueError(k)


def config_inputs(k, rows=0):
    """The inputs of BASELINE config k as numpy arrays: Generator(PCG64(k)),
    arrays drawn in config_spec order.  N(0,1) arrays are float32 draws;
    weights are U(0.5, 1.5) float64 draws cast to float32; the LayerNorm bias
    is an N(0,1) float32 draw times 0.1; logits are N(0,1) float32 draws times
    2 with `rng.random(shape) < 0.01` (float64 draws, taken in row blocks,
    which is the same stream) set to +20, then targets `rng.integers(0,
    32000, rows)`; embedding ids are min(zipf(1.1, (64, 2048)) - 1, 31999)
    (with `rows`, zipf(1.1, rows))."""
    import numpy as np
    rng = np.random.default_rng(k)
    out = {}

    def normal(shape):
        a = np.empty(shape, np.float32)
        rng.standard_normal(out=a, dtype=np.float32)
        return a

    for name, shape, _ in config_spec(k, rows):
        if name in ("w",):
            out[name] = rng.uniform(0.5, 1.5, shape).astype(np.float32)
        elif name == "b":
            out[name] = (rng.standard_normal(shape, dtype=np.float32)
                         * np.float32(0.1)).astype(np.float32)
        elif name == "logits":
            x = normal(shape)
            x *= np.float32(2.0)
            step = 256
            for r in range(0, shape[0], step):
                blk = x[r:r + step]
                blk[rng.random(blk.shape) < 0.01] = np.float32(20.0)
            out[name] = x
        elif name == "targets":
            out[name] = rng.integers(0, 32000, shape[0]).astype(np.int64)
        elif name == "ids":
            zshape = (64, 2048) if shape[0] == 64 * 2048 and not rows else shape
            out[name] = np.minimum(rng.zipf(1.1, zshape) - 1, 31999).astype(np.int64).reshape(-1)
        else:
            out[name] = normal(shape)
    return out


def device_inputs(k, dev, rank, world, rows=0):
    """config_inputs(k) on this rank's device: rank 0 draws them on its host
    and uploads them, the other ranks receive them by broadcast."""
    import torch
    spec = config_spec(k, rows)
    t0 = time.perf_counter()
    if rank == 0:
        host = config_inputs(k, rows)
        t1 = time.perf_counter()
        out = {n: torch.from_numpy(host[n]).to(dev) for n, _, _ in spec}
        del host
        log(f"config {k} inputs: drawn in {t1 - t0:.1f} s, uploaded in "
            f"{time.perf_counter() - t1:.1f} s")
    else:
        out = {n: torch.empty(s, dtype=getattr(torch, d), device=dev) for n, s, d in spec}
    if world > 1:
        import torch.distributed as dist
        for n, _, _ in spec:
            dist.broadcast(out[n], 0)
    return out


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


# ---- CPU reference samples (oracle port) ------------------------------------------------

# rows (tokens, ids, samples) per CPU sample of each workload
SAMPLE_ROWS = {"ln_gelu": 1024, "rms": 1024, "embedding": 1024, "ce": 64, "mlp_block": 64,
               "registry": 64, "optim": 1 << 20, "loader": 512}


def cpu_sample(workload, seed):
    """One bounded sample of `workload` through the oracle port of the
    reference CPU path: SAMPLE_ROWS[workload] rows of the config's shapes and
    distributions.  Returns (seconds, algorithmic bytes of the sample)."""
    import numpy as np
    from oracle import oxiref as R
    rng = np.random.default_rng(seed)
    rows = SAMPLE_ROWS[workload]
    if workload in ("ln_gelu", "rms"):
        cols = 4096
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        b = (rng.standard_normal(cols, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        dy = rng.standard_normal((rows, cols), dtype=np.float32)
        t0 = time.perf_counter()
        xt, wt = R.from_numpy(x, True), R.from_numpy(w, True)
        if workload == "rms":
            y = R.rms_norm(xt, wt, 1e-6)
            nbytes = rows * (20 * cols + 8) + 12 * cols
        else:
            y = R.gelu(R.layer_norm(xt, wt, R.from_numpy(b, True), 1e-5))
            nbytes = rows * (20 * cols + 16) + 24 * cols
        y.backward(dy)
        return time.perf_counter() - t0, nbytes
    if workload == "ce":
        cols = 32000
        x = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(2)).astype(np.float32)
        x[rng.random((rows, cols)) < 0.01] = 20.0
        t = [int(v) for v in rng.integers(0, cols, rows)]
        t0 = time.perf_counter()
        xt = R.from_numpy(x, True)
        R.cross_entropy(xt, t).backward()
        return time.perf_counter() - t0, rows * cols * 12 + rows * 36
    if workload == "embedding":
        v, d, n = 32000, 4096, rows
        table = rng.standard_normal((v, d), dtype=np.float32)
        ids = np.minimum(rng.zipf(1.1, n) - 1, v - 1).astype(np.int64)
        dout = rng.standard_normal((n, d), dtype=np.float32)
        t0 = time.perf_counter()
        tt = R.from_numpy(table, True)
        out = R.embedding([int(i) for i in ids], tt)
        out.backward(dout)
        return time.perf_counter() - t0, n * 8 * 2 + n * d * 4 * 3 + v * d * 4
    if workload == "mlp_block":
        m, dmod, hid = rows, 4096, 11008
        x = rng.standard_normal((m, dmod), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, dmod).astype(np.float32)
        g = rng.standard_normal((m, hid), dtype=np.float32)
        u = rng.standard_normal((m, hid), dtype=np.float32)
        dy = rng.standard_normal((m, dmod), dtype=np.float32)
        dh = rng.standard_normal((m, hid), dtype=np.float32)
        t0 = time.perf_counter()
        xt, wt = R.from_numpy(x, True), R.from_numpy(w, True)
        R.rms_norm(xt, wt, 1e-6).backward(dy)
        gt, ut = R.from_numpy(g, True), R.from_numpy(u, True)
        h = R.silu(gt) * ut
        hv = h.numpy()
        R.t_reduce("sum", hv, 1, False), R.t_reduce("max", hv, 1, False), R.t_reduce("argmax", hv, 1, False)
        h.backward(dh)
        for grad in (xt.grad.numpy(), gt.grad.numpy(), ut.grad.numpy()):
            R.sumsq_all_f64(grad)
        return time.perf_counter() - t0, m * (20 * dmod + 32 * hid) + 12 * dmod
    if workload == "optim":
        n = rows
        p = rng.standard_normal(n, dtype=np.float32)
        g = rng.standard_normal(n, dtype=np.float32)
        t0 = time.perf_counter()
        R.adamw_step(p, g, None, None, 1e-3, 0.9, 0.999, 1e-8, 0.01, True, 1)
        R.sgd_step(p, g, None, 1e-2, 0.9, True)
        return time.perf_counter() - t0, 48 * n
    if workload == "loader":
        nrows, bs = 4096, rows
        images = rng.standard_normal((nrows, 3, 32, 32), dtype=np.float32)
        labels = rng.integers(0, 10, nrows).astype(np.float32)
        t0 = time.perf_counter()
        idx = [int(v) for v in rng.permutation(nrows)[:bs]]
        R.gather_columns([images, labels], idx)
        img, _ = R.gather_columns([images, labels], idx)
        R.apply_transforms(img, LOADER_STEPS, R.batch_rng(R.batch_seed(1, R.indices_seed(idx))))
        return time.perf_counter() - t0, bs * (LOADER_PLAIN_BYTES + LOADER_AUG_BYTES)
    if workload == "registry":
        m, hid = rows, 11008
        g = rng.standard_normal((m, hid), dtype=np.float32)
        u = rng.standard_normal((m, hid), dtype=np.float32)
        dh = rng.standard_normal((m, hid), dtype=np.float32)
        t0 = time.perf_counter()
        gt, ut = R.from_numpy(g, True), R.from_numpy(u, True)
        h = R.silu(gt) * ut
        hv = h.numpy()
        R.t_reduce("sum", hv, 1, False), R.t_reduce("max", hv, 1, False), R.t_reduce("argmax", hv, 1, False)
        h.backward(dh)
        return time.perf_counter() - t0, m * hid * (44 + 92) + 12 * m
    raise ValueError(workload)


def cpu_baseline(workload, budget_s=10.0):
    """Single-threaded oracle port on repeated samples for ~budget_s."""
    cpu_sample(workload, 0)  # build/load the C oracle, warm caches
    total, nbytes, reps = 0.0, 0, 0
    while total < budget_s or reps < 1:
        dt, b = cpu_sample(workload, 1 + reps)
        total += dt
        nbytes += b
        reps += 1
    return {"value": nbytes / total / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{reps} samples of {SAMPLE_ROWS[workload]} rows of the {workload} "
                      f"workload (oracle port of the reference CPU path, one thread), "
                      f"{total:.1f} s"}


def _pool_worker(args):
    return cpu_sample(*args)


def _reference_steps(pool, cores, workload, steps, warmup):
    """Seconds per step (one bounded sample per process, the step ends when the
    slowest process finishes) and bytes per step."""
    pool.map(_pool_worker, [(workload, 0)] * cores)
    times, nbytes = [], 0
    for step in range(warmup + steps):
        res = pool.map(_pool_worker, [(workload, 1000 * step + i) for i in range(cores)])
        if step >= warmup:
            # input generation and process-pool IPC are not counted
            times.append(max(dt for dt, _ in res))
            nbytes = sum(b for _, b in res)
    return sum(times) / len(times), nbytes


def _reference_config(workload, cores):
    return {"workload": WORKLOADS[workload].DESC, "rows_per_sample": SAMPLE_ROWS[workload],
            "processes": cores, "samples_per_step": cores,
            "threading": "one single-threaded oracle process per host core (spawn-started "
                         "pool), each computing its own bounded sample; a step ends when "
                         "the slowest process finishes",
            "scaling_note": "rank 0 alone runs the host cores of the box; the figure does "
                            "not change with the number of GPUs"}


def run_reference(args, rank, world):
    """--impl reference: the oracle port on all host cores (spawn-started
    process pool, one bounded sample per process per step)."""
    if rank != 0:
        return
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        per_step, nbytes = _reference_steps(pool, cores, args.workload, args.steps, args.warmup)
        per_workload = {}
        if args.workload == "ln_gelu" and not args.no_per_workload:
            for name in PER_WORKLOAD:
                s, b = _reference_steps(pool, cores, name, 3, 1)
                per_workload[name] = {"value": b / s / 1e9, "unit": "GB/s",
                                      "ms_per_step": s * 1e3, "steps": 3, "warmup": 1,
                                      "config": _reference_config(name, cores)}
    gbs = nbytes / per_step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded inputs with the BASELINE config's shapes and distributions)",
        "config": _reference_config(args.workload, cores),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{cores} processes x one {SAMPLE_ROWS[args.workload]}-row "
                                   f"{args.workload} sample per step (oracle port of the "
                                   "reference CPU path; the Rust reference is not buildable "
                                   "here: no cargo)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if per_workload:
        line["per_workload"] = per_workload
    print(json.dumps(line), flush=True)


# ---- GPU workloads --------------------------------------------------------------------------

def _time_ops(torch, ops):
    """GB/s of each kernel on its own: {name: (callable, bytes)}, CUDA events,
    median of 5 runs after 2 warm-ups."""
    out = {}
    for name, (fn, nbytes) in ops.items():
        for _ in range(2):
            fn()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        out[name] = round(nbytes / (statistics.median(ts) * 1e-3) / 1e9, 1)
    return out


def _shard(n, rank, world, mode):
    """Rows [lo, hi) of n that this rank works on: all of them in weak mode
    (every rank owns a full config) and in single mode (one GPU's run of the
    config inside a multi-GPU job), its balanced share in strong mode."""
    if mode != "strong":
        return 0, n
    from oxitorch_b200.sharded import shard_range
    return shard_range(n, rank, world)


class _EventWait:
    """A pending exchange recorded as an event: wait() orders the current
    stream after it (the interface of an async collective's work)."""

    def __init__(self, event):
        self.event = event

    def wait(self):
        import torch
        torch.cuda.current_stream().wait_event(self.event)


class Workload:
    """Inputs resident on the device; fwd()/bwd() launch the path's kernels on
    the current stream; exchange() issues the step's data-parallel collective
    (N > 1) asynchronously on the gradient slot of the step; begin(i) selects
    step i's slot and waits for the exchange that last used it; drain() waits
    for every exchange in flight."""

    dominant = "bwd"       # the kernel the roofline reports
    launches = 0           # our kernels per step
    ROWS = ("rows", "rows")  # (attribute holding the rows per GPU step, unit)
    CONFIG = None          # BASELINE config index of the inputs
    GRAPHS = True          # fwd/bwd phases replayed as CUDA graphs in the timed loop
    VARIANTS = 2           # distinct steps (buffer slots) a graph is captured for

    def __init__(self, dev, rank, world, args, inp=None, mode="weak"):
        import torch
        from oxitorch_b200 import _native as N
        self.torch, self.N, self.L = torch, N, N.load()
        self.dev, self.rank, self.world, self.args, self.mode = dev, rank, world, args, mode
        self.s = torch.cuda.current_stream().cuda_stream
        self.slot = 0
        self.pending = [None, None]

    def close(self):
        """Releases what other ranks hold of this workload (collective)."""

    def begin(self, i):
        self.slot = i % 2
        work = self.pending[self.slot]
        if work is not None:
            work.wait()
            self.pending[self.slot] = None

    def graph_key(self):
        """Identifies the buffers of the current step (its captured graphs)."""
        return self.slot

    def drain(self):
        for k in range(2):
            if self.pending[k] is not None:
                self.pending[k].wait()
                self.pending[k] = None

    def _allreduce_async(self, *tensors):
        """One all-reduce (sum) of the slot's partials, on NCCL's stream; a
        single flat buffer keeps it to one collective."""
        if self.world > 1:
            import torch.distributed as dist
            assert len(tensors) == 1
            self.pending[self.slot] = dist.all_reduce(tensors[0], op=dist.ReduceOp.SUM,
                                                      async_op=True)

    def exchange(self):
        pass

    def partials(self):
        """The tensors the exchange sums (for the post-timing check)."""
        return []

    def inputs_note(self):
        return (f"BASELINE config {self.CONFIG} inputs: numpy Generator(PCG64({self.CONFIG})), "
                "the arrays the parity tests check (bench.config_inputs)"
                if self.CONFIG else "torch generator on the device")

    def config(self):
        return {"workload": self.DESC}


class LnGelu(Workload):
    DESC = ("layer_norm(affine)+gelu(tanh) fwd+bwd, fp32, x [16384, 4096] per GPU "
            "(BASELINE config 2)")
    CONFIG = 2
    KERNEL = "ln_bwd_pipe_kernel (layer_norm+gelu VJP) + dweight/dbias finisher"
    launches = 3  # forward, VJP, dweight+dbias finisher

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        lo, hi = _shard(inp["x"].shape[0], rank, world, mode)
        self.x, self.dy = inp["x"][lo:hi], inp["dy"][lo:hi]
        self.w, self.b = inp["w"], inp["b"]
        self.rows, self.cols = hi - lo, 4096
        R, C = self.rows, self.cols
        self.y, self.dx = t.empty_like(self.x), t.empty_like(self.x)
        self.mean, self.rstd = t.empty(R, device=dev), t.empty(R, device=dev)
        self.dwdb = [t.empty(2 * C, device=dev) for _ in range(2)]
        self.ws_bytes = self.L.oxc_layer_norm_bwd_workspace_size(R, C)
        self.ws = t.empty(max(self.ws_bytes, 16), dtype=t.uint8, device=dev)
        self.fwd_bytes = R * (8 * C + 8) + 8 * C
        self.bwd_bytes = R * (12 * C + 8) + 16 * C

    def fwd(self, x=None):
        N, L = self.N, self.L
        N.check(L.oxc_layer_norm_fwd((x if x is not None else self.x).data_ptr(), self.w.data_ptr(),
                                     self.b.data_ptr(), self.y.data_ptr(), self.mean.data_ptr(),
                                     self.rstd.data_ptr(), self.rows, self.cols, 1e-5,
                                     N.ACT_GELU_TANH, self.s))

    def bwd(self, x=None, dy=None):
        N, L = self.N, self.L
        dwdb = self.dwdb[self.slot]
        N.check(L.oxc_layer_norm_bwd((x if x is not None else self.x).data_ptr(), self.w.data_ptr(),
                                     self.b.data_ptr(), self.mean.data_ptr(), self.rstd.data_ptr(),
                                     (dy if dy is not None else self.dy).data_ptr(),
                                     self.dx.data_ptr(), dwdb.data_ptr(),
                                     dwdb.data_ptr() + self.cols * F32, self.rows, self.cols,
                                     N.ACT_GELU_TANH, N.GRAD_REF, self.ws.data_ptr(),
                                     self.ws_bytes, self.s))

    def exchange(self):
        self._allreduce_async(self.dwdb[self.slot])

    def partials(self):
        return [self.dwdb[self.slot]]

    def e2e_io(self):
        return [self.x, self.dy], [self.y, self.dx, self.dwdb[0]]

    def e2e_step(self, dev_in):
        self.slot = 0
        self.fwd(dev_in[0])
        self.bwd(dev_in[0], dev_in[1])
        self.exchange()
        self.drain()

    def config(self):
        return {"workload": self.DESC, "rows_per_gpu": self.rows, "cols": self.cols, "eps": 1e-5,
                "parallelism": f"row-sharded data parallel x{self.world}, dweight/dbias "
                               "all-reduce overlapped with the next step's forward",
                "grad_mode": "ref (reference graph: rsqrt detached)",
                "inputs": self.inputs_note(),
                "l2": "no flush: every input (268 MB) is larger than the 126 MB L2"}


class Rms(Workload):
    DESC = "rms_norm fwd+bwd, fp32, x [4096, 4096] per GPU (BASELINE config 1)"
    CONFIG = 1
    KERNEL = "rms_bwd_stream_kernel (RMSNorm VJP) + dweight finisher"
    launches = 3
    SETS = 3  # rotating input/output sets: 3 x 268 MB, far more than the 126 MB L2

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        lo, hi = _shard(inp["x"].shape[0], rank, world, mode)
        self.rows, self.cols = hi - lo, 4096
        R, C = self.rows, self.cols
        self.w = inp["w"]
        # Every tensor of config 1 fits in L2, so consecutive steps rotate over
        # SETS copies of (x, dy, y, dx): a step reads a set that the previous
        # step did not touch, and the only dirty lines it meets in L2 are the
        # previous step's own outputs.  (A flush by writing a large buffer left
        # up to 126 MB of the flush buffer's dirty lines to be written back
        # inside the timed step.)  Every set holds the config's x and dy.
        x, dy = inp["x"][lo:hi], inp["dy"][lo:hi]
        self.sets = [(x, dy, t.empty_like(x), t.empty_like(x))]
        for _ in range(self.SETS - 1):
            self.sets.append((x.clone(), dy.clone(), t.empty_like(x), t.empty_like(x)))
        self.cur = 0
        self.x, self.dy, self.y, self.dx = self.sets[0]
        self.rstd = t.empty(R, device=dev)
        self.dws = [t.empty(C, device=dev) for _ in range(2)]
        self.ws_bytes = self.L.oxc_rms_norm_bwd_workspace_size(R, C)
        self.ws = t.empty(max(self.ws_bytes, 16), dtype=t.uint8, device=dev)
        self.fwd_bytes = R * (8 * C + 4) + 4 * C
        self.bwd_bytes = R * (12 * C + 4) + 8 * C

    VARIANTS = 6  # 3 input sets x 2 gradient slots

    def begin(self, i):
        super().begin(i)
        self.cur = i % self.SETS  # the set this step reads

    def graph_key(self):
        return (self.cur, self.slot)

    def fwd(self, x=None):
        if x is None:  # the timed loop: this step's set
            x, _, y, _ = self.sets[self.cur]
        else:          # e2e: the uploaded input, set 0's outputs
            y = self.sets[0][2]
        self.N.check(self.L.oxc_rms_norm_fwd(x.data_ptr(), self.w.data_ptr(), y.data_ptr(),
                                             self.rstd.data_ptr(), self.rows, self.cols, 1e-6,
                                             self.s))

    def bwd(self, x=None, dy=None):
        cx, cdy, _, cdx = self.sets[self.cur] if x is None else self.sets[0]
        self.N.check(self.L.oxc_rms_norm_bwd((x if x is not None else cx).data_ptr(),
                                             self.w.data_ptr(), self.rstd.data_ptr(),
                                             (dy if dy is not None else cdy).data_ptr(),
                                             cdx.data_ptr(), self.dws[self.slot].data_ptr(),
                                             self.rows, self.cols, self.N.GRAD_REF,
                                             self.ws.data_ptr(), self.ws_bytes, self.s))

    def exchange(self):
        self._allreduce_async(self.dws[self.slot])

    def partials(self):
        return [self.dws[self.slot]]

    def e2e_io(self):
        return [self.x, self.dy], [self.y, self.dx, self.dws[0]]

    def e2e_step(self, dev_in):
        self.slot = 0
        self.fwd(dev_in[0])
        self.bwd(dev_in[0], dev_in[1])
        self.exchange()
        self.drain()

    def config(self):
        return {"workload": self.DESC, "rows_per_gpu": self.rows, "cols": self.cols, "eps": 1e-6,
                "inputs": self.inputs_note(),
                "l2": "no flush: each 67 MB tensor fits the 126 MB L2, so steps rotate over "
                      "3 sets of x/dy/y/dx (804 MB in all); a step's inputs were last "
                      "touched two steps earlier and are not in L2"}


class CrossEntropy(Workload):
    DESC = ("log_softmax+cross_entropy (mean) fwd+bwd, fp32, logits [32768, 32000] per GPU "
            "(BASELINE config 3)")
    CONFIG = 3
    KERNEL = "ce_bwd_rows_kernel (cross-entropy VJP)"
    launches = 3

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        lo, hi = _shard(inp["logits"].shape[0], rank, world, mode)
        self.x, self.t = inp["logits"][lo:hi], inp["targets"][lo:hi]
        self.rows, self.cols = hi - lo, 32000
        R, C = self.rows, self.cols
        self.losses = [t.empty(1, device=dev) for _ in range(2)]
        self.rmax, self.rsum, self.rnll = (t.empty(R, device=dev) for _ in range(3))
        self.dx = t.empty_like(self.x)
        self.flag = t.zeros(4, dtype=t.int32, device=dev)
        # the global row count of the mean: every rank's rows (weak) or the
        # config's rows (strong)
        self.total = R * world if mode == "weak" else inp["logits"].shape[0]
        self.fwd_bytes = R * (4 * C + 8 + 12) + 4
        self.bwd_bytes = R * (8 * C + 8 + 8)

    def per_op(self):
        """The standalone F.softmax / F.log_softmax kernels on the same logits
        (forward reads x and writes y; the VJP reads y and dy and writes dx)."""
        t = self.torch
        y, dx = self.dx, t.empty_like(self.x)
        R, C = self.rows, self.cols
        L, N, s = self.L, self.N, self.s
        ops = {}
        for log_ in (0, 1):
            name = "log_softmax" if log_ else "softmax"
            ops[f"{name} forward"] = (lambda log_=log_: N.check(L.oxc_softmax_fwd(
                self.x.data_ptr(), y.data_ptr(), R, C, log_, s)), 8 * R * C)
            ops[f"{name} VJP"] = (lambda log_=log_: N.check(L.oxc_softmax_bwd(
                y.data_ptr(), self.x.data_ptr(), dx.data_ptr(), R, C, log_, s)), 12 * R * C)
        out = _time_ops(t, ops)
        del dx
        return out

    def fwd(self, x=None):
        self.N.check(self.L.oxc_cross_entropy_fwd(
            (x if x is not None else self.x).data_ptr(), self.t.data_ptr(),
            self.losses[self.slot].data_ptr(), self.rmax.data_ptr(), self.rsum.data_ptr(),
            self.rnll.data_ptr(), self.rows, self.cols, self.total, self.flag.data_ptr(), self.s))

    def bwd(self, x=None):
        self.N.check(self.L.oxc_cross_entropy_bwd(
            (x if x is not None else self.x).data_ptr(), self.t.data_ptr(), self.rmax.data_ptr(),
            self.rsum.data_ptr(), None, self.dx.data_ptr(), self.rows, self.cols, self.total, self.s))

    def exchange(self):
        self._allreduce_async(self.losses[self.slot])

    def partials(self):
        return [self.losses[self.slot]]

    def e2e_io(self):
        return [self.x], [self.losses[0], self.dx]

    def e2e_step(self, dev_in):
        self.slot = 0
        self.fwd(dev_in[0])
        self.bwd(dev_in[0])
        self.exchange()
        self.drain()

    def config(self):
        return {"workload": self.DESC, "rows_per_gpu": self.rows, "classes": self.cols,
                "parallelism": f"row-sharded x{self.world}, loss all-reduce (global mean)",
                "inputs": self.inputs_note(),
                "l2": "no flush: logits (4.19 GB) are larger than L2"}


class Embedding(Workload):
    DESC = ("embedding gather + duplicate-id VJP, fp32, table [32000, 4096], ids [64, 2048] "
            "Zipf(1.1) clipped to 31999 (BASELINE config 4)")
    CONFIG = 4
    KERNEL = "emb_rows_kernel + emb_split_kernel (duplicate-id VJP)"
    dominant = "bwd"
    launches = 9  # gather; prepare, sort (4 CUB passes), offsets, split, rows
    ROWS = ("n", "tokens")

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        self.v, self.d = 32000, 4096
        lo, hi = _shard(inp["ids"].shape[0], rank, world, mode)
        self.ids, self.dout = inp["ids"][lo:hi], inp["dout"][lo:hi]
        self.n = n = hi - lo
        self.table = inp["table"]
        self.out = t.empty(n, self.d, device=dev)
        self.flag = t.zeros(4, dtype=t.int32, device=dev)
        self.fwd_bytes = n * 8 + 2 * n * self.d * 4
        if world == 1 or mode == "single":
            self.world = 1  # the single-GPU VJP, no exchange
            self.dtable = t.empty_like(self.table)
            self.ws_bytes = self.L.oxc_embedding_bwd_workspace_size(n, self.v, self.d)
            self.ws = t.empty(max(self.ws_bytes, 16), dtype=t.uint8, device=dev)
            self.bwd_bytes = n * 8 + n * self.d * 4 + self.v * self.d * 4
        else:
            # token-sharded, replicated table: the VJP's rows go to their vocab
            # shard's owner, which sums them in rank order into its dense shard
            # of the gradient on a communication stream that overlaps the next
            # step's forward.  The fused form stores the rows into the owner's
            # memory from the VJP kernel itself (peer memory over NVLink); where
            # peer memory cannot be mapped, the compact VJP + NCCL all-to-all.
            from oxitorch_b200.sharded import PeerGradExchange, SparseGradExchange
            self.GRAPHS = False  # the exchange holds a collective
            self.ex = None
            kind = getattr(args, "exchange", "push")
            if kind != "nccl":
                try:
                    self.ex = PeerGradExchange(n, self.v, self.d, dev, slots=2, mode=kind)
                    self.exchange_kind = "peer"
                    self.launches = 11  # + present, scan (2), meta, map, reduce (and NCCL's)
                except RuntimeError as e:  # raised on every rank alike
                    self.exchange_fallback = str(e)
            if self.ex is None:
                self.ex = SparseGradExchange(n, self.v, self.d, dev, slots=2)
                self.exchange_kind = "nccl"
                self.launches = 14
            self.dshard = self.ex.dshard[0]
            # this rank's share of the job's bytes: its tokens' ids and dout,
            # and its shard of the dense table gradient
            self.bwd_bytes = n * 8 + n * self.d * 4 + self.ex.shard_rows * self.d * 4

    def fwd(self, dout=None):
        self.N.check(self.L.oxc_embedding_fwd(self.table.data_ptr(), self.ids.data_ptr(),
                                              self.out.data_ptr(), self.n, self.v, 0, self.v,
                                              self.d, self.flag.data_ptr(), self.s))

    def bwd(self, dout=None):
        dout = dout if dout is not None else self.dout
        if self.world == 1:
            self.N.check(self.L.oxc_embedding_bwd(dout.data_ptr(), self.ids.data_ptr(),
                                                  self.dtable.data_ptr(), self.n, self.v, 0,
                                                  self.v, self.d, self.flag.data_ptr(),
                                                  self.ws.data_ptr(), self.ws_bytes, self.s))
            return
        self.ex.vjp(self.ids, dout, self.slot)

    def exchange(self):
        if self.world == 1:
            return
        _, done = self.ex.exchange(self.slot)
        self.pending[self.slot] = _EventWait(done)

    def e2e_io(self):
        return [self.dout], [self.out, self.dtable if self.world == 1 else self.dshard]

    def e2e_step(self, dev_in):
        self.fwd()
        self.bwd(dev_in[0])
        self.exchange()

    def close(self):
        if self.world > 1 and self.exchange_kind == "peer":
            self.ex.close()

    def check_exchange(self):
        """After timing (N > 1): one more VJP through the workload's exchange,
        against an independent route: every rank's dense single-GPU VJP of its
        tokens (oxc_embedding_bwd over the whole table), summed over ranks in
        f64 by a reduce-scatter onto the vocab shards.  Tolerance 1e-6 x the sum
        over ranks of |partial|; rows touched by one rank only are that rank's
        position-order sums, so they agree to the bit."""
        t = self.torch
        import torch.distributed as dist
        from oxitorch_b200 import functional as F
        self.begin(0)
        self.bwd()
        self.exchange()
        self.drain()
        got = self.ex.dshard[self.slot].double()
        dense, flag = F.embedding_bwd(self.ids, self.dout, self.v)
        part = dense.double()
        del dense
        lo, rows = self.ex.lo, self.ex.shard_rows
        if self.v % self.world:
            return {"ok": None, "what": "vocab not divisible by the ranks: not checked"}
        cyclic = getattr(self.ex, "cyclic", False)
        if cyclic:  # owner p's rows p, p + N, ...: order the table owner-major
            part = part.view(self.v // self.world, self.world, self.d).transpose(0, 1).contiguous()
        want = t.empty(rows, self.d, dtype=t.float64, device=self.dev)
        dist.reduce_scatter_tensor(want, part)
        tol = t.empty_like(want)
        dist.reduce_scatter_tensor(tol, part.abs_())
        del part
        tol.mul_(1e-6).add_(1e-30)
        err = (got - want).abs_()
        ok = bool((err <= tol).all().item()) and int(flag.abs().sum().item()) == 0 \
            and int(self.ex.flag.abs().sum().item()) == 0
        worst = float((err / tol).max().item())
        return {"ok": ok, "worst_err_over_tolerance": worst,
                "shard_rows": (f"{lo}, {lo} + {self.world}, ... ({rows} rows)" if cyclic
                               else [lo, lo + rows]),
                "what": "exchanged dtable shard vs the f64 reduce-scatter of every rank's dense "
                        "single-GPU VJP, tolerance 1e-6 x sum over ranks of |partial|"}

    def _exchange_desc(self):
        if self.exchange_kind == "peer":
            own = ("rows owned cyclically, row r by rank r mod N, which spreads the Zipf-hot "
                   "low ids")
            if self.ex.mode == "pull":
                return ("exchange over NVLink peer memory (CUDA IPC), pull form: the VJP kernel "
                        "writes each touched row into this GPU's region for the row's owner; after "
                        "a stream-ordered barrier each owner's kernel reads its regions from every "
                        "rank's memory and sums them in rank order, overlapping the next forward; "
                        + own)
            return ("exchange over NVLink peer memory (CUDA IPC), push form: the VJP kernel "
                    "stores each touched row into its owner's memory; a stream-ordered barrier; "
                    "the owner's rank-order sum; " + own)
        why = getattr(self, "exchange_fallback", None)
        return ("compact VJP + NCCL all-to-all of the touched rows to their vocab shard's owner "
                "+ rank-order sum (sparse exchange)" + (f"; peer memory unavailable: {why}"
                                                        if why else ""))

    def config(self):
        return {"workload": self.DESC, "ids_per_gpu": self.n, "table": [self.v, self.d],
                "parallelism": (f"token-sharded data parallel x{self.world}, replicated table; "
                                + self._exchange_desc() if self.world > 1 else "one GPU"),
                "inputs": self.inputs_note(),
                "roofline_note": "the VJP is the HBM-bound phase; the gather's hot table rows are "
                                 "L2 hits, so its algorithmic bytes exceed its DRAM bytes "
                                 "(fwd_dram_gbs)",
                "l2": "no flush: dout (2.1 GB) is larger than L2"}


class EmbeddingVocab(Workload):
    """The vocab-sharded scheme: every rank holds a 1/N row shard of the table
    and all the ids; the forward is a masked gather (zeros for other shards'
    ids) followed by an all-reduce of the [131072, 4096] output; each rank's
    VJP writes its own shard's rows from the replicated dout, with no exchange.
    Communication-bound by construction: reported beside the token-sharded
    scheme, as strong scaling of the one config."""
    DESC = ("embedding, vocab-sharded table: masked gather + all-reduce of the [131072, 4096] "
            "output, per-shard duplicate-id VJP (BASELINE config 4)")
    CONFIG = 4
    KERNEL = "emb_gather_kernel + NCCL all-reduce of the output (the step is communication-bound)"
    dominant = "fwd"
    launches = 9
    GRAPHS = False  # the forward holds the output all-reduce
    ROWS = ("n", "tokens")

    def __init__(self, dev, rank, world, args, inp, mode="strong"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        from oxitorch_b200.sharded import vocab_shard
        self.v, self.d = 32000, 4096
        self.ids, self.dout = inp["ids"], inp["dout"]
        self.n = n = self.ids.shape[0]
        self.lo, self.rows = vocab_shard(self.v, rank, world)
        self.table = inp["table"][self.lo:self.lo + self.rows]
        self.out = t.empty(n, self.d, device=dev)
        self.dshard = t.empty(self.rows, self.d, device=dev)
        self.flag = t.zeros(4, dtype=t.int32, device=dev)
        self.ws_bytes = self.L.oxc_embedding_bwd_workspace_size(n, self.rows, self.d)
        self.ws = t.empty(max(self.ws_bytes, 16), dtype=t.uint8, device=dev)
        # the job's algorithmic bytes are the one config's, shared by the ranks
        self.fwd_bytes = (n * 8 + 2 * n * self.d * 4) // world
        self.bwd_bytes = (n * 8 + n * self.d * 4 + self.v * self.d * 4) // world

    def fwd(self):
        self.N.check(self.L.oxc_embedding_fwd(self.table.data_ptr(), self.ids.data_ptr(),
                                              self.out.data_ptr(), self.n, self.v, self.lo,
                                              self.rows, self.d, self.flag.data_ptr(), self.s))
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(self.out, op=dist.ReduceOp.SUM)

    def bwd(self):
        self.N.check(self.L.oxc_embedding_bwd(self.dout.data_ptr(), self.ids.data_ptr(),
                                              self.dshard.data_ptr(), self.n, self.v, self.lo,
                                              self.rows, self.d, self.flag.data_ptr(),
                                              self.ws.data_ptr(), self.ws_bytes, self.s))

    def config(self):
        return {"workload": self.DESC, "ids": self.n, "table_rows_per_gpu": self.rows,
                "parallelism": f"vocab-sharded x{self.world}: output all-reduce "
                               f"({self.n * self.d * 4 / 1e9:.2f} GB) in the forward",
                "inputs": self.inputs_note()}


class MlpBlock(Workload):
    E2E_LARGE = True
    DESC = ("decoder-MLP activation block fwd+bwd, fp32, 65536 tokens: RMSNorm [.., 4096] "
            "(broadcast weight view), SwiGLU [.., 11008] (transposed gate view), dim-1 "
            "sum/max/argmax, whole-tensor L2 of {dx, dg, du} (BASELINE config 5)")
    CONFIG = 5
    KERNEL = "swiglu_bwd_tile_kernel (SwiGLU VJP, sum-of-squares fused)"
    launches = 8
    ROWS = ("M", "tokens")

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        lo, hi = _shard(inp["x"].shape[0], rank, world, mode)
        M = hi - lo
        D, H = 4096, 11008
        self.M, self.D, self.H = M, D, H
        self.x, self.up = inp["x"][lo:hi], inp["up"][lo:hi]
        self.dy, self.dh = inp["dy"][lo:hi], inp["dh"][lo:hi]
        self.wbuf = inp["w"]
        self.gate_buf = inp["gate_buf"][:, lo:hi]
        self.y, self.dx = t.empty_like(self.x), t.empty_like(self.x)
        self.rstd = t.empty(M, device=dev)
        self.h, self.dg, self.du = (t.empty(M, H, device=dev) for _ in range(3))
        self.hs, self.hm, self.ha = (t.empty(M, device=dev) for _ in range(3))
        # one flat exchange buffer per slot: dweight [D] then the two f64 sums
        # of squares (as 4 floats)
        self.xbuf = [t.empty(D + 4, device=dev) for _ in range(2)]
        self.rws_bytes = self.L.oxc_rms_norm_bwd_workspace_size(M, D)
        self.rws = t.empty(max(self.rws_bytes, 16), dtype=t.uint8, device=dev)
        self.sws_bytes = self.L.oxc_swiglu_bwd_workspace_size(M, H)
        self.sws = t.empty(max(self.sws_bytes, 16), dtype=t.uint8, device=dev)
        import ctypes
        self.ctypes = ctypes
        self.fwd_bytes = M * (8 * D + 4) + 4 * D + M * 12 * H + 12 * M
        self.bwd_bytes = M * (12 * D + 4) + 8 * D + M * 20 * H + 16

    def _v(self, tensor):
        return self.ctypes.byref(self.N.make_view(tensor))

    def fwd(self, x=None, gate=None):
        N, L = self.N, self.L
        x = x if x is not None else self.x
        gate = gate if gate is not None else self.gate_buf.t()
        N.check(L.oxc_rms_norm_fwd(x.data_ptr(), self.wbuf.data_ptr(), self.y.data_ptr(),
                                   self.rstd.data_ptr(), self.M, self.D, 1e-6, self.s))
        N.check(L.oxc_swiglu_fwd(self._v(gate), self._v(self.up), self.h.data_ptr(),
                                 self.hs.data_ptr(), self.hm.data_ptr(), self.ha.data_ptr(), self.s))

    def bwd(self, x=None, gate=None):
        N, L = self.N, self.L
        x = x if x is not None else self.x
        gate = gate if gate is not None else self.gate_buf.t()
        xb = self.xbuf[self.slot]
        sq = xb.data_ptr() + self.D * F32
        N.check(L.oxc_rms_norm_bwd(x.data_ptr(), self.wbuf.data_ptr(), self.rstd.data_ptr(),
                                   self.dy.data_ptr(), self.dx.data_ptr(), xb.data_ptr(),
                                   self.M, self.D, N.GRAD_REF, self.rws.data_ptr(), self.rws_bytes,
                                   self.s))
        N.check(L.oxc_swiglu_bwd(self._v(gate), self._v(self.up), self._v(self.dh),
                                 self.dg.data_ptr(), self.du.data_ptr(), sq,
                                 self.sws.data_ptr(), self.sws_bytes, self.s))
        views = (N.View * 1)(N.make_view(self.dx))
        N.check(L.oxc_sum_squares(views, 1, sq + 8, self.sws.data_ptr(), self.sws_bytes, self.s))

    def exchange(self):
        # dweight (f32) and the f64 sums of squares travel as one buffer: the
        # f64 pair is summed by a separate f64 all-reduce of its view
        if self.world > 1:
            import torch.distributed as dist
            xb = self.xbuf[self.slot]
            dist.all_reduce(xb[self.D:].view(self.torch.float64), op=dist.ReduceOp.SUM,
                            async_op=True)
            self.pending[self.slot] = dist.all_reduce(xb[:self.D], op=dist.ReduceOp.SUM,
                                                      async_op=True)

    def partials(self):
        return [self.xbuf[self.slot][:self.D]]

    def e2e_io(self):
        return ([self.x, self.gate_buf, self.up, self.dy, self.dh],
                [self.y, self.h, self.hs, self.hm, self.ha, self.dx, self.xbuf[0], self.dg,
                 self.du])

    def e2e_step(self, dev_in):
        x, gate_buf, up, dy, dh = dev_in
        saved = (self.up, self.dy, self.dh)
        self.up, self.dy, self.dh = up, dy, dh
        self.slot = 0
        self.fwd(x, gate_buf.t())
        self.bwd(x, gate_buf.t())
        self.exchange()
        self.drain()
        self.up, self.dy, self.dh = saved

    def config(self):
        return {"workload": self.DESC, "tokens_per_gpu": self.M, "hidden": self.D,
                "ffn": self.H, "gate_strides": [1, 65536], "weight_strides": [0, 1],
                "inputs": self.inputs_note(),
                "l2": "no flush: every tensor (1-2.9 GB) is larger than L2"}


class Registry(Workload):
    DESC = ("config-5 SwiGLU composed from the elementwise registry and dim reductions, as the "
            "reference's F.silu(g) * u graph runs it: sigmoid, mul, mul, dim-1 sum/max/argmax "
            "forward; the graph's eight elementwise VJP ops backward; gate a transposed view "
            "(BASELINE config 5, strided engine)")
    CONFIG = 5
    KERNEL = "elem_dense_kernel / elem_pipe_kernel (registry binary ops of the VJP)"
    launches = 14  # sigmoid, 2 mul, 3 reductions; 7 binary + 1 scalar-binary
    E2E_LARGE = True
    MUL, ADD, SUB, SIGMOID = 2, 0, 1, 12
    R_SUM, R_MAX, R_ARGMAX = 0, 2, 4
    ROWS = ("M", "tokens")

    def __init__(self, dev, rank, world, args, inp, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        import ctypes
        t = self.torch
        lo, hi = _shard(inp["up"].shape[0], rank, world, mode)
        M = hi - lo
        H = 11008
        self.M, self.H = M, H
        self.ctypes = ctypes
        self.gate_buf = inp["gate_buf"][:, lo:hi]
        self.up, self.dh = inp["up"][lo:hi], inp["dh"][lo:hi]
        (self.sg, self.silu, self.h, self.du, self.t, self.dg1, self.ds, self.oms, self.sds,
         self.dg2, self.dg) = (t.empty(M, H, device=dev) for _ in range(11))
        self.hs, self.hm, self.ha = (t.empty(M, device=dev) for _ in range(3))
        self.fwd_bytes = M * H * (8 + 12 + 12 + 3 * 4) + 3 * 4 * M
        self.bwd_bytes = M * H * (7 * 12 + 8)

    def _v(self, x):
        return self.ctypes.byref(self.N.make_view(x))

    def _bin(self, op, a, b, out):
        self.N.check(self.L.oxc_binary(op, self._v(a), self._v(b), self._v(out), self.s))

    def _red(self, kind, x, out):
        self.N.check(self.L.oxc_reduce(kind, self._v(x), 1, 0, self._v(out), None, 0, self.s))

    def fwd(self):
        g = self.gate_buf.t()
        self.N.check(self.L.oxc_unary(self.SIGMOID, self._v(g), self._v(self.sg), self.s))
        self._bin(self.MUL, g, self.sg, self.silu)
        self._bin(self.MUL, self.silu, self.up, self.h)
        self._red(self.R_SUM, self.h, self.hs)
        self._red(self.R_MAX, self.h, self.hm)
        self._red(self.R_ARGMAX, self.h, self.ha)

    def bwd(self):
        # h = silu * u;  silu = g * s;  s = sigmoid(g)  (autograd/ops.rs mul and sigmoid VJPs)
        g = self.gate_buf.t()
        self._bin(self.MUL, self.dh, self.silu, self.du)
        self._bin(self.MUL, self.dh, self.up, self.t)
        self._bin(self.MUL, self.t, self.sg, self.dg1)
        self._bin(self.MUL, self.t, g, self.ds)
        self.N.check(self.L.oxc_binary_scalar(self.SUB, self._v(self.sg), 1.0, 1, self._v(self.oms),
                                              self.s))
        self._bin(self.MUL, self.sg, self.oms, self.sds)
        self._bin(self.MUL, self.ds, self.sds, self.dg2)
        self._bin(self.ADD, self.dg1, self.dg2, self.dg)

    def per_op(self):
        """GB/s of each kernel on its own (CUDA events, median of 5 after 2 warm-ups)."""
        g = self.gate_buf.t()
        MH = self.M * self.H
        ops = {
            "sigmoid(transposed gate)": (lambda: self.N.check(self.L.oxc_unary(
                self.SIGMOID, self._v(g), self._v(self.sg), self.s)), 8 * MH),
            "mul(transposed gate, dense)": (lambda: self._bin(self.MUL, g, self.sg, self.silu),
                                            12 * MH),
            "mul(dense, dense)": (lambda: self._bin(self.MUL, self.silu, self.up, self.h), 12 * MH),
            "sub(1, dense) scalar": (lambda: self.N.check(self.L.oxc_binary_scalar(
                self.SUB, self._v(self.sg), 1.0, 1, self._v(self.oms), self.s)), 8 * MH),
            "sum over dim 1": (lambda: self._red(self.R_SUM, self.h, self.hs), 4 * MH + 4 * self.M),
            "max over dim 1": (lambda: self._red(self.R_MAX, self.h, self.hm), 4 * MH + 4 * self.M),
            "argmax over dim 1": (lambda: self._red(self.R_ARGMAX, self.h, self.ha),
                                  4 * MH + 4 * self.M),
        }
        return _time_ops(self.torch, ops)

    def e2e_io(self):
        return [self.gate_buf, self.up, self.dh], [self.h, self.hs, self.hm, self.ha, self.dg,
                                                    self.du]

    def e2e_step(self, dev_in):
        saved = (self.gate_buf, self.up, self.dh)
        self.gate_buf, self.up, self.dh = dev_in
        self.fwd()
        self.bwd()
        self.gate_buf, self.up, self.dh = saved

    def config(self):
        return {"workload": self.DESC, "tokens_per_gpu": self.M, "ffn": self.H,
                "gate_strides": [1, 65536], "inputs": self.inputs_note(),
                "l2": "no flush: every tensor (2.9 GB) is larger than L2"}


class Optim(Workload):
    DESC = ("optimizer step on device, fp32: AdamW (forward phase) and SGD with Nesterov "
            "momentum (backward phase), each over a flat parameter of 2^28 elements per GPU")
    KERNEL = "adam_kernel (AdamW step)"
    dominant = "fwd"
    launches = 2
    GRAPHS = False  # the step counter (bias corrections) changes every step
    E2E_LARGE = True
    ROWS = ("n", "elements")

    def __init__(self, dev, rank, world, args, inp=None, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        t = self.torch
        gen = t.Generator(device=dev)
        gen.manual_seed(7 + 1000 * rank)
        n = self.n = args.rows or (1 << 28)
        self.p = t.randn(n, device=dev, generator=gen)
        self.g = t.randn(n, device=dev, generator=gen) * 0.01
        self.m = t.zeros(n, device=dev)
        self.v = t.zeros(n, device=dev)
        self.p2 = t.randn(n, device=dev, generator=gen)
        self.vel = t.zeros(n, device=dev)
        self.t = 0
        self.fwd_bytes = 28 * n  # read p, g, m, v; write p, m, v
        self.bwd_bytes = 20 * n  # read p, g, buf; write p, buf

    def fwd(self, g=None):
        self.t += 1
        self.N.check(self.L.oxc_adamw_step(
            self.p.data_ptr(), (g if g is not None else self.g).data_ptr(), self.m.data_ptr(),
            self.v.data_ptr(), self.n, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1, self.t, self.s))

    def bwd(self, g=None):
        self.N.check(self.L.oxc_sgd_step(
            self.p2.data_ptr(), (g if g is not None else self.g).data_ptr(), self.vel.data_ptr(),
            self.n, 1e-2, 0.9, 1, self.s))

    def e2e_io(self):
        return [self.g], [self.p, self.p2]

    def e2e_step(self, dev_in):
        self.fwd(dev_in[0])
        self.bwd(dev_in[0])

    def config(self):
        return {"workload": self.DESC, "elements_per_gpu": self.n,
                "hyperparameters": "AdamW lr 1e-3, betas (0.9, 0.999), eps 1e-8, wd 0.01; "
                                   "SGD lr 1e-2, momentum 0.9, Nesterov",
                "parallelism": f"data-parallel replicas x{self.world}, no exchange in the step",
                "inputs": self.inputs_note(),
                "l2": "no flush: every tensor (1.07 GB) is larger than the 126 MB L2"}


# CIFAR-10-shaped loader epoch: per sample, the plain epoch moves the 12288-byte
# image and the 4-byte label in and out and reads the 8-byte order entry once
# per column; the augmented epoch reads and writes the 3 x 28 x 28 crop (9408
# bytes), reads three 24-byte plane maps and the order entry, and gathers the
# label.
LOADER_STEPS = [("crop", 28), ("flip",),
                ("normalize", [0.4914, 0.4822, 0.4465], [0.247, 0.243, 0.261])]
LOADER_PLAIN_BYTES = 2 * 12288 + 2 * 4 + 2 * 8
LOADER_AUG_BYTES = 2 * 9408 + 3 * 24 + 8 + (2 * 4 + 8)


class Loader(Workload):
    DESC = ("data loader epoch on device, fp32 CIFAR-10-shaped columns (50000 x 3 x 32 x 32 "
            "images, 50000 labels), batch 512, shuffled: the plain epoch gather (forward phase) "
            "and the augmented epoch, RandomCrop(28) + RandomHorizontalFlip + Normalize "
            "(backward phase)")
    KERNEL = "image_epoch_kernel (gather + crop + flip + normalize) + label gather"
    dominant = "bwd"
    launches = 3
    GRAPHS = False  # epochs upload their plans from the host
    ROWS = ("n", "samples")

    def __init__(self, dev, rank, world, args, inp=None, mode="weak"):
        super().__init__(dev, rank, world, args, inp, mode)
        from oxitorch_b200 import data as D
        t = self.torch
        gen = t.Generator(device=dev)
        gen.manual_seed(9 + 1000 * rank)
        n = self.n = args.rows or 50000
        self.images = t.randn(n, 3, 32, 32, device=dev, generator=gen)
        self.labels = t.randint(0, 10, (n,), device=dev, generator=gen).float()
        wire = D.NativeTransform([("crop", [28]), ("flip", []),
                                  ("normalize", LOADER_STEPS[2][1] + LOADER_STEPS[2][2])])
        self.plain = D.DataLoader([self.images, self.labels], batch_size=512, shuffle=True, seed=1)
        self.aug = D.DataLoader([self.images, self.labels], batch_size=512, shuffle=True, seed=1,
                                transforms=wire, transform_seed=2)
        # the host half (order, draws, uploads) once; the timed steps re-launch them
        self.ep_plain = self.plain._plan_epoch(self.L)
        self.ep_aug = self.aug._plan_epoch(self.L)
        self.fwd_bytes = n * LOADER_PLAIN_BYTES
        self.bwd_bytes = n * LOADER_AUG_BYTES
        self.last = t.empty(512, device=dev)

    def fwd(self):
        self.plain._launch_epoch(self.L, self.ep_plain)

    def bwd(self):
        self.aug._launch_epoch(self.L, self.ep_aug)

    def e2e_io(self):
        return [], [self.last]

    def e2e_step(self, dev_in):
        """Both epochs through the public API: host order and draws, their
        uploads, the launches, and every batch taken; the step's result read
        back is the last augmented batch's labels."""
        for _ in self.plain:
            pass
        for batch in self.aug:
            pass
        self.last[:batch[1].shape[0]].copy_(batch[1])

    def config(self):
        return {"workload": self.DESC, "samples_per_gpu": self.n,
                "parallelism": f"data-parallel replicas x{self.world}, each loading its own copy",
                "inputs": self.inputs_note(),
                "l2": "no flush: the 614 MB image column and the epoch buffers exceed the 126 MB L2",
                "e2e_note": "the dataset stays resident; per epoch the API uploads the order "
                            "(8 B/sample) and the plane maps (72 B/sample) itself"}


WORKLOADS = {"ln_gelu": LnGelu, "rms": Rms, "ce": CrossEntropy, "embedding": Embedding,
             "embedding_vocab": EmbeddingVocab, "mlp_block": MlpBlock, "registry": Registry,
             "optim": Optim, "loader": Loader}


# ---- timing ----------------------------------------------------------------------------------

def _max_over_ranks(torch, dev, world, value):
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([value], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return value


def time_steps(wl, steps, warmup, world, local_rank, exchange=True, solo=False):
    """Device time of exactly `steps` steps after `warmup` untimed ones: CUDA
    events on the launching stream around the whole loop, a barrier and a
    synchronize on both sides, the max over ranks.  The last step's exchange
    is inside the timed region (drain() before the end event).  `solo`: this
    rank runs alone (no barrier, no max), the others wait.

    A step is one replay of a graph holding the forward and the VJP (or their
    eager launches); no event is recorded between the phases, because a timing
    event between two kernels makes the GPU drain the first before the second
    starts (on config 1 that cost 9 us of a 59 us step).  The phases' own
    durations (the roofline's kernel time) come from two more loops right
    after, timed the same way: `steps` forward launches back to back, then
    `steps` VJP launches, on the same rotating buffers.
    Returns (ms_per_step, fwd_ms, bwd_ms, clocks)."""
    torch = wl.torch
    stream = torch.cuda.current_stream()
    multi = world > 1 and not solo
    if multi:
        import torch.distributed as dist

    graphs = capture_graphs(wl) if wl.GRAPHS else None

    def run(phase):
        if graphs:
            graphs[(phase, wl.graph_key())].replay()
        else:
            if phase in ("step", "fwd"):
                wl.fwd()
            if phase in ("step", "bwd"):
                wl.bwd()

    def one(i):
        wl.begin(i)
        run("step")
        if exchange:
            wl.exchange()

    for i in range(warmup):
        one(i)
    wl.drain()
    torch.cuda.synchronize()

    def timed(body, first):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if multi:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(steps):
            body(first + i)
        wl.drain()
        end.record(stream)
        torch.cuda.synchronize()
        if multi:
            dist.barrier()
        ms = start.elapsed_time(end)
        if multi:
            ms = _max_over_ranks(torch, wl.dev, world, ms)
        return ms / steps

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    ms = timed(one, warmup)
    clocks = sampler.stop()

    def phase_body(phase):
        def body(i):
            wl.begin(i)
            run(phase)
        return body

    fwd_ms = timed(phase_body("fwd"), warmup + steps)
    bwd_ms = timed(phase_body("bwd"), warmup + 2 * steps)
    wl.graphs_used = bool(graphs)
    return ms, fwd_ms, bwd_ms, clocks


def capture_graphs(wl):
    """One CUDA graph per phase (fwd, bwd, and the whole step) and step variant,
    so the timed loops launch each with one replay instead of a Python call
    per kernel (configs whose steps last tens of microseconds are otherwise
    bound by the host).  The kernels and their launch geometry are exactly the
    eager ones.  Returns None (eager launches) if a capture fails."""
    torch = wl.torch
    stream = torch.cuda.current_stream()
    graphs = {}

    def both():
        wl.fwd()
        wl.bwd()
    try:
        for i in range(wl.VARIANTS):
            wl.begin(i)
            key = wl.graph_key()
            for phase, fn in (("fwd", wl.fwd), ("bwd", wl.bwd), ("step", both)):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                    fn()
                graphs[(phase, key)] = g
        wl.drain()
        torch.cuda.synchronize()
        return graphs
    except Exception as e:  # noqa: BLE001 -- reported, and the loop runs eagerly
        log(f"graph capture failed for {type(wl).__name__} ({e}); launching eagerly")
        torch.cuda.synchronize()
        return None


def exchange_check(wl):
    """After timing: one more VJP, then its partials all-reduced through the
    workload's own exchange, compared with the f64 sum of every rank's partial
    (all-gathered).  Tolerance 1e-6 x sum over ranks of |partial| (NCCL's
    reduction order is its own)."""
    torch = wl.torch
    import torch.distributed as dist
    wl.begin(0)
    wl.fwd()
    wl.bwd()
    parts = [p.clone() for p in wl.partials()]
    wl.exchange()
    wl.drain()
    worst, ok = 0.0, True
    for before, after in zip(parts, wl.partials()):
        gathered = [torch.empty_like(before) for _ in range(wl.world)]
        dist.all_gather(gathered, before)
        stack = torch.stack(gathered).double()
        want = stack.sum(0)
        tol = 1e-6 * stack.abs().sum(0) + 1e-30
        err = (after.double() - want).abs()
        worst = max(worst, float((err / tol).max().item()))
        ok = ok and bool((err <= tol).all().item())
    return {"ok": ok, "worst_err_over_tolerance": worst,
            "what": "all-reduced partials vs the f64 sum of the all-gathered per-rank partials, "
                    "tolerance 1e-6 x sum of |partials|"}


def measure(name, args, rank, world, local_rank, inp, steps, warmup, mode="weak",
            cpu_budget=0.0, with_per_op=False):
    """Times one workload and returns its report (rank 0) or None."""
    import torch
    dev = torch.device("cuda", local_rank)
    cls = WORKLOADS[name]
    wl = cls(dev, rank, world, args, inp, mode)
    ms, fwd_ms, bwd_ms, clocks = time_steps(wl, steps, warmup, world, local_rank)
    check = None
    if world > 1 and hasattr(wl, "check_exchange"):
        check = wl.check_exchange()
    elif world > 1 and wl.partials():
        check = exchange_check(wl)
    total_bytes = world * (wl.fwd_bytes + wl.bwd_bytes)
    peak, peak_kind = measured_peak()
    dom_ms, dom_bytes = (bwd_ms, wl.bwd_bytes) if wl.dominant == "bwd" else (fwd_ms, wl.fwd_bytes)
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    prof = _profiled_traffic(name)
    traffic = prof.get("dram_bytes_per_launch")
    rep = {
        "workload": name,
        "value": total_bytes / (ms * 1e-3) / 1e9,
        "unit": "GB/s",
        "ms_per_step": ms,
        "steps": steps, "warmup": warmup,
        "scaling": "weak" if mode == "weak" else "strong",
        "rows_per_s": {"value": world * getattr(wl, wl.ROWS[0]) / (ms * 1e-3),
                       "unit": f"{wl.ROWS[1]}/s"},
        "config": {**wl.config(), "algorithmic_bytes_per_gpu_step": wl.fwd_bytes + wl.bwd_bytes},
        "roofline": {
            "bound": "hbm",
            "kernel": wl.KERNEL,
            "achieved": achieved,
            "peak": peak,
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs: torch copy read+write)",
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            # the same phase time with the profiled DRAM bytes
            "dram_gbs": traffic / (dom_ms * 1e-3) / 1e9 if traffic else None,
            "fwd_gbs": wl.fwd_bytes / (fwd_ms * 1e-3) / 1e9,
            "bwd_gbs": wl.bwd_bytes / (bwd_ms * 1e-3) / 1e9,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        },
        "gpu_launches": wl.launches * steps,
        "clocks": clocks,
    }
    rep["config"]["launch"] = ("each step replayed as one CUDA graph of the same kernels (forward "
                               "then VJP), one per step variant" if wl.graphs_used
                               else "eager launches through the C ABI")
    rep["roofline"]["phase_timing"] = (
        "fwd_ms / bwd_ms: each phase timed over its own loop of `steps` back-to-back launches "
        "(CUDA events on the launching stream, max over ranks) right after the step loop, on "
        "the same rotating buffers; the step loop itself records no event between the phases, "
        "since a timing event between two kernels makes the GPU drain the first before the "
        "second starts")
    if prof.get("fwd_dram_bytes_per_launch"):
        rep["roofline"]["fwd_dram_gbs"] = prof["fwd_dram_bytes_per_launch"] / (fwd_ms * 1e-3) / 1e9
    if check is not None:
        rep["exchange_check"] = check
    if rank == 0 and with_per_op and hasattr(wl, "per_op"):
        rep["config"]["per_op_gbs"] = wl.per_op()
    if rank == 0 and world == 1 and cpu_budget > 0:
        rep["cpu_baseline"] = cpu_baseline(name, cpu_budget)
    return wl, rep


# the input whose rows the strong-scaling split divides
GLOBAL_ROWS_KEY = {"ln_gelu": "x", "rms": "x", "ce": "logits", "embedding": "ids",
                   "embedding_vocab": "ids", "mlp_block": "x", "registry": "up"}


def strong_scaling(name, args, rank, world, local_rank, inp, steps, warmup):
    """The global config split `world` ways, timed with every rank, against
    the same global config on rank 0 alone (no exchange) in the same run:
    efficiency T1 / (N * T_N)."""
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    t1 = None
    if rank == 0:
        wl1 = WORKLOADS[name](dev, rank, world, args, inp, "single")
        t1, _, _, _ = time_steps(wl1, steps, warmup, world, local_rank, exchange=False, solo=True)
        del wl1
    dist.barrier()
    wl, rep = measure(name, args, rank, world, local_rank, inp, steps, warmup, mode="strong")
    wl.close()
    del wl
    if rank != 0:
        return None
    tn = rep["ms_per_step"]
    return {"value": rep["value"], "unit": "GB/s", "ms_per_step": tn, "t1_ms_per_step": t1,
            "global_rows": inp[GLOBAL_ROWS_KEY[name]].shape[0],
            "per_gpu": rep["config"], "efficiency": t1 / (world * tn),
            "exchange_check": rep.get("exchange_check"),
            "note": "T1: the global config on rank 0 alone with no exchange; T_N: each rank its "
                    "1/N row share plus the step's exchange"}


def run_ours(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    # every launch of the run goes to one non-default stream, which CUDA graphs
    # can be captured on
    with torch.cuda.stream(torch.cuda.Stream()):
        _run_ours(args, rank, world, local_rank)


def _run_ours(args, rank, world, local_rank):
    import torch
    dev = torch.device("cuda", local_rank)
    name = args.workload
    cls = WORKLOADS[name]
    inp = device_inputs(cls.CONFIG, dev, rank, world, args.rows) if cls.CONFIG else None
    wl, rep = measure(name, args, rank, world, local_rank, inp, args.steps, args.warmup,
                      cpu_budget=10.0 if not args.no_cpu_baseline else 0.0,
                      with_per_op=(name in ("ce", "registry")))

    # ---- e2e: host buffers through the C ABI --------------------------------------------
    e2e = None
    if getattr(wl, "E2E_LARGE", False) and not args.e2e_large:
        ins, outs = wl.e2e_io()
        gb = sum(t.numel() * t.element_size() for t in ins + outs) / 1e9
        e2e = {"value": None, "unit": "GB/s",
               "skipped": f"this workload moves {gb:.1f} GB per step through pinned host "
                          "buffers; pass --e2e-large to measure it"}
    elif not args.skip_e2e:
        e2e = run_e2e(torch, wl, args, dev, world)
    wl.close()
    del wl
    torch.cuda.empty_cache()

    strong = None
    if world > 1 and cls.CONFIG and not args.no_strong:
        strong = strong_scaling(name, args, rank, world, local_rank, inp, args.steps,
                                args.warmup)
    del inp
    torch.cuda.empty_cache()

    per_workload = {}
    if name == "ln_gelu" and not args.no_per_workload:
        psteps = max(5, min(args.steps, 50))
        for other in PER_WORKLOAD:
            oinp = device_inputs(WORKLOADS[other].CONFIG, dev, rank, world, args.rows)
            owl, orep = measure(other, args, rank, world, local_rank, oinp, psteps, 3,
                                cpu_budget=3.0 if not args.no_cpu_baseline else 0.0)
            owl.close()
            del owl
            if world > 1 and not args.no_strong:
                orep["strong_scaling"] = strong_scaling(other, args, rank, world, local_rank,
                                                        oinp, psteps, 3)
            per_workload[other] = orep
            if other == "mlp_block":
                # config 5 once more, composed from the generic registry (the
                # reference's own graph of F.silu(g) * u), on the same arrays
                rwl, rrep = measure("registry", args, rank, world, local_rank, oinp, psteps, 3)
                del rwl
                per_workload["registry"] = rrep
            if other == "embedding" and world > 1:
                # the vocab-sharded scheme beside the token-sharded one
                vwl, vrep = measure("embedding_vocab", args, rank, world, local_rank, oinp,
                                    psteps, 3, mode="strong")
                del vwl
                if rank == 0 and orep.get("strong_scaling"):
                    t1 = orep["strong_scaling"]["t1_ms_per_step"]
                    vrep["strong_scaling"] = {"t1_ms_per_step": t1,
                                              "ms_per_step": vrep["ms_per_step"],
                                              "efficiency": t1 / (world * vrep["ms_per_step"])}
                per_workload["embedding_vocab_sharded"] = vrep
            del oinp
            torch.cuda.synchronize()
            torch.cuda.empty_cache()

    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": rep["value"],
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": rep["ms_per_step"],
        "rows_per_s": rep["rows_per_s"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (numpy-seeded inputs with the BASELINE config's shapes and "
                "distributions; no dataset)",
        "config": rep["config"],
        "roofline": rep["roofline"],
        "e2e": e2e,
        "gpu_launches": rep["gpu_launches"],
        "clocks": rep["clocks"],
        "cpu_baseline": rep.get("cpu_baseline"),
    }
    if "exchange_check" in rep:
        line["exchange_check"] = rep["exchange_check"]
    if strong:
        line["strong_scaling"] = strong
    if per_workload:
        line["per_workload"] = per_workload
    print(json.dumps(line), flush=True)


def run_e2e(torch, wl, args, dev, world):
    """The step through the C ABI with host buffers: every step uploads its
    inputs and downloads its outputs inside the timed region."""
    stream = torch.cuda.current_stream()
    ins, outs = wl.e2e_io()
    h_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t) for t in ins]
    d_in = [[torch.empty_like(t) for t in ins] for _ in range(2)]
    h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs]
    up_s, down_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_run(n):
        """n steps through the C ABI.  Step i uploads its inputs into
        d_in[i % 2] on one copy stream and downloads its outputs on the
        other; step i+1's upload runs while step i computes and downloads
        (PCIe is full duplex).  Ordering: an upload waits until the step
        that last used its buffer has computed; a step computes after its
        upload and after the previous step's download (the outputs are
        reused).  Returns the event of the last download."""
        comp, up, down = [None] * n, [None] * n, [None] * n

        def upload(i):
            with torch.cuda.stream(up_s):
                if i >= 2:
                    up_s.wait_event(comp[i - 2])
                for d, h in zip(d_in[i % 2], h_in):
                    d.copy_(h, non_blocking=True)
                up[i] = torch.cuda.Event()
                up[i].record(up_s)

        up_s.wait_stream(stream)
        down_s.wait_stream(stream)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            stream.wait_event(up[i])
            if i >= 1:
                stream.wait_event(down[i - 1])
            wl.e2e_step(d_in[i % 2])
            comp[i] = torch.cuda.Event()
            comp[i].record(stream)
            with torch.cuda.stream(down_s):
                down_s.wait_event(comp[i])
                for h, d in zip(h_out, outs):
                    h.copy_(d, non_blocking=True)
                down[i] = torch.cuda.Event()
                down[i].record(down_s)
        return down[n - 1]

    # 16 steps: the first upload and the last download cannot overlap other
    # work, and over 16 steps they weigh 1/16 instead of 1/6
    e2e_steps = max(2, min(args.steps, 16))
    stream.wait_event(e2e_run(2))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    stream.wait_event(e2e_run(e2e_steps))
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(torch, dev, world, e0.elapsed_time(e1))
    return {"value": world * (wl.fwd_bytes + wl.bwd_bytes) / (e2e_ms / e2e_steps * 1e-3) / 1e9,
            "unit": "GB/s",
            "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in ins),
            "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in outs),
            "ms_per_step": e2e_ms / e2e_steps,
            "steps": e2e_steps,
            "path": "pinned host -> C ABI fwd/bwd entry points -> pinned host; every step uploads "
                    "its inputs and downloads its outputs inside the timed region, the next "
                    "step's upload overlapping this step's compute and download; the first "
                    "upload and the last download are not overlapped"}


def _profiled_traffic(workload):
    """DRAM bytes per launch of the roofline kernel at this workload's full
    size, from the committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(workload, {}) or {}
    except Exception:
        return {}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="ln_gelu", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-workload", action="store_true",
                    help="headline workload only (profiling runs)")
    ap.add_argument("--no-strong", action="store_true", help="no strong-scaling legs at N > 1")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows / tokens / ids per GPU (0 = the BASELINE config's; smaller only "
                         "for profiling: other shapes draw other arrays)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs: no host-buffer leg")
    ap.add_argument("--exchange", choices=("push", "pull", "nccl"), default="push",
                    help="embedding at N > 1: the peer-memory exchange (pull or push form) or "
                         "the NCCL all-to-all one")
    ap.add_argument("--e2e-large", action="store_true",
                    help="also run the host-buffer leg of the mlp_block workload")
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
