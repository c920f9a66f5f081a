"""Benchmark of the k-means distance engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|lloyd]

Workloads
  c2 (default): pairwise distance + argmin, no center update.  X is 2^20 x 128 fp32
      N(0,1), C is 1024 x 128 fp32 N(0,1); fp16 tensor-core GEMM (fp32 accumulate),
      cancellation test with kappa = 5 (the reference default) and selective fp32
      recompute (pairwise_euclidean_fp16_fp32 semantics).  One step = one pass over
      X.  Weak scaling: every rank owns its own 2^20-row shard (seed 1 + rank); there
      is no data-path collective.  Metric unit GFLOP/s = 2 n k d / time.
  lloyd: full Lloyd iterations, n = 2^24 x 64 (sharded across ranks), k = 4096,
      bf16 GEMM + fp32 recompute (kappa stated in config), fp32 centers, one NCCL
      all-reduce of the k x (d+1) fp64 statistics per iteration.  Unit iter/s.

Timing: W untimed steps, then K steps bracketed by a barrier + synchronize, CUDA
events on the launching stream, max over ranks.  Inputs are resident in HBM and
larger than L2 (X = 512 MiB for c2).  `e2e` repeats the metric through the public
API with pinned host buffers: every step copies X and C host->device and the labels
device->host inside the timed region.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "euclid-cuda_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, REPO)

# euc_argmin's `exact` argument and the Python modules' `exact`, per argmin mode
MODE_ARG = {"fast": 0, "exact": 1, "certified": 2}
MODE_PY = {"fast": False, "exact": True, "certified": "certified"}
METRIC = "distance GFLOP/s vs TC/HBM roofline; Lloyd iters/sec at 1/2/4/8 B200"
C2 = dict(n=1 << 20, d=128, k=1024, op="fp16_fp32", kappa=5.0, seed=1)
LLOYD = dict(n=1 << 24, d=64, k=4096, op="bf16_fp32", kappa=0.1, seed=3)


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained"), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def traffic_from_profiles(kernel, workload, rows):
    """Per-launch DRAM bytes of `kernel` recorded from an ncu capture under profiles/, for
    a launch over `rows` rows (the recorded figure is for the workload's full row count;
    every term of it is proportional to the rows a launch processes)."""
    path = os.path.join(REPO, "profiles", f"{kernel}_{workload}.md")
    full = C2["n"] if workload == "c2" else LLOYD["n"]
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0]) * rows / full
    except OSError:
        pass
    return None


class Clocks:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, index):
        self.index, self.samples, self.reasons = index, [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            names = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                     "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                        r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for nm, bit in names.items():
                            if r & bit:
                                self.reasons.add(nm)
                    except Exception:
                        pass
                    time.sleep(0.01)

            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
        except Exception:
            self._t = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline(k, d, seconds=10.0, rows=4096, seed=1):
    """fp64 distance + argmin (the oracle's host implementation) on a bounded row sample,
    all host threads; returns GFLOP/s and a description of the sample."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    C = rng.normal(size=(k, d))
    P = rng.normal(size=(rows, d))
    O.dist_argmin_f64(P[:64], C)  # warm-up (thread pool, page faults)
    t0 = time.perf_counter()
    reps, used = 0, 1
    while True:
        _, _, used = O.dist_argmin_f64(P, C)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    flops = 2.0 * rows * k * d * reps
    return flops / el / 1e9, used, f"{reps} x {rows} rows x {k} centers x {d} dims, fp64 ({el:.1f} s)"


def count_launches(step, torch):
    """Kernels of this library (namespace euc::) that one step launches, counted from the
    CUDA activity trace of one untimed step."""
    try:
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        return sum(1 for ev in prof.events() if ev.device_type.name == "CUDA" and "euc::" in ev.name)
    except Exception:
        return None


def workload_name(workload, n):
    """The config's workload string, the same on both arms."""
    if workload == "c2":
        return f"c2: distance+argmin n={n} x d=128, k=1024, fp16 GEMM + fp32 recompute, kappa=5"
    return f"c4: Lloyd n={n} x d=64, k=4096, bf16 GEMM + fp32 recompute, kappa=0.1"


def run_reference(a):
    """--impl reference: the reference path's CPU implementation (the oracle port; the
    reference itself is CUDA-only) on the host cores, rank 0 only."""
    rank, world, _ = env_rank()
    if rank != 0:
        return
    cfg = C2 if a.workload == "c2" else LLOYD
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(cfg["seed"])
    rows = 2048
    C = rng.normal(size=(cfg["k"], cfg["d"]))
    P = rng.normal(size=(rows, cfg["d"]))
    for _ in range(a.warmup):
        O.dist_argmin_f64(P, C)
    times = []
    used = 1
    for _ in range(a.steps):
        t0 = time.perf_counter()
        _, _, used = O.dist_argmin_f64(P, C)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    flops = 2.0 * rows * cfg["k"] * cfg["d"] * a.steps
    val = flops / tot / 1e9
    unit = "GFLOP/s"
    if a.workload == "lloyd":
        # one iteration = distances for all n points (sample scaled) + the center update
        val = 1.0 / (tot / a.steps * cfg["n"] / rows)
        unit = "iter/s"
    sample = f"{rows} of {cfg['n']} rows x {cfg['k']} centers x {cfg['d']} dims per step, fp64 distance+argmin"
    line = {"metric": METRIC, "value": val, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": tot / a.steps * 1e3, "higher_is_better": True,
            "scaling": "weak" if a.workload == "c2" else "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": {"workload": workload_name(a.workload, cfg["n"]), **cfg, "sample_rows": rows},
            "cpu_baseline": {"value": val, "unit": unit, "cores": used, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "lloyd", "c5a", "configs"],
                    help="c5a: the D-materialising small-dimension sweep; configs: C1, C3 and C5b (one GPU, "
                         "one line per measurement)")
    ap.add_argument("--mode", default="fast", choices=["fast", "exact", "certified"],
                    help="argmin mode of euc_argmin (the headline line uses the default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg (profiling runs)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--rows", type=int, default=None,
                    help="override the workload's row count (smaller cases for profiler captures)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":
        return run_reference(a)

    import ctypes

    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import _ops
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    hbm, tc_peak, tc_sus, peak_src = peaks()
    if a.workload == "c5a":
        return run_c5a(a, dev, hbm)
    if a.workload == "configs":
        return run_configs(a, dev, tc_peak)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    L = lib()
    st = torch.cuda.current_stream(dev)
    cfg = dict(C2 if a.workload == "c2" else LLOYD)
    if a.rows:
        cfg["n"] = a.rows
    n, d, k = cfg["n"], cfg["d"], cfg["k"]
    if a.workload == "lloyd":
        from kmeans import shard_rows
        lo, hi = shard_rows(n, rank, world)
        n_local = hi - lo
    else:
        n_local = n
    g = torch.Generator(device=dev)
    g.manual_seed(cfg["seed"] + (rank if a.workload == "c2" else 0))
    if a.workload == "c2":
        X = torch.randn(n_local, d, generator=g, device=dev, dtype=torch.float32)
        gc = torch.Generator(device=dev)
        gc.manual_seed(cfg["seed"])
        Cm = torch.randn(k, d, generator=gc, device=dev, dtype=torch.float32)
    else:
        # C4 blobs: centers U[-5,5]^64, points = random true center + N(0, 0.5^2).  Every rank
        # generates the same full set (4 GiB) and keeps its shard, so the initial centers
        # (k points sampled without replacement) are identical on all ranks.
        gc = torch.Generator(device=dev)
        gc.manual_seed(cfg["seed"])
        true_c = torch.rand(k, d, generator=gc, device=dev) * 10 - 5
        lab = torch.randint(0, k, (n,), generator=gc, device=dev)
        X_full = true_c[lab] + 0.5 * torch.randn(n, d, generator=gc, device=dev)
        del true_c, lab
        Cm = X_full[torch.randperm(n, generator=gc, device=dev)[:k]].contiguous()
        X = X_full[lo:hi].clone()
        del X_full
    X = X.contiguous()
    torch.cuda.synchronize()

    op_id = OPS[cfg["op"]]
    labels = torch.empty(n_local, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = workspace(L.euc_argmin_workspace_bytes(op_id, n_local, k, d), dev)
    sp = stream_of(X)
    kappa = ctypes.c_float(cfg["kappa"])

    if a.workload == "c2":
        def step():
            check(L.euc_argmin(op_id, ptr(X), ptr(Cm), n_local, k, d, kappa, MODE_ARG[a.mode], None, ptr(labels),
                               None, ptr(cnt), ptr(ws), ws.numel(), sp))
        work_units = 2.0 * n_local * k * d * world  # flop per step, all ranks
    else:
        from kmeans import LloydKMeans
        km = LloydKMeans(k, op=cfg["op"], kappa=cfg["kappa"], mode=a.mode)
        state = {"C": Cm}

        def step():
            state["C"], _, _ = km.step(X, state["C"])
        work_units = 1.0  # one iteration (of the whole job) per step

    for _ in range(a.warmup):
        step()
    barrier()
    launches_per_step = count_launches(step, torch)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(st)
        for _ in range(a.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    ms_step = ms / a.steps
    value = work_units / (ms_step / 1e3) / (1e9 if a.workload == "c2" else 1.0)
    unit = "GFLOP/s" if a.workload == "c2" else "iter/s"

    # dominant kernel duration (CUDA events around the tcgen05 launch, same stream)
    L.euc_set_kernel_timing(1)
    kms = []
    for _ in range(min(a.steps, 50)):
        if a.workload == "c2":
            step()
        else:
            check(L.euc_argmin(op_id, ptr(X), ptr(Cm), n_local, k, d, kappa, MODE_ARG[a.mode], None, ptr(labels),
                               None, ptr(cnt), ptr(ws), ws.numel(), sp))
        kms.append(L.euc_last_kernel_ms())
    L.euc_set_kernel_timing(0)
    kname = L.euc_last_kernel_name().decode()
    kernel_ms = statistics.mean(kms)
    flop_launch = 2.0 * n_local * k * d
    achieved = flop_launch / (kernel_ms / 1e3) / 1e12
    traffic = traffic_from_profiles(kname, a.workload, n_local) if not a.rows else None
    roof = {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
            "frac": achieved / tc_peak, "traffic": traffic, "kernel": kname, "kernel_ms": kernel_ms,
            "peak_source": f"{peak_src} bf16 dense burst"}

    # end to end through the public API, host buffers
    if a.no_e2e:
        e2e = None
    else:
        e2e = run_e2e(a, cfg, X, Cm, dev, st, barrier, max_over_ranks, world)
    del X

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        v, cores, sample = cpu_baseline(k, d, seconds=a.cpu_seconds)
        if a.workload == "lloyd":
            v = v * 1e9 / (2.0 * n * k * d)
            cu = "iter/s"
        else:
            cu = "GFLOP/s"
        cpu = {"value": v, "unit": cu, "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "weak" if a.workload == "c2" else "strong", "vs_baseline": None,
                "dtype": "fp16" if cfg["op"].startswith("fp16") else "bf16", "data": "synthetic",
                "config": {"workload": workload_name(a.workload, n),
                           "n_per_rank": n_local, "k": k, "d": d, "op": cfg["op"], "kappa": cfg["kappa"],
                           "l2": "inputs larger than L2 (X fp32 >= 512 MiB per rank)",
                           "parallelism": f"dp{world}", "argmin_mode": a.mode},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
                "gpu_launches": None if launches_per_step is None else launches_per_step * a.steps,
                "launches_per_step": launches_per_step, "flagged_last_step": int(cnt.item())}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_configs(a, dev, tc_peak):
    """The other benchmark configurations, each timed with CUDA events (inputs resident,
    larger than L2 except C1's 12.8 MB, whose step reads them once):
      C1  one fp64 Lloyd iteration, n = 100 000, d = 32, k = 64 (iter/s);
      C3  the cancellation regime, n = 2^22, d = 64, k = 256 at offset 1000, bf16_fp64:
          D with every pair recomputed in fp64, and the fused argmin (exact and certified);
      C5b d = 1024, n = 2^21, k = 8192, fp16-representable values: the tensorcore_fp16_fp32
          D (64 GiB) and the fused argmin (TFLOP/s = 2 n k d / t)."""
    import ctypes

    import torch
    import _ops
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    from kmeans import LloydKMeans
    L = lib()
    g = torch.Generator(device=dev)
    g.manual_seed(11)

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(dev.index) as clk:
            e0.record()
            for _ in range(steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps, clk.summary()

    def emit(cfg, value, unit, ms, clk, extra):
        line = {"metric": f"{cfg} {unit}", "value": value, "unit": unit, "n_gpus": 1, "ms_per_step": ms,
                "higher_is_better": True, "data": "synthetic", "clocks": clk}
        line.update(extra)
        print(json.dumps(line), flush=True)

    # C1
    n, d, k = 100_000, 32, 64
    true_c = torch.rand(k, d, generator=g, device=dev, dtype=torch.float64) * 20 - 10
    X = true_c[torch.randint(0, k, (n,), generator=g, device=dev)] + torch.randn(n, d, generator=g, device=dev,
                                                                                 dtype=torch.float64)
    C0 = X[torch.randperm(n, generator=g, device=dev)[:k]].contiguous()
    km = LloydKMeans(k, op="double", kappa=5.0)
    ms, clk = timed(lambda: km.step(X, C0), 20, 5)
    emit("C1", 1e3 / ms, "iter/s", ms, clk, {"dtype": "fp64", "config": {"workload": "c1: Lloyd n=100000 x d=32, "
                                                                          "k=64, fp64", "op": "double"}})
    del X, C0, true_c
    # C3
    n, d, k = 1 << 22, 64, 256
    mu = torch.randn(k, d, generator=g, device=dev) * 0.1
    X = 1000.0 + mu[torch.randint(0, k, (n,), generator=g, device=dev)] + 0.01 * torch.randn(n, d, generator=g,
                                                                                             device=dev)
    C = X[torch.randperm(n, generator=g, device=dev)[:k]].contiguous()
    D = torch.empty((n, k), dtype=torch.float32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = workspace(L.euc_workspace_bytes(OPS["bf16_fp64"], n, k, d), dev)
    sp = stream_of(X)

    def c3_d():
        check(L.euc_mix_bf16_fp64(ptr(X), ptr(C), n, k, d, ctypes.c_float(5.0), ptr(D), ptr(cnt), ptr(ws),
                                  ws.numel(), sp))
    ms, clk = timed(c3_d, 3, 2)
    emit("C3", 2.0 * n * k * d / (ms / 1e3) / 1e9, "GFLOP/s", ms, clk,
         {"dtype": "bf16", "recomputed": int(cnt.item()), "recompute_rate": int(cnt.item()) / (n * k),
          "config": {"workload": "c3: D of n=4194304 x d=64 to k=256 at offset 1000, bf16_fp64 (fp64 recompute)",
                     "op": "bf16_fp64"}})
    del D, ws
    for mode in ("exact", "certified"):
        ex = True if mode == "exact" else "certified"
        out = {}

        def c3_a():
            out["r"] = _ops.run_argmin("bf16_fp64", X, C, 5.0, exact=ex, labels_dtype=torch.int32, min_dist=False)
        ms, clk = timed(c3_a, 3, 2)
        emit("C3 argmin", 2.0 * n * k * d / (ms / 1e3) / 1e9, "GFLOP/s", ms, clk,
             {"dtype": "bf16", "count": int(out["r"][2].item()),
              "config": {"workload": f"c3: argmin n=4194304 x d=64, k=256, bf16_fp64, {mode}", "op": "bf16_fp64",
                         "argmin_mode": mode}})
    del X, C
    # C5b
    n, d, k = 1 << 21, 1024, 8192
    X = torch.randn(n, d, generator=g, device=dev).half().float()
    C = torch.randn(k, d, generator=g, device=dev).half().float()
    D = torch.empty((n, k), dtype=torch.float32, device=dev)
    ws = workspace(L.euc_workspace_bytes(OPS["tensorcore_fp16_fp32"], n, k, d), dev)
    sp = stream_of(X)

    def c5b_d():
        check(L.euc_tensorcore_fp16_fp32(ptr(X), ptr(C), n, k, d, ctypes.c_float(5.0), 32, ptr(D), None, ptr(ws),
                                         ws.numel(), sp))
    ms, clk = timed(c5b_d, 3, 2)
    tf = 2.0 * n * k * d / (ms / 1e3) / 1e12
    emit("C5b", tf * 1e3, "GFLOP/s", ms, clk,
         {"dtype": "fp16", "roofline": {"bound": "tensor", "achieved": tf, "peak": tc_peak, "unit": "TFLOP/s",
                                        "frac": tf / tc_peak},
          "config": {"workload": "c5b: D (64 GiB) of n=2097152 x d=1024 to k=8192, tensorcore_fp16_fp32",
                     "op": "tensorcore_fp16_fp32"}})
    del D, ws
    for mode in ("fast", "exact"):
        out = {}

        def c5b_a():
            out["r"] = _ops.run_argmin("tensorcore_fp16_fp32", X, C, 5.0, exact=(mode == "exact"),
                                       labels_dtype=torch.int32, min_dist=False)
        ms, clk = timed(c5b_a, 3, 2)
        tf = 2.0 * n * k * d / (ms / 1e3) / 1e12
        emit("C5b argmin", tf * 1e3, "GFLOP/s", ms, clk,
             {"dtype": "fp16", "count": int(out["r"][2].item()),
              "roofline": {"bound": "tensor", "achieved": tf, "peak": tc_peak, "unit": "TFLOP/s", "frac": tf / tc_peak},
              "config": {"workload": f"c5b: argmin n=2097152 x d=1024, k=8192, tensorcore_fp16_fp32, {mode}",
                         "op": "tensorcore_fp16_fp32", "argmin_mode": mode}})
    return 0


def run_c5a(a, dev, hbm):
    """C5a: D = distances of n = 2^27 rows to k = 64 centers at d = 2, 4, 8 (fp32), through
    the D-materialising operators pairwise_euclidean_fp32_fp32 (GEMM form, cancellation
    test, direct recompute) and pairwise_euclidean_uniform_fp32_direct.  HBM-bound on the
    D store: GB/s = 4 (n d + k d + n k) / t, one JSON line per operator and d.  D (32 GiB)
    is written once per step, far larger than L2."""
    import ctypes

    import torch
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    L = lib()
    n, k = a.rows or (1 << 27), 64
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    D = torch.empty((n, k), dtype=torch.float32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    for d in (2, 4, 8):
        X = torch.randn(n, d, generator=g, device=dev)
        C = torch.randn(k, d, generator=g, device=dev)
        sp = stream_of(X)
        for op in ("fp32_fp32", "uniform_fp32_direct"):
            if op == "fp32_fp32":
                ws = workspace(L.euc_workspace_bytes(OPS[op], n, k, d), dev)

                def step():
                    check(L.euc_mix_fp32_fp32(ptr(X), ptr(C), n, k, d, ctypes.c_float(5.0), ptr(D), ptr(cnt),
                                              ptr(ws), ws.numel(), sp))
            else:
                def step():
                    check(L.euc_uniform_fp32_direct(ptr(X), ptr(C), n, k, d, ptr(D), sp))
            for _ in range(a.warmup):
                step()
            torch.cuda.synchronize()
            launches = count_launches(step, torch)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with Clocks(dev.index) as clk:
                e0.record()
                for _ in range(a.steps):
                    step()
                e1.record()
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.steps
            gbs = 4.0 * (n * d + k * d + n * k) / (ms / 1e3) / 1e9
            print(json.dumps({"metric": "C5a D GB/s = 4(nd+kd+nk)/t", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                              "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
                              "dtype": "fp32", "data": "synthetic",
                              "config": {"workload": f"c5a: D of n={n} x d={d} to k={k}, {op}", "op": op, "d": d,
                                         "l2": f"D ({n * k * 4 / 2 ** 30:.1f} GiB) larger than L2"},
                              "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                           "frac": gbs / hbm},
                              "flagged_last_step": int(cnt.item()) if op == "fp32_fp32" else None,
                              "gpu_launches": None if launches is None else launches * a.steps,
                              "clocks": clk.summary()}), flush=True)
        del X, C
    return 0


def run_e2e(a, cfg, X, Cm, dev, st, barrier, max_over_ranks, world):
    """The metric through the public API with pinned host buffers: every step copies X and
    C host->device and the labels device->host inside the timed region."""
    import torch

    import _ops
    import euclidean_cuda_mix
    n_local, d = X.shape
    k = Cm.shape[0]
    Xh = X.cpu().pin_memory()
    Ch = Cm.cpu().pin_memory()
    out_h = torch.empty(n_local, dtype=torch.int64).pin_memory()
    e2e_steps = max(3, min(a.steps, 20))

    def e2e_step():
        Xd = Xh.to(dev, non_blocking=True)
        Cd = Ch.to(dev, non_blocking=True)
        lab, _, _ = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin(Xd, Cd, C2["kappa"], exact=MODE_PY[a.mode]) \
            if a.workload == "c2" else _ops.run_argmin(cfg["op"], Xd, Cd, cfg["kappa"], exact=MODE_PY[a.mode],
                                                       min_dist=False)
        out_h.copy_(lab, non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(st)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(st)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / e2e_steps
    flop_step = 2.0 * n_local * k * d * world
    e2e = {"value": flop_step / (e2e_ms / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": Xh.numel() * 4 + Ch.numel() * 4, "d2h_bytes_per_step": out_h.numel() * 8,
           "api": "euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin" if a.workload == "c2"
           else "_ops.run_argmin"}
    if a.workload == "lloyd":
        e2e["note"] = "distance+argmin phase of one iteration through the public API"

    return e2e


if __name__ == "__main__":
    main()
