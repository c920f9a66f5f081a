"""Benchmark of the k-means distance engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload lloyd|c2|c5a|configs] [--mode fast|exact|certified]

Workloads
  lloyd (default): full Lloyd iterations, n = 2^24 points x d = 64 (Gaussian blobs:
      4096 true centers U[-5,5]^64, point noise N(0, 0.5^2), seed 3), k = 4096, bf16
      GEMM + fp32 recompute (kappa stated in config), fp32 centers.  One step = one
      iteration of the whole job: every rank's fused distance + argmin on its shard of
      the points, its center statistics, ONE NCCL all-reduce of the k x (d+1) fp64
      statistics, the new centers.  Strong scaling: the 2^24 points are split across
      the ranks.  Unit iter/s.  `e2e` is k-means through the public API
      (kmeans.LloydKMeans.fit, 20 iterations) from pinned host memory: the shard and
      the initial centers copied host->device, the centers and labels copied back,
      all inside the timed region.
      At N = 1 the line also carries
        "c2":      the distance + argmin sweep below, with its own roofline and e2e;
        "configs": C1, C3, C5a and C5b measured one after another (run_configs).
  c2: pairwise distance + argmin, no center update, as the headline.  X is 2^20 x 128
      fp32 N(0,1), C is 1024 x 128 fp32 N(0,1); fp16 tensor-core GEMM (fp32
      accumulate), cancellation test with kappa = 5 (the reference default) and
      selective fp32 recompute (pairwise_euclidean_fp16_fp32 semantics).  Weak scaling:
      every rank owns its own 2^20 rows (seed 1 + rank), no data-path collective.
      Unit GFLOP/s = 2 n k d / time.
  c5a / configs: the extra measurements, one JSON line each.

Timing: W untimed steps, then K steps bracketed by a barrier + synchronize, CUDA
events on the launching stream, max over ranks.  Inputs are resident in HBM and
larger than L2 (X = 4 GiB for lloyd, 512 MiB for c2).

CPU baseline: the same computation in fp64 on the host cores (the oracle's OpenMP C
code), on a bounded row sample, scaled to the workload's row count; run before any
CUDA work, by the same function in both arms.
"""
import argparse
import json
import os
import statistics
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
FIT_ITERS = 20  # C4: full k-means, 20 Lloyd iterations


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


# ------------------------------------------------------------------ CPU baseline
def _blobs_np(rows, cfg):
    """A row sample with the Lloyd workload's distribution (numpy): k true centers
    U[-5,5]^d, points = a random true center + N(0, 0.5^2); the initial centers are k
    further points of the same mixture."""
    import numpy as np
    rng = np.random.default_rng(cfg["seed"])
    k, d = cfg["k"], cfg["d"]
    true_c = rng.uniform(-5, 5, size=(k, d))
    X = true_c[rng.integers(0, k, rows)] + 0.5 * rng.normal(size=(rows, d))
    C = true_c[rng.integers(0, k, k)] + 0.5 * rng.normal(size=(k, d))
    return X, C


def cpu_lloyd_sample(rows=2048):
    """One fp64 Lloyd iteration (distance + argmin + center update, the oracle's OpenMP C
    code on all host threads) on `rows` rows of the Lloyd workload; returns the
    iteration time scaled to the full 2^24 rows (the per-row part scaled by n / rows,
    the reduction of the per-thread tables and the means counted once), the threads
    used and the raw part times."""
    from oracle import oracle as O
    X, C = _blobs_np(rows, LLOYD)
    _, _, used, t_rows, t_fixed = O.lloyd_step_f64(X, C)
    return t_rows * LLOYD["n"] / rows + t_fixed, used, t_rows, t_fixed


def cpu_c2_sample(rows=2048):
    """fp64 distance + argmin on `rows` rows of the C2 workload (N(0,1)); returns the
    time in ms, the threads used and the flop count."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(C2["seed"])
    C = rng.normal(size=(C2["k"], C2["d"]))
    P = rng.normal(size=(rows, C2["d"]))
    t0 = time.perf_counter()
    _, _, used = O.dist_argmin_f64(P, C)
    return (time.perf_counter() - t0) * 1e3, used, 2.0 * rows * C2["k"] * C2["d"]


def cpu_baselines(seconds=10.0):
    """The CPU baseline of both workloads, each on repeated bounded samples for about
    `seconds` (best sample taken): Lloyd in iter/s, C2 in GFLOP/s."""
    from oracle import oracle as O
    rows = 2048
    O.dist_argmin_f64(_blobs_np(64, LLOYD)[0], _blobs_np(64, LLOYD)[1])  # thread pool, page faults
    t0, best, used = time.perf_counter(), None, 1
    reps = 0
    while time.perf_counter() - t0 < seconds or reps == 0:
        it_ms, used, _, _ = cpu_lloyd_sample(rows)
        best = it_ms if best is None else min(best, it_ms)
        reps += 1
    lloyd = {"value": 1e3 / best, "unit": "iter/s", "cores": used, "kind": "port",
             "sample": f"{reps} x one fp64 Lloyd iteration on {rows} of {LLOYD['n']} rows x {LLOYD['k']} centers x "
                       f"{LLOYD['d']} dims (distance + argmin + center sums), per-row time scaled to all rows, "
                       f"best sample"}
    t0, best, reps = time.perf_counter(), None, 0
    while time.perf_counter() - t0 < seconds / 2 or reps == 0:
        ms, used2, flop = cpu_c2_sample(rows)
        best = ms if best is None else min(best, ms)
        reps += 1
    c2 = {"value": flop / (best / 1e3) / 1e9, "unit": "GFLOP/s", "cores": used2, "kind": "port",
          "sample": f"{reps} x {rows} of {C2['n']} rows x {C2['k']} centers x {C2['d']} dims, fp64 distance + argmin, "
                    f"best sample"}
    return lloyd, c2


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
    return f"c4: Lloyd n={n} x d=64, k=4096, bf16 GEMM + fp32 recompute, kappa=0.1, fp32 centers"


def workload_config(workload, n, world):
    """The line's `config`, built by this one function in both arms."""
    cfg = C2 if workload == "c2" else LLOYD
    return {"workload": workload_name(workload, n), "n": n, "k": cfg["k"], "d": cfg["d"], "op": cfg["op"],
            "kappa": cfg["kappa"], "seed": cfg["seed"], "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (X fp32: 4 GiB lloyd, 512 MiB c2 per rank)"}


# ------------------------------------------------------------------ reference arm
def run_reference(a):
    """--impl reference: the reference path's CPU implementation (the oracle port; the
    reference itself is CUDA-only) on the host cores, rank 0 only.  Every step is one
    bounded sample of the workload: for lloyd one fp64 iteration (distance + argmin +
    center update) on 2048 rows, scaled to all rows; for c2 fp64 distance + argmin on
    2048 rows."""
    rank, world, _ = env_rank()
    if rank != 0:
        return
    cfg = C2 if a.workload == "c2" else LLOYD
    rows = 2048
    sample = cpu_c2_sample if a.workload == "c2" else cpu_lloyd_sample
    for _ in range(a.warmup):
        sample(rows)
    times, used, wall = [], 1, time.perf_counter()
    for _ in range(a.steps):
        r = sample(rows)
        times.append(r[0])
        used = r[1]
    wall_ms = (time.perf_counter() - wall) * 1e3 / a.steps
    ms = sum(times) / len(times)
    if a.workload == "c2":
        val, unit = 2.0 * rows * cfg["k"] * cfg["d"] / (ms / 1e3) / 1e9, "GFLOP/s"
        desc = f"{rows} of {cfg['n']} rows x {cfg['k']} centers x {cfg['d']} dims per step, fp64 distance + argmin"
    else:
        val, unit = 1e3 / ms, "iter/s"
        desc = (f"one fp64 Lloyd iteration (distance + argmin + center update) on {rows} of {cfg['n']} rows per "
                f"step, per-row time scaled to all rows ({ms / 1e3:.1f} s per full iteration)")
    # ms_per_step is the wall time of one sampled step; `value` is scaled to the workload
    ref_gpu = reference_gpu(a.workload) if not a.no_reference_gpu else None
    line = {"metric": METRIC, "value": val, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": wall_ms, "higher_is_better": True,
            "scaling": "weak" if a.workload == "c2" else "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": workload_config(a.workload, cfg["n"], world), "sample_rows": rows,
            "cpu_baseline": {"value": val, "unit": unit, "cores": used, "kind": "port", "sample": desc},
            "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    print(json.dumps(line), flush=True)


def reference_gpu(workload):
    """The reference's own CUDA operators on the same workload (informational; the line's
    value is the CPU implementation): its extensions as built from its sources into
    oracle/_ref, one B200.  c2: pairwise_euclidean_fp16_fp32(X, C, 5) + D.argmin(1) (in
    two row halves: its form kernel's grid.y exceeds 65535 at n = 2^20).  lloyd: one
    iteration, pairwise_euclidean_bf16_fp32(kappa 0.1) in 2^18-row chunks (N*M < 2^32)
    + argmin per chunk, then update_centers_fp32 timed on the first 2^20 points and
    scaled linearly in n (its cost is k * n * d).  None when the extensions are absent."""
    ref = os.path.join(REPO, "oracle", "_ref")
    if not os.path.exists(os.path.join(ref, "ref_euclidean_mix.so")):
        return None
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        sys.path.insert(0, ref)
        import ref_center_kernels as rcen
        import ref_euclidean_mix as rmix
        dev = torch.device("cuda", 0)

        def timed(fn, iters):
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / iters

        if workload == "c2":
            g = torch.Generator(device=dev).manual_seed(C2["seed"])
            X = torch.randn(C2["n"], C2["d"], generator=g, device=dev)
            C = torch.randn(C2["k"], C2["d"], generator=g, device=dev)
            half = X.shape[0] // 2
            ms = timed(lambda: torch.cat([rmix.pairwise_euclidean_fp16_fp32(X[:half], C, 5.0).argmin(1),
                                          rmix.pairwise_euclidean_fp16_fp32(X[half:], C, 5.0).argmin(1)]), 5)
            return {"op": "pairwise_euclidean_fp16_fp32 + argmin", "ms_per_step": ms,
                    "value": 2.0 * C2["n"] * C2["k"] * C2["d"] / (ms / 1e3) / 1e9, "unit": "GFLOP/s"}
        n, d, k = LLOYD["n"], LLOYD["d"], LLOYD["k"]
        g = torch.Generator(device=dev).manual_seed(LLOYD["seed"])
        true_c = torch.rand(k, d, generator=g, device=dev) * 10 - 5
        X = true_c[torch.randint(0, k, (n,), generator=g, device=dev)] + 0.5 * torch.randn(n, d, generator=g,
                                                                                           device=dev)
        del true_c
        C = X[torch.randperm(n, generator=g, device=dev)[:k]].contiguous()
        chunk = 1 << 18
        labels = torch.empty(n, dtype=torch.int64, device=dev)

        def dist():
            for r0 in range(0, n, chunk):
                labels[r0:r0 + chunk] = rmix.pairwise_euclidean_bf16_fp32(X[r0:r0 + chunk], C, LLOYD["kappa"]).argmin(1)
        ms_d = timed(dist, 1)
        sub = 1 << 20
        Xs, ls = X[:sub].contiguous(), labels[:sub].contiguous()
        ms_c = timed(lambda: rcen.update_centers_fp32(Xs, ls, k), 1) * (n / sub)
        return {"op": "pairwise_euclidean_bf16_fp32 chunks + argmin + update_centers_fp32",
                "ms_distance": ms_d, "ms_centers_scaled": ms_c, "ms_per_step": ms_d + ms_c,
                "value": 1e3 / (ms_d + ms_c), "unit": "iter/s", "centers_timed_rows": sub}
    except Exception as e:  # informational only: never fail the arm
        return {"error": f"{type(e).__name__}: {e}"}


# ------------------------------------------------------------------ our arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="lloyd", choices=["lloyd", "c2", "c5a", "configs"],
                    help="lloyd: the headline (C4 Lloyd iterations); c2: the distance sweep as the headline; "
                         "c5a, configs: the extra measurements, one line each")
    ap.add_argument("--mode", default="fast", choices=["fast", "exact", "certified"],
                    help="argmin mode of euc_argmin (the headline line uses the default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="reference arm: skip the reference's own CUDA operators (the reference_gpu key)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end legs (profiling runs)")
    ap.add_argument("--no-extras", action="store_true", help="skip the c2 and configs keys of the N = 1 line")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--rows", type=int, default=None,
                    help="override the workload's row count (smaller cases for profiler captures)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":
        return run_reference(a)
    rank, world, local = env_rank()

    # the CPU baseline first, before any CUDA work in this process
    cpu_lloyd = cpu_c2 = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and a.workload in ("lloyd", "c2"):
        cpu_lloyd, cpu_c2 = cpu_baselines(a.cpu_seconds)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    hbm, tc_peak, tc_sus, peak_src = peaks()
    if a.workload == "c5a":
        for r in run_c5a(a, dev, hbm):
            print(json.dumps(r), flush=True)
        return 0
    if a.workload == "configs":
        for r in run_configs(dev, tc_peak, hbm, full=True, tc_sus=tc_sus):
            print(json.dumps(r), flush=True)
        return 0

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

    ctx = dict(a=a, dev=dev, rank=rank, world=world, barrier=barrier, max_over_ranks=max_over_ranks,
               tc_peak=tc_peak, peak_src=peak_src)
    if a.workload == "c2":
        head = bench_c2(ctx, weak=True)
        cpu = cpu_c2
    else:
        head = bench_lloyd(ctx)
        cpu = cpu_lloyd
    extras = {}
    if a.workload == "lloyd" and world == 1 and not a.no_extras and not a.rows:
        torch.cuda.empty_cache()
        extras["c2"] = bench_c2(ctx, weak=False)
        if cpu_c2 is not None:
            extras["c2"]["cpu_baseline"] = cpu_c2
        torch.cuda.empty_cache()
        extras["configs"] = run_configs(dev, tc_peak, hbm, full=False, tc_sus=tc_sus)

    if rank == 0:
        cfg = C2 if a.workload == "c2" else LLOYD
        n = a.rows or cfg["n"]
        line = {"metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
                "scaling": "weak" if a.workload == "c2" else "strong", "vs_baseline": None,
                "dtype": "fp16" if cfg["op"].startswith("fp16") else "bf16", "data": "synthetic",
                "config": workload_config(a.workload, n, world), "n_per_rank": head["n_local"],
                "argmin_mode": a.mode, "roofline": head["roofline"], "cpu_baseline": cpu, "e2e": head.get("e2e"),
                "clocks": head["clocks"], "gpu_launches": head["gpu_launches"],
                "launches_per_step": head["launches_per_step"]}
        for key in ("phases_ms", "per_rank", "store_low", "flagged_last_step"):
            if key in head:
                line[key] = head[key]
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _time_steps(step, steps, st, dev_index, torch):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev_index) as clk:
        e0.record(st)
        for _ in range(steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1), clk.summary()


def _screen_roofline(L, launch, flop, tc_peak, peak_src, workload, rows, reps):
    """Mean CUDA-event duration of the screening kernel (the dominant kernel) over `reps`
    calls of `launch`, as achieved TFLOP/s against the bf16 dense peak."""
    L.euc_set_kernel_timing(1)
    kms = []
    for _ in range(reps):
        launch()
        kms.append(L.euc_last_kernel_ms())
    L.euc_set_kernel_timing(0)
    kname = L.euc_last_kernel_name().decode()
    kernel_ms = statistics.mean(kms)
    achieved = flop / (kernel_ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s", "frac": achieved / tc_peak,
            "traffic": traffic_from_profiles(kname, workload, rows), "kernel": kname, "kernel_ms": kernel_ms,
            "peak_source": f"{peak_src} bf16 dense burst"}


def bench_lloyd(ctx):
    """C4 Lloyd iterations on this rank's shard (one NCCL all-reduce per iteration)."""
    import ctypes

    import torch
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    from kmeans import LloydKMeans, shard_rows
    a, dev, rank, world = ctx["a"], ctx["dev"], ctx["rank"], ctx["world"]
    L = lib()
    st = torch.cuda.current_stream(dev)
    cfg = dict(LLOYD)
    if a.rows:
        cfg["n"] = a.rows
    n, d, k = cfg["n"], cfg["d"], cfg["k"]
    lo, hi = shard_rows(n, rank, world)
    n_local = hi - lo
    # C4 blobs: centers U[-5,5]^64, points = random true center + N(0, 0.5^2).  Every rank
    # generates the same full set (4 GiB) and keeps its shard, so the initial centers (k
    # points sampled without replacement, seed 3) are identical on all ranks.
    gc = torch.Generator(device=dev)
    gc.manual_seed(cfg["seed"])
    true_c = torch.rand(k, d, generator=gc, device=dev) * 10 - 5
    lab = torch.randint(0, k, (n,), generator=gc, device=dev)
    X_full = true_c[lab] + 0.5 * torch.randn(n, d, generator=gc, device=dev)
    del true_c, lab
    C0 = X_full[torch.randperm(n, generator=gc, device=dev)[:k]].contiguous()
    X = X_full[lo:hi].clone().contiguous()
    del X_full
    torch.cuda.empty_cache()
    torch.cuda.synchronize()

    km = LloydKMeans(k, op=cfg["op"], kappa=cfg["kappa"], mode=a.mode)
    state = {"C": C0}

    def step():
        state["C"], _, state["cnt"] = km.step(X, state["C"])

    for _ in range(a.warmup):
        step()
    ctx["barrier"]()
    ms, clk = _time_steps(step, a.steps, st, dev.index, torch)
    ctx["barrier"]()
    launches_per_step = count_launches(step, torch)  # after the timed region
    ctx["barrier"]()
    ms_own = ms
    ms = ctx["max_over_ranks"](ms)
    ms_step = ms / a.steps
    phases = lloyd_phases(km, X, state["C"], st, torch)

    # the same iterations screening from a low-precision copy of the points stored once
    # (LloydKMeans(store_low=True)): the fp32 points are read only for the recompute and
    # the center statistics
    prep = km.prepare(X)
    state_low = {"C": C0}

    def step_low():
        state_low["C"], _, _ = km.step(X, state_low["C"], prep)
    for _ in range(a.warmup):
        step_low()
    ctx["barrier"]()
    ms_low, _ = _time_steps(step_low, a.steps, st, dev.index, torch)
    ctx["barrier"]()
    ms_low = ctx["max_over_ranks"](ms_low) / a.steps
    del prep

    # the screening kernel alone (CUDA events around its launch, same stream)
    op_id = OPS[cfg["op"]]
    labels = torch.empty(n_local, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = workspace(L.euc_argmin_workspace_bytes(op_id, n_local, k, d), dev)
    sp = stream_of(X)
    Cc = state["C"]

    def launch():
        check(L.euc_argmin(op_id, ptr(X), ptr(Cc), n_local, k, d, ctypes.c_float(cfg["kappa"]), MODE_ARG[a.mode],
                           None, ptr(labels), None, ptr(cnt), ptr(ws), ws.numel(), sp))
    roof = _screen_roofline(L, launch, 2.0 * n_local * k * d, ctx["tc_peak"], ctx["peak_src"], "lloyd", n_local,
                            min(a.steps, 20))
    del ws, labels
    # what each rank saw: its own timed step, its phases, its screening kernel and clock
    mine = {"rank": rank, "ms_per_step": ms_own / a.steps, "phases_ms": phases, "screen_ms": roof["kernel_ms"],
            "sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons")}
    per_rank = [mine]
    if world > 1:
        import torch.distributed as dist
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
    e2e = None if a.no_e2e else lloyd_e2e(ctx, km, X, C0)
    return {"value": 1e3 / ms_step, "unit": "iter/s", "ms_per_step": ms_step, "n_local": n_local, "roofline": roof,
            "e2e": e2e, "clocks": clk,
            "gpu_launches": None if launches_per_step is None else launches_per_step * a.steps,
            "launches_per_step": launches_per_step, "phases_ms": phases, "per_rank": per_rank,
            "store_low": {"value": 1e3 / ms_low, "unit": "iter/s", "ms_per_step": ms_low,
                          "note": "X screened from a stored bf16 copy, fp32 read for recompute and centers"},
            "flagged_last_step": int(state["cnt"].item())}


def lloyd_phases(km, X, C, st, torch):
    """CUDA-event time of each phase of one iteration on this rank (after the timed
    region): assignment (all of euc_argmin), center statistics, all-reduce, new centers.
    A device-side sleep (about 2 ms) ahead of the first event lets the host queue every
    launch of the iteration first, so each phase is device time, as in the timed loop, and
    not the host's launch latency of an idle GPU."""
    import torch.distributed as dist
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    torch.cuda.synchronize()
    torch.cuda._sleep(4_000_000)
    ev[0].record(st)
    labels, _ = km.assign(X, C)
    ev[1].record(st)
    stats = km.center_stats(X, labels)
    ev[2].record(st)
    if km._world() > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=km.group)
    ev[3].record(st)
    km.finalize(stats, C)
    ev[4].record(st)
    torch.cuda.synchronize()
    names = ("assign", "center_stats", "all_reduce", "finalize")
    return {nm: ev[i].elapsed_time(ev[i + 1]) for i, nm in enumerate(names)}


def lloyd_e2e(ctx, km, X, C0):
    """k-means through the public API (LloydKMeans.fit, 20 iterations) from pinned host
    memory: every e2e step copies this rank's shard and the initial centers host->device,
    runs the 20 iterations (one all-reduce each) and copies the centers and the labels
    back; iter/s = 20 / (time of one e2e step), max over ranks."""
    import torch
    a, dev = ctx["a"], ctx["dev"]
    st = torch.cuda.current_stream(dev)
    Xh = X.cpu().pin_memory()
    Ch = C0.cpu().pin_memory()
    C_out = torch.empty_like(Ch).pin_memory()
    lab_out = torch.empty(X.shape[0], dtype=torch.int32).pin_memory()

    def fit():
        # the host shard goes to fit itself: its upload overlaps the first assignment
        Cd = Ch.to(dev, non_blocking=True)
        C, labels = km.fit(Xh, Cd, FIT_ITERS)
        C_out.copy_(C, non_blocking=True)
        lab_out.copy_(labels, non_blocking=True)

    fit()
    ctx["barrier"]()
    reps = 2
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(st)
    for _ in range(reps):
        fit()
    f1.record(st)
    torch.cuda.synchronize()
    ctx["barrier"]()
    ms_fit = ctx["max_over_ranks"](f0.elapsed_time(f1)) / reps
    return {"value": FIT_ITERS / (ms_fit / 1e3), "unit": "iter/s", "ms_per_step": ms_fit,
            "iters_per_step": FIT_ITERS,
            "h2d_bytes_per_step": Xh.numel() * 4 + Ch.numel() * 4,
            "d2h_bytes_per_step": C_out.numel() * 4 + lab_out.numel() * 4,
            "api": "kmeans.LloydKMeans.fit (one e2e step = one 20-iteration fit from pinned host buffers; the upload overlaps the first assignment)"}


def bench_c2(ctx, weak):
    """C2 distance + argmin: this rank's own 2^20 rows (weak scaling) when `weak`, else
    the single-GPU measurement carried as the lloyd line's "c2" key."""
    import ctypes

    import torch
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    a, dev, rank = ctx["a"], ctx["dev"], ctx["rank"]
    world = ctx["world"] if weak else 1
    L = lib()
    st = torch.cuda.current_stream(dev)
    cfg = dict(C2)
    if a.rows and weak:
        cfg["n"] = a.rows
    n, d, k = cfg["n"], cfg["d"], cfg["k"]
    g = torch.Generator(device=dev)
    g.manual_seed(cfg["seed"] + (rank if weak else 0))
    X = torch.randn(n, d, generator=g, device=dev, dtype=torch.float32)
    gc = torch.Generator(device=dev)
    gc.manual_seed(cfg["seed"])
    Cm = torch.randn(k, d, generator=gc, device=dev, dtype=torch.float32)
    torch.cuda.synchronize()
    op_id = OPS[cfg["op"]]
    labels = torch.empty(n, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = workspace(L.euc_argmin_workspace_bytes(op_id, n, k, d), dev)
    sp = stream_of(X)
    kappa = ctypes.c_float(cfg["kappa"])

    def step_mode(mode):
        def step():
            check(L.euc_argmin(op_id, ptr(X), ptr(Cm), n, k, d, kappa, MODE_ARG[mode], None, ptr(labels),
                               None, ptr(cnt), ptr(ws), ws.numel(), sp))
        return step

    step = step_mode(a.mode)
    barrier = ctx["barrier"] if weak else torch.cuda.synchronize
    mor = ctx["max_over_ranks"] if weak else (lambda x: x)
    for _ in range(a.warmup):
        step()
    barrier()
    steps = a.steps if weak else max(a.steps, 50)
    ms, clk = _time_steps(step, steps, st, dev.index, torch)
    barrier()
    launches_per_step = count_launches(step, torch)  # after the timed region
    ms_step = mor(ms) / steps
    flop = 2.0 * n * k * d
    out = {"value": flop * world / (ms_step / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": ms_step, "n_local": n,
           "clocks": clk, "gpu_launches": None if launches_per_step is None else launches_per_step * steps,
           "launches_per_step": launches_per_step, "flagged_last_step": int(cnt.item())}
    out["roofline"] = _screen_roofline(L, step, flop, ctx["tc_peak"], ctx["peak_src"], "c2", n, min(steps, 50))
    if not weak:
        out["config"] = {"workload": workload_name("c2", n), "n": n, "k": k, "d": d, "op": cfg["op"],
                         "kappa": cfg["kappa"], "argmin_mode": a.mode}
        # the reference-semantics (exact epilogue) and certified modes beside the default
        for mode in ("exact", "certified"):
            if mode == a.mode:
                continue
            s2 = step_mode(mode)
            for _ in range(3):
                s2()
            torch.cuda.synchronize()
            ms2, _ = _time_steps(s2, 20, st, dev.index, torch)
            out[f"{mode}_mode_ms_per_step"] = ms2 / 20
    del ws
    if not a.no_e2e:
        out["e2e"] = c2_e2e(ctx, a, X, Cm, dev, st, barrier, mor, world)
    return out


def c2_e2e(ctx, a, X, Cm, dev, st, barrier, mor, world):
    """C2 through the public API with pinned host buffers: every step copies X and C
    host->device and the labels device->host inside the timed region."""
    import torch

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
        lab, _, _ = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin(Xd, Cd, C2["kappa"], exact=MODE_PY[a.mode])
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
    e2e_ms = mor(f0.elapsed_time(f1)) / e2e_steps
    return {"value": 2.0 * n_local * k * d * world / (e2e_ms / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": Xh.numel() * 4 + Ch.numel() * 4, "d2h_bytes_per_step": out_h.numel() * 8,
            "api": "euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin"}


# ------------------------------------------------------------------ the other configs
def run_configs(dev, tc_peak, hbm, full, tc_sus=None):
    """The other benchmark configurations, each timed with CUDA events (inputs resident,
    larger than L2 except C1's 12.8 MB, whose step reads them once); returns one dict
    per measurement:
      C1  one fp64 Lloyd iteration, n = 100 000, d = 32, k = 64 (iter/s);
      C3  the cancellation regime, n = 2^22, d = 64, k = 256 at offset 1000, bf16_fp64:
          D with every pair recomputed in fp64, and the fused argmin (exact and
          certified; labels compared);
      C5a D of n = 2^27 rows at d = 2, 4, 8 to k = 64 (fp32_fp32 and uniform_fp32_direct),
          GB/s = 4 (n d + k d + n k) / t against the HBM peak;
      C5b d = 1024, n = 2^21, k = 8192, fp16-representable values, tensorcore_fp16_fp32:
          at kappa = 0.5 (no pair flagged) the D operator and the fused argmin against the
          tensor peak; at the reference default kappa = 5 (every pair flagged) the fused
          argmin, and with `full` the D operator (its direct recompute of all 1.7e10
          pairs takes seconds)."""
    import ctypes

    import torch
    import _ops
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    from kmeans import LloydKMeans
    L = lib()
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    out = []

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

    def emit(name, value, unit, ms, clk, extra):
        r = {"metric": f"{name} {unit}", "value": value, "unit": unit, "n_gpus": 1, "ms_per_step": ms,
             "higher_is_better": True, "data": "synthetic", "clocks": clk}
        r.update(extra)
        out.append(r)

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
                     "op": "bf16_fp64", "kappa": 5.0}})
    lab_d = D.argmin(1)
    del D, ws
    labs = {}
    for mode in ("exact", "certified"):
        ex = True if mode == "exact" else "certified"
        res = {}

        def c3_a():
            res["r"] = _ops.run_argmin("bf16_fp64", X, C, 5.0, exact=ex, labels_dtype=torch.int64, min_dist=False)
        ms, clk = timed(c3_a, 3, 2)
        labs[mode] = res["r"][0]
        emit("C3 argmin", 2.0 * n * k * d / (ms / 1e3) / 1e9, "GFLOP/s", ms, clk,
             {"dtype": "bf16", "count": int(res["r"][2].item()),
              "label_agreement_vs_D_argmin": float((res["r"][0] == lab_d).double().mean().item()),
              "config": {"workload": f"c3: argmin n=4194304 x d=64, k=256, bf16_fp64, {mode}", "op": "bf16_fp64",
                         "kappa": 5.0, "argmin_mode": mode}})
    del X, C, lab_d, labs
    torch.cuda.empty_cache()
    # C5a
    out.extend(run_c5a(None, dev, hbm, steps=10, warmup=3))
    torch.cuda.empty_cache()
    # C5b: launches of 30-40 ms run under the power cap, so the sustained GEMM peak (a
    # seconds-long cuBLAS loop under the same cap) is given beside the burst one
    def c5b_roof(tf):
        r = {"bound": "tensor", "achieved": tf, "peak": tc_peak, "unit": "TFLOP/s", "frac": tf / tc_peak}
        if tc_sus:
            r["peak_sustained"] = tc_sus
            r["frac_sustained"] = tf / tc_sus
        return r

    n, d, k = 1 << 21, 1024, 8192
    X = torch.randn(n, d, generator=g, device=dev).half().float()
    C = torch.randn(k, d, generator=g, device=dev).half().float()
    sp = stream_of(X)
    D = torch.empty((n, k), dtype=torch.float32, device=dev)
    ws = workspace(L.euc_workspace_bytes(OPS["tensorcore_fp16_fp32"], n, k, d), dev)
    flop = 2.0 * n * k * d
    for kappa in ((0.5, 5.0) if full else (0.5,)):
        def c5b_d():
            check(L.euc_tensorcore_fp16_fp32(ptr(X), ptr(C), n, k, d, ctypes.c_float(kappa), 32, ptr(D), ptr(cnt),
                                             ptr(ws), ws.numel(), sp))
        ms, clk = timed(c5b_d, 3 if kappa < 1 else 1, 2 if kappa < 1 else 1)
        tf = flop / (ms / 1e3) / 1e12
        emit("C5b", tf * 1e3, "GFLOP/s", ms, clk,
             {"dtype": "fp16", "recomputed": int(cnt.item()), "recompute_rate": int(cnt.item()) / (n * k),
              "roofline": c5b_roof(tf),
              "config": {"workload": f"c5b: D (64 GiB) of n=2097152 x d=1024 to k=8192, tensorcore_fp16_fp32, "
                                     f"kappa={kappa}", "op": "tensorcore_fp16_fp32", "kappa": kappa}})
    del D, ws
    torch.cuda.empty_cache()
    for kappa in (0.5, 5.0):
        res = {}

        def c5b_a():
            res["r"] = _ops.run_argmin("tensorcore_fp16_fp32", X, C, kappa, exact=False, labels_dtype=torch.int32,
                                       min_dist=False)
        ms, clk = timed(c5b_a, 3, 2)
        tf = flop / (ms / 1e3) / 1e12
        emit("C5b argmin", tf * 1e3, "GFLOP/s", ms, clk,
             {"dtype": "fp16", "count": int(res["r"][2].item()), "recompute_rate": int(res["r"][2].item()) / (n * k),
              "roofline": c5b_roof(tf),
              "config": {"workload": f"c5b: argmin n=2097152 x d=1024, k=8192, tensorcore_fp16_fp32, kappa={kappa}",
                         "op": "tensorcore_fp16_fp32", "kappa": kappa, "argmin_mode": "fast"}})
    del X, C
    torch.cuda.empty_cache()
    return out


def run_c5a(a, dev, hbm, steps=None, warmup=None):
    """C5a: D = distances of n = 2^27 rows to k = 64 centers at d = 2, 4, 8 (fp32), through
    the D-materialising operators pairwise_euclidean_fp32_fp32 (GEMM form, cancellation
    test, direct recompute) and pairwise_euclidean_uniform_fp32_direct.  HBM-bound on the
    D store: GB/s = 4 (n d + k d + n k) / t, one result per operator and d.  D (32 GiB)
    is written once per step, far larger than L2."""
    import ctypes

    import torch
    from _lib import OPS, check, lib, ptr, stream_of, workspace
    L = lib()
    steps = steps or a.steps
    warmup = warmup or a.warmup
    n, k = (a.rows if a is not None and a.rows else (1 << 27)), 64
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    D = torch.empty((n, k), dtype=torch.float32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    out = []
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
            for _ in range(warmup):
                step()
            torch.cuda.synchronize()
            launches = count_launches(step, torch)
            ms, clk = _time_steps(step, steps, torch.cuda.current_stream(dev), dev.index, torch)
            ms /= steps
            gbs = 4.0 * (n * d + k * d + n * k) / (ms / 1e3) / 1e9
            out.append({"metric": "C5a D GB/s = 4(nd+kd+nk)/t", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                        "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
                        "dtype": "fp32", "data": "synthetic",
                        "config": {"workload": f"c5a: D of n={n} x d={d} to k={k}, {op}", "op": op, "d": d,
                                   "l2": f"D ({n * k * 4 / 2 ** 30:.1f} GiB) larger than L2"},
                        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm},
                        "flagged_last_step": int(cnt.item()) if op == "fp32_fp32" else None,
                        "gpu_launches": None if launches is None else launches * steps, "clocks": clk})
        del X, C
    del D
    return out


if __name__ == "__main__":
    main()
