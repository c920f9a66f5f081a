"""Time the REFERENCE's own CUDA operators (built by oracle/build_ref.py) on the bench
workloads, on one B200 (the comparison numbers for the engine's own measurements).

    python tests/golden/time_reference_gpu.py [--iters 5]

c2: pairwise_euclidean_fp16_fp32(X, C, kappa=5) + D.argmin(1), X 2^20 x 128, C 1024 x 128
    (the reference has no fused argmin; its callers argmin the materialised D), and the
    same with pairwise_euclidean_tensorcore_fp16_fp32(..., tile_size=32).
c4: one Lloyd iteration, n = 2^24 x 64, k = 4096, bf16 GEMM + fp32 recompute, kappa 0.1:
    the distance op in row chunks of 2^18 (its N*M <= 2^32 limit), argmin per chunk, then
    update_centers_fp32.  The center update scans all N labels per (cluster, dim) and is
    timed on the first 2^20 points and scaled linearly in N (its cost is K*N*D).
Prints one JSON line per measurement.
"""
import argparse
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle", "_ref")


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--only", default="c2,c4")
    a = ap.parse_args()
    sys.path.insert(0, REF)
    import ref_center_kernels as rcen
    import ref_euclidean_mix as rmix
    import ref_euclidean_tiled as rtil
    dev = torch.device("cuda:0")
    if "c2" in a.only:
        g = torch.Generator(device=dev).manual_seed(1)
        X = torch.randn(1 << 20, 128, generator=g, device=dev)
        C = torch.randn(1024, 128, generator=g, device=dev)
        flop = 2.0 * X.shape[0] * C.shape[0] * X.shape[1]
        # the reference's form kernel launches a (M/16, N/16) grid: N = 2^20 gives
        # gridDim.y = 65536 > 65535 (invalid configuration), so it runs in two row halves
        half = X.shape[0] // 2

        def mix_c2():
            return torch.cat([rmix.pairwise_euclidean_fp16_fp32(X[:half], C, 5.0).argmin(1),
                              rmix.pairwise_euclidean_fp16_fp32(X[half:], C, 5.0).argmin(1)])
        ms = timed(mix_c2, a.iters)
        print(json.dumps({"workload": "c2", "op": "pairwise_euclidean_fp16_fp32 + argmin (2 row halves)",
                          "ms": ms, "GFLOP/s": flop / ms / 1e6}), flush=True)
        ms = timed(lambda: rtil.pairwise_euclidean_tensorcore_fp16_fp32(X, C, 5.0, 32).argmin(1), a.iters)
        print(json.dumps({"workload": "c2", "op": "pairwise_euclidean_tensorcore_fp16_fp32 + argmin", "ms": ms,
                          "GFLOP/s": flop / ms / 1e6}), flush=True)
        del X, C
        torch.cuda.empty_cache()
    if "c4" in a.only:
        n, d, k = 1 << 24, 64, 4096
        g = torch.Generator(device=dev).manual_seed(3)
        true_c = torch.rand(k, d, generator=g, device=dev) * 10 - 5
        lab = torch.randint(0, k, (n,), generator=g, device=dev)
        X = true_c[lab] + 0.5 * torch.randn(n, d, generator=g, device=dev)
        del true_c, lab
        C = X[torch.randperm(n, generator=g, device=dev)[:k]].contiguous()
        chunk = 1 << 18

        def dist():
            out = torch.empty(n, dtype=torch.int64, device=dev)
            for r0 in range(0, n, chunk):
                out[r0:r0 + chunk] = rmix.pairwise_euclidean_bf16_fp32(X[r0:r0 + chunk], C, 0.1).argmin(1)
            return out

        labels = dist()
        ms_d = timed(dist, max(1, a.iters // 2))
        sub = 1 << 20
        ms_c_sub = timed(lambda: rcen.update_centers_fp32(X[:sub].contiguous(), labels[:sub].contiguous(), k), 1)
        ms_c = ms_c_sub * (n / sub)
        print(json.dumps({"workload": "c4", "op": "bf16_fp32 chunks + argmin + update_centers_fp32",
                          "ms_distance": ms_d, "ms_centers_scaled": ms_c, "ms_iter": ms_d + ms_c,
                          "iter/s": 1e3 / (ms_d + ms_c), "centers_timed_rows": sub}), flush=True)


if __name__ == "__main__":
    main()
