"""One rank of the data-parallel Lloyd loop on CPU tensors over gloo (test helper).

Run by tests/test_dist_gloo.py as `python tests/dist_worker.py OUT.npy` with RANK,
WORLD_SIZE, MASTER_ADDR and MASTER_PORT in the environment.  With LEAVE_AFTER=s the last
rank exits after step s (between steps: nothing of it is in flight); every other rank
must then see its next step raise within the process group's timeout (PG_TIMEOUT
seconds) instead of waiting for good: it writes the error to OUT.npy.err and exits 3.  The host logic under test
is kmeans.LloydKMeans.step and kmeans.shard_rows (sharding, the one all-reduce of the
k x (d+1) statistics, identical finalisation on every rank); the per-rank compute is
the oracle's (assignment by fp64 distance, fp64 center statistics), standing in for
the device kernels that need a B200.
"""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "euclid-cuda_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import kmeans  # noqa: E402
from oracle import oracle as O  # noqa: E402


class HostLloyd(kmeans.LloydKMeans):
    """LloydKMeans with the per-rank compute on the host (oracle)."""

    def assign(self, X, C, prepared=None):
        lab, _, _ = O.dist_argmin_f64(X.numpy(), C.numpy(), threads=1)
        return torch.from_numpy(lab.astype(np.int32)), torch.zeros((), dtype=torch.int64)

    def center_stats(self, X, labels):
        return torch.from_numpy(O.center_stats(X.numpy(), labels.numpy(), self.k))

    def finalize(self, stats, prev):
        s = stats.numpy()
        cnt = s[:, -1:]
        mean = s[:, :-1] / np.maximum(cnt, 1.0)
        keep = prev.numpy().astype(np.float64) if self.empty == 1 else np.zeros_like(mean)
        return torch.from_numpy(np.where(cnt > 0, mean, keep).astype(prev.numpy().dtype))


def data(n, d, k, seed):
    """Blobs on a 2^-8 grid: every fp64 partial sum is exact, so any sharding gives
    bit-identical statistics."""
    rng = np.random.default_rng(seed)
    cen = rng.integers(-64, 64, (k, d)) / 8.0
    X = (cen[rng.integers(0, k, n)] + rng.integers(-32, 32, (n, d)) / 256.0).astype(np.float32)
    C0 = X[rng.choice(n, k, replace=False)].copy()
    return X, C0


def main():
    out = sys.argv[1]
    n, d, k, iters = 3001, 8, 7, 4
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    leave_after = int(os.environ.get("LEAVE_AFTER", "0"))
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=float(os.environ.get("PG_TIMEOUT", "60"))))
    X, C0 = data(n, d, k, seed=12)
    lo, hi = kmeans.shard_rows(n, rank, world)
    km = HostLloyd(k, op="double", empty="keep")
    C = torch.from_numpy(C0)
    Xl = torch.from_numpy(X[lo:hi].copy())
    for step in range(iters):
        if leave_after and rank == world - 1 and step == leave_after:
            os._exit(0)  # this rank leaves between steps
        try:
            C, _, _ = km.step(Xl, C)
        except Exception as e:  # a peer is gone: the collective ended with an error
            if not leave_after:
                raise
            with open(out + ".err", "w") as f:
                f.write(f"step {step}: {type(e).__name__}: {e}")
            os._exit(3)
    np.save(out, C.numpy())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
