"""Lloyd iterations on the B200 engine, data-parallel over the GPUs of one node.

The reference ships the pieces (distance operators, update_centers_*) but not the
loop; this is the caller those pieces are meant for (distances -> argmin labels ->
center update), composed without materialising D:

    labels      = euc_argmin(op, X_local, C)            fused GEMM + test + argmin
    stats       = euc_center_stats(X_local, labels)     k x (dim+1) fp64 sums, counts
    all_reduce(stats)                                    one collective per iteration
    C           = euc_center_finalize(stats)            mean; empty -> 0 (reference) or keep

Points are sharded by rows, centers replicated.  With one process per GPU
(torchrun), every rank runs the same sequence on its shard and the single
all-reduce (NCCL over NVLink) makes the centers identical on all ranks.  Cluster
counts are exact integers in fp64, so they are bit-identical for any GPU count.
"""
import ctypes

import torch
import torch.distributed as dist

import _ops
from _lib import check, lib, ptr, stream_of, workspace

EMPTY_POLICY = {"zero": 0, "keep": 1}


class _phase:
    """NVTX range around one phase of an iteration (a no-op without CUDA)."""

    def __init__(self, name):
        self.name = name
        self.on = torch.cuda.is_available()

    def __enter__(self):
        if self.on:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if self.on:
            torch.cuda.nvtx.range_pop()
# labels: the screen (exact wherever the top-two gap exceeds its resolution), the exact
# epilogue, or the certified first index of the smallest direct distance
ASSIGN_MODE = {"fast": False, "exact": True, "certified": "certified"}


class LloydKMeans:
    """One Lloyd iteration per `step`; `op` is the distance operator (e.g. 'bf16_fp32',
    'fp16_fp32', 'double') whose cancellation test and recompute define the labels;
    `mode` ('fast', 'exact', 'certified') is the argmin mode of euc_argmin."""

    def __init__(self, n_clusters, op="bf16_fp32", kappa=5.0, empty="zero", group=None, mode="fast",
                 store_low=False):
        self.k = int(n_clusters)
        self.op = op
        self.kappa = float(kappa)
        self.empty = EMPTY_POLICY[empty]
        self.group = group
        self.mode = ASSIGN_MODE[mode]
        # screen from a low-precision copy of the points made once per fit (prepare), the
        # fp32 points read only for the recompute and the center statistics
        self.store_low = bool(store_low)
        self._ws = None

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    def center_stats(self, X, labels):
        n, d = X.shape
        nbytes = lib().euc_center_stats_workspace_bytes(n, d, self.k)
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != X.device:
            self._ws = workspace(nbytes, X.device)
        stats = torch.empty((self.k, d + 1), dtype=torch.float64, device=X.device)
        check(lib().euc_center_stats(ptr(X), int(X.dtype == torch.float64), ptr(labels),
                                     int(labels.dtype == torch.int64), n, d, self.k, ptr(stats),
                                     ptr(self._ws), self._ws.numel(), stream_of(X)))
        return stats

    def finalize(self, stats, prev):
        d = stats.size(1) - 1
        out = torch.empty((self.k, d), dtype=prev.dtype, device=stats.device)
        check(lib().euc_center_finalize(ptr(stats), d, self.k, ptr(out), int(prev.dtype == torch.float64),
                                        ptr(prev), self.empty, stream_of(stats)))
        return out

    def prepare(self, X):
        """The points' low-precision copy and norms for the screen (store_low); reuse it
        for every iteration over the same X."""
        return _ops.prepare_points(self.op, X)

    def assign(self, X, C, prepared=None):
        """Labels (int32) of the local rows and the flagged-pair count (0-d tensor; the
        number of direct distances taken in the certified mode)."""
        labels, _, cnt = _ops.run_argmin(self.op, X, C, self.kappa, exact=self.mode, labels_dtype=torch.int32,
                                         min_dist=False, prepared=prepared)
        return labels, cnt

    def step(self, X, C, prepared=None):
        """One iteration on the local shard X; returns (new centers, labels int32,
        flagged-pair count of this shard as a 0-d device tensor).  `prepared`: the
        result of prepare(X) (store_low).  Each phase is an NVTX range (lloyd:assign,
        lloyd:center_stats, lloyd:all_reduce, lloyd:finalize)."""
        with _phase("lloyd:assign"):
            labels, cnt = self.assign(X, C, prepared)
        return self._update(X, labels, C), labels, cnt

    def fit(self, X, C0, n_iter, upload_chunks=8):
        """n_iter Lloyd iterations from initial centers C0 (on the GPU); returns (centers,
        labels int32).  X is the local shard, on C0's device or in host memory (pinned
        for an asynchronous copy): a host X is copied in `upload_chunks` row blocks on a
        side stream, and the first iteration assigns each block as soon as it has landed,
        so the copy overlaps the first assignment (a row's label does not depend on the
        other rows, so the labels are those of one assignment of the whole shard)."""
        C = C0.contiguous()
        labels = None
        n_iter = int(n_iter)
        if not X.is_cuda and C.is_cuda:
            X, labels = self._upload_and_assign(X, C, upload_chunks if n_iter > 0 and not self.store_low else 1)
            if n_iter > 0 and not self.store_low:
                C = self._update(X, labels, C)
                n_iter -= 1
        prepared = self.prepare(X) if self.store_low else None
        for _ in range(n_iter):
            C, labels, _ = self.step(X, C, prepared)
        return C, labels

    def _upload_and_assign(self, Xh, C, chunks):
        """Xh (host) copied to C's device in row blocks on a side stream; with chunks > 1
        each block is assigned on the current stream once it has landed."""
        dev = C.device
        n = Xh.size(0)
        Xd = torch.empty(Xh.shape, dtype=Xh.dtype, device=dev)
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(cur)  # Xd is allocated on the current stream
        bounds = [shard_rows(n, c, max(1, chunks)) for c in range(max(1, chunks))]
        events = []
        with torch.cuda.stream(side):
            for lo, hi in bounds:
                if hi > lo:
                    Xd[lo:hi].copy_(Xh[lo:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(side)
                events.append(ev)
        if chunks <= 1:
            cur.wait_event(events[-1])
            return Xd, None
        labels = torch.empty(n, dtype=torch.int32, device=dev)
        with _phase("lloyd:assign"):
            for (lo, hi), ev in zip(bounds, events):
                cur.wait_event(ev)
                if hi > lo:
                    lab, _ = self.assign(Xd[lo:hi], C)
                    labels[lo:hi].copy_(lab)
        return Xd, labels

    def _update(self, X, labels, C):
        """The center update of one iteration from its labels."""
        with _phase("lloyd:center_stats"):
            stats = self.center_stats(X, labels)
        if self._world() > 1:
            with _phase("lloyd:all_reduce"):
                dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=self.group)
        with _phase("lloyd:finalize"):
            return self.finalize(stats, C)


def kmeanspp(X, k, seed=0):
    """k-means++ seeding on X's device (euc_kmeanspp): returns (centers k x dim in X's
    type, row indices int64[k]); deterministic for a given seed.  Single device: with
    sharded rows, seed on one rank and broadcast the centers."""
    X = X.contiguous()
    n, d = X.shape
    if X.dtype not in (torch.float32, torch.float64):
        raise RuntimeError("kmeanspp: X must be float32 or float64")
    idx = torch.empty(int(k), dtype=torch.int64, device=X.device)
    centers = torch.empty((int(k), d), dtype=X.dtype, device=X.device)
    ws = workspace(lib().euc_kmeanspp_workspace_bytes(n, d, int(k)), X.device)
    check(lib().euc_kmeanspp(ptr(X), int(X.dtype == torch.float64), n, d, int(k), int(seed) & (2 ** 64 - 1),
                             ptr(idx), ptr(centers), ptr(ws), ws.numel(), stream_of(X)))
    return centers, idx


def shard_rows(n, rank, world):
    """Contiguous row range [lo, hi) of rank `rank` out of `world`."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)
