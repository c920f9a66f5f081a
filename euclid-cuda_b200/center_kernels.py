"""Drop-in for the reference extension bound in center_kernels.cu:252-270.

update_centers_fp32 / _fp64(X, labels, n_clusters): per-cluster mean of the rows of
X with each label (labels int64; out-of-range labels ignored; empty clusters -> 0),
computed by one pass over X with fp64 accumulation instead of the reference's
O(K*N) scan (center_kernels.cu:37-95).  The `_with_reinit` twins replace empty
clusters with random points drawn exactly as center_kernels.cu:195-246 does
(torch.randint on X's device, one draw per empty cluster in cluster order).
"""
import torch

import _ops
from _lib import OPS, check, lib, ptr, stream_of, workspace


def _update(X, labels, n_clusters, dtype, want_counts=False):
    _ops.check_input(X, "X")
    _ops.check_input(labels, "labels")
    if X.dtype != dtype:
        raise RuntimeError("X must be float32" if dtype == torch.float32 else "X must be float64")
    if labels.dtype != torch.int64:
        raise RuntimeError("labels must be int64")
    N, D = X.size(0), X.size(1)
    K = int(n_clusters)
    centers = torch.zeros((K, D), dtype=dtype, device=X.device)
    counts = torch.zeros(K, dtype=torch.int64, device=X.device)
    op = "centers_fp32" if dtype == torch.float32 else "centers_fp64"
    ws = workspace(lib().euc_workspace_bytes(OPS[op], N, K, D), X.device)
    fn = lib().euc_update_centers_fp32 if dtype == torch.float32 else lib().euc_update_centers_fp64
    check(fn(ptr(X), ptr(labels), N, D, K, ptr(centers), ptr(counts), ptr(ws), ws.numel(), stream_of(X)))
    return (centers, counts) if want_counts else centers


def update_centers_fp32(X, labels, n_clusters):
    """Update KMeans centers in FP32."""
    return _update(X, labels, n_clusters, torch.float32)


def update_centers_fp64(X, labels, n_clusters):
    """Update KMeans centers in FP64."""
    return _update(X, labels, n_clusters, torch.float64)


def _reinit(X, centers, counts):
    empty = counts == 0
    n_empty = int(empty.sum().item())
    if n_empty > 0:
        idx = torch.nonzero(empty).squeeze(1)
        pts = torch.randint(0, X.size(0), (n_empty,), dtype=torch.long, device=X.device)
        centers[idx] = X[pts]
    return centers


def update_centers_fp32_with_reinit(X, labels, n_clusters):
    """Update KMeans centers in FP32 with empty cluster reinitialization."""
    c, cnt = _update(X, labels, n_clusters, torch.float32, True)
    return _reinit(X, c, cnt)


def update_centers_fp64_with_reinit(X, labels, n_clusters):
    """Update KMeans centers in FP64 with empty cluster reinitialization."""
    c, cnt = _update(X, labels, n_clusters, torch.float64, True)
    return _reinit(X, c, cnt)
