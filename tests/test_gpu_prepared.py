"""Prepared points (the points stored in the GEMM's low precision, the
fp32 originals read only for the recompute): euc_argmin_prepared against euc_argmin.

euc_prepare_points writes the rounded copy and the norms that euc_argmin would form
itself on every call (or that the screening kernel forms from the fp32 points), so the
outputs -- labels, minimum distances, flagged counts -- must be identical, in the
screen's mode and in the exact mode, and a Lloyd fit that screens from the stored copy
must reach the same centers and labels as one that reads the fp32 points.
"""
import ctypes

import numpy as np
import pytest
import torch

import _ops
from _lib import OPS, device_check, lib, ptr, workspace
from kmeans import LloydKMeans

pytestmark = pytest.mark.gpu


def data(n, m, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    C = torch.randn(m, d, generator=g, device="cuda")
    P = C[torch.randint(0, m, (n,), generator=g, device="cuda")] + 0.2 * torch.randn(n, d, generator=g, device="cuda")
    return P.contiguous(), C


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp32", "bf16_fp64", "tf32_fp64", "tiled_bf16_fp32",
                                "tensorcore_fp16_fp64"])
@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("n,m,d", [(3001, 517, 96), (1000, 300, 70)])
def test_prepared_matches_direct(op, exact, n, m, d):
    P, C = data(n, m, d, seed=n + d)
    kappa = 0.1 if "bf16" in op else 0.5
    prep = _ops.prepare_points(op, P)
    a = _ops.run_argmin(op, P, C, kappa, exact=exact)
    b = _ops.run_argmin(op, P, C, kappa, exact=exact, prepared=prep)
    device_check()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and int(a[2].item()) == int(b[2].item())


def test_prepared_every_pair_flagged():
    # K >= 2.5: euc_argmin takes the all-flagged route (certified argmin), the prepared
    # call the exact epilogue; both give the reference's labels and distances
    P, C = data(700, 200, 64, seed=5)
    prep = _ops.prepare_points("bf16_fp64", P)
    a = _ops.run_argmin("bf16_fp64", P, C, 50.0)
    b = _ops.run_argmin("bf16_fp64", P, C, 50.0, prepared=prep)
    device_check()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and int(a[2].item()) == int(b[2].item()) == 700 * 200


def test_prepared_rejects_certified_and_non_tensor_core_ops():
    P, C = data(100, 20, 32, seed=1)
    prep = _ops.prepare_points("fp16_fp32", P)
    with pytest.raises(RuntimeError, match="certified"):
        _ops.run_argmin("fp16_fp32", P, C, 5.0, exact="certified", prepared=prep)
    with pytest.raises(RuntimeError, match="tensor-core"):
        _ops.prepare_points("fp32_fp32", P)


def test_lloyd_fit_from_stored_copy():
    rng = np.random.default_rng(3)
    n, d, k = 20000, 64, 512
    true_c = rng.uniform(-5, 5, (k, d))
    X = torch.from_numpy((true_c[rng.integers(0, k, n)] + rng.normal(0, 0.5, (n, d))).astype(np.float32)).cuda()
    C0 = X[torch.from_numpy(rng.choice(n, k, replace=False)).cuda()].contiguous()
    Ca, la = LloydKMeans(k, op="bf16_fp32", kappa=0.1).fit(X, C0, 4)
    Cb, lb = LloydKMeans(k, op="bf16_fp32", kappa=0.1, store_low=True).fit(X, C0, 4)
    device_check()
    assert torch.equal(la, lb)
    assert torch.equal(Ca, Cb)


@pytest.mark.parametrize("store_low", [False, True])
def test_lloyd_fit_from_host_shard(store_low):
    """fit from a pinned host shard (uploaded in row blocks, each assigned as it lands)
    gives the centers and labels of fit from the shard already on the device."""
    rng = np.random.default_rng(4)
    n, d, k = 30011, 64, 300
    true_c = rng.uniform(-5, 5, (k, d))
    Xh = torch.from_numpy((true_c[rng.integers(0, k, n)] + rng.normal(0, 0.5, (n, d))).astype(np.float32))
    Xh = Xh.pin_memory()
    X = Xh.cuda()
    C0 = X[torch.from_numpy(rng.choice(n, k, replace=False)).cuda()].contiguous()
    Ca, la = LloydKMeans(k, op="bf16_fp32", kappa=0.1, store_low=store_low).fit(X, C0, 3)
    Cb, lb = LloydKMeans(k, op="bf16_fp32", kappa=0.1, store_low=store_low).fit(Xh, C0, 3, upload_chunks=7)
    Cc, lc = LloydKMeans(k, op="bf16_fp32", kappa=0.1, store_low=store_low).fit(Xh, C0, 1, upload_chunks=5)
    Cd, ld = LloydKMeans(k, op="bf16_fp32", kappa=0.1, store_low=store_low).fit(X, C0, 1)
    device_check()
    assert torch.equal(la, lb) and torch.equal(Ca, Cb)
    assert torch.equal(lc, ld) and torch.equal(Cc, Cd)


def test_prepared_workspace_is_smaller():
    L = lib()
    op, n, m, d = OPS["bf16_fp32"], 1 << 20, 4096, 64
    full = L.euc_argmin_workspace_bytes(op, n, m, d)
    prep = L.euc_argmin_prepared_workspace_bytes(op, n, m, d)
    assert full - prep >= n * 64 * 2 + n * 4  # the copy (2 bytes a value) and the norms
