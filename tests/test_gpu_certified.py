"""Certified argmin (euc_argmin with EUC_ARGMIN_CERTIFIED) against the oracle on the GPU.

The certified label is the first index of the smallest direct distance over all
centers in the operator's recompute arithmetic, and min_dist is that distance: both are
compared bit for bit with oracle.certified_argmin, on data where the screen separates
almost every row (clusters), where it separates few (Gaussian rows in 256 dimensions,
exact ties between duplicated centers) and none (the cancellation regime at offset
1000), on ragged shapes that reach both the fused and the prepared point path, and at
the C2 size on a sample of rows.
"""
import numpy as np
import pytest
import torch

import _ops
from _lib import device_check
from kmeans import LloydKMeans
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

OPS = ["fp16_fp32", "bf16_fp32", "fp16_fp64", "bf16_fp64", "tf32_fp64", "tiled_fp16_fp32", "tiled_bf16_fp64",
       "tensorcore_fp16_fp64", "tensorcore_bf16_fp32"]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def clustered(n, m, d, seed, spread=1.0, offset=0.0):
    rng = np.random.default_rng(seed)
    C = rng.uniform(-5, 5, (m, d)) + offset
    X = C[rng.integers(0, m, n)] + rng.normal(0, spread, (n, d))
    return X.astype(np.float32), C.astype(np.float32)


def run(op, X, C):
    lab, md, cnt = _ops.run_argmin(op, cuda(X), cuda(C), 5.0, exact="certified")
    return lab.cpu().numpy(), md.cpu().numpy(), int(cnt.item())


def check(op, X, C):
    lab, md, cnt = run(op, X, C)
    lo, mo = O.certified_argmin(op, X, C)
    np.testing.assert_array_equal(lab, lo)
    np.testing.assert_array_equal(md, mo)
    n, m = X.shape[0], C.shape[0]
    assert min(m, 1) * n <= cnt <= n * m
    device_check()
    return cnt


@pytest.mark.parametrize("op", OPS)
def test_certified_clustered(op):
    X, C = clustered(3000, 100, 32, 1)
    cnt = check(op, X, C)
    assert cnt <= 8 * 3000 + 100 * 300  # at most a tenth of the rows evaluated whole


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp64", "tf32_fp64"])
def test_certified_gaussian_high_dim(op):
    rng = np.random.default_rng(2)
    X = rng.normal(size=(700, 256)).astype(np.float32)
    C = rng.normal(size=(520, 256)).astype(np.float32)
    check(op, X, C)


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp32"])
def test_certified_duplicate_centers_take_the_first_index(op):
    X, C = clustered(2000, 64, 16, 3)
    C = np.concatenate([C, C[::-1], C[:5]])  # every center twice or three times, in other groups
    lab, md, _ = run(op, X, C)
    lo, mo = O.certified_argmin(op, X, C)
    np.testing.assert_array_equal(lab, lo)
    np.testing.assert_array_equal(md, mo)
    assert (lab < 64).all()
    device_check()


@pytest.mark.parametrize("op", ["bf16_fp64", "fp16_fp32"])
def test_certified_cancellation_regime(op):
    # offset 1000: the screen's rounding swamps the distances, every row is evaluated whole
    rng = np.random.default_rng(5)
    mu = rng.normal(0, 0.1, (64, 16))
    X = (1000.0 + mu[rng.integers(0, 64, 1500)] + rng.normal(0, 0.01, (1500, 16))).astype(np.float32)
    C = X[rng.choice(1500, 64, replace=False)].copy()
    cnt = check(op, X, C)
    assert cnt == 1500 * 64


@pytest.mark.parametrize("n,m,d", [(1, 1, 1), (5, 7, 3), (130, 9, 17), (257, 300, 4), (129, 1, 8), (1000, 257, 64),
                                   (300, 2000, 12)])
def test_certified_ragged_shapes(n, m, d):
    X, C = clustered(n, m, d, n + m + d, spread=0.3)
    for op in ("fp16_fp32", "bf16_fp64"):
        check(op, X, C)


def test_certified_prepared_and_fused_points_agree():
    # a 16-byte misaligned view of the points takes the prepared path
    X, C = clustered(1024, 200, 32, 7)
    buf = np.zeros((1024 * 32 + 1,), np.float32)
    buf[1:] = X.ravel()
    Xt = cuda(buf)[1:].view(1024, 32)
    assert Xt.data_ptr() % 16 != 0
    lab_p, md_p, _ = _ops.run_argmin("fp16_fp32", Xt, cuda(C), 5.0, exact="certified")
    lab_f, md_f, _ = _ops.run_argmin("fp16_fp32", cuda(X), cuda(C), 5.0, exact="certified")
    np.testing.assert_array_equal(lab_p.cpu().numpy(), lab_f.cpu().numpy())
    np.testing.assert_array_equal(md_p.cpu().numpy(), md_f.cpu().numpy())
    np.testing.assert_array_equal(lab_f.cpu().numpy(), O.certified_argmin("fp16_fp32", X, C)[0])
    device_check()


def test_certified_lloyd_step_labels():
    X, C = clustered(20000, 256, 64, 9, spread=0.5)
    C0 = X[np.random.default_rng(1).choice(20000, 256, replace=False)]
    km = LloydKMeans(256, op="bf16_fp32", kappa=0.1, mode="certified")
    C1, lab, cnt = km.step(cuda(X), cuda(C0))
    lo, _ = O.certified_argmin("bf16_fp32", X, C0)
    np.testing.assert_array_equal(lab.cpu().numpy().astype(np.int64), lo)
    st = O.center_stats(X, lo, 256)
    means = np.where(st[:, 64:] > 0, st[:, :64] / np.maximum(st[:, 64:], 1), 0.0)
    np.testing.assert_allclose(C1.cpu().numpy(), means.astype(np.float32), rtol=1e-6, atol=1e-6)
    device_check()


def test_certified_c2_size_sampled_rows():
    # the C2 configuration (2^20 x 1024 x 128, fp16 GEMM, fp32 recompute), checked on a
    # sample of rows against the oracle
    g = torch.Generator(device=DEV)
    g.manual_seed(11)
    C = torch.randn(1024, 128, device=DEV, generator=g) * 2.0
    X = C[torch.randint(0, 1024, (1 << 20,), device=DEV, generator=g)] + torch.randn(1 << 20, 128, device=DEV,
                                                                                       generator=g)
    lab, md, cnt = _ops.run_argmin("fp16_fp32", X, C, 5.0, exact="certified")
    rows = np.random.default_rng(0).choice(1 << 20, 1500, replace=False)
    Xs = X[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    lo, mo = O.certified_argmin("fp16_fp32", Xs, C.cpu().numpy())
    np.testing.assert_array_equal(lab.cpu().numpy()[rows], lo)
    np.testing.assert_array_equal(md.cpu().numpy()[rows], mo)
    assert int(cnt.item()) < 16 * (1 << 20)  # nearly every row decided by its group of 8
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp16", "bf16_bf16", "single", "fp32_fp32"])
def test_certified_rejects_operators_without_a_screen(op):
    X, C = clustered(64, 8, 8, 0)
    with pytest.raises(RuntimeError, match="certified"):
        _ops.run_argmin(op, cuda(X), cuda(C), 5.0, exact="certified")
