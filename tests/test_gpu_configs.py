"""The benchmark configurations as parity cases (engine vs oracle on the GPU).

Each case builds its inputs with the configuration's recipe (shapes, value
distributions, operator, kappa) at a row count the oracle finishes in seconds:

* C1  fp64 Lloyd iteration, n = 100 000, d = 32, k = 64 (full size);
* C3  bf16 GEMM -> fp64 recompute at offset 1000, d = 64, k = 256 (8192 of 2^22 rows):
      every pair meets the cancellation test, so the labels come from the recompute;
* C4  one bf16_fp32 Lloyd iteration, d = 64, k = 4096 (16384 of 2^24 rows);
* C5a the D-materialising fp16_fp32 operator at d = 2, 4, 8, k = 64 (65536 of 2^27 rows);
* C5b fp16-representable inputs, d = 1024, k = 8192 (512 of 2^21 rows).

Tolerances as in test_gpu_parity: the CUDA-core fp64 path is bit-exact; tensor-core
D entries within 8 u_low (pp + cc); labels equal wherever the oracle's top-two gap
exceeds the screen's stated bound.
"""
import numpy as np
import pytest
import torch

import euclidean_cuda_mix
from _lib import device_check
from kmeans import LloydKMeans
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_c1_lloyd_fp64():
    rng = np.random.default_rng(0)
    n, d, k = 100_000, 32, 64
    true_c = rng.uniform(-10, 10, (k, d))
    X = true_c[rng.integers(0, k, n)] + rng.normal(0, 1, (n, d))
    C = X[rng.choice(n, k, replace=False)].copy()
    km = LloydKMeans(k, op="double", kappa=5.0)
    C1, lab, _ = km.step(cuda(X), cuda(C))
    lab = lab.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(lab, O.argmin_first(O.double(X, C)))  # fp64 path: same order, bit-exact
    co, cnt = O.update_centers(X, lab, k)
    np.testing.assert_allclose(C1.cpu().numpy(), co, rtol=1e-12, atol=1e-12)
    device_check()


def test_c3_offset_full_recompute():
    rng = np.random.default_rng(2)
    n, d, k = 8192, 64, 256
    mu = rng.normal(0, 0.1, (k, d))
    X = (1000.0 + mu[rng.integers(0, k, n)] + rng.normal(0, 0.01, (n, d))).astype(np.float32)
    C = X[rng.choice(n, k, replace=False)].copy()
    Do, flag, cnt_o = O.mix("bf16_fp64", X, C, 5.0)
    assert cnt_o == n * k  # every pair cancels: the labels are the fp64 recompute's
    for exact in (True, False):
        lab, md, cnt = euclidean_cuda_mix.pairwise_euclidean_bf16_fp64_argmin(cuda(X), cuda(C), 5.0, exact=exact)
        assert int(cnt.item()) == cnt_o
        np.testing.assert_array_equal(lab.cpu().numpy(), O.argmin_first(Do))
        np.testing.assert_array_equal(md.cpu().numpy(), Do[np.arange(n), O.argmin_first(Do)])
    device_check()


def test_c4_lloyd_bf16_fp32():
    rng = np.random.default_rng(3)
    n, d, k = 16384, 64, 4096
    true_c = rng.uniform(-5, 5, (k, d))
    X = (true_c[rng.integers(0, k, n)] + rng.normal(0, 0.5, (n, d))).astype(np.float32)
    C = X[rng.choice(n, k, replace=False)].copy()
    km = LloydKMeans(k, op="bf16_fp32", kappa=0.1)
    C1, lab, cnt = km.step(cuda(X), cuda(C))
    lab = lab.cpu().numpy().astype(np.int64)
    Do, flag, cnt_o = O.mix("bf16_fp32", X, C, 0.1)
    lo = O.argmin_first(Do)
    pp = O.norms_f32(X, "low_bf16").astype(np.float64)
    ccmax = float(O.norms_f32(C, "low_bf16").max())
    sure = O.top2_gap(Do) > 2.0 ** -7 * (pp + ccmax)
    assert sure.mean() > 0.5
    np.testing.assert_array_equal(lab[sure], lo[sure])
    assert abs(int(cnt.item()) - cnt_o) <= 2 + 0.01 * cnt_o
    # the new centers are the means of the engine's own labels
    st = O.center_stats(X, lab, k)
    cntk = st[:, d]
    means = np.where(cntk[:, None] > 0, st[:, :d] / np.maximum(cntk[:, None], 1), 0.0)
    np.testing.assert_allclose(C1.cpu().numpy(), means.astype(np.float32), rtol=1e-6, atol=1e-6)
    device_check()


@pytest.mark.parametrize("d", [2, 4, 8])
def test_c5a_small_dims_D(d):
    rng = np.random.default_rng(4)
    n, k = 65536, 64
    P = rng.normal(size=(n, d)).astype(np.float32)
    C = rng.normal(size=(k, d)).astype(np.float32)
    De, cnt_e = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_with_stats(cuda(P), cuda(C), 5.0)
    De = De.cpu().numpy()
    Do, flag, cnt_o = O.mix("fp16_fp32", P, C, 5.0)
    pp = O.norms_f32(P, "low_fp16").astype(np.float64)
    cc = O.norms_f32(C, "low_fp16").astype(np.float64)
    tol = 8 * 2.0 ** -11 * (pp[:, None] + cc[None, :]) + 1e-6 * np.abs(Do)
    assert (np.abs(De.astype(np.float64) - Do) <= tol).all()
    assert abs(cnt_e - cnt_o) <= 2 + 0.01 * cnt_o
    assert (De == Do).mean() > 0.9
    device_check()


def test_c5b_wide_fp16_inputs():
    rng = np.random.default_rng(4)
    n, d, k = 512, 1024, 8192
    P = rng.normal(size=(n, d)).astype(np.float16).astype(np.float32)  # fp16-representable values
    C = rng.normal(size=(k, d)).astype(np.float16).astype(np.float32)
    Pt, Ct = cuda(P), cuda(C)
    De, cnt_e = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_with_stats(Pt, Ct, 5.0)
    De = De.cpu().numpy()
    Do, flag, cnt_o = O.mix("fp16_fp32", P, C, 5.0)
    pp = O.norms_f32(P, "low_fp16").astype(np.float64)
    cc = O.norms_f32(C, "low_fp16").astype(np.float64)
    tol = 8 * 2.0 ** -11 * (pp[:, None] + cc[None, :]) + 1e-6 * np.abs(Do)
    assert (np.abs(De.astype(np.float64) - Do) <= tol).all()
    assert abs(cnt_e - cnt_o) <= 2 + 0.01 * cnt_o
    lab, md, cnt = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin(Pt, Ct, 5.0)
    lo = O.argmin_first(Do)
    sure = O.top2_gap(Do) > 2.0 ** -10 * (pp + cc.max())
    assert sure.mean() > 0.25
    np.testing.assert_array_equal(lab.cpu().numpy()[sure], lo[sure])
    device_check()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("n,d,k,seed", [(5000, 16, 20, 1), (3000, 64, 64, 7), (1025, 3, 10, 123), (7, 2, 7, 5)])
def test_kmeanspp_matches_oracle(n, d, k, seed, dtype):
    """k-means++ seeding on the device picks the same rows as the oracle's restatement
    (integer weights: the draw does not depend on summation order)."""
    from kmeans import kmeanspp
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, d)).astype(dtype)
    X[: n // 10] = X[0]  # duplicated rows: weight 0 once one of them is chosen
    C, idx = kmeanspp(cuda(X), k, seed=seed)
    io = O.kmeanspp(X, k, seed=seed)
    np.testing.assert_array_equal(idx.cpu().numpy(), io)
    np.testing.assert_array_equal(C.cpu().numpy(), X[io])
    device_check()


def test_kmeanspp_all_rows_equal_draws_uniformly():
    from kmeans import kmeanspp
    X = np.ones((300, 4), np.float32)
    _, idx = kmeanspp(cuda(X), 5, seed=3)
    np.testing.assert_array_equal(idx.cpu().numpy(), O.kmeanspp(X, 5, seed=3))
    device_check()
