"""The fused argmin's all-flagged route on the GPU, against the oracle.

With K >= 2.5 the reference's cancellation test flags every pair whose norms lie in
the safe range (tests/test_oracle.py::test_all_flagged_route_flags_every_pair pins
that on the oracle), so its D is the direct recompute of every pair.  The engine then
runs the certified argmin in both the screen and the exact mode (a dense sweep of all
pairs when there are at most 512 centers) and reports n * m flagged pairs; a call with a row or center outside the range (NaN, a norm below
2^-13, above 6.0e4 for the fp16 operators) takes the exact epilogue instead.  Either
way the labels (first index of the smallest D value), the minimum distances and the
count must equal the oracle's bit for bit.
"""
import numpy as np
import pytest
import torch

import _ops
from _lib import device_check, lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def oracle_op(name, P, C, kappa):
    if name.startswith(("tiled_", "tensorcore_")):
        D, flag, cnt, _ = O.tiled(name.split("_", 1)[1], P, C, kappa)
    else:
        D, flag, cnt = O.mix(name, P, C, kappa)
    return D, flag, cnt


def check_against_oracle(name, P, C, kappa, exact):
    D, flag, cnt_o = oracle_op(name, P, C, kappa)
    lab, md, cnt = _ops.run_argmin(name, cuda(P), cuda(C), kappa, exact=exact)
    lo = O.argmin_first(D)
    np.testing.assert_array_equal(lab.cpu().numpy(), lo)
    np.testing.assert_array_equal(md.cpu().numpy(), D[np.arange(P.shape[0]), lo])
    assert int(cnt.item()) == cnt_o
    return flag


OPS = ["bf16_fp64", "fp16_fp32", "tf32_fp64", "bf16_fp32", "tiled_bf16_fp32", "tensorcore_fp16_fp64"]


@pytest.mark.parametrize("name", OPS)
@pytest.mark.parametrize("exact", [False, True])
def test_all_flagged_route_matches_oracle(name, exact):
    rng = np.random.default_rng(7)
    n, d, k = 700, 128, 600
    true_c = rng.normal(size=(k // 4, d))
    P = (true_c[rng.integers(0, k // 4, n)] + 0.3 * rng.normal(size=(n, d))).astype(np.float32)
    C = np.concatenate([P[rng.choice(n, k - 8, replace=False)], P[:8]]).astype(np.float32)  # duplicates: first index
    flag = check_against_oracle(name, P, C, 50.0, exact)
    assert flag.all()
    device_check()


@pytest.mark.parametrize("name", OPS)
@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("n,d,k", [(701, 64, 300), (600, 70, 512), (65, 36, 7)])
def test_all_flagged_few_centers(name, exact, n, d, k):
    # few centers, clustered data: the certified bounds decide most rows and the route
    # stays certified (the dense sweep takes over only where they fail, below); labels,
    # distances and count as the oracle's.  d = 70 and 36 are not multiples of 16, 7 and
    # 300 centers leave partial tiles, 512 is the most the dense sweep would take
    rng = np.random.default_rng(n + k)
    true_c = rng.normal(size=(max(2, k // 4), d))
    P = (true_c[rng.integers(0, true_c.shape[0], n)] + 0.3 * rng.normal(size=(n, d))).astype(np.float32)
    C = np.concatenate([P[rng.choice(n, k - 2, replace=False)], P[:2]]).astype(np.float32)  # duplicates
    flag = check_against_oracle(name, P, C, 50.0, exact)
    assert flag.all()
    device_check()


@pytest.mark.parametrize("name", ["bf16_fp64", "bf16_fp32"])
def test_c3_shape_offset_dense_sweep(name):
    # C3's recipe (offset 1000, kappa 5: K = 5.16 flags every pair) on 2048 rows: the
    # norms dwarf the distances, the certified screen decides few rows and the route
    # sweeps every pair densely.  Centers 3 and 5 differ by one fp32 ulp in dimension 7
    # and rows 0..39 sit on center 5 there: center 3 is farther by ulp^2 in fp64, far
    # below the stored distance's fp32 ulp, so the stored values tie and the first
    # index, 3, is the label (a comparison in fp64 would give 5).
    rng = np.random.default_rng(11)
    n, d, k = 2048, 64, 256
    P = (rng.normal(size=(n, d)) + 1000.0).astype(np.float32)
    C = (rng.normal(size=(k, d)) + 1000.0).astype(np.float32)
    C[5] = C[3]
    C[5, 7] = np.nextafter(C[3, 7], np.float32(2000.0))
    P[:40] = C[5] + 0.3 * rng.normal(size=(40, d)).astype(np.float32)
    P[:40, 7] = C[5, 7]
    L = lib()
    for exact in (False, True):
        L.euc_set_kernel_timing(1)
        try:
            flag = check_against_oracle(name, P, C, 5.0, exact)
            assert L.euc_last_kernel_name() == b"dense_argmin_kernel"
        finally:
            L.euc_set_kernel_timing(0)
        assert flag.all()
    lab, _, _ = _ops.run_argmin(name, cuda(P), cuda(C), 5.0)
    assert (lab[:40].cpu().numpy() == 3).all()
    # the certified mode takes the same sweep; its count is the n k direct distances
    L.euc_set_kernel_timing(1)
    try:
        lab, md, cnt = _ops.run_argmin(name, cuda(P), cuda(C), 5.0, exact="certified")
        assert L.euc_last_kernel_name() == b"dense_argmin_kernel"
    finally:
        L.euc_set_kernel_timing(0)
    lo, mo = O.certified_argmin(name, P, C)
    np.testing.assert_array_equal(lab.cpu().numpy(), lo)
    np.testing.assert_array_equal(md.cpu().numpy(), mo)
    assert int(cnt.item()) == n * k and (lo[:40] == 3).all()
    device_check()


@pytest.mark.parametrize("bad", ["nan_row", "tiny_row", "fp16_overflow"])
def test_out_of_range_rows_take_the_exact_path(bad):
    rng = np.random.default_rng(3)
    n, d, k = 300, 64, 200
    P = rng.normal(size=(n, d)).astype(np.float32)
    C = rng.normal(size=(k, d)).astype(np.float32)
    name = "bf16_fp64"
    if bad == "nan_row":
        P[17, 5] = np.nan
    elif bad == "tiny_row":
        P[17] = 1e-6  # norm 6.4e-11 < 2^-13
    else:
        name = "fp16_fp32"
        P[17] *= 40.0  # norm about 1e5 > 6.0e4: fp16 S and norm may overflow
    for exact in (False, True):
        flag = check_against_oracle(name, P, C, 50.0, exact)
        if bad == "nan_row":
            assert not flag[17].any() and flag[np.arange(n) != 17].all()
    device_check()


def test_c5b_shape_reference_kappa():
    # C5b's shape at the reference default kappa = 5: K = 5 (2 * 1024 + 4) 2^-11 = 5.01,
    # every pair flagged; fp16-representable N(0,1) values (512 of 2^21 rows)
    rng = np.random.default_rng(4)
    n, d, k = 512, 1024, 8192
    P = rng.normal(size=(n, d)).astype(np.float16).astype(np.float32)
    C = rng.normal(size=(k, d)).astype(np.float16).astype(np.float32)
    lab, md, cnt = _ops.run_argmin("tensorcore_fp16_fp32", cuda(P), cuda(C), 5.0)
    assert int(cnt.item()) == n * k
    lo, mo = O.certified_argmin("tensorcore_fp16_fp32", P, C)
    np.testing.assert_array_equal(lab.cpu().numpy(), lo)
    np.testing.assert_array_equal(md.cpu().numpy(), mo)
    device_check()
