"""Failure detection on the GPU, without a GPU fault.

Every pipeline wait of the tensor-core kernels is bounded.  The test shortens the
bound (euc_set_wait_limit_ns) and arms a host-side injection
(euc_test_withhold_arrival): in the next screening launch one epilogue warp of the
first CTA keeps its first accumulator, so that CTA's MMA warp waits on a barrier that
nothing will complete.  After the bound the kernel records the error, stops its
pipeline, lets its copies and MMAs in flight land, frees its tensor memory and returns.
The host reads the status with euc_device_check (EUC_ERR_TIMEOUT), and the next call on
the same context is correct.
"""
import numpy as np
import pytest
import torch

import _ops
from _lib import device_check, lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu
EUC_ERR_TIMEOUT = 5


def test_expired_wait_is_reported_and_the_context_stays_usable():
    rng = np.random.default_rng(9)
    # 1024 centers: 4 center tiles per row tile, so the first CTA's MMA warp comes back to
    # the withheld accumulator (tile 2) and waits for it
    n, d, k = 5000, 128, 1024
    C = rng.normal(size=(k, d)).astype(np.float32)
    P = (C[rng.integers(0, k, n)] + 0.05 * rng.normal(size=(n, d))).astype(np.float32)
    Pt, Ct = torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda()
    L = lib()
    device_check()
    L.euc_set_wait_limit_ns(2_000_000)  # 2 ms
    try:
        L.euc_test_withhold_arrival()
        _ops.run_argmin("fp16_fp32", Pt, Ct, 5.0)  # the launch itself succeeds
        rc = L.euc_device_check()
        assert rc == EUC_ERR_TIMEOUT, L.euc_last_error()
        assert b"bounded device wait expired" in L.euc_last_error()
    finally:
        L.euc_set_wait_limit_ns(0)
    assert L.euc_device_check() == 0  # the status was read and cleared
    # the same context, the next call: correct
    lab, md, cnt = _ops.run_argmin("fp16_fp32", Pt, Ct, 5.0)
    device_check()
    Do, _, cnt_o = O.mix("fp16_fp32", P, C, 5.0)
    lo = O.argmin_first(Do)
    pp = O.norms_f32(P, "low_fp16").astype(np.float64)
    sure = O.top2_gap(Do) > 2.0 ** -10 * (pp + float(O.norms_f32(C, "low_fp16").max()))
    assert sure.mean() > 0.9
    np.testing.assert_array_equal(lab.cpu().numpy()[sure], lo[sure])
    assert abs(int(cnt.item()) - cnt_o) <= 2 + cnt_o // 100


def test_wait_limit_default_restored_and_injection_is_one_shot():
    rng = np.random.default_rng(1)
    P = rng.normal(size=(3000, 64)).astype(np.float32)
    C = rng.normal(size=(512, 64)).astype(np.float32)
    Pt, Ct = torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda()
    lab1, _, _ = _ops.run_argmin("bf16_fp32", Pt, Ct, 0.1)
    lab2, _, _ = _ops.run_argmin("bf16_fp32", Pt, Ct, 0.1)
    device_check()
    assert torch.equal(lab1, lab2)
