"""D operators whose flagged pairs overflow the recompute list (more than max(n m / 256,
2^16) of them): the tiled recompute re-derives every flag from the stored distance and
recomputes the flagged pairs, bit-identical with the oracle's direct recompute.  The
cancellation regime (offset 1000) flags every pair; a half-offset set flags the offset
rows only, so whole tiles without a flag are skipped.
"""
import numpy as np
import pytest
import torch

import euclidean_cuda_advanced
import euclidean_cuda_mix
import euclidean_cuda_tiled
from _lib import device_check
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def offset_data(n, m, d, seed, half=False):
    rng = np.random.default_rng(seed)
    mu = rng.normal(0, 0.1, (m, d))
    X = mu[rng.integers(0, m, n)] + rng.normal(0, 0.01, (n, d))
    X[: (n // 2 if half else n)] += 1000.0
    C = (1000.0 + mu + rng.normal(0, 0.01, (m, d))).astype(np.float32)
    return X.astype(np.float32), C


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("name", ["bf16_fp64", "bf16_fp32", "fp16_fp32"])
def test_overflow_mix(name, half):
    P, C = offset_data(640, 300, 24, 1, half)
    D, cnt = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{name}_with_stats")(cuda(P), cuda(C), 5.0)
    Do, flag, cnt_o = O.mix(name, P, C, 5.0)
    assert cnt_o > 65536  # the list overflows
    assert cnt == cnt_o
    np.testing.assert_array_equal(D.cpu().numpy()[flag], Do[flag])  # every flagged pair recomputed, bit-exact
    device_check()


@pytest.mark.parametrize("name", ["fp16_fp32", "bf16_fp64"])
def test_overflow_tensorcore(name):
    P, C = offset_data(512, 320, 32, 2)
    D = getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{name}")(cuda(P), cuda(C), 5.0, 32)
    Do, flag, cnt_o, _ = O.tiled(name, P, C, 5.0)
    assert cnt_o > 65536
    np.testing.assert_array_equal(D.cpu().numpy()[flag], Do[flag])
    device_check()


def test_overflow_fp64_form():
    P, C = offset_data(600, 300, 40, 3)
    D = euclidean_cuda_advanced.pairwise_euclidean_fp64_tf32(cuda(P), cuda(C), 1e9)
    Do, cnt_o = O.advanced("fp64_tf32", P, C, 1e9)
    assert cnt_o > 65536
    np.testing.assert_array_equal(D.cpu().numpy(), Do)  # CUDA-core form: every entry bit-exact
    device_check()
