"""D-materialising operators at small dim (the C5a shapes): the one-pass kernel that forms,
tests, recomputes in place and stores D against the oracle, bit for bit (CUDA-core
arithmetic in the same order), with the flagged-pair counts equal.
"""
import numpy as np
import pytest
import torch

import euclidean_cuda
import euclidean_cuda_mix
import euclidean_cuda_uniform
from _lib import device_check
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


# dims 5..8 pad to 8 and 9..16 to 16 (centers held in registers, 64-column slices: 12,
# 68 and 200 columns end in a partial slice), the others to 2 and 4 (centers in shared
# memory)
SHAPES = [(1, 4, 1), (1000, 64, 2), (4097, 64, 3), (777, 64, 4), (2048, 200, 8), (513, 12, 16), (300, 1024, 8),
          (1500, 68, 6), (129, 8, 5), (3000, 64, 7), (2000, 64, 16), (777, 200, 12), (301, 68, 9)]


def data(n, m, d, seed):
    rng = np.random.default_rng(seed)
    P = rng.normal(size=(n, d)).astype(np.float32)
    C = rng.normal(size=(m, d)).astype(np.float32)
    P[: min(n, m) // 2] = C[: min(n, m) // 2]  # exact matches: distance 0, flagged
    if n > 10:
        P[5:9] += 1e-4  # near matches: cancellation
    return P, C


@pytest.mark.parametrize("n,m,d", SHAPES)
def test_thin_mix_fp32(n, m, d):
    P, C = data(n, m, d, n + m + d)
    for name, fn in (("fp32_fp32", euclidean_cuda_mix.pairwise_euclidean_fp32_fp32_with_stats),
                     ("fp32_fp64", euclidean_cuda_mix.pairwise_euclidean_fp32_fp64_with_stats)):
        D, cnt = fn(cuda(P), cuda(C), 5.0)
        Do, flag, cnt_o = O.mix(name, P, C, 5.0)
        np.testing.assert_array_equal(D.cpu().numpy(), Do)
        assert cnt == cnt_o
    device_check()


@pytest.mark.parametrize("n,m,d", SHAPES)
def test_thin_single_and_direct(n, m, d):
    P, C = data(n, m, d, 7 * n + d)
    np.testing.assert_array_equal(euclidean_cuda.pairwise_euclidean_single(cuda(P), cuda(C)).cpu().numpy(),
                                  O.single(P, C))
    U = euclidean_cuda_uniform
    for nm in ("fp32_direct", "tf32_direct", "tf32"):
        np.testing.assert_array_equal(getattr(U, f"pairwise_euclidean_uniform_{nm}")(cuda(P), cuda(C)).cpu().numpy(),
                                      O.uniform(nm, P, C))
    device_check()


def test_thin_two_calls_in_a_row_keep_counts_separate():
    P, C = data(3000, 64, 4, 3)
    _, c1 = euclidean_cuda_mix.pairwise_euclidean_fp32_fp32_with_stats(cuda(P), cuda(C), 5.0)
    _, c2 = euclidean_cuda_mix.pairwise_euclidean_fp32_fp32_with_stats(cuda(P), cuda(C), 5.0)
    assert c1 == c2 == O.mix("fp32_fp32", P, C, 5.0)[2]
    device_check()
