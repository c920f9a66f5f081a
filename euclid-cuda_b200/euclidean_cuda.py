"""Drop-in for the reference extension bound in euclidean_cuda.cpp:21-32.

pairwise_euclidean_single / _double (euclidean_kernels.cu:83-152): expanded-form
squared distances D = max(|p|^2 - 2 p.c + |c|^2, 0) in fp32 / fp64, computed by the
B200 engine (libeuclid_b200.so) instead of norms + torch::mm + a form kernel.
"""
import torch

import _ops


def pairwise_euclidean_single(P, C):
    """Pairwise Euclidean distance in single precision (FP32)."""
    return _ops.run_plain("euc_pairwise_single", "single", P, C, torch.float32)


def pairwise_euclidean_double(P, C):
    """Pairwise Euclidean distance in double precision (FP64)."""
    return _ops.run_plain("euc_pairwise_double", "double", P, C, torch.float64)


# fused distance + first-index argmin (no counterpart in the reference: the caller's D.argmin(1))
def pairwise_euclidean_single_argmin(P, C):
    return _ops.run_argmin("single", P, C)


def pairwise_euclidean_double_argmin(P, C):
    return _ops.run_argmin("double", P, C)
