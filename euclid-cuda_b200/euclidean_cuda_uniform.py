"""Drop-in for the reference extension bound in euclidean_cuda_uniform.cpp:7-41.

Uniform-precision distances without fallback (euclidean_kernels_uniform.cu):
expanded form in fp16 / bf16 / fp32 (D in the input's type) and the direct formula
sum (p - c)^2 in fp16 / bf16 / tf32 / fp32 / fp64.
"""
import torch

import _ops


def pairwise_euclidean_uniform_fp16(P, C):
    """Pure FP16 Euclidean distance (no fallback) (euclidean_kernels_uniform.cu:138)."""
    return _ops.run_plain("euc_uniform_fp16", "uniform_fp16", P, C, torch.float16)


def pairwise_euclidean_uniform_bf16(P, C):
    """Pure BF16 Euclidean distance (no fallback) (euclidean_kernels_uniform.cu:177)."""
    return _ops.run_plain("euc_uniform_bf16", "uniform_bf16", P, C, torch.bfloat16)


def pairwise_euclidean_uniform_tf32(P, C):
    """Pure TF32 Euclidean distance (no fallback) (euclidean_kernels_uniform.cu:215)."""
    return _ops.run_plain("euc_uniform_tf32", "uniform_tf32", P, C, torch.float32)


def pairwise_euclidean_uniform_fp16_direct(P, C):
    """Pure FP16 Euclidean distance using direct formula sum((p-c)^2) (:288)."""
    return _ops.run_plain("euc_uniform_fp16_direct", None, P, C, torch.float16)


def pairwise_euclidean_uniform_bf16_direct(P, C):
    """Pure BF16 Euclidean distance using direct formula (:345)."""
    return _ops.run_plain("euc_uniform_bf16_direct", None, P, C, torch.bfloat16)


def pairwise_euclidean_uniform_tf32_direct(P, C):
    """Pure TF32/FP32 Euclidean distance using direct formula (:398)."""
    return _ops.run_plain("euc_uniform_tf32_direct", None, P, C, torch.float32)


def pairwise_euclidean_uniform_fp32_direct(P, C):
    """Pure FP32 Euclidean distance using direct formula (:453)."""
    return _ops.run_plain("euc_uniform_fp32_direct", None, P, C, torch.float32)


def pairwise_euclidean_uniform_fp64_direct(P, C):
    """Pure FP64 Euclidean distance using direct formula (:507)."""
    return _ops.run_plain("euc_uniform_fp64_direct", None, P, C, torch.float64)
