"""Drop-in for the reference extension bound in euclidean_cuda_advanced.cpp:8-31.

fp64-GEMM / fp32-GEMM variants with fp64 recompute (euclidean_kernels_advanced.cu:225-453).
"""
import torch

import _ops


def pairwise_euclidean_fp64_fp16(P, C, kappa=5.0):
    """Double-precision GEMM with FP16 storage and fallback (:225)."""
    return _ops.run_advanced("fp64_fp16", P, C, kappa, torch.float16, torch.float32)


def pairwise_euclidean_fp64_bf16(P, C, kappa=5.0):
    """Double-precision GEMM with BF16 storage and fallback (:283)."""
    return _ops.run_advanced("fp64_bf16", P, C, kappa, torch.bfloat16, torch.float32)


def pairwise_euclidean_fp64_tf32(P, C, kappa=5.0):
    """FP64 reference with TF32 GEMM acceleration (:341)."""
    return _ops.run_advanced("fp64_tf32", P, C, kappa, torch.float32, torch.float64)


def pairwise_euclidean_fp64_fp32_gemm(P, C, kappa=5.0):
    """FP64 with FP32 GEMM and adaptive correction (:398)."""
    return _ops.run_advanced("fp64_fp32_gemm", P, C, kappa, torch.float64, torch.float64)


def get_last_fallback_count(list_count_tensor):
    """Get count of fallback corrections from last run (euclidean_kernels_advanced.cu:455-460)."""
    return _ops.read_count_i32(list_count_tensor)
