"""Drop-in for the reference extension bound in euclidean_cuda_mix.cpp:6-95.

pairwise_euclidean_<low>_<fallback>(P, C, kappa=5.0): low-precision distance with the
cancellation test d <= kappa * gamma * (|p|^2 + |c|^2) and a selective recompute of the
flagged pairs by the direct formula (euclidean_kernels_mix.cu).  `_with_stats` also
returns the number of recomputed pairs.  Each `_argmin` variant (new) returns
(labels int64, min distance fp32, flagged count) without materialising D.
"""
import _ops


def pairwise_euclidean_fp16_fp64(P, C, kappa=5.0):
    """FP16 GEMM with FP64 fallback for unstable entries (euclidean_kernels_mix.cu:515)."""
    return _ops.run_mix("fp16_fp64", P, C, kappa, False)


def pairwise_euclidean_fp16_fp64_with_stats(P, C, kappa=5.0):
    """FP16 GEMM with FP64 fallback for unstable entries; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("fp16_fp64", P, C, kappa, True)


def pairwise_euclidean_fp16_fp64_argmin(P, C, kappa=5.0, exact=False):
    """Fused fp16_fp64 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("fp16_fp64", P, C, kappa, exact)


def pairwise_euclidean_bf16_fp64(P, C, kappa=5.0):
    """BF16 GEMM with FP64 fallback for unstable entries (euclidean_kernels_mix.cu:584)."""
    return _ops.run_mix("bf16_fp64", P, C, kappa, False)


def pairwise_euclidean_bf16_fp64_with_stats(P, C, kappa=5.0):
    """BF16 GEMM with FP64 fallback for unstable entries; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("bf16_fp64", P, C, kappa, True)


def pairwise_euclidean_bf16_fp64_argmin(P, C, kappa=5.0, exact=False):
    """Fused bf16_fp64 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("bf16_fp64", P, C, kappa, exact)


def pairwise_euclidean_tf32_fp64(P, C, kappa=5.0):
    """TF32 GEMM with FP64 fallback for unstable entries (euclidean_kernels_mix.cu:648)."""
    return _ops.run_mix("tf32_fp64", P, C, kappa, False)


def pairwise_euclidean_tf32_fp64_with_stats(P, C, kappa=5.0):
    """TF32 GEMM with FP64 fallback for unstable entries; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("tf32_fp64", P, C, kappa, True)


def pairwise_euclidean_tf32_fp64_argmin(P, C, kappa=5.0, exact=False):
    """Fused tf32_fp64 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("tf32_fp64", P, C, kappa, exact)


def pairwise_euclidean_fp32_fp64(P, C, kappa=5.0):
    """FP32 GEMM with FP64 fallback for unstable entries (euclidean_kernels_mix.cu:918)."""
    return _ops.run_mix("fp32_fp64", P, C, kappa, False)


def pairwise_euclidean_fp32_fp64_with_stats(P, C, kappa=5.0):
    """FP32 GEMM with FP64 fallback for unstable entries; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("fp32_fp64", P, C, kappa, True)


def pairwise_euclidean_fp32_fp64_argmin(P, C, kappa=5.0, exact=False):
    """Fused fp32_fp64 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("fp32_fp64", P, C, kappa, exact)


def pairwise_euclidean_fp16_fp16(P, C, kappa=5.0):
    """FP16 GEMM with FP16 direct formula fallback (euclidean_kernels_mix.cu:1041)."""
    return _ops.run_mix("fp16_fp16", P, C, kappa, False)


def pairwise_euclidean_fp16_fp16_with_stats(P, C, kappa=5.0):
    """FP16 GEMM with FP16 direct formula fallback; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("fp16_fp16", P, C, kappa, True)


def pairwise_euclidean_fp16_fp16_argmin(P, C, kappa=5.0, exact=False):
    """Fused fp16_fp16 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("fp16_fp16", P, C, kappa, exact)


def pairwise_euclidean_fp16_fp32(P, C, kappa=5.0):
    """FP16 GEMM with FP32 direct formula fallback (euclidean_kernels_mix.cu:1163)."""
    return _ops.run_mix("fp16_fp32", P, C, kappa, False)


def pairwise_euclidean_fp16_fp32_with_stats(P, C, kappa=5.0):
    """FP16 GEMM with FP32 direct formula fallback; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("fp16_fp32", P, C, kappa, True)


def pairwise_euclidean_fp16_fp32_argmin(P, C, kappa=5.0, exact=False):
    """Fused fp16_fp32 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("fp16_fp32", P, C, kappa, exact)


def pairwise_euclidean_bf16_bf16(P, C, kappa=5.0):
    """BF16 GEMM with BF16 direct formula fallback (euclidean_kernels_mix.cu:1284)."""
    return _ops.run_mix("bf16_bf16", P, C, kappa, False)


def pairwise_euclidean_bf16_bf16_with_stats(P, C, kappa=5.0):
    """BF16 GEMM with BF16 direct formula fallback; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("bf16_bf16", P, C, kappa, True)


def pairwise_euclidean_bf16_bf16_argmin(P, C, kappa=5.0, exact=False):
    """Fused bf16_bf16 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("bf16_bf16", P, C, kappa, exact)


def pairwise_euclidean_bf16_fp32(P, C, kappa=5.0):
    """BF16 GEMM with FP32 direct formula fallback (euclidean_kernels_mix.cu:1405)."""
    return _ops.run_mix("bf16_fp32", P, C, kappa, False)


def pairwise_euclidean_bf16_fp32_with_stats(P, C, kappa=5.0):
    """BF16 GEMM with FP32 direct formula fallback; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("bf16_fp32", P, C, kappa, True)


def pairwise_euclidean_bf16_fp32_argmin(P, C, kappa=5.0, exact=False):
    """Fused bf16_fp32 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("bf16_fp32", P, C, kappa, exact)


def pairwise_euclidean_fp32_fp32(P, C, kappa=5.0):
    """FP32 GEMM with FP32 direct formula fallback (euclidean_kernels_mix.cu:1525)."""
    return _ops.run_mix("fp32_fp32", P, C, kappa, False)


def pairwise_euclidean_fp32_fp32_with_stats(P, C, kappa=5.0):
    """FP32 GEMM with FP32 direct formula fallback; returns (D, number of recomputed pairs)."""
    return _ops.run_mix("fp32_fp32", P, C, kappa, True)


def pairwise_euclidean_fp32_fp32_argmin(P, C, kappa=5.0, exact=False):
    """Fused fp32_fp32 distance + row argmin: (labels, min distance, flagged count tensor)."""
    return _ops.run_argmin("fp32_fp32", P, C, kappa, exact)


def get_fallback_count_low(list_count_tensor):
    """Get fallback count from last computation (euclidean_kernels_mix.cu:1028-1033)."""
    return _ops.read_count_i32(list_count_tensor)
