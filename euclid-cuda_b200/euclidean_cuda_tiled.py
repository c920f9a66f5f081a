"""Drop-in for the reference extension bound in euclidean_cuda_tiled.cpp:4-65.

Tiled operators pairwise_euclidean_tiled_<low>_<high>(P, C, kappa, tile_size) with
`_with_stats` twins returning (D, total, per-tile counts), and the tensor-core
operators pairwise_euclidean_tensorcore_<low>_<high>(P, C, kappa, tile_size=64).
Defaults and argument rules are the reference's: tiled accepts tile_size 16 or 32
(<= 0 picks one), so the fp32 variants' default of 64 raises; the tensor-core ops
accept only 32 (their default 64 raises) and need dim % 16 == 0.
"""
import _ops


def pairwise_euclidean_tiled_fp16_fp64(P, C, kappa, tile_size=32):
    """euclidean_kernels_tiled.cu:440."""
    return _ops.run_tiled("fp16_fp64", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_fp16_fp64_with_stats(P, C, kappa, tile_size=32):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("fp16_fp64", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_fp16_fp64_argmin(P, C, kappa, exact=False):
    """Fused tiled_fp16_fp64 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_fp16_fp64", P, C, kappa, exact)


def pairwise_euclidean_tiled_fp16_fp32(P, C, kappa, tile_size=32):
    """euclidean_kernels_tiled.cu:447."""
    return _ops.run_tiled("fp16_fp32", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_fp16_fp32_with_stats(P, C, kappa, tile_size=32):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("fp16_fp32", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_fp16_fp32_argmin(P, C, kappa, exact=False):
    """Fused tiled_fp16_fp32 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_fp16_fp32", P, C, kappa, exact)


def pairwise_euclidean_tiled_bf16_fp64(P, C, kappa, tile_size=32):
    """euclidean_kernels_tiled.cu:470."""
    return _ops.run_tiled("bf16_fp64", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_bf16_fp64_with_stats(P, C, kappa, tile_size=32):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("bf16_fp64", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_bf16_fp64_argmin(P, C, kappa, exact=False):
    """Fused tiled_bf16_fp64 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_bf16_fp64", P, C, kappa, exact)


def pairwise_euclidean_tiled_bf16_fp32(P, C, kappa, tile_size=32):
    """euclidean_kernels_tiled.cu:477."""
    return _ops.run_tiled("bf16_fp32", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_bf16_fp32_with_stats(P, C, kappa, tile_size=32):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("bf16_fp32", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_bf16_fp32_argmin(P, C, kappa, exact=False):
    """Fused tiled_bf16_fp32 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_bf16_fp32", P, C, kappa, exact)


def pairwise_euclidean_tiled_fp32_fp64(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled.cu:500."""
    return _ops.run_tiled("fp32_fp64", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_fp32_fp64_with_stats(P, C, kappa, tile_size=64):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("fp32_fp64", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_fp32_fp64_argmin(P, C, kappa, exact=False):
    """Fused tiled_fp32_fp64 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_fp32_fp64", P, C, kappa, exact)


def pairwise_euclidean_tiled_fp32_fp32(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled.cu:507."""
    return _ops.run_tiled("fp32_fp32", P, C, kappa, tile_size, False)


def pairwise_euclidean_tiled_fp32_fp32_with_stats(P, C, kappa, tile_size=64):
    """Returns (D, total flagged, per-tile flagged counts)."""
    return _ops.run_tiled("fp32_fp32", P, C, kappa, tile_size, True)


def pairwise_euclidean_tiled_fp32_fp32_argmin(P, C, kappa, exact=False):
    """Fused tiled_fp32_fp32 distance + row argmin (new)."""
    return _ops.run_argmin("tiled_fp32_fp32", P, C, kappa, exact)


def pairwise_euclidean_tensorcore_fp16_fp64(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled_tc.cu:274 (tile_size must be 32)."""
    return _ops.run_tensorcore("fp16_fp64", P, C, kappa, tile_size)


def pairwise_euclidean_tensorcore_fp16_fp64_argmin(P, C, kappa, exact=False):
    """Fused tensorcore_fp16_fp64 distance + row argmin (new)."""
    return _ops.run_argmin("tensorcore_fp16_fp64", P, C, kappa, exact)


def pairwise_euclidean_tensorcore_fp16_fp32(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled_tc.cu:281 (tile_size must be 32)."""
    return _ops.run_tensorcore("fp16_fp32", P, C, kappa, tile_size)


def pairwise_euclidean_tensorcore_fp16_fp32_argmin(P, C, kappa, exact=False):
    """Fused tensorcore_fp16_fp32 distance + row argmin (new)."""
    return _ops.run_argmin("tensorcore_fp16_fp32", P, C, kappa, exact)


def pairwise_euclidean_tensorcore_bf16_fp64(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled_tc.cu:288 (tile_size must be 32)."""
    return _ops.run_tensorcore("bf16_fp64", P, C, kappa, tile_size)


def pairwise_euclidean_tensorcore_bf16_fp64_argmin(P, C, kappa, exact=False):
    """Fused tensorcore_bf16_fp64 distance + row argmin (new)."""
    return _ops.run_argmin("tensorcore_bf16_fp64", P, C, kappa, exact)


def pairwise_euclidean_tensorcore_bf16_fp32(P, C, kappa, tile_size=64):
    """euclidean_kernels_tiled_tc.cu:295 (tile_size must be 32)."""
    return _ops.run_tensorcore("bf16_fp32", P, C, kappa, tile_size)


def pairwise_euclidean_tensorcore_bf16_fp32_argmin(P, C, kappa, exact=False):
    """Fused tensorcore_bf16_fp32 distance + row argmin (new)."""
    return _ops.run_argmin("tensorcore_bf16_fp32", P, C, kappa, exact)
