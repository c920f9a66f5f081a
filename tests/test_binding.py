"""Host-side behaviour of the reference-named modules (no GPU): the public names,
argument names and defaults are the reference's pybind11 bindings, and invalid
arguments raise RuntimeError with the reference's TORCH_CHECK messages."""
import inspect

import pytest
import torch

import center_kernels
import euclidean_cuda
import euclidean_cuda_advanced
import euclidean_cuda_mix
import euclidean_cuda_tiled
import euclidean_cuda_uniform

MIX = ["fp16_fp64", "bf16_fp64", "tf32_fp64", "fp32_fp64", "fp16_fp16", "fp16_fp32", "bf16_bf16", "bf16_fp32",
       "fp32_fp32"]


def sig(f):
    return [(p.name, p.default) for p in inspect.signature(f).parameters.values()]


E = inspect.Parameter.empty


def test_base_names():  # euclidean_cuda.cpp:26-31
    for f in ("pairwise_euclidean_single", "pairwise_euclidean_double"):
        assert sig(getattr(euclidean_cuda, f)) == [("P", E), ("C", E)]


def test_mix_names_and_defaults():  # euclidean_cuda_mix.cpp:13-94
    for op in MIX:
        for suffix in ("", "_with_stats"):
            assert sig(getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}{suffix}")) == \
                [("P", E), ("C", E), ("kappa", 5.0)]
    assert sig(euclidean_cuda_mix.get_fallback_count_low) == [("list_count_tensor", E)]


def test_tiled_names_and_defaults():  # euclidean_cuda_tiled.cpp:12-62
    for op, T in (("fp16_fp64", 32), ("fp16_fp32", 32), ("bf16_fp64", 32), ("bf16_fp32", 32),
                  ("fp32_fp64", 64), ("fp32_fp32", 64)):
        for suffix in ("", "_with_stats"):
            assert sig(getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tiled_{op}{suffix}")) == \
                [("P", E), ("C", E), ("kappa", E), ("tile_size", T)]
    for op in ("fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32"):
        assert sig(getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{op}")) == \
            [("P", E), ("C", E), ("kappa", E), ("tile_size", 64)]


def test_uniform_and_advanced_names():  # euclidean_cuda_uniform.cpp:9-40, euclidean_cuda_advanced.cpp:10-30
    for op in ("fp16", "bf16", "tf32", "fp16_direct", "bf16_direct", "tf32_direct", "fp32_direct", "fp64_direct"):
        assert sig(getattr(euclidean_cuda_uniform, f"pairwise_euclidean_uniform_{op}")) == [("P", E), ("C", E)]
    for op in ("fp64_fp16", "fp64_bf16", "fp64_tf32", "fp64_fp32_gemm"):
        assert sig(getattr(euclidean_cuda_advanced, f"pairwise_euclidean_{op}")) == \
            [("P", E), ("C", E), ("kappa", 5.0)]
    assert sig(euclidean_cuda_advanced.get_last_fallback_count) == [("list_count_tensor", E)]


def test_centers_names():  # center_kernels.cu:255-269
    for f in ("update_centers_fp32", "update_centers_fp64", "update_centers_fp32_with_reinit",
              "update_centers_fp64_with_reinit"):
        assert sig(getattr(center_kernels, f)) == [("X", E), ("labels", E), ("n_clusters", E)]


def test_validation_messages_cpu_tensors():
    P = torch.zeros(4, 3)
    with pytest.raises(RuntimeError, match="P must be a CUDA tensor"):
        euclidean_cuda_mix.pairwise_euclidean_fp16_fp64(P, P)
    with pytest.raises(RuntimeError, match="P must be CUDA tensor"):  # tiled.cu:27 wording
        euclidean_cuda_tiled.pairwise_euclidean_tiled_fp16_fp64(P, P, 5.0)
    with pytest.raises(RuntimeError, match="X must be a CUDA tensor"):
        center_kernels.update_centers_fp32(P, torch.zeros(4, dtype=torch.int64), 2)
    with pytest.raises(TypeError):
        euclidean_cuda.pairwise_euclidean_single(P.numpy(), P)


def test_kmeans_shard_rows():
    from kmeans import shard_rows
    n = 1003
    parts = [shard_rows(n, r, 8) for r in range(8)]
    assert parts[0][0] == 0 and parts[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    assert max(h - l for l, h in parts) - min(h - l for l, h in parts) <= 1
