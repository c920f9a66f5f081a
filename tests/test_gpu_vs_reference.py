"""Engine vs the reference's own CUDA extensions on the same GPU and inputs.

The reference modules are the unmodified sources compiled by oracle/build_ref.py
into oracle/_ref/ (skipped if they were not built).  Shapes respect the
reference's hazards: N, M multiples of 32 for its tiled kernel, tile_size=32 and
dim % 16 == 0 for its tensor-core kernel.

Tolerance (both sides use a library/tensor-core GEMM with an unspecified fp32
summation order): |D - D_ref| <= 8 u_low (pp + cc) + 1e-6 |D_ref| elementwise,
flag counts within 0.1 % + 2, labels equal where the reference's top-two gap
exceeds 8 u_low (pp_i + max cc), recomputed pairs (direct formula) bit-identical.
"""
import os
import sys

import numpy as np
import pytest
import torch

import center_kernels
import euclidean_cuda_mix
import euclidean_cuda_tiled
from _lib import device_check
from oracle import oracle as O

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(os.path.join(REF, "ref_euclidean_mix.so")),
                                 reason="reference extensions not built (oracle/build_ref.py)")]


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REF)
    import importlib
    mods = {}
    for key, name in (("mix", "ref_euclidean_mix"), ("tiled", "ref_euclidean_tiled"),
                      ("centers", "ref_center_kernels")):
        try:
            mods[key] = importlib.import_module(name)
        except ImportError:
            pass
    return mods


def _c2_like(n, m, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(n, d, generator=g, device="cuda"), torch.randn(m, d, generator=g, device="cuda"))


@pytest.mark.parametrize("op,kappa", [("fp16_fp32", 5.0), ("fp16_fp64", 5.0), ("bf16_fp32", 0.1),
                                      ("tf32_fp64", 5.0), ("fp32_fp32", 5.0), ("fp16_fp16", 5.0)])
def test_mix_vs_reference(ref, op, kappa):
    P, C = _c2_like(16384, 1024, 128, 1)
    # add close pairs so the cancellation test fires
    P[:2048] = C[torch.arange(2048, device="cuda") % 1024] + 1e-3 * P[:2048]
    Dr, cr = getattr(ref["mix"], f"pairwise_euclidean_{op}_with_stats")(P, C, kappa)
    De, ce = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_with_stats")(P, C, kappa)
    low = O.MIX[op][0]
    u = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -7, "tf32": 2.0 ** -11, "fp32": 2.0 ** -18}[low]
    Pn, Cn = P.cpu().numpy(), C.cpu().numpy()
    pp = torch.from_numpy(O.norms_f32(Pn, O.MIX[op][2]).astype(np.float64)).cuda()
    cc = torch.from_numpy(O.norms_f32(Cn, O.MIX[op][2]).astype(np.float64)).cuda()
    tol = 8 * u * (pp[:, None] + cc[None]) + 1e-6 * Dr.double().abs()
    err = (De.double() - Dr.double()).abs()
    assert bool((err <= tol).all()), float((err - tol).max())
    assert abs(ce - cr) <= 2 + 1e-3 * cr, (ce, cr)
    gap = torch.topk(Dr, 2, dim=1, largest=False).values
    sure = (gap[:, 1] - gap[:, 0]).double() > 8 * u * (pp + cc.max())
    assert bool((De.argmin(1)[sure] == Dr.argmin(1)[sure]).all())
    lab, _, cnt = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")(P, C, kappa)
    assert bool((lab[sure] == Dr.argmin(1)[sure]).all())
    device_check()


@pytest.mark.parametrize("op,kappa", [("fp16_fp64", 5.0), ("bf16_fp32", 0.1), ("fp32_fp64", 5.0)])
def test_tiled_vs_reference(ref, op, kappa):
    P, C = _c2_like(2048, 256, 64, 2)
    P[:256] = C + 1e-3 * P[:256]
    for T in (16, 32):
        Dr, tr, per_r = getattr(ref["tiled"], f"pairwise_euclidean_tiled_{op}_with_stats")(P, C, kappa, T)
        De, te, per_e = getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tiled_{op}_with_stats")(P, C, kappa, T)
        assert len(per_r) == len(per_e)
        u = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8, "fp32": 2.0 ** -18}[op[:4]]
        nrm = (P * P).sum(1).double(), (C * C).sum(1).double()
        tol = 8 * u * (nrm[0][:, None] + nrm[1][None]) + 1e-6 * Dr.double().abs()
        assert bool(((De.double() - Dr.double()).abs() <= tol).all())
        assert abs(te - tr) <= 2 + 1e-3 * tr
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp64"])
def test_tensorcore_vs_reference(ref, op):
    P, C = _c2_like(1024, 512, 128, 3)
    P[:512] = C + 1e-3 * P[:512]
    kappa = 5.0 if op.startswith("fp16") else 0.1
    Dr = getattr(ref["tiled"], f"pairwise_euclidean_tensorcore_{op}")(P, C, kappa, 32)
    De = getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{op}")(P, C, kappa, 32)
    torch.cuda.synchronize()
    u = 2.0 ** -11 if op.startswith("fp16") else 2.0 ** -8
    nrm = (P * P).sum(1).double(), (C * C).sum(1).double()
    tol = 8 * u * (nrm[0][:, None] + nrm[1][None]) + 1e-6 * Dr.double().abs()
    assert bool(((De.double() - Dr.double()).abs() <= tol).all())
    device_check()


def test_centers_vs_reference(ref):
    if "centers" not in ref:
        pytest.skip("reference center_kernels not built")
    g = torch.Generator(device="cuda").manual_seed(4)
    X = torch.randn(200000, 64, generator=g, device="cuda")
    lab = torch.randint(0, 512, (200000,), generator=g, device="cuda")
    lab[lab == 7] = 8
    cr = ref["centers"].update_centers_fp32(X, lab, 512)
    ce = center_kernels.update_centers_fp32(X, lab, 512)
    cnt = torch.bincount(lab, minlength=512).double()
    # the reference sums sequentially in fp32: error <= n_k * 2^-24 * sum|x| / n_k per entry
    tol = (cnt * 2.0 ** -24 * 4).clamp(min=1e-6)[:, None]
    assert bool(((ce.double() - cr.double()).abs() <= tol).all())
    assert bool((ce[7] == 0).all()) and bool((cr[7] == 0).all())
    X64 = X.double()
    torch.testing.assert_close(center_kernels.update_centers_fp64(X64, lab, 512),
                               ref["centers"].update_centers_fp64(X64, lab, 512), rtol=1e-12, atol=1e-13)
    device_check()
