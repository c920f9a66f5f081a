"""Engine vs oracle on the GPU, through the C ABI (via the reference-named modules).

Tolerances:
* CUDA-core paths (fp32 / fp64 GEMM, direct formulas, the advanced operators) use
  the same sequential fused multiply-add order as the oracle: bit-exact.
* Tensor-core paths: the MMA's fp32 accumulation order differs from any sequential
  sum, so S (and with it a pair's flag) can differ in the last place.  Checked:
  - pairs recomputed by both are bit-identical (same direct formula);
  - every entry |D - D_oracle| <= 8 u_low (pp_i + cc_j) + 1e-6 |D_oracle|;
  - flag counts agree within 2 + 1 % (only pairs at the threshold may flip);
  - >= 90 % of all entries are bit-identical (S rounds to the same fp16/bf16);
  - labels equal wherever the oracle's top-two gap exceeds 8 u_low (pp_i + max cc).
"""
import zlib

import numpy as np
import pytest
import torch

import center_kernels
import euclidean_cuda
import euclidean_cuda_advanced
import euclidean_cuda_mix
import euclidean_cuda_tiled
import euclidean_cuda_uniform
from _lib import device_check
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

SHAPES = [(1, 1, 1), (7, 3, 5), (130, 257, 37), (257, 100, 100), (64, 64, 16), (200, 33, 128), (96, 300, 300)]
U_LOW = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8, "tf32": 2.0 ** -11, "fp32": 2.0 ** -23}


def data(n, m, d, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "gauss":
        return rng.normal(size=(n, d)).astype(np.float32), rng.normal(size=(m, d)).astype(np.float32)
    C = rng.normal(size=(m, d)).astype(np.float32)
    lab = rng.integers(0, m, n)
    P = (C[lab] + rng.normal(0, 0.02, (n, d))).astype(np.float32)
    return P, C


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def norms_for(P, C, mode):
    return O.norms_f32(P, mode).astype(np.float64), O.norms_f32(C, mode).astype(np.float64)


def check_tc_D(De, Do, flag_o, cnt_e, cnt_o, pp, cc, u, min_same=0.0):
    assert De.shape == Do.shape
    tol = 8 * u * (pp[:, None] + cc[None, :]) + 1e-6 * np.abs(Do)
    bad = ~(np.abs(De.astype(np.float64) - Do) <= tol)
    assert not bad.any(), f"{bad.sum()} entries out of tolerance, worst {np.abs(De - Do)[bad].max()}"
    assert abs(cnt_e - cnt_o) <= 2 + 0.01 * cnt_o, (cnt_e, cnt_o)
    # pairs recomputed by the oracle and flagged by the engine too carry the direct value
    same = (De == Do).mean()
    assert same >= min_same, same


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("kind", ["gauss", "blobs"])
@pytest.mark.parametrize("op", sorted(O.MIX))
def test_mix_vs_oracle(op, shape, kind):
    n, m, d = shape
    P, C = data(n, m, d, kind, seed=zlib.crc32(repr((op, shape, kind)).encode()))
    for kappa in (5.0, 0.05):
        De, cnt_e = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_with_stats")(cuda(P), cuda(C), kappa)
        De = De.cpu().numpy()
        Do, flag_o, cnt_o = O.mix(op, P, C, kappa)
        low = O.MIX[op][0]
        if low == "fp32":  # CUDA-core fp32 GEMM: same order as the oracle
            np.testing.assert_array_equal(De, Do)
            assert cnt_e == cnt_o
        else:
            nm = O.MIX[op][2]
            pp, cc = norms_for(P, C, nm)
            # S rounded to fp16/bf16 (as the reference's cuBLAS output) makes most entries bit-identical
            check_tc_D(De, Do, flag_o, cnt_e, cnt_o, pp, cc, 2.0 ** -7 if low == "bf16" else U_LOW[low],
                       min_same=0.9 if O.MIX[op][1] else 0.0)
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp32", "fp16_fp64", "fp16_fp16", "bf16_bf16", "tf32_fp64",
                                "fp32_fp64", "fp32_fp32"])
@pytest.mark.parametrize("shape", [(300, 257, 64), (129, 1000, 37), (5, 1, 3), (200, 600, 300)])
def test_mix_argmin_vs_oracle(op, shape):
    n, m, d = shape
    P, C = data(n, m, d, "blobs", seed=11)
    kappa = 5.0 if not op.startswith("bf16") else 0.05
    lab, md, cnt = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")(cuda(P), cuda(C), kappa)
    lab, md, cnt = lab.cpu().numpy(), md.cpu().numpy(), int(cnt.item())
    Do, flag_o, cnt_o = O.mix(op, P, C, kappa)
    lo = O.argmin_first(Do)
    low = O.MIX[op][0]
    if low == "fp32":
        np.testing.assert_array_equal(lab, lo)
        np.testing.assert_array_equal(md, Do[np.arange(n), lo])
        assert cnt == cnt_o
        return
    pp, cc = norms_for(P, C, O.MIX[op][2])
    u = 2.0 ** -7 if low == "bf16" else U_LOW[low]
    gap = O.top2_gap(Do) if m > 1 else np.full(n, np.inf)
    sure = gap > 8 * u * (pp + cc.max())
    assert sure.mean() > 0.5
    np.testing.assert_array_equal(lab[sure], lo[sure])
    # the reported minimum is the distance at the label, within the GEMM tolerance
    assert (np.abs(md - Do[np.arange(n), lab]) <= 8 * u * (pp + cc[lab]) + 1e-6 * np.abs(md)).all()
    assert abs(cnt - cnt_o) <= 2 + 0.01 * cnt_o
    device_check()


def test_argmin_matches_engine_D():
    """Exact fused argmin == argmin of the engine's own D (same kernels, same S); the
    fast screen agrees wherever the top-two gap exceeds its stated bound."""
    P, C = data(1000, 300, 72, "blobs", seed=3)
    Pt, Ct = cuda(P), cuda(C)
    for op in ("fp16_fp32", "bf16_fp64", "tf32_fp64", "fp16_fp16"):
        kappa = 5.0 if op != "bf16_fp64" else 0.05
        D = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}")(Pt, Ct, kappa)
        lab, md, c1 = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")(Pt, Ct, kappa, exact=True)
        torch.testing.assert_close(lab, D.argmin(1), rtol=0, atol=0)
        torch.testing.assert_close(md, D.min(1).values, rtol=0, atol=0)
        labf, mdf, c2 = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")(Pt, Ct, kappa)
        assert int(c1.item()) == int(c2.item())  # same accumulators, same cancellation test
        u = 2.0 ** -7 if op.startswith("bf16") else 2.0 ** -10
        nrm = O.norms_f32(P, O.MIX[op][2]).astype(np.float64)
        bound = torch.from_numpy(u * (nrm + O.norms_f32(C, O.MIX[op][2]).max())).to(DEV)
        top2 = torch.topk(D, 2, dim=1, largest=False).values.double()
        sure = (top2[:, 1] - top2[:, 0]) > bound
        assert float(sure.double().mean()) > 0.9
        assert bool((labf[sure] == lab[sure]).all())
        assert bool(((mdf.double() - md.double()).abs() <= bound + 1e-5 * md.double()).all())
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp32", "fp16_fp64"])
def test_fast_argmin_c2_like(op):
    """Fast screen at a C2-like shape (1024 centers, d=128) against the exact epilogue."""
    g = torch.Generator(device=DEV).manual_seed(7)
    P = torch.randn(65536, 128, generator=g, device=DEV)
    C = torch.randn(1024, 128, generator=g, device=DEV)
    P[:4096] = C[torch.arange(4096, device=DEV) % 1024] + 1e-3 * P[:4096]  # near-duplicates -> flagged pairs
    kappa = 5.0 if op.startswith("fp16") else 0.1
    fn = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")
    le, me, ce = fn(P, C, kappa, exact=True)
    lf, mf, cf = fn(P, C, kappa)
    assert int(ce.item()) == int(cf.item()) and int(cf.item()) >= 4096
    # labels agree wherever the row's top-two gap (of the exact D) exceeds the fast screen's bound
    D = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}")(P, C, kappa)
    top2 = torch.topk(D, 2, dim=1, largest=False).values.double()
    nm = "low_fp16" if op.startswith("fp16") else "low_bf16"
    pp = torch.from_numpy(O.norms_f32(P.cpu().numpy(), nm).astype(np.float64)).to(DEV)
    ccmax = float(O.norms_f32(C.cpu().numpy(), nm).max())
    u = 2.0 ** -10 if op.startswith("fp16") else 2.0 ** -7
    sure = (top2[:, 1] - top2[:, 0]) > u * (pp + ccmax)
    assert float(sure.double().mean()) > (0.9 if op.startswith("fp16") else 0.6)
    assert bool((lf[sure] == le[sure]).all())
    assert bool((lf[:4096] == torch.arange(4096, device=DEV) % 1024).all())
    device_check()


def test_flag_list_overflow():
    """kappa so large that every pair is flagged: the compact list (capacity 2^16 here)
    overflows; argmin folds the excess in place, D mode falls back to a dense sweep."""
    P, C = data(300, 400, 24, "gauss", seed=21)  # 120000 pairs > 65536
    Do, flag_o, cnt_o = O.mix("fp16_fp32", P, C, 1.0e6)
    assert cnt_o == 300 * 400
    D, cnt = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_with_stats(cuda(P), cuda(C), 1.0e6)
    assert cnt == cnt_o
    np.testing.assert_array_equal(D.cpu().numpy(), Do)  # every value is the direct fp32 formula
    for exact in (True, False):
        lab, md, c = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin(cuda(P), cuda(C), 1.0e6, exact=exact)
        np.testing.assert_array_equal(lab.cpu().numpy(), O.argmin_first(Do))
        np.testing.assert_array_equal(md.cpu().numpy(), Do.min(1))
        assert int(c.item()) == cnt_o
    device_check()


def test_fast_argmin_region_overflow_redo():
    """Cancellation-heavy input (every pair flagged, every chunk a candidate): the fast
    path's candidate list overflows its per-CTA regions and the overflowing rows are
    evaluated whole by the redo pass.  All distances are then direct fp32 values, so
    labels, minima and counts equal the exact path's and the oracle's."""
    rng = np.random.default_rng(5)
    n, m, d = 4096, 2048, 64
    C = (1000.0 + rng.normal(0, 0.1, (m, d))).astype(np.float32)
    P = (C[rng.integers(0, m, n)] + rng.normal(0, 0.01, (n, d))).astype(np.float32)
    Pt, Ct = cuda(P), cuda(C)
    fn = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin
    le, me, ce = fn(Pt, Ct, 5.0, exact=True)
    lf, mf, cf = fn(Pt, Ct, 5.0)
    assert int(ce.item()) == n * m and int(cf.item()) == n * m
    torch.testing.assert_close(lf, le, rtol=0, atol=0)
    torch.testing.assert_close(mf, me, rtol=0, atol=0)
    Do, _, cnt_o = O.mix("fp16_fp32", P, C, 5.0)
    assert cnt_o == n * m
    np.testing.assert_array_equal(lf.cpu().numpy(), O.argmin_first(Do))
    device_check()


@pytest.mark.parametrize("op,variants", [("fp16_fp16", ("fp16", "fp16_fused")), ("bf16_bf16", ("bf16", "bf16_fused"))])
def test_half_arith_recompute_rounding(op, variants):
    """With every pair flagged, D is entirely the half/bf16-arithmetic recompute; it must
    equal one of the two rounding sequences bit for bit (the test reports which)."""
    P, C = data(64, 48, 40, "gauss", seed=12)
    D = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}")(cuda(P), cuda(C), 1.0e6).cpu().numpy()
    ii, jj = np.nonzero(np.ones((64, 48), bool))
    match = {}
    for v in variants:
        ref = O.direct_pairs(v, P, C, ii, jj).astype(np.float32).reshape(64, 48)
        match[v] = float((ref == D).mean())
    print(op, match)
    assert max(match.values()) == 1.0, match


TILED = ["fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32", "fp32_fp64", "fp32_fp32"]


@pytest.mark.parametrize("op", TILED)
@pytest.mark.parametrize("shape", [(64, 64, 48), (100, 70, 33), (33, 300, 128)])
def test_tiled_vs_oracle(op, shape):
    n, m, d = shape
    P, C = data(n, m, d, "blobs", seed=5)
    for T in (16, 32):
        kappa = 5.0 if not op.startswith("bf16") else 0.1
        De, tot, tiles = getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tiled_{op}_with_stats")(
            cuda(P), cuda(C), kappa, T)
        Do, flag_o, cnt_o, tiles_o = O.tiled(op, P, C, kappa, tile=T)
        De = De.cpu().numpy()
        assert len(tiles) == len(tiles_o) and tot == sum(tiles)
        if op.startswith("fp32"):
            np.testing.assert_array_equal(De, Do)
            np.testing.assert_array_equal(np.array(tiles), tiles_o)
        else:
            pp, cc = norms_for(P, C, "sumsq")
            check_tc_D(De, Do, flag_o, tot, cnt_o, pp, cc, U_LOW[O.TILED[op][0]])
            assert np.abs(np.array(tiles) - tiles_o).sum() <= 2 + 0.01 * cnt_o
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32"])
def test_tensorcore_vs_oracle(op):
    P, C = data(96, 80, 64, "blobs", seed=9)
    kappa = 5.0 if op.startswith("fp16") else 0.1
    De = getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{op}")(cuda(P), cuda(C), kappa, 32)
    Do, flag_o, cnt_o, _ = O.tiled(op, P, C, kappa)
    pp, cc = norms_for(P, C, "sumsq")
    check_tc_D(De.cpu().numpy(), Do, flag_o, int(flag_o.sum()), cnt_o, pp, cc, U_LOW[O.TILED[op][0]])
    with pytest.raises(RuntimeError, match="tile_size=32 only"):
        getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{op}")(cuda(P), cuda(C), kappa)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        getattr(euclidean_cuda_tiled, f"pairwise_euclidean_tensorcore_{op}")(cuda(P[:, :60]), cuda(C[:, :60]),
                                                                             kappa, 32)
    device_check()


@pytest.mark.parametrize("shape", SHAPES)
def test_base_ops_exact(shape):
    n, m, d = shape
    P, C = data(n, m, d, "gauss", seed=1)
    np.testing.assert_array_equal(euclidean_cuda.pairwise_euclidean_single(cuda(P), cuda(C)).cpu().numpy(),
                                  O.single(P, C))
    np.testing.assert_array_equal(
        euclidean_cuda.pairwise_euclidean_double(cuda(P).double(), cuda(C).double()).cpu().numpy(),
        O.double(P.astype(np.float64), C.astype(np.float64)))
    lab, md, _ = euclidean_cuda.pairwise_euclidean_double_argmin(cuda(P).double(), cuda(C).double())
    Do = O.double(P.astype(np.float64), C.astype(np.float64))
    np.testing.assert_array_equal(lab.cpu().numpy(), O.argmin_first(Do))
    np.testing.assert_array_equal(md.cpu().numpy(), Do.min(1))
    device_check()


@pytest.mark.parametrize("shape", SHAPES)
def test_uniform_vs_oracle(shape):
    n, m, d = shape
    P, C = data(n, m, d, "gauss", seed=2)
    P16, C16 = P.astype(np.float16), C.astype(np.float16)
    Pb, Cb = O.bf16_bits(P), O.bf16_bits(C)
    tp16, tc16 = cuda(P16), cuda(C16)
    tpb, tcb = cuda(Pb.view(np.int16)).view(torch.bfloat16), cuda(Cb.view(np.int16)).view(torch.bfloat16)
    U = euclidean_cuda_uniform
    # direct formulas: deterministic sequential fma -> bit exact
    np.testing.assert_array_equal(U.pairwise_euclidean_uniform_fp16_direct(tp16, tc16).cpu().numpy(),
                                  O.uniform("fp16_direct", P16, C16))
    np.testing.assert_array_equal(
        U.pairwise_euclidean_uniform_bf16_direct(tpb, tcb).view(torch.int16).cpu().numpy().view(np.uint16),
        O.uniform("bf16_direct", Pb, Cb))
    for nm in ("tf32_direct", "fp32_direct"):
        np.testing.assert_array_equal(getattr(U, f"pairwise_euclidean_uniform_{nm}")(cuda(P), cuda(C)).cpu().numpy(),
                                      O.uniform(nm, P, C))
    P64, C64 = P.astype(np.float64), C.astype(np.float64)
    np.testing.assert_array_equal(U.pairwise_euclidean_uniform_fp64_direct(cuda(P64), cuda(C64)).cpu().numpy(),
                                  O.uniform("fp64_direct", P64, C64))
    np.testing.assert_array_equal(U.pairwise_euclidean_uniform_tf32(cuda(P), cuda(C)).cpu().numpy(),
                                  O.uniform("tf32", P, C))
    # expanded fp16 / bf16 (tensor cores, output in the low type)
    D16 = U.pairwise_euclidean_uniform_fp16(tp16, tc16).cpu().numpy().astype(np.float64)
    Do16 = O.uniform("fp16", P16, C16).astype(np.float64)
    pp, cc = norms_for(P16.astype(np.float32), C16.astype(np.float32), "low_fp16")
    assert (np.abs(D16 - Do16) <= 8 * 2.0 ** -11 * (pp[:, None] + cc[None]) + 2e-3 * np.abs(Do16)).all()
    Db = O.bf16_from_bits(U.pairwise_euclidean_uniform_bf16(tpb, tcb).view(torch.int16).cpu().numpy().view(np.uint16))
    Dob = O.bf16_from_bits(O.uniform("bf16", Pb, Cb))
    ppb, ccb = norms_for(O.bf16_from_bits(Pb), O.bf16_from_bits(Cb), "low_bf16")
    assert (np.abs(Db.astype(np.float64) - Dob) <= 8 * 2.0 ** -8 * (ppb[:, None] + ccb[None]) + 1e-2 * np.abs(Dob)).all()
    device_check()


@pytest.mark.parametrize("shape", SHAPES)
def test_advanced_exact(shape):
    n, m, d = shape
    P, C = data(n, m, d, "blobs", seed=4)
    A = euclidean_cuda_advanced
    for kappa in (5.0, 1e5):
        P16, C16 = P.astype(np.float16), C.astype(np.float16)
        De = A.pairwise_euclidean_fp64_fp16(cuda(P16), cuda(C16), kappa).cpu().numpy()
        np.testing.assert_array_equal(De, O.advanced("fp64_fp16", P16, C16, kappa)[0])
        Pb, Cb = O.bf16_bits(P), O.bf16_bits(C)
        tpb, tcb = cuda(Pb.view(np.int16)).view(torch.bfloat16), cuda(Cb.view(np.int16)).view(torch.bfloat16)
        np.testing.assert_array_equal(A.pairwise_euclidean_fp64_bf16(tpb, tcb, kappa).cpu().numpy(),
                                      O.advanced("fp64_bf16", Pb, Cb, kappa)[0])
        np.testing.assert_array_equal(A.pairwise_euclidean_fp64_tf32(cuda(P), cuda(C), kappa).cpu().numpy(),
                                      O.advanced("fp64_tf32", P, C, kappa)[0])
        P64, C64 = P.astype(np.float64), C.astype(np.float64)
        np.testing.assert_array_equal(
            A.pairwise_euclidean_fp64_fp32_gemm(cuda(P64), cuda(C64), kappa).cpu().numpy(),
            O.advanced("fp64_fp32_gemm", P64, C64, kappa)[0])
    device_check()


# shapes reach: the shared-memory table (first), the block-private counting sort (k <= 16384,
# one and several row blocks) and the global-atomic counting sort (k > 16384)
@pytest.mark.parametrize("n,d,k", [(500, 8, 10), (20000, 64, 300), (4097, 130, 4096), (3, 2, 5),
                                   (100000, 16, 4096), (30000, 4, 20000)])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_centers_vs_oracle(n, d, k, dtype):
    rng = np.random.default_rng(n + k)
    X = rng.normal(size=(n, d)).astype(dtype)
    lab = rng.integers(-1, k + 1, n).astype(np.int64)  # includes out-of-range labels
    lab[lab == 1] = 0                                     # cluster 1 empty
    fn = center_kernels.update_centers_fp32 if dtype == np.float32 else center_kernels.update_centers_fp64
    ce = fn(cuda(X), cuda(lab), k).cpu().numpy()
    st = O.center_stats(X, lab, k)
    cnt = st[:, d]
    exact = np.where(cnt[:, None] > 0, st[:, :d] / np.maximum(cnt[:, None], 1), 0.0)
    assert (ce[1] == 0).all()
    np.testing.assert_allclose(ce, exact.astype(dtype), rtol=1e-6 if dtype == np.float32 else 1e-12,
                               atol=1e-7 if dtype == np.float32 else 1e-14)
    co, _ = O.update_centers(X, lab, k)  # reference semantics (sequential sums)
    tol = (np.maximum(cnt, 1) * (2.0 ** -24 if dtype == np.float32 else 2.0 ** -53))[:, None] * 8
    assert (np.abs(ce - co) <= tol * np.maximum(np.abs(co), 1)).all()
    device_check()


def test_centers_reinit_uses_reference_rng_draws():
    rng = np.random.default_rng(0)
    X = rng.normal(size=(100, 4)).astype(np.float32)
    lab = rng.integers(0, 3, 100).astype(np.int64)  # clusters 3..5 empty
    torch.manual_seed(123)
    ce = center_kernels.update_centers_fp32_with_reinit(cuda(X), cuda(lab), 6)
    torch.manual_seed(123)
    pts = torch.randint(0, 100, (3,), dtype=torch.long, device=DEV).cpu().numpy()
    np.testing.assert_array_equal(ce[3:].cpu().numpy(), X[pts])


def test_lloyd_step_matches_composition():
    from kmeans import LloydKMeans
    P, C = data(5000, 50, 24, "blobs", seed=8)
    km = LloydKMeans(50, op="fp16_fp32", kappa=5.0)
    C1, lab, cnt = km.step(cuda(P), cuda(C))
    lab_ref, _, _ = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32_argmin(cuda(P), cuda(C), 5.0)
    torch.testing.assert_close(lab.long(), lab_ref, rtol=0, atol=0)
    st = O.center_stats(P, lab.cpu().numpy().astype(np.int64), 50)
    exact = np.where(st[:, -1:] > 0, st[:, :-1] / np.maximum(st[:, -1:], 1), 0.0)
    np.testing.assert_allclose(C1.cpu().numpy(), exact.astype(np.float32), rtol=1e-6, atol=1e-7)
    device_check()


def test_error_paths_on_gpu():
    P = cuda(np.zeros((4, 3), np.float32))
    with pytest.raises(RuntimeError, match="P must be float32"):
        euclidean_cuda_mix.pairwise_euclidean_fp16_fp64(P.double(), P)
    with pytest.raises(RuntimeError, match="Dimension mismatch"):
        euclidean_cuda_mix.pairwise_euclidean_fp16_fp64(P, cuda(np.zeros((4, 2), np.float32)))
    with pytest.raises(RuntimeError, match="must be contiguous"):
        euclidean_cuda_mix.pairwise_euclidean_fp16_fp64(cuda(np.zeros((3, 4), np.float32)).t(), P)
    with pytest.raises(RuntimeError, match="Supported tile_size: 16 or 32"):
        euclidean_cuda_tiled.pairwise_euclidean_tiled_fp32_fp32(P, P, 5.0)  # default tile_size=64
    with pytest.raises(RuntimeError, match="labels must be int64"):
        center_kernels.update_centers_fp32(P, cuda(np.zeros(4, np.int32)), 2)
    # empty inputs
    e = euclidean_cuda_mix.pairwise_euclidean_fp16_fp32(cuda(np.zeros((0, 3), np.float32)), P)
    assert e.shape == (0, 4)
    device_check()


@pytest.mark.parametrize("op", ["fp16_fp32", "bf16_fp32"])
def test_fast_argmin_fused_rows_equal_prepared_rows(op):
    """The screen reads 16-byte aligned fp32 points itself; a point matrix one float off
    that alignment takes the prepared low-precision copy instead.  Both round, and sum
    the norms, the same way: identical outputs."""
    g = torch.Generator(device=DEV).manual_seed(5)
    n, m, d = 5000, 700, 96
    base = torch.randn(n * d + 1, generator=g, device=DEV)
    P_off = base[1:].view(n, d)  # 4 bytes past a 16-byte boundary
    P = P_off.clone()            # aligned copy of the same values
    C = torch.randn(m, d, generator=g, device=DEV)
    kappa = 5.0 if op.startswith("fp16") else 0.1
    fn = getattr(euclidean_cuda_mix, f"pairwise_euclidean_{op}_argmin")
    la, ma, ca = fn(P, C, kappa)
    lb, mb, cb = fn(P_off, C, kappa)
    torch.testing.assert_close(la, lb, rtol=0, atol=0)
    torch.testing.assert_close(ma, mb, rtol=0, atol=0)
    assert int(ca.item()) == int(cb.item())
    device_check()
