"""Pin the CPU oracle to the reference's own outputs (no GPU needed).

tests/golden/*.npz hold inputs and outputs of the unmodified reference extensions,
run on a B200 by tests/golden/make_golden.py.  Checked here, per fixture and kappa:

* flag counts of every mix operator: equal;
* every pair the oracle recomputes: bit-identical to the reference (the direct
  formulas are deterministic, including the fp16/bf16-arithmetic ones);
* everything downstream of the reference's library GEMM (cuBLAS / torch::mm, whose
  summation order the oracle cannot reproduce): |D - D_ref| <= 8 u (pp + cc);
* per-tile flag counts of the tiled operators: equal;
* direct (uniform *_direct) operators and the fp32/fp64 center update: bit-identical;
* the caller-side argmin of a reference D: equal to the oracle's.
"""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIX = sorted(f for f in glob.glob(os.path.join(HERE, "*.npz")) if not f.endswith("centers_empty.npz"))
U = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -7, "tf32": 2.0 ** -11, "fp32": 2.0 ** -20}


def load(f):
    z = np.load(f)
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="module", params=FIX, ids=[os.path.basename(f)[:-4] for f in FIX])
def g(request):
    return load(request.param)


def test_fixtures_present():
    assert len(FIX) >= 6 and os.path.exists(os.path.join(HERE, "centers_empty.npz"))


@pytest.mark.parametrize("op", sorted(O.MIX))
def test_mix_pinned(g, op):
    P, C = g["P"], g["C"]
    low, s_round, nmode = O.MIX[op][0], O.MIX[op][1], O.MIX[op][2]
    pp = O.norms_f32(P, nmode).astype(np.float64)
    cc = O.norms_f32(C, nmode).astype(np.float64)
    for ki, kappa in enumerate(g["kappas"]):
        Dr = g[f"mix_{op}_k{ki}"]
        Do, flag, cnt = O.mix(op, P, C, float(kappa))
        assert cnt == int(g[f"mix_{op}_k{ki}_count"])
        np.testing.assert_array_equal(Do[flag], Dr[flag])
        tol = 8 * U[low] * (pp[:, None] + cc[None]) + 1e-6 * np.abs(Dr)
        assert (np.abs(Do.astype(np.float64) - Dr) <= tol).all()
        if s_round:  # S rounded to fp16/bf16: the library GEMM's order rarely changes a value
            assert (Do == Dr).mean() > 0.95


@pytest.mark.parametrize("op", sorted(O.TILED))
def test_tiled_pinned(g, op):
    P, C = g["P"], g["C"]
    for ki, kappa in enumerate(g["kappas"]):
        for T in (16, 32):
            key = f"tiled_{op}_T{T}_k{ki}"
            if key not in g:
                continue
            Do, flag, cnt, tiles = O.tiled(op, P, C, float(kappa), tile=T)
            np.testing.assert_array_equal(tiles, g[key + "_tiles"])
            np.testing.assert_array_equal(Do[flag], g[key][flag])
            nrm = O.norms_f32(P, "sumsq").astype(np.float64), O.norms_f32(C, "sumsq").astype(np.float64)
            tol = 8 * U[O.TILED[op][0]] * (nrm[0][:, None] + nrm[1][None]) + 1e-6 * np.abs(g[key])
            assert (np.abs(Do.astype(np.float64) - g[key]) <= tol).all()


@pytest.mark.parametrize("op", ["fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32"])
def test_tensorcore_pinned(g, op):
    P, C = g["P"], g["C"]
    for ki, kappa in enumerate(g["kappas"]):
        key = f"tc_{op}_k{ki}"
        if key not in g:
            continue
        Do, flag, cnt, _ = O.tiled(op, P, C, float(kappa))
        nrm = O.norms_f32(P, "sumsq").astype(np.float64), O.norms_f32(C, "sumsq").astype(np.float64)
        tol = 8 * U[O.TILED[op][0]] * (nrm[0][:, None] + nrm[1][None]) + 1e-6 * np.abs(g[key])
        assert (np.abs(Do.astype(np.float64) - g[key]) <= tol).all()
        # pairs both sides recomputed carry the identical direct value
        both = flag & (Do == g[key])
        assert both.sum() >= 0.9 * flag.sum()


def test_base_and_uniform_pinned(g):
    P, C = g["P"], g["C"]
    pp, cc = O.norms_f32(P, "fma").astype(np.float64), O.norms_f32(C, "fma").astype(np.float64)
    assert (np.abs(O.single(P, C) - g["single"]) <= 2.0 ** -18 * (pp[:, None] + cc[None])).all()
    D64 = O.double(P.astype(np.float64), C.astype(np.float64))
    assert (np.abs(D64 - g["double"]) <= 2.0 ** -48 * (pp[:, None] + cc[None])).all()
    # direct formulas: bit-identical
    np.testing.assert_array_equal(O.uniform("fp32_direct", P, C), g["uni_fp32_direct"])
    np.testing.assert_array_equal(O.uniform("tf32_direct", P, C), g["uni_tf32_direct"])
    np.testing.assert_array_equal(O.uniform("fp64_direct", P.astype(np.float64), C.astype(np.float64)),
                                  g["uni_fp64_direct"])
    np.testing.assert_array_equal(O.uniform("fp16_direct", P.astype(np.float16), C.astype(np.float16)),
                                  g["uni_fp16_direct"])
    np.testing.assert_array_equal(O.uniform("bf16_direct", g["P_bf16"], g["C_bf16"]), g["uni_bf16_direct"])
    np.testing.assert_array_equal(O.bf16_bits(P), g["P_bf16"])  # the oracle's bf16 rounding is torch's
    # expanded fp16 / bf16 / fp32 forms
    D16 = O.uniform("fp16", P.astype(np.float16), C.astype(np.float16)).astype(np.float64)
    assert (np.abs(D16 - g["uni_fp16"]) <= 8 * 2.0 ** -11 * (pp[:, None] + cc[None]) + 2e-3 * np.abs(D16)).all()
    Db = O.bf16_from_bits(O.uniform("bf16", g["P_bf16"], g["C_bf16"])).astype(np.float64)
    Dbr = O.bf16_from_bits(g["uni_bf16"])
    assert (np.abs(Db - Dbr) <= 8 * 2.0 ** -8 * (pp[:, None] + cc[None]) + 1e-2 * np.abs(Dbr)).all()
    assert (np.abs(O.uniform("tf32", P, C) - g["uni_tf32"]) <= 2.0 ** -18 * (pp[:, None] + cc[None])).all()


def test_advanced_pinned(g):
    P, C = g["P"], g["C"]
    for ki, kappa in enumerate(g["kappas"]):
        for op, args in (("fp64_fp16", (P.astype(np.float16), C.astype(np.float16))),
                         ("fp64_bf16", (g["P_bf16"], g["C_bf16"])),
                         ("fp64_tf32", (P, C)),
                         ("fp64_fp32_gemm", (P.astype(np.float64), C.astype(np.float64)))):
            Do, _ = O.advanced(op, *args, float(kappa))
            Dr = g[f"adv_{op}_k{ki}"]
            nrm = (P.astype(np.float64) ** 2).sum(1), (C.astype(np.float64) ** 2).sum(1)
            tol = 2.0 ** -18 * (nrm[0][:, None] + nrm[1][None]) + 1e-6 * np.abs(Dr)
            assert (np.abs(Do.astype(np.float64) - Dr) <= tol).all(), op
            assert (Do == Dr).mean() > 0.9, op


def test_argmin_and_centers_pinned(g):
    P, C = g["P"], g["C"]
    Dr = g["mix_fp16_fp32_k0"]
    np.testing.assert_array_equal(O.argmin_first(Dr), g["argmin_mix_fp16_fp32_k0"])
    lab = g["centers_labels"]
    c32, _ = O.update_centers(P, lab, C.shape[0])
    np.testing.assert_array_equal(c32, g["centers_fp32"])  # same sequential fp32 sums
    c64, _ = O.update_centers(P.astype(np.float64), lab, C.shape[0])
    np.testing.assert_array_equal(c64, g["centers_fp64"])


def test_centers_empty_and_out_of_range_pinned():
    z = load(os.path.join(HERE, "centers_empty.npz"))
    c32, cnt = O.update_centers(z["X"], z["labels"], 10)
    np.testing.assert_array_equal(c32, z["centers_fp32"])
    c64, _ = O.update_centers(z["X"].astype(np.float64), z["labels"], 10)
    np.testing.assert_array_equal(c64, z["centers_fp64"])
    assert cnt[4] == 0 and (z["centers_fp32"][4] == 0).all()
