"""Known-answer tests of the CPU oracle (no GPU): rounding helpers, norms, GEMM
order, direct formulas, flag constants and the center update, on cases whose
answers are exact by construction."""
import numpy as np
import pytest

from oracle import oracle as O


def test_round_f16_matches_numpy_rne():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 1, 10000), rng.normal(0, 1e4, 1000), rng.normal(0, 1e-5, 1000),
                        [65504.0, 65519.9, 65520.0, 1e6, -1e6, 0.0, -0.0, 2.0 ** -25, 3 * 2.0 ** -26]])
    x = x.astype(np.float32)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(O.round_f16(x), ref)


def test_round_bf16_matches_torch_rne():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.normal(0, 1, 10000), rng.normal(0, 1e30, 100), [3.4e38, 1e-40, 0.0]]).astype(np.float32)
    ref = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(O.round_bf16(x), ref)


def test_round_tf32_is_round_half_away():
    # 1 + 2^-11 is the midpoint between 1 and 1 + 2^-10: tf32 RNA rounds it up
    x = np.array([1 + 2.0 ** -11, -(1 + 2.0 ** -11), 1 + 2.0 ** -12, 1 + 3 * 2.0 ** -11], np.float32)
    np.testing.assert_array_equal(O.round_tf32(x), np.array([1 + 2.0 ** -10, -(1 + 2.0 ** -10), 1.0,
                                                            1 + 2 * 2.0 ** -10], np.float32))


def test_norm_modes():
    X = np.array([[1.0, 2.0, 3.0], [0.1, 0.2, 0.3]], np.float32)
    np.testing.assert_array_equal(O.norms_f32(X[:1], "fma"), np.float32([14.0]))
    # low_fp16: fp16 inputs, fp32 fma accumulation, fp16 result
    h = X[1].astype(np.float16).astype(np.float32)
    s = np.float32(0)
    for v in h:
        s = np.float32(np.float64(v) * v + s)  # exact product in fp64, single rounding == fmaf
    assert O.norms_f32(X[1:], "low_fp16")[0] == np.float32(np.float16(s))
    X64 = X.astype(np.float64)
    np.testing.assert_allclose(O.norms_f64(X64), (X64 ** 2).sum(1), rtol=1e-15)


def test_gemm_sequential_order():
    # exact integer data: any order gives the same result, check the shape convention S = A B^T
    A = np.arange(12, dtype=np.float32).reshape(3, 4)
    B = np.arange(8, dtype=np.float32).reshape(2, 4)
    np.testing.assert_array_equal(O.gemm_f32(A, B), A @ B.T)
    np.testing.assert_array_equal(O.gemm_f64(A.astype(np.float64), B.astype(np.float64)), (A @ B.T).astype(np.float64))


def test_lattice_distances_exact():
    # integer lattice points: every formula is exact
    rng = np.random.default_rng(2)
    P = rng.integers(-8, 8, (40, 6)).astype(np.float32)
    C = rng.integers(-8, 8, (9, 6)).astype(np.float32)
    exact = ((P[:, None, :].astype(np.float64) - C[None]) ** 2).sum(-1)
    np.testing.assert_array_equal(O.single(P, C), exact.astype(np.float32))
    np.testing.assert_array_equal(O.double(P, C), exact)
    np.testing.assert_array_equal(O.direct_all(P, C), exact)
    ii, jj = np.nonzero(np.ones_like(exact, bool))
    for rec in ("fp64", "fp32", "fp16"):  # sums <= 2048 are exact in fp16
        np.testing.assert_array_equal(O.direct_pairs(rec, P, C, ii, jj), exact[ii, jj])
    # bf16 arithmetic (8 significant bits) rounds: compare with torch's per-op bf16 rounding
    torch = pytest.importorskip("torch")
    pb, cb = torch.from_numpy(P).bfloat16(), torch.from_numpy(C).bfloat16()
    acc = torch.zeros(len(ii), dtype=torch.bfloat16)
    for k in range(P.shape[1]):
        diff = pb[ii, k] - cb[jj, k]
        acc = acc + diff * diff
    np.testing.assert_array_equal(O.direct_pairs("bf16", P, C, ii, jj), acc.float().numpy())
    for name in O.MIX:
        if name == "bf16_bf16":
            continue
        D, flag, cnt = O.mix(name, P, C, 5.0)
        np.testing.assert_array_equal(D, exact.astype(np.float32))
    np.testing.assert_array_equal(O.argmin_first(exact), np.argmin(exact, 1))


def test_fp16_arithmetic_recompute_rounds_each_step():
    # (p - c)^2 accumulated in fp16: 2049 is not representable, 2048 + 1 -> 2048
    P = np.zeros((1, 3), np.float32)
    C = np.array([[32.0, 32.0, 1.0]], np.float32)  # 1024 + 1024 + 1
    v = O.direct_pairs("fp16", P, C, [0], [0])[0]
    assert v == 2048.0
    assert O.direct_pairs("fp64", P, C, [0], [0])[0] == 2049.0


def test_flag_constants_follow_reference_expressions():
    # kform 0: kappa * ((2d+4) * u) ; kform 1: (kappa * 2) * (d * u)
    assert O._k_float(0, 5.0, 128, 2.0 ** -11) == np.float32(5.0) * np.float32(260 * 2.0 ** -11)
    assert O._k_float(1, 5.0, 128, 2.0 ** -23) == np.float32(10.0) * np.float32(128 * 2.0 ** -23)


def test_mix_flags_close_pairs_only():
    rng = np.random.default_rng(3)
    C = rng.normal(size=(16, 32)).astype(np.float32)
    lab = rng.integers(0, 16, 64)
    P = (C[lab] + rng.normal(0, 1e-3, (64, 32))).astype(np.float32)
    D, flag, cnt = O.mix("fp16_fp64", P, C, 5.0)
    # every point's own center is flagged and recomputed exactly; far pairs are not
    assert flag[np.arange(64), lab].all()
    assert cnt == flag.sum() and cnt < 64 * 16 // 4
    exact = ((P[:, None, :].astype(np.float64) - C[None]) ** 2).sum(-1)
    np.testing.assert_allclose(D[np.arange(64), lab], exact[np.arange(64), lab].astype(np.float32), rtol=1e-6)
    assert (O.argmin_first(D) == lab).all()


def test_centers_reference_semantics():
    X = np.arange(20, dtype=np.float32).reshape(10, 2)
    lab = np.array([0, 0, 1, 1, 1, 5, -1, 9, 0, 3])  # 5, -1, 9 out of range for k=4; cluster 2 empty
    c, cnt = O.update_centers(X, lab, 4)
    np.testing.assert_array_equal(cnt, [3, 3, 0, 1])
    np.testing.assert_array_equal(c[2], [0.0, 0.0])
    np.testing.assert_allclose(c[0], X[[0, 1, 8]].mean(0))
    st = O.center_stats(X, lab, 4)
    np.testing.assert_array_equal(st[:, 2], [3, 3, 0, 1])
    np.testing.assert_array_equal(st[1, :2], X[[2, 3, 4]].sum(0))


def test_cpu_baseline_argmin():
    rng = np.random.default_rng(4)
    P = rng.normal(size=(300, 12))
    C = rng.normal(size=(17, 12))
    lab, md, used = O.dist_argmin_f64(P, C, threads=2)
    D = ((P[:, None] - C[None]) ** 2).sum(-1)
    np.testing.assert_array_equal(lab, D.argmin(1))
    np.testing.assert_allclose(md, D.min(1), rtol=1e-12, atol=1e-12)
    assert used >= 1


def test_kmeanspp_oracle_draws_distinct_rows():
    """D^2 sampling never re-draws a chosen row while another row has weight > 0; the
    first row is the uniform draw floor(r_0 n / 2^53)."""
    rng = np.random.default_rng(0)
    X = rng.normal(size=(400, 5))
    idx = O.kmeanspp(X, 30, seed=11)
    assert len(set(idx.tolist())) == 30
    assert idx[0] == (O.seed_draw53(11, 0) * 400) >> 53
    assert 0 <= O.seed_draw53(2 ** 64 - 1, 5) < 2 ** 53


@pytest.mark.parametrize("name", ["fp16_fp32", "bf16_fp64", "tf32_fp64"])
def test_certified_oracle_is_the_fully_flagged_operator(name):
    # with every pair flagged (kappa large enough that K >= 2), the operator's D is the
    # direct distance of every pair: its first-index argmin is the certified label
    rng = np.random.default_rng(4)
    P = rng.normal(size=(120, 9)).astype(np.float32)
    C = np.concatenate([rng.normal(size=(30, 9)), P[:3]]).astype(np.float32)
    D, flag, cnt = O.mix(name, P, C, kappa=1e6)
    assert flag.all()
    lab, md = O.certified_argmin(name, P, C)
    np.testing.assert_array_equal(lab, O.argmin_first(D))
    np.testing.assert_array_equal(md, D[np.arange(120), lab])
    assert (lab[:3] == 30 + np.arange(3)).all()  # the points themselves, at distance 0
    assert (md[:3] == 0).all()


@pytest.mark.parametrize("name", ["bf16_fp64", "bf16_fp32"])
def test_certified_oracle_ties_on_the_stored_fp32_value(name):
    # the label is the first index among distances equal AS STORED (fp32): centers 3 and
    # 5 differ by one fp32 ulp in dimension 7 and the rows sit on center 5 there, so
    # center 3 is farther by ulp^2 in exact arithmetic but the stored values tie and 3
    # wins, as argmin_first of the operator's D gives (C3's offset-1000 regime, where the
    # engine sweeps every pair densely)
    rng = np.random.default_rng(11)
    n, d, k = 64, 64, 16
    P = (rng.normal(size=(n, d)) + 1000.0).astype(np.float32)
    C = (rng.normal(size=(k, d)) + 1000.0).astype(np.float32)
    C[5] = C[3]
    C[5, 7] = np.nextafter(C[3, 7], np.float32(2000.0))
    P[:10] = C[5] + 0.3 * rng.normal(size=(10, d)).astype(np.float32)
    P[:10, 7] = C[5, 7]
    exact = ((P[:10, None, :].astype(np.float64) - C[None, [3, 5], :].astype(np.float64)) ** 2).sum(-1)
    assert (exact[:, 0] > exact[:, 1]).all()  # center 5 is closer before rounding
    D, flag, _ = O.mix(name, P, C, kappa=5.0)
    assert flag.all()
    lab, md = O.certified_argmin(name, P, C)
    np.testing.assert_array_equal(lab, O.argmin_first(D))
    np.testing.assert_array_equal(md, D[np.arange(n), lab])
    assert (D[:10, 3] == D[:10, 5]).all() and (lab[:10] == 3).all()


def test_certified_oracle_rejects_half_arithmetic_recompute():
    P = np.ones((2, 3), np.float32)
    with pytest.raises(ValueError):
        O.certified_argmin("fp16_fp16", P, P)


def _kappa_for(K, dim, u):
    # the smallest float kappa whose K = kappa * ((2 dim + 4) u) (the reference's float
    # expression) reaches K
    kappa = np.float32(K / ((2 * dim + 4) * u))
    while O._k_float(0, kappa, dim, u) < np.float32(K):
        kappa = np.nextafter(kappa, np.float32(np.inf))
    return kappa


ALL_FLAGGED_OPS = [("mix", n) for n in ("fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32", "tf32_fp64")] + \
                  [("tiled", n) for n in ("fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32")]


def _adversarial(rng, dim, lo, hi):
    """Rows whose fp32 norms span [lo, hi] (log-uniform, ends included) and centers that
    are the rows negated and rescaled (anti-aligned pairs: the most negative s, so the
    largest distance relative to pp + cc), plus Gaussian rows."""
    n = 96
    P = rng.normal(size=(n, dim))
    P /= np.linalg.norm(P, axis=1, keepdims=True)
    tgt = np.exp(rng.uniform(np.log(lo), np.log(hi), n))
    tgt[:4] = [lo, lo, hi, hi]
    P *= np.sqrt(tgt)[:, None] * (1 + 2.0 ** -20)
    C = -P[rng.permutation(n)[:48]] * rng.uniform(0.5, 1.0, (48, 1))
    C = np.concatenate([C, -P[:8], rng.normal(size=(8, dim))])
    P = P.astype(np.float32)
    C = C.astype(np.float32)
    norms = np.concatenate([O.norms_f32(P, "sumsq"), O.norms_f32(C, "sumsq")])
    keep = (norms >= lo) & (norms <= hi)  # what the engine's range check lets through
    return P[keep[:len(P)]], C[keep[len(P):]]


@pytest.mark.parametrize("kind,name", ALL_FLAGGED_OPS)
@pytest.mark.parametrize("dim", [3, 64, 1024])
def test_all_flagged_route_flags_every_pair(kind, name, dim):
    """The engine's all-flagged route (fused argmin with K >= 2.5 and every norm in
    [2^-13, hi], hi = 6.0e4 where S or the norms are rounded to fp16) replaces the
    exact epilogue by the certified argmin and reports n * m flagged pairs.  That needs
    the reference's cancellation test to flag every such pair, anti-aligned pairs at the
    ends of the range included."""
    rng = np.random.default_rng(dim)
    f16 = name.startswith("fp16")
    lo, hi = 2.0 ** -13, (6.0e4 if f16 else 1.0e30)
    P, C = _adversarial(rng, dim, lo, hi)
    if kind == "mix":
        _, _, _, u, _, _ = O.MIX[name]
        D, flag, cnt = O.mix(name, P, C, kappa=_kappa_for(2.5, dim, u))
    else:
        _, u, _ = O.TILED[name]
        D, flag, cnt, _ = O.tiled(name, P, C, _kappa_for(2.5, dim, u))
    assert flag.all() and cnt == P.shape[0] * C.shape[0]
    lab, md = O.certified_argmin(("" if kind == "mix" else "tiled_") + name, P, C)
    np.testing.assert_array_equal(lab, O.argmin_first(D))
    np.testing.assert_array_equal(md, D[np.arange(P.shape[0]), lab])


def test_all_flagged_route_needs_its_threshold():
    # below the route's K an anti-aligned pair (s < 0) escapes the test: d_exp is about
    # 2 (pp + cc) there, so K = 1.9 leaves it unflagged
    rng = np.random.default_rng(0)
    P = rng.normal(size=(16, 32)).astype(np.float32)
    _, _, _, u, _, _ = O.MIX["bf16_fp32"]
    _, flag, _ = O.mix("bf16_fp32", P, -P, kappa=_kappa_for(1.9, 32, u))
    assert not flag[np.arange(16), np.arange(16)].any()
