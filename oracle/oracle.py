"""CPU oracle for the euclid-cuda distance path -- TEST INFRASTRUCTURE ONLY.

Restates, operator by operator, the arithmetic of the reference extensions
(inEXASCALE/euclid-cuda) on the CPU: numpy float32/float64 for the elementwise
steps (IEEE round-to-nearest, no fusion), and the C routines of euclid_oracle.c
(liboracle.so) for everything that has a required accumulation order.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module; the engine never does.

Parity status: pinned against golden vectors that the reference's own CUDA
extensions produced on a B200 (tests/golden/, see tests/golden/make_golden.py).
The one step the oracle cannot reproduce bit for bit is the reference's library
GEMM (cuBLAS / torch::mm, summation order unspecified); the oracle uses a
sequential fused multiply-add and the tests compare through that step with a
tolerance.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        src = os.path.join(HERE, "euclid_oracle.c")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
        L = ctypes.CDLL(path)
        P, I64, I, D = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.orc_round.argtypes = [P, P, I64, I]
        L.orc_norms_f32.argtypes = [P, I64, I64, I, P]
        L.orc_norms_f64.argtypes = [P, I64, I64, P]
        L.orc_gemm_f32.argtypes = [P, P, I64, I64, I64, P]
        L.orc_gemm_f64.argtypes = [P, P, I64, I64, I64, P]
        L.orc_direct_pairs.argtypes = [I, I, P, P, I64, P, P, I64, P]
        L.orc_direct_all.argtypes = [I, P, P, I64, I64, I64, P]
        L.orc_centers_f32.argtypes = [P, P, I64, I64, I64, P, P]
        L.orc_centers_f64.argtypes = [P, P, I64, I64, I64, P, P]
        L.orc_center_stats.argtypes = [P, I, P, I64, I64, I64, P]
        L.orc_dist_argmin_f64.argtypes = [P, P, I64, I64, I64, P, P, I]
        L.orc_dist_argmin_f64.restype = I
        L.orc_lloyd_step_f64.argtypes = [P, P, I64, I64, I64, P, P, I, P]
        L.orc_lloyd_step_f64.restype = I
        L.orc_max_threads.restype = I
        _LIB = L
    return _LIB


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ----------------------------------------------------------------- rounding
def round_f16(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_round(_p(x), _p(y), x.size, 1)
    return y


def round_bf16(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_round(_p(x), _p(y), x.size, 2)
    return y


def round_tf32(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_round(_p(x), _p(y), x.size, 3)
    return y


def bf16_bits(x):
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b):
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


LOW_ROUND = {"fp16": round_f16, "bf16": round_bf16, "tf32": round_tf32}


# -------------------------------------------------------------------- norms
def norms_f32(X, mode):
    """mode: 'low_fp16' | 'low_bf16' | 'fma' | 'sumsq' (see euclid_oracle.c)."""
    X = _c(X, np.float32)
    out = np.empty(X.shape[0], np.float32)
    code = {"low_fp16": 0, "low_bf16": 1, "fma": 2, "sumsq": 3}[mode]
    lib().orc_norms_f32(_p(X), X.shape[0], X.shape[1], code, _p(out))
    return out


def norms_f64(X):
    X = _c(X, np.float64)
    out = np.empty(X.shape[0], np.float64)
    lib().orc_norms_f64(_p(X), X.shape[0], X.shape[1], _p(out))
    return out


# -------------------------------------------------------------------- GEMMs
def gemm_f32(A, B):
    A, B = _c(A, np.float32), _c(B, np.float32)
    S = np.empty((A.shape[0], B.shape[0]), np.float32)
    lib().orc_gemm_f32(_p(A), _p(B), A.shape[0], B.shape[0], A.shape[1], _p(S))
    return S


def gemm_f64(A, B):
    A, B = _c(A, np.float64), _c(B, np.float64)
    S = np.empty((A.shape[0], B.shape[0]), np.float64)
    lib().orc_gemm_f64(_p(A), _p(B), A.shape[0], B.shape[0], A.shape[1], _p(S))
    return S


# ------------------------------------------------------------------- direct
REC = {"fp64": 1, "fp32": 2, "fp16": 3, "bf16": 4, "fp16_fused": 5, "bf16_fused": 6}
IN = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.float64): 3}


def _in_code(X, bf16):
    return 2 if bf16 else IN[X.dtype]


def direct_pairs(rec, P, C, ii, jj, bf16_inputs=False):
    ii = _c(ii, np.int64)
    jj = _c(jj, np.int64)
    out = np.empty(ii.size, np.float64)
    if ii.size:
        lib().orc_direct_pairs(REC[rec], _in_code(P, bf16_inputs), _p(P), _p(C), P.shape[1], _p(ii), _p(jj),
                               ii.size, _p(out))
    return out


def direct_all(P, C, bf16_inputs=False):
    out = np.empty((P.shape[0], C.shape[0]), np.float64)
    lib().orc_direct_all(_in_code(P, bf16_inputs), _p(P), _p(C), P.shape[0], C.shape[0], P.shape[1], _p(out))
    return out


# ----------------------------------------------------------- form and flag
def _form_f32(S, pp, cc):
    """d = max((pp - 2 s) + cc, 0) in fp32 (form_mixed_and_list_*, euclidean_kernels_mix.cu:203-205)."""
    with np.errstate(invalid="ignore", over="ignore"):
        d = (pp[:, None] - np.float32(2.0) * S) + cc[None, :]
        d = np.where(np.isnan(d), np.float32(0.0), d)  # fmaxf(NaN, 0) = 0
        return np.maximum(d, np.float32(0.0)).astype(np.float32)


def _k_float(kform, kappa, dim, u):
    kappa = np.float32(kappa)
    u = np.float32(u)
    if kform == 0:  # kappa * ((float)(2*dim+4) * u), euclidean_kernels_mix.cu:207-211
        return np.float32(kappa * np.float32(np.float32(2 * dim + 4) * u))
    # (kappa * 2) * (dim * u), euclidean_kernels.cu:71 and euclidean_kernels_mix.cu:930-931
    return np.float32(np.float32(kappa * np.float32(2.0)) * np.float32(np.float32(dim) * u))


def _flag_f32(d, pp, cc, K):
    with np.errstate(invalid="ignore", over="ignore"):
        eps = np.float32(K) * (pp[:, None] + cc[None, :])
        return d <= eps


# Operator recipes: (gemm/low precision, S rounded to low?, norm mode, u, kform, recompute).
# The fp16/bf16-arithmetic recompute (direct_fp16_on_list / direct_bf16_on_list,
# euclidean_kernels_mix.cu:412-469) is `acc = __hadd(acc, __hmul(diff, diff))`; nvcc
# built for sm_100 contracts the product and the sum into one rounding, and the
# reference's own outputs on a B200 (tests/golden) match that sequence bit for bit.
MIX = {
    "fp16_fp64": ("fp16", True, "low_fp16", 2.0 ** -11, 0, "fp64"),   # euclidean_kernels_mix.cu:515
    "bf16_fp64": ("bf16", True, "low_bf16", 2.0 ** -7, 0, "fp64"),    # :584
    "tf32_fp64": ("tf32", False, "fma", 2.0 ** -11, 0, "fp64"),       # :648
    "fp32_fp64": ("fp32", False, "fma", 2.0 ** -23, 1, "fp64"),       # :918
    "fp16_fp16": ("fp16", True, "low_fp16", 2.0 ** -11, 0, "fp16_fused"),   # :1041
    "fp16_fp32": ("fp16", True, "low_fp16", 2.0 ** -11, 0, "fp32"),   # :1163
    "bf16_bf16": ("bf16", True, "low_bf16", 2.0 ** -7, 0, "bf16_fused"),    # :1284
    "bf16_fp32": ("bf16", True, "low_bf16", 2.0 ** -7, 0, "fp32"),    # :1405
    "fp32_fp32": ("fp32", False, "fma", 2.0 ** -23, 0, "fp32"),       # :1525
}
# euclidean_kernels_tiled.cu:440-528 (u_bf16 = 2^-8 there) and euclidean_kernels_tiled_tc.cu:274-300
TILED = {
    "fp16_fp64": ("fp16", 2.0 ** -11, "fp64"), "fp16_fp32": ("fp16", 2.0 ** -11, "fp32"),
    "bf16_fp64": ("bf16", 2.0 ** -8, "fp64"), "bf16_fp32": ("bf16", 2.0 ** -8, "fp32"),
    "fp32_fp64": ("fp32", 2.0 ** -23, "fp64"), "fp32_fp32": ("fp32", 2.0 ** -23, "fp32"),
}


def _low_s(P, C, low):
    if low == "fp32":
        return gemm_f32(P, C)
    r = LOW_ROUND[low]
    return gemm_f32(r(P), r(C))


def mix(name, P, C, kappa=5.0, S=None):
    """pairwise_euclidean_<name> (euclidean_kernels_mix.cu): returns (D, flag mask, n flagged).
    `S` optionally supplies the GEMM result (to check everything downstream of it)."""
    low, s_round, nmode, u, kform, rec = MIX[name]
    P = _c(P, np.float32)
    C = _c(C, np.float32)
    n, dim = P.shape
    pp, cc = norms_f32(P, nmode), norms_f32(C, nmode)
    if S is None:
        S = _low_s(P, C, low)
    if s_round:
        S = LOW_ROUND[low](S)  # cuBLAS writes S in the low precision (mix.cu:538)
    d = _form_f32(S, pp, cc)
    flag = _flag_f32(d, pp, cc, _k_float(kform, kappa, dim, u))
    ii, jj = np.nonzero(flag)
    D = d.copy()
    D[ii, jj] = direct_pairs(rec, P, C, ii, jj).astype(np.float32)
    return D, flag, int(flag.sum())


def tiled(name, P, C, kappa, S=None, tile=32):
    """pairwise_euclidean_tiled_<name> and pairwise_euclidean_tensorcore_<name>:
    norms are (P*P).sum(1) in fp32, S is the fp32-accumulated product of the low inputs
    (not rounded), the recompute reads the fp32 originals.  Returns (D, flag, count,
    per-tile counts in the reference's tile order)."""
    low, u, rec = TILED[name]
    P = _c(P, np.float32)
    C = _c(C, np.float32)
    n, dim = P.shape
    m = C.shape[0]
    pp, cc = norms_f32(P, "sumsq"), norms_f32(C, "sumsq")
    if S is None:
        S = _low_s(P, C, low)
    d = _form_f32(S, pp, cc)
    flag = _flag_f32(d, pp, cc, _k_float(0, kappa, dim, u))
    ii, jj = np.nonzero(flag)
    D = d.copy()
    D[ii, jj] = direct_pairs(rec, P, C, ii, jj).astype(np.float32)
    tn, tm = -(-n // tile), -(-m // tile)
    tiles = np.zeros(tn * tm, np.int64)
    np.add.at(tiles, (ii // tile) * tm + jj // tile, 1)
    return D, flag, int(flag.sum()), tiles


def single(P, C, S=None):
    """pairwise_euclidean_single (euclidean_kernels.cu:83-118)."""
    P, C = _c(P, np.float32), _c(C, np.float32)
    pp, cc = norms_f32(P, "fma"), norms_f32(C, "fma")
    if S is None:
        S = gemm_f32(P, C)
    return _form_f32(S, pp, cc)


def double(P, C, S=None):
    """pairwise_euclidean_double (euclidean_kernels.cu:120-152)."""
    P, C = _c(P, np.float64), _c(C, np.float64)
    pp, cc = norms_f64(P), norms_f64(C)
    if S is None:
        S = gemm_f64(P, C)
    d = (pp[:, None] - 2.0 * S) + cc[None, :]
    return np.where(d < 0.0, 0.0, d)


def uniform(name, P, C, S=None):
    """pairwise_euclidean_uniform_* (euclidean_kernels_uniform.cu:138-532).  fp16 inputs
    are float16 arrays, bf16 inputs are uint16 bit patterns; returns D in the op's type
    (bf16 as uint16 bits)."""
    if name == "fp16":
        P16, C16 = np.asarray(P, np.float16), np.asarray(C, np.float16)
        Pf, Cf = P16.astype(np.float32), C16.astype(np.float32)
        pp, cc = norms_f32(Pf, "low_fp16"), norms_f32(Cf, "low_fp16")
        if S is None:
            S = gemm_f32(Pf, Cf)
        S = round_f16(S)
        return _form_f32(S, pp, cc).astype(np.float16)
    if name == "bf16":
        Pf, Cf = bf16_from_bits(P), bf16_from_bits(C)
        pp, cc = norms_f32(Pf, "low_bf16"), norms_f32(Cf, "low_bf16")
        if S is None:
            S = gemm_f32(Pf, Cf)
        S = round_bf16(S)
        return bf16_bits(_form_f32(S, pp, cc))
    if name == "tf32":
        return single(P, C, S)
    if name in ("fp16_direct", "fp32_direct", "tf32_direct", "fp64_direct"):
        D = direct_all(np.ascontiguousarray(P), np.ascontiguousarray(C))
        return D.astype({"fp16_direct": np.float16, "fp64_direct": np.float64}.get(name, np.float32))
    if name == "bf16_direct":
        D = direct_all(_c(P, np.uint16), _c(C, np.uint16), bf16_inputs=True)
        return bf16_bits(D.astype(np.float32))
    raise KeyError(name)


def advanced(name, P, C, kappa=5.0, S=None):
    """pairwise_euclidean_fp64_* (euclidean_kernels_advanced.cu:225-453); returns (D, count)."""
    dim = P.shape[1]
    if name in ("fp64_fp16", "fp64_bf16"):
        bf = name == "fp64_bf16"
        Pf = bf16_from_bits(P) if bf else np.asarray(P, np.float16).astype(np.float32)
        Cf = bf16_from_bits(C) if bf else np.asarray(C, np.float16).astype(np.float32)
        pp, cc = norms_f32(Pf, "fma"), norms_f32(Cf, "fma")
        if S is None:
            S = gemm_f64(Pf.astype(np.float64), Cf.astype(np.float64))
        d64 = (pp.astype(np.float64)[:, None] - 2.0 * S) + cc.astype(np.float64)[None, :]
        d = np.maximum(d64, 0.0).astype(np.float32)
        flag = _flag_f32(d, pp, cc, _k_float(1, kappa, dim, 2.0 ** -23))
        ii, jj = np.nonzero(flag)
        D = d.copy()
        D[ii, jj] = direct_pairs("fp64", _c(P, np.uint16) if bf else np.asarray(P, np.float16),
                                 _c(C, np.uint16) if bf else np.asarray(C, np.float16), ii, jj,
                                 bf16_inputs=bf).astype(np.float32)
        return D, int(flag.sum())
    # fp64_tf32 (fp32 inputs) / fp64_fp32_gemm (fp64 inputs): fp64 norms, fp32 GEMM
    P64, C64 = np.asarray(P, np.float64), np.asarray(C, np.float64)
    pp, cc = norms_f64(P64), norms_f64(C64)
    if S is None:
        S = gemm_f32(P64.astype(np.float32), C64.astype(np.float32))
    d = (pp[:, None] - 2.0 * S.astype(np.float64)) + cc[None, :]
    d = np.maximum(d, 0.0)
    K = (np.float64(np.float32(kappa)) * 2.0) * (np.float64(dim) * 2.0 ** -52)
    flag = d <= K * (pp[:, None] + cc[None, :])
    ii, jj = np.nonzero(flag)
    D = d.copy()
    D[ii, jj] = direct_pairs("fp64", P64, C64, ii, jj)
    return D, int(flag.sum())


# ------------------------------------------------------------------ argmin
def argmin_first(D):
    """torch.argmin(D, 1): index of the first minimum of each row."""
    return np.argmin(D, axis=1).astype(np.int64)


def certified_argmin(name, P, C):
    """The certified argmin of operator `name` (a MIX or TILED key whose recompute is
    fp32 or fp64): label = first index of the smallest direct distance over all
    centers in the operator's recompute arithmetic (direct_dist of the reference's
    fallback kernels, euclidean_kernels_mix.cu:156-177, 481-504), stored as fp32 as
    the operator stores a recomputed pair; returns (labels, min_dist).  Equal to
    argmin_first of the operator's D when every pair is flagged."""
    rec = MIX[name][5] if name in MIX else TILED[name.split("_", 1)[1]][2]
    if rec not in ("fp32", "fp64"):
        raise ValueError(f"{name}: the certified argmin needs an fp32 or fp64 recompute")
    P = _c(P, np.float32)
    C = _c(C, np.float32)
    n, m = P.shape[0], C.shape[0]
    ii = np.repeat(np.arange(n, dtype=np.int64), m)
    jj = np.tile(np.arange(m, dtype=np.int64), n)
    D = direct_pairs(rec, P, C, ii, jj).astype(np.float32).reshape(n, m)
    lab = argmin_first(D)
    return lab, D[np.arange(n), lab]


def top2_gap(D):
    part = np.partition(D, 1, axis=1)[:, :2]
    return part[:, 1] - part[:, 0]


# ----------------------------------------------------------------- centers
def update_centers(X, labels, k):
    """update_centers_fp32 / _fp64 (center_kernels.cu:101-139): sequential sums in the
    working precision; returns (centers, counts)."""
    labels = _c(labels, np.int64)
    if X.dtype == np.float64:
        X = _c(X, np.float64)
        out = np.empty((k, X.shape[1]), np.float64)
        cnt = np.empty(k, np.int64)
        lib().orc_centers_f64(_p(X), _p(labels), X.shape[0], X.shape[1], k, _p(out), _p(cnt))
    else:
        X = _c(X, np.float32)
        out = np.empty((k, X.shape[1]), np.float32)
        cnt = np.empty(k, np.int64)
        lib().orc_centers_f32(_p(X), _p(labels), X.shape[0], X.shape[1], k, _p(out), _p(cnt))
    return out, cnt


def center_stats(X, labels, k):
    """k x (dim+1) table: per-cluster sums (extended precision) and counts."""
    labels = _c(labels, np.int64)
    is64 = X.dtype == np.float64
    X = _c(X, np.float64 if is64 else np.float32)
    st = np.empty((k, X.shape[1] + 1), np.float64)
    lib().orc_center_stats(_p(X), int(is64), _p(labels), X.shape[0], X.shape[1], k, _p(st))
    return st


# ------------------------------------------------------------- k-means++
_GOLDEN_GAMMA = 0x9E3779B97F4A7C15
_M64 = (1 << 64) - 1


def seed_draw53(seed, s):
    """Top 53 bits of SplitMix64(seed + (s + 1) * golden gamma) (the published SplitMix64
    finaliser), as the engine's k-means++ draws them."""
    z = (seed + (s + 1) * _GOLDEN_GAMMA) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    z ^= z >> 31
    return z >> 11


def kmeanspp(X, k, seed=0):
    """Deterministic k-means++ seeding as euc_kmeanspp defines it: row 0 uniform, then
    D^2 sampling with the fp64 direct distance (dimension order), weights scaled to
    exact integers q = floor(D 2^S), S = 62 - ceil(log2 n) - (floor(log2 max D) + 1),
    target floor(r * sum q / 2^53), the first row whose running sum exceeds it; all
    weights 0 -> uniform.  Returns the int64 row indices."""
    n = X.shape[0]
    idx = [(seed_draw53(seed, 0) * n) >> 53]
    D = None
    lg = (n - 1).bit_length()  # ceil(log2 n)
    rows = np.arange(n)
    for s in range(1, k):
        d2 = direct_pairs("fp64", X, X, rows, np.full(n, idx[-1]))
        d2 = np.where(np.isnan(d2), 0.0, d2)
        D = d2 if D is None else np.fmin(D, d2)
        r = seed_draw53(seed, s)
        maxd = float(D.max())
        if maxd > 0.0:
            S = 62 - lg - int(np.frexp(maxd)[1])  # frexp exponent = floor(log2) + 1
            q = np.ldexp(D, S).astype(np.uint64)
            total = int(q.sum(dtype=np.uint64))
        else:
            total = 0
        if total == 0:
            idx.append((r * n) >> 53)
            continue
        t = (r * total) >> 53
        run = np.cumsum(q, dtype=np.uint64)
        idx.append(int(np.searchsorted(run, np.uint64(t), side="right")))
    return np.asarray(idx, np.int64)


# ------------------------------------------------------------ CPU baseline
def dist_argmin_f64(P, C, threads=0):
    """fp64 distance + argmin on the host cores; returns (labels, min dist, threads used)."""
    P, C = _c(P, np.float64), _c(C, np.float64)
    lab = np.empty(P.shape[0], np.int64)
    md = np.empty(P.shape[0], np.float64)
    used = lib().orc_dist_argmin_f64(_p(P), _p(C), P.shape[0], C.shape[0], P.shape[1], _p(lab), _p(md), threads)
    return lab, md, used


def lloyd_step_f64(X, C, threads=0):
    """One fp64 Lloyd iteration on the host cores (CPU baseline): returns (new centers,
    labels, threads used, ms of the per-row part, ms of the reduction and means)."""
    X, C = _c(X, np.float64), _c(C, np.float64)
    lab = np.empty(X.shape[0], np.int64)
    out = np.empty_like(C)
    ms = np.zeros(2, np.float64)
    used = lib().orc_lloyd_step_f64(_p(X), _p(C), X.shape[0], C.shape[0], X.shape[1], _p(lab), _p(out), threads,
                                    _p(ms))
    return out, lab, used, float(ms[0]), float(ms[1])


def max_threads():
    return lib().orc_max_threads()
