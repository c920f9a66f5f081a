"""The C ABI library (no GPU needed): it loads, exports every entry point declared
in include/euclid_b200.h, and its host-only queries behave.  No compute call is
made here."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "euclid_b200.h")
LIB = os.path.join(REPO, "euclid-cuda_b200", "libeuclid_b200.so")


def declared():
    src = open(HEADER).read()
    names = set(re.findall(r"EUC_API\s+[\w\s\*]+?\b(euc_\w+)\s*\(", src))
    names |= set(re.findall(r"EUC_(?:MIX|TILED|TC)_DECL\((euc_\w+)\)", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        import subprocess
        import sys
        subprocess.run([sys.executable, os.path.join(REPO, "euclid-cuda_b200", "build.py")], check=True)
    return ctypes.CDLL(LIB)


def test_header_declares_the_reference_surface():
    names = declared()
    # one entry per reference operator family member: 2 base + 9 mix + 6 tiled +
    # 4 tensorcore + 8 uniform + 4 advanced + 2 centers, plus counter reads and new entries
    for fam, n in (("euc_mix_", 9), ("euc_tiled_", 6), ("euc_tensorcore_", 4), ("euc_uniform_", 8),
                   ("euc_advanced_", 4), ("euc_update_centers_", 2), ("euc_pairwise_", 2)):
        assert sum(x.startswith(fam) for x in names) == n, fam
    assert "euc_argmin" in names and "euc_center_stats" in names and "euc_center_finalize" in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    import sys
    sys.path.insert(0, os.path.join(REPO, "euclid-cuda_b200"))
    import _lib
    assert set(declared()) <= set(_lib.exported_symbols()) | {"euc_device_check"}


def test_host_queries(lib):
    lib.euc_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.euc_version()
    lib.euc_status_string.restype = ctypes.c_char_p
    assert lib.euc_status_string(6) == b"workspace too small"
    lib.euc_workspace_bytes.restype = ctypes.c_size_t
    lib.euc_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
    # fp16 tensor-core op: norms + padded fp16 copies (dim 100 -> 128) + flag list
    n, m, d = 1000, 300, 100
    ws = lib.euc_workspace_bytes(10, n, m, d)
    assert ws >= n * 128 * 2 + m * 128 * 2 + (n + m) * 4
    # direct operators need no workspace; unknown ids report 0
    assert lib.euc_workspace_bytes(46, n, m, d) == 0
    assert lib.euc_workspace_bytes(999, n, m, d) == 0
    lib.euc_argmin_workspace_bytes.restype = ctypes.c_size_t
    lib.euc_argmin_workspace_bytes.argtypes = lib.euc_workspace_bytes.argtypes
    # the fused argmin adds the norm-sorted centers (copy, and norms and original index
    # padded to 256-center tiles), per-CTA list counts, a redo byte per point, the
    # candidate-chunk list and a 64-bit row key per point
    al = lambda b: (b + 255) // 256 * 256
    mpad = (m + 255) // 256 * 256
    ccap = min(n * ((m + 31) // 32), max(2 * n, 1 << 16))  # candidate chunks: entry + 32 fp32 accumulators
    # plus the centers' extra-K rows of the screening MMA (32 bytes per sorted center)
    assert lib.euc_argmin_workspace_bytes(10, n, m, d) == (ws + al(m * 128 * 2) + 2 * al(mpad * 4) + al(1024 * 4)
                                                           + al(n) + al(mpad * 32) + al(ccap * 8)
                                                           + al(ccap * 128) + al(n * 8))


def test_compute_entry_rejects_missing_device(lib):
    """Without a GPU every compute entry returns EUC_ERR_DEVICE before touching memory."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    lib.euc_argmin.restype = ctypes.c_int
    lib.euc_last_error.restype = ctypes.c_char_p
    rc = lib.euc_argmin(15, None, None, ctypes.c_int64(10), ctypes.c_int64(10), ctypes.c_int64(4),
                        ctypes.c_float(5.0), 0, None, None, None, None, None, ctypes.c_size_t(0), None)
    assert rc == 8
    assert b"sm_100" in lib.euc_last_error()


def test_kmeanspp_entry_checks_shapes_before_the_device(lib):
    """euc_kmeanspp rejects k outside [1, n] with EUC_ERR_SHAPE, and otherwise needs an
    sm_100 device; the workspace is one fp64 weight per row plus block sums."""
    import torch
    lib.euc_kmeanspp.restype = ctypes.c_int
    lib.euc_kmeanspp.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                 ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                 ctypes.c_void_p]
    lib.euc_kmeanspp_workspace_bytes.restype = ctypes.c_size_t
    lib.euc_kmeanspp_workspace_bytes.argtypes = [ctypes.c_int64] * 3
    al = lambda b: (b + 255) // 256 * 256
    n = 5000
    assert lib.euc_kmeanspp_workspace_bytes(n, 8, 10) == al(n * 8) + al(((n + 1023) // 1024) * 8) + 256
    for k in (0, n + 1):
        assert lib.euc_kmeanspp(None, 0, n, 8, k, 1, None, None, None, 0, None) == 1  # EUC_ERR_SHAPE
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert lib.euc_kmeanspp(ctypes.c_void_p(16), 0, n, 8, 10, 1, ctypes.c_void_p(16), None, ctypes.c_void_p(16),
                            1 << 20, None) == 8  # EUC_ERR_DEVICE


def test_noalloc_entry_checks_arguments_before_the_scratch(lib):
    """euc_argmin_noalloc checks its arguments before the scratch-size test and before it
    takes the array's address: an unknown operator is EUC_ERR_ARG, a negative size
    EUC_ERR_SHAPE (not a wrapped, huge workspace), and without an sm_100 device a valid
    call is EUC_ERR_DEVICE (no module load is attempted)."""
    import torch
    f = lib.euc_argmin_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    lib.euc_last_error.restype = ctypes.c_char_p
    assert f(999, None, None, 10, 10, 4, 5.0, 0, None, None, None, None, None) == 7  # EUC_ERR_ARG
    for n, m, d in ((-1, 10, 4), (10, -3, 4), (10, 10, -2)):
        assert f(15, None, None, n, m, d, 5.0, 0, None, None, None, None, None) == 1  # EUC_ERR_SHAPE
        assert b"negative" in lib.euc_last_error()
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert f(15, None, None, 10, 10, 4, 5.0, 0, None, None, None, None, None) == 8  # EUC_ERR_DEVICE
    assert b"sm_100" in lib.euc_last_error()


def test_prepared_points_sizes_and_checks(lib):
    """euc_prepared_points_bytes: the rounded copy (rows padded to whole 128-byte boxes)
    then fp32 norms, each 256-byte aligned; 0 for operators without a tensor-core GEMM.
    euc_prepare_points rejects bad sizes before the device check."""
    import torch
    al = lambda b: (b + 255) // 256 * 256
    f = lib.euc_prepared_points_bytes
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int64]
    assert f(17, 1000, 70) == al(1000 * 128 * 2) + al(1000 * 4)    # bf16_fp32: 70 -> 128 per row
    assert f(12, 1000, 70) == al(1000 * 96 * 4) + al(1000 * 4)     # tf32_fp64: 70 -> 96 per row
    assert f(18, 1000, 70) == 0                                    # fp32_fp32: CUDA-core GEMM
    g = lib.euc_prepare_points
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t,
                  ctypes.c_void_p]
    assert g(17, None, -1, 8, None, 0, None) == 1   # EUC_ERR_SHAPE
    assert g(18, None, 10, 8, None, 0, None) == 3   # EUC_ERR_UNSUPPORTED
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert g(17, ctypes.c_void_p(16), 10, 8, ctypes.c_void_p(16), 1 << 20, None) == 8  # EUC_ERR_DEVICE
