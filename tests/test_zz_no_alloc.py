"""euc_argmin_noalloc (static device scratch, no allocation) against euc_argmin (caller
workspace), both called through the C ABI on the same inputs.

Both run the same kernels on the same inputs, so the tolerance is zero: labels,
min_dist and the flag count must be identical, on two calls in a row (the second call
reuses the scratch the first one left behind).  Shapes whose workspace exceeds the
static scratch are rejected with EUC_ERR_WORKSPACE before any launch.
"""
import ctypes

import pytest
import torch

from _lib import lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EUC_ERR_WORKSPACE = 6
# (op id, exact): fp16 tensor-core mix op (fast screen, exact epilogue, certified
# labels), the bf16 one (fast, certified), and the fp32 CUDA-core mix op
CASES = [(15, 0), (15, 1), (15, 2), (17, 0), (17, 2), (18, 1)]


def _inputs(n, m, d, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    C = torch.randn(m, d, generator=g, device=DEV)
    lab = torch.randint(0, m, (n,), generator=g, device=DEV)
    P = C[lab] + 0.05 * torch.randn(n, d, generator=g, device=DEV)
    return P.contiguous(), C.contiguous()


def _outs(n):
    return (torch.full((n,), -1, dtype=torch.int64, device=DEV), torch.full((n,), -1, dtype=torch.int32, device=DEV),
            torch.full((n,), float("nan"), dtype=torch.float32, device=DEV),
            torch.zeros(1, dtype=torch.int64, device=DEV))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("op,exact", CASES)
def test_noalloc_matches_workspace_entry(op, exact):
    L = lib()
    n, m, d, kappa = 3001, 517, 100, 5.0
    P, C = _inputs(n, m, d, seed=op * 10 + exact)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws_bytes = L.euc_argmin_workspace_bytes(op, n, m, d)
    assert 0 < ws_bytes <= L.euc_argmin_noalloc_max_bytes()
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    lab, lab32, md, cnt = _outs(n)
    rc = L.euc_argmin(op, _p(P), _p(C), n, m, d, kappa, exact, _p(lab), _p(lab32), _p(md), _p(cnt), _p(ws),
                      ws_bytes, stream)
    assert rc == 0, L.euc_last_error()
    torch.cuda.synchronize()
    for call in range(2):
        lab_s, lab32_s, md_s, cnt_s = _outs(n)
        rc = L.euc_argmin_noalloc(op, _p(P), _p(C), n, m, d, kappa, exact, _p(lab_s), _p(lab32_s), _p(md_s),
                                  _p(cnt_s), stream)
        assert rc == 0, L.euc_last_error()
        torch.cuda.synchronize()
        assert torch.equal(lab_s, lab), call
        assert torch.equal(lab32_s, lab32), call
        assert torch.equal(md_s, md), call
        assert int(cnt_s.item()) == int(cnt.item()), call
    assert ((lab >= 0) & (lab < m)).all()


def test_noalloc_rejects_oversized_shape():
    L = lib()
    op, m, d = 15, 1024, 128
    cap = L.euc_argmin_noalloc_max_bytes()
    n = 1 << 20  # fp16 copies alone need 2^20 * 128 * 2 bytes = 256 MiB
    assert L.euc_argmin_workspace_bytes(op, n, m, d) > cap
    lab = torch.full((4,), -7, dtype=torch.int64, device=DEV)
    null = ctypes.c_void_p(0)
    rc = L.euc_argmin_noalloc(op, null, null, n, m, d, 5.0, 0, _p(lab), null, null, null,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == EUC_ERR_WORKSPACE
    assert b"static scratch" in L.euc_last_error()
    torch.cuda.synchronize()
    assert (lab == -7).all()  # nothing launched


def _with_workspace(L, op, P, C, exact, kappa, stream):
    """euc_argmin on a freshly allocated workspace filled with junk bytes."""
    n, d = P.shape
    m = C.shape[0]
    ws_bytes = L.euc_argmin_workspace_bytes(op, n, m, d)
    ws = torch.full((ws_bytes,), 0xAB, dtype=torch.uint8, device=DEV)
    out = _outs(n)
    lab, lab32, md, cnt = out
    rc = L.euc_argmin(op, _p(P), _p(C), n, m, d, kappa, exact, _p(lab), _p(lab32), _p(md), _p(cnt), _p(ws),
                      ws_bytes, stream)
    assert rc == 0, L.euc_last_error()
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("op,exact", [(15, 0), (15, 2)])
def test_noalloc_after_larger_and_smaller_calls(op, exact):
    """A call after a larger one (whose leftovers fill the scratch) and after a smaller one
    gives the same outputs as euc_argmin on a fresh workspace: nothing of an earlier
    call's scratch leaks into a later result."""
    L = lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    shapes = [(40000, 700, 96), (1000, 40, 16), (40000, 700, 96), (777, 300, 64)]
    for i, (n, m, d) in enumerate(shapes):
        assert L.euc_argmin_workspace_bytes(op, n, m, d) <= L.euc_argmin_noalloc_max_bytes()
        P, C = _inputs(n, m, d, seed=100 + i)
        ref = _with_workspace(L, op, P, C, exact, 5.0, stream)
        got = _outs(n)
        rc = L.euc_argmin_noalloc(op, _p(P), _p(C), n, m, d, 5.0, exact, *(_p(t) for t in got), stream)
        assert rc == 0, L.euc_last_error()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b), (i, n, m, d)
