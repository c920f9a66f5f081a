"""Shared validation and launch helpers behind the reference-named modules.

The checks and their messages mirror the reference's TORCH_CHECKs (a failed check
raises RuntimeError, as TORCH_CHECK does), e.g.
CHECK_CUDA / CHECK_CONTIGUOUS (euclidean_kernels_mix.cu:17-19), the dtype and
rank checks (euclidean_kernels_mix.cu:518-525) and the tiled/tensor-core tile rules
(euclidean_kernels_tiled.cu:331-336, euclidean_kernels_tiled_tc.cu:246-248).
Differences, by design: outputs are produced asynchronously on the current stream
(the reference ends every op with cudaDeviceSynchronize), and the reference's
size limits (N*M <= 2^32, smem <= 48 KiB) do not exist here.
"""
import ctypes

import torch

from _lib import OPS, check, lib, ptr, stream_of, workspace

_TORCH_DT = {"fp32": torch.float32, "fp64": torch.float64, "fp16": torch.float16, "bf16": torch.bfloat16}
_DT_NAME = {torch.float32: "float32", torch.float64: "float64", torch.float16: "float16",
            torch.bfloat16: "bfloat16"}


def check_input(t, name, cuda_msg="must be a CUDA tensor"):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} {cuda_msg}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def check_pair(P, C, dtype, rank_msg="Inputs must be 2D", dim_msg="Dimension mismatch",
               cuda_msg="must be a CUDA tensor", dtype_first=False):
    if dtype_first:  # tiled / tensorcore: CHECK_INPUT includes the float32 check
        for t, nm in ((P, "P"), (C, "C")):
            check_input(t, nm, cuda_msg)
            if t.dtype != dtype:
                raise RuntimeError(f"{nm} must be {_DT_NAME[dtype]}")
    else:
        check_input(P, "P", cuda_msg)
        check_input(C, "C", cuda_msg)
        if P.dtype != dtype:
            raise RuntimeError(f"P must be {_DT_NAME[dtype]}")
        if C.dtype != dtype:
            raise RuntimeError(f"C must be {_DT_NAME[dtype]}")
    if P.dim() != 2 or C.dim() != 2:
        raise RuntimeError(rank_msg)
    if C.size(1) != P.size(1):
        raise RuntimeError(dim_msg)
    if P.device != C.device:
        raise RuntimeError("P and C must be on the same device")


def _count_value(cnt):
    return int(cnt.item())


def run_mix(name, P, C, kappa, with_stats):
    check_pair(P, C, torch.float32)
    n, d = P.shape
    m = C.size(0)
    D = torch.empty((n, m), dtype=torch.float32, device=P.device)
    cnt = torch.zeros(1, dtype=torch.int64, device=P.device)
    ws = workspace(lib().euc_workspace_bytes(OPS[name], n, m, d), P.device)
    st = stream_of(P)
    fn = getattr(lib(), "euc_mix_" + name)
    check(fn(ptr(P), ptr(C), n, m, d, ctypes.c_float(kappa), ptr(D), ptr(cnt), ptr(ws), ws.numel(), st))
    if with_stats:
        return D, _count_value(cnt)
    return D


def run_tiled(name, P, C, kappa, tile_size, with_stats):
    check_pair(P, C, torch.float32, rank_msg="P and C must be 2D", dim_msg="dimension mismatch",
               cuda_msg="must be CUDA tensor", dtype_first=True)
    n, d = P.shape
    m = C.size(0)
    T = tile_size if tile_size > 0 else (32 if d <= 128 else 16)
    D = torch.empty((n, m), dtype=torch.float32, device=P.device)
    cnt = torch.zeros(1, dtype=torch.int64, device=P.device)
    tiles = None
    if with_stats and T in (16, 32):
        tiles = torch.zeros(((n + T - 1) // T) * ((m + T - 1) // T), dtype=torch.int32, device=P.device)
    ws = workspace(lib().euc_workspace_bytes(OPS["tiled_" + name], n, m, d), P.device)
    st = stream_of(P)
    fn = getattr(lib(), "euc_tiled_" + name)
    check(fn(ptr(P), ptr(C), n, m, d, ctypes.c_float(kappa), int(tile_size), ptr(D), ptr(tiles), ptr(cnt),
             ptr(ws), ws.numel(), st))
    if with_stats:
        per_tile = tiles.cpu().tolist() if tiles is not None else []
        return D, int(sum(per_tile)), per_tile
    return D


def run_tensorcore(name, P, C, kappa, tile_size):
    check_pair(P, C, torch.float32, rank_msg="P and C must be 2D", dim_msg="dimension mismatch",
               dtype_first=True)
    n, d = P.shape
    m = C.size(0)
    D = torch.empty((n, m), dtype=torch.float32, device=P.device)
    ws = workspace(lib().euc_workspace_bytes(OPS["tensorcore_" + name], n, m, d), P.device)
    st = stream_of(P)
    fn = getattr(lib(), "euc_tensorcore_" + name)
    check(fn(ptr(P), ptr(C), n, m, d, ctypes.c_float(kappa), int(tile_size), ptr(D), None, ptr(ws), ws.numel(),
             st))
    return D


def run_plain(cname, opname, P, C, dtype, out_dtype=None):
    check_pair(P, C, dtype)
    n, d = P.shape
    m = C.size(0)
    D = torch.empty((n, m), dtype=out_dtype or dtype, device=P.device)
    st = stream_of(P)
    fn = getattr(lib(), cname)
    if opname is None:  # direct operators take no workspace
        check(fn(ptr(P), ptr(C), n, m, d, ptr(D), st))
    else:
        ws = workspace(lib().euc_workspace_bytes(OPS[opname], n, m, d), P.device)
        check(fn(ptr(P), ptr(C), n, m, d, ptr(D), ptr(ws), ws.numel(), st))
    return D


def run_advanced(name, P, C, kappa, in_dtype, out_dtype):
    check_pair(P, C, in_dtype)
    n, d = P.shape
    m = C.size(0)
    D = torch.empty((n, m), dtype=out_dtype, device=P.device)
    cnt = torch.zeros(1, dtype=torch.int64, device=P.device)
    ws = workspace(lib().euc_workspace_bytes(OPS[name], n, m, d), P.device)
    st = stream_of(P)
    fn = getattr(lib(), "euc_advanced_" + name)
    check(fn(ptr(P), ptr(C), n, m, d, ctypes.c_float(kappa), ptr(D), ptr(cnt), ptr(ws), ws.numel(), st))
    _LAST_COUNT[0] = cnt
    return D


_LAST_COUNT = [None]


ARGMIN_CERTIFIED = 2  # EUC_ARGMIN_CERTIFIED


def prepare_points(op_name, P):
    """The points' low-precision copy and norms for tensor-core operator `op_name`
    (euc_prepare_points): a uint8 device buffer for run_argmin(..., prepared=...)."""
    check_input(P, "P")
    if P.dtype != torch.float32 or P.dim() != 2:
        raise RuntimeError("P must be a 2D float32 tensor")
    P = P.contiguous()
    n, d = P.shape
    nbytes = lib().euc_prepared_points_bytes(OPS[op_name], n, d)
    if nbytes == 0 and n > 0:
        raise RuntimeError(f"{op_name}: no prepared points (tensor-core operators only)")
    buf = workspace(nbytes, P.device)
    check(lib().euc_prepare_points(OPS[op_name], ptr(P), n, d, ptr(buf), buf.numel(), stream_of(P)))
    return buf


def run_argmin(op_name, P, C, kappa=5.0, exact=False, labels_dtype=torch.int64, min_dist=True, prepared=None):
    """Fused distance + argmin for distance operator `op_name` (a key of _lib.OPS):
    returns (labels, min_dist, flagged-pair count as a 0-d device tensor).  `exact`
    True selects the epilogue that forms every distance exactly as the D-producing
    operator does; "certified" labels every row with the first index of its smallest
    direct distance in the operator's recompute arithmetic, recomputing only the
    centers that can win, and the count is then the number of direct distances taken
    (see euc_argmin in include/euclid_b200.h)."""
    want = torch.float64 if op_name == "double" else torch.float32
    check_pair(P, C, want)
    n, d = P.shape
    m = C.size(0)
    dev = P.device
    labels = torch.empty(n, dtype=labels_dtype, device=dev)
    md = torch.empty(n, dtype=want, device=dev) if min_dist else None
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    st = stream_of(P)
    l64 = labels if labels_dtype == torch.int64 else None
    l32 = labels if labels_dtype == torch.int32 else None
    mode = ARGMIN_CERTIFIED if isinstance(exact, str) and exact == "certified" else int(bool(exact))
    if prepared is not None:
        ws = workspace(lib().euc_argmin_prepared_workspace_bytes(OPS[op_name], n, m, d), dev)
        check(lib().euc_argmin_prepared(OPS[op_name], ptr(P), ptr(prepared), ptr(C), n, m, d, ctypes.c_float(kappa),
                                        mode, ptr(l64), ptr(l32), ptr(md), ptr(cnt), ptr(ws), ws.numel(), st))
        return labels, md, cnt[0]
    ws = workspace(lib().euc_argmin_workspace_bytes(OPS[op_name], n, m, d), dev)
    check(lib().euc_argmin(OPS[op_name], ptr(P), ptr(C), n, m, d, ctypes.c_float(kappa), mode,
                           ptr(l64), ptr(l32),
                           ptr(md), ptr(cnt), ptr(ws), ws.numel(), st))
    return labels, md, cnt[0]


def read_count_i32(t):
    """get_fallback_count_low / get_last_fallback_count: first int32 of a device tensor."""
    check_input(t, "list_count_tensor")
    out = ctypes.c_int32(0)
    check(lib().euc_read_count_i32(ptr(t), ctypes.byref(out)))
    return int(out.value)
