"""ctypes binding of libeuclid_b200.so (the C ABI in include/euclid_b200.h).

torch is used here only for device memory (outputs, workspace) and the current
CUDA stream.  There is no CPU fallback: if the library is missing or the device is
not an sm_100 part every call raises.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeuclid_b200.so")

# operator ids (euc_op in include/euclid_b200.h)
OPS = {
    "single": 0, "double": 1,
    "fp16_fp64": 10, "bf16_fp64": 11, "tf32_fp64": 12, "fp32_fp64": 13, "fp16_fp16": 14,
    "fp16_fp32": 15, "bf16_bf16": 16, "bf16_fp32": 17, "fp32_fp32": 18,
    "tiled_fp16_fp64": 20, "tiled_fp16_fp32": 21, "tiled_bf16_fp64": 22, "tiled_bf16_fp32": 23,
    "tiled_fp32_fp64": 24, "tiled_fp32_fp32": 25,
    "tensorcore_fp16_fp64": 30, "tensorcore_fp16_fp32": 31, "tensorcore_bf16_fp64": 32,
    "tensorcore_bf16_fp32": 33,
    "uniform_fp16": 40, "uniform_bf16": 41, "uniform_tf32": 42, "uniform_fp16_direct": 43,
    "uniform_bf16_direct": 44, "uniform_tf32_direct": 45, "uniform_fp32_direct": 46,
    "uniform_fp64_direct": 47,
    "fp64_fp16": 50, "fp64_bf16": 51, "fp64_tf32": 52, "fp64_fp32_gemm": 53,
    "centers_fp32": 60, "centers_fp64": 61,
}

_lib = None
_dev = None
_V, _I64, _I, _F, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

_SIGS = {
    "euc_version": ([], ctypes.c_char_p),
    "euc_status_string": ([_I], ctypes.c_char_p),
    "euc_last_error": ([], ctypes.c_char_p),
    "euc_device_check": ([], _I),
    "euc_workspace_bytes": ([_I, _I64, _I64, _I64], _SZ),
    "euc_argmin_workspace_bytes": ([_I, _I64, _I64, _I64], _SZ),
    "euc_set_kernel_timing": ([_I], None),
    "euc_set_wait_limit_ns": ([ctypes.c_uint64], None),
    "euc_test_withhold_arrival": ([], None),
    "euc_set_screen_pairs": ([_I], None),
    "euc_last_kernel_ms": ([], ctypes.c_float),
    "euc_last_kernel_name": ([], ctypes.c_char_p),
    "euc_pairwise_single": ([_V, _V, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_pairwise_double": ([_V, _V, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_uniform_fp16": ([_V, _V, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_uniform_bf16": ([_V, _V, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_uniform_tf32": ([_V, _V, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_read_count_i32": ([_V, _V], _I),
    "euc_read_count_u64": ([_V, _V], _I),
    "euc_update_centers_fp32": ([_V, _V, _I64, _I64, _I64, _V, _V, _V, _SZ, _V], _I),
    "euc_update_centers_fp64": ([_V, _V, _I64, _I64, _I64, _V, _V, _V, _SZ, _V], _I),
    "euc_argmin": ([_I, _V, _V, _I64, _I64, _I64, _F, _I, _V, _V, _V, _V, _V, _SZ, _V], _I),
    "euc_prepared_points_bytes": ([_I, _I64, _I64], _SZ),
    "euc_prepare_points": ([_I, _V, _I64, _I64, _V, _SZ, _V], _I),
    "euc_argmin_prepared_workspace_bytes": ([_I, _I64, _I64, _I64], _SZ),
    "euc_argmin_prepared": ([_I, _V, _V, _V, _I64, _I64, _I64, _F, _I, _V, _V, _V, _V, _V, _SZ, _V], _I),
    "euc_argmin_noalloc_max_bytes": ([], _SZ),
    "euc_argmin_noalloc": ([_I, _V, _V, _I64, _I64, _I64, _F, _I, _V, _V, _V, _V, _V], _I),
    "euc_center_stats_workspace_bytes": ([_I64, _I64, _I64], _SZ),
    "euc_center_stats": ([_V, _I, _V, _I, _I64, _I64, _I64, _V, _V, _SZ, _V], _I),
    "euc_center_finalize": ([_V, _I64, _I64, _V, _I, _V, _I, _V], _I),
    "euc_kmeanspp_workspace_bytes": ([_I64, _I64, _I64], _SZ),
    "euc_kmeanspp": ([_V, _I, _I64, _I64, _I64, ctypes.c_uint64, _V, _V, _V, _SZ, _V], _I),
}
for _n in ("fp16_fp64", "bf16_fp64", "tf32_fp64", "fp32_fp64", "fp16_fp16", "fp16_fp32", "bf16_bf16",
           "bf16_fp32", "fp32_fp32"):
    _SIGS["euc_mix_" + _n] = ([_V, _V, _I64, _I64, _I64, _F, _V, _V, _V, _SZ, _V], _I)
for _n in ("fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32", "fp32_fp64", "fp32_fp32"):
    _SIGS["euc_tiled_" + _n] = ([_V, _V, _I64, _I64, _I64, _F, _I, _V, _V, _V, _V, _SZ, _V], _I)
for _n in ("fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32"):
    _SIGS["euc_tensorcore_" + _n] = ([_V, _V, _I64, _I64, _I64, _F, _I, _V, _V, _V, _SZ, _V], _I)
for _n in ("fp16", "bf16", "tf32", "fp32", "fp64"):
    _SIGS["euc_uniform_%s_direct" % _n] = ([_V, _V, _I64, _I64, _I64, _V, _V], _I)
for _n in ("fp16", "bf16", "tf32"):
    _SIGS["euc_advanced_fp64_" + _n] = ([_V, _V, _I64, _I64, _I64, _F, _V, _V, _V, _SZ, _V], _I)
_SIGS["euc_advanced_fp64_fp32_gemm"] = ([_V, _V, _I64, _I64, _I64, _F, _V, _V, _V, _SZ, _V], _I)


def lib():
    """Load libeuclid_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"euclid_b200: {LIB_PATH} is missing; build it with "
                               "`python euclid-cuda_b200/build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(rc):
    if rc != 0:
        msg = lib().euc_last_error().decode() or lib().euc_status_string(rc).decode()
        raise RuntimeError(msg)


def _bind_device(t):
    # the library keeps its own CUDA runtime; make its current device match the tensor's
    global _dev
    d = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if _dev != d:
        torch.cuda.set_device(d)
        _dev = d


def stream_of(t):
    _bind_device(t)
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def device_check():
    """Synchronise and raise if a bounded device-side wait expired since the last check."""
    check(lib().euc_device_check())
