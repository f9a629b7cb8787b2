"""Locating and loading the native libraries of the package.

``libptparaconv2d.so`` registers ``torch.ops.ptparaconv2d`` (the reference
schema).  ``libpc2d_sm100.so`` holds the CUDA kernels behind the C ABI of
``include/paraconv2d.h``; :func:`cabi` binds it through ctypes for callers
that work with raw device pointers.

There is no fallback: if a library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
KERNEL_LIB = os.path.join(PKG_DIR, "libpc2d_sm100.so")
OP_LIB = os.path.join(PKG_DIR, "libptparaconv2d.so")

# pc2d_status / pc2d_dtype / pc2d_algo of include/paraconv2d.h
PC2D_OK = 0
PC2D_ERR_INVALID_ARGUMENT = 1
PC2D_ERR_UNSUPPORTED = 2
PC2D_ERR_WORKSPACE = 3
PC2D_ERR_CUDA = 4
PC2D_ERR_TIMEOUT = 5
PC2D_DTYPE_F32 = 0
PC2D_DTYPE_F64 = 1
PC2D_ALGO_AUTO = 0
PC2D_ALGO_SIMT = 1
PC2D_ALGO_TC = 2

_lock = threading.Lock()
_op_loaded = False
_cabi = None


class NativeLibraryMissing(ImportError):
    pass


def _require(path: str) -> str:
    if not os.path.exists(path):
        raise NativeLibraryMissing(
            f"{os.path.basename(path)} is not built; run `python paraconv2d_b200/build.py` "
            "(there is no CPU or Python fallback for this op)")
    return path


def load_op_library() -> None:
    """Registers torch.ops.ptparaconv2d from libptparaconv2d.so (once)."""
    global _op_loaded
    with _lock:
        if _op_loaded:
            return
        import torch

        _require(KERNEL_LIB)
        torch.ops.load_library(_require(OP_LIB))
        _op_loaded = True


def cabi() -> ctypes.CDLL:
    """ctypes binding of the C ABI in libpc2d_sm100.so (argument types set)."""
    global _cabi
    with _lock:
        if _cabi is not None:
            return _cabi
        lib = ctypes.CDLL(_require(KERNEL_LIB))
        I, L, D, P, S = ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_void_p, ctypes.c_size_t
        sig = {
            "pc2d_abi_version": ([], I),
            "pc2d_out_size": ([I, I, I, I], I),
            "pc2d_infer_m": ([L, I, I, I], L),
            "pc2d_set_algo": ([I], I),
            "pc2d_get_algo": ([], I),
            "pc2d_forward_workspace_size": ([I] * 12, S),
            "pc2d_forward": ([I, P, P, D] + [I] * 11 + [P, P, P, S, P], I),
            "pc2d_backward_workspace_size": ([I] * 13, S),
            "pc2d_backward": ([I, P, P, P, P, D] + [I] * 12 + [P, P, P, S, P], I),
            "pc2d_backward_interior": ([I, P, P, P, P, D] + [I] * 16 + [D, P, P, P, S, P], I),
            "pc2d_pad_scale": ([I, P] + [I] * 8 + [D, P, P], I),
            "pc2d_comm_handle_bytes": ([], S),
            "pc2d_comm_create": ([I, I, S, ctypes.POINTER(P), P], I),
            "pc2d_comm_connect": ([P, P], I),
            "pc2d_comm_destroy": ([P], I),
            "pc2d_backward_sum": ([P, I, P, P, P, P, D] + [I] * 12 + [P, P, P, S, P], I),
            "pc2d_comm_allreduce": ([P, P, P, S, P], I),
            "pc2d_param_step": ([I, P, P, P, I, I] + [D] * 6 + [I, P], I),
            "pc2d_status_string": ([I], ctypes.c_char_p),
            "pc2d_last_error": ([], ctypes.c_char_p),
            "pc2d_device_status": ([], I),
            "pc2d_clear_device_status": ([], I),
            "pc2d_selftest_bounded_wait": ([ctypes.c_uint, P], I),
            "pc2d_timing_enable": ([I], I),
            "pc2d_timing_reset": ([], I),
            "pc2d_timing_read": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int)], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _cabi = lib
        return lib


def status_message(st: int) -> str:
    lib = cabi()
    return f"{lib.pc2d_status_string(st).decode()}: {lib.pc2d_last_error().decode()}"


def set_algo(algo: int) -> int:
    """Process-wide kernel family (PC2D_ALGO_AUTO / _SIMT / _TC); returns the previous one."""
    prev = cabi().pc2d_set_algo(int(algo))
    if prev < 0:
        raise ValueError(f"invalid algo {algo}")
    return prev


def kernel_times(names=("forward", "dgrad", "wgrad", "simt_forward", "simt_dgrad", "simt_wgrad")):
    """{family: (total_ms, launches)} recorded since the last pc2d_timing_reset."""
    lib = cabi()
    out = {}
    for n in names:
        t = ctypes.c_double(0.0)
        c = ctypes.c_int(0)
        st = lib.pc2d_timing_read(n.encode(), ctypes.byref(t), ctypes.byref(c))
        if st != PC2D_OK:
            raise RuntimeError(status_message(st))
        out[n] = (t.value, c.value)
    return out
