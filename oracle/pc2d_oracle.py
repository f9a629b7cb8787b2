"""ORACLE -- test infrastructure only.

ctypes front end of ``oracle/pc2d_oracle.c`` (a plain-C restatement of the
reference CPU op, GeoND-tech/ParaConv2d ``paraconv2d.cc:70-239``) and loader
of the reference op built from its own source (``oracle/build_ref.sh``).

All arrays are numpy, C-contiguous, float32 or float64.  ``pars`` is the flat
``[h0 | h | p | p0]`` vector of the reference (``paraconv2d.cc:23-37``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "pc2d_oracle.c")
_LIB_DIR = os.path.join(_HERE, "_build")
_LIB = os.path.join(_LIB_DIR, "libpc2d_oracle.so")
REF_LIB = os.path.join(_HERE, "_ref", "libptparaconv2d_ref.so")

_lib: Optional[ctypes.CDLL] = None
_ref_loaded = False


def build_oracle(force: bool = False) -> str:
    """Compile the C restatement (no FMA contraction, so the fp32 results
    match the reference op bit for bit)."""
    if force or not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(_SRC):
        os.makedirs(_LIB_DIR, exist_ok=True)
        tmp = _LIB + f".tmp{os.getpid()}"
        subprocess.check_call(
            ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-std=c11",
             "-o", tmp, _SRC]
        )
        os.replace(tmp, _LIB)
    return _LIB


def _get() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build_oracle())
        P = ctypes.c_void_p
        I = ctypes.c_int
        D = ctypes.c_double
        for suf in ("f32", "f64"):
            fw = getattr(_lib, f"pc2d_oracle_forward_{suf}")
            fw.argtypes = [P, P, D] + [I] * 11 + [P, P]
            fw.restype = None
            bw = getattr(_lib, f"pc2d_oracle_backward_{suf}")
            bw.argtypes = [P, P, P, P, D] + [I] * 13 + [P, P, I]
            bw.restype = None
        _lib.pc2d_oracle_out_size.argtypes = [I, I, I, I]
        _lib.pc2d_oracle_out_size.restype = I
    return _lib


def out_size(inp: int, k: int, s: int, dl: int) -> int:
    """Output extent, reference ``paraconv2d.cc:268-269``."""
    return ((inp - (dl * (k - 1)) - 1) // s) + 1


def _pair(v) -> Tuple[int, int]:
    if isinstance(v, int):
        return (v, v)
    return (int(v[0]), int(v[1]))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _suffix(dtype) -> str:
    if dtype == np.float32:
        return "f32"
    if dtype == np.float64:
        return "f64"
    raise TypeError(f"oracle supports float32/float64, got {dtype}")


def forward(x: np.ndarray, pars: np.ndarray, factor: float, kernel_size, stride=1, dilation=1):
    """Reference forward (``paraconv2d.cc:70-124``) on an already padded input.
    Returns ``(output, hsum)``, both ``[N, m, P, Q]``."""
    x = np.ascontiguousarray(x)
    pars = np.ascontiguousarray(pars, dtype=x.dtype)
    (k0, k1), (s0, s1), (d0, d1) = _pair(kernel_size), _pair(stride), _pair(dilation)
    n, c, h, w = x.shape
    d = c * k0 * k1
    m = pars.size // (2 * (d + 1))
    P, Q = out_size(h, k0, s0, d0), out_size(w, k1, s1, d1)
    out = np.zeros((n, m, P, Q), dtype=x.dtype)
    hsum = np.zeros((n, m, P, Q), dtype=x.dtype)
    fn = getattr(_get(), f"pc2d_oracle_forward_{_suffix(x.dtype)}")
    fn(_ptr(x), _ptr(pars), float(factor), k0, k1, s0, s1, d0, d1, n, c, h, w, m, P, Q, _ptr(out), _ptr(hsum))
    return out, hsum


def backward(grad: np.ndarray, x: np.ndarray, pars: np.ndarray, hsum: np.ndarray, factor: float,
             kernel_size, stride=1, dilation=1, skip_input_grad: bool = False):
    """Reference backward (``paraconv2d.cc:128-239``).  Returns
    ``(inputgrad [N,C,H,W], parsgrad [2m(d+1)])``."""
    x = np.ascontiguousarray(x)
    dt = x.dtype
    grad = np.ascontiguousarray(grad, dtype=dt)
    pars = np.ascontiguousarray(pars, dtype=dt)
    hsum = np.ascontiguousarray(hsum, dtype=dt)
    (k0, k1), (s0, s1), (d0, d1) = _pair(kernel_size), _pair(stride), _pair(dilation)
    n, c, h, w = x.shape
    d = c * k0 * k1
    m = pars.size // (2 * (d + 1))
    P, Q = out_size(h, k0, s0, d0), out_size(w, k1, s1, d1)
    assert grad.shape == (n, m, P, Q) and hsum.shape == (n, m, P, Q)
    dx = np.zeros_like(x)
    dpars = np.zeros(m * 2 * (d + 1), dtype=dt)
    fn = getattr(_get(), f"pc2d_oracle_backward_{_suffix(dt)}")
    fn(_ptr(grad), _ptr(x), _ptr(pars), _ptr(hsum), float(factor), k0, k1, s0, s1, d0, d1,
       n, c, h, w, m, P, Q, _ptr(dx), _ptr(dpars), int(bool(skip_input_grad)))
    return dx, dpars


# ---------------------------------------------------------------------------
# The reference op itself (built from its own sources by oracle/build_ref.sh)
# ---------------------------------------------------------------------------

def reference_available() -> bool:
    return os.path.exists(REF_LIB)


def load_reference() -> bool:
    """Register ``torch.ops.ptparaconv2d_ref`` if the reference build exists."""
    global _ref_loaded
    if _ref_loaded:
        return True
    if not reference_available():
        return False
    import torch

    torch.ops.load_library(REF_LIB)
    _ref_loaded = True
    return True


def _int_tensor(v):
    import torch

    return torch.tensor(list(_pair(v)), dtype=torch.int)


def ref_forward(x, pars, factor, kernel_size, stride=1, dilation=1):
    """The reference op's CPU forward on torch CPU tensors."""
    import torch

    if not load_reference():
        raise RuntimeError("reference op not built (oracle/build_ref.sh)")
    return torch.ops.ptparaconv2d_ref.forward(x, pars, float(factor), _int_tensor(kernel_size),
                                              _int_tensor(stride), _int_tensor(dilation))


def ref_backward(grad, x, pars, hsum, factor, kernel_size, stride=1, dilation=1, skip_input_grad=False):
    """The reference op's CPU backward on torch CPU tensors."""
    import torch

    if not load_reference():
        raise RuntimeError("reference op not built (oracle/build_ref.sh)")
    return torch.ops.ptparaconv2d_ref.backward(grad, x, pars, hsum, float(factor), _int_tensor(kernel_size),
                                               _int_tensor(stride), _int_tensor(dilation), bool(skip_input_grad))
