"""Calls the C ABI of libpc2d_sm100.so (include/paraconv2d.h) through ctypes
with torch CUDA tensors as device memory (torch is only the allocator and
the stream here)."""
from __future__ import annotations

import torch

from paraconv2d_b200 import _lib


def _dt(t):
    if t.dtype == torch.float32:
        return _lib.PC2D_DTYPE_F32
    if t.dtype == torch.float64:
        return _lib.PC2D_DTYPE_F64
    raise TypeError(t.dtype)


def _pair(v):
    return (v, v) if isinstance(v, int) else (int(v[0]), int(v[1]))


def _stream():
    return torch.cuda.current_stream().cuda_stream


def forward(x, pars, factor, k, s=1, dl=1):
    lib = _lib.cabi()
    (k0, k1), (s0, s1), (d0, d1) = _pair(k), _pair(s), _pair(dl)
    n, C, H, W = x.shape
    m = lib.pc2d_infer_m(pars.numel(), C, k0, k1)
    assert m > 0
    P, Q = lib.pc2d_out_size(H, k0, s0, d0), lib.pc2d_out_size(W, k1, s1, d1)
    out = torch.empty((n, m, P, Q), dtype=x.dtype, device=x.device)
    hsum = torch.empty_like(out)
    wsb = lib.pc2d_forward_workspace_size(_dt(x), n, C, H, W, m, k0, k1, s0, s1, d0, d1)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
    st = lib.pc2d_forward(_dt(x), x.data_ptr(), pars.data_ptr(), float(factor), k0, k1, s0, s1, d0, d1, n, C, H, W, m,
                          out.data_ptr(), hsum.data_ptr(), ws.data_ptr() if wsb else None, wsb, _stream())
    assert st == 0, _lib.status_message(st)
    return out, hsum


def backward(grad, x, pars, hsum, factor, k, s=1, dl=1, skip_input_grad=False):
    lib = _lib.cabi()
    (k0, k1), (s0, s1), (d0, d1) = _pair(k), _pair(s), _pair(dl)
    n, C, H, W = x.shape
    m = lib.pc2d_infer_m(pars.numel(), C, k0, k1)
    dx = torch.empty_like(x)
    dpars = torch.empty_like(pars)
    wsb = lib.pc2d_backward_workspace_size(_dt(x), n, C, H, W, m, k0, k1, s0, s1, d0, d1, int(skip_input_grad))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
    st = lib.pc2d_backward(_dt(x), grad.data_ptr(), x.data_ptr(), pars.data_ptr(), hsum.data_ptr(), float(factor),
                           k0, k1, s0, s1, d0, d1, n, C, H, W, m, int(skip_input_grad), dx.data_ptr(), dpars.data_ptr(),
                           ws.data_ptr() if wsb else None, wsb, _stream())
    assert st == 0, _lib.status_message(st)
    return dx, dpars


class algo:
    """Context manager selecting the kernel family (PC2D_ALGO_*)."""

    def __init__(self, a):
        self.a = a

    def __enter__(self):
        self.prev = _lib.set_algo(self.a)
        return self

    def __exit__(self, *exc):
        _lib.set_algo(self.prev)
        return False
