"""pc2d_forward_noalloc: the forward pass for callers that may not allocate
device memory while the op runs (plugin hosts that pass only input and
output buffers, fixed-budget real-time code).  It uses a static device
scratch array instead of a caller workspace; its results must equal those of
pc2d_forward, call after call, although every call reuses the same array.

This file is collected last on purpose (tests/test_zz_*): if it fails, a run
that stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from cabi_runner import forward
from paraconv2d_b200 import _lib, workloads
from pc2d_testutil import check_outputs

pytestmark = pytest.mark.gpu


def _noalloc():
    lib = _lib.cabi()
    fn = lib.pc2d_forward_noalloc
    I, D, P = ctypes.c_int, ctypes.c_double, ctypes.c_void_p
    fn.argtypes = [I, P, P, D] + [I] * 11 + [P, P, P]
    fn.restype = I
    return fn


def _call(fn, x, pars, L, m):
    n, C, H, W = x.shape
    P = (H - (L.k - 1) - 1) // L.s + 1
    Q = (W - (L.k - 1) - 1) // L.s + 1
    out = torch.full((n, m, P, Q), float("nan"), device=x.device)
    hsum = torch.full_like(out, float("nan"))
    st = fn(0, x.data_ptr(), pars.data_ptr(), 1.0, L.k, L.k, L.s, L.s, 1, 1, n, C, H, W, m, out.data_ptr(),
            hsum.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_message(st)
    return out, hsum


@pytest.mark.parametrize("name,n", [("c2", 4), ("c3", 1), ("c4", 1), ("c1", 2)])
def test_noalloc_forward_matches_forward_twice(name, n):
    wl = workloads.WORKLOADS[name]
    L = wl.layer
    x, pars, g = workloads.draw(wl, n=n)
    xp = workloads.pad_input(x, L.p).cuda()
    p = pars[0].cuda()
    ref_out, ref_hs = forward(xp, p, 1.0, L.k, L.s, 1)
    fn = _noalloc()
    # two calls in a row: the second reuses the scratch the first one left behind
    for _ in range(2):
        out, hs = _call(fn, xp, p, L, L.cout)
        torch.cuda.synchronize()
        check_outputs(out.cpu().numpy(), hs.cpu().numpy(), ref_out.cpu().numpy(), ref_hs.cpu().numpy())
    assert _lib.cabi().pc2d_device_status() == 0


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    # 512 -> 512 channels, 3x3: the split weights alone need ~38 MB > 8 MiB.
    fn = _noalloc()
    st = fn(0, None, None, 1.0, 3, 3, 1, 1, 1, 1, 1, 512, 10, 10, 512, None, None, None)
    assert st == _lib.PC2D_ERR_WORKSPACE
    assert b"static scratch" in _lib.cabi().pc2d_last_error()
