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

import oracle
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
        if name == "c1":
            # and against the reference CPU op directly
            o_out, o_hs = oracle.forward(xp.cpu().numpy(), pars[0].numpy(), 1.0, L.k, L.s, 1)
            check_outputs(out.cpu().numpy(), hs.cpu().numpy(), o_out, o_hs)
    assert _lib.cabi().pc2d_device_status() == 0


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    # 512 -> 512 channels, 3x3: the split weights alone need ~38 MB > 8 MiB.
    fn = _noalloc()
    st = fn(0, None, None, 1.0, 3, 3, 1, 1, 1, 1, 1, 512, 10, 10, 512, None, None, None)
    assert st == _lib.PC2D_ERR_WORKSPACE
    assert b"static scratch" in _lib.cabi().pc2d_last_error()


def _call64(fn, x, pars, k, m):
    n, C, H, W = x.shape
    P, Q = H - k + 1, W - k + 1
    out = torch.full((n, m, P, Q), float("nan"), dtype=x.dtype, device=x.device)
    hsum = torch.full_like(out, float("nan"))
    st = fn(_lib.PC2D_DTYPE_F64 if x.dtype == torch.float64 else _lib.PC2D_DTYPE_F32, x.data_ptr(), pars.data_ptr(),
            1.0, k, k, 1, 1, 1, 1, n, C, H, W, m, out.data_ptr(), hsum.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_message(st)
    return out, hsum


def test_noalloc_paths_without_scratch():
    """Problems whose kernel path needs no scratch (fp64, or the CUDA-core
    kernels forced process-wide) give the same results as pc2d_forward, and a
    rejected call leaves the array usable for the next valid call."""
    from cabi_runner import algo
    from paraconv2d_b200 import PC2D_ALGO_SIMT

    fn = _noalloc()
    gen = torch.Generator().manual_seed(11)
    x64 = (torch.rand(2, 3, 9, 9, generator=gen, dtype=torch.float64) * 2 - 1).cuda()
    p64 = (torch.randn(2 * 5 * 28, generator=gen, dtype=torch.float64) * 0.1).cuda()
    ref = forward(x64, p64, 1.0, 3)
    for _ in range(2):
        got = _call64(fn, x64, p64, 3, 5)
        torch.cuda.synchronize()
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    wl = workloads.WORKLOADS["c2"]
    L = wl.layer
    x, pars, _ = workloads.draw(wl, n=2)
    xp = workloads.pad_input(x, L.p).cuda()
    p = pars[0].cuda()
    with algo(PC2D_ALGO_SIMT):
        ref = forward(xp, p, 1.0, L.k, L.s, 1)
        got = _call(fn, xp, p, L, L.cout)
        torch.cuda.synchronize()
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    # a call rejected for its size, then a valid tensor-core call
    st = fn(0, None, None, 1.0, 3, 3, 1, 1, 1, 1, 1, 512, 10, 10, 512, None, None, None)
    assert st == _lib.PC2D_ERR_WORKSPACE
    ref = forward(xp, p, 1.0, L.k, L.s, 1)
    got = _call(fn, xp, p, L, L.cout)
    torch.cuda.synchronize()
    check_outputs(got[0].cpu().numpy(), got[1].cpu().numpy(), ref[0].cpu().numpy(), ref[1].cpu().numpy())
    assert _lib.cabi().pc2d_device_status() == 0
