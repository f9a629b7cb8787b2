"""Runs the forward and backward passes of one seeded workload a few times
through the C ABI, for profilers (ncu) to capture.

    python -m paraconv2d_b200.profile_case c2 [--reps 2] [--n 128] [--simt]

The input, parameters and upstream gradient are the seeded draw of
``paraconv2d_b200.workloads``; device memory holds only that problem's
tensors and workspaces.
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import _lib, workloads


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", nargs="?", default="c2")
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--n", type=int, default=None, help="images (default: the workload's batch)")
    ap.add_argument("--simt", action="store_true", help="force the CUDA-core kernels")
    a = ap.parse_args(argv)
    wl = workloads.WORKLOADS[a.workload]
    L = wl.layer
    lib = _lib.cabi()
    if a.simt:
        _lib.set_algo(_lib.PC2D_ALGO_SIMT)
    x, pars, g = workloads.draw(wl, n=a.n)
    grad = workloads.draw_grad(wl, g, n=a.n)
    dev = torch.device("cuda", 0)
    xp = workloads.pad_input(x, L.p).to(dev)
    p = pars[0].to(dev)
    gd = grad.to(dev)
    n, C, H, W = xp.shape
    P, Q = wl.out_hw(0)
    out = torch.empty((n, L.cout, P, Q), device=dev)
    hs = torch.empty_like(out)
    dx = torch.empty_like(xp)
    dp = torch.empty_like(p)
    fws = lib.pc2d_forward_workspace_size(0, n, C, H, W, L.cout, L.k, L.k, L.s, L.s, 1, 1)
    bws = lib.pc2d_backward_workspace_size(0, n, C, H, W, L.cout, L.k, L.k, L.s, L.s, 1, 1, 0)
    fw = torch.empty(max(fws, 1), dtype=torch.uint8, device=dev)
    bw = torch.empty(max(bws, 1), dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(a.reps):
        st = lib.pc2d_forward(0, xp.data_ptr(), p.data_ptr(), 1.0, L.k, L.k, L.s, L.s, 1, 1, n, C, H, W, L.cout,
                              out.data_ptr(), hs.data_ptr(), fw.data_ptr(), fws, s)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))
        st = lib.pc2d_backward(0, gd.data_ptr(), xp.data_ptr(), p.data_ptr(), hs.data_ptr(), 1.0, L.k, L.k, L.s, L.s,
                               1, 1, n, C, H, W, L.cout, 0, dx.data_ptr(), dp.data_ptr(), bw.data_ptr(), bws, s)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))
    torch.cuda.synchronize()
    st = lib.pc2d_device_status()
    if st != 0:
        raise RuntimeError(_lib.status_message(st))
    print(f"{a.workload}: {a.reps} x (forward + backward) of n={n} done")
    return 0


if __name__ == "__main__":
    sys.exit(main())
