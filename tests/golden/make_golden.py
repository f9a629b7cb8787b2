"""Generates the golden fixtures in this directory from the reference op.

Every expected tensor stored here is produced by the reference ParaConv2d op
(GeoND-tech/ParaConv2d, CPU path of ``paraconv2d.cc``) compiled from its own
sources by ``oracle/build_ref.sh`` and loaded as ``torch.ops.ptparaconv2d_ref``.
The fixtures pin the C restatement in ``oracle/`` (``tests/test_oracle.py``)
and the CUDA kernels (``tests/test_gpu_parity.py``) on machines where the
reference sources are absent.

Inputs follow the seeded recipe used throughout the tests and the bench: on a
CPU ``torch.Generator`` seeded per case, draw the (unpadded) input, then the
flat parameter vector ``pars ~ N(0, sigma^2)``, then the upstream gradient
``N(0, 1)``; the input is padded with zeros exactly as the module does
(``F.pad``) before it reaches the op.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

# name: (N, C, H, W, m, (k0,k1), (s0,s1), (dl0,dl1), pad(l,r,t,b), sigma, input dist, factor, skip, dtype, seed)
CASES = {
    # BASELINE correctness case c1: N=2, C=3, 32x32, m=8, k3 s1 p1, U(-1,1), N(0, 0.1^2), seed 0
    "c1": (2, 3, 32, 32, 8, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), 0.1, "uniform", 1.0, False, "f32", 0),
    # reduced-size shapes of c2..c5 (same channels/kernels/strides, smaller N and spatial size)
    "c2_small": (1, 64, 8, 8, 64, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), 0.05, "uniform", 1.0, False, "f32", 1),
    "c3_small": (1, 64, 6, 6, 128, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), 0.05, "absnormal", 1.0, False, "f32", 2),
    "c4_small": (1, 3, 20, 20, 64, (7, 7), (2, 2), (1, 1), (3, 3, 3, 3), 0.1, "uniform", 1.0, False, "f32", 3),
    "c5_l2_small": (2, 32, 8, 8, 64, (3, 3), (2, 2), (1, 1), (1, 1, 1, 1), 0.05, "uniform", 1.0, False, "f32", 4),
    # odd shapes: non-square, stride 2, dilation 2, rectangular kernel, m not a multiple of 8
    "odd_s2": (2, 5, 13, 11, 3, (3, 3), (2, 2), (1, 1), (0, 0, 0, 0), 0.1, "uniform", 1.0, False, "f32", 10),
    "odd_dil2": (1, 2, 15, 12, 5, (3, 3), (1, 1), (2, 2), (0, 0, 0, 0), 0.1, "uniform", 0.5, False, "f32", 11),
    "odd_rect": (2, 4, 9, 14, 7, (3, 5), (1, 2), (1, 1), (0, 0, 0, 0), 0.1, "uniform", 1.0, False, "f32", 12),
    "k1": (3, 6, 5, 7, 9, (1, 1), (1, 1), (1, 1), (0, 0, 0, 0), 0.1, "uniform", 1.0, False, "f32", 13),
    "m1_n1": (1, 1, 3, 3, 1, (3, 3), (1, 1), (1, 1), (0, 0, 0, 0), 0.3, "uniform", 2.0, False, "f32", 14),
    "skip_grad": (2, 3, 10, 10, 4, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), 0.1, "uniform", 1.0, True, "f32", 15),
    "factor": (1, 4, 9, 9, 8, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), 0.1, "uniform", 0.1, False, "f32", 16),
    "f64": (2, 3, 9, 10, 4, (3, 3), (1, 2), (1, 1), (1, 1, 1, 1), 0.1, "uniform", 1.0, False, "f64", 17),
}


def make_inputs(N, C, H, W, m, k, pad, sigma, dist, seed, dtype=torch.float32):
    """Seeded draw: input, then pars, then the upstream gradient (shape known after padding)."""
    g = torch.Generator().manual_seed(seed)
    if dist == "uniform":
        x = torch.rand((N, C, H, W), generator=g, dtype=torch.float64) * 2 - 1
    elif dist == "absnormal":
        x = torch.randn((N, C, H, W), generator=g, dtype=torch.float64).abs()
    else:
        raise ValueError(dist)
    d = C * k[0] * k[1]
    pars = torch.randn(2 * m * (d + 1), generator=g, dtype=torch.float64) * sigma
    xp = F.pad(x, pad)
    return x.to(dtype), xp.to(dtype), pars.to(dtype), g


def make_case(name):
    N, C, H, W, m, k, s, dl, pad, sigma, dist, factor, skip, dts, seed = CASES[name]
    dt = torch.float32 if dts == "f32" else torch.float64
    _, xp, pars, g = make_inputs(N, C, H, W, m, k, pad, sigma, dist, seed, dt)
    out, hsum = oracle.ref_forward(xp, pars, factor, k, s, dl)
    grad = torch.randn(out.shape, generator=g, dtype=torch.float64).to(dt)
    dx, dpars = oracle.ref_backward(grad, xp, pars, hsum, factor, k, s, dl, skip)
    arrays = dict(x=xp.numpy(), pars=pars.numpy(), grad=grad.numpy(), out=out.numpy(), hsum=hsum.numpy(),
                  dx=dx.numpy(), dpars=dpars.numpy())
    meta = dict(N=N, C=C, H=H, W=W, m=m, kernel_size=list(k), stride=list(s), dilation=list(dl), pad=list(pad),
                sigma=sigma, dist=dist, factor=factor, skip_input_grad=skip, dtype=dts, seed=seed)
    return arrays, meta


def kat_one_hot():
    """Hand-checkable known-answer case: 1x1x4x4 input 0..15, k=3, m=1, h one-hot at tap
    (0,0), p = 0, h0 = 0, p0 = 0.  With the flipped window, tap (0,0) reads input row
    oy+2, col ox+2, so hsum[oy,ox] = x[oy+2, ox+2] and out = hsum^2 - sum(window^2)."""
    x = torch.arange(16, dtype=torch.float32).reshape(1, 1, 4, 4)
    d = 9
    pars = torch.zeros(2 * (d + 1))
    pars[1 + 0] = 1.0  # h[0, c=0, ix2=0, iy2=0]
    out, hsum = oracle.ref_forward(x, pars, 1.0, 3, 1, 1)
    exp_hsum = x[0, 0, 2:4, 2:4]
    win_sq = torch.stack([torch.stack([(x[0, 0, i:i + 3, j:j + 3] ** 2).sum() for j in range(2)])
                          for i in range(2)])
    assert torch.equal(hsum[0, 0], exp_hsum), (hsum, exp_hsum)
    assert torch.equal(out[0, 0], exp_hsum ** 2 - win_sq), (out, exp_hsum ** 2 - win_sq)
    grad = torch.ones_like(out)
    dx, dpars = oracle.ref_backward(grad, x, pars, hsum, 1.0, 3, 1, 1, False)
    arrays = dict(x=x.numpy(), pars=pars.numpy(), grad=grad.numpy(), out=out.numpy(), hsum=hsum.numpy(),
                  dx=dx.numpy(), dpars=dpars.numpy())
    meta = dict(N=1, C=1, H=4, W=4, m=1, kernel_size=[3, 3], stride=[1, 1], dilation=[1, 1], pad=[0, 0, 0, 0],
                sigma=0.0, dist="arange", factor=1.0, skip_input_grad=False, dtype="f32", seed=-1)
    return arrays, meta


def main():
    if not oracle.load_reference():
        sys.exit("reference op not built: run oracle/build_ref.sh first")
    manifest = {}
    items = [(name, make_case(name)) for name in CASES] + [("kat_one_hot", kat_one_hot())]
    for name, (arrays, meta) in items:
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        manifest[name] = meta
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"wrote {len(manifest)} fixtures")


if __name__ == "__main__":
    main()
