"""Shared helpers of the test suite: golden fixtures, tolerance policy and a
float64 torch restatement of the op used as a second reference at sizes the
CPU oracle cannot reach quickly.

Tolerance policy (per tensor, against the fp32 oracle = the reference CPU op):
  output, hsum                elementwise |a - b| <= 1e-5 + 1e-4 |b|
  inputgrad, h0/h/p/p0 grads  max |a - b| <= 1e-4 * max |b|
The gradients are long reductions whose fp32 value depends on summation
order; the reference's own fp32 result is not elementwise within 1e-5/1e-4 of
the exact (fp64) value, so no other summation order can be.  Where both the
fp32 oracle's result and an fp64 reference exist, each gradient tensor must
also be about as close to the fp64 value as fp32 arithmetic gets:
  max |a - b64| <= max(2 max |oracle32 - b64|, 2^-18 max |b64|)
(check_vs_float64).  The floor is 64 units in the last place of the tensor's
largest value.  It is needed because the oracle's own error is one sample of
one summation order: on short reductions it is often a few ulps, and any
other order -- this library's fp32 CUDA-core kernels included -- lands a few
times further away (measured: up to 1.1e-6 max|b64| for those kernels, 1.3e-6
for the 3xTF32 tensor-core kernels, against the oracle's 2e-7 to 1e-6).
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch
import torch.nn.functional as F

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

OUT_ATOL, OUT_RTOL = 1e-5, 1e-4
GRAD_REL = 1e-4


def golden_manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def load_golden(name):
    meta = golden_manifest()[name]
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    return arrays, meta


def _pair64(a, b):
    """Both operands as float64, as torch tensors on the device of whichever
    is a torch tensor (large comparisons stay on the GPU), else numpy."""
    if isinstance(a, torch.Tensor) or isinstance(b, torch.Tensor):
        dev = a.device if isinstance(a, torch.Tensor) else b.device
        return (torch.as_tensor(a).to(dev, torch.float64), torch.as_tensor(b).to(dev, torch.float64))
    return np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)


def _max(t):
    return float(t.max()) if isinstance(t, torch.Tensor) else float(np.max(t))


def _numel(t):
    return t.numel() if isinstance(t, torch.Tensor) else t.size


def elementwise_excess(a, b, atol=OUT_ATOL, rtol=OUT_RTOL):
    """max over elements of |a-b| / (atol + rtol |b|); <= 1 passes."""
    a, b = _pair64(a, b)
    if _numel(a) == 0:
        return 0.0
    return _max(abs(a - b) / (atol + rtol * abs(b)))


def maxrel_excess(a, b, rel=GRAD_REL):
    """max |a-b| / (rel * max |b|); <= 1 passes."""
    a, b = _pair64(a, b)
    if _numel(a) == 0:
        return 0.0
    scale = _max(abs(b))
    err = _max(abs(a - b))
    if scale == 0.0:
        return 0.0 if err == 0.0 else float("inf")
    return err / (rel * scale)


def split_pars(pars, m, d):
    pars = np.asarray(pars)
    return pars[:m], pars[m:m + m * d], pars[m + m * d:m + 2 * m * d], pars[m + 2 * m * d:]


def check_outputs(out, hsum, ref_out, ref_hsum):
    e_out = elementwise_excess(out, ref_out)
    e_hs = elementwise_excess(hsum, ref_hsum)
    assert e_out <= 1.0, f"output exceeds 1e-5/1e-4 elementwise by {e_out:.3g}x"
    assert e_hs <= 1.0, f"hsum exceeds 1e-5/1e-4 elementwise by {e_hs:.3g}x"
    return e_out, e_hs


def check_grads(dx, dpars, ref_dx, ref_dpars, m, d, skip_input_grad=False):
    res = {}
    if skip_input_grad:
        assert np.all(np.asarray(dx) == 0), "inputgrad must be all zero when skip_input_grad"
        res["dx"] = 0.0
    else:
        res["dx"] = maxrel_excess(dx, ref_dx)
    for name, a, b in zip(("dh0", "dh", "dp", "dp0"), split_pars(dpars, m, d), split_pars(ref_dpars, m, d)):
        res[name] = maxrel_excess(a, b)
    bad = {k: v for k, v in res.items() if v > 1.0}
    assert not bad, f"gradients exceed max|a-b| <= 1e-4 max|b|: {bad}"
    return res


# Floor of the fp32-oracle comparison, relative to the tensor's largest value
# (64 fp32 ulps): where the oracle's own error is a few ulps by luck of its
# summation order, "twice the oracle's error" would hold any other fp32
# summation order to that luck.
VS64_FLOOR = 2.0 ** -18


def check_vs_float64(dx, dpars, oracle_dx, oracle_dpars, ref_dx, ref_dpars, m, d, skip_input_grad=False,
                     factor=2.0):
    """Second half of the gradient policy: per tensor, our max error against
    the fp64 reference is at most `factor` times the fp32 oracle's own max
    error against it, or VS64_FLOOR * max|b64| where that is larger.
    Returns {tensor: (our error, oracle error)}."""
    pairs = []
    if not skip_input_grad:
        pairs.append(("dx", dx, oracle_dx, ref_dx))
    for name, a, o, b in zip(("dh0", "dh", "dp", "dp0"), split_pars(dpars, m, d), split_pars(oracle_dpars, m, d),
                             split_pars(ref_dpars, m, d)):
        pairs.append((name, a, o, b))
    res, bad = {}, {}
    for name, a, o, b in pairs:
        a, o, b = (np.asarray(t, dtype=np.float64) for t in (a, o, b))
        if b.size == 0:
            continue
        ours = float(np.max(np.abs(a - b)))
        orc = float(np.max(np.abs(o - b)))
        scale = float(np.max(np.abs(b)))
        res[name] = (ours, orc)
        if ours > max(factor * orc, VS64_FLOOR * scale):
            bad[name] = {"ours": ours, "oracle": orc, "max|b64|": scale}
    assert not bad, f"gradients further from fp64 than {factor}x the fp32 oracle's own error: {bad}"
    return res


# --------------------------------------------------------------------------
# Layer stacks (the data-parallel workload): float64 chained restatement
# --------------------------------------------------------------------------

def ref_layer64(x, pars, L):
    """One ParaConv2d layer (module semantics: constant pad L.p on all sides,
    then the op) in float64 torch on x's device, differentiable in x and
    pars.  The op's input gradient carries no output factor (f = 1 here)."""
    xp = F.pad(x, (L.p, L.p, L.p, L.p))
    k, C = L.k, L.cin
    m, d = L.cout, L.cin * L.k * L.k
    h0, h, p, p0 = pars[:m], pars[m:m + m * d], pars[m + m * d:m + 2 * m * d], pars[m + 2 * m * d:]
    H = h.reshape(m, C, k, k).flip(2, 3)
    Pw = p.reshape(m, C, k, k).flip(2, 3)
    ones = torch.ones(1, C, k, k, dtype=x.dtype, device=x.device)
    hs = F.conv2d(xp, H, stride=L.s) + h0.view(1, m, 1, 1)
    px = F.conv2d(xp, Pw, stride=L.s)
    s2 = F.conv2d(xp * xp, ones, stride=L.s)
    pp = (p.reshape(m, d) ** 2).sum(1).view(1, m, 1, 1)
    return hs * hs - (s2 - 2 * px + pp) - (p0 * p0).view(1, m, 1, 1)


def stack_reference64(x, pars_list, layers, loss_fn):
    """Forward and backward of a layer stack in float64: returns (outputs of
    every layer, gradient of every layer's input, every layer's pars grad),
    all float64 tensors on x's device.  `loss_fn(y)` maps the last output to
    the scalar loss."""
    acts = [x.to(torch.float64).detach().requires_grad_(True)]
    params = [p.to(x.device, torch.float64).detach().requires_grad_(True) for p in pars_list]
    h = acts[0]
    outs = []
    for L, pr in zip(layers, params):
        h = ref_layer64(h, pr, L)
        h.retain_grad()
        outs.append(h)
    loss_fn(h).backward()
    in_grads = [acts[0].grad] + [o.grad for o in outs[:-1]]
    return [o.detach() for o in outs], in_grads, [p.grad for p in params]


# --------------------------------------------------------------------------
# float64 torch restatement (test reference for large sizes)
# --------------------------------------------------------------------------

def torch_reference(x, pars, factor, k, s, dl, grad=None, skip_input_grad=False):
    """Forward (and, with `grad`, backward) of the op in float64 torch, from
    the conv decomposition: hsum = h0 + conv(x, flip(h)), |win - p|^2 =
    conv(x^2, 1) - 2 conv(x, flip(p)) + |p|^2.  Returns numpy arrays
    (out, hsum[, dx, dpars]) with dx in the op's convention (2 * scatter, no
    output factor) and dpars packed like pars."""
    k0, k1 = k
    x = torch.as_tensor(x).to(torch.float64).clone().requires_grad_(grad is not None)
    pars = torch.as_tensor(pars).to(x.device, torch.float64).clone().requires_grad_(grad is not None)
    C = x.shape[1]
    d = C * k0 * k1
    m = pars.numel() // (2 * (d + 1))
    h0, h, p, p0 = pars[:m], pars[m:m + m * d], pars[m + m * d:m + 2 * m * d], pars[m + 2 * m * d:]
    H = h.reshape(m, C, k0, k1).flip(2, 3)
    Pw = p.reshape(m, C, k0, k1).flip(2, 3)
    ones = torch.ones(1, C, k0, k1, dtype=torch.float64, device=x.device)
    hs = F.conv2d(x, H, stride=s, dilation=dl) + h0.view(1, m, 1, 1)
    px = F.conv2d(x, Pw, stride=s, dilation=dl)
    s2 = F.conv2d(x * x, ones, stride=s, dilation=dl)
    pp = (p.reshape(m, d) ** 2).sum(1).view(1, m, 1, 1)
    out = factor * (hs * hs - (s2 - 2 * px + pp) - (p0 * p0).view(1, m, 1, 1))
    if grad is None:
        return out.detach().cpu().numpy(), hs.detach().cpu().numpy()
    g = torch.as_tensor(grad).to(x.device, torch.float64)
    dx, dpars = torch.autograd.grad(out, (x, pars), g)
    dx = torch.zeros_like(dx) if skip_input_grad else dx / factor
    return (out.detach().cpu().numpy(), hs.detach().cpu().numpy(), dx.cpu().numpy(), dpars.cpu().numpy())
