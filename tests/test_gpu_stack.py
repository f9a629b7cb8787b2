"""The c5 layer stack (3->32->64->64->64, k3 p1, stride 2 on layers 2 and 3,
64x64 input, loss sum((2^-40 out)^2)) through the ParaConv2d module chain on
the GPU, against

* a float64 chained restatement (every layer's output, every layer's input
  gradient, every layer's parameter gradient) at the per-GPU shard of an
  8-GPU run (128 images) and at the full batch (1024 images);
* the reference CPU op chained layer by layer in fp32 (the oracle) on the
  first 4 images, with the second half of the gradient policy: no further
  from fp64 than twice the oracle's own error.

Tolerances (pc2d_testutil): outputs elementwise 1e-5 + 1e-4|b|, gradients
max|a-b| <= 1e-4 max|b|.  Layer 0 runs with skip_input_grad, as in the
data-parallel step; a second case checks its input gradient (the narrow-input
GEMM + col2im path at 64x64) with skip_input_grad off.
"""
import numpy as np
import pytest
import torch

import oracle
import paraconv2d_b200 as pc
from paraconv2d_b200 import workloads
from pc2d_testutil import (check_grads, check_vs_float64, elementwise_excess, maxrel_excess, ref_layer64,
                           stack_reference64)

pytestmark = pytest.mark.gpu

WL = workloads.WORKLOADS["c5"]


def _stack(pars, skip_first=True):
    mods = []
    for i, (L, pr) in enumerate(zip(WL.layers, pars)):
        m = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p, skip_input_grad=(skip_first and i == 0)).cuda()
        with torch.no_grad():
            m.pars.copy_(pr.cuda())
        mods.append(m)
    return mods


def _run_stack(mods, x, input_grad=False):
    """Our chain: outputs of every layer, gradients of every layer's input
    (None where not computed) and every layer's parameter gradient."""
    h = x.cuda().requires_grad_(input_grad)
    acts = [h]
    for m in mods:
        h = m(h)
        h.retain_grad()
        acts.append(h)
    workloads.stack_loss(h).backward()
    torch.cuda.synchronize()
    outs = [a.detach() for a in acts[1:]]
    in_grads = [a.grad for a in acts[:-1]]
    return outs, in_grads, [m.pars.grad for m in mods]


def _d(L):
    return L.cin * L.k * L.k


@pytest.mark.parametrize("n", [128, 1024])
def test_c5_stack_vs_float64(n):
    x, pars, _ = workloads.draw(WL, n=n)
    outs, in_grads, pgrads = _run_stack(_stack(pars), x)
    r_outs, r_in, r_p = stack_reference64(x.cuda(), pars, WL.layers, workloads.stack_loss)
    for i, L in enumerate(WL.layers):
        e = elementwise_excess(outs[i], r_outs[i])
        assert e <= 1.0, f"layer {i} output exceeds 1e-5/1e-4 elementwise by {e:.3g}x"
        check_grads(np.zeros(1), pgrads[i].cpu().numpy(), np.zeros(1), r_p[i].cpu().numpy(), L.cout, _d(L))
        if i > 0:
            e = maxrel_excess(in_grads[i], r_in[i])
            assert e <= 1.0, f"layer {i} input gradient exceeds 1e-4 max|b| by {e:.3g}x"
        assert torch.isfinite(pgrads[i]).all()


def test_c5_first_layer_input_gradient():
    """Layer 0 alone (C=3 -> 32, 64x64, the narrow-input dgrad path) with its
    input gradient computed, 128 images, against float64."""
    x, pars, g = workloads.draw(WL, n=128)
    L = WL.layers[0]
    m = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p).cuda()
    with torch.no_grad():
        m.pars.copy_(pars[0].cuda())
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    gy = torch.randn(y.shape, generator=g).cuda()
    y.backward(gy)
    rdx, rdp = torch.autograd.functional.vjp(
        lambda xx, pp: ref_layer64(xx, pp, L), (x.cuda().double(), pars[0].cuda().double()), gy.double())[1]
    assert maxrel_excess(xd.grad, rdx) <= 1.0
    check_grads(np.zeros(1), m.pars.grad.cpu().numpy(), np.zeros(1), rdp.cpu().numpy(), L.cout, _d(L))


def _oracle_chain(x, pars):
    """The reference CPU op chained in fp32 (module semantics: pad 1, factors
    1, layer 0 skips its input gradient), loss sum((2^-40 y)^2): outputs,
    input gradients (None for layer 0) and parameter gradients."""
    h = x.numpy()
    saved, outs = [], []
    for L, pr in zip(WL.layers, pars):
        xp = np.ascontiguousarray(np.pad(h, ((0, 0), (0, 0), (L.p, L.p), (L.p, L.p))))
        out, hs = oracle.forward(xp, pr.numpy(), 1.0, L.k, L.s, 1)
        saved.append((xp, hs))
        outs.append(out)
        h = out
    # d/dy sum((s y)^2) = 2 s^2 y, a power of two times y: exact in fp32
    g = (outs[-1] * np.float32(2.0 * workloads.STACK_OUTPUT_SCALE ** 2)).astype(np.float32)
    in_grads, pgrads = [None] * 4, [None] * 4
    for i in range(3, -1, -1):
        L, (xp, hs) = WL.layers[i], saved[i]
        dxp, dp = oracle.backward(g, xp, pars[i].numpy(), hs, 1.0, L.k, L.s, 1, i == 0)
        pgrads[i] = dp
        if i > 0:
            g = np.ascontiguousarray(dxp[:, :, L.p:-L.p, L.p:-L.p])
            in_grads[i] = g
    return outs, in_grads, pgrads


def test_c5_stack_small_vs_oracle_chain():
    """First 4 images: our chain against the oracle chain (same policy) and
    against fp64 no worse than twice the oracle chain's own error."""
    n = 4
    x, pars, _ = workloads.draw(WL, n=n)
    outs, in_grads, pgrads = _run_stack(_stack(pars), x)
    o_outs, o_in, o_p = _oracle_chain(x, pars)
    r_outs, r_in, r_p = stack_reference64(x, pars, WL.layers, workloads.stack_loss)
    for i, L in enumerate(WL.layers):
        e = elementwise_excess(outs[i].cpu().numpy(), o_outs[i])
        assert e <= 1.0, f"layer {i} output exceeds 1e-5/1e-4 elementwise against the oracle by {e:.3g}x"
        d = _d(L)
        dx = in_grads[i].cpu().numpy() if i > 0 else np.zeros(1)
        odx = o_in[i] if i > 0 else np.zeros(1)
        rdx = r_in[i].numpy() if i > 0 else np.zeros(1)
        check_grads(dx, pgrads[i].cpu().numpy(), odx, o_p[i], L.cout, d, skip_input_grad=False)
        check_vs_float64(dx, pgrads[i].cpu().numpy(), odx, o_p[i], rdx, r_p[i].numpy(), L.cout, d,
                         skip_input_grad=(i == 0))
