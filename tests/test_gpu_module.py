"""The ParaConv2d module and torch.ops.ptparaconv2d on CUDA against the
oracle: padding, input/output/grad factors, fp16 inputs, skip_input_grad,
non-contiguous upstream gradients and the op's argument checks."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import paraconv2d_b200 as pc
from pc2d_testutil import check_grads, check_outputs, elementwise_excess, maxrel_excess

pytestmark = pytest.mark.gpu


def _module(cin, cout, k, **kw):
    torch.manual_seed(7)
    m = pc.ParaConv2d(cin, cout, k, **kw)
    with torch.no_grad():
        m.pars.normal_(0.0, 0.1)
    return m.cuda()


def _oracle_layer(m, x_cpu, grad_cpu=None):
    """Oracle output/gradients of module `m` on input x (the module's own pad and factors applied)."""
    k = tuple(int(v) for v in m.kernel_size)
    s = tuple(int(v) for v in m.stride)
    dl = tuple(int(v) for v in m.dilation)
    xp = F.pad(m.input_factor * x_cpu.double(), m.padding, mode=m.padding_mode).numpy()
    pars = m.pars.detach().cpu().double().numpy()
    out, hs = oracle.forward(xp, pars, m.output_factor, k, s, dl)
    if grad_cpu is None:
        return out, hs
    dxp, dpars = oracle.backward(grad_cpu.double().numpy(), xp, pars, hs, m.output_factor, k, s, dl,
                                 m.skip_input_grad)
    return out, hs, dxp, dpars


@pytest.mark.parametrize("kw", [
    dict(padding=1),
    dict(padding=(1, 2)),                      # a 2-tuple goes to F.pad as is: pads width only
    dict(padding=2, stride=2, dilation=2),
    dict(padding=1, output_factor=0.3, input_factor=1.7, grad_factor=0.5),
    dict(padding=1, skip_input_grad=True),
])
def test_module_forward_backward(kw):
    m = _module(4, 8, 3, **kw)
    torch.manual_seed(3)
    x = torch.rand(2, 4, 11, 9) * 2 - 1
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    g = torch.randn(y.shape)
    y.backward(g.cuda())
    out, hs, dxp, dpars = _oracle_layer(m, x, g)
    assert elementwise_excess(y.detach().cpu().numpy(), out) <= 1.0
    d = 4 * 9
    check_grads(np.zeros(1), m.pars.grad.cpu().numpy(), np.zeros(1), dpars, 8, d, skip_input_grad=False)
    # input gradient: the op's dx (no output factor) through F.pad's and the factors' backward
    l, r, t, b = m.padding if len(m.padding) == 4 else (m.padding[0], m.padding[1], 0, 0)
    H, W = dxp.shape[2], dxp.shape[3]
    ref_dx = dxp[:, :, t:H - b, l:W - r] * m.input_factor * m.grad_factor
    if kw.get("skip_input_grad"):
        assert torch.count_nonzero(xd.grad) == 0
    else:
        assert maxrel_excess(xd.grad.cpu().numpy(), ref_dx) <= 1.0


def test_module_fp16_input():
    m = _module(3, 8, 3, padding=1)
    x = (torch.rand(2, 3, 8, 8) * 2 - 1).half()
    y = m(x.cuda()).detach()
    assert y.dtype == torch.float16
    out, _ = _oracle_layer(m, x.float())
    assert np.allclose(y.float().cpu().numpy(), out, rtol=1e-2, atol=1e-2)


def test_noncontiguous_upstream_gradient():
    """y.sum().backward() hands the op an expanded (stride-0) gradient; the
    reference reads it as contiguous memory, this op makes it contiguous."""
    m = _module(3, 4, 3, padding=1)
    x = torch.rand(1, 3, 6, 6).cuda().requires_grad_(True)
    m(x).sum().backward()
    _, _, _, dpars = _oracle_layer(m, x.detach().cpu(), torch.ones(1, 4, 6, 6))
    check_grads(np.zeros(1), m.pars.grad.cpu().numpy(), np.zeros(1), dpars, 4, 27)


def test_op_float64():
    torch.manual_seed(0)
    x = torch.rand(1, 2, 7, 7, dtype=torch.float64)
    pars = torch.randn(2 * 3 * (18 + 1), dtype=torch.float64) * 0.2
    k = torch.tensor([3, 3], dtype=torch.int)
    one = torch.tensor([1, 1], dtype=torch.int)
    out, hs = torch.ops.ptparaconv2d.forward(x.cuda(), pars.cuda(), 1.0, k, one, one)
    ro, rh = oracle.forward(x.numpy(), pars.numpy(), 1.0, 3, 1, 1)
    assert np.allclose(out.cpu().numpy(), ro, rtol=1e-12, atol=1e-12)
    assert np.allclose(hs.cpu().numpy(), rh, rtol=1e-12, atol=1e-12)


def test_op_rejects_bad_arguments():
    x = torch.rand(1, 3, 8, 8).cuda()
    one = torch.tensor([1, 1], dtype=torch.int)
    k3 = torch.tensor([3, 3], dtype=torch.int)
    with pytest.raises(RuntimeError, match="multiple of"):
        torch.ops.ptparaconv2d.forward(x, torch.zeros(5).cuda(), 1.0, k3, one, one)
    with pytest.raises(RuntimeError, match="even kernel"):
        k2 = torch.tensor([2, 2], dtype=torch.int)
        torch.ops.ptparaconv2d.forward(x, torch.zeros(2 * (12 + 1)).cuda(), 1.0, k2, one, one)
    with pytest.raises(NotImplementedError):
        torch.ops.ptparaconv2d.forward(x.bfloat16(), torch.zeros(2 * 28).cuda().bfloat16(), 1.0, k3, one, one)
