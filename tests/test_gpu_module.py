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


def _reference_route(m, x):
    """The reference module's route: input_factor * x, F.pad, the op's
    autograd Function (ptparaconv2d.py:215-218)."""
    xx = F.pad(m.input_factor * x, m.padding, mode=m.padding_mode)
    return pc.ParaConv2dFunction.apply(xx, m.pars, m.output_factor, m.kernel_size, m.stride, m.dilation,
                                       m.skip_input_grad, m.grad_factor)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("cin", [5, 16], ids=["narrow_input", "implicit_dgrad"])
@pytest.mark.parametrize("kw", [
    dict(padding=1),
    dict(padding=(1, 2)),
    dict(padding=(2, 0, 1, 3), stride=2),
    dict(padding=1, input_factor=1.7, grad_factor=0.5, output_factor=0.3),
])
def test_fused_route_equals_reference_route(kw, cin, dtype):
    """The module's fused route (one pad+scale pass; input gradient written
    unpadded and scaled by the kernels) gives the reference route's results:
    outputs and parameter gradients bitwise, the input gradient to within two
    roundings (the scale is applied once, as 2*input_factor*grad_factor)."""
    m = _module(cin, 24, 3, **kw).to(dtype)
    assert m._fused(torch.zeros(1, cin, 4, 4, device="cuda", dtype=dtype))
    torch.manual_seed(5)
    x = (torch.rand(3, cin, 13, 11, dtype=dtype) * 2 - 1).cuda()
    xa = x.clone().requires_grad_(True)
    xb = x.clone().requires_grad_(True)
    ya = m(xa)
    g = torch.randn(ya.shape, dtype=dtype, device="cuda")
    ya.backward(g)
    ga = m.pars.grad.clone()
    m.pars.grad = None
    yb = _reference_route(m, xb)
    yb.backward(g)
    assert torch.equal(ya, yb)
    assert torch.equal(ga, m.pars.grad)
    eps = torch.finfo(dtype).eps
    assert float((xa.grad - xb.grad).abs().max()) <= 4 * eps * float(xb.grad.abs().max())


def test_fused_route_first_layer_skips_input_gradient():
    """An input that needs no gradient: the input-gradient kernels do not run,
    and the parameter gradient is the same (bitwise) as when they do."""
    m = _module(3, 8, 3, padding=1)
    x = (torch.rand(2, 3, 16, 16) * 2 - 1).cuda()
    y = m(x)
    g = torch.randn(y.shape, device="cuda")
    y.backward(g)
    ga = m.pars.grad.clone()
    m.pars.grad = None
    xr = x.clone().requires_grad_(True)
    m(xr).backward(g)
    assert torch.equal(ga, m.pars.grad)
    assert xr.grad is not None and float(xr.grad.abs().max()) > 0


def test_fused_route_skip_input_grad_gives_zeros():
    m = _module(3, 4, 3, padding=1, skip_input_grad=True)
    x = torch.rand(2, 3, 8, 8, device="cuda", requires_grad=True)
    m(x).sum().backward()
    assert x.grad is not None and x.grad.shape == x.shape and torch.count_nonzero(x.grad) == 0


def test_other_padding_modes_take_the_reference_route():
    m = _module(3, 4, 3, padding=1, padding_mode='reflect')
    x = torch.rand(2, 3, 8, 8, device="cuda")
    assert not m._fused(x)
    y = m(x)
    out, _ = _oracle_layer(m, x.cpu())
    assert elementwise_excess(y.detach().cpu().numpy(), out) <= 1.0


@pytest.mark.parametrize("shape,pads", [((3, 5, 64, 64), (1, 1, 1, 1)), ((64, 32, 64, 64), (1, 1, 1, 1)),
                                        ((7, 3, 16, 16), (1, 1, 1, 1)), ((1, 2, 7, 100), (0, 0, 5, 0)),
                                        ((2, 2, 3, 3), (2, 2, 2, 2)), ((5, 1, 1, 1), (0, 0, 0, 0))])
def test_cabi_pad_scale_shapes(shape, pads):
    """pc2d_pad_scale equals F.pad(scale * x) bitwise on wide and narrow rows
    (segments of several padded rows, planes crossing segments, rows shorter
    than a warp), including a c5 layer's 64x64 planes."""
    from paraconv2d_b200 import _lib

    lib = _lib.cabi()
    n, C, H, W = shape
    pt, pb, pl, pr = pads
    torch.manual_seed(3)
    x = (torch.rand(n, C, H, W) * 2 - 1).cuda()
    xp = torch.full((n, C, H + pt + pb, W + pl + pr), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.pc2d_pad_scale(0, x.data_ptr(), n, C, H, W, pt, pb, pl, pr, 0.75, xp.data_ptr(), stream) == 0
    assert torch.equal(xp, F.pad(0.75 * x, (pl, pr, pt, pb)))


@pytest.mark.parametrize("dtype,code", [(torch.float32, 0), (torch.float64, 1)])
def test_cabi_pad_scale_and_interior_backward(dtype, code):
    """pc2d_pad_scale equals F.pad(scale * x) bitwise; pc2d_backward_interior
    equals pc2d_backward's padded input gradient, sliced and scaled (bitwise
    for scale 1), with the same parameter gradient."""
    from cabi_runner import backward, forward
    from paraconv2d_b200 import _lib

    lib = _lib.cabi()
    torch.manual_seed(9)
    n, C, H, W, m_, k = 2, 6, 10, 9, 7, 3
    pt, pb, pl, pr = 1, 2, 0, 3
    x = (torch.rand(n, C, H, W, dtype=dtype) * 2 - 1).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for scale in (1.0, 0.375):
        xp = torch.empty(n, C, H + pt + pb, W + pl + pr, dtype=dtype, device="cuda")
        assert lib.pc2d_pad_scale(code, x.data_ptr(), n, C, H, W, pt, pb, pl, pr, scale, xp.data_ptr(), stream) == 0
        assert torch.equal(xp, F.pad(scale * x, (pl, pr, pt, pb)))
    pars = (torch.randn(2 * m_ * (C * k * k + 1), dtype=dtype) * 0.1).cuda()
    out, hsum = forward(xp, pars, 1.0, k)
    g = torch.randn(out.shape, dtype=dtype, device="cuda")
    dx_full, dp_full = backward(g, xp, pars, hsum, 1.0, k)
    Hp, Wp = xp.shape[2], xp.shape[3]
    wsb = lib.pc2d_backward_workspace_size(code, n, C, Hp, Wp, m_, k, k, 1, 1, 1, 1, 0)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
    for scale in (1.0, 2.5):
        dx = torch.full((n, C, H, W), float("nan"), dtype=dtype, device="cuda")
        dp = torch.empty_like(pars)
        st = lib.pc2d_backward_interior(code, g.data_ptr(), xp.data_ptr(), pars.data_ptr(), hsum.data_ptr(), 1.0,
                                        k, k, 1, 1, 1, 1, n, C, Hp, Wp, m_, 0, pt, pb, pl, pr, scale, dx.data_ptr(),
                                        dp.data_ptr(), ws.data_ptr(), wsb, stream)
        assert st == 0, _lib.status_message(st)
        ref = dx_full[:, :, pt:Hp - pb, pl:Wp - pr] * scale
        if scale == 1.0:
            assert torch.equal(dx, ref)
        else:
            assert float((dx - ref).abs().max()) <= 2 * torch.finfo(dtype).eps * float(ref.abs().max())
        assert torch.equal(dp, dp_full)
    # skip_input_grad with no input-gradient array: parameter gradient only
    dp = torch.empty_like(pars)
    st = lib.pc2d_backward_interior(code, g.data_ptr(), xp.data_ptr(), pars.data_ptr(), hsum.data_ptr(), 1.0, k, k,
                                    1, 1, 1, 1, n, C, Hp, Wp, m_, 1, pt, pb, pl, pr, 1.0, None, dp.data_ptr(),
                                    ws.data_ptr(), wsb, stream)
    assert st == 0, _lib.status_message(st)
    assert torch.equal(dp, dp_full)
