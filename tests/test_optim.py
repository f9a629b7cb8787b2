"""ParaboloidSGD (paraconv2d_b200/optim.py): the optimizer tags of the
module's ``pars`` (reference ptparaconv2d.py:194-198) applied per parameter
group.  CPU tests cover the update rule and its agreement with
torch.optim.SGD; the GPU tests compare the fused kernel (pc2d_param_step)
with the same update in torch ops."""
import pytest
import torch

import paraconv2d_b200 as pc
from paraconv2d_b200.optim import ParaboloidSGD, paraboloid_split, sgd_step_reference


def _layer(cin=3, cout=5, k=3, dev="cpu", dtype=torch.float32, **kw):
    torch.manual_seed(0)
    m = pc.ParaConv2d(cin, cout, k, **kw)
    return m.to(device=dev, dtype=dtype)


def _grads(mod, seed):
    g = torch.Generator().manual_seed(seed)
    for p in mod.parameters():
        p.grad = torch.randn(p.shape, generator=g, dtype=torch.float64).to(p.dtype).to(p.device)


def test_split_follows_the_packing():
    mod = _layer(3, 5, 3)
    m, d = paraboloid_split(mod.pars)
    assert (m, d) == (5, 27)
    assert mod.pars.numel() == 2 * m * (1 + d)


def test_untagged_parameters_take_torch_sgd():
    torch.manual_seed(1)
    a = torch.nn.Linear(7, 3)
    b = torch.nn.Linear(7, 3)
    b.load_state_dict(a.state_dict())
    oa = ParaboloidSGD(a.parameters(), lr=0.1, momentum=0.9, weight_decay=0.01)
    ob = torch.optim.SGD(b.parameters(), lr=0.1, momentum=0.9, weight_decay=0.01, foreach=False)
    for step in range(3):
        for pa, pb in zip(a.parameters(), b.parameters()):
            pa.grad = torch.full_like(pa, 0.5 + step)
            pb.grad = pa.grad.clone()
        oa.step()
        ob.step()
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.allclose(pa, pb, rtol=0, atol=1e-6)


def test_tags_scale_the_update_per_part():
    """With momentum 0 and no weight decay the [h0 | h] part moves by
    lr*h_lr_factor*grad and the [p | p0] part by lr*p_lr_factor*grad;
    weight decay is scaled by wd_factor."""
    mod = _layer(3, 5, 3, h_lr_factor=4.0, p_lr_factor=0.25, wd_factor=0.5)
    m, d = paraboloid_split(mod.pars)
    nh = m * (1 + d)
    w0 = mod.pars.detach().clone()
    _grads(mod, 3)
    g = mod.pars.grad.clone()
    ParaboloidSGD(mod.parameters(), lr=0.1, weight_decay=0.2).step()
    dd = g + 0.2 * 0.5 * w0
    want = w0.clone()
    want[:nh] -= 0.1 * 4.0 * dd[:nh]
    want[nh:] -= 0.1 * 0.25 * dd[nh:]
    assert torch.allclose(mod.pars.detach(), want, rtol=0, atol=1e-7)


def test_momentum_buffer_starts_at_the_first_gradient():
    w = torch.zeros(6)
    buf = torch.empty(6)
    sgd_step_reference(w, torch.ones(6), buf, True, 3, 1.0, 2.0, 0.0, 0.9)
    assert torch.equal(buf, torch.ones(6))
    assert torch.equal(w, torch.tensor([-1.0, -1, -1, -2, -2, -2]))
    sgd_step_reference(w, torch.ones(6), buf, False, 3, 1.0, 2.0, 0.0, 0.9)
    assert torch.allclose(buf, torch.full((6,), 1.9))


def test_bad_split_and_arguments_are_refused():
    p = torch.nn.Parameter(torch.zeros(10))
    p.d = 3  # 10 is not a multiple of 2*(3+1)
    with pytest.raises(ValueError):
        paraboloid_split(p)
    with pytest.raises(ValueError):
        ParaboloidSGD([p], lr=-1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("momentum", [0.0, 0.9])
def test_fused_step_equals_the_torch_update(dtype, momentum):
    """Three steps of the fused kernel on a 64->64 3x3 layer (73,856 values)
    against the same update in torch ops; fp32 within a few ulps (the kernel
    may contract multiply-adds), fp64 within 1e-15 relative."""
    dev = torch.device("cuda", 0)
    kw = dict(h_lr_factor=3.0, p_lr_factor=0.5, wd_factor=0.1)
    fused = _layer(64, 64, 3, dev=dev, dtype=dtype, **kw)
    ref = _layer(64, 64, 3, dev=dev, dtype=dtype, **kw)
    opt = ParaboloidSGD(fused.parameters(), lr=0.05, momentum=momentum, weight_decay=0.01)
    m, d = paraboloid_split(ref.pars)
    buf = torch.empty_like(ref.pars)
    for step in range(3):
        _grads(fused, 10 + step)
        _grads(ref, 10 + step)
        opt.step()
        with torch.no_grad():
            sgd_step_reference(ref.pars, ref.pars.grad, buf, step == 0, m * (1 + d), 0.05 * 3.0, 0.05 * 0.5,
                               0.01 * 0.1, momentum)
    torch.cuda.synchronize()
    a, b = fused.pars.detach(), ref.pars.detach()
    tol = 1e-6 if dtype == torch.float32 else 1e-15
    assert float((a - b).abs().max()) <= tol * float(b.abs().max())
    assert pc.cabi().pc2d_device_status() == 0


@pytest.mark.gpu
def test_fused_step_unaligned_tail():
    """A parameter count that is not a multiple of four (m=3, d=2: 18 values)
    takes the element-wise tail of the kernel."""
    dev = torch.device("cuda", 0)
    p = torch.nn.Parameter(torch.arange(18, dtype=torch.float32, device=dev) / 7)
    p.d, p.isParaboloid, p.h_lr_factor, p.p_lr_factor, p.wd_factor = 2, True, 2.0, 0.5, 1.0
    q = p.detach().clone()
    p.grad = torch.ones_like(p)
    ParaboloidSGD([p], lr=0.1).step()
    sgd_step_reference(q, torch.ones_like(q), None, True, 9, 0.2, 0.05, 0.0, 0.0)
    torch.cuda.synchronize()
    assert torch.allclose(p.detach(), q, rtol=0, atol=1e-7)
