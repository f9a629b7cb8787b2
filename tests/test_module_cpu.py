"""The ParaConv2d module mirror on CPU: constructor semantics of the
reference module (ptparaconv2d.py:62-221) without running the op."""
import math

import numpy as np
import pytest
import torch

import paraconv2d_b200 as pc
from paraconv2d_b200 import ptparaconv2d


def test_parameter_layout_and_tags():
    torch.manual_seed(0)
    m = pc.ParaConv2d(3, 5, (3, 5), stride=(2, 1), padding=2, dilation=(1, 2), h_factor=0.25, p_factor=0.5,
                      h_lr_factor=3.0, p_lr_factor=4.0, wd_factor=0.2)
    d = 3 * 3 * 5
    assert m.pars.shape == (2 * 5 * (d + 1),)
    assert m.pars.d == d and m.pars.isParaboloid
    assert (m.pars.h_lr_factor, m.pars.p_lr_factor, m.pars.wd_factor) == (3.0, 4.0, 0.2)
    h0, h, p, p0 = m.pars[:5], m.pars[5:5 + 5 * d], m.pars[5 + 5 * d:5 + 10 * d], m.pars[5 + 10 * d:]
    assert torch.all(h0 == 0.25) and torch.all(p0 == 0.5)         # spotlight: h0 = h_factor, p0 = p_factor
    assert float(h.abs().max()) <= 1e-4 and float(p.abs().max()) <= 1.0
    for t, v in ((m.kernel_size, [3, 5]), (m.stride, [2, 1]), (m.dilation, [1, 2])):
        assert t.dtype == torch.int32 and t.device.type == "cpu" and t.tolist() == v
    assert m.padding == (2, 2, 2, 2)


def test_two_tuple_padding_is_passed_to_pad_unchanged():
    m = pc.ParaConv2d(2, 2, 3, padding=(1, 2))
    assert m.padding == (1, 2)


def test_same_random_draws_as_the_reference_constructor():
    """The constructor draws, in order: a (m, d+1) uniform(+-1/sqrt(d+1))
    matrix, then h ~ U(+-input_factor*1e-4), then p ~ U(+-input_factor)
    (reference ptparaconv2d.py:12-19, 166-171), so a seeded construction gives
    the same pars as the reference."""
    torch.manual_seed(123)
    m = pc.ParaConv2d(2, 3, 3, input_factor=2.0)
    torch.manual_seed(123)
    d = 18
    tmp = torch.empty(3, d + 1).uniform_(-1 / math.sqrt(d + 1), 1 / math.sqrt(d + 1))
    h = torch.empty(3, d).uniform_(-2e-4, 2e-4)
    p = torch.empty(3, d).uniform_(-2.0, 2.0)
    expect = torch.cat((0.01 * torch.ones(3), h.reshape(-1), p.reshape(-1), 0.0001 * torch.ones(3)))
    assert torch.equal(m.pars.detach(), expect)


def test_linear_init_matches_pnnconvert():
    torch.manual_seed(5)
    m = pc.ParaConv2d(2, 4, 1, init="linear")
    torch.manual_seed(5)
    tmp = torch.empty(4, 3).uniform_(-1 / math.sqrt(3), 1 / math.sqrt(3))
    h, p, h0 = ptparaconv2d.pnnconvert(tmp[:, :2], tmp[:, 2], 20.0)
    expect = torch.cat((h0, h.reshape(-1), p.reshape(-1), 0.01 * torch.ones(4)))
    assert torch.allclose(m.pars.detach(), expect)
    # pnnconvert: h = w/|w|, h0 = b/|w| + 20, p = h*(20 - b/|w|)
    w, b = tmp[:, :2], tmp[:, 2]
    nw = w.norm(dim=1, keepdim=True)
    assert torch.allclose(h, w / nw) and torch.allclose(h0, b / nw[:, 0] + 20)


def test_unknown_init_and_init_from_numpy():
    with pytest.raises(Exception, match="Unknown Paraboloid initialization"):
        pc.ParaConv2d(2, 2, 3, init="xavier")
    arr = np.arange(2 * 2 * (18 + 1), dtype=np.float32)
    m = pc.ParaConv2d(2, 2, 3, init_from_numpy=arr)
    assert np.array_equal(m.pars.detach().numpy(), arr)


def test_state_dict_holds_the_flat_parameter_only():
    m = pc.ParaConv2d(3, 4, 3)
    sd = m.state_dict()
    assert list(sd) == ["pars"] and sd["pars"].shape == (2 * 4 * 28,)
