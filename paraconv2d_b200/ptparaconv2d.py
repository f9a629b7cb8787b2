"""Drop-in mirror of the reference Python module ``ptparaconv2d``
(GeoND-tech/ParaConv2d ``ptparaconv2d.py``) on top of the B200 op library.

Same names, constructor signature, parameter layout, defaults and
forward/backward semantics as the reference:

* ``spotlightinit`` / ``pnnconvert``: parameter initialisers (``ptparaconv2d.py:12-32``);
* ``ParaConv2dFunction``: autograd function calling ``torch.ops.ptparaconv2d``
  with fp16 inputs computed in fp32 (``ptparaconv2d.py:36-58``);
* ``ParaConv2d``: the module (``ptparaconv2d.py:62-221``); ``forward`` scales
  by ``input_factor``, pads with ``F.pad`` and calls the op.

One deliberate difference: the reference constructor runs a CPU warm-up
forward (``ptparaconv2d.py:212-213``).  This op has no CPU kernel, so the
warm-up runs on the current CUDA device when one is available and is skipped
otherwise; it has no side effects either way.

``ParaConv2d.forward`` computes what the reference's does: ``input_factor *
input``, a constant ``F.pad``, the op.  With constant padding on fp32/fp64
CUDA inputs it takes a fused route (``_PaddedParaConv2d``): the scale and the
pad are one pass (``paraconv2d_b200.pad_scale``), and the backward writes the
gradient of the unpadded input, times ``input_factor * grad_factor``,
directly from the kernels (``paraconv2d_b200.backward_interior``), instead of
slicing the padded gradient and scaling it twice.  When the input needs no
gradient (a network's first layer), the input-gradient kernels do not run at
all.  Other padding modes and fp16 inputs take the reference's route.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

from ._lib import load_op_library

load_op_library()


def spotlightinit(m, d, input_factor, h_factor=1.0, p_factor=-0.000001):
    """'spotlight' initialisation (reference ``ptparaconv2d.py:12-19``): h tiny
    uniform, h0 = h_factor, p uniform in +-input_factor, p0 = p_factor."""
    h = torch.empty(m, d)
    h.data.uniform_(-input_factor * 0.0001, input_factor * 0.0001)
    h0 = h_factor * torch.ones(m)
    p = torch.empty(m, d)
    p.data.uniform_(-input_factor, input_factor)
    p0 = p_factor * torch.ones(m)
    return (h, p, h0, p0)


def pnnconvert(w, b, offset=20.0):
    """Converts a linear layer (w, b) into paraboloid parameters (reference
    ``ptparaconv2d.py:23-32``): h = w/|w|, h0 = b/|w| + offset,
    p = h * (offset - b/|w|)."""
    H, D = w.size()
    tmpd = torch.sqrt(torch.sum(torch.square(w), dim=1))
    h = torch.div(w, tmpd.repeat(D, 1).t()).detach()
    tmpb = torch.div(b, tmpd)
    factor = 1.0
    h0 = (factor * (tmpb + offset)).detach()
    p = h.mul((factor * offset) - tmpb.repeat(D, 1).t()).detach()
    h = factor * h
    return (h, p, h0)


class ParaConv2dFunction(Function):
    """Autograd function of the op (reference ``ptparaconv2d.py:36-58``)."""

    @staticmethod
    def forward(ctx, input, pars, output_factor, kernel_size, stride, dilation, skip_input_grad, grad_factor):
        inputdtype = input.dtype
        if inputdtype == torch.float16:
            input = input.float()
        output, hsum = torch.ops.ptparaconv2d.forward(input, pars, float(output_factor), kernel_size, stride, dilation)
        ctx.save_for_backward(input, pars, hsum)
        ctx.output_factor = output_factor
        ctx.kernel_size = kernel_size
        ctx.stride = stride
        ctx.dilation = dilation
        ctx.skip_input_grad = skip_input_grad
        ctx.grad_factor = grad_factor
        return output.to(inputdtype)

    @staticmethod
    def backward(ctx, grad_output):
        input, pars, hsum = ctx.saved_tensors
        if grad_output.dtype == torch.float16:
            grad_output = grad_output.float()
        grad_input, grad_pars = torch.ops.ptparaconv2d.backward(
            grad_output, input, pars, hsum, float(ctx.output_factor), ctx.kernel_size, ctx.stride, ctx.dilation,
            ctx.skip_input_grad)
        if ctx.grad_factor != 1:
            grad_input = ctx.grad_factor * grad_input
        return grad_input, grad_pars, None, None, None, None, None, None


class _PaddedParaConv2d(Function):
    """input_factor * input -> constant pad -> op, with the backward of all
    three in the op's own kernels (see the module docstring)."""

    @staticmethod
    def forward(ctx, input, pars, output_factor, kernel_size, stride, dilation, skip_input_grad, grad_factor,
                padding, input_factor):
        xp = torch.ops.paraconv2d_b200.pad_scale(input, list(padding), float(input_factor))
        output, hsum = torch.ops.ptparaconv2d.forward(xp, pars, float(output_factor), kernel_size, stride, dilation)
        ctx.save_for_backward(xp, pars, hsum)
        ctx.output_factor = output_factor
        ctx.kernel_size = kernel_size
        ctx.stride = stride
        ctx.dilation = dilation
        ctx.skip_input_grad = skip_input_grad
        ctx.padding = list(padding)
        ctx.dx_scale = float(input_factor) * float(grad_factor)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        xp, pars, hsum = ctx.saved_tensors
        need = bool(ctx.needs_input_grad[0])
        grad_input, grad_pars = torch.ops.paraconv2d_b200.backward_interior(
            grad_output, xp, pars, hsum, float(ctx.output_factor), ctx.kernel_size, ctx.stride, ctx.dilation,
            ctx.skip_input_grad, ctx.padding, ctx.dx_scale, need)
        return (grad_input if need else None), grad_pars, None, None, None, None, None, None, None, None


class ParaConv2d(nn.Module):
    r"""2-D convolution with paraboloid neurons (reference ``ptparaconv2d.py:62-221``).

    For every output pixel and output channel j, with ``win`` the (flipped)
    input window:

    * ``hsum = h0[j] + h[j] . win``
    * ``out = output_factor * (hsum^2 - |win - p[j]|^2 - p0[j]^2)``

    Arguments (same names and defaults as the reference): ``in_channels``,
    ``out_channels``, ``kernel_size``, ``stride=1``, ``padding=0`` (an int pads
    all four sides; a tuple is passed to ``F.pad`` unchanged), ``dilation=1``,
    ``bias`` (ignored), ``padding_mode='constant'``, ``device``, ``dtype``,
    ``output_factor=1.0``, ``input_factor=1.0``, ``h_lr_factor``,
    ``p_lr_factor``, ``wd_factor`` (optimizer tags on ``pars``),
    ``skip_input_grad=False``, ``init='spotlight'|'linear'``, ``h_factor``,
    ``p_factor``, ``grad_factor=1.0``, ``init_from_numpy=None``.

    The parameters are one flat vector ``pars = [h0 (m) | h (m*d) | p (m*d) | p0 (m)]``,
    ``d = in_channels*k0*k1``, interchangeable with the reference's
    ``state_dict``.  Kernel sizes must be odd.
    """

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, bias=True,
                 padding_mode='constant', device=None, dtype=None, output_factor=1.0, input_factor=1.0,
                 h_lr_factor=1., p_lr_factor=1., wd_factor=0.1, skip_input_grad=False, init='spotlight',
                 h_factor=0.01, p_factor=0.0001, grad_factor=1., init_from_numpy=None):
        super().__init__()
        if type(kernel_size) == int:
            kernel_size = [kernel_size, kernel_size]
        if type(dilation) == int:
            dilation = [dilation, dilation]
        if type(stride) == int:
            stride = [stride, stride]
        if type(padding) == int:
            padding = (padding, padding, padding, padding)
        input_features = in_channels * kernel_size[0] * kernel_size[1]
        tmp = torch.empty(out_channels, input_features + 1)
        stdv = 1. / math.sqrt(tmp.size(1))
        tmp.data.uniform_(-stdv, stdv)
        if init == 'spotlight':
            tmph, tmpp, tmph0, tmpp0 = spotlightinit(out_channels, input_features, input_factor, h_factor, p_factor)
        elif init == "linear":
            w = tmp[:, 0:input_features]
            b = tmp[:, input_features]
            tmph, tmpp, tmph0 = pnnconvert(w, b, 20.0)
            tmpp0 = 0.01 * torch.ones(out_channels)
        else:
            raise Exception("Unknown Paraboloid initialization.")
        if dtype is not None:
            tmph0, tmph, tmpp0, tmpp = (t.to(dtype) for t in (tmph0, tmph, tmpp0, tmpp))
        if device is not None:
            tmph0, tmph, tmpp0, tmpp = (t.to(device) for t in (tmph0, tmph, tmpp0, tmpp))
        if init_from_numpy is not None:
            self.pars = nn.Parameter(torch.from_numpy(init_from_numpy))
        else:
            self.pars = nn.Parameter(torch.concat((tmph0, torch.reshape(tmph, (-1,)), torch.reshape(tmpp, (-1,)),
                                                   tmpp0), dim=0))
        self.pars.d = int(in_channels * kernel_size[0] * kernel_size[1])
        self.pars.isParaboloid = True
        self.pars.h_lr_factor = h_lr_factor
        self.pars.p_lr_factor = p_lr_factor
        self.pars.wd_factor = wd_factor
        self.output_factor = output_factor
        self.in_channels = in_channels
        self.out_channels = out_channels
        # CPU int32 tensors, read on the host by the op (reference ptparaconv2d.py:203-205).
        self.kernel_size = torch.tensor(kernel_size, dtype=torch.int)
        self.stride = torch.tensor(stride, dtype=torch.int)
        self.dilation = torch.tensor(dilation, dtype=torch.int)
        self.skip_input_grad = skip_input_grad
        self.padding = padding
        self.padding_mode = padding_mode
        self.input_factor = input_factor
        self.grad_factor = grad_factor
        self._warmup(dilation, kernel_size)

    def _warmup(self, dilation, kernel_size):
        if not torch.cuda.is_available():
            return
        dev = self.pars.device if self.pars.is_cuda else torch.device("cuda", torch.cuda.current_device())
        with torch.no_grad():
            pars = self.pars.detach().to(dev)
            dt = pars.dtype if pars.dtype in (torch.float32, torch.float64) else torch.float32
            x = torch.zeros(1, self.in_channels, dilation[0] * kernel_size[0], dilation[1] * kernel_size[1],
                            device=dev, dtype=dt)
            x = F.pad(self.input_factor * x, self.padding, mode=self.padding_mode)
            torch.ops.ptparaconv2d.forward(x, pars.to(dt), float(self.output_factor), self.kernel_size, self.stride,
                                           self.dilation)

    def _fused(self, input):
        return (self.padding_mode == 'constant' and input.is_cuda and input.dim() == 4
                and input.dtype in (torch.float32, torch.float64) and self.pars.dtype == input.dtype
                and len(self.padding) in (2, 4) and all(int(v) >= 0 for v in self.padding))

    def forward(self, input):
        if self._fused(input):
            return _PaddedParaConv2d.apply(input, self.pars, self.output_factor, self.kernel_size, self.stride,
                                           self.dilation, self.skip_input_grad, self.grad_factor,
                                           tuple(int(v) for v in self.padding), self.input_factor)
        x = self.input_factor * input
        x = F.pad(x, self.padding, mode=self.padding_mode)
        return ParaConv2dFunction.apply(x, self.pars, self.output_factor, self.kernel_size, self.stride,
                                        self.dilation, self.skip_input_grad, self.grad_factor)

    def extra_repr(self) -> str:
        return (f"in_channels={self.in_channels}, out_channels={self.out_channels}, "
                f"input_factor={self.input_factor}, output_factor={self.output_factor}, "
                f"kernel_size={self.kernel_size}")
