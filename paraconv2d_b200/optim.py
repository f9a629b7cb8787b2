"""SGD for networks of ParaConv2d layers, honouring the optimizer tags the
module sets on its flat parameter vector (reference ptparaconv2d.py:194-198):
``pars.h_lr_factor`` and ``pars.p_lr_factor`` multiply the learning rate of
the [h0 | h] and [p | p0] parts, ``pars.wd_factor`` multiplies the weight
decay ("Multiplies the learning rate / weight decay applied to the parameters
by the optimizer", the reference module's docstring).

The update is torch.optim.SGD's (momentum without dampening or Nesterov,
weight decay added to the gradient):

    d = grad + weight_decay * wd_factor * w
    buf = momentum * buf + d            (buf = d on the first step)
    w -= lr * lr_factor * buf

For a tagged ``pars`` on the GPU it is one fused kernel (``pc2d_param_step``:
one pass over the parameters, the gradient and the momentum buffer); other
parameters, and tagged ones on the CPU, take the same update in torch ops.
"""
from __future__ import annotations

import torch
from torch.optim import Optimizer

from . import _lib


def paraboloid_split(p: torch.Tensor):
    """(m, d) of a tagged flat parameter vector [h0 | h | p | p0] of
    2*m*(1+d) values, d = ``p.d`` (input channels x window)."""
    d = int(p.d)
    n = p.numel()
    if d < 0 or n % (2 * (d + 1)) != 0:
        raise ValueError(f"a paraboloid parameter vector of {n} values does not split with d = {d}")
    return n // (2 * (d + 1)), d


def sgd_step_reference(w, g, buf, first, nh, lr_h, lr_p, wd, momentum):
    """The update in torch ops (in place on w and buf): the first nh values
    use lr_h, the rest lr_p."""
    d = g.add(w, alpha=wd) if wd != 0 else g
    if momentum != 0:
        if first:
            buf.copy_(d)
        else:
            buf.mul_(momentum).add_(d)
        d = buf
    if nh >= w.numel():
        w.add_(d, alpha=-lr_h)
        return
    flat_w, flat_d = w.view(-1), d.reshape(-1)
    flat_w[:nh].add_(flat_d[:nh], alpha=-lr_h)
    flat_w[nh:].add_(flat_d[nh:], alpha=-lr_p)


class ParaboloidSGD(Optimizer):
    """SGD with the ParaConv2d tags applied per parameter (see the module
    docstring).  Parameters without the tags get plain SGD."""

    def __init__(self, params, lr: float, momentum: float = 0.0, weight_decay: float = 0.0):
        if lr < 0 or momentum < 0 or weight_decay < 0:
            raise ValueError("ParaboloidSGD: lr, momentum and weight_decay must be non-negative")
        super().__init__(params, dict(lr=lr, momentum=momentum, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self.state[p]
                first = "momentum_buffer" not in state
                if mom != 0 and first:
                    state["momentum_buffer"] = torch.empty_like(p, memory_format=torch.contiguous_format)
                buf = state.get("momentum_buffer")
                if getattr(p, "isParaboloid", False):
                    m, d = paraboloid_split(p)
                    hf, pf, wdf = float(p.h_lr_factor), float(p.p_lr_factor), float(p.wd_factor)
                    if p.is_cuda and p.dtype in (torch.float32, torch.float64):
                        g = p.grad.contiguous()
                        if not p.is_contiguous():
                            raise ValueError("ParaboloidSGD: the paraboloid parameter vector must be contiguous")
                        lib = _lib.cabi()
                        st = lib.pc2d_param_step(0 if p.dtype == torch.float32 else 1, p.data_ptr(), g.data_ptr(),
                                                 buf.data_ptr() if buf is not None else None, m, d, lr, hf, pf, wd,
                                                 wdf, mom, 1 if first else 0,
                                                 torch.cuda.current_stream(p.device).cuda_stream)
                        if st != 0:
                            raise RuntimeError(_lib.status_message(st))
                    else:
                        sgd_step_reference(p, p.grad, buf, first, m * (1 + d), lr * hf, lr * pf, wd * wdf, mom)
                else:
                    sgd_step_reference(p, p.grad, buf, first, p.numel(), lr, lr, wd, mom)
                if mom != 0:
                    state["momentum_buffer"] = buf
        return loss
