"""Seeded synthetic workloads of the ParaConv2d layer (no dataset is involved).

The five cases are the layer shapes the op is measured and checked on:

* ``c1``: N=2, 3->8 channels, 32x32, k3 s1 p1; U(-1,1) input, pars N(0, 0.1^2), seed 0
* ``c2``: N=128, 64->64, 32x32, k3 s1 p1; U(-1,1), N(0, 0.05^2), seed 1
* ``c3``: N=64, 64->128, 56x56, k3 s1 p1; |N(0,1)| input, N(0, 0.05^2), seed 2
* ``c4``: N=32, 3->64, 224x224, k7 s2 p3; U(-1,1), N(0, 0.1^2), seed 3
* ``c5``: a 4-layer stack 3->32->64->64->64, k3 p1, stride 2 on layers 2 and 3,
  64x64 input, global batch 1024, loss sum of squares of the output (scaled
  by an exact power of two, see ``stack_loss``); U(-1,1), N(0, 0.05^2), seed 4

Draw order on a CPU ``torch.Generator`` seeded per case: the unpadded input,
then the flat parameter vector of each layer, then the upstream gradient
N(0,1) (for c5 the gradient is that of the loss).  Every rank of a
data-parallel run draws the same full batch and keeps its own shard, so the
result does not depend on the number of GPUs.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Tuple

import torch


@dataclass(frozen=True)
class Layer:
    cin: int
    cout: int
    k: int
    s: int
    p: int


@dataclass(frozen=True)
class Workload:
    name: str
    n: int
    h: int
    w: int
    layers: Tuple[Layer, ...]
    sigma: float
    dist: str
    seed: int
    description: str = field(default="", compare=False)

    @property
    def layer(self) -> Layer:
        return self.layers[0]

    def out_hw(self, i: int = 0) -> Tuple[int, int]:
        h, w = self.h, self.w
        for L in self.layers[: i + 1]:
            h = (h + 2 * L.p - (L.k - 1) - 1) // L.s + 1
            w = (w + 2 * L.p - (L.k - 1) - 1) // L.s + 1
        return h, w

    def npars(self, i: int = 0) -> int:
        L = self.layers[i]
        return 2 * L.cout * (L.cin * L.k * L.k + 1)


WORKLOADS = {
    "c1": Workload("c1", 2, 32, 32, (Layer(3, 8, 3, 1, 1),), 0.1, "uniform", 0,
                   "N=2, 3->8ch, 32x32, k3 s1 p1"),
    "c2": Workload("c2", 128, 32, 32, (Layer(64, 64, 3, 1, 1),), 0.05, "uniform", 1,
                   "N=128, 64->64ch, 32x32, k3 s1 p1"),
    "c3": Workload("c3", 64, 56, 56, (Layer(64, 128, 3, 1, 1),), 0.05, "absnormal", 2,
                   "N=64, 64->128ch, 56x56, k3 s1 p1"),
    "c4": Workload("c4", 32, 224, 224, (Layer(3, 64, 7, 2, 3),), 0.1, "uniform", 3,
                   "N=32, 3->64ch, 224x224, k7 s2 p3"),
    "c5": Workload("c5", 1024, 64, 64, (Layer(3, 32, 3, 1, 1), Layer(32, 64, 3, 2, 1), Layer(64, 64, 3, 2, 1),
                                        Layer(64, 64, 3, 1, 1)), 0.05, "uniform", 4,
                   "4-layer stack 3->32->64->64->64, k3 p1, s2 on layers 2-3, 64x64, global N=1024"),
}


def layer_workload(wl: Workload, i: int) -> Workload:
    """Layer i of a stack as a single-layer workload of its own: the stack's
    batch and the layer's input size, with seeded U(-1,1) inputs (a benchmark
    stand-in for the previous layer's output) and the stack's parameter
    distribution."""
    L = wl.layers[i]
    h, w = wl.out_hw(i - 1) if i > 0 else (wl.h, wl.w)
    return Workload(f"{wl.name}.L{i}", wl.n, h, w, (L,), wl.sigma, "uniform", wl.seed + 100 * (i + 1),
                    f"layer {i} of {wl.name}: N={wl.n}, {L.cin}->{L.cout}ch, {h}x{w}, k{L.k} s{L.s} p{L.p}")


def draw(wl: Workload, n: int = None, dtype=torch.float32):
    """Seeded draw of (input [n,C,H,W] unpadded, [pars per layer], generator).
    With ``n`` smaller than the workload's batch, the first n images of the
    full draw are returned (the draw itself is always the full batch)."""
    g = torch.Generator().manual_seed(wl.seed)
    shape = (wl.n, wl.layers[0].cin, wl.h, wl.w)
    if wl.dist == "uniform":
        x = torch.rand(shape, generator=g, dtype=torch.float32) * 2 - 1
    elif wl.dist == "absnormal":
        x = torch.randn(shape, generator=g, dtype=torch.float32).abs()
    else:
        raise ValueError(wl.dist)
    pars: List[torch.Tensor] = []
    for i in range(len(wl.layers)):
        pars.append(torch.randn(wl.npars(i), generator=g, dtype=torch.float32) * wl.sigma)
    if n is not None:
        x = x[:n].contiguous()
    return x.to(dtype), [p.to(dtype) for p in pars], g


def draw_grad(wl: Workload, g: torch.Generator, n: int = None, dtype=torch.float32):
    """Upstream gradient N(0,1) of the (single-layer) output, drawn after the input and pars."""
    P, Q = wl.out_hw(0)
    grad = torch.randn((wl.n, wl.layers[0].cout, P, Q), generator=g, dtype=torch.float32)
    if n is not None:
        grad = grad[:n].contiguous()
    return grad.to(dtype)


def pad_input(x: torch.Tensor, p: int) -> torch.Tensor:
    return torch.nn.functional.pad(x, (p, p, p, p))


# Loss of the c5 stack.  sum(out^2) itself is about 4e56 at the full batch and
# every parameter gradient lies between 1e41 and 1e57: far beyond the fp32
# range (3.4e38), so in fp32 the loss is inf and all parameter gradients are
# inf/NaN, in the reference CPU op as much as here.  The stack's loss is
# therefore sum((2^-40 out)^2) = 2^-80 sum(out^2): multiplying by a power of
# two is exact, so every gradient is exactly 2^-80 times that of sum(out^2)
# wherever the latter is representable, and the step does the same work.
STACK_OUTPUT_SCALE = 2.0 ** -40


def stack_loss(y: torch.Tensor) -> torch.Tensor:
    """sum((2^-40 y)^2), the c5 training loss (see STACK_OUTPUT_SCALE)."""
    ys = y * STACK_OUTPUT_SCALE
    return (ys * ys).sum()


def fwd_flops_per_image(wl: Workload, i: int = 0) -> float:
    """Algorithmic flops of the forward contractions per image: 4*m*d*P*Q
    (h.win and p.win, 2 flops per multiply-add)."""
    L = wl.layers[i]
    P, Q = wl.out_hw(i)
    return 4.0 * L.cout * L.cin * L.k * L.k * P * Q


def bwd_flops_per_image(wl: Workload, i: int = 0, skip_input_grad: bool = False) -> float:
    """Algorithmic flops of the backward contractions per image: 8*m*d*P*Q
    (dgrad and wgrad), 4*m*d*P*Q without the input gradient."""
    return fwd_flops_per_image(wl, i) * (1.0 if skip_input_grad else 2.0)


def fwd_bytes_per_image(wl: Workload, i: int = 0) -> float:
    """Compulsory fp32 HBM bytes of the forward per image: padded input read
    plus output and hsum written."""
    L = wl.layers[i]
    P, Q = wl.out_hw(i)
    H, W = wl.out_hw(i - 1) if i > 0 else (wl.h, wl.w)
    return 4.0 * (L.cin * (H + 2 * L.p) * (W + 2 * L.p) + 2 * L.cout * P * Q)
