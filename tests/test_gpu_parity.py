"""Parity of the CUDA kernels with the reference CPU op, through the C ABI.

Reference values come from the golden fixtures (produced by the reference
op itself) and from the oracle (the C restatement pinned bit-for-bit to the
reference) on seeded subsets of the measured workloads.  Tolerances: see
pc2d_testutil (output/hsum elementwise 1e-5 + 1e-4|b|; gradients
max|a-b| <= 1e-4 max|b|).  Both kernel families are checked: AUTO (tcgen05
3xTF32 kernels where they apply) and SIMT (CUDA-core FMA).
"""
import zlib

import numpy as np
import pytest
import torch

import oracle
import paraconv2d_b200  # noqa: F401  (registers torch.ops.ptparaconv2d)
from cabi_runner import algo, backward, forward
from paraconv2d_b200 import PC2D_ALGO_AUTO, PC2D_ALGO_SIMT, _lib, workloads
from pc2d_testutil import (check_grads, check_outputs, check_vs_float64, elementwise_excess, golden_manifest,
                           load_golden, maxrel_excess, split_pars, torch_reference)

pytestmark = pytest.mark.gpu

ALGOS = {"auto": PC2D_ALGO_AUTO, "simt": PC2D_ALGO_SIMT}
NAMES = sorted(golden_manifest())


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("algo_name", sorted(ALGOS))
@pytest.mark.parametrize("name", NAMES)
def test_golden(name, algo_name):
    a, meta = load_golden(name)
    k, s, dl, f = meta["kernel_size"], meta["stride"], meta["dilation"], meta["factor"]
    C = meta["C"]
    d = C * k[0] * k[1]
    with algo(ALGOS[algo_name]):
        x, pars = _cuda(a["x"]), _cuda(a["pars"])
        out, hsum = forward(x, pars, f, k, s, dl)
        dx, dpars = backward(_cuda(a["grad"]), x, pars, _cuda(a["hsum"]), f, k, s, dl, meta["skip_input_grad"])
        torch.cuda.synchronize()
    check_outputs(out.cpu().numpy(), hsum.cpu().numpy(), a["out"], a["hsum"])
    check_grads(dx.cpu().numpy(), dpars.cpu().numpy(), a["dx"], a["dpars"], meta["m"], d, meta["skip_input_grad"])
    # the fixture holds the reference op's own result: ours may be no further
    # from the exact (fp64) gradients than twice as far as that result is
    _, _, rdx, rdp = torch_reference(a["x"], a["pars"], f, k, s, dl, grad=a["grad"],
                                     skip_input_grad=meta["skip_input_grad"])
    check_vs_float64(dx.cpu().numpy(), dpars.cpu().numpy(), a["dx"], a["dpars"], rdx, rdp, meta["m"], d,
                     meta["skip_input_grad"])


def _subset_case(name, n):
    wl = workloads.WORKLOADS[name]
    L = wl.layer
    x, pars, g = workloads.draw(wl, n=n)
    grad = workloads.draw_grad(wl, g, n=n)
    xp = workloads.pad_input(x, L.p)
    return wl, L, xp.numpy(), pars[0].numpy(), grad.numpy()


@pytest.mark.parametrize("algo_name", sorted(ALGOS))
@pytest.mark.parametrize("name,n", [("c1", 2), ("c2", 2), ("c3", 1), ("c4", 1)])
def test_workload_subset_vs_oracle(name, n, algo_name):
    """The first n images of each measured workload against the oracle."""
    wl, L, xp, pars, grad = _subset_case(name, n)
    ref_out, ref_hs = oracle.forward(xp, pars, 1.0, L.k, L.s, 1)
    ref_dx, ref_dp = oracle.backward(grad, xp, pars, ref_hs, 1.0, L.k, L.s, 1, False)
    d = L.cin * L.k * L.k
    with algo(ALGOS[algo_name]):
        x, p = _cuda(xp), _cuda(pars)
        out, hsum = forward(x, p, 1.0, L.k, L.s, 1)
        dx, dp = backward(_cuda(grad), x, p, _cuda(ref_hs), 1.0, L.k, L.s, 1)
        torch.cuda.synchronize()
    check_outputs(out.cpu().numpy(), hsum.cpu().numpy(), ref_out, ref_hs)
    check_grads(dx.cpu().numpy(), dp.cpu().numpy(), ref_dx, ref_dp, L.cout, d)
    _, _, rdx, rdp = torch_reference(xp, pars, 1.0, (L.k, L.k), L.s, 1, grad=grad)
    check_vs_float64(dx.cpu().numpy(), dp.cpu().numpy(), ref_dx, ref_dp, rdx, rdp, L.cout, d)


@pytest.mark.parametrize("name", ["c2", "c3", "c4"])
def test_full_size_forward_vs_float64(name):
    """Full-size forward of each measured workload against the float64 torch
    restatement: same elementwise tolerance as against the oracle."""
    wl = workloads.WORKLOADS[name]
    L = wl.layer
    x, pars, g = workloads.draw(wl)
    xp = workloads.pad_input(x, L.p).cuda()
    p = pars[0].cuda()
    out, hsum = forward(xp, p, 1.0, L.k, L.s, 1)
    ref_out, ref_hs = torch_reference(xp, p, 1.0, (L.k, L.k), L.s, 1)
    torch.cuda.synchronize()
    assert elementwise_excess(out.cpu().numpy(), ref_out) <= 1.0
    assert elementwise_excess(hsum.cpu().numpy(), ref_hs) <= 1.0


@pytest.mark.parametrize("name", ["c2", "c3"])
def test_full_size_backward_vs_float64(name):
    """Full-size c2 and c3 backward (c3 takes the two-stage wgrad variant):
    gradients against the float64 torch restatement, max|a-b| <= 1e-4 max|b|,
    and batch additivity (grads of the full batch = sum over two halves)."""
    wl = workloads.WORKLOADS[name]
    L = wl.layer
    x, pars, g = workloads.draw(wl)
    grad = workloads.draw_grad(wl, g).cuda()
    xp = workloads.pad_input(x, L.p).cuda()
    p = pars[0].cuda()
    out, hsum = forward(xp, p, 1.0, L.k, L.s, 1)
    dx, dp = backward(grad, xp, p, hsum, 1.0, L.k, L.s, 1)
    _, _, rdx, rdp = torch_reference(xp, p, 1.0, (L.k, L.k), L.s, 1, grad=grad)
    d = L.cin * L.k * L.k
    check_grads(dx.cpu().numpy(), dp.cpu().numpy(), rdx, rdp, L.cout, d)
    h = wl.n // 2
    dpa = backward(grad[:h].contiguous(), xp[:h].contiguous(), p, hsum[:h].contiguous(), 1.0, L.k, L.s, 1)[1]
    dpb = backward(grad[h:].contiguous(), xp[h:].contiguous(), p, hsum[h:].contiguous(), 1.0, L.k, L.s, 1)[1]
    assert maxrel_excess((dpa + dpb).cpu().numpy(), dp.cpu().numpy()) <= 1.0


@pytest.mark.parametrize("name", ["c2", "c3"])
def test_full_size_gradient_error_within_twice_the_oracle(name):
    """Full-size c2 and c3 gradients: per tensor, max|a - b64| / max|b64| is
    at most twice the reference fp32 op's own (the oracle, whole batch in one
    call, as the reference computes it), or 2^-18 -- the two-part policy of
    the fixtures, here at the configured sizes, where the parameter
    gradients sum 131k (c2) and 200k (c3) pixels per element.  The oracle
    takes about 35 s (c2) and 110 s (c3) of one host core."""
    wl = workloads.WORKLOADS[name]
    L = wl.layer
    x, pars, g = workloads.draw(wl)
    grad = workloads.draw_grad(wl, g)
    xp = workloads.pad_input(x, L.p)
    p = pars[0]
    out, hsum = forward(xp.cuda(), p.cuda(), 1.0, L.k, L.s, 1)
    dx, dp = backward(grad.cuda(), xp.cuda(), p.cuda(), hsum, 1.0, L.k, L.s, 1)
    _, _, rdx, rdp = torch_reference(xp.cuda().double(), p.cuda().double(), 1.0, (L.k, L.k), L.s, 1,
                                     grad=grad.cuda().double())
    o_out, o_hs = oracle.forward(xp.numpy(), p.numpy(), 1.0, L.k, L.s, 1)
    o_dx, o_dp = oracle.backward(grad.numpy(), xp.numpy(), p.numpy(), o_hs, 1.0, L.k, L.s, 1)
    d = L.cin * L.k * L.k
    names = ("dx", "dh0", "dh", "dp", "dp0")
    ours = (dx.cpu().numpy(),) + tuple(split_pars(dp.cpu().numpy(), L.cout, d))
    orac = (np.asarray(o_dx),) + tuple(split_pars(o_dp, L.cout, d))
    ref = (np.asarray(rdx),) + tuple(split_pars(np.asarray(rdp), L.cout, d))
    bad = []
    for nm, a, o, b in zip(names, ours, orac, ref):
        b = np.asarray(b, np.float64)
        scale = np.abs(b).max()
        e_ours = np.abs(np.asarray(a, np.float64) - b).max() / scale
        e_orac = np.abs(np.asarray(o, np.float64) - b).max() / scale
        if e_ours > max(2.0 * e_orac, 2.0 ** -18):
            bad.append(f"{nm}: {e_ours:.3g} vs oracle {e_orac:.3g}")
    assert not bad, f"{name}: gradient error above twice the fp32 oracle's: {bad}"


# Medium problems that take the tensor-core paths the measured workloads do
# not: 64-K forward stages with per-channel halo copies (odd planes), 48-wide
# channel blocks, two output-channel blocks, strided + dilated dgrad phases,
# and the single-tensor-copy halo with 32-wide blocks.
MEDIUM = {
    "c40_m48_k3x5_s2x1_dl1x2_odd": dict(n=3, C=40, H=23, W=23, m=48, k=(3, 5), s=(2, 1), dl=(1, 2)),
    "c64_m32_k3_aligned": dict(n=2, C=64, H=18, W=18, m=32, k=(3, 3), s=(1, 1), dl=(1, 1)),
    "c48_m80_k3_s2": dict(n=2, C=48, H=21, W=21, m=80, k=(3, 3), s=(2, 2), dl=(1, 1)),
    # few input channels: the output-pixel GEMM + col2im input gradient
    "c5_m24_k5x3_s1x2_dl2x1_narrow": dict(n=16, C=5, H=60, W=60, m=24, k=(5, 3), s=(1, 2), dl=(2, 1)),
    # narrow windows (d <= 31, m <= 32): CUDA-core parameter gradients; 154
    # output pixels per image (not a multiple of 4: element-wise staging)
    "c1_m20_k5_s2_dl2x1_window25": dict(n=3, C=1, H=29, W=31, m=20, k=(5, 5), s=(2, 2), dl=(2, 1)),
    # the widest such window (31 elements, ones column at 31), 32 channels
    "c31_m32_k1_window31": dict(n=2, C=31, H=12, W=12, m=32, k=(1, 1), s=(1, 1), dl=(1, 1)),
    # strided and dilated, 40 input channels, odd m, 24 images
    "c40_m21_k3_s2_dl1x2": dict(n=24, C=40, H=63, W=63, m=21, k=(3, 3), s=(2, 2), dl=(1, 2)),
}


@pytest.mark.parametrize("name", sorted(MEDIUM))
def test_medium_shapes_vs_float64(name):
    """Forward and backward of seeded medium problems against the float64
    torch restatement (outputs elementwise 1e-5 + 1e-4|b|, gradients
    max|a-b| <= 1e-4 max|b|)."""
    cfg = MEDIUM[name]
    n, C, H, W, m = cfg["n"], cfg["C"], cfg["H"], cfg["W"], cfg["m"]
    k, s, dl = cfg["k"], cfg["s"], cfg["dl"]
    d = C * k[0] * k[1]
    gen = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    x = torch.rand(n, C, H, W, generator=gen) * 2 - 1
    pars = torch.cat([torch.full((m,), 0.01), torch.randn(m * d, generator=gen) * 0.05,
                      (torch.rand(m * d, generator=gen) * 2 - 1) * 0.5, torch.full((m,), 0.01)])
    xd, pd = x.cuda(), pars.cuda()
    with algo(PC2D_ALGO_AUTO):
        out, hsum = forward(xd, pd, 1.0, k, s, dl)
        g = torch.randn(out.shape, generator=gen)
        dx, dp = backward(g.cuda(), xd, pd, hsum, 1.0, k, s, dl)
        torch.cuda.synchronize()
    ref_out, ref_hs, rdx, rdp = torch_reference(xd, pd, 1.0, k, s, dl, grad=g.cuda())
    check_outputs(out.cpu().numpy(), hsum.cpu().numpy(), ref_out, ref_hs)
    check_grads(dx.cpu().numpy(), dp.cpu().numpy(), rdx, rdp, m, d)


def test_full_size_backward_c4_vs_float64():
    """Full-size c4 backward (3 input channels: the output-pixel GEMM + col2im
    input gradient, k7 stride 2) against the float64 torch restatement."""
    wl = workloads.WORKLOADS["c4"]
    L = wl.layer
    x, pars, g = workloads.draw(wl)
    grad = workloads.draw_grad(wl, g).cuda()
    xp = workloads.pad_input(x, L.p).cuda()
    p = pars[0].cuda()
    out, hsum = forward(xp, p, 1.0, L.k, L.s, 1)
    dx, dp = backward(grad, xp, p, hsum, 1.0, L.k, L.s, 1)
    _, _, rdx, rdp = torch_reference(xp, p, 1.0, (L.k, L.k), L.s, 1, grad=grad)
    check_grads(dx.cpu().numpy(), dp.cpu().numpy(), rdx, rdp, L.cout, L.cin * L.k * L.k)


@pytest.mark.parametrize("algo_name", sorted(ALGOS))
def test_deterministic(algo_name):
    """No floating-point atomics: two runs are bitwise identical."""
    wl, L, xp, pars, grad = _subset_case("c2", 4)
    with algo(ALGOS[algo_name]):
        x, p, g = _cuda(xp), _cuda(pars), _cuda(grad)
        r1 = forward(x, p, 1.0, L.k, L.s, 1)
        r2 = forward(x, p, 1.0, L.k, L.s, 1)
        b1 = backward(g, x, p, r1[1], 1.0, L.k, L.s, 1)
        b2 = backward(g, x, p, r1[1], 1.0, L.k, L.s, 1)
    for u, v in zip(r1 + b1, r2 + b2):
        assert torch.equal(u, v)


def test_forward_batch_independent():
    """Each image's output does not depend on the rest of the batch (bitwise)."""
    wl, L, xp, pars, grad = _subset_case("c2", 3)
    x, p = _cuda(xp), _cuda(pars)
    full = forward(x, p, 1.0, L.k, L.s, 1)
    one = forward(x[1:2].contiguous(), p, 1.0, L.k, L.s, 1)
    assert torch.equal(full[0][1:2], one[0]) and torch.equal(full[1][1:2], one[1])


def test_tc_and_simt_agree():
    """The two kernel families agree to well within the tolerance."""
    wl, L, xp, pars, grad = _subset_case("c3", 1)
    x, p = _cuda(xp), _cuda(pars)
    with algo(PC2D_ALGO_AUTO):
        a = forward(x, p, 1.0, L.k, L.s, 1)
    with algo(PC2D_ALGO_SIMT):
        b = forward(x, p, 1.0, L.k, L.s, 1)
    assert elementwise_excess(a[0].cpu().numpy(), b[0].cpu().numpy()) <= 0.5
    assert elementwise_excess(a[1].cpu().numpy(), b[1].cpu().numpy()) <= 0.5


def test_edge_empty_batch_and_m1():
    x = torch.zeros((0, 3, 8, 8), device="cuda")
    pars = torch.randn(2 * 1 * (27 + 1), device="cuda")
    out, hs = forward(x, pars, 1.0, 3, 1, 1)
    assert out.shape == (0, 1, 6, 6)
    dx, dp = backward(torch.zeros_like(out), x, pars, hs, 1.0, 3, 1, 1)
    assert dx.shape == x.shape and torch.count_nonzero(dp) == 0


def test_bounded_wait_selftest():
    """A device-side wait on a barrier nothing completes returns by itself
    and records PC2D_ERR_TIMEOUT; the next call of the op raises it (read from
    the host mirror of the status word, without synchronising), until the
    status is cleared; the context stays usable."""
    lib = _lib.cabi()
    x = torch.rand(1, 3, 8, 8, device="cuda")
    pars = torch.randn(2 * 4 * 28, device="cuda") * 0.1
    k = torch.tensor([3, 3], dtype=torch.int)
    one = torch.tensor([1, 1], dtype=torch.int)
    ref = torch.ops.ptparaconv2d.forward(x, pars, 1.0, k, one, one)
    assert lib.pc2d_clear_device_status() == 0
    assert lib.pc2d_selftest_bounded_wait(200000, None) == 0
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="PC2D_ERR_TIMEOUT"):
        torch.ops.ptparaconv2d.forward(x, pars, 1.0, k, one, one)
    with pytest.raises(RuntimeError, match="PC2D_ERR_TIMEOUT"):
        torch.ops.ptparaconv2d.backward(torch.ones_like(ref[0]), x, pars, ref[1], 1.0, k, one, one, False)
    assert lib.pc2d_device_status() == _lib.PC2D_ERR_TIMEOUT
    assert lib.pc2d_clear_device_status() == 0
    assert lib.pc2d_device_status() == 0
    out = torch.ops.ptparaconv2d.forward(x, pars, 1.0, k, one, one)
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])


def test_no_device_errors_after_suite():
    assert _lib.cabi().pc2d_device_status() == 0


@pytest.mark.parametrize("name,n", [("c2", 16), ("c4", 4)])
def test_backward_outputs_ordered_on_stream(name, n):
    """wgrad may start while dgrad still runs (programmatic launch) and waits
    for it only at its end; work queued on the stream right after the
    backward, with no host synchronisation in between, must still see the
    finished input gradient and parameter gradient.  c2 takes the implicit
    dgrad kernel, c4 (3 input channels) the GEMM + col2im path."""
    wl, L, xp, pars, grad = _subset_case(name, n)
    x, p, g = _cuda(xp), _cuda(pars), _cuda(grad)
    _, hsum = forward(x, p, 1.0, L.k, L.s, 1)
    torch.cuda.synchronize()
    sums = []
    for _ in range(3):
        dx, dp = backward(g, x, p, hsum, 1.0, L.k, L.s, 1)
        # queued behind the backward on the same stream, no sync
        early = torch.stack([dx.double().abs().sum(), dp.double().abs().sum(), dx.double().sum()])
        torch.cuda.synchronize()
        late = torch.stack([dx.double().abs().sum(), dp.double().abs().sum(), dx.double().sum()])
        assert torch.equal(early, late)
        sums.append(late)
    assert all(torch.equal(sums[0], s) for s in sums[1:])

