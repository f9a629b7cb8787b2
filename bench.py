#!/usr/bin/env python
"""Throughput of the ParaConv2d layer on B200: forward and forward+backward
images/s on the 64->64-channel, 32x32, k3 layer with a batch of 128 images
per GPU (fp32, seeded synthetic data), plus the fraction of the op's
tensor-core roofline; and the data-parallel training step of the 4-layer
stack (3->32->64->64->64, 64x64 input, global batch 1024 split across the
GPUs) in the same line.

A "step" of the headline is one forward + backward pass of the layer over
the per-GPU batch (with --gpus N > 1, followed by an NCCL all-reduce of the
parameter gradient; scaling is weak: 128 images per GPU).  Output: one JSON
line on rank 0.

  value     fwd+bwd images/s over all GPUs, inputs resident in HBM, through
            the C ABI (include/paraconv2d.h); L2 flushed before every step,
            outside the timed events
  e2e       the same through the public module (ParaConv2d forward +
            autograd backward), with the step's input and upstream gradient
            copied from pinned host memory and the output, the input gradient
            and the parameter gradient copied back, all inside the timed
            region; steps are pipelined as a training loop with an
            asynchronous loader runs them (the next step's inputs and the
            previous step's results cross PCIe while a step computes)
  roofline  the dominant kernel (largest summed CUDA-event time, timed per
            launch by the library's pc2d_timing_* hooks in a second timed
            pass of the same steps; the hooks stay off in the pass that gives
            value, because their events cost ~20 us per step and keep wgrad
            from starting while dgrad finishes) against the 3xTF32 tensor
            peak (a measured TF32 GEMM rate / 3)
  cpu_baseline  the reference CPU op on the host cores (bounded sample; N=1)
  dp_step   the stack's data-parallel training step (strong scaling): its
            images/s, the all-reduce time, and a check on rank 0 that the
            all-reduced gradients equal those of the whole batch computed in
            one process

--impl reference times the reference's own CPU implementation of the op
(built from its sources into oracle/_ref; the oracle port where that build
is absent) on the host cores, same metric and workload: each step is the
forward + backward of one image per host thread.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

UNIT = "images/s"
L2_FLUSH_BYTES = 512 << 20
STACK = "c5"

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of
# each main kernel on the c2 layer, from one ncu capture per kernel
# (the command is in TRAFFIC_SOURCE).  Writes still in L2 when a kernel ends
# are not counted by that capture.
NCU_TRAFFIC_BYTES = {
    ("c2", "forward"): 38.548480e6 + 14.362112e6,
    ("c2", "dgrad"): 105.651456e6 + 16.430592e6,
    ("c2", "wgrad"): 105.120000e6 + 14.597120e6,
}
TRAFFIC_SOURCE = ("ncu --set full --clock-control none -k regex:tc_<kernel>_kernel -c 1, one capture per kernel, of "
                  "python bench.py --workload c2 --steps 1 --warmup 1 --no-stack --no-cpu-baseline (not this run)")

# Kernel families the library can time (pc2d_timing_read).
KERNELS = ("forward", "dgrad", "wgrad", "simt_forward", "simt_dgrad", "simt_wgrad")


def load_workloads():
    """paraconv2d_b200/workloads.py by path: importing the package would load
    the op libraries, which the reference arm must not do."""
    name = "pc2d_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "paraconv2d_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def metric_of(wl):
    if len(wl.layers) > 1:
        return f"{wl.name} data-parallel training step images/s ({wl.description})"
    return f"fwd & fwd+bwd images/s ({wl.description}) on B200; % of roofline"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c2")
    ap.add_argument("--layer", type=int, default=None,
                    help="benchmark this layer of a multi-layer workload on its own (single-layer line)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-stack", action="store_true", help="skip the data-parallel stack block")
    ap.add_argument("--stack-steps", type=int, default=20)
    ap.add_argument("--grad-sum", choices=["peer", "nccl"], default="peer",
                    help="N > 1: sum the parameter gradient inside the backward over NVLink peer memory "
                         "(pc2d_backward_sum; the c5 step: one bucket by pc2d_comm_allreduce), or with NCCL "
                         "all-reduces (after the backward; the c5 step: one per layer, overlapped)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU work of the baseline sample")
    return ap.parse_args()


# ------------------------------------------------------------------ helpers

def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
            self.proc = None

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def measure_tf32_tflops(device):
    """Dense TF32 GEMM rate of this GPU (cuBLAS, 8192^3, best of 5), the
    denominator of the 3xTF32 roofline (not a number of this library)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device=device)
        b = torch.randn(n, n, device=device)
        for _ in range(3):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(5):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e) / 1e3)
        del a, b
        return 2.0 * n ** 3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


class Dist:
    """The process group of a torchrun launch (None at N=1), with the helpers
    every rank calls in the same order."""

    def __init__(self, world, dev):
        self.pg = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
            self.pg = dist
        self.dev = dev

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, v):
        if self.pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=self.dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def all_reduce(self, t):
        if self.pg is not None:
            self.pg.all_reduce(t)

    def close(self):
        if self.pg is not None:
            self.pg.barrier()
            self.pg.destroy_process_group()


# --------------------------------------------------------- CPU reference arm

def cpu_reference_step(wl, threads, use_ref):
    """One reference step on the host: forward + backward of `threads` images
    of the layer, one image per thread (the reference op is single-threaded
    and releases the GIL).  Returns (seconds, images, kind)."""
    import oracle

    workloads = load_workloads()
    L = wl.layer
    if not hasattr(cpu_reference_step, "cache"):
        x, pars, g = workloads.draw(wl, n=None)
        grad = workloads.draw_grad(wl, g)
        cpu_reference_step.cache = (workloads.pad_input(x, L.p), pars[0], grad)
        cpu_reference_step.next = 0
    xp, pars, grad = cpu_reference_step.cache
    if use_ref:
        oracle.load_reference()
    kind = "reference" if use_ref else "port"

    def one(i):
        xi = xp[i:i + 1].contiguous()
        if use_ref:
            out, hs = oracle.ref_forward(xi, pars, 1.0, L.k, L.s, 1)
            oracle.ref_backward(grad[i:i + 1].contiguous(), xi, pars, hs, 1.0, L.k, L.s, 1, False)
        else:
            xn = xi.numpy()
            out, hs = oracle.forward(xn, pars.numpy(), 1.0, L.k, L.s, 1)
            oracle.backward(grad[i:i + 1].numpy(), xn, pars.numpy(), hs, 1.0, L.k, L.s, 1, False)

    idx = [(cpu_reference_step.next + i) % wl.n for i in range(threads)]
    cpu_reference_step.next = (cpu_reference_step.next + threads) % wl.n
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        list(ex.map(one, idx))
        wall = time.perf_counter() - t0
    return wall, threads, kind


def cpu_reference_rate(wl, cpu_seconds, threads):
    """images/s of the reference CPU op (fwd+bwd) on `threads` host threads,
    over as many one-image-per-thread steps as fit in ~cpu_seconds."""
    import oracle

    use_ref = oracle.reference_available()
    wall, imgs, kind = cpu_reference_step(wl, threads, use_ref)
    steps = max(1, int(cpu_seconds / max(wall, 1e-3)) - 1)
    tot, n = 0.0, 0
    for _ in range(steps):
        w, i, _ = cpu_reference_step(wl, threads, use_ref)
        tot += w
        n += i
    rate = n / tot
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n} images of the {wl.name} layer ({wl.description}) in {steps} steps of {threads}, fwd+bwd, "
                      f"one image per thread on {threads} threads ({tot:.1f} s)"}


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import oracle

    workloads = load_workloads()
    wl = workloads.WORKLOADS[args.workload]
    if len(wl.layers) > 1:
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no multi-layer or data-parallel path"}))
        return 0
    cores = host_cores()
    use_ref = oracle.reference_available()
    for _ in range(args.warmup):
        cpu_reference_step(wl, cores, use_ref)
    walls, imgs, kind = [], 0, None
    for _ in range(args.steps):
        w, i, kind = cpu_reference_step(wl, cores, use_ref)
        walls.append(w)
        imgs += i
    tot = sum(walls)
    value = imgs / tot
    line = {
        "impl": "reference", "metric": metric_of(wl), "value": value, "unit": UNIT, "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": layer_config(wl, wl.n, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"each step: forward + backward of {cores} images of the {wl.name} layer "
                                   f"({wl.description}; images taken in turn from the seeded batch), one image per "
                                   f"thread on {cores} host threads; {imgs} images in {tot:.1f} s"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def layer_config(wl, n, world):
    """The `config` of the headline line (both arms)."""
    return {"workload": f"{wl.name}: {wl.description}", "per_gpu_batch": n, "global_batch": n * world,
            "parallelism": f"dp{world}" if world > 1 else "single GPU",
            "l2": f"value: flushed ({L2_FLUSH_BYTES >> 20} MiB write) before every step, outside the timed events; "
                  "e2e: pipelined steps without a flush, inputs copied fresh from the host every step, working set "
                  "per step larger than L2",
            "kernel_timing": "per-kernel CUDA events in a second pass of the same steps (off in the value pass)",
            "precision": "fp32 via 3xTF32 tensor-core split where the tcgen05 kernels apply"}


# ------------------------------------------------------------------ our arm

def bench_layer(args, wl, lib, D, rank, world):
    """The single-layer headline: device-resident steps through the C ABI,
    per-kernel times, the end-to-end leg through the module."""
    import paraconv2d_b200 as pc
    from paraconv2d_b200 import _lib

    workloads = load_workloads()
    dev = D.dev
    L = wl.layer
    x, pars, g = workloads.draw(wl)
    grad = workloads.draw_grad(wl, g)
    xp = workloads.pad_input(x, L.p).to(dev)
    p = pars[0].to(dev)
    gd = grad.to(dev)
    n, C, H, W = xp.shape
    m = L.cout
    P, Q = wl.out_hw(0)
    out = torch.empty((n, m, P, Q), device=dev)
    hsum = torch.empty_like(out)
    dx = torch.empty_like(xp)
    dp = torch.empty_like(p)
    fws = lib.pc2d_forward_workspace_size(0, n, C, H, W, m, L.k, L.k, L.s, L.s, 1, 1)
    bws = lib.pc2d_backward_workspace_size(0, n, C, H, W, m, L.k, L.k, L.s, L.s, 1, 1, 0)
    fwsb = torch.empty(max(fws, 1), dtype=torch.uint8, device=dev)
    bwsb = torch.empty(max(bws, 1), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def fwd():
        st = lib.pc2d_forward(0, xp.data_ptr(), p.data_ptr(), 1.0, L.k, L.k, L.s, L.s, 1, 1, n, C, H, W, m,
                              out.data_ptr(), hsum.data_ptr(), fwsb.data_ptr(), fws, sptr)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))

    def bwd_local(dst):
        st = lib.pc2d_backward(0, gd.data_ptr(), xp.data_ptr(), p.data_ptr(), hsum.data_ptr(), 1.0, L.k, L.k, L.s,
                               L.s, 1, 1, n, C, H, W, m, 0, dx.data_ptr(), dst.data_ptr(), bwsb.data_ptr(), bws, sptr)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))

    # N > 1: the data-parallel step sums the parameter gradient over the
    # ranks, inside the backward (NVLink peer memory) or with NCCL after it
    comm, grad_sum = None, None
    if world > 1:
        grad_sum = "NCCL all_reduce(SUM) of the parameter gradient after the backward"
        if args.grad_sum == "peer":
            from paraconv2d_b200.dp import PeerGradComm

            comm = PeerGradComm(p.numel())
            grad_sum = ("parameter gradient summed over the ranks inside the backward, over NVLink peer memory "
                        "(pc2d_backward_sum)")

    def bwd():
        if comm is None:
            bwd_local(dp)
            D.all_reduce(dp)
            return
        st = lib.pc2d_backward_sum(comm.comm, 0, gd.data_ptr(), xp.data_ptr(), p.data_ptr(), hsum.data_ptr(), 1.0,
                                   L.k, L.k, L.s, L.s, 1, 1, n, C, H, W, m, 0, dx.data_ptr(), dp.data_ptr(),
                                   bwsb.data_ptr(), bws, sptr)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))

    for _ in range(args.warmup):
        fwd()
        bwd()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    D.barrier()
    torch.cuda.synchronize()
    # The headline pass runs with the library's per-kernel event timing off:
    # those events (two per kernel) cost ~20 us per step and sit between
    # dgrad and wgrad, which stops wgrad from starting on the SMs dgrad has
    # left.  A second pass of the same steps, with them on, gives the
    # per-kernel durations of the roofline.
    clk = ClockSampler(D.dev.index).start()
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        fwd()
        ev[i][1].record(stream)
        bwd()
        ev[i][2].record(stream)
        ev[i][3].record(stream)
    torch.cuda.synchronize()
    D.barrier()
    lib.pc2d_timing_reset()
    lib.pc2d_timing_enable(1)
    for i in range(args.steps):
        flush.zero_()
        fwd()
        bwd()
    torch.cuda.synchronize()
    lib.pc2d_timing_enable(0)
    ktimes = _lib.kernel_times(KERNELS)
    D.barrier()
    t_fwd = [e[0].elapsed_time(e[1]) / 1e3 for e in ev]
    t_bwd = [e[1].elapsed_time(e[2]) / 1e3 for e in ev]
    t_step = [e[0].elapsed_time(e[3]) / 1e3 for e in ev]
    tot_step = D.max(sum(t_step))
    tot_fwd = D.max(sum(t_fwd))
    tot_bwd = D.max(sum(t_bwd))
    images = n * world * args.steps
    sum_check = None
    if comm is not None:
        # the fused sum against NCCL's all-reduce of this rank's own gradient
        ref = torch.empty_like(dp)
        bwd_local(ref)
        D.all_reduce(ref)
        bwd()
        torch.cuda.synchronize()
        err = float((dp - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
        sum_check = {"max_rel_diff_vs_nccl": D.max(err), "bitwise_equal_here": bool(torch.equal(dp, ref))}

    # ---- end to end through the public module, host buffers
    layer = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p).to(dev)
    with torch.no_grad():
        layer.pars.copy_(p)
    x_host = x.pin_memory()
    g_host = grad.pin_memory()
    out_host = torch.empty((n, m, P, Q), dtype=torch.float32).pin_memory()
    dx_host = torch.empty(x.shape, dtype=torch.float32).pin_memory()
    dp_host = torch.empty(p.numel(), dtype=torch.float32).pin_memory()
    # Steps are pipelined the way a training loop with an asynchronous data
    # loader runs them: step i+1's input and upstream gradient cross PCIe
    # (host -> device stream) while step i computes, and step i's output,
    # input gradient and parameter gradient go back (device -> host stream)
    # while step i+1 computes.  Two device slots for the inputs; a slot is
    # refilled only after the step that read it has finished its backward.
    # Every step's copies lie inside the timed region.
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    x_slots = [torch.empty(x.shape, device=dev) for _ in range(2)]
    g_slots = [torch.empty(grad.shape, device=dev) for _ in range(2)]
    slot_free = [None, None]
    slot_out = [None, None]

    def e2e_step(i):
        s = i % 2
        # at most two steps in flight, as with a loader's bounded queue: the
        # host waits for step i-2's results before it queues step i (an
        # unbounded run-ahead would grow the allocator's pool step by step)
        if slot_out[s] is not None:
            slot_out[s].synchronize()
        with torch.cuda.stream(h2d_stream):
            if slot_free[s] is not None:
                h2d_stream.wait_event(slot_free[s])
            x_slots[s].copy_(x_host, non_blocking=True)
            g_slots[s].copy_(g_host, non_blocking=True)
            in_ready = torch.cuda.Event()
            in_ready.record(h2d_stream)
        stream.wait_event(in_ready)
        xd = x_slots[s].detach().requires_grad_(True)
        layer.pars.grad = None
        y = layer(xd)
        y_ready = torch.cuda.Event()
        y_ready.record(stream)
        y.backward(g_slots[s])
        D.all_reduce(layer.pars.grad)
        done = torch.cuda.Event()
        done.record(stream)
        slot_free[s] = done
        yv, dxv, dpv = y.detach(), xd.grad, layer.pars.grad
        for t in (yv, dxv, dpv):
            t.record_stream(d2h_stream)
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(y_ready)
            out_host.copy_(yv, non_blocking=True)
            d2h_stream.wait_event(done)
            dx_host.copy_(dxv, non_blocking=True)
            dp_host.copy_(dpv, non_blocking=True)
            out_done = torch.cuda.Event()
            out_done.record(d2h_stream)
        slot_out[s] = out_done

    def e2e_run(steps, start_event=None, end_event=None):
        if start_event is not None:
            start_event.record(stream)
        h2d_stream.wait_stream(stream)
        for i in range(steps):
            e2e_step(i)
        stream.wait_stream(d2h_stream)
        if end_event is not None:
            end_event.record(stream)

    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize()
    D.barrier()
    flush.zero_()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_run(args.steps, e_s, e_e)
    e_e.synchronize()
    e_tot = D.max(e_s.elapsed_time(e_e) / 1e3)
    clk.stop()
    D.barrier()
    e2e_value = images / e_tot
    # one more step, checked against the device-resident step's results
    e2e_run(1)
    torch.cuda.synchronize()
    e2e_check = {
        "out_equal": bool(torch.equal(out_host, out.cpu())),
        "dx_max_rel_diff": float((dx_host - dx[:, :, L.p:H - L.p, L.p:W - L.p].cpu()).abs().max()
                                 / dx.abs().max().clamp_min(1e-30).cpu()),
        "dpars_max_rel_diff": float((dp_host - dp.cpu()).abs().max() / dp.abs().max().clamp_min(1e-30).cpu()),
    }
    h2d = (x_host.numel() + g_host.numel()) * 4
    d2h = (out_host.numel() + dx_host.numel() + dp_host.numel()) * 4

    # ---- roofline of the dominant kernel (per-launch CUDA-event times of
    # the second timed pass; each main kernel does 4*m*d*n*P*Q algorithmic
    # flops)
    peaks = measured_peaks()
    tf32 = measure_tf32_tflops(dev)
    peak_3x = tf32 / 3.0
    mean_fwd = tot_fwd / args.steps
    mean_bwd = tot_bwd / args.steps
    timed = {k: v for k, v in ktimes.items() if v[1] > 0}
    dom = max(timed, key=lambda k: timed[k][0]) if timed else "forward"
    dom_ms = timed[dom][0] / timed[dom][1] if timed else 1e3 * mean_fwd
    kflops = workloads.fwd_flops_per_image(wl) * n  # forward, dgrad and wgrad kernels alike
    achieved = kflops / (dom_ms / 1e3) / 1e12
    tr = NCU_TRAFFIC_BYTES.get((wl.name, dom))
    bf16_burst = peaks.get("bf16_tflops")
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak_3x, "unit": "TFLOP/s", "frac": achieved / peak_3x,
        "traffic": tr, "traffic_source": TRAFFIC_SOURCE if tr else None, "kernel": dom, "kernel_ms": dom_ms,
        "algorithmic_flops_per_launch": kflops,
        "kernel_ms_all": {k: v[0] / v[1] for k, v in timed.items()},
        "peak_source": f"measured TF32 cuBLAS GEMM {tf32:.0f} TFLOP/s on this GPU / 3 (3xTF32 issues three MMAs per "
                       f"algorithmic multiply-add); bf16 dense {bf16_burst} TFLOP/s of measured (MEASURED_PEAKS.json)",
        "frac_of_bf16_half": (achieved / (bf16_burst / 6.0)) if bf16_burst else None,
        "fwd_frac": workloads.fwd_flops_per_image(wl) * n / mean_fwd / 1e12 / peak_3x,
        "bwd_frac": workloads.bwd_flops_per_image(wl) * n / mean_bwd / 1e12 / peak_3x,
        "hbm_gbs_fwd": workloads.fwd_bytes_per_image(wl) * n / mean_fwd / 1e9,
        "hbm_peak_gbs": peaks.get("hbm_gbs"),
    }
    return {
        "value": images / tot_step, "ms_per_step": 1e3 * tot_step / args.steps,
        "fwd_images_per_s": images / tot_fwd, "fwd_ms": 1e3 * mean_fwd, "bwd_ms": 1e3 * mean_bwd,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": 1e3 * e_tot / args.steps,
                "pipelined": "step i+1's host->device copies and step i-1's device->host copies overlap step i "
                             "(two streams, two device input slots); no L2 flush between steps: each step's inputs "
                             "arrive fresh over PCIe and its working set exceeds the 126 MB L2",
                "check_vs_device_step": e2e_check},
        "gpu_launches": args.steps * (launches_per_step(ktimes, args.steps) + (1 if comm is not None else 0)),
        "roofline": roofline, "clock": clk, "algo": {0: "auto", 1: "simt", 2: "tc"}[lib.pc2d_get_algo()],
        "grad_sum": grad_sum, "grad_sum_check": sum_check, "comm": comm,
    }


def launches_per_step(ktimes, steps):
    """Our kernel launches per device-resident step, from the timed main
    kernels: tcgen05 forward = 1 prep kernel + the main kernel; tcgen05
    dgrad = 1 prep + main; tcgen05 wgrad = main + fixed-order reduction;
    CUDA-core forward = 1; CUDA-core dgrad = 1; CUDA-core wgrad = 2."""
    per_main = {"forward": 2, "dgrad": 2, "wgrad": 2, "simt_forward": 1, "simt_dgrad": 1, "simt_wgrad": 2}
    total = sum(per_main[k] * v[1] for k, v in ktimes.items())
    return total // max(1, steps)


def bench_stack(args, wl, lib, D, rank, world, steps):
    """Data-parallel training step of the layer stack (the c5 workload:
    3->32->64->64->64, k3 p1, stride 2 on layers 2-3, 64x64 input, global
    batch 1024, loss sum((2^-40 out)^2)).  The global batch is split across
    the ranks (strong scaling); the parameter gradients are summed across
    the ranks: one bucket of all layers' gradients over NVLink peer memory
    after the backward (--grad-sum peer, the default), or one asynchronous
    NCCL all-reduce per layer issued as soon as its gradient is accumulated
    (--grad-sum nccl)."""
    import paraconv2d_b200 as pc
    from paraconv2d_b200 import _lib
    from paraconv2d_b200.dp import GradAllReduce, PeerGradComm, shard

    workloads = load_workloads()
    dev = D.dev
    x, pars, _ = workloads.draw(wl)
    xs = shard(x, rank, world).contiguous()

    def make_model():
        mods = []
        for i, (L, pr) in enumerate(zip(wl.layers, pars)):
            # the first layer's input needs no gradient: skip_input_grad, as
            # the reference module documents for the first layer of a network
            m = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p, skip_input_grad=(i == 0)).to(dev)
            with torch.no_grad():
                m.pars.copy_(pr.to(dev))
            mods.append(m)
        return torch.nn.Sequential(*mods)

    model = make_model()
    params = list(model.parameters())
    # the gradient sum over the ranks: one bucket summed over NVLink peer
    # memory after the backward (--grad-sum peer), or one asynchronous NCCL
    # all-reduce per layer from its post-accumulate-grad hook (--grad-sum nccl)
    comm = None
    reducer = None
    if world > 1:
        if args.grad_sum == "peer":
            comm = PeerGradComm(sum(prm.numel() for prm in params))
            reducer = GradAllReduce(params, bucketed=True, peer=comm)
        else:
            reducer = GradAllReduce(params, bucketed=False)
    xd = xs.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(inp):
        for prm in params:
            prm.grad = None
        loss = workloads.stack_loss(model(inp))
        loss.backward()
        if reducer is not None:
            reducer()
        return loss

    for _ in range(args.warmup):
        step(xd)
    torch.cuda.synchronize()
    D.barrier()
    tot = 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(steps):
        flush.zero_()
        e0.record(stream)
        step(xd)
        e1.record(stream)
        e1.synchronize()
        tot += e0.elapsed_time(e1) / 1e3
    tot = D.max(tot)
    # per-kernel durations from a second pass with the library's event timing
    # on (kept out of the headline pass, as in the layer bench)
    D.barrier()
    lib.pc2d_timing_reset()
    lib.pc2d_timing_enable(1)
    for _ in range(steps):
        flush.zero_()
        step(xd)
    torch.cuda.synchronize()
    lib.pc2d_timing_enable(0)
    ktimes = _lib.kernel_times(KERNELS)
    # end to end: the shard's input from pinned host memory; the loss and the
    # summed gradients read back
    x_host = xs.pin_memory()
    grads_host = [torch.empty(prm.numel()).pin_memory() for prm in params]
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    D.barrier()
    e_tot = 0.0
    for _ in range(steps):
        flush.zero_()
        e0.record(stream)
        loss = step(x_host.to(dev, non_blocking=True))
        loss_host.copy_(loss.detach(), non_blocking=True)
        for gh, prm in zip(grads_host, params):
            gh.copy_(prm.grad, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        e_tot += e0.elapsed_time(e1) / 1e3
    e_tot = D.max(e_tot)
    # the sum on its own: one flat bucket of all gradients, blocking, by the
    # step's backend
    ar_ms = None
    if world > 1:
        flat = torch.cat([prm.grad.reshape(-1) for prm in params])

        def flat_sum():
            if comm is not None:
                comm.allreduce_(flat)
            else:
                D.all_reduce(flat)

        for _ in range(3):
            flat_sum()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(steps):
            flat_sum()
        a1.record(stream)
        a1.synchronize()
        ar_ms = D.max(a0.elapsed_time(a1) / steps)
    # data-parallel parity: the all-reduced gradients of the last step
    # against the gradient of the whole batch in one process (rank 0)
    got = [prm.grad.detach().clone() for prm in params]
    parity = None
    D.barrier()
    if rank == 0:
        ref_model = make_model()
        workloads.stack_loss(ref_model(x.to(dev))).backward()
        errs = []
        for a, prm in zip(got, ref_model.parameters()):
            b = prm.grad.detach()
            errs.append(float((a - b).abs().max() / b.abs().max().clamp_min(1e-300)))
        finite = all(bool(torch.isfinite(a).all()) for a in got)
        parity = {"max_rel_err_per_layer": errs, "tolerance": 1e-4, "finite": finite,
                  "pass": finite and max(errs) <= 1e-4,
                  "what": "max|allreduced - one-process full-batch| / max|full-batch| per layer's pars.grad"}
        del ref_model
    D.barrier()
    peak_3x = None
    if rank == 0:
        peak_3x = measure_tf32_tflops(dev) / 3.0
    images = wl.n * steps
    flops_img = sum((2 if i == 0 else 3) * workloads.fwd_flops_per_image(wl, i) for i in range(len(wl.layers)))
    timed = {k: v for k, v in ktimes.items() if v[1] > 0}
    res = {
        "metric": metric_of(wl), "value": images / tot, "unit": UNIT, "n_gpus": world, "steps": steps,
        "ms_per_step": 1e3 * tot / steps, "scaling": "strong", "global_batch": wl.n, "per_gpu_batch": int(xs.shape[0]),
        "allreduce": (None if world == 1 else
                      "one bucket of all layers' gradients summed over NVLink peer memory after the backward "
                      "(pc2d_comm_allreduce)" if comm is not None else
                      "one async NCCL all-reduce (SUM) per layer, issued from its post-accumulate-grad hook"),
        "allreduce_ms_flat_bucket": ar_ms,
        "e2e": {"value": images / e_tot, "unit": UNIT, "h2d_bytes_per_step": x_host.numel() * 4,
                "d2h_bytes_per_step": sum(g.numel() * 4 for g in grads_host) + 4},
        "kernel_ms_per_step": {k: v[0] / steps for k, v in timed.items()},
        "dp_parity": parity,
    }
    if peak_3x:
        res["tensor_frac_of_step"] = flops_img * wl.n / (tot / steps) / 1e12 / peak_3x / world
    if reducer is not None:
        reducer.remove()
    if comm is not None:
        comm.close()
    return res


def run_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D = Dist(world, dev)
    from paraconv2d_b200 import _lib

    workloads = load_workloads()
    lib = _lib.cabi()
    wl = workloads.WORKLOADS[args.workload]
    if args.layer is not None:
        wl = workloads.layer_workload(wl, args.layer)
    if len(wl.layers) > 1:
        clk = ClockSampler(local).start()
        res = bench_stack(args, wl, lib, D, rank, world, args.steps)
        clk.stop()
        if rank == 0:
            line = dict(res)
            line.update({"warmup": args.warmup, "higher_is_better": True, "vs_baseline": None, "dtype": "f32",
                         "data": "synthetic (seeded)",
                         "config": {"workload": f"{wl.name}: {wl.description}", "global_batch": wl.n,
                                    "per_gpu_batch": res["per_gpu_batch"], "parallelism": f"dp{world}"},
                         "clocks": clk.summary()})
            print(json.dumps(line), flush=True)
        D.close()
        return 0

    r = bench_layer(args, wl, lib, D, rank, world)
    stack = None
    if not args.no_stack:
        clk_s = ClockSampler(local).start()
        stack = bench_stack(args, workloads.WORKLOADS[STACK], lib, D, rank, world, args.stack_steps)
        clk_s.stop()
        stack["clocks"] = clk_s.summary()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference_rate(wl, args.cpu_seconds, host_cores())
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": host_cores(), "kind": "port", "sample": f"failed: {exc}"}
    if rank == 0:
        cfg = layer_config(wl, wl.n, world)
        line = {
            "metric": metric_of(wl), "value": r["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": cfg,
            "fwd_images_per_s": r["fwd_images_per_s"], "fwd_ms": r["fwd_ms"], "bwd_ms": r["bwd_ms"],
            "e2e": r["e2e"], "gpu_launches": r["gpu_launches"], "roofline": r["roofline"], "cpu_baseline": cpu,
            "clocks": r["clock"].summary(), "algo": r["algo"], "grad_sum": r["grad_sum"],
            "grad_sum_check": r["grad_sum_check"], "dp_step": stack,
        }
        print(json.dumps(line), flush=True)
    if r["comm"] is not None:
        r["comm"].close()
    D.close()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
