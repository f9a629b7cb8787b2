#!/usr/bin/env python
"""Throughput of the ParaConv2d layer on B200: forward and forward+backward
images/s on the 64->64-channel, 32x32, k3 layer with a batch of 128 images
per GPU (fp32, seeded synthetic data), plus the fraction of the op's
tensor-core roofline.

A "step" is one forward + backward pass of the layer over the per-GPU batch
(with --gpus N > 1, followed by an NCCL all-reduce of the parameter
gradient, the data-parallel training step; scaling is weak: 128 images per
GPU).  Output: one JSON line on rank 0.

  value     fwd+bwd images/s over all GPUs, inputs resident in HBM, through
            the C ABI (include/paraconv2d.h); L2 flushed before every step,
            outside the timed events
  e2e       the same through the public module (ParaConv2d forward +
            autograd backward), with the step's input and upstream gradient
            copied from pinned host memory and the parameter gradient read
            back, all inside the timed region
  roofline  the dominant kernel (largest summed CUDA-event time, timed per
            launch by the library's pc2d_timing_* hooks in a second timed
            pass of the same steps; the hooks stay off in the pass that gives
            value, because their events cost ~20 us per step and keep wgrad
            from starting while dgrad finishes) against the 3xTF32 tensor
            peak (a measured TF32 GEMM rate / 3)
  cpu_baseline  the reference CPU op on the host cores (bounded sample)

--impl reference times the reference's own CPU implementation of the op
(built from its sources into oracle/_ref; the oracle port where that build
is absent) on the host cores, same metric and workload.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
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

WORKLOAD = "c2"
METRIC = "fwd & fwd+bwd images/s (N=128, 64→64ch, 32×32, k3) on B200; % of roofline"
UNIT = "images/s"
L2_FLUSH_BYTES = 512 << 20

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of
# each main kernel on the c2 layer, from the ncu --set full capture summarised
# in profiles/tc_kernels_c2.md.  Writes that are still in L2 when a kernel ends
# are not counted by that capture.
NCU_TRAFFIC_BYTES = {
    ("c2", "forward"): 38.542336e6 + 13.854464e6,
    ("c2", "dgrad"): 105.669376e6 + 16.545280e6,
    ("c2", "wgrad"): 105.206016e6 + 14.017024e6,
}

# Kernel families the library can time (pc2d_timing_read).
KERNELS = ("forward", "dgrad", "wgrad", "simt_forward", "simt_dgrad", "simt_wgrad")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
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

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
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


# --------------------------------------------------------- CPU reference arm

def cpu_reference_rate(wl, cpu_seconds, threads):
    """images/s of the reference CPU op (fwd+bwd and fwd) on `threads` host
    threads, one image per task; the sample is sized to ~cpu_seconds of work."""
    import numpy as np

    import oracle
    from paraconv2d_b200 import workloads

    L = wl.layer
    x, pars, g = workloads.draw(wl, n=None)
    grad = workloads.draw_grad(wl, g)
    xp = workloads.pad_input(x, L.p)
    use_ref = oracle.load_reference()
    kind = "reference" if use_ref else "port"

    def one(i, with_bwd=True):
        xi = xp[i:i + 1].contiguous()
        if use_ref:
            out, hs = oracle.ref_forward(xi, pars[0], 1.0, L.k, L.s, 1)
            if with_bwd:
                oracle.ref_backward(grad[i:i + 1].contiguous(), xi, pars[0], hs, 1.0, L.k, L.s, 1, False)
        else:
            xn = xi.numpy()
            out, hs = oracle.forward(xn, pars[0].numpy(), 1.0, L.k, L.s, 1)
            if with_bwd:
                oracle.backward(grad[i:i + 1].numpy(), xn, pars[0].numpy(), hs, 1.0, L.k, L.s, 1, False)

    # calibrate on one image, single thread
    t0 = time.perf_counter()
    one(0)
    t1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    one(0, with_bwd=False)
    tf1 = time.perf_counter() - t0
    n_img = int(max(threads, min(wl.n, round(cpu_seconds / max(t1, 1e-6)))))
    n_img = max(threads, (n_img // threads) * threads)
    idx = [i % wl.n for i in range(n_img)]
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        list(ex.map(one, idx))
        wall = time.perf_counter() - t0
    rate = n_img / wall
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n_img} images of the {wl.name} layer ({wl.description}), fwd+bwd, one image per task on "
                      f"{threads} threads; single-thread fwd {1.0 / tf1:.3g} img/s, fwd+bwd {1.0 / t1:.3g} img/s",
            "fwd_value": threads / tf1 if tf1 > 0 else None, "seconds": wall}


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from paraconv2d_b200 import workloads

    wl = workloads.WORKLOADS[args.workload]
    cores = host_cores()
    per_step = max(2.0, args.cpu_seconds / max(1, args.steps))
    for _ in range(args.warmup):
        pass  # the reference CPU op has no warm-up state worth timing
    vals = []
    last = None
    for _ in range(args.steps):
        last = cpu_reference_rate(wl, per_step, cores)
        vals.append(last["value"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * wl.n / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": f"{wl.name}: {wl.description}", "per_gpu_batch": wl.n, "host_cores": cores},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": last["kind"], "sample": last["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm

def run_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    import paraconv2d_b200 as pc
    from paraconv2d_b200 import _lib, workloads

    wl = workloads.WORKLOADS[args.workload]
    L = wl.layer
    lib = _lib.cabi()
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

    def bwd():
        st = lib.pc2d_backward(0, gd.data_ptr(), xp.data_ptr(), p.data_ptr(), hsum.data_ptr(), 1.0, L.k, L.k, L.s,
                               L.s, 1, 1, n, C, H, W, m, 0, dx.data_ptr(), dp.data_ptr(), bwsb.data_ptr(), bws, sptr)
        if st != 0:
            raise RuntimeError(_lib.status_message(st))

    def allreduce():
        if pg is not None:
            pg.all_reduce(dp)

    def barrier():
        if pg is not None:
            pg.barrier()

    def max_over_ranks(v):
        if pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident steps, split into forward / backward events
    for _ in range(args.warmup):
        fwd()
        bwd()
        allreduce()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    # The headline pass runs with the library's per-kernel event timing off:
    # those events (two per kernel) cost ~20 us per step and sit between
    # dgrad and wgrad, which stops wgrad from starting on the SMs dgrad has
    # left.  A second pass of the same steps, with them on, gives the
    # per-kernel durations of the roofline.
    clk = ClockSampler(local)
    clk.__enter__()
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        fwd()
        ev[i][1].record(stream)
        bwd()
        ev[i][2].record(stream)
        allreduce()
        ev[i][3].record(stream)
    torch.cuda.synchronize()
    barrier()
    lib.pc2d_timing_reset()
    lib.pc2d_timing_enable(1)
    for i in range(args.steps):
        flush.zero_()
        fwd()
        bwd()
        allreduce()
    torch.cuda.synchronize()
    lib.pc2d_timing_enable(0)
    ktimes = _lib.kernel_times(KERNELS)
    barrier()
    t_fwd = [e[0].elapsed_time(e[1]) / 1e3 for e in ev]
    t_bwd = [e[1].elapsed_time(e[2]) / 1e3 for e in ev]
    t_step = [e[0].elapsed_time(e[3]) / 1e3 for e in ev]
    tot_step = max_over_ranks(sum(t_step))
    tot_fwd = max_over_ranks(sum(t_fwd))
    tot_bwd = max_over_ranks(sum(t_bwd))
    images = n * world * args.steps
    value = images / tot_step
    fwd_value = images / tot_fwd

    # ---- end to end through the public module, host buffers
    layer = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p).to(dev)
    with torch.no_grad():
        layer.pars.copy_(p)
    x_host = x.pin_memory()
    g_host = grad.pin_memory()
    dp_host = torch.empty(p.numel(), dtype=torch.float32).pin_memory()

    copy_stream = torch.cuda.Stream(dev)

    def e2e_step(start_event=None):
        # the upstream gradient crosses PCIe on a second stream, concurrently
        # with the input copy and the forward; it starts after the step's
        # start event, and the backward waits for it
        if start_event is not None:
            copy_stream.wait_event(start_event)
        else:
            copy_stream.wait_stream(stream)
        with torch.cuda.stream(copy_stream):
            gdd = g_host.to(dev, non_blocking=True)
            g_ready = torch.cuda.Event()
            g_ready.record(copy_stream)
        gdd.record_stream(stream)
        xd = x_host.to(dev, non_blocking=True)
        layer.pars.grad = None
        y = layer(xd)
        stream.wait_event(g_ready)
        y.backward(gdd)
        allreduce_e2e(layer.pars.grad)
        dp_host.copy_(layer.pars.grad, non_blocking=True)

    def allreduce_e2e(t):
        if pg is not None:
            pg.all_reduce(t)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_tot = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e_s.record(stream)
        e2e_step(e_s)
        e_e.record(stream)
        e_e.synchronize()
        e_tot += e_s.elapsed_time(e_e) / 1e3
    e_tot = max_over_ranks(e_tot)
    clk.__exit__(None, None, None)
    barrier()
    e2e_value = images / e_tot
    h2d = x_host.numel() * 4 + g_host.numel() * 4
    d2h = dp_host.numel() * 4

    # ---- roofline of the dominant kernel (per-launch CUDA-event times of
    # the second timed pass; each main kernel does 4*m*d*n*P*Q algorithmic
    # flops)
    peaks = measured_peaks()
    tf32 = measure_tf32_tflops(dev)
    peak_3x = tf32 / 3.0
    f_fwd = workloads.fwd_flops_per_image(wl) * n
    f_bwd = workloads.bwd_flops_per_image(wl) * n
    mean_fwd = tot_fwd / args.steps
    mean_bwd = tot_bwd / args.steps
    timed = {k: v for k, v in ktimes.items() if v[1] > 0}
    dom = max(timed, key=lambda k: timed[k][0]) if timed else "forward"
    dom_ms = timed[dom][0] / timed[dom][1] if timed else 1e3 * mean_fwd
    kflops = workloads.fwd_flops_per_image(wl) * n  # forward, dgrad and wgrad kernels alike
    achieved = kflops / (dom_ms / 1e3) / 1e12
    fwd_frac = f_fwd / mean_fwd / 1e12 / peak_3x
    bwd_frac = f_bwd / mean_bwd / 1e12 / peak_3x
    tr = NCU_TRAFFIC_BYTES.get((args.workload, dom))
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak_3x, "unit": "TFLOP/s", "frac": achieved / peak_3x,
        "traffic": tr, "kernel": dom, "kernel_ms": dom_ms,
        "kernel_ms_all": {k: v[0] / v[1] for k, v in timed.items()},
        "peak_source": f"measured TF32 cuBLAS GEMM {tf32:.0f} TFLOP/s on this GPU / 3 (3xTF32 issues three MMAs per "
                       f"algorithmic multiply-add); bf16 dense {peaks.get('bf16_tflops')} TFLOP/s of measured "
                       f"(MEASURED_PEAKS.json)",
        "fwd_frac": fwd_frac, "bwd_frac": bwd_frac,
        "hbm_gbs_fwd": workloads.fwd_bytes_per_image(wl) * n / mean_fwd / 1e9,
        "hbm_peak_gbs": peaks.get("hbm_gbs"),
    }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_reference_rate(wl, args.cpu_seconds, host_cores())
            cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": host_cores(), "kind": "port", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * tot_step / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": f"{wl.name}: {wl.description}", "per_gpu_batch": n, "global_batch": n * world,
                       "parallelism": f"dp{world}" if world > 1 else "single GPU",
                       "l2": f"flushed ({L2_FLUSH_BYTES >> 20} MiB write) before every step, outside the timed events",
                       "kernel_timing": "per-kernel CUDA events in a second pass of the same steps (off in the value pass)",
                       "precision": "fp32 via 3xTF32 tensor-core split where the tcgen05 kernels apply",
                       "algo": {0: "auto", 1: "simt", 2: "tc"}[lib.pc2d_get_algo()]},
            "fwd_images_per_s": fwd_value, "fwd_ms": 1e3 * mean_fwd, "bwd_ms": 1e3 * mean_bwd,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * launches_per_step(lib, ktimes, args.steps),
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def launches_per_step(lib, ktimes, steps):
    """Our kernel launches per device-resident step, from the timed main
    kernels: tcgen05 forward = 1 prep kernel + the main kernel; tcgen05
    dgrad = 1 prep + main; tcgen05 wgrad = main + fixed-order reduction;
    CUDA-core forward = 1; CUDA-core dgrad = 1; CUDA-core wgrad = 2."""
    per_main = {"forward": 2, "dgrad": 2, "wgrad": 2, "simt_forward": 1, "simt_dgrad": 1, "simt_wgrad": 2}
    total = sum(per_main[k] * v[1] for k, v in ktimes.items())
    return total // max(1, steps)


def run_stack(args):
    """Data-parallel training step of a multi-layer stack (the c5 workload:
    3->32->64->64->64, k3 p1, stride 2 on layers 2-3, 64x64 input, global batch
    1024, loss = sum(out^2)).  The global batch is split across the ranks
    (strong scaling); one bucketed NCCL all-reduce (SUM) of all parameter
    gradients per step."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    import paraconv2d_b200 as pc
    from paraconv2d_b200 import _lib, workloads
    from paraconv2d_b200.dp import GradAllReduce, shard

    wl = workloads.WORKLOADS[args.workload]
    lib = _lib.cabi()
    x, pars, _ = workloads.draw(wl)
    xs = shard(x, rank, world).contiguous()
    layers = []
    for i, (L, pr) in enumerate(zip(wl.layers, pars)):
        # the first layer's input needs no gradient: skip_input_grad, as the
        # reference module documents for the first layer of a network
        m = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p, skip_input_grad=(i == 0)).to(dev)
        with torch.no_grad():
            m.pars.copy_(pr.to(dev))
        layers.append(m)
    model = torch.nn.Sequential(*layers)
    reducer = GradAllReduce(model.parameters()) if world > 1 else None
    xd = xs.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(inp):
        for prm in model.parameters():
            prm.grad = None
        y = model(inp)
        (y * y).sum().backward()
        if reducer is not None:
            reducer()

    def max_over_ranks(v):
        if pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(xd)
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    clk = ClockSampler(local)
    clk.__enter__()
    tot = 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        flush.zero_()
        e0.record(stream)
        step(xd)
        e1.record(stream)
        e1.synchronize()
        tot += e0.elapsed_time(e1) / 1e3
    # per-kernel durations from a second pass with the library's event timing
    # on (kept out of the headline pass, as in run_layer)
    lib.pc2d_timing_reset()
    lib.pc2d_timing_enable(1)
    for _ in range(args.steps):
        flush.zero_()
        step(xd)
    torch.cuda.synchronize()
    lib.pc2d_timing_enable(0)
    ktimes = _lib.kernel_times(KERNELS)
    tot = max_over_ranks(tot)
    # end to end: the shard's input from pinned host memory, gradients read back
    x_host = xs.pin_memory()
    grads_host = [torch.empty(prm.numel()).pin_memory() for prm in model.parameters()]
    e_tot = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0.record(stream)
        step(x_host.to(dev, non_blocking=True))
        for gh, prm in zip(grads_host, model.parameters()):
            gh.copy_(prm.grad, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        e_tot += e0.elapsed_time(e1) / 1e3
    e_tot = max_over_ranks(e_tot)
    clk.__exit__(None, None, None)
    images = wl.n * args.steps
    flops_img = sum((2 if i == 0 else 3) * workloads.fwd_flops_per_image(wl, i) for i in range(len(wl.layers)))
    peak_3x = measure_tf32_tflops(dev) / 3.0
    if rank == 0:
        timed = {k: v for k, v in ktimes.items() if v[1] > 0}
        line = {
            "metric": f"{wl.name} data-parallel training step images/s", "value": images / tot, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)",
            "config": {"workload": f"{wl.name}: {wl.description}", "global_batch": wl.n,
                       "per_gpu_batch": xs.shape[0], "parallelism": f"dp{world}",
                       "l2": f"flushed ({L2_FLUSH_BYTES >> 20} MiB write) before every step, outside the timed events",
                       "kernel_timing": "per-kernel CUDA events in a second pass of the same steps (off in the value pass)"},
            "e2e": {"value": images / e_tot, "unit": UNIT, "h2d_bytes_per_step": x_host.numel() * 4,
                    "d2h_bytes_per_step": sum(g.numel() * 4 for g in grads_host)},
            "tensor_frac_of_step": flops_img * wl.n / (tot / args.steps) / 1e12 / peak_3x / world,
            "kernel_ms_per_step": {k: v[0] / args.steps for k, v in timed.items()},
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    from paraconv2d_b200 import workloads
    if len(workloads.WORKLOADS[args.workload].layers) > 1:
        return run_stack(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
