"""Data-parallel gradient of the c5 stack through the CUDA kernels: two ranks,
each with its shard of the batch, sum their parameter gradients; the result
must equal the gradient of the whole batch computed in one process
(max|a-b| <= 1e-4 max|b| per layer: the two differ only in the order of the
fp32 sums).  Three modes of GradAllReduce are checked: one NCCL bucket after
the backward, one asynchronous NCCL all-reduce per layer issued as soon as
that layer's gradient is accumulated, and (two GPUs) one bucket summed over
NVLink peer memory (pc2d_comm_allreduce).

The ranks use NCCL with one GPU each when two GPUs are visible, else gloo
with both ranks on GPU 0 (no kernel of one rank waits for the other's; the
ranks meet only in the host-side all-reduce).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

GLOBAL_BATCH = 32


def _model(dev):
    import paraconv2d_b200 as pc
    from paraconv2d_b200 import workloads

    wl = workloads.WORKLOADS["c5"]
    _, pars, _ = workloads.draw(wl, n=1)
    mods = []
    for i, (L, pr) in enumerate(zip(wl.layers, pars)):
        m = pc.ParaConv2d(L.cin, L.cout, L.k, stride=L.s, padding=L.p, skip_input_grad=(i == 0)).to(dev)
        with torch.no_grad():
            m.pars.copy_(pr.to(dev))
        mods.append(m)
    return torch.nn.Sequential(*mods)


def _batch():
    from paraconv2d_b200 import workloads

    x, _, _ = workloads.draw(workloads.WORKLOADS["c5"], n=GLOBAL_BATCH)
    return x


def _grads(model):
    return torch.cat([p.grad.reshape(-1) for p in model.parameters()]).cpu()


def _worker(rank, world, port, mode, outdir):
    import torch.distributed as dist

    from paraconv2d_b200 import workloads
    from paraconv2d_b200.dp import GradAllReduce, PeerGradComm, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    ngpu = torch.cuda.device_count()
    dev = torch.device("cuda", rank % ngpu)
    torch.cuda.set_device(dev)
    backend = "nccl" if ngpu >= world else "gloo"
    kw = {"device_id": dev} if backend == "nccl" else {}
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), **kw)
    try:
        model = _model(dev)
        comm = None
        if mode == "peer_bucket":
            comm = PeerGradComm(sum(p.numel() for p in model.parameters()))
            red = GradAllReduce(model.parameters(), bucketed=True, peer=comm)
        else:
            red = GradAllReduce(model.parameters(), bucketed=(mode == "one_bucket"))
        x = shard(_batch(), rank, world).to(dev)
        workloads.stack_loss(model(x)).backward()
        red()
        torch.cuda.synchronize()
        torch.save(_grads(model), os.path.join(outdir, f"rank{rank}.pt"))
        red.remove()
        if comm is not None:
            comm.close()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("mode", ["one_bucket", "per_layer_overlapped", "peer_bucket"])
def test_two_rank_gradient_equals_full_batch(mode, tmp_path):
    from paraconv2d_b200 import workloads
    from pc2d_testutil import maxrel_excess

    dev = torch.device("cuda", 0)
    model = _model(dev)
    workloads.stack_loss(model(_batch().to(dev))).backward()
    ref = [p.grad.detach().cpu().clone() for p in model.parameters()]
    if mode == "peer_bucket" and torch.cuda.device_count() < 2:
        pytest.skip("the peer sum needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), mode, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        got = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        off = 0
        for i, g in enumerate(ref):
            e = maxrel_excess(got[off:off + g.numel()], g.reshape(-1))
            assert e <= 1.0, f"rank {r} layer {i}: all-reduced gradient differs from the full batch by {e:.3g}x"
            off += g.numel()
        assert torch.isfinite(got).all()


def _peer_worker(rank, world, port, outdir):
    import torch.distributed as dist

    from cabi_runner import backward, forward
    from paraconv2d_b200 import _lib
    from paraconv2d_b200.dp import PeerGradComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        lib = _lib.cabi()
        gen = torch.Generator().manual_seed(100 + rank)  # each rank its own shard
        n, C, H, W, m, k = 4, 16, 18, 18, 24, 3
        x = (torch.rand(n, C, H, W, generator=gen) * 2 - 1).to(dev)
        pars = (torch.randn(2 * m * (C * k * k + 1), generator=torch.Generator().manual_seed(7)) * 0.05).to(dev)
        out, hsum = forward(x, pars, 1.0, k)
        g = torch.randn(out.shape, generator=gen).to(dev)
        comm = PeerGradComm(pars.numel())
        wsb = lib.pc2d_backward_workspace_size(0, n, C, H, W, m, k, k, 1, 1, 1, 1, 0)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        results = []
        for _ in range(3):  # both exchange slots, then the first again
            ref_dx, ref = backward(g, x, pars, hsum, 1.0, k)
            dist.all_reduce(ref)
            dx = torch.empty_like(x)
            dp = torch.empty_like(pars)
            st = lib.pc2d_backward_sum(comm.comm, 0, g.data_ptr(), x.data_ptr(), pars.data_ptr(), hsum.data_ptr(),
                                       1.0, k, k, 1, 1, 1, 1, n, C, H, W, m, 0, dx.data_ptr(), dp.data_ptr(),
                                       ws.data_ptr(), wsb, stream)
            assert st == 0, _lib.status_message(st)
            torch.cuda.synchronize()
            results.append((torch.equal(dp, ref), torch.equal(dx, ref_dx)))
        assert lib.pc2d_device_status() == 0
        comm.close()
        torch.save({"results": results, "dp": dp.cpu()}, os.path.join(outdir, f"peer{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_sum_equals_nccl_allreduce(tmp_path):
    """pc2d_backward_sum on two GPUs: the parameter gradient summed over
    NVLink peer memory equals NCCL's all-reduce of the ranks' own gradients
    bit for bit (two addends: both round the exact sum once), on both ranks
    and over three calls (both exchange slots); the input gradient is the
    rank's own."""
    mp.start_processes(_peer_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = torch.load(os.path.join(tmp_path, "peer0.pt"))
    r1 = torch.load(os.path.join(tmp_path, "peer1.pt"))
    assert all(a and b for a, b in r0["results"] + r1["results"])
    assert torch.equal(r0["dp"], r1["dp"])


def _allreduce_worker(rank, world, port, outdir):
    import torch.distributed as dist

    from paraconv2d_b200.dp import PeerGradComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        comm = PeerGradComm(186_496)
        results = []
        for count in (1001, 186_496, 3):  # both exchange slots, a ragged tail, the full bucket
            gen = torch.Generator().manual_seed(1000 * count + rank)
            t = (torch.randn(count, generator=gen) * 1e-3).to(dev)
            ref = t.clone()
            dist.all_reduce(ref)
            comm.allreduce_(t)
            torch.cuda.synchronize()
            results.append(torch.equal(t, ref))
        from paraconv2d_b200 import _lib
        assert _lib.cabi().pc2d_device_status() == 0
        comm.close()
        torch.save({"results": results, "last": t.cpu()}, os.path.join(outdir, f"ar{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_equals_nccl(tmp_path):
    """pc2d_comm_allreduce on two GPUs: in place, counts that are and are not
    multiples of four, equal to NCCL's all-reduce bit for bit on both ranks."""
    mp.start_processes(_allreduce_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = torch.load(os.path.join(tmp_path, "ar0.pt"))
    r1 = torch.load(os.path.join(tmp_path, "ar1.pt"))
    assert all(r0["results"]) and all(r1["results"])
    assert torch.equal(r0["last"], r1["last"])
