"""Data-parallel gradient of the c5 stack through the CUDA kernels: two ranks,
each with its shard of the batch, sum their parameter gradients with one
all-reduce; the result must equal the gradient of the whole batch computed
in one process (max|a-b| <= 1e-4 max|b| per layer: the two differ only in
the order of the fp32 sums).  Both all-reduce modes of GradAllReduce are
checked: one bucket after the backward, and one asynchronous all-reduce per
layer issued as soon as that layer's gradient is accumulated.

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


def _worker(rank, world, port, bucketed, outdir):
    import torch.distributed as dist

    from paraconv2d_b200 import workloads
    from paraconv2d_b200.dp import GradAllReduce, shard

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
        red = GradAllReduce(model.parameters(), bucketed=bucketed)
        x = shard(_batch(), rank, world).to(dev)
        workloads.stack_loss(model(x)).backward()
        red()
        torch.cuda.synchronize()
        torch.save(_grads(model), os.path.join(outdir, f"rank{rank}.pt"))
        red.remove()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("bucketed", [True, False], ids=["one_bucket", "per_layer_overlapped"])
def test_two_rank_gradient_equals_full_batch(bucketed, tmp_path):
    from paraconv2d_b200 import workloads
    from pc2d_testutil import maxrel_excess

    dev = torch.device("cuda", 0)
    model = _model(dev)
    workloads.stack_loss(model(_batch().to(dev))).backward()
    ref = [p.grad.detach().cpu().clone() for p in model.parameters()]
    mp.start_processes(_worker, args=(2, _free_port(), bucketed, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        got = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        off = 0
        for i, g in enumerate(ref):
            e = maxrel_excess(got[off:off + g.numel()], g.reshape(-1))
            assert e <= 1.0, f"rank {r} layer {i}: all-reduced gradient differs from the full batch by {e:.3g}x"
            off += g.numel()
        assert torch.isfinite(got).all()
