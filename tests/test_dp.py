"""Data-parallel logic on CPU: two gloo ranks, each with its shard of the
batch, must reproduce the full-batch gradient of a single process after the
SUM all-reduce (bucketed and per-parameter).  The model is the float64 torch
restatement of the op (test-only); the kernels themselves are checked on the
GPU elsewhere."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from paraconv2d_b200.dp import GradAllReduce, shard, shard_bounds


class RefLayer(torch.nn.Module):
    """Float64 restatement of ParaConv2d (conv decomposition, flipped window)."""

    def __init__(self, cin, cout, k, s, p, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        d = cin * k * k
        self.cin, self.cout, self.k, self.s, self.p = cin, cout, k, s, p
        self.pars = torch.nn.Parameter(torch.randn(2 * cout * (d + 1), generator=g, dtype=torch.float64) * 0.1)

    def forward(self, x):
        m, C, k = self.cout, self.cin, self.k
        d = C * k * k
        pr = self.pars
        h0, h, p, p0 = pr[:m], pr[m:m + m * d], pr[m + m * d:m + 2 * m * d], pr[m + 2 * m * d:]
        x = F.pad(x, (self.p,) * 4)
        H = h.reshape(m, C, k, k).flip(2, 3)
        Pw = p.reshape(m, C, k, k).flip(2, 3)
        hs = F.conv2d(x, H, stride=self.s) + h0.view(1, m, 1, 1)
        px = F.conv2d(x, Pw, stride=self.s)
        s2 = F.conv2d(x * x, torch.ones(1, C, k, k, dtype=x.dtype), stride=self.s)
        pp = (p.reshape(m, d) ** 2).sum(1).view(1, m, 1, 1)
        return hs * hs - (s2 - 2 * px + pp) - (p0 * p0).view(1, m, 1, 1)


def make_model():
    return torch.nn.Sequential(RefLayer(3, 8, 3, 1, 1, 1), RefLayer(8, 8, 3, 2, 1, 2))


def batch():
    g = torch.Generator().manual_seed(4)
    return torch.rand(6, 3, 8, 8, generator=g, dtype=torch.float64) * 2 - 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, bucketed, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = make_model()
        red = GradAllReduce(model.parameters(), bucketed=bucketed)
        x = shard(batch(), rank, world)
        (model(x) ** 2).sum().backward()
        red()
        out[rank] = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bucketed", [True, False])
def test_two_rank_sum_equals_full_batch(bucketed):
    model = make_model()
    (model(batch()) ** 2).sum().backward()
    ref = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    mgr = mp.Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), bucketed, out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert torch.allclose(out[r], ref, rtol=1e-12, atol=1e-12)


def test_shard_bounds_cover_the_batch():
    for n in (1, 7, 1024):
        for world in (1, 2, 3, 8):
            got = [shard_bounds(n, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1


def _worker_missing(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = make_model()
        red = GradAllReduce(model.parameters(), bucketed=True)
        if rank == 0:
            x = shard(batch(), rank, world)
            (model(x) ** 2).sum().backward()
        # rank 1 has no gradient at all this step: it still joins the same
        # collective (zeros) and receives rank 0's sum
        red()
        out[rank] = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    finally:
        dist.destroy_process_group()


def test_bucket_spans_parameters_without_gradient():
    model = make_model()
    (model(shard(batch(), 0, 2)) ** 2).sum().backward()
    ref = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    mgr = mp.Manager()
    out = mgr.dict()
    mp.start_processes(_worker_missing, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert torch.allclose(out[r], ref, rtol=1e-12, atol=1e-12)


def test_peer_sum_needs_the_bucketed_mode():
    """The NVLink peer sum works on the flat bucket only: asking for it with
    per-parameter all-reduces is refused before any hook is registered."""
    from paraconv2d_b200.dp import GradAllReduce

    p = torch.nn.Parameter(torch.zeros(4))
    with pytest.raises(ValueError):
        GradAllReduce([p], bucketed=False, peer=object())
