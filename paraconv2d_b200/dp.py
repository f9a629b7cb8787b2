"""Data-parallel training of ParaConv2d layers: one process per GPU, the batch
split across ranks, the parameter gradients summed with one NCCL all-reduce.

The global loss of a ParaConv2d stack is a sum over images, so the gradient
of the full batch is the SUM of the ranks' gradients (not the mean that
DistributedDataParallel takes).  Every rank draws or receives the same
global batch and keeps its own contiguous shard, so the result does not
depend on the number of ranks.
"""
from __future__ import annotations

import contextlib
import ctypes
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def _range(name: str, t: torch.Tensor):
    """A named profiler range (NVTX) around host code that issues work for a
    CUDA tensor; nothing for CPU tensors."""
    return torch.cuda.nvtx.range(name) if t.is_cuda else contextlib.nullcontext()


def shard_bounds(n: int, rank: int, world: int):
    """[start, stop) of rank's contiguous shard of n items (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(batch: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's contiguous shard of the leading (batch) dimension."""
    a, b = shard_bounds(batch.shape[0], rank, world)
    return batch[a:b]


class GradAllReduce:
    """Sums the gradients of `params` across the ranks of `group`.

    ``bucketed=True`` (default) flattens all gradients into one buffer and
    issues a single all-reduce after the backward: for a 4-layer
    3->32->64->64->64 stack that is 186,496 floats.  The buffer always spans
    every parameter (a parameter without a gradient on this rank contributes
    zeros and receives the others' sum), so every rank issues a collective of
    the same length.  ``bucketed=False`` issues one asynchronous all-reduce
    per parameter as soon as its gradient is accumulated, overlapping the
    backward of the layers below it; ``wait()`` completes them.  In that mode
    every parameter must receive a gradient on every rank in every step (the
    ranks must issue the same collectives in the same order).

    ``peer`` (a ``PeerGradComm``, bucketed mode only) sums the bucket over
    NVLink peer memory on the current stream instead of through NCCL: one
    small kernel after the backward, where NCCL's all-reduce kernels would
    wait for SMs that the layer kernels (one CTA per SM) hold."""

    def __init__(self, params: Iterable[torch.nn.Parameter], group: Optional[dist.ProcessGroup] = None,
                 bucketed: bool = True, peer: Optional["PeerGradComm"] = None):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        self.group = group
        self.bucketed = bucketed
        if peer is not None and not bucketed:
            raise ValueError("GradAllReduce: the peer sum works on the bucket (bucketed=True)")
        self.peer = peer
        self._works = []
        self._hooks = []
        self._flat = None
        if not bucketed:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))

    def _on_grad(self, p):
        with _range("pc2d.allreduce.param", p.grad):
            self._works.append(dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def __call__(self):
        """Call after backward: completes the sum of every gradient."""
        if not self.bucketed:
            self.wait()
            return
        if not self.params:
            return
        ref = self.params[0]
        total = sum(p.numel() for p in self.params)
        if self._flat is None or self._flat.numel() != total or self._flat.device != ref.device:
            self._flat = torch.empty(total, dtype=ref.dtype, device=ref.device)
        off = 0
        for p in self.params:
            seg = self._flat[off:off + p.numel()]
            if p.grad is None:
                seg.zero_()
            else:
                seg.copy_(p.grad.reshape(-1))
            off += p.numel()
        if self.peer is not None:
            self.peer.allreduce_(self._flat)
        else:
            with _range("pc2d.allreduce.bucket", self._flat):
                dist.all_reduce(self._flat, op=dist.ReduceOp.SUM, group=self.group)
        off = 0
        for p in self.params:
            seg = self._flat[off:off + p.numel()].view_as(p)
            if p.grad is None:
                p.grad = seg.clone()
            else:
                p.grad.copy_(seg)
            off += p.numel()

    def wait(self):
        n = len(self._works)
        for w in self._works:
            w.wait()
        self._works.clear()
        if n != len(self.params):
            raise RuntimeError(f"GradAllReduce: {n} of {len(self.params)} parameters received a gradient this step; "
                               "per-parameter all-reduce needs every parameter's gradient on every rank")

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks.clear()


class PeerGradComm:
    """The communicator of ``pc2d_backward_sum`` (include/paraconv2d.h) for
    this rank: each rank's exchange buffer mapped by every other rank over
    CUDA IPC, so that the backward pass itself sums the parameter gradient
    over the ranks (NVLink peer loads, fixed rank order), with no all-reduce
    after it.  One process per GPU, at most 8 GPUs of one node.

    Creating it is collective over ``group`` (the IPC handles are exchanged
    with ``all_gather_object``); so is ``close``, which waits for every rank
    before unmapping.  ``max_params`` bounds the parameter count of the
    layers it serves."""

    def __init__(self, max_params: int, group: Optional[dist.ProcessGroup] = None):
        from ._lib import cabi, status_message

        self._lib = cabi()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        nb = self._lib.pc2d_comm_handle_bytes()
        handle = (ctypes.c_char * nb)()
        comm = ctypes.c_void_p()
        st = self._lib.pc2d_comm_create(self.rank, self.world, int(max_params), ctypes.byref(comm), handle)
        if st != 0:
            raise RuntimeError(status_message(st))
        self.comm = comm
        gathered = [None] * self.world
        dist.all_gather_object(gathered, bytes(handle), group=group)
        blob = b"".join(gathered)
        st = self._lib.pc2d_comm_connect(self.comm, blob)
        if st != 0:
            raise RuntimeError(status_message(st))

    def allreduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In place: t = the sum over the ranks of every rank's t (fp32,
        contiguous, on this rank's GPU, at most ``max_params`` values), on the
        current stream, the same bits on every rank.  Collective: every rank
        calls it in the same order."""
        from ._lib import status_message

        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("PeerGradComm.allreduce_: a contiguous float32 CUDA tensor")
        st = self._lib.pc2d_comm_allreduce(self.comm, t.data_ptr(), t.data_ptr(), t.numel(),
                                           torch.cuda.current_stream(t.device).cuda_stream)
        if st != 0:
            raise RuntimeError(status_message(st))
        return t

    def close(self):
        if self.comm is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self._lib.pc2d_comm_destroy(self.comm)
            self.comm = None
