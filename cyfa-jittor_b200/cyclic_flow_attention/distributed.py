"""Data-parallel plumbing for multi-GPU CyFA training (one process per GPU).

The CyFA op shards over (batch x head) with no exchange inside it, so a step
on N GPUs is: each rank runs its own batch shard, and the weight gradients are
averaged across ranks (the reference averages one flat fp32 bucket with Jittor
MPI, training/optim.py:52-63).  `allreduce_gradients` is that single flat
bucket after the backward; `GradientBuckets` splits it into buckets that are
all-reduced while the backward is still running.  NCCL over NVLink on B200; the
same code runs on gloo for CPU tests.
"""

import contextlib

import torch
import torch.distributed as dist


def shard_batch(x, rank, world):
    """Rank's contiguous slice of the batch dimension (weak or strong scaling)."""
    B = x.shape[0]
    if B % world:
        raise ValueError(f"batch {B} does not divide over {world} ranks")
    n = B // world
    return x[rank * n:(rank + 1) * n]


def allreduce_gradients(params, group=None, op="avg"):
    """Averages (or sums) the .grad of `params` across ranks with ONE flat fp32
    bucket, in a fixed parameter order.  Parameters without a gradient
    contribute zeros, so every rank issues the same collective."""
    params = list(params)
    if not params:
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    dev = params[0].device
    sizes = [p.numel() for p in params]
    flat = torch.zeros(sum(sizes), dtype=torch.float32, device=dev)
    off = 0
    for p, n in zip(params, sizes):
        if p.grad is not None:
            flat[off:off + n].copy_(p.grad.reshape(-1))
        off += n
    if op == "avg" and dist.get_backend(group) == "nccl":
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        if op == "avg":
            flat /= world
    off = 0
    for p, n in zip(params, sizes):
        g = flat[off:off + n].view_as(p)
        if p.grad is None:
            p.grad = g.to(p.dtype).clone()
        else:
            p.grad.copy_(g)
        off += n


class GradientBuckets:
    """Bucketed gradient averaging overlapped with the backward pass.

    Parameters are grouped, in reverse registration order (the order in which
    backward produces their gradients), into fp32 buckets of about
    `bucket_bytes`.  A post-accumulate-grad hook copies each gradient into its
    bucket slot as soon as autograd has it; a completed bucket is all-reduced
    asynchronously while the rest of the backward runs.  Buckets are launched
    strictly in index order, so every rank issues the same collectives in the
    same order even if its gradients arrive in another order.  `finish()`
    launches what is left (parameters without a gradient contribute zeros),
    waits, and writes the averages back into `.grad`.

    The reference averages one flat fp32 bucket after the backward
    (training/optim.py:52-63); the arithmetic is the same, the transfer overlaps.
    """

    def __init__(self, params, group=None, bucket_bytes=8 << 20):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.world = dist.get_world_size(group)
        self.avg_op = dist.get_backend(group) == "nccl"
        order = list(reversed(self.params))
        self.buckets = []
        cur, size = [], 0
        for p in order:
            cur.append(p)
            size += p.numel() * 4
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.flat = []
        self.slot = {}
        for i, bucket in enumerate(self.buckets):
            n = sum(p.numel() for p in bucket)
            flat = torch.zeros(n, dtype=torch.float32, device=bucket[0].device)
            off = 0
            for p in bucket:
                self.slot[p] = (i, flat[off:off + p.numel()])
                off += p.numel()
            self.flat.append(flat)
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]
        self.sync = True
        self._reset()

    def _reset(self):
        self.pending = [len(b) for b in self.buckets]
        self.filled = [set() for _ in self.buckets]
        self.works = [None] * len(self.buckets)
        self.next = 0

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside accumulate locally only (gradient accumulation
        over micro-batches); the last backward, outside, averages the sums."""
        self.sync = False
        try:
            yield
        finally:
            self.sync = True

    def _on_grad(self, p):
        if self.world == 1 or not self.sync:
            return
        i, view = self.slot[p]
        if p in self.filled[i]:
            return
        view.copy_(p.grad.reshape(-1))
        self.filled[i].add(p)
        self.pending[i] -= 1
        self._launch_ready()

    def _launch(self, i):
        op = dist.ReduceOp.AVG if self.avg_op else dist.ReduceOp.SUM
        self.works[i] = dist.all_reduce(self.flat[i], op=op, group=self.group, async_op=True)
        self.next = i + 1

    def _launch_ready(self):
        while self.next < len(self.buckets) and self.pending[self.next] == 0:
            self._launch(self.next)

    def finish(self):
        """Completes the averaging of this step's gradients (call after backward)."""
        if self.world == 1:
            self._reset()
            return
        for i in range(self.next, len(self.buckets)):
            for p in self.buckets[i]:
                view = self.slot[p][1]
                if p in self.filled[i]:
                    continue
                if p.grad is None:
                    view.zero_()
                else:
                    view.copy_(p.grad.reshape(-1))
            self._launch(i)
        dsts, srcs = [], []
        for i, bucket in enumerate(self.buckets):
            self.works[i].wait()
            if not self.avg_op:
                self.flat[i].div_(self.world)
            for p in bucket:
                view = self.slot[p][1].view_as(p)
                if p.grad is None:
                    p.grad = view.to(p.dtype).clone()
                else:
                    dsts.append(p.grad)
                    srcs.append(view)
        if dsts:
            torch._foreach_copy_(dsts, srcs)
        self._reset()

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []


def broadcast_parameters(params, src=0, group=None):
    """Copies rank `src`'s parameters to every rank (reference train.py:86-90)."""
    for p in params:
        dist.broadcast(p.data, src=src, group=group)
