"""Data-parallel plumbing for multi-GPU CyFA training (one process per GPU).

The CyFA op shards over (batch x head) with no exchange inside it, so a step
on N GPUs is: each rank runs its own batch shard, then the weight gradients are
averaged with one flat all-reduce (the reference averages one flat fp32 bucket
with Jittor MPI, training/optim.py:52-63).  NCCL over NVLink on B200; the same
code runs on gloo for CPU tests.
"""

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


def broadcast_parameters(params, src=0, group=None):
    """Copies rank `src`'s parameters to every rank (reference train.py:86-90)."""
    for p in params:
        dist.broadcast(p.data, src=src, group=group)
