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

from . import _lib


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

    Parameters are grouped into fp32 buckets of about `bucket_bytes`: first in
    reverse registration order, then, from the second synced step on, in the
    order in which the first backward produced their gradients.  A post-accumulate-grad hook copies each gradient into its
    bucket slot as soon as autograd has it; a completed bucket is all-reduced
    asynchronously while the rest of the backward runs (on CUDA one library
    kernel gathers a bucket's bf16/f32 gradients into it and one scatters the
    averages back).  Buckets are launched
    strictly in index order, so every rank issues the same collectives in the
    same order even if its gradients arrive in another order.  `finish()`
    launches what is left (parameters without a gradient contribute zeros),
    waits, and writes the averages back into `.grad`.

    The reference averages one flat fp32 bucket after the backward
    (training/optim.py:52-63); the arithmetic is the same, the transfer overlaps.
    """

    def __init__(self, params, group=None, bucket_bytes=8 << 20, groups=None):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.bucket_bytes = bucket_bytes
        self.world = dist.get_world_size(group)
        self.avg_op = dist.get_backend(group) == "nccl"
        self._arrivals = []  # parameter indices in the order of the first backward
        self._param_index = {id(p): k for k, p in enumerate(self.params)}
        if groups is not None:
            # explicit buckets, in the order the backward fills them (a model
            # knows which gradients arrive together); leftovers go last
            self._rebuilt = True
            listed = {id(p) for g in groups for p in g}
            buckets = [[p for p in g if p.requires_grad] for g in groups]
            rest = [p for p in reversed(self.params) if id(p) not in listed]
            self._build_groups([b for b in buckets if b] + ([rest] if rest else []))
        else:
            self._rebuilt = False
            self._build(list(reversed(self.params)))
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]
        self.sync = True
        self._reset()

    def _build(self, order):
        buckets = []
        cur, size = [], 0
        for p in order:
            cur.append(p)
            size += p.numel() * 4
            if size >= self.bucket_bytes:
                buckets.append(cur)
                cur, size = [], 0
        if cur:
            buckets.append(cur)
        self._build_groups(buckets)

    def _build_groups(self, buckets):
        self.buckets = buckets
        self.flat = []
        self.slot = {}  # param -> (bucket, element offset, flat view)
        for i, bucket in enumerate(self.buckets):
            offs, off = [], 0
            for p in bucket:
                offs.append(off)
                off += (p.numel() + 63) // 64 * 64  # 256-byte aligned slots
            flat = torch.zeros(off, dtype=torch.float32, device=bucket[0].device)
            for p, o in zip(bucket, offs):
                self.slot[p] = (i, o, flat[o:o + p.numel()])
            self.flat.append(flat)

    def _rebuild_by_arrival(self):
        """After the first synced step: regroup the buckets in the order in which
        that backward produced the gradients (rank 0's order, broadcast, so all
        ranks agree), so that early buckets fill early.  Not during stream capture."""
        self._rebuilt = True
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            return
        seen = list(dict.fromkeys(self._arrivals))
        seen_set = set(seen)
        rest = [k for k in reversed(range(len(self.params))) if k not in seen_set]
        order = torch.tensor(seen + rest, dtype=torch.int64, device=self.flat[0].device)
        dist.broadcast(order, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                       group=self.group)
        self._build([self.params[k] for k in order.tolist()])

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
        i = self.slot[p][0]
        if p in self.filled[i]:
            return
        if not self._rebuilt:
            self._arrivals.append(self._param_index[id(p)])
        self.filled[i].add(p)
        self.pending[i] -= 1
        self._launch_ready()

    def early(self, params, grads):
        """Gradients handed over by the op that computes them, before autograd
        accumulates them (e.g. weight gradients formed ahead of the input
        gradient).  If they complete a bucket (its other parameters' gradients
        have already arrived) and every earlier bucket has been launched, the
        bucket is gathered (these from `grads`, the others from `.grad`) and
        all-reduced now, overlapping the rest of the op; the parameters' hooks
        then do nothing.  Otherwise nothing happens and the hooks work as usual."""
        if self.world == 1 or not self.sync or not params:
            return
        first = self.slot.get(params[0])
        if first is None:
            return
        i = first[0]
        given = dict(zip(params, grads))
        if any(self.slot.get(p, (None,))[0] != i for p in params):
            return
        if any(p not in given and p not in self.filled[i] for p in self.buckets[i]):
            return
        self._launch_ready()
        if self.next != i:
            return
        self.filled[i] = set(self.buckets[i])
        self.pending[i] = 0
        self._launch(i, given)

    def _pieces(self, i, given=None):
        """Bucket i's gradients as library pieces, or None if one of them does
        not fit the kernel (not CUDA, other dtype, non-contiguous, unaligned)."""
        pieces = []
        for p in self.buckets[i]:
            g = given.get(p, p.grad) if given is not None else p.grad
            if g is None:
                continue
            if (not g.is_cuda or g.dtype not in (torch.float32, torch.bfloat16)
                    or not g.is_contiguous() or g.data_ptr() % 16):
                return None
            pieces.append((g.data_ptr(), g.numel(), self.slot[p][1],
                           0 if g.dtype == torch.float32 else 1))
        arr = (_lib.BucketPiece * max(len(pieces), 1))()
        for k, pc in enumerate(pieces):
            arr[k] = _lib.BucketPiece(*pc)
        return arr, len(pieces)

    def _gather(self, i, given=None):
        """Copies bucket i's gradients (or the `given` ones) into its flat fp32
        buffer; slots of parameters without a gradient are zero."""
        flat = self.flat[i]
        grad = (lambda p: given.get(p, p.grad)) if given is not None else (lambda p: p.grad)
        for p in self.buckets[i]:
            if grad(p) is None:
                self.slot[p][2].zero_()
        packed = self._pieces(i, given) if flat.is_cuda else None
        if packed is not None:
            arr, n = packed
            _lib.call("cyfa_bucket_gather", arr, n, _lib.ptr(flat), _lib.stream())
            return
        for p in self.buckets[i]:
            if grad(p) is not None:
                self.slot[p][2].copy_(grad(p).reshape(-1))

    def _scatter(self, i, scale):
        """Writes scale * bucket i back into the gradients (allocating missing ones)."""
        flat = self.flat[i]
        for p in self.buckets[i]:
            if p.grad is None:
                p.grad = torch.empty_like(p)
        packed = self._pieces(i) if flat.is_cuda else None
        if packed is not None:
            arr, n = packed
            _lib.call("cyfa_bucket_scatter", arr, n, _lib.ptr(flat), float(scale), _lib.stream())
            return
        for p in self.buckets[i]:
            view = self.slot[p][2].view_as(p)
            p.grad.copy_(view * scale if scale != 1.0 else view)

    def _launch(self, i, given=None):
        self._gather(i, given)
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
            self._launch(i)
        scale = 1.0 if self.avg_op else 1.0 / self.world
        for i in range(len(self.buckets)):
            self.works[i].wait()
            self._scatter(i, scale)
        if not self._rebuilt:
            self._rebuild_by_arrival()
        self._reset()

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []


def broadcast_parameters(params, src=0, group=None):
    """Copies rank `src`'s parameters to every rank (reference train.py:86-90)."""
    for p in params:
        dist.broadcast(p.data, src=src, group=group)
