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
from torch import nn

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

    def __init__(self, params, group=None, bucket_bytes=8 << 20, groups=None,
                 comm_sms=0):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        # SMs that a GEMM issued right after an early hand-over leaves to the
        # all-reduce it launched (`early` returns it; 0: the GEMM takes them all)
        self.comm_sms = comm_sms
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
        then do nothing, and the return value is `comm_sms` (the SMs the op's next
        GEMM should leave to the collective).  Otherwise nothing happens, the hooks
        work as usual and the return value is 0."""
        if self.world == 1 or not self.sync or not params:
            return 0
        first = self.slot.get(params[0])
        if first is None:
            return 0
        i = first[0]
        given = dict(zip(params, grads))
        if any(self.slot.get(p, (None,))[0] != i for p in params):
            return 0
        if any(p not in given and p not in self.filled[i] for p in self.buckets[i]):
            return 0
        self._launch_ready()
        if self.next != i:
            return 0
        self.filled[i] = set(self.buckets[i])
        self.pending[i] = 0
        self._launch(i, given)
        return self.comm_sms

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


# ---------------------------------------------------------------- head parallelism
class _ReplicatedInput(torch.autograd.Function):
    """Identity in the forward; in the backward the input gradient, a partial
    sum over this rank's heads, is summed over the head group."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, dx):
        dx = dx.contiguous()
        dist.all_reduce(dx, op=dist.ReduceOp.SUM, group=ctx.group)
        return dx, None


class _GatherHeads(torch.autograd.Function):
    """[..., H_l * V] per rank -> [..., world * H_l * V] on every rank, rank r's
    heads at block r (one all_gather_into_tensor).  The computation after it is
    replicated, so the adjoint is the rank's own block of the gradient."""

    @staticmethod
    def forward(ctx, o, group):
        world = dist.get_world_size(group)
        ctx.group, ctx.world, ctx.rank = group, world, dist.get_rank(group)
        lead, width = o.shape[:-1], o.shape[-1]
        flat = o.reshape(-1, width).contiguous()
        out = torch.empty(world * flat.shape[0], width, device=o.device, dtype=o.dtype)
        dist.all_gather_into_tensor(out, flat, group=group)
        return out.view(world, -1, width).permute(1, 0, 2).reshape(*lead, world * width)

    @staticmethod
    def backward(ctx, dy):
        width = dy.shape[-1] // ctx.world
        return dy[..., ctx.rank * width:(ctx.rank + 1) * width].contiguous(), None


# parameters of CyclicFlowAttention split by heads: name -> (rows per head of
# the head dimension: "k" = head_k_dim, "v" = head_v_dim, 1 = one per head)
_HEAD_ROWS = {
    "q_proj.weight": "k", "k_proj.weight": "k", "v_proj.weight": "v",
    "a_proj.weight": 1, "b_proj.weight": 1, "b_proj.bias": 1, "d_proj.weight": 1,
    "d_proj.bias": 1, "dt_bias": 1, "A_log": 1, "readout": 1,
    "q_conv1d.weight": "k", "k_conv1d.weight": "k", "v_conv1d.weight": "v",
    "q_conv1d.bias": "k", "k_conv1d.bias": "k", "v_conv1d.bias": "v",
    "g_proj.1.weight": "v", "g_proj.1.bias": "v",
}
# shared across heads: every rank holds all of it and contributes a partial gradient
_SHARED = ("q_norm.weight", "k_norm.weight", "o_norm.weight", "g_proj.0.weight")


def _head_rows(layer, name):
    unit = _HEAD_ROWS[name]
    return {"k": layer.head_k_dim, "v": layer.head_v_dim, 1: 1}[unit]


class HeadParallelAttention(nn.Module):
    """A CyclicFlowAttention layer split over the ranks of `group` by heads, for
    batches too small to split over the ranks (B < #GPUs).

    Every rank gets the whole input batch.  Rank r keeps heads [r*H_l, (r+1)*H_l)
    of every per-head parameter (the q/k/v/a/b/d projection rows, short
    convolutions, readout, A_log, dt_bias and the output gate's second linear)
    and a copy of the shared ones (q/k/o norm weights, the output gate's first
    linear, o_proj), and runs the fused layer on its heads up to the gated
    output norm.  The head outputs [B, T, H_l*V] are gathered with one
    all_gather_into_tensor into [B, T, H*V] and projected by o_proj on every
    rank, so the output is replicated.  Backward: each rank keeps its block of
    the gathered gradient, its head-sharded weight gradients are final, the
    input gradient is summed over the group (one all-reduce), and
    ``sync_grads()`` sums the shared parameters' partial gradients (one flat
    all-reduce).  The math is the unsplit layer's (layers/cyfa.py:299-357)."""

    def __init__(self, layer, group=None):
        super().__init__()
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        H = layer.num_heads
        if H % world:
            raise ValueError(f"{H} heads do not split over {world} ranks")
        self.group, self.world, self.rank = group, world, rank
        self.heads_local = H // world
        from .layers.cyfa import CyclicFlowAttention

        hidden = layer.q_proj.weight.shape[1]
        conv = layer.q_conv1d.width if layer.use_short_conv else 4
        bias = layer.use_short_conv and layer.q_conv1d.bias is not None
        local = CyclicFlowAttention(hidden, self.heads_local, layer.head_k_dim,
                                    expand_v=layer.head_v_dim / layer.head_k_dim,
                                    num_slots=layer.num_slots,
                                    use_short_conv=layer.use_short_conv, conv_size=conv,
                                    conv_bias=bias, norm_eps=layer.q_norm.eps,
                                    chunk_size=layer.chunk_size)
        full = dict(layer.named_parameters())
        with torch.no_grad():
            for name, p in local.named_parameters():
                src = full[name]
                if name in _HEAD_ROWS:
                    n = self.heads_local * _head_rows(layer, name)
                    src = src[rank * n:(rank + 1) * n]
                p.data = src.detach().clone()
        self.local = local
        self.o_proj = nn.Linear(layer.o_proj.weight.shape[1], hidden, bias=False,
                                device=layer.o_proj.weight.device,
                                dtype=layer.o_proj.weight.dtype)
        with torch.no_grad():
            self.o_proj.weight.copy_(layer.o_proj.weight)
        self.local.o_proj = None  # the projection happens after the gather

    def forward(self, x):
        x = _ReplicatedInput.apply(x, self.group)
        o, _ = self.local._forward_fused(x, False, project=False)
        o = _GatherHeads.apply(o, self.group)
        return torch.nn.functional.linear(o, self.o_proj.weight)

    def shared_parameters(self):
        named = dict(self.local.named_parameters())
        return [named[n] for n in _SHARED if n in named]

    def sync_grads(self):
        """Sums the shared parameters' partial gradients over the group."""
        ps = [p for p in self.shared_parameters() if p.grad is not None]
        if not ps:
            return
        flat = torch.cat([p.grad.float().reshape(-1) for p in ps])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        off = 0
        for p in ps:
            n = p.numel()
            p.grad.copy_(flat[off:off + n].view_as(p.grad))
            off += n

    def gather_grads(self):
        """{reference name: full gradient} on every rank: the head-sharded
        gradients gathered in head order, the others as held (for checking
        against the unsplit layer)."""
        out = {}
        for name, p in self.local.named_parameters():
            if p.grad is None:
                continue
            g = p.grad.contiguous()
            if name in _HEAD_ROWS:
                parts = torch.empty((self.world * g.shape[0],) + tuple(g.shape[1:]),
                                    device=g.device, dtype=g.dtype)
                dist.all_gather_into_tensor(parts, g, group=self.group)
                g = parts
            out[name] = g
        if self.o_proj.weight.grad is not None:
            out["o_proj.weight"] = self.o_proj.weight.grad
        return out
