"""AdamW with fp32 master weights and moments, for data-parallel training.

Counterpart of the reference's ``training.optim.AdamW`` (training/optim.py:8-124):
the same constructor, hyperparameter checks, ``backward(loss)`` /
``clip_grad_norm`` / ``step`` / ``zero_grad`` protocol and per-group lists
``master``, ``m``, ``v``, ``grads``, ``parameter_dtypes``.

Layout: every parameter's fp32 master copy, moments and gradient accumulator
are segments of four flat fp32 buffers (each segment starts at a multiple of 8
elements), so that

* ``backward`` gathers all gradients into one flat buffer (one libcyfa launch
  per 64 tensors on CUDA) and, across data-parallel ranks, averages it with ONE
  all-reduce, as the reference averages one concatenated fp32 bucket
  (training/optim.py:52-63);
* ``clip_grad_norm`` is one fixed-order norm over that buffer;
* ``step`` is one fused libcyfa launch per 64 parameters (``cyfa_adamw_step``)
  that updates master, m and v and writes each parameter rounded to its own
  dtype (bf16 weights, fp32 norms / readout / A_log / dt_bias).

The update arithmetic runs only in libcyfa.so: on CPU tensors ``step`` and
``clip_grad_norm`` raise.  Gradient gathering and the all-reduce are plain
tensor copies and collectives, so they also run on CPU (gloo) for tests.
"""

import ctypes

import torch
import torch.distributed as dist

from cyclic_flow_attention import _lib

_ALIGN = 8  # elements: 32-byte segment starts for the vectorised kernels


def _dtype_code(t):
    if t.dtype == torch.float32:
        return 0
    if t.dtype == torch.bfloat16:
        return 1
    raise TypeError(f"AdamW parameters must be float32 or bfloat16, got {t.dtype}")


class AdamW:
    """Keep moments and master weights in FP32; round model weights once per step.

    ``params`` is an iterable of tensors, of (name, tensor) pairs (e.g.
    ``model.named_parameters()``), or of param-group dicts with a "params" list
    and optional "lr", "betas", "eps", "weight_decay".  The names are what
    ``restore_training`` checks; plain tensors are named by their position.
    """

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01):
        if lr < 0 or eps <= 0 or weight_decay < 0 or not all(0 <= b < 1 for b in betas):
            raise ValueError("Invalid AdamW hyperparameters")
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.update_step = 0
        self.n_step = 0
        self._have_grad = False
        items = list(params)
        if items and isinstance(items[0], dict):
            groups = [dict(g) for g in items]
        else:
            groups = [{"params": items}]
        self.param_groups = []
        for gi, group in enumerate(groups):
            plist, names = [], []
            for i, p in enumerate(group["params"]):
                if isinstance(p, tuple):
                    names.append(p[0])
                    p = p[1]
                else:
                    names.append(f"{gi}.{i}")
                plist.append(p)
            group["params"] = plist
            group["names"] = names
            self.param_groups.append(group)
        self._layout()

    # ------------------------------------------------------------ flat buffers
    def _layout(self):
        params = [p for g in self.param_groups for p in g["params"]]
        if not params:
            raise ValueError("AdamW got an empty parameter list")
        dev = params[0].device
        if any(p.device != dev for p in params):
            raise ValueError("all AdamW parameters must live on one device")
        offsets, n = [], 0
        for p in params:
            _dtype_code(p)
            offsets.append(n)
            n += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN
        self._numel = n
        self.device = dev
        f32 = dict(device=dev, dtype=torch.float32)
        self._master = torch.zeros(n, **f32)
        self._m = torch.zeros(n, **f32)
        self._v = torch.zeros(n, **f32)
        self._grads = torch.zeros(n, **f32)
        self._incoming = torch.zeros(n, **f32)
        k = 0
        for group in self.param_groups:
            group["offsets"] = []
            for key in ("master", "m", "v", "grads"):
                group[key] = []
            for p in group["params"]:
                off = offsets[k]
                k += 1
                group["offsets"].append(off)
                for key, buf in (("master", self._master), ("m", self._m), ("v", self._v),
                                 ("grads", self._grads)):
                    group[key].append(buf[off:off + p.numel()].view(p.shape))
            group["parameter_dtypes"] = [str(p.dtype).replace("torch.", "")
                                         for p in group["params"]]
        with torch.no_grad():
            for group in self.param_groups:
                for p, w in zip(group["params"], group["master"]):
                    w.copy_(p.detach().float())

    def _trainable(self):
        for group in self.param_groups:
            for p, off in zip(group["params"], group["offsets"]):
                if p.requires_grad:
                    yield group, p, off

    # ------------------------------------------------------------ protocol
    def zero_grad(self):
        self._have_grad = False

    def backward(self, loss, retain_graph=False):
        """Gradients of `loss` into the fp32 accumulator, averaged over the
        data-parallel ranks with one flat all-reduce (training/optim.py:39-72)."""
        entries = list(self._trainable())
        if not entries:
            return
        params = [p for _, p, _ in entries]
        grads = torch.autograd.grad(loss, params, retain_graph=retain_graph, allow_unused=True)
        self._accumulate([(g, p, off) for g, (_, p, off) in zip(grads, entries)], reduce=True)

    def accumulate_param_grads(self):
        """Like ``backward`` for gradients already in ``p.grad`` (for example
        averaged during the backward by ``GradientBuckets``): gathers them into
        the fp32 accumulator without another all-reduce."""
        entries = list(self._trainable())
        self._accumulate([(p.grad, p, off) for _, p, off in entries], reduce=False)

    def _accumulate(self, triples, reduce):
        dst = self._incoming if self._have_grad else self._grads
        if any(g is None for g, _, _ in triples):
            dst.zero_()
        if self.device.type == "cuda":
            pieces = [(g, off) for g, _, off in triples if g is not None]
            self._gather(pieces, dst)
        else:
            for g, p, off in triples:
                if g is not None:
                    dst[off:off + p.numel()].copy_(g.reshape(-1))
        if reduce and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            if dist.get_backend() == "nccl":
                dist.all_reduce(dst, op=dist.ReduceOp.AVG)
            else:
                dist.all_reduce(dst, op=dist.ReduceOp.SUM)
                dst /= dist.get_world_size()
        if self._have_grad:
            self._grads.add_(self._incoming)
        self._have_grad = True
        self.n_step += 1

    def _gather(self, pieces, dst):
        arr = (_lib.BucketPiece * max(1, len(pieces)))()
        keep = []
        for i, (g, off) in enumerate(pieces):
            g = g.contiguous()
            if g.dtype not in (torch.float32, torch.bfloat16):
                g = g.float()
            if g.data_ptr() % 16:
                g = g.clone()  # the gather kernel reads 16-byte vectors
            keep.append(g)
            arr[i] = _lib.BucketPiece(g.data_ptr(), g.numel(), off, _dtype_code(g))
        _lib.call("cyfa_bucket_gather", arr, len(pieces), _lib.ptr(dst), _lib.stream())

    def clip_grad_norm(self, max_norm, norm_type=2):
        """Scales the accumulated gradients so that their global L2 norm is at
        most `max_norm` (training/optim.py:74-89).  Returns the norm before
        clipping as a 0-d device tensor (None when there are no gradients)."""
        if norm_type != 2 or max_norm <= 0:
            raise ValueError("Use a positive maximum L2 gradient norm")
        if not self._have_grad:
            return None
        _lib.require_cuda(self._grads)
        norm = torch.empty((), device=self.device, dtype=torch.float32)
        nwork = _lib.lib().cyfa_grad_clip_work_bytes()
        work = torch.empty(nwork, device=self.device, dtype=torch.uint8)
        _lib.call("cyfa_grad_clip", _lib.ptr(self._grads), self._numel, float(max_norm),
                  _lib.ptr(norm), _lib.ptr(work), ctypes.c_size_t(nwork), _lib.stream())
        return norm

    def step(self, loss=None, retain_graph=False):
        """One AdamW update of every trainable parameter from the accumulated
        gradients (``backward(loss)`` first when `loss` is given), then clears
        the accumulator, as the reference's pre_step / post_step do."""
        if loss is not None:
            self.backward(loss, retain_graph)
        _lib.require_cuda(self._master)
        self.update_step += 1
        for group in self.param_groups:
            lr = group.get("lr", self.lr)
            b0, b1 = group.get("betas", self.betas)
            eps = group.get("eps", self.eps)
            decay = group.get("weight_decay", self.weight_decay)
            live = [(p, off) for p, off in zip(group["params"], group["offsets"])
                    if p.requires_grad]
            if not live:
                continue
            arr = (_lib.BucketPiece * len(live))()
            for i, (p, off) in enumerate(live):
                if not p.is_contiguous():
                    raise ValueError("AdamW parameters must be contiguous")
                arr[i] = _lib.BucketPiece(p.data_ptr(), p.numel(), off, _dtype_code(p))
            _lib.call("cyfa_adamw_step", arr, len(live), _lib.ptr(self._master),
                      _lib.ptr(self._m), _lib.ptr(self._v), _lib.ptr(self._grads), float(lr),
                      float(b0), float(b1), float(eps), float(decay), self.update_step,
                      _lib.stream())
        self.zero_grad()
