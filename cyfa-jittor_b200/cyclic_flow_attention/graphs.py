"""CUDA-graph capture of a whole training (or inference) step.

A CyFA layer step is ~100 kernel launches (the core's own plus cuBLAS and the
torch glue); launched one by one from Python the host needs about as long to
issue them as the GPU needs to run them.  `GraphedStep` records the step once
into a CUDA graph and replays it, so a step costs one graph launch on the host.

The step function is captured with its inputs at fixed device addresses
(`static_inputs`); calling the step copies new inputs into them first.
Parameter gradients are produced inside the graph: they are set to None before
capture, allocated from the graph's memory pool during it, and every replay
overwrites them (no accumulation across replays).  Gradient-averaging hooks
(`distributed.GradientBuckets`) that run during the capture are recorded with
their collectives, so a data-parallel step replays its all-reduces too.

The reference has no equivalent (Jittor traces and fuses through its own
compiler); this is the B200 build's replacement for that tracing path.
"""

import torch

from . import _lib


def _detach(t):
    return t.detach() if isinstance(t, torch.Tensor) else t


class GraphedStep:
    """fn(*static_inputs) -> output tensor(s), captured after `warmup` eager runs
    on a side stream.  `params` are the tensors whose .grad the step produces."""

    def __init__(self, fn, static_inputs, params=(), warmup=3, pool=None):
        if not torch.cuda.is_available():
            raise RuntimeError("GraphedStep needs a CUDA device")
        self.fn = fn
        self.static_inputs = list(static_inputs)
        self.params = list(params)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._clear_grads()
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self._clear_grads()
        self.graph = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count()
        with torch.cuda.graph(self.graph, pool=pool):
            out = fn(*self.static_inputs)
        # detached views: holding the captured autograd graph would keep its
        # AccumulateGrad nodes (bound to the capture stream) alive for later eager steps
        self.static_output = (tuple(_detach(o) for o in out) if isinstance(out, (tuple, list))
                              else _detach(out))
        del out
        # kernels of this library that one replay launches
        self.library_launches = _lib.launch_count() - n0
        self.static_grads = [p.grad for p in self.params]

    def pool(self):
        """Memory pool of this graph, to share with another graph of the same step."""
        return self.graph.pool()

    def _clear_grads(self):
        for p in self.params:
            p.grad = None

    def replay(self):
        self.graph.replay()
        for p, g in zip(self.params, self.static_grads):
            if p.grad is not g:
                p.grad = g
        return self.static_output

    def __call__(self, *inputs):
        if len(inputs) != len(self.static_inputs):
            raise ValueError(f"expected {len(self.static_inputs)} inputs, got {len(inputs)}")
        with torch.no_grad():  # static inputs may be leaves that require grad
            for dst, src in zip(self.static_inputs, inputs):
                if src is not dst:
                    dst.copy_(src, non_blocking=True)
        return self.replay()
