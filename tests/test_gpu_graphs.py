"""GPU checks of the CUDA-graph step: a captured layer training step replays
to the same output and gradients as the eager step, on inputs that change
between replays, and it replays this library's kernels (not a fallback)."""

import pytest
import torch

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu


def _setup(B, T, hidden, H, hd):
    from cyclic_flow_attention import CyclicFlowAttention

    torch.manual_seed(3)
    m = CyclicFlowAttention(hidden, H, hd)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if p.dim() >= 2 and name != "readout":
                p.normal_(0, 0.02)
    m = m.keep_fp32().cuda()
    params = list(m.parameters())

    def step(x, dy):
        for p in params:
            p.grad = None
        y, _ = m(x)
        loss = torch.dot(y.reshape(-1).float(), dy.reshape(-1).float())
        loss.backward()
        return loss

    return m, params, step


@pytest.mark.parametrize("B,T,hidden,H,hd", [(2, 384, 512, 2, 256), (1, 200, 256, 2, 128)])
def test_graphed_step_matches_eager(B, T, hidden, H, hd):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention.graphs import GraphedStep

    m, params, step = _setup(B, T, hidden, H, hd)
    gen = torch.Generator().manual_seed(5)
    inputs = [(torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda(),
               torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda())
              for _ in range(3)]
    static = [torch.empty_like(inputs[0][0]), torch.empty_like(inputs[0][1])]
    static[0].copy_(inputs[0][0])
    static[1].copy_(inputs[0][1])
    graphed = GraphedStep(step, static, params, warmup=2)
    assert graphed.library_launches > 10  # the core's kernels are in the graph
    for x, dy in inputs[1:] + inputs[:1]:
        loss_g = graphed(x, dy).clone()
        grads_g = [p.grad.clone() for p in params]
        loss_e = step(x, dy)
        torch.cuda.synchronize()
        assert rel_l2(loss_g, loss_e) <= 1e-5
        for (name, p), g in zip(m.named_parameters(), grads_g):
            err = rel_l2(g, p.grad)
            assert err <= 1e-5, (name, err)
    del graphed


def test_pdl_launch_matches_stream_order():
    """Programmatic dependent launch (kernels may start while their predecessor
    drains) gives bitwise the same step as plain stream order, eager and graphed."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib
    from cyclic_flow_attention.graphs import GraphedStep

    B, T, hidden, H, hd = 2, 384, 512, 2, 256
    m, params, step = _setup(B, T, hidden, H, hd)
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda()
    dy = torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda()
    results = {}
    prev = _lib.set_pdl(True)
    try:
        for on in (False, True):
            _lib.set_pdl(on)
            # detached: a live autograd graph would keep the eager AccumulateGrad
            # nodes (bound to this stream) for the capture below
            loss = step(x, dy).detach().clone()
            grads = [p.grad.clone() for p in params]
            static = [x.clone(), dy.clone()]
            graphed = GraphedStep(step, static, params, warmup=2)
            loss_g = graphed(x, dy).clone()
            grads_g = [p.grad.clone() for p in params]
            del graphed
            torch.cuda.synchronize()
            results[on] = (loss, grads, loss_g, grads_g)
    finally:
        _lib.set_pdl(prev)
    off, on_ = results[False], results[True]
    assert torch.equal(off[0], on_[0]) and torch.equal(off[2], on_[2])
    for a, b, c, d in zip(off[1], on_[1], off[3], on_[3]):
        assert torch.equal(a, b) and torch.equal(c, d)


def test_deferred_weight_gradients_match_inline():
    """The o_proj and output-gate weight gradients computed on the layer's side
    stream (deferred, joined in the front's backward) equal the inline ones: a
    hook on a parameter turns its deferral off."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    B, T, hidden, H, hd = 2, 384, 512, 2, 256
    m, params, step = _setup(B, T, hidden, H, hd)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda()
    dy = torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16).cuda()
    step(x, dy)
    torch.cuda.synchronize()
    deferred = [p.grad.clone() for p in params]
    handles = [p.register_post_accumulate_grad_hook(lambda p: None)
               for p in (m.o_proj.weight, m.g_proj[1].weight)]
    try:
        step(x, dy)
        torch.cuda.synchronize()
    finally:
        for h in handles:
            h.remove()
    for (name, p), g in zip(m.named_parameters(), deferred):
        assert torch.equal(p.grad, g), name
