"""GPU checks of the fused AdamW update (cyfa_adamw_step) and the gradient
clipping (cyfa_grad_clip) against a plain fp32 PyTorch restatement of the
reference's formulas (training/optim.py:74-124), over several steps, two
parameter groups, bf16 and fp32 parameters and gradient accumulation."""

import pytest
import torch

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def AdamW():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from training.optim import AdamW as A

    return A


def _reference_step(state, grads, lr, betas, eps, decay, step):
    b0, b1 = betas
    bc1, bc2 = 1 - b0 ** step, 1 - b1 ** step
    for s, g in zip(state, grads):
        s["m"] = b0 * s["m"] + (1 - b0) * g
        s["v"] = b1 * s["v"] + (1 - b1) * g * g
        s["w"] = s["w"] * (1 - lr * decay) - (lr / bc1) * s["m"] / (torch.sqrt(s["v"] / bc2) + eps)


@pytest.mark.parametrize("clip", [None, 0.05])
def test_adamw_matches_reference_formula(AdamW, clip):
    torch.manual_seed(0)
    shapes = [(300, 129), (1027,), (64, 8), (5,)]
    dtypes = [torch.bfloat16, torch.float32, torch.bfloat16, torch.float32]
    ps = [torch.randn(s, device="cuda").to(dt).requires_grad_(True) for s, dt in zip(shapes, dtypes)]
    groups = [{"params": ps[:2]}, {"params": ps[2:], "lr": 3e-3, "weight_decay": 0.0}]
    opt = AdamW(groups, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    hp = [(1e-2, 0.1), (3e-3, 0.0)]
    state = [{"w": p.detach().float().clone(), "m": torch.zeros_like(p, dtype=torch.float32),
              "v": torch.zeros_like(p, dtype=torch.float32)} for p in ps]
    xs = [torch.randn(s, device="cuda") for s in shapes]
    for step in range(1, 4):
        # two micro-batches accumulated, as gradient accumulation does
        total = [torch.zeros_like(s["w"]) for s in state]
        for micro in range(2):
            loss = sum(((p.float() - (micro + 1) * x) ** 2).sum() for p, x in zip(ps, xs))
            gs = torch.autograd.grad(loss, ps, retain_graph=True)
            total = [t + g.float() for t, g in zip(total, gs)]
            opt.backward(loss)
        if clip is not None:
            norm = opt.clip_grad_norm(clip)
            want = torch.sqrt(sum((t.double() ** 2).sum() for t in total))
            assert abs(norm.item() - want.item()) <= 1e-4 * want.item()
            coef = min(clip / (want.item() + 1e-6), 1.0)
            total = [t * coef for t in total]
        for gi, (lr, decay) in enumerate(hp):
            idx = [0, 1] if gi == 0 else [2, 3]
            _reference_step([state[i] for i in idx], [total[i] for i in idx], lr, (0.9, 0.95),
                            1e-8, decay, step)
        opt.step()
        torch.cuda.synchronize()
        masters = [w for g in opt.param_groups for w in g["master"]]
        for i, (p, s) in enumerate(zip(ps, state)):
            assert rel_l2(masters[i], s["w"]) < 1e-5, (step, i)
            # the parameter holds the master rounded once to its dtype
            assert torch.equal(p.detach(), masters[i].to(p.dtype)), (step, i)
    assert opt.update_step == 3


def test_adamw_trains_a_layer(AdamW):
    """A CyFA layer on the fused path, three AdamW steps on a fixed batch: the
    loss decreases and every parameter stays finite."""
    from cyclic_flow_attention import CyclicFlowAttention

    torch.manual_seed(0)
    m = CyclicFlowAttention(256, 2, 128).keep_fp32().cuda()
    opt = AdamW(m.named_parameters(), lr=1e-3)
    x = torch.randn(2, 128, 256, device="cuda").to(torch.bfloat16)
    target = torch.randn(2, 128, 256, device="cuda")
    losses = []
    for _ in range(4):
        y, _ = m(x)
        loss = (y.float() - target).pow(2).mean()
        losses.append(loss.item())
        opt.step(loss)
    assert losses[-1] < losses[0]
    assert all(torch.isfinite(p).all() for p in m.parameters())
