"""Host logic of the data-parallel training support (CPU, no GPU needed): the
fp32-master AdamW's flat layout, gradient accumulation and one-bucket
all-reduce over world_size-2 gloo ranks, and the resumable training
checkpoints (reference training/optim.py:8-124, training/checkpoint.py:13-63).
The update arithmetic itself is a libcyfa kernel, tested on the GPU."""

import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from training.checkpoint import restore_training, save_training
from training.optim import AdamW


def _params():
    torch.manual_seed(0)
    return [torch.randn(3, 5, requires_grad=True), torch.randn(7, requires_grad=True),
            torch.randn(2, 2).to(torch.bfloat16).requires_grad_(True)]


def test_hyperparameter_checks():
    for kw in (dict(lr=-1), dict(eps=0), dict(weight_decay=-0.1), dict(betas=(1.0, 0.9))):
        with pytest.raises(ValueError):
            AdamW(_params(), **kw)


def test_flat_layout_and_masters():
    ps = _params()
    opt = AdamW(ps)
    g = opt.param_groups[0]
    assert [m.shape for m in g["master"]] == [p.shape for p in ps]
    for p, w in zip(ps, g["master"]):
        assert w.dtype == torch.float32 and torch.equal(w, p.detach().float())
    assert all(off % 8 == 0 for off in g["offsets"])
    assert g["parameter_dtypes"] == ["float32", "float32", "bfloat16"]


def test_backward_accumulates_and_zero_grad_restarts():
    ps = _params()
    opt = AdamW(ps)
    x = torch.randn(5)

    def loss(scale):
        return scale * ((ps[0] @ x).sum() + ps[1].pow(2).sum() + ps[2].float().sum())

    opt.backward(loss(1.0))
    first = [g.clone() for g in opt.param_groups[0]["grads"]]
    opt.backward(loss(2.0))
    for a, b in zip(opt.param_groups[0]["grads"], first):
        assert torch.allclose(a, 3 * b)
    assert opt.n_step == 2
    opt.zero_grad()
    opt.backward(loss(1.0))
    for a, b in zip(opt.param_groups[0]["grads"], first):
        assert torch.allclose(a, b)


def test_update_needs_cuda():
    opt = AdamW(_params())
    opt.backward(sum(p.float().sum() for p in opt.param_groups[0]["params"]))
    with pytest.raises(RuntimeError):
        opt.step()
    with pytest.raises(RuntimeError):
        opt.clip_grad_norm(1.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, q):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from training.optim import AdamW as A

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        w = torch.randn(4, 3, requires_grad=True)
        b = torch.randn(3, requires_grad=True)
        opt = A([w, b])
        x = torch.arange(8, dtype=torch.float32).reshape(2, 4) + 10 * rank
        opt.backward(((x @ w) + b).pow(2).sum())
        q.put((rank, [g.tolist() for g in opt.param_groups[0]["grads"]], x.tolist()))
    finally:
        dist.destroy_process_group()


def test_backward_averages_over_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, grads, x = q.get(timeout=120)
        res[r] = ([torch.tensor(g) for g in grads], torch.tensor(x))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.manual_seed(0)
    w = torch.randn(4, 3, requires_grad=True)
    b = torch.randn(3, requires_grad=True)
    local = []
    for r in range(world):
        w.grad = b.grad = None
        ((res[r][1] @ w) + b).pow(2).sum().backward()
        local.append((w.grad.clone(), b.grad.clone()))
    want = [(local[0][i] + local[1][i]) / 2 for i in range(2)]
    for r in range(world):
        for got, exp in zip(res[r][0], want):
            assert torch.allclose(got, exp, rtol=1e-6, atol=1e-5)


def _tiny_model():
    from cyclic_flow_attention.models.cyfa import (CyclicFlowAttentionConfig,
                                                   CyclicFlowAttentionForCausalLM)

    cfg = CyclicFlowAttentionConfig(hidden_size=128, num_heads=1, head_dim=128, num_slots=128,
                                    num_hidden_layers=1, vocab_size=64)
    torch.manual_seed(1)
    return CyclicFlowAttentionForCausalLM(cfg).to_bfloat16()


def test_checkpoint_roundtrip_and_errors(tmp_path):
    model = _tiny_model()
    opt = AdamW(model.named_parameters())
    gen = torch.Generator().manual_seed(5)
    for kind in ("master", "m", "v"):
        for t in opt.param_groups[0][kind]:
            t.copy_(torch.randn(t.shape, generator=gen))
    opt.update_step = 7
    rng = np.random.default_rng(3)
    rng.random(4)
    args = {"gradient_accumulation_steps": 2, "lr": 1e-3}
    d = tmp_path / "ckpt"
    save_training(model, opt, None, d, step=5, rng=rng, arguments=args)
    assert (d / "config.json").exists() and (d / "model.safetensors").exists()
    assert (d / "training_state" / "optimizer.safetensors").exists()
    assert not (tmp_path / "ckpt.incomplete").exists()
    with pytest.raises(FileExistsError):
        save_training(model, opt, None, d, step=5, rng=rng, arguments=args)
    expect_next = np.random.default_rng(3)
    expect_next.random(4)

    fresh = AdamW(model.named_parameters())
    rng2 = np.random.default_rng(99)
    state = restore_training(fresh, d, rng2)
    assert state["step"] == 5 and fresh.update_step == 7 and fresh.n_step == 10
    for kind in ("master", "m", "v"):
        for a, b in zip(fresh.param_groups[0][kind], opt.param_groups[0][kind]):
            assert torch.equal(a, b)
    assert rng2.random() == expect_next.random()

    # names / order, shapes, world size, leftover tensors
    names = list(model.named_parameters())
    with pytest.raises(ValueError):
        restore_training(AdamW(names[::-1]), d, np.random.default_rng())
    meta = json.loads((d / "training.json").read_text())
    meta["world_size"] = 2
    (d / "training.json").write_text(json.dumps(meta))
    with pytest.raises(ValueError):
        restore_training(AdamW(model.named_parameters()), d, np.random.default_rng())
