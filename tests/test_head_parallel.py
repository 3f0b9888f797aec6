"""Head-parallel layer plumbing on world_size-2 gloo ranks (CPU): the
parameter split by heads, and the two collectives of the split -- the gather
of the head outputs (all_gather_into_tensor; adjoint: the rank's own block) and
the input gradient summed over the ranks -- against the unsplit computation.
The fused layer itself runs on the GPU (tests/test_gpu_head_parallel.py)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from cyclic_flow_attention import CyclicFlowAttention
    from cyclic_flow_attention.distributed import (HeadParallelAttention, _GatherHeads,
                                                   _ReplicatedInput)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # parameter split: rank r holds heads [2r, 2r+2) of the 4-head layer
        torch.manual_seed(0)
        full = CyclicFlowAttention(64, 4, 32)
        hp = HeadParallelAttention(full, None)
        fp = dict(full.named_parameters())
        split_ok = True
        for name, p in hp.local.named_parameters():
            rows = {"q_proj.weight": 32, "k_proj.weight": 32, "v_proj.weight": 32,
                    "q_conv1d.weight": 32, "k_conv1d.weight": 32, "v_conv1d.weight": 32,
                    "g_proj.1.weight": 32, "g_proj.1.bias": 32}.get(name, 1)
            if name in ("q_norm.weight", "k_norm.weight", "o_norm.weight", "g_proj.0.weight"):
                want = fp[name]
            else:
                want = fp[name][rank * 2 * rows:(rank + 1) * 2 * rows]
            split_ok &= torch.equal(p, want)
        split_ok &= torch.equal(hp.o_proj.weight, full.o_proj.weight)
        split_ok &= hp.local.o_proj is None and hp.heads_local == 2

        # collectives: y = gather_r(x W_r^T) U^T against x W^T U^T
        gen = torch.Generator().manual_seed(1)
        x = torch.randn(3, 5, 8, generator=gen)
        W = torch.randn(6, 8, generator=gen)   # 2 ranks x 3 output columns
        U = torch.randn(4, 6, generator=gen)
        dy = torch.randn(3, 5, 4, generator=gen)
        xl = x.clone().requires_grad_(True)
        Wl = W[3 * rank:3 * rank + 3].clone().requires_grad_(True)
        h = _ReplicatedInput.apply(xl, None) @ Wl.t()
        y = _GatherHeads.apply(h, None) @ U.t()
        (y * dy).sum().backward()
        xf = x.clone().requires_grad_(True)
        Wf = W.clone().requires_grad_(True)
        yf = xf @ Wf.t() @ U.t()
        (yf * dy).sum().backward()
        ok = (torch.allclose(y, yf, atol=1e-5) and torch.allclose(xl.grad, xf.grad, atol=1e-5)
              and torch.allclose(Wl.grad, Wf.grad[3 * rank:3 * rank + 3], atol=1e-5))
        q.put((rank, bool(split_ok), bool(ok)))
    finally:
        dist.destroy_process_group()


def test_head_split_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, split_ok, ok in res:
        assert split_ok, rank
        assert ok, rank
