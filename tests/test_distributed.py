"""Multi-process (world_size 2, gloo, CPU) tests of the data-parallel plumbing:
batch sharding, the flat-bucket gradient all-reduce and parameter broadcast
(the reference's distributed test checks the mean all-reduce of an fp32 gradient,
tests/test_distributed.py:8-21)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from cyclic_flow_attention.distributed import (
        allreduce_gradients,
        broadcast_parameters,
        shard_batch,
    )

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(rank)
        lin = torch.nn.Linear(4, 3)
        broadcast_parameters(lin.parameters())
        x = torch.arange(24, dtype=torch.float32).reshape(6, 4)
        xs = shard_batch(x, rank, world)
        loss = lin(xs).pow(2).sum()
        loss.backward()
        grads_local = [p.grad.clone() for p in lin.parameters()]
        allreduce_gradients(lin.parameters())
        # plain lists: tensors sent through the queue would be shared-memory
        # handles that die with this process
        out = {
            "w": lin.weight.detach().tolist(),
            "shard": xs.tolist(),
            "local": [g.tolist() for g in grads_local],
            "avg": [p.grad.tolist() for p in lin.parameters()],
        }
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_dp_step_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out = q.get(timeout=120)
        res[r] = {k: (torch.tensor(v) if k in ("w", "shard") else [torch.tensor(x) for x in v])
                  for k, v in out.items()}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # broadcast: identical parameters
    assert torch.equal(res[0]["w"], res[1]["w"])
    # shards: disjoint halves of the batch
    assert torch.equal(torch.cat([res[0]["shard"], res[1]["shard"]]),
                       torch.arange(24, dtype=torch.float32).reshape(6, 4))
    # all-reduce: mean of the local gradients, identical on both ranks
    for i in range(2):
        mean = (res[0]["local"][i] + res[1]["local"][i]) / 2
        assert torch.allclose(res[0]["avg"][i], mean)
        assert torch.equal(res[0]["avg"][i], res[1]["avg"][i])


def test_shard_batch_rejects_uneven():
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from cyclic_flow_attention.distributed import shard_batch

    with pytest.raises(ValueError):
        shard_batch(torch.zeros(5, 2), 0, 2)


def _bucket_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from cyclic_flow_attention.distributed import (
        GradientBuckets,
        allreduce_gradients,
        broadcast_parameters,
    )

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(rank)

        def make():
            torch.manual_seed(7)
            m = torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Tanh(),
                                    torch.nn.Linear(7, 3), torch.nn.Linear(3, 2))
            m.unused = torch.nn.Parameter(torch.ones(4))  # never receives a gradient
            return m

        ref, net = make(), make()
        broadcast_parameters(ref.parameters())
        broadcast_parameters(net.parameters())
        # tiny buckets: several collectives, launched while backward runs
        buckets = GradientBuckets(net.parameters(), bucket_bytes=64)
        xs = [torch.randn(6, 5) for _ in range(3)]
        out = {"n_buckets": len(buckets.buckets)}
        for step in range(2):  # the same buckets are reused every step
            for m in (ref, net):
                for p in m.parameters():
                    p.grad = None
            # micro-batch accumulation: the first two backward passes stay local
            with buckets.no_sync():
                for x in xs[:2]:
                    net(x * (step + 1)).pow(2).sum().backward()
            net(xs[2] * (step + 1)).pow(2).sum().backward()
            buckets.finish()
            for x in xs:
                ref(x * (step + 1)).pow(2).sum().backward()
            allreduce_gradients(ref.parameters())
            out[f"ref{step}"] = [(p.grad if p.grad is not None else torch.zeros_like(p)).tolist()
                                 for p in ref.parameters()]
            out[f"net{step}"] = [p.grad.tolist() for p in net.parameters()]
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_gradient_buckets_match_flat_allreduce():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out = q.get(timeout=120)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0]["n_buckets"] > 2
    for r in range(world):
        for step in range(2):
            for a, b in zip(res[r][f"ref{step}"], res[r][f"net{step}"]):
                assert torch.allclose(torch.tensor(a), torch.tensor(b), rtol=1e-6, atol=1e-6)
    for step in range(2):
        for a, b in zip(res[0][f"net{step}"], res[1][f"net{step}"]):
            assert torch.equal(torch.tensor(a), torch.tensor(b))


class _EarlyLinear(torch.autograd.Function):
    """y = x w^T + b whose backward hands (w, b)'s gradients over before dx."""

    leave = []  # what each hand-over returned (SMs to leave to the collective)

    @staticmethod
    def forward(ctx, x, w, b, ready):
        ctx.save_for_backward(x, w)
        ctx.ready, ctx.params = ready, (w, b)
        return x @ w.t() + b

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dw, db = dy.t() @ x, dy.sum(0)
        _EarlyLinear.leave.append(ctx.ready(ctx.params, (dw, db)))
        return dy @ w, dw, db, None


def _early_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cyfa-jittor_b200"))
    from cyclic_flow_attention.distributed import GradientBuckets, allreduce_gradients

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        def make():
            torch.manual_seed(3)
            return torch.nn.Linear(5, 6), torch.nn.Linear(6, 2)

        l1, l2 = make()
        r1, r2 = make()
        params = list(l1.parameters()) + list(l2.parameters())
        # explicit groups in backward order: l2 first, then l1 (handed over early)
        buckets = GradientBuckets(params, groups=[list(l2.parameters()), list(l1.parameters())],
                                  comm_sms=24)
        torch.manual_seed(10 + rank)
        x = torch.randn(4, 5)
        out = {"n": len(buckets.buckets)}
        for step in range(2):
            for p in params + list(r1.parameters()) + list(r2.parameters()):
                p.grad = None
            y = l2(_EarlyLinear.apply(x * (step + 1), l1.weight, l1.bias, buckets.early))
            y.pow(2).sum().backward()
            out[f"early_used{step}"] = buckets.next  # bucket 1 launched before finish()
            buckets.finish()
            r2(r1(x * (step + 1))).pow(2).sum().backward()
            allreduce_gradients(list(r1.parameters()) + list(r2.parameters()))
            out[f"net{step}"] = [p.grad.tolist() for p in params]
            out[f"ref{step}"] = [p.grad.tolist() for p in list(r1.parameters()) + list(r2.parameters())]
        out["leave"] = list(_EarlyLinear.leave)
        # a hand-over that cannot complete its bucket launches nothing: 0
        out["leave_incomplete"] = buckets.early([l2.weight], [torch.zeros_like(l2.weight)])
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_gradient_buckets_groups_and_early_handover():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_early_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out = q.get(timeout=120)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r]["n"] == 2
        # each early launch asks the next GEMM to leave comm_sms SMs to it
        assert res[r]["leave"] == [24, 24]
        assert res[r]["leave_incomplete"] == 0
        for step in range(2):
            assert res[r][f"early_used{step}"] == 2  # both buckets launched during backward
            for a, b in zip(res[r][f"net{step}"], res[r][f"ref{step}"]):
                assert torch.allclose(torch.tensor(a), torch.tensor(b), rtol=1e-6, atol=1e-6)
