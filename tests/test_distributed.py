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
