"""The head-parallel layer on 2 GPUs (one process each, NCCL): output, input
gradient and every parameter gradient equal the unsplit layer's on the same
inputs (bf16 tolerance 1e-2).  Needs at least two CUDA devices."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "cyfa-jittor_b200"), os.path.join(root, "tests")]
    from gpu_util import rel_l2

    from cyclic_flow_attention import CyclicFlowAttention
    from cyclic_flow_attention.distributed import HeadParallelAttention

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        torch.manual_seed(0)
        full = CyclicFlowAttention(512, 4, 128)
        with torch.no_grad():
            for name, p in full.named_parameters():
                if p.dim() >= 2 and name != "readout":
                    p.normal_(0, 0.02)
        full = full.keep_fp32().to(dev)
        gen = torch.Generator().manual_seed(1)
        x = torch.randn(2, 300, 512, generator=gen).to(torch.bfloat16).to(dev)
        dy = torch.randn(2, 300, 512, generator=gen).to(torch.bfloat16).to(dev)
        hp = HeadParallelAttention(full, None)
        xh = x.clone().requires_grad_(True)
        y = hp(xh)
        y.backward(dy)
        hp.sync_grads()
        grads = hp.gather_grads()
        xf = x.clone().requires_grad_(True)
        yf, _ = full(xf)
        yf.backward(dy)
        errs = {"y": rel_l2(y, yf), "x": rel_l2(xh.grad, xf.grad)}
        errs.update({n: rel_l2(g, p.grad) for n, p in full.named_parameters()
                     for g in [grads.get(n)] if g is not None})
        missing = [n for n, _ in full.named_parameters() if n not in grads]
        q.put((rank, errs, missing, None))
        dist.barrier()
    except Exception as e:  # report instead of hanging the other rank's queue read
        q.put((rank, {}, [], repr(e)))
    finally:
        dist.destroy_process_group()


def test_head_parallel_matches_unsplit_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, missing, err in res:
        assert err is None, (rank, err)
        print("head-parallel rank", rank, {k: round(v, 5) for k, v in errs.items()})
        assert not missing, missing
        for n, e in errs.items():
            assert e < 1e-2, (rank, n, e)
