"""Helpers shared by the GPU parity tests."""

import torch


def rel_l2(a, b):
    """Relative L2 error ||a - b|| / ||b|| in float64."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def bf16_cpu(x):
    """Rounds to bf16 and returns fp32 on the CPU (the values the GPU sees)."""
    return x.to(torch.bfloat16).float()


def seeded(seed):
    return torch.Generator().manual_seed(seed)
