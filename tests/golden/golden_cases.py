"""Seeded inputs of the golden-vector cases (shared by make_golden.py, which
runs the reference's own kernels on them, and the tests that compare against
the committed outputs).  Deterministic: torch's CPU generator."""

import torch

# name, B, H, K, V, dtype, seed, T (decode steps), initial clock scale
CASES = [
    ("bf16_k128", 1, 2, 128, 128, torch.bfloat16, 101, 48, 3000.0),
    ("f32_k128", 1, 2, 128, 128, torch.float32, 102, 48, 150.0),
    ("bf16_k256", 1, 2, 256, 256, torch.bfloat16, 103, 32, 700.0),
]
EPS = 1e-6
SAMPLES = 512  # sampled entries of each final state


def case_inputs(case):
    """q, k, v [B,T,H,D] in the case dtype; g, delta, beta [B,T,H]; readout
    [H,127,127]; q/k norm weights [K]; initial state (hk0, hv0, clock0); all on
    the CPU."""
    name, B, H, K, V, dtype, seed, T, cscale = case
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen).to(dtype)
    k = torch.randn(B, T, H, K, generator=gen).to(dtype)
    v = torch.randn(B, T, H, V, generator=gen).to(dtype)
    g = torch.log(0.9 + 0.1 * torch.rand(B, T, H, generator=gen))
    delta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    readout = torch.eye(127).expand(H, -1, -1) + 0.05 * torch.randn(H, 127, 127, generator=gen)
    qw = 1 + 0.1 * torch.randn(K, generator=gen)
    kw = 1 + 0.1 * torch.randn(K, generator=gen)
    hk0 = 0.05 * torch.randn(B, H, K, 128, generator=gen)
    hv0 = 0.05 * torch.randn(B, H, 128, V, generator=gen)
    clock0 = cscale * torch.rand(B, H, generator=gen)
    return dict(q=q, k=k, v=v, g=g, delta=delta, beta=beta, readout=readout, qw=qw, kw=kw,
                hk0=hk0, hv0=hv0, clock0=clock0)


def sample_index(case, shape):
    """Fixed flat indices of the sampled final-state entries."""
    gen = torch.Generator().manual_seed(case[6] + 7)
    n = 1
    for s in shape:
        n *= s
    return torch.randint(0, n, (SAMPLES,), generator=gen)


def summarize_state(case, hk, hv):
    """Small fingerprint of the final states: row and column sums and sampled
    entries (float64)."""
    hk = hk.double().cpu()
    hv = hv.double().cpu()
    return {
        "hk_rows": hk.sum(-1), "hk_cols": hk.sum(-2),
        "hv_rows": hv.sum(-1), "hv_cols": hv.sum(-2),
        "hk_sample": hk.reshape(-1)[sample_index(case, hk.shape)],
        "hv_sample": hv.reshape(-1)[sample_index(case, hv.shape)],
    }
