"""Known-answer tests that pin the CPU oracle (no GPU needed).

The reference ships no golden vectors and cannot run here (Jittor + CUDA only),
so the oracle is pinned against the paper's own relative-time definition
(README.md:32-106 of the reference) and against algebraic identities.
"""

import math

import pytest
import torch

from oracle import cyfa_oracle as O


def _rand_inputs(B, T, H, K, V, seed=0, dtype=torch.float64):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen, dtype=dtype)
    k = torch.randn(B, T, H, K, generator=gen, dtype=dtype)
    v = torch.randn(B, T, H, V, generator=gen, dtype=dtype)
    g = torch.log(torch.rand(B, T, H, generator=gen, dtype=dtype) * 0.1 + 0.9)
    delta = torch.sigmoid(torch.randn(B, T, H, generator=gen, dtype=dtype))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen, dtype=dtype))
    return q, k, v, g, delta, beta


def test_basis_is_orthonormal():
    phi = O.basis(128)
    assert phi.shape == (127, 128)
    assert torch.allclose(phi @ phi.T, torch.eye(127, dtype=torch.float64), atol=1e-12)
    assert torch.all(phi[:, 1] == 0)


def test_chunk_equals_token_recurrence():
    gen = torch.Generator().manual_seed(1)
    B, H, T, K, V = 2, 3, 48, 8, 5
    q = torch.randn(B, H, T, K, generator=gen, dtype=torch.float64)
    k = torch.randn(B, H, T, K, generator=gen, dtype=torch.float64)
    v = torch.randn(B, H, T, V, generator=gen, dtype=torch.float64)
    g = -torch.rand(B, H, T, generator=gen, dtype=torch.float64)
    h0 = torch.randn(B, H, K, V, generator=gen, dtype=torch.float64)
    for C in (4, 16, 48):
        oc, fc = O.scalar_la_chunk(q, k, v, g, h0, C, 0.7)
        orr, fr = O.scalar_la_recurrent(q, k, v, g, h0, 0.7)
        assert torch.allclose(oc, orr, atol=1e-10, rtol=1e-10)
        assert torch.allclose(fc, fr, atol=1e-10, rtol=1e-10)


def test_two_pass_equals_relative_time_recurrence():
    """KAT (i): the absolute-clock two-pass form equals K_t = a P(d) K + b e0 k^T."""
    B, T, H, K, V, M = 1, 37, 2, 8, 6, 128
    q, k, v, g, delta, beta = _rand_inputs(B, T, H, K, V, seed=2)
    gen = torch.Generator().manual_seed(3)
    readout = torch.eye(M - 1, dtype=torch.float64).expand(H, -1, -1) + 0.05 * torch.randn(
        H, M - 1, M - 1, generator=gen, dtype=torch.float64)
    qw = torch.ones(K, dtype=torch.float64)
    kw = torch.ones(K, dtype=torch.float64)
    out, _ = O.chunk_cyfa(q, k, v, g, delta, beta, readout, qw, kw, chunk_size=8)
    qn = O.head_rmsnorm(q, qw, 1e-6)
    kn = O.head_rmsnorm(k, kw, 1e-6)
    ref = O.relative_time_reference(qn, kn, v.permute(0, 2, 1, 3), g.permute(0, 2, 1),
                                    delta.permute(0, 2, 1), beta.permute(0, 2, 1),
                                    readout, K ** -0.5, M)
    assert torch.allclose(out.permute(0, 2, 1, 3), ref, atol=1e-9, rtol=1e-8)


def test_clock_wrap_invariance():
    """KAT (iv): lam -> lam + 127 leaves the write vector unchanged (integer wrap)."""
    gen = torch.Generator().manual_seed(4)
    lam = torch.rand(1000, generator=gen, dtype=torch.float64) * 300
    beta = torch.rand(1000, generator=gen, dtype=torch.float64)
    w0, _, _ = O.write_vector(lam, beta, 128)
    w1, _, _ = O.write_vector(lam + 127, beta, 128)
    assert torch.allclose(w0, w1, atol=1e-9)
    # and the phase is the exact angle 2*pi*p*lam/127 (mod 2*pi)
    c, s = O.phase_cos_sin(lam, 128)
    ang = 2 * math.pi * torch.arange(64, dtype=torch.float64) * lam[:, None] / 127
    assert torch.allclose(c, torch.cos(ang), atol=1e-9)
    assert torch.allclose(s, torch.sin(ang), atol=1e-9)


def test_decode_matches_chunk_every_step():
    """Decode after a prefill equals the chunked forward at every step."""
    B, T, H, K, V, M = 2, 12, 2, 16, 8, 128
    q, k, v, g, delta, beta = _rand_inputs(B, T, H, K, V, seed=5)
    readout = torch.eye(M - 1, dtype=torch.float64).expand(H, -1, -1).clone()
    qw = torch.ones(K, dtype=torch.float64) * 1.1
    kw = torch.ones(K, dtype=torch.float64) * 0.9
    full, _ = O.chunk_cyfa(q, k, v, g, delta, beta, readout, qw, kw, chunk_size=4)
    P = 5
    _, state = O.chunk_cyfa(q[:, :P], k[:, :P], v[:, :P], g[:, :P], delta[:, :P], beta[:, :P],
                            readout, qw, kw, chunk_size=4, output_final_state=True)
    for t in range(P, T):
        sl = slice(t, t + 1)
        o, state = O.fused_recurrent_cyfa(q[:, sl], k[:, sl], v[:, sl], g[:, sl], delta[:, sl],
                                          beta[:, sl], readout, qw, kw, initial_state=state,
                                          output_final_state=True, dtype=torch.float64)
        assert torch.allclose(o[:, 0], full[:, t], atol=1e-9, rtol=1e-8)


def test_initial_state_continuation():
    """Two chunk calls chained through the returned state equal one call."""
    B, T, H, K, V, M = 1, 40, 2, 8, 8, 128
    q, k, v, g, delta, beta = _rand_inputs(B, T, H, K, V, seed=6)
    readout = torch.eye(M - 1, dtype=torch.float64).expand(H, -1, -1).clone()
    w = torch.ones(K, dtype=torch.float64)
    full, fs = O.chunk_cyfa(q, k, v, g, delta, beta, readout, w, w, chunk_size=8,
                            output_final_state=True)
    a, st = O.chunk_cyfa(q[:, :17], k[:, :17], v[:, :17], g[:, :17], delta[:, :17],
                         beta[:, :17], readout, w, w, chunk_size=8, output_final_state=True)
    b, st2 = O.chunk_cyfa(q[:, 17:], k[:, 17:], v[:, 17:], g[:, 17:], delta[:, 17:],
                          beta[:, 17:], readout, w, w, chunk_size=8, initial_state=st,
                          output_final_state=True)
    assert torch.allclose(torch.cat([a, b], 1), full, atol=1e-9)
    for x, y in zip(st2, fs):
        assert torch.allclose(x, y, atol=1e-9)


def test_chunk_size_independence():
    """The chunk size is an implementation detail: C=64 and C=128 agree."""
    B, T, H, K, V, M = 1, 256, 1, 16, 16, 128
    q, k, v, g, delta, beta = _rand_inputs(B, T, H, K, V, seed=7)
    readout = torch.eye(M - 1, dtype=torch.float64).expand(H, -1, -1).clone()
    w = torch.ones(K, dtype=torch.float64)
    a, sa = O.chunk_cyfa(q, k, v, g, delta, beta, readout, w, w, chunk_size=64,
                         output_final_state=True)
    b, sb = O.chunk_cyfa(q, k, v, g, delta, beta, readout, w, w, chunk_size=128,
                         output_final_state=True)
    assert torch.allclose(a, b, atol=1e-9)
    for x, y in zip(sa, sb):
        assert torch.allclose(x, y, atol=1e-9)


@pytest.mark.parametrize("T", [1, 63, 65])
def test_ragged_lengths_pad_neutrally(T):
    """T not a multiple of the chunk: zero padding changes nothing (chunk.py:198-207)."""
    B, H, K, V, M = 1, 2, 8, 8, 128
    q, k, v, g, delta, beta = _rand_inputs(B, T, H, K, V, seed=8)
    readout = torch.eye(M - 1, dtype=torch.float64).expand(H, -1, -1).clone()
    w = torch.ones(K, dtype=torch.float64)
    o, st = O.chunk_cyfa(q, k, v, g, delta, beta, readout, w, w, chunk_size=64,
                         output_final_state=True)
    qn = O.head_rmsnorm(q, w, 1e-6)
    kn = O.head_rmsnorm(k, w, 1e-6)
    ref = O.relative_time_reference(qn, kn, v.permute(0, 2, 1, 3), g.permute(0, 2, 1),
                                    delta.permute(0, 2, 1), beta.permute(0, 2, 1),
                                    readout, K ** -0.5, M)
    assert torch.allclose(o.permute(0, 2, 1, 3), ref, atol=1e-9)
    assert torch.allclose(st[2], delta.permute(0, 2, 1).sum(-1))


def test_oracle_gate_param_conditioning():
    """The gate/clock parameter gradients of the layer are ill-conditioned: a single
    bf16-sized relative perturbation (2^-9) of the layer inputs and parameters moves
    them by percent-level amounts, while well-conditioned weights move by < 1.5 %.
    This fixes the looser tolerances used for them in the GPU layer test."""
    gen = torch.Generator().manual_seed(3)
    B, T, hid, H, hd = 1, 128, 128, 2, 128
    shapes = {"q_proj.weight": (H * hd, hid), "k_proj.weight": (H * hd, hid),
              "v_proj.weight": (H * hd, hid), "a_proj.weight": (H, hid), "b_proj.weight": (H, hid),
              "b_proj.bias": (H,), "d_proj.weight": (H, hid), "d_proj.bias": (H,),
              "q_conv1d.weight": (H * hd, 1, 4), "k_conv1d.weight": (H * hd, 1, 4),
              "v_conv1d.weight": (H * hd, 1, 4), "g_proj.0.weight": (hd, hid),
              "g_proj.1.weight": (H * hd, hd), "g_proj.1.bias": (H * hd,),
              "o_proj.weight": (hid, H * hd)}
    base = {n: torch.randn(*s, generator=gen) * 0.02 for n, s in shapes.items()}
    base["dt_bias"] = torch.tensor([-5.6, -5.0])
    base["A_log"] = torch.tensor([1.5, 2.5])
    base["readout"] = torch.eye(127).expand(H, -1, -1).clone()
    for n in ("q_norm.weight", "k_norm.weight", "o_norm.weight"):
        base[n] = torch.ones(hd)
    x = torch.randn(B, T, hid, generator=gen)
    dy = torch.randn(B, T, hid, generator=gen)

    def grads(eps, seed):
        g = torch.Generator().manual_seed(seed)
        P = {n: (v * (1 + eps * torch.randn(v.shape, generator=g))).requires_grad_(True)
             for n, v in base.items()}
        xr = x * (1 + eps * torch.randn(x.shape, generator=g))
        (O.cyfa_layer(P, xr, H, hd, hd) * dy).sum().backward()
        return {n: p.grad for n, p in P.items()}

    g0 = grads(0.0, 0)
    g1 = grads(2.0 ** -9, 1)
    rel = {n: ((g1[n] - g0[n]).norm() / g0[n].norm()).item() for n in g0}
    assert rel["q_proj.weight"] < 1.5e-2
    assert max(rel["d_proj.bias"], rel["dt_bias"], rel["A_log"]) > 2 * rel["q_proj.weight"]
