"""The allocation-free entry point cyfa_gated_norm_bwd_static.

Some callers cannot give the library a workspace: bindings whose FFI signature
carries only the op's own tensors, and processes whose device memory belongs to
a framework allocator that third-party code may not draw from.  For them the
gated-norm backward keeps its weight-gradient partials in a fixed device array
inside the library.  On two calls in a row through the C ABI it must match both
cyfa_gated_norm_bwd (which takes a caller-provided work buffer) and a plain fp32
PyTorch reference of the same backward.  The file name makes pytest collect it
last."""

import ctypes

import pytest
import torch

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the bf16 tolerance of the GPU parity tests
SCALE, EPS = 127.0, 1e-6


def _case(rows, D, seed, L):
    gen = torch.Generator().manual_seed(seed)
    x = (0.01 * torch.randn(rows, D, generator=gen)).to(torch.bfloat16).cuda()
    gate = torch.randn(rows, D, generator=gen).to(torch.bfloat16).cuda()
    w = (1 + 0.1 * torch.randn(D, generator=gen)).cuda()
    dy = torch.randn(rows, D, generator=gen).to(torch.bfloat16).cuda()
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device="cuda")
    L.call("cyfa_gated_norm_fwd", L.ptr(x), L.ptr(gate), L.ptr(w), EPS, SCALE, L.ptr(y),
           L.ptr(rstd), rows, D, L.stream())
    return x, gate, w, rstd, dy


def _fp32_reference(x, gate, w, dy):
    """y = u rsqrt(mean(u^2) + eps) w sigmoid(gate), u = scale x, in fp32 autograd."""
    xr = x.detach().float().requires_grad_(True)
    gr = gate.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    u = xr * SCALE
    y = u * torch.rsqrt(u.pow(2).mean(-1, keepdim=True) + EPS) * wr * torch.sigmoid(gr)
    (y * dy.float()).sum().backward()
    return xr.grad, gr.grad, wr.grad


def _with_work(L, x, gate, w, rstd, dy, rows, D):
    dx, dg, dw = torch.empty_like(x), torch.empty_like(gate), torch.empty(D, device="cuda")
    n = L.lib().cyfa_gated_norm_work_bytes(rows, D)
    work = torch.empty(n, device="cuda", dtype=torch.uint8)
    L.call("cyfa_gated_norm_bwd", L.ptr(x), L.ptr(gate), L.ptr(w), SCALE, L.ptr(rstd), L.ptr(dy),
           L.ptr(dx), L.ptr(dg), L.ptr(dw), rows, D, L.ptr(work), ctypes.c_size_t(n), L.stream())
    return dx, dg, dw


def _static(L, x, gate, w, rstd, dy, rows, D):
    dx, dg, dw = torch.empty_like(x), torch.empty_like(gate), torch.empty(D, device="cuda")
    L.call("cyfa_gated_norm_bwd_static", L.ptr(x), L.ptr(gate), L.ptr(w), SCALE, L.ptr(rstd),
           L.ptr(dy), L.ptr(dx), L.ptr(dg), L.ptr(dw), rows, D, L.stream())
    return dx, dg, dw


def test_static_scratch_entry_matches_workspace_entry():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib as L

    # two calls in a row, different sizes, so a stale scratch would show up
    for rows, D, seed in ((5000, 256, 1), (777, 128, 2)):
        args = _case(rows, D, seed, L)
        ref = _with_work(L, *args, rows, D)
        got = _static(L, *args, rows, D)
        x, gate, w, _, dy = args
        f32 = _fp32_reference(x, gate, w, dy)
        torch.cuda.synchronize()
        for a, b, c in zip(got, ref, f32):
            assert rel_l2(a, b) < TOL
            assert rel_l2(a, c) < TOL
    assert L.device_error() == 0
