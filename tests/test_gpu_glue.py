"""GPU parity of the layer glue kernels (short conv, gate activations, gated
output norm) against plain fp32 torch references with autograd."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def LO():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention.ops import layer_ops

    return layer_ops


def _conv_ref(x, w, b=None):
    B, T, C = x.shape
    W = w.shape[-1]
    y = F.conv1d(F.pad(x.transpose(1, 2), (W - 1, 0)), w, b, groups=C)
    return y.transpose(1, 2)


# C % 128 == 0 takes the TMA-streamed kernels (T not a multiple of their 64-token
# tiles, T = 1, every width); other C the register-window kernels.
@pytest.mark.parametrize("B,T,C,W,bias", [(2, 300, 256, 4, False), (1, 128, 3072, 4, False),
                                          (2, 17, 64, 3, False), (1, 200, 384, 3, True),
                                          (3, 64, 128, 2, False), (1, 1, 128, 4, True),
                                          (2, 70, 256, 1, False)])
def test_short_conv(LO, B, T, C, W, bias):
    gen = torch.Generator().manual_seed(T + C)
    x = torch.randn(B, T, C, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    w = (0.3 * torch.randn(C, 1, W, generator=gen)).cuda().requires_grad_(True)
    b = (0.1 * torch.randn(C, generator=gen)).cuda().requires_grad_(True) if bias else None
    dy = torch.randn(B, T, C, generator=gen).cuda()
    y = LO.ShortConvFunction.apply(x, w, b)
    (y.float() * dy).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    br = b.detach().clone().requires_grad_(True) if bias else None
    yr = _conv_ref(xr, wr, br)
    (yr * dy).sum().backward()
    assert rel_l2(y, yr) < 1e-2
    assert rel_l2(x.grad, xr.grad) < 1e-2
    assert rel_l2(w.grad, wr.grad) < 1e-2  # dy enters in bf16
    if bias:
        assert rel_l2(b.grad, br.grad) < 1e-2


def test_gate_act(LO):
    B, T, H, width = 2, 100, 4, 264
    gen = torch.Generator().manual_seed(7)
    aux = torch.randn(B, T, width, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    dlin = torch.randn(B, T, H, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    A_log = torch.log(torch.rand(H, generator=gen) * 16 + 1e-3).cuda().requires_grad_(True)
    dt = (torch.randn(H, generator=gen) - 4).cuda().requires_grad_(True)
    bb = (0.1 * torch.randn(H, generator=gen)).cuda().requires_grad_(True)
    db = (0.1 * torch.randn(H, generator=gen)).cuda().requires_grad_(True)
    a_col, b_col = 256, 260
    g, d, b = LO.GateActFunction.apply(aux, dlin, A_log, dt, bb, db, a_col, b_col, H)
    ups = [torch.randn(B, T, H, generator=gen).cuda() for _ in range(3)]
    sum((x * u).sum() for x, u in zip((g, d, b), ups)).backward()
    auxr = aux.detach().float().requires_grad_(True)
    dlr = dlin.detach().float().requires_grad_(True)
    Ar = A_log.detach().clone().requires_grad_(True)
    dtr = dt.detach().clone().requires_grad_(True)
    bbr = bb.detach().clone().requires_grad_(True)
    dbr = db.detach().clone().requires_grad_(True)
    gr = -Ar.exp() * F.softplus(auxr[..., a_col:a_col + H] + dtr)
    drr = torch.sigmoid(dlr + dbr)
    brr = torch.sigmoid(auxr[..., b_col:b_col + H] + bbr)
    sum((x * u).sum() for x, u in zip((gr, drr, brr), ups)).backward()
    for a_, b_ in zip((g, d, b), (gr, drr, brr)):
        assert rel_l2(a_, b_) < 1e-5
    assert rel_l2(aux.grad, auxr.grad) < 1e-2
    assert rel_l2(dlin.grad, dlr.grad) < 1e-2
    assert rel_l2(A_log.grad, Ar.grad) < 1e-4
    assert rel_l2(dt.grad, dtr.grad) < 1e-4
    assert rel_l2(bb.grad, bbr.grad) < 1e-4
    assert rel_l2(db.grad, dbr.grad) < 1e-4


@pytest.mark.parametrize("D", [256, 128])
@pytest.mark.parametrize("B,T,H", [(2, 70, 3), (4, 700, 4)])
def test_gated_norm(LO, D, B, T, H):
    gen = torch.Generator().manual_seed(D)
    x = (0.01 * torch.randn(B, T, H, D, generator=gen)).to(torch.bfloat16).cuda().requires_grad_(True)
    gin = torch.randn(B, T, D, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    gw = (0.05 * torch.randn(H * D, D, generator=gen)).to(torch.bfloat16).cuda().requires_grad_(True)
    gb = (0.1 * torch.randn(H * D, generator=gen)).to(torch.bfloat16).cuda().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(D, generator=gen)).cuda().requires_grad_(True)
    dy = torch.randn(B, T, H * D, generator=gen).cuda()
    y = LO.GatedNormFunction.apply(x, gin, gw, gb, w, 1e-6, 127.0)
    (y.float() * dy).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    ginr = gin.detach().float().requires_grad_(True)
    gwr = gw.detach().float().requires_grad_(True)
    gbr = gb.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    gr = F.linear(ginr, gwr, gbr)
    u = xr * 127.0
    yr = u * torch.rsqrt(u.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    yr = (yr * torch.sigmoid(gr.reshape(B, T, H, D))).reshape(B, T, H * D)
    (yr * dy).sum().backward()
    assert rel_l2(y, yr) < 1e-2
    assert rel_l2(x.grad, xr.grad) < 1e-2
    for a, b in ((gin, ginr), (gw, gwr), (gb, gbr)):
        assert rel_l2(a.grad, b.grad) < 1e-2
    assert rel_l2(w.grad, wr.grad) < 1e-2  # dy enters in bf16


@pytest.mark.parametrize("D,Kg,H,tokens,bias", [(256, 256, 4, 16384, True), (256, 192, 3, 333, True),
                                                (128, 128, 2, 1, False), (128, 320, 5, 700, True)])
def test_gated_norm_gate_fused(D, Kg, H, tokens, bias):
    """cyfa_gated_norm_gate_fwd (the gate linear on tcgen05 inside the norm
    kernel) against the gate linear in fp32 rounded to bf16 followed by the
    norm in fp32, with gin a strided column view of a wider packed tensor, a
    partial last 128-token tile, and the optional gate output."""
    from cyclic_flow_attention import _lib

    gen = torch.Generator().manual_seed(D + Kg + H)
    width = Kg + 72  # gin sits at column 40 of a [tokens, Kg + 72] projection
    P = torch.randn(tokens, width, generator=gen).to(torch.bfloat16).cuda()
    gin = P[:, 40:40 + Kg]
    x = (0.01 * torch.randn(tokens, H, D, generator=gen)).to(torch.bfloat16).cuda()
    gw = (0.05 * torch.randn(H * D, Kg, generator=gen)).to(torch.bfloat16).cuda()
    gb = (0.1 * torch.randn(H * D, generator=gen)).to(torch.bfloat16).cuda() if bias else None
    w = (1 + 0.1 * torch.randn(D, generator=gen)).cuda()
    y = torch.empty(tokens, H * D, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(tokens * H, device="cuda")
    gate = torch.empty(tokens, H * D, device="cuda", dtype=torch.bfloat16)
    p = _lib.ptr
    _lib.call("cyfa_gated_norm_gate_fwd", p(x), p(gin), width, p(gw), p(gb), H, Kg, p(w), 1e-6,
              127.0, p(y), p(rstd), p(gate), tokens, D, _lib.stream())
    torch.cuda.synchronize()
    g_ref = (gin.float() @ gw.float().t())
    # the gate: fp32 accumulation in another order, then bf16 rounding
    assert (gate.float() - g_ref).abs().max() <= 2 ** -7 * g_ref.abs().max() + 1e-3
    assert rel_l2(gate, g_ref) < 4e-3
    u = x.float() * 127.0
    rs = torch.rsqrt(u.pow(2).mean(-1) + 1e-6)
    gt = g_ref.to(torch.bfloat16).float() + (gb.float() if bias else 0.0)
    yr = (u * rs[..., None] * w) * torch.sigmoid(gt.reshape(tokens, H, D))
    assert rel_l2(rstd, rs.reshape(-1)) < 1e-5
    assert rel_l2(y, yr.reshape(tokens, H * D)) < 1e-2
    # no gate output requested: same y
    y2 = torch.empty_like(y)
    _lib.call("cyfa_gated_norm_gate_fwd", p(x), p(gin), width, p(gw), p(gb), H, Kg, p(w), 1e-6,
              127.0, p(y2), p(rstd), None, tokens, D, _lib.stream())
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    assert _lib.device_error() == 0


def test_gated_norm_inference_path(LO):
    """gated_norm_infer (the inference path: the gate linear inside the norm
    kernel) matches GatedNormFunction (cuBLAS linear, then the norm) up to the
    bf16 rounding of a gate accumulated in another order."""
    gen = torch.Generator().manual_seed(7)
    B, T, H, D = 2, 300, 4, 256
    P = torch.randn(B, T, 3 * D, generator=gen).to(torch.bfloat16).cuda()
    gin = P[..., D:2 * D]  # a column view, as the layer passes it
    x = (0.01 * torch.randn(B, T, H, D, generator=gen)).to(torch.bfloat16).cuda()
    gw = (0.05 * torch.randn(H * D, D, generator=gen)).to(torch.bfloat16).cuda()
    gb = (0.1 * torch.randn(H * D, generator=gen)).to(torch.bfloat16).cuda()
    w = (1 + 0.1 * torch.randn(D, generator=gen)).cuda()
    with torch.no_grad():
        y_inf = LO.gated_norm_infer(x, gin, gw, gb, w, 1e-6, 127.0)
    y_train = LO.GatedNormFunction.apply(x, gin, gw, gb, w.clone().requires_grad_(True), 1e-6,
                                         127.0)
    assert rel_l2(y_inf, y_train) < 2e-3
