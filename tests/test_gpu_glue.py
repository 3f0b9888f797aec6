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
