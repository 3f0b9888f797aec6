"""GPU parity of the tcgen05 self-test GEMM, the decode step and the per-token
prep kernels against the CPU oracle (bf16 paths: rel-L2 <= 1e-2; fp32-accumulated
paths: <= 1e-4)."""

import math

import pytest
import torch

from gpu_util import bf16_cpu, rel_l2, seeded
from oracle import cyfa_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
F32_TOL = 1e-4


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib

    return _lib


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("K,N", [(64, 64), (128, 128), (256, 256), (192, 128)])
def test_umma_selftest(L, a_mn, b_mn, K, N):
    gen = seeded(K * 7 + N + a_mn * 3 + b_mn)
    A = torch.randn(128, K, generator=gen).to(torch.bfloat16)
    Bm = torch.randn(K, N, generator=gen).to(torch.bfloat16)
    a_store = (A.t().contiguous() if a_mn else A).cuda()
    b_store = (Bm if b_mn else Bm.t().contiguous()).cuda()
    c = torch.zeros(128, N, device="cuda")
    L.call("cyfa_selftest_umma", L.ptr(a_store), L.ptr(b_store), L.ptr(c), K, N, a_mn, b_mn,
           L.stream())
    torch.cuda.synchronize()
    ref = A.float() @ Bm.float()
    assert rel_l2(c, ref) < 1e-5
    assert L.device_error() == 0


def _decode_inputs(B, H, K, V, seed, with_state=True):
    gen = seeded(seed)
    q = torch.randn(B, 1, H, K, generator=gen)
    k = torch.randn(B, 1, H, K, generator=gen)
    v = torch.randn(B, 1, H, V, generator=gen)
    g = torch.log(torch.rand(B, 1, H, generator=gen) * 0.1 + 0.9)
    delta = torch.sigmoid(torch.randn(B, 1, H, generator=gen))
    beta = torch.sigmoid(torch.randn(B, 1, H, generator=gen))
    readout = torch.eye(127).expand(H, -1, -1) + 0.05 * torch.randn(H, 127, 127, generator=gen)
    qw = 1 + 0.1 * torch.randn(K, generator=gen)
    kw = 1 + 0.1 * torch.randn(K, generator=gen)
    state = None
    if with_state:
        state = (0.1 * torch.randn(B, H, K, 128, generator=gen),
                 0.1 * torch.randn(B, H, 128, V, generator=gen),
                 torch.rand(B, H, generator=gen) * 3000)
    return q, k, v, g, delta, beta, readout, qw, kw, state


@pytest.mark.parametrize("K,V", [(256, 256), (128, 128), (256, 128)])
@pytest.mark.parametrize("with_state", [True, False])
def test_decode_step_matches_oracle(L, K, V, with_state):
    B, H = 3, 2
    q, k, v, g, delta, beta, readout, qw, kw, state = _decode_inputs(B, H, K, V, 11, with_state)
    qb, kb, vb = bf16_cpu(q), bf16_cpu(k), bf16_cpu(v)
    ref_o, ref_state = O.fused_recurrent_cyfa(qb, kb, vb, g, delta, beta, readout, qw, kw,
                                              initial_state=state, output_final_state=True)
    table = O.readout_table(readout).float().cuda()
    dev = lambda x: x.contiguous().cuda()
    out = torch.empty(B, 1, H, V, device="cuda", dtype=torch.bfloat16)
    hk = torch.empty(B, H, K, 128, device="cuda")
    hv = torch.empty(B, H, 128, V, device="cuda")
    clk = torch.empty(B, H, device="cuda")
    st = [dev(x) for x in state] if state is not None else [None, None, None]
    args = [dev(q.to(torch.bfloat16)), dev(k.to(torch.bfloat16)), dev(v.to(torch.bfloat16)),
            dev(g), dev(delta), dev(beta), table, dev(qw), dev(kw)] + st + [hk, hv, clk, out]
    L.call("cyfa_decode_step", *[L.ptr(a) for a in args], B, H, K, V, 0, 1e-6, 1e-6,
           K ** -0.5, L.stream())
    torch.cuda.synchronize()
    assert rel_l2(out, ref_o) < BF16_TOL
    assert rel_l2(hk, ref_state[0]) < BF16_TOL
    assert rel_l2(hv, ref_state[1]) < BF16_TOL
    assert rel_l2(clk, ref_state[2]) < F32_TOL
    assert L.device_error() == 0


def test_decode_fp32_inputs(L):
    B, H, K, V = 2, 2, 256, 256
    q, k, v, g, delta, beta, readout, qw, kw, state = _decode_inputs(B, H, K, V, 12)
    ref_o, ref_state = O.fused_recurrent_cyfa(q, k, v, g, delta, beta, readout, qw, kw,
                                              initial_state=state, output_final_state=True)
    table = O.readout_table(readout).float().cuda()
    out = torch.empty(B, 1, H, V, device="cuda")
    hk = torch.empty(B, H, K, 128, device="cuda")
    hv = torch.empty(B, H, 128, V, device="cuda")
    clk = torch.empty(B, H, device="cuda")
    args = [x.contiguous().cuda() for x in (q, k, v, g, delta, beta)] + [table] + \
        [qw.cuda(), kw.cuda()] + [x.cuda() for x in state] + [hk, hv, clk, out]
    L.call("cyfa_decode_step", *[L.ptr(a) for a in args], B, H, K, V, 1, 1e-6, 1e-6,
           K ** -0.5, L.stream())
    torch.cuda.synchronize()
    assert rel_l2(out, ref_o) < F32_TOL
    assert rel_l2(hk, ref_state[0]) < F32_TOL
    assert rel_l2(hv, ref_state[1]) < F32_TOL


def test_decode_inplace_matches_out_of_place(L):
    """hk/hv/clock outputs aliased to their inputs (the graphed decoder's static
    cache) give bitwise the same steps as separate outputs, over many (b, h) and
    several repeated calls (the clock is read by every warp before it is stored)."""
    B, H, K, V = 64, 8, 256, 256
    q, k, v, g, delta, beta, readout, qw, kw, state = _decode_inputs(B, H, K, V, 21)
    table = O.readout_table(readout).float().cuda()
    ins = [x.to(torch.bfloat16).contiguous().cuda() for x in (q, k, v)] + \
        [x.contiguous().cuda() for x in (g, delta, beta)] + [table, qw.cuda(), kw.cuda()]
    a = [x.contiguous().cuda() for x in state]          # in place
    b = [x.contiguous().cuda() for x in state]          # out of place, ping-pong
    b2 = [torch.empty_like(x) for x in b]
    out_a = torch.empty(B, 1, H, V, device="cuda", dtype=torch.bfloat16)
    out_b = torch.empty_like(out_a)
    for _ in range(6):
        L.call("cyfa_decode_step", *[L.ptr(x) for x in ins + a + a + [out_a]], B, H, K, V, 0,
               1e-6, 1e-6, K ** -0.5, L.stream())
        L.call("cyfa_decode_step", *[L.ptr(x) for x in ins + b + b2 + [out_b]], B, H, K, V, 0,
               1e-6, 1e-6, K ** -0.5, L.stream())
        b, b2 = b2, b
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b)
        for x, y in zip(a, b):
            assert torch.equal(x, y)
    assert L.device_error() == 0


@pytest.mark.parametrize("T", [1, 100, 128, 300])
def test_gates_fwd(L, T):
    B, H = 2, 3
    gen = seeded(T)
    g = torch.log(torch.rand(B, T, H, generator=gen) * 0.1 + 0.9)
    delta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    clock0 = torch.rand(B, H, generator=gen) * 500
    TP = (T + 127) // 128 * 128
    G = torch.empty(B, H, TP, device="cuda")
    lam = torch.empty_like(G)
    bh = torch.empty_like(G)
    clk = torch.empty(B, H, device="cuda")
    L.call("cyfa_gates_fwd", *[L.ptr(x) for x in (g.cuda(), delta.cuda(), beta.cuda(),
                                                   clock0.cuda(), G, lam, bh, clk)],
           B, T, H, L.stream())
    torch.cuda.synchronize()
    ref_lam = O.clock_scan(delta.double().permute(0, 2, 1), clock0.double())
    assert rel_l2(lam[..., :T], ref_lam) < F32_TOL
    gp = torch.nn.functional.pad(g.double().permute(0, 2, 1), (0, TP - T))
    ref_G = gp.reshape(B, H, TP // 128, 128).cumsum(-1).reshape(B, H, TP) / math.log(2)
    assert rel_l2(G, ref_G) < F32_TOL
    assert torch.equal(bh[..., :T].cpu(), beta.permute(0, 2, 1))
    assert rel_l2(clk, delta.double().sum(1) + clock0.double()) < F32_TOL
    # padded tail: the clock stops and beta is zero
    if TP > T:
        assert torch.all(bh[..., T:] == 0)
        assert torch.all(lam[..., T:] == lam[..., T - 1:T])


@pytest.mark.parametrize("K", [256, 128])
def test_token_fwd_bwd(L, K):
    B, T, H = 2, 130, 2
    TP = 256
    gen = seeded(K)
    q = torch.randn(B, T, H, K, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, H, K, generator=gen).to(torch.bfloat16)
    qw = 1 + 0.1 * torch.randn(K, generator=gen)
    kw = 1 + 0.1 * torch.randn(K, generator=gen)
    lam = torch.rand(B, H, TP, generator=gen) * 4000
    beta = torch.rand(B, H, TP, generator=gen)
    beta[..., T:] = 0
    dev = lambda x: x.contiguous().cuda()
    qn = torch.empty(B, H, TP, K, device="cuda", dtype=torch.bfloat16)
    kn = torch.empty_like(qn)
    w = torch.empty(B, H, TP, 128, device="cuda", dtype=torch.bfloat16)
    qrs = torch.empty(B, H, TP, device="cuda")
    krs = torch.empty_like(qrs)
    L.call("cyfa_token_fwd", *[L.ptr(x) for x in (dev(q), dev(k), dev(qw), dev(kw), dev(lam),
                                                   dev(beta), qn, kn, w, qrs, krs)],
           B, T, H, K, 1e-6, 1e-6, L.stream())
    torch.cuda.synchronize()
    # forward parity
    qf = q.float().requires_grad_()
    kf = k.float().requires_grad_()
    qwf = qw.clone().requires_grad_()
    kwf = kw.clone().requires_grad_()
    lamf = lam[..., :T].clone().double().requires_grad_()
    betaf = beta[..., :T].clone().double().requires_grad_()
    ref_q = O.head_rmsnorm(qf, qwf, 1e-6)
    ref_k = O.head_rmsnorm(kf, kwf, 1e-6)
    ref_w, _, _ = O.write_vector(lamf, betaf, 128)
    assert rel_l2(qn[:, :, :T], ref_q) < BF16_TOL
    assert rel_l2(kn[:, :, :T], ref_k) < BF16_TOL
    assert rel_l2(w[:, :, :T], ref_w) < BF16_TOL
    assert torch.all(qn[:, :, T:] == 0) and torch.all(w[:, :, T:] == 0)
    # backward parity
    dqn = torch.randn(B, H, TP, K, generator=gen)
    dkn = torch.randn(B, H, TP, K, generator=gen)
    dw = torch.randn(B, H, TP, 128, generator=gen)
    (ref_q * dqn[:, :, :T]).sum().backward()
    (ref_k * dkn[:, :, :T]).sum().backward()
    (ref_w * dw[:, :, :T].double()).sum().backward()
    nblk = min((B * H * TP + 7) // 8, 444)  # partial rows, as the header states
    dq = torch.empty(B, T, H, K, device="cuda", dtype=torch.bfloat16)
    dk = torch.empty_like(dq)
    dqw = torch.zeros(nblk, K, device="cuda")
    dkw = torch.zeros_like(dqw)
    dlam = torch.empty(B, H, TP, device="cuda")
    dbeta = torch.empty_like(dlam)
    L.call("cyfa_token_bwd", *[L.ptr(x) for x in (dev(q), dev(k), dev(qw), dev(kw), qrs, krs,
                                                   dev(dqn), dev(dkn), dev(lam), dev(beta),
                                                   dev(dw), dq, dk, dqw, dkw, dlam, dbeta)],
           B, T, H, K, L.stream())
    torch.cuda.synchronize()
    assert rel_l2(dq, qf.grad) < BF16_TOL
    assert rel_l2(dk, kf.grad) < BF16_TOL
    assert rel_l2(dqw.sum(0), qwf.grad) < 1e-3
    assert rel_l2(dkw.sum(0), kwf.grad) < 1e-3
    assert rel_l2(dlam[..., :T], lamf.grad) < 1e-3
    assert rel_l2(dbeta[..., :T], betaf.grad) < 1e-3


@pytest.mark.parametrize("T", [5, 128, 333])
def test_gates_bwd(L, T):
    B, H = 2, 2
    TP = (T + 127) // 128 * 128
    gen = seeded(T + 1)
    dG = torch.randn(B, H, TP, generator=gen)
    dlam = torch.randn(B, H, TP, generator=gen)
    dbeta = torch.randn(B, H, TP, generator=gen)
    dclock = torch.randn(B, H, generator=gen)
    outs = [torch.empty(B, T, H, device="cuda") for _ in range(3)] + [torch.empty(B, H, device="cuda")]
    L.call("cyfa_gates_bwd", *[L.ptr(x) for x in (dG.cuda(), dlam.cuda(), dbeta.cuda(),
                                                   dclock.cuda(), *outs)], B, T, H, L.stream())
    torch.cuda.synchronize()
    # autograd through the forward definitions
    g = torch.zeros(B, T, H, dtype=torch.float64, requires_grad=True)
    d = torch.zeros(B, T, H, dtype=torch.float64, requires_grad=True)
    c0 = torch.zeros(B, H, dtype=torch.float64, requires_grad=True)
    gp = torch.nn.functional.pad(g.permute(0, 2, 1), (0, TP - T))
    # dG is the gradient w.r.t. the natural-log in-tile cumsum
    G = gp.reshape(B, H, TP // 128, 128).cumsum(-1).reshape(B, H, TP)
    dp = torch.nn.functional.pad(d.permute(0, 2, 1), (0, TP - T))
    lam = dp.cumsum(-1) + c0.unsqueeze(-1)
    clock = dp.sum(-1) + c0
    ((G * dG).sum() + (lam * dlam).sum() + (clock * dclock).sum()).backward()
    assert rel_l2(outs[0], g.grad) < 1e-5
    assert rel_l2(outs[1], d.grad) < 1e-5
    assert torch.equal(outs[2].cpu(), dbeta[..., :T].permute(0, 2, 1))
    assert rel_l2(outs[3], c0.grad) < 1e-5


def test_readout_table_kernels(L):
    """cyfa_readout_table / cyfa_readout_table_grad against the oracle's fp64
    table product and its adjoint (bf16 table: rel-L2 <= 1e-2; fp32 gradient:
    rel-L2 <= 1e-4)."""
    from cyclic_flow_attention.ops.chunk import readout_grad, table_bf16

    H = 3
    gen = torch.Generator().manual_seed(21)
    readout = torch.eye(127).expand(H, -1, -1) + 0.05 * torch.randn(H, 127, 127, generator=gen)
    tb = table_bf16(readout.cuda())
    torch.cuda.synchronize()
    ref = O.readout_table(readout)  # [H, 127, 128] fp64
    assert tb.shape == (H, 128, 128) and tb.dtype == torch.bfloat16
    assert rel_l2(tb[:, :127].float().cpu(), ref) < BF16_TOL
    assert torch.count_nonzero(tb[:, 127]).item() == 0
    dtab = torch.randn(H, 128, 128, generator=gen)
    dr = readout_grad(dtab.cuda(), readout.cuda())
    torch.cuda.synchronize()
    ref_dr = dtab[:, :127].double() @ O.basis(128).t()
    assert dr.shape == (H, 127, 127)
    assert rel_l2(dr.cpu(), ref_dr) < F32_TOL
    assert L.device_error() == 0


@pytest.mark.parametrize("K,V,W", [(256, 256, 4), (128, 256, 3), (256, 128, 2)])
def test_decode_layer_matches_separate_kernels(L, K, V, W):
    """cyfa_decode_layer (convolutions, gate activations, decode step and gated
    output norm of a layer's T = 1 step in one launch) against the chain of
    separate launches it replaces (cyfa_decode_conv, cyfa_gate_act_fwd,
    cyfa_decode_step, cyfa_gated_norm_bias_fwd): bitwise equal convolution
    histories, states and clock; the output equal up to the order of the norm's
    row sum (rare one-ulp bf16 differences)."""
    import ctypes

    gen = seeded(K + V + W)
    B, H = 6, 4
    HK, HV = H * K, H * V
    a_col = 2 * HK + HV + V
    NB = (a_col + 3 * H + 7) // 8 * 8
    bf = torch.bfloat16
    P = torch.randn(B, NB, generator=gen).to(bf).cuda()
    caches = [(0.5 * torch.randn(B, W - 1, C, generator=gen)).to(bf).cuda() for C in (HK, HK, HV)]
    wconv = [(0.3 * torch.randn(C, W, generator=gen)).cuda() for C in (HK, HK, HV)]
    A_log = torch.randn(H, generator=gen).cuda()
    dt_bias = torch.randn(H, generator=gen).cuda()
    b_bias = torch.randn(H, generator=gen).cuda()
    d_bias = torch.randn(H, generator=gen).cuda()
    table = (0.1 * torch.randn(H, 127, 128, generator=gen)).cuda()
    qn = (1 + 0.1 * torch.randn(K, generator=gen)).cuda()
    kn = (1 + 0.1 * torch.randn(K, generator=gen)).cuda()
    hk = (0.1 * torch.randn(B * H, K, 128, generator=gen)).cuda()
    hv = (0.1 * torch.randn(B * H, 128, V, generator=gen)).cuda()
    clock = (100 * torch.rand(B * H, generator=gen)).cuda()
    gate = torch.randn(B, HV, generator=gen).to(bf).cuda()
    gbias = (0.1 * torch.randn(HV, generator=gen)).to(bf).cuda()
    onorm = (1 + 0.1 * torch.randn(V, generator=gen)).cuda()
    p, st, ps = L.ptr, L.stream(), NB
    # ---- the separate launches
    c1 = [t.clone() for t in caches]
    q = torch.empty(B, 1, H, K, device="cuda", dtype=bf)
    k = torch.empty_like(q)
    v = torch.empty(B, 1, H, V, device="cuda", dtype=bf)
    L.call("cyfa_decode_conv", p(P), ps, p(c1[0]), p(c1[1]), p(c1[2]), p(wconv[0]), p(wconv[1]),
           p(wconv[2]), p(q), p(k), p(v), B, HK, HK, HV, W, st)
    g = torch.empty(B, 1, H, device="cuda")
    delta, beta = torch.empty_like(g), torch.empty_like(g)
    L.call("cyfa_gate_act_fwd", p(P[:, a_col:]), ps, p(P[:, a_col + H:]), ps,
           p(P[:, a_col + 2 * H:]), ps, p(A_log), p(dt_bias), p(b_bias), p(d_bias), p(g),
           p(delta), p(beta), B, H, st)
    hk1, hv1, clock1 = torch.empty_like(hk), torch.empty_like(hv), torch.empty_like(clock)
    o = torch.empty(B, 1, H, V, device="cuda", dtype=bf)
    L.call("cyfa_decode_step", p(q), p(k), p(v), p(g), p(delta), p(beta), p(table), p(qn), p(kn),
           p(hk), p(hv), p(clock), p(hk1), p(hv1), p(clock1), p(o), B, H, K, V, 0, 1e-6, 1e-6,
           K ** -0.5, st)
    y1 = torch.empty(B, HV, device="cuda", dtype=bf)
    rstd = torch.empty(B * H, device="cuda")
    L.call("cyfa_gated_norm_bias_fwd", p(o), p(gate), p(gbias), H, p(onorm), 1e-5, 127.0, p(y1),
           p(rstd), B * H, V, st)
    # ---- one launch
    c2 = [t.clone() for t in caches]
    hk2, hv2, clock2 = torch.empty_like(hk), torch.empty_like(hv), torch.empty_like(clock)
    y2 = torch.empty_like(y1)
    a = L.DecodeLayerArgs(
        B=B, H=H, K=K, V=V, W=W, a_col=a_col, P_stride=NB, P=p(P), cache_q=p(c2[0]),
        cache_k=p(c2[1]), cache_v=p(c2[2]), wconv_q=p(wconv[0]), wconv_k=p(wconv[1]),
        wconv_v=p(wconv[2]), A_log=p(A_log), dt_bias=p(dt_bias), b_bias=p(b_bias),
        d_bias=p(d_bias), table=p(table), q_norm_weight=p(qn), k_norm_weight=p(kn), hk_in=p(hk),
        hv_in=p(hv), clock_in=p(clock), hk_out=p(hk2), hv_out=p(hv2), clock_out=p(clock2),
        gate=p(gate), gate_bias=p(gbias), o_norm_weight=p(onorm), y=p(y2), q_eps=1e-6,
        k_eps=1e-6, scale=K ** -0.5, o_eps=1e-5, o_scale=127.0)
    L.call("cyfa_decode_layer", ctypes.byref(a), st)
    torch.cuda.synchronize()
    for x1, x2 in zip(c1, c2):
        assert torch.equal(x1, x2)
    assert torch.equal(hk1, hk2) and torch.equal(hv1, hv2) and torch.equal(clock1, clock2)
    assert rel_l2(y2, y1) < 2e-3
    assert L.device_error() == 0
