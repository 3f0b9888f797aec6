"""GPU parity of chunk_cyfa (forward and backward) against the CPU oracle.

Tolerances: bf16 outputs and gradients rel-L2 <= 1e-2 of
the fp32 oracle; the fp32 clock <= 1e-4.  Two gate gradients are suffix sums:
ddelta_t = sum_{s>=t} dlam_s (+ the final clock's gradient), and dg_t, the
in-tile suffix sum of the per-token gate terms.  Their per-token terms (the
differences of consecutive entries) must meet 1e-2; the sums themselves then
meet 1e-2 times the summation's condition number (suffix sums of |terms| over
suffix sums of terms, from the oracle), the forward error bound of summation.
"""

import pytest
import torch

from gpu_util import rel_l2, seeded, suffix_condition, suffix_terms
from oracle import cyfa_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
F32_TOL = 1e-4


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import ops as _ops

    return _ops


def make_inputs(B, T, H, K, V, seed=0, with_state=False, gate_scale=1.0):
    gen = seeded(seed)
    q = torch.randn(B, T, H, K, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, H, K, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, T, H, V, generator=gen).to(torch.bfloat16)
    g = torch.log(1 - gate_scale * 0.1 * torch.rand(B, T, H, generator=gen))
    delta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    readout = torch.eye(127).expand(H, -1, -1) + 0.05 * torch.randn(H, 127, 127, generator=gen)
    qw = 1 + 0.1 * torch.randn(K, generator=gen)
    kw = 1 + 0.1 * torch.randn(K, generator=gen)
    state = None
    if with_state:
        state = (0.05 * torch.randn(B, H, K, 128, generator=gen),
                 0.05 * torch.randn(B, H, 128, V, generator=gen),
                 torch.rand(B, H, generator=gen) * 1000)
    return [q, k, v, g, delta, beta, readout, qw, kw], state


FWD_CASES = [
    (1, 256, 2, 256, 256, False),
    (2, 300, 1, 256, 256, True),
    (1, 200, 2, 128, 128, False),
    (1, 384, 1, 256, 128, True),
    (2, 130, 2, 128, 256, False),
    (1, 1, 1, 256, 256, True),
]


@pytest.mark.parametrize("B,T,H,K,V,with_state", FWD_CASES)
def test_chunk_forward(ops, B, T, H, K, V, with_state):
    ins, state = make_inputs(B, T, H, K, V, seed=B * 1000 + T + K + V, with_state=with_state)
    dev = [x.cuda() for x in ins]
    st = None if state is None else tuple(x.cuda() for x in state)
    with torch.no_grad():
        o, fs = ops.chunk_cyfa(*dev, initial_state=st, output_final_state=True)
    torch.cuda.synchronize()
    ref_o, ref_s = O.chunk_cyfa(*[x.float() for x in ins[:6]], *ins[6:], initial_state=state,
                                output_final_state=True, dtype=torch.float32)
    assert rel_l2(fs[0], ref_s[0]) < BF16_TOL, "key state"
    assert rel_l2(fs[1], ref_s[1]) < BF16_TOL, "value state"
    assert rel_l2(fs[2], ref_s[2]) < F32_TOL, "clock"
    assert rel_l2(o, ref_o) < BF16_TOL, "output"
    from cyclic_flow_attention import _lib

    assert _lib.device_error() == 0


def test_chunk_forward_deterministic(ops):
    ins, _ = make_inputs(2, 512, 2, 256, 256, seed=3)
    dev = [x.cuda() for x in ins]
    with torch.no_grad():
        a, sa = ops.chunk_cyfa(*dev, output_final_state=True)
        b, sb = ops.chunk_cyfa(*dev, output_final_state=True)
    assert torch.equal(a, b)
    for x, y in zip(sa, sb):
        assert torch.equal(x, y)


def test_chunk_strong_decay_stays_finite(ops):
    """Gates near zero (alpha ~ 0) must not overflow the in-tile decay factors."""
    ins, _ = make_inputs(1, 256, 1, 256, 256, seed=9)
    ins[3] = torch.full_like(ins[3], -30.0)
    dev = [x.cuda() for x in ins]
    with torch.no_grad():
        o, fs = ops.chunk_cyfa(*dev, output_final_state=True)
    assert torch.isfinite(o).all() and all(torch.isfinite(x).all() for x in fs)
    ref_o, _ = O.chunk_cyfa(*[x.float() for x in ins[:6]], *ins[6:], dtype=torch.float32)
    assert rel_l2(o, ref_o) < BF16_TOL


BWD_CASES = [
    (1, 256, 2, 256, 256, False),
    (2, 200, 1, 256, 256, True),
    (1, 256, 2, 128, 128, True),
    (1, 130, 1, 256, 128, False),
    (1, 384, 1, 128, 256, True),
]


@pytest.mark.parametrize("B,T,H,K,V,with_state", BWD_CASES)
def test_chunk_backward(ops, B, T, H, K, V, with_state):
    ins, state = make_inputs(B, T, H, K, V, seed=B * 77 + T + K + 3 * V, with_state=with_state)
    gen = seeded(T + 5)
    do = torch.randn(B, T, H, V, generator=gen)
    dst = None
    if with_state:
        dst = (torch.randn(B, H, K, 128, generator=gen), torch.randn(B, H, 128, V, generator=gen),
               torch.randn(B, H, generator=gen))
    # GPU
    dev = [x.cuda().requires_grad_(True) for x in ins]
    st = None if state is None else tuple(x.cuda().requires_grad_(True) for x in state)
    o, fs = ops.chunk_cyfa(*dev, initial_state=st, output_final_state=True)
    loss = (o.float() * do.cuda()).sum()
    if dst is not None:
        loss = loss + sum((a * b.cuda()).sum() for a, b in zip(fs, dst))
    loss.backward()
    torch.cuda.synchronize()
    # oracle (fp32 autograd)
    ref_in = [x.float().clone().requires_grad_(True) for x in ins]
    ref_st = None if state is None else tuple(x.clone().requires_grad_(True) for x in state)
    ro, rs = O.chunk_cyfa(*ref_in, initial_state=ref_st, output_final_state=True,
                          dtype=torch.float32)
    rl = (ro * do).sum()
    if dst is not None:
        rl = rl + sum((a * b).sum() for a, b in zip(rs, dst))
    rl.backward()
    names = ["q", "k", "v", "g", "delta", "beta", "readout", "q_norm_weight", "k_norm_weight"]
    errs = {n: rel_l2(a.grad, b.grad) for n, a, b in zip(names, dev, ref_in)}
    tols = [BF16_TOL] * len(names)
    # suffix sums: per-token terms at 1e-2, the sums at 1e-2 x their condition number
    tg = [x.grad.permute(0, 2, 1) for x in (dev[3], ref_in[3], dev[4], ref_in[4])]
    errs["g_terms"] = rel_l2(suffix_terms(tg[0], 128), suffix_terms(tg[1], 128))
    errs["delta_terms"] = rel_l2(suffix_terms(tg[2]), suffix_terms(tg[3]))
    tols[3] = BF16_TOL * max(1.0, suffix_condition(suffix_terms(tg[1], 128), 128))
    tols[4] = BF16_TOL * max(1.0, suffix_condition(suffix_terms(tg[3])))
    names += ["g_terms", "delta_terms"]
    tols += [BF16_TOL, BF16_TOL]
    if st is not None:
        for n, a, b in zip(["hk0", "hv0", "clock0"], st, ref_st):
            errs[n] = rel_l2(a.grad, b.grad)
        # dclock0 = ddelta_0: the sum of all the clock terms of a sequence
        ct = suffix_terms(tg[3])
        tols += [BF16_TOL, BF16_TOL,
                 BF16_TOL * max(1.0, (ct.abs().sum(-1).norm() / ct.sum(-1).norm()).item())]
        names += ["hk0", "hv0", "clock0"]
    print("chunk grad errors", B, T, H, K, V, with_state, {k: round(v, 5) for k, v in errs.items()},
          "tolerances", [round(t, 4) for t in tols])
    bad = {n: errs[n] for n, t in zip(names, tols) if errs[n] >= t}
    assert not bad, f"gradient errors over tolerance: {bad} (all: {errs})"
    from cyclic_flow_attention import _lib

    assert _lib.device_error() == 0


def test_chunk_backward_deterministic(ops):
    ins, _ = make_inputs(2, 300, 2, 256, 256, seed=21)
    do = torch.randn(2, 300, 2, 256, generator=seeded(1)).cuda()
    grads = []
    for _ in range(2):
        dev = [x.cuda().requires_grad_(True) for x in ins]
        o, _ = ops.chunk_cyfa(*dev)
        (o.float() * do).sum().backward()
        grads.append([x.grad.clone() for x in dev])
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("K,V", [(256, 256), (256, 128), (128, 256)])
def test_chunk_batched_matches_per_sequence(ops, K, V):
    """(b, h) pairs are independent, so a batch of 8 sequences (512 tiles at
    T = 2048, H = 4: several tiles per persistent CTA, ring and TMEM buffers
    wrapping around) must give exactly the per-token outputs and gradients of
    the same sequences run one at a time (64 tiles, one per CTA).  Parameter
    gradients are sums over the batch, reduced in another order: 1e-5."""
    B, T, H = 8, 2048, 4
    ins, state = make_inputs(B, T, H, K, V, seed=K + V, with_state=True)
    do = torch.randn(B, T, H, V, generator=seeded(9)).to(torch.bfloat16).cuda()
    from cyclic_flow_attention import _lib

    # one serial scan per state slice at every batch size (a single sequence
    # would otherwise get segmented scans, another summation order)
    prev_split = _lib.set_scan_split(False)

    def run(sl):
        dev = [x[sl].cuda().requires_grad_(True) if i < 6 else x.cuda().requires_grad_(True)
               for i, x in enumerate(ins)]
        st = tuple(x[sl].cuda().requires_grad_(True) for x in state)
        o, fs = ops.chunk_cyfa(*dev, initial_state=st, output_final_state=True)
        (o.float() * do[sl].float()).sum().backward()
        return o.detach(), [x.grad for x in dev] + [x.grad for x in st]

    try:
        o_all, g_all = run(slice(0, B))
        per = [run(slice(b, b + 1)) for b in range(B)]
        torch.cuda.synchronize()
    finally:
        _lib.set_scan_split(prev_split)
    assert torch.equal(o_all, torch.cat([p[0] for p in per]))
    # per-token tensors: q k v g delta beta and the initial-state grads (batch dim 0)
    for i in list(range(6)) + [9, 10, 11]:
        want = torch.cat([p[1][i] for p in per])
        assert torch.equal(g_all[i], want), i
    # batch-reduced parameters: readout, q/k norm weights
    for i in (6, 7, 8):
        want = sum(p[1][i] for p in per)
        assert rel_l2(g_all[i], want) <= 1e-5, i
    from cyclic_flow_attention import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("B,T,H,K,V", [(1, 4096, 1, 256, 256), (1, 8192, 1, 128, 128),
                                       (2, 4100, 1, 256, 128)])
def test_segmented_scans_match_serial(ops, B, T, H, K, V):
    """With few sequences x heads the state scans split their tiles into
    segments scanned side by side (summary pass, carries, real pass): outputs,
    final states and every gradient equal the one-serial-pass result up to
    fp32 summation order, and the oracle to the usual tolerances."""
    from cyclic_flow_attention import _lib

    # weak decay (alpha ~ 0.9995 per token), so the carried states matter
    ins, state = make_inputs(B, T, H, K, V, seed=T + K, with_state=True, gate_scale=0.01)
    gen = seeded(T)
    do = torch.randn(B, T, H, V, generator=gen).to(torch.bfloat16).cuda()
    dst = (torch.randn(B, H, K, 128, generator=gen).cuda(),
           torch.randn(B, H, 128, V, generator=gen).cuda(), torch.randn(B, H, generator=gen).cuda())

    def run(split):
        prev = _lib.set_scan_split(split)
        try:
            dev = [x.cuda().requires_grad_(True) for x in ins]
            st = tuple(x.cuda().requires_grad_(True) for x in state)
            o, fs = ops.chunk_cyfa(*dev, initial_state=st, output_final_state=True)
            loss = (o.float() * do.float()).sum() + sum((a * b).sum() for a, b in zip(fs, dst))
            loss.backward()
            torch.cuda.synchronize()
        finally:
            _lib.set_scan_split(prev)
        return [o.detach()] + [x.detach() for x in fs] + [x.grad for x in dev] + \
            [x.grad for x in st]

    seg, ser = run(True), run(False)
    names = ["o", "hk", "hv", "clock", "dq", "dk", "dv", "dg", "ddelta", "dbeta", "dreadout",
             "dqw", "dkw", "dhk0", "dhv0", "dclock0"]
    errs = {n: rel_l2(a, b) for n, a, b in zip(names, seg, ser)}
    # the carries round differently; bf16 histories pass that on as occasional
    # one-ulp flips.  The clock gradients are suffix sums over the whole sequence:
    # compared per term, and as sums within their condition number.
    dd_seg, dd_ser = (x.permute(0, 2, 1) for x in (seg[8], ser[8]))
    errs["ddelta_terms"] = rel_l2(suffix_terms(dd_seg), suffix_terms(dd_ser))
    terms = suffix_terms(dd_ser)
    kappa = {"ddelta": suffix_condition(terms),
             "dclock0": (terms.abs().sum(-1).norm() / terms.sum(-1).norm()).item()}
    print("segmented vs serial", B, T, H, K, V, {k: float(f"{v:.3g}") for k, v in errs.items()},
          "kappa", {k: round(v, 1) for k, v in kappa.items()})
    assert errs["hk"] < 1e-5 and errs["hv"] < 1e-5 and errs["clock"] < 1e-6
    for n, e in errs.items():
        assert e < BF16_TOL * max(1.0, kappa.get(n, 1.0)), (n, e)
    ref_o, ref_s = O.chunk_cyfa(*[x.float() for x in ins[:6]], *ins[6:], initial_state=state,
                                output_final_state=True, dtype=torch.float32)
    assert rel_l2(seg[0], ref_o) < BF16_TOL
    assert rel_l2(seg[1], ref_s[0]) < BF16_TOL and rel_l2(seg[2], ref_s[1]) < BF16_TOL
    assert _lib.device_error() == 0
