"""GPU checks of the CyclicFlowAttention layer: parity with the oracle layer
(forward and backward), and the reference's own hot-path test
(tests/test_inference.py:20-34 of the reference): decoding the next token from
a prefill cache matches the full-sequence forward (rel-RMS < 0.02 there; the
bf16 tolerance 1e-2 is used here)."""

import pytest
import torch

from gpu_util import gate_param_tolerances, rel_l2
from oracle import cyfa_oracle as O


pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Layer():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import CyclicFlowAttention

    return CyclicFlowAttention


def _layer(Layer, hidden, H, hd, seed):
    torch.manual_seed(seed)
    m = Layer(hidden, H, hd)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if p.dim() >= 2 and name != "readout":
                p.normal_(0, 0.02)
        m.readout.add_(0.05 * torch.randn_like(m.readout))
    return m.keep_fp32().cuda()


@pytest.mark.parametrize("B,T,hidden,H,hd", [(2, 256, 512, 2, 256), (1, 200, 256, 2, 128)])
def test_layer_forward_backward(Layer, B, T, hidden, H, hd):
    m = _layer(Layer, hidden, H, hd, seed=T)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, T, hidden, generator=gen).to(torch.bfloat16)
    dy = torch.randn(B, T, hidden, generator=gen)
    xg = x.cuda().requires_grad_(True)
    y, _ = m(xg)
    (y.float() * dy.cuda()).sum().backward()
    params = {n: p.detach().float().cpu().clone().requires_grad_(True)
              for n, p in m.named_parameters()}
    xr = x.float().requires_grad_(True)
    taps = {}
    yr = O.cyfa_layer(params, xr, H, hd, hd, taps=taps)
    (yr * dy).sum().backward()
    errs = {"y": rel_l2(y, yr), "x": rel_l2(xg.grad, xr.grad)}
    errs.update({n: rel_l2(p.grad, params[n].grad) for n, p in m.named_parameters()})
    # gate/clock parameters: within 1e-2 x their condition number (the provable
    # bound given per-term parity) and within 4x the shift that the reference's
    # own bf16 storage points produce in the oracle (bf16_points)
    kappa = gate_param_tolerances(taps, xr.detach(), params)
    rparams = {n: p.detach().clone().requires_grad_(True) for n, p in params.items()}
    (O.cyfa_layer(rparams, x.float(), H, hd, hd, bf16_points=True) * dy).sum().backward()
    tols = {n: max(1e-2, min(k, 4.0 * rel_l2(rparams[n].grad, params[n].grad)))
            for n, k in kappa.items()}
    print("layer errors", B, T, hidden, H, hd, {k: round(v, 5) for k, v in errs.items()},
          "gate tolerances", {k: round(v, 4) for k, v in tols.items()})
    for n, e in errs.items():
        assert e < tols.get(n, 1e-2), (n, e)


def test_layer_decode_matches_prefill(Layer):
    B, T, hidden, H, hd = 2, 65, 512, 2, 256
    m = _layer(Layer, hidden, H, hd, seed=4).eval()
    x = torch.randn(B, T, hidden, generator=torch.Generator().manual_seed(2)).to(
        torch.bfloat16).cuda()
    with torch.no_grad():
        full, _ = m(x)
        _, cache = m(x[:, :64], use_cache=True)
        y1, cache = m(x[:, 64:65], cache=cache, use_cache=True)
    assert rel_l2(y1[:, 0], full[:, 64]) < 1e-2


def test_layer_state_dict_roundtrip(Layer, tmp_path):
    m = _layer(Layer, 256, 1, 256, seed=5)
    path = tmp_path / "layer.pt"
    torch.save(m.state_dict(), path)
    m2 = _layer(Layer, 256, 1, 256, seed=6)
    m2.load_state_dict(torch.load(path))
    for (n, a), (_, b) in zip(m.state_dict().items(), m2.state_dict().items()):
        assert torch.equal(a, b), n


def test_sm_target_gemm_precision(Layer):
    """The GEMM path a layer uses beside a running collective (cuBLASLt with an
    SM-count target, fp32 split-K sums) is as precise as the default path: both
    against an fp32 product of the same bf16 operands, at the c3 dx GEMM's
    inner size."""
    from cyclic_flow_attention.ops.layer_ops import _sm_carveout

    gen = torch.Generator().manual_seed(5)
    a = torch.randn(4096, 3336, generator=gen).to(torch.bfloat16).cuda()
    b = (0.02 * torch.randn(3336, 1024, generator=gen)).to(torch.bfloat16).cuda()
    ref = a.float() @ b.float()
    c0 = a @ b
    with _sm_carveout(32):
        c1 = a @ b
    e0, e1 = rel_l2(c0, ref), rel_l2(c1, ref)
    print("bf16 GEMM rel-L2 against fp32: default", e0, "SM target", e1)
    assert e0 < 2.5e-3 and e1 < 2.5e-3
    assert e1 < 1.25 * e0


def test_dx_gemm_sm_target_after_early_handover(Layer):
    """When the early gradient hand-over launches a collective it returns a number
    of SMs; the layer's input-gradient GEMM then runs through cuBLASLt targeting
    that many fewer SMs.  Its input gradient is as close to the fp32 oracle's as
    the default path's, the weight gradients are unchanged (formed before), and
    the BLAS backend, SM target and reduction mode are restored afterwards."""
    hidden, H, hd = 512, 2, 256
    m = _layer(Layer, hidden, H, hd, seed=7)
    gen = torch.Generator().manual_seed(2)
    x = torch.randn(2, 256, hidden, generator=gen).to(torch.bfloat16)
    dy = torch.randn(2, 256, hidden, generator=gen)
    mm = torch.backends.cuda.matmul
    lib0 = torch.backends.cuda.preferred_blas_library()
    carve0 = torch._C._get_sm_carveout_experimental()
    red0 = mm.allow_bf16_reduced_precision_reduction
    seen = []

    def run(ready):
        m.grad_ready = ready
        for p in m.parameters():
            p.grad = None
        xg = x.cuda().requires_grad_(True)
        y, _ = m(xg)
        (y.float() * dy.cuda()).sum().backward()
        torch.cuda.synchronize()
        return xg.grad.clone(), {n: p.grad.clone() for n, p in m.named_parameters()}

    try:
        dx0, g0 = run(None)
        dx1, g1 = run(lambda params, grads: seen.append(len(params)) or 32)
    finally:
        m.grad_ready = None
    assert seen, "the fused backward did not hand its weight gradients over"
    params = {n: p.detach().float().cpu().clone().requires_grad_(True)
              for n, p in m.named_parameters()}
    xr = x.float().requires_grad_(True)
    (O.cyfa_layer(params, xr, H, hd, hd) * dy).sum().backward()
    e0, e1 = rel_l2(dx0, xr.grad), rel_l2(dx1, xr.grad)
    print("dx rel-L2 against the oracle: default", e0, "SM target", e1)
    assert e1 < 1e-2 and e1 < 1.1 * e0 + 1e-4
    for n in g0:
        assert torch.equal(g0[n], g1[n]), n
    assert torch.backends.cuda.preferred_blas_library() == lib0
    assert torch._C._get_sm_carveout_experimental() == carve0
    assert mm.allow_bf16_reduced_precision_reduction == red0
