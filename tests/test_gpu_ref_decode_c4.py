"""The library's decode step against the reference's OWN decode kernel at
BASELINE configs[3]'s shape (batch 256, 8 heads, K = V = 256, bf16 inputs,
fp32 states), one step from a seeded state.

The reference kernel (cyclic_flow_attention/ops/fused_recurrent.py:55-188) is
built for this shape from the reference tree by oracle/ref_build.py into
oracle/_ref/ (test infrastructure; the test is skipped when that build is
absent).  Both kernels get the same inputs and the same fp32 readout table.
Tolerances: outputs (bf16) rel-L2 <= 1e-2, states (fp32) <= 1e-4, at clocks up
to 3000 and up to 1e6.  The test also prints both kernels' device times on this
shape (informational)."""

import ctypes
import os

import pytest
import torch

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "ref_decode_bf16_c4.so")
B, H, K, V = 256, 8, 256, 256


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _time(fn, reps=10):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps * 1000.0  # us


@pytest.mark.parametrize("clock_scale", [3000.0, 1.0e6])
def test_decode_step_matches_reference_kernel_c4(clock_scale):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    if not os.path.exists(REF_SO):
        pytest.skip("reference decode kernel not built (oracle/ref_build.py)")
    from cyclic_flow_attention import _lib
    from cyclic_flow_attention.ops.chunk import readout_table

    gen = torch.Generator().manual_seed(404)
    bf = torch.bfloat16
    q = torch.randn(B, 1, H, K, generator=gen).to(bf).cuda()
    k = torch.randn(B, 1, H, K, generator=gen).to(bf).cuda()
    v = torch.randn(B, 1, H, V, generator=gen).to(bf).cuda()
    g = torch.log(0.9 + 0.1 * torch.rand(B, 1, H, generator=gen)).cuda()
    delta = torch.sigmoid(torch.randn(B, 1, H, generator=gen)).cuda()
    beta = torch.sigmoid(torch.randn(B, 1, H, generator=gen)).cuda()
    readout = (torch.eye(127).expand(H, -1, -1)
               + 0.05 * torch.randn(H, 127, 127, generator=gen)).cuda()
    qw = (1 + 0.1 * torch.randn(K, generator=gen)).cuda()
    kw = (1 + 0.1 * torch.randn(K, generator=gen)).cuda()
    hk = (0.05 * torch.randn(B, H, K, 128, generator=gen)).cuda()
    hv = (0.05 * torch.randn(B, H, 128, V, generator=gen)).cuda()
    # clocks up to 3000 (a long generation) and up to 1e6, where the fp32 clock's
    # fractional part is coarse (ulp 1/16) and the phase rule's integer reduction
    # carries the whole angle
    clock = (clock_scale * torch.rand(B, H, generator=gen)).cuda()
    table = readout_table(readout).contiguous()  # [H, 127, 128] fp32
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    ref = ctypes.CDLL(REF_SO)
    o_r = torch.empty(B, 1, H, V, device="cuda", dtype=bf)
    hk_r, hv_r, clock_r = torch.empty_like(hk), torch.empty_like(hv), torch.empty_like(clock)
    ins = _ptrs([q, k, v, g, delta, beta, table, qw, kw, hk, hv, clock])
    outs = _ptrs([o_r, hk_r, hv_r, clock_r])

    def run_ref():
        rc = ref.ref_decode(ins, outs, stream)
        assert rc == 0

    o_c = torch.empty_like(o_r)
    hk_c, hv_c, clock_c = torch.empty_like(hk), torch.empty_like(hv), torch.empty_like(clock)
    p = _lib.ptr

    def run_cyfa():
        _lib.call("cyfa_decode_step", p(q), p(k), p(v), p(g), p(delta), p(beta), p(table),
                  p(qw), p(kw), p(hk), p(hv), p(clock), p(hk_c), p(hv_c), p(clock_c), p(o_c),
                  B, H, K, V, 0, 1e-6, 1e-6, K ** -0.5, _lib.stream())

    run_ref()
    run_cyfa()
    torch.cuda.synchronize()
    assert rel_l2(o_c, o_r) < 1e-2
    assert rel_l2(hk_c, hk_r) < 1e-4
    assert rel_l2(hv_c, hv_r) < 1e-4
    assert rel_l2(clock_c, clock_r) < 1e-6
    assert _lib.device_error() == 0

    if clock_scale != 3000.0:
        return
    state_bytes = B * H * 2 * (K * 128 + 128 * V) * 4
    t_ref, t_cyfa = _time(run_ref), _time(run_cyfa)
    print(f"\nconfigs[3] decode step, batch {B}, {H} x {K}: reference kernel {t_ref:.1f} us "
          f"({state_bytes / t_ref / 1e3:.0f} GB/s of state traffic), libcyfa {t_cyfa:.1f} us "
          f"({state_bytes / t_cyfa / 1e3:.0f} GB/s); out rel-L2 {rel_l2(o_c, o_r):.2e}, "
          f"hk {rel_l2(hk_c, hk_r):.2e}, hv {rel_l2(hv_c, hv_r):.2e}")
