"""The decode projections' weight-streaming GEMM (cyfa_skinny_gemm) against a
plain fp32 PyTorch product of the same bf16 operands: the shapes of a batched
decode step at configs[3] (hidden 2048, 8 x 256 heads, MLP 5632, vocab 32000,
batch 256 -- K-split with fp32 partials for the narrow outputs), ragged M and
N, and a strided x (a column slice of a packed projection).  bf16 output:
rel-L2 <= 1e-2."""

import pytest
import torch

from gpu_util import rel_l2, seeded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mm():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention.ops.gemm import _fits, decode_mm

    return decode_mm, _fits


@pytest.mark.parametrize("M,N,K", [
    (256, 6424, 2048),   # packed q|k|v|g0|a|b|d projection
    (256, 2048, 256),    # output gate's second linear
    (256, 2048, 2048),   # o_proj (K split)
    (256, 11264, 2048),  # MLP gate|up
    (256, 2048, 5632),   # MLP down (K split)
    (256, 32000, 2048),  # lm_head
    (200, 1000, 320),
    (1, 512, 128),
    (129, 136, 192),
])
def test_skinny_gemm_matches_fp32(mm, M, N, K):
    decode_mm, fits = mm
    gen = seeded(M * 7 + N + K)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (0.02 * torch.randn(N, K, generator=gen)).to(torch.bfloat16).cuda()
    assert fits(x, w)
    y = decode_mm(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    assert rel_l2(y, ref) < 1e-2
    # deterministic: a second call gives the same bits
    assert torch.equal(decode_mm(x, w), y)
    from cyclic_flow_attention import _lib

    assert _lib.device_error() == 0


def test_skinny_gemm_strided_input(mm):
    decode_mm, fits = mm
    gen = seeded(5)
    P = torch.randn(64, 1024, generator=gen).to(torch.bfloat16).cuda()
    x = P[:, 512:768]  # a column slice, rows 1024 elements apart
    w = (0.05 * torch.randn(384, 256, generator=gen)).to(torch.bfloat16).cuda()
    assert fits(x, w)
    y = decode_mm(x, w)
    assert rel_l2(y, x.float() @ w.float().t()) < 1e-2
