"""Projections of a batched decode step on libcyfa's weight-streaming GEMM.

``decode_mm(x, w)`` is ``x @ w.T`` for an nn.Linear weight ``w`` [N, K] and a
few bf16 rows ``x`` [M, K] (M <= 256: one row per sequence of the decode
batch).  At that M the product sits at the B200's FLOP/byte ridge, so it should
run at the HBM rate of the weights; ``cyfa_skinny_gemm`` streams each weight
from HBM once by TMA into tcgen05 MMAs.  Larger M (prefill) is an ordinary
library GEMM and goes to torch.
"""

import ctypes

import torch

from .. import _lib


def _fits(x, w):
    M, K = x.shape
    N = w.shape[0]
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and 0 < M <= 256 and K % 64 == 0 and N % 8 == 0 and w.shape[1] == K
            and x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0
            and w.is_contiguous() and w.data_ptr() % 16 == 0)


def decode_mm(x, w, out=None):
    """x [M, K] @ w[N, K]^T -> [M, N] bf16 (into `out` when given)."""
    if not _fits(x, w):
        return torch.mm(x, w.t(), out=out) if out is not None else torch.mm(x, w.t())
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16) if out is None else out
    nwork = _lib.lib().cyfa_skinny_gemm_work_bytes(M, N, K)
    work = torch.empty(max(nwork, 16), device=x.device, dtype=torch.uint8) if nwork else None
    _lib.call("cyfa_skinny_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w), _lib.ptr(y), y.stride(0),
              M, N, K, _lib.ptr(work), ctypes.c_size_t(nwork), _lib.stream())
    return y
