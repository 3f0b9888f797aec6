"""GPU checks of the gradient-bucket kernels (cyfa_bucket_gather/_scatter):
bf16 and f32 tensors of ragged sizes, more pieces than one launch takes,
exact fp32 widening on the way in and round-to-nearest on the way out."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bucket_gather_scatter_roundtrip():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib

    gen = torch.Generator().manual_seed(11)
    sizes = [1, 7, 8, 9, 2047, 2048, 2049, 5000, 3, 65536 + 5] * 8  # 80 pieces: two launches
    tensors = []
    for k, n in enumerate(sizes):
        dt = torch.bfloat16 if k % 3 else torch.float32
        tensors.append(torch.randn(n, generator=gen).to(dt).cuda())
    offs, off = [], 0
    for t in tensors:
        offs.append(off)
        off += (t.numel() + 63) // 64 * 64
    flat = torch.full((off,), float("nan"), device="cuda")
    arr = (_lib.BucketPiece * len(tensors))()
    for k, (t, o) in enumerate(zip(tensors, offs)):
        arr[k] = _lib.BucketPiece(t.data_ptr(), t.numel(), o, 0 if t.dtype == torch.float32 else 1)
    _lib.call("cyfa_bucket_gather", arr, len(tensors), _lib.ptr(flat), _lib.stream())
    for t, o in zip(tensors, offs):
        assert torch.equal(flat[o:o + t.numel()], t.float())
    flat.mul_(3.0)
    _lib.call("cyfa_bucket_scatter", arr, len(tensors), _lib.ptr(flat), 0.5, _lib.stream())
    torch.cuda.synchronize()
    for t, o in zip(tensors, offs):
        want = (flat[o:o + t.numel()] * 0.5).to(t.dtype)
        assert torch.equal(t, want)


def test_bucket_rejects_misaligned_offset():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib

    t = torch.ones(16, device="cuda")
    flat = torch.zeros(64, device="cuda")
    arr = (_lib.BucketPiece * 1)(_lib.BucketPiece(t.data_ptr(), 16, 4, 0))
    with pytest.raises(_lib.CyfaError):
        _lib.call("cyfa_bucket_gather", arr, 1, _lib.ptr(flat), _lib.stream())
