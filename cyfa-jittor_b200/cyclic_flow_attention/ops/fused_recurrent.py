"""Constant-state autoregressive CyFA decoding on B200.

Drop-in for the reference's ``fused_recurrent_cyfa``
(cyclic_flow_attention/ops/fused_recurrent.py:10-200): same signature, return
convention and errors; the step runs in libcyfa.so (cyfa_decode_step).
"""

import torch

from .. import _lib
from .chunk import readout_table


def fused_recurrent_cyfa(
    q,
    k,
    v,
    g,
    delta,
    beta,
    readout,
    q_norm_weight,
    k_norm_weight,
    q_norm_eps=1e-6,
    k_norm_eps=1e-6,
    scale=None,
    initial_state=None,
    output_final_state=False,
    cu_seqlens=None,
    inplace=False,
):
    """Decode one token using constant-size key, value and clock states.

    Uses the same input layout and return convention as chunk_cyfa.  This path
    is inference-only and needs one token per sequence.  With ``inplace=True``
    the new states overwrite ``initial_state`` (same bytes, no allocation).
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    M = readout.shape[-1] + 1
    tracked = (q, k, v, g, delta, beta, readout, q_norm_weight, k_norm_weight)
    if initial_state is not None:
        tracked = tracked + tuple(initial_state)
    if torch.is_grad_enabled() and any(x.requires_grad for x in tracked):
        raise ValueError(
            "fused_recurrent_cyfa is inference-only; use torch.no_grad() or chunk_cyfa for gradients"
        )
    if T != 1 or cu_seqlens is not None:
        raise NotImplementedError("native fused decode currently needs dense T=1")
    if M > 256 or K > 1024 or V > 1024:
        raise ValueError("decode shape exceeds block limits")
    if M != 128 or K not in (128, 256) or V not in (128, 256):
        raise ValueError("the B200 decode kernel needs 128 slots and head dims 128 or 256")
    _lib.require_cuda(*tracked)
    dev = q.device
    dtype = q.dtype
    if dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"unsupported dtype {dtype}")
    code = 0 if dtype == torch.bfloat16 else 1
    q, k, v = (x.to(dtype).contiguous() for x in (q, k, v))
    g, delta, beta = (x.float().contiguous() for x in (g, delta, beta))
    table = readout_table(readout).contiguous()
    sc = K ** -0.5 if scale is None else float(scale)
    if initial_state is None:
        hk_in = hv_in = clock_in = None
    else:
        hk_in, hv_in, clock_in = (x.float().contiguous() for x in initial_state)
    if inplace and initial_state is not None:
        hk_out, hv_out, clock_out = hk_in, hv_in, clock_in
    else:
        hk_out = torch.empty(B, H, K, M, device=dev, dtype=torch.float32)
        hv_out = torch.empty(B, H, M, V, device=dev, dtype=torch.float32)
        clock_out = torch.empty(B, H, device=dev, dtype=torch.float32)
    out = torch.empty(B, 1, H, V, device=dev, dtype=dtype)
    P = _lib.ptr
    _lib.call("cyfa_decode_step", P(q), P(k), P(v), P(g), P(delta), P(beta), P(table),
              P(q_norm_weight.float().contiguous()), P(k_norm_weight.float().contiguous()),
              P(hk_in), P(hv_in), P(clock_in), P(hk_out), P(hv_out), P(clock_out), P(out),
              B, H, K, V, code, float(q_norm_eps), float(k_norm_eps), sc, _lib.stream())
    return out, ((hk_out, hv_out, clock_out) if output_final_state else None)
