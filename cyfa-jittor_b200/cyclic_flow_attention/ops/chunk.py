"""Chunkwise Cyclic Flow Attention on B200 (sm_100a).

Drop-in for the reference's ``chunk_cyfa`` (cyclic_flow_attention/ops/chunk.py:164-353):
same signature, layouts, defaults and errors.  The whole op (gates, clock,
q/k RMSNorm, write vector, both ScalarGatedLA passes and the softmax slot
readout, forward and backward) runs in libcyfa.so; torch only allocates
buffers, builds the readout table R.Phi and differentiates through it.
"""

import ctypes
import math

import torch

from .. import _lib

_c = ctypes


class _FwdArgs(_c.Structure):
    _fields_ = [(n, _c.c_int) for n in ("B", "T", "H", "K", "V")] + \
        [(n, _c.c_float) for n in ("q_eps", "k_eps", "scale")] + \
        [(n, _c.c_void_p) for n in ("q", "k", "v", "g", "delta", "beta", "q_norm_weight",
                                     "k_norm_weight", "table_bf", "hk0", "hv0", "clock0",
                                     "o", "hk", "hv", "clock")] + \
        [(n, _c.c_longlong) for n in ("q_stride", "k_stride", "v_stride")] + \
        [("lengths", _c.c_void_p)]


class _BwdArgs(_c.Structure):
    _fields_ = [("fwd", _FwdArgs)] + \
        [(n, _c.c_void_p) for n in ("d_o", "dhk", "dhv", "dclock", "dq", "dk", "dv", "dg",
                                     "ddelta", "dbeta", "dtable", "dq_norm_weight",
                                     "dk_norm_weight", "dhk0", "dhv0", "dclock0")] + \
        [(n, _c.c_longlong) for n in ("dq_stride", "dk_stride", "dv_stride")] + \
        [(n, _c.c_void_p) for n in ("readout_basis_t", "dreadout")]


_BASIS = {}


def basis(M, device):
    """Real Fourier basis Phi [M-1, M] (reference ops/chunk.py:82-103), built once
    per device in fp64 and kept in fp32."""
    key = (M, str(device))
    if key not in _BASIS:
        period = M - 1
        row = torch.arange(period, dtype=torch.float64, device=device).unsqueeze(1)
        col = torch.arange(M, device=device)
        pair = (col // 2).to(torch.float64)
        phase = row * (pair * (2 * math.pi / period)).unsqueeze(0)
        z = torch.where((col % 2 == 1).unsqueeze(0), torch.sin(phase), torch.cos(phase))
        scale = torch.full((M,), (2.0 / period) ** 0.5, dtype=torch.float64, device=device)
        scale[:2] = period ** -0.5
        out = z * scale
        out[:, 1] = 0.0
        _BASIS[key] = out.float()
    return _BASIS[key]


_BASIS_T = {}


def basis_t(M, device):
    """Phi^T [M, M-1] fp32 (contiguous), for the readout gradient kernel."""
    key = (M, str(device))
    if key not in _BASIS_T:
        _BASIS_T[key] = basis(M, device).t().contiguous()
    return _BASIS_T[key]


def readout_table(readout):
    """Table_h = R_h . Phi in fp32, [H, M-1, M] (reference ops/chunk.py:281)."""
    M = readout.shape[-1] + 1
    return readout.float() @ basis(M, readout.device)


def table_bf16(readout, out=None):
    """The readout table in the kernels' layout: bf16 [H, 128, 128], Table_h =
    R_h . Phi rounded once, last row zero (one libcyfa launch, into `out` if
    given)."""
    H = readout.shape[0]
    r = readout.detach().to(torch.float32).contiguous()
    tb = torch.empty(H, 128, 128, device=readout.device, dtype=torch.bfloat16) if out is None \
        else out
    _lib.call("cyfa_readout_table", _p(r), _p(basis(128, readout.device)), _p(tb), H,
              _lib.stream())
    return tb


def readout_grad(dtable, readout):
    """Gradient of the readout from the kernels' table gradient dtable [H,128,128]
    fp32 (one libcyfa launch); returned in the readout's dtype."""
    H = dtable.shape[0]
    dr = torch.empty(H, 127, 127, device=dtable.device, dtype=torch.float32)
    _lib.call("cyfa_readout_table_grad", _p(dtable), _p(basis_t(128, dtable.device)), _p(dr),
              H, _lib.stream())
    return dr if readout.dtype == torch.float32 else dr.to(readout.dtype)


def _contig(x, dtype):
    return x.to(dtype).contiguous()


def _p(t):
    return None if t is None else t.data_ptr()


class ChunkCyfaFunction(torch.autograd.Function):
    """Autograd wrapper over cyfa_chunk_fwd / cyfa_chunk_bwd."""

    @staticmethod
    def forward(ctx, q, k, v, g, delta, beta, readout, qw, kw, hk0, hv0, clock0,
                q_eps, k_eps, scale):
        ctx.set_materialize_grads(False)  # the final states usually get no gradient
        B, T, H, K = q.shape
        V = v.shape[-1]
        dev = q.device
        tb = table_bf16(readout)
        o = torch.empty(B, T, H, V, device=dev, dtype=torch.bfloat16)
        hk = torch.empty(B, H, K, 128, device=dev, dtype=torch.float32)
        hv = torch.empty(B, H, 128, V, device=dev, dtype=torch.float32)
        clock = torch.empty(B, H, device=dev, dtype=torch.float32)
        nbytes = _lib.lib().cyfa_chunk_saved_bytes(B, T, H, K, V)
        if nbytes == 0:
            raise ValueError(f"unsupported chunk_cyfa shape B={B} T={T} H={H} K={K} V={V}")
        saved = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        args = _FwdArgs(B, T, H, K, V, q_eps, k_eps, scale,
                        _p(q), _p(k), _p(v), _p(g), _p(delta), _p(beta), _p(qw), _p(kw),
                        _p(tb), _p(hk0), _p(hv0), _p(clock0), _p(o), _p(hk), _p(hv), _p(clock))
        _lib.call("cyfa_chunk_fwd", _c.byref(args), _lib.ptr(saved), _c.c_size_t(nbytes),
                  _lib.stream())
        ctx.save_for_backward(q, k, v, g, delta, beta, qw, kw, tb, hk0, hv0, clock0,
                              hk, hv, clock, saved)
        ctx.readout_meta = readout.detach()[:0]  # dtype and device of the readout
        ctx.eps = (q_eps, k_eps, scale)
        ctx.has_init = (hk0 is not None, hv0 is not None, clock0 is not None)
        return o, hk, hv, clock

    @staticmethod
    def backward(ctx, do, dhk, dhv, dclock):
        (q, k, v, g, delta, beta, qw, kw, tb, hk0, hv0, clock0, hk, hv, clock,
         saved) = ctx.saved_tensors
        B, T, H, K = q.shape
        V = v.shape[-1]
        dev = q.device
        q_eps, k_eps, scale = ctx.eps
        fwd = _FwdArgs(B, T, H, K, V, q_eps, k_eps, scale,
                       _p(q), _p(k), _p(v), _p(g), _p(delta), _p(beta), _p(qw), _p(kw),
                       _p(tb), _p(hk0), _p(hv0), _p(clock0), None, _p(hk), _p(hv), _p(clock))
        do = torch.zeros(B, T, H, V, device=dev, dtype=torch.bfloat16) if do is None \
            else _contig(do, torch.bfloat16)
        dhk = None if dhk is None else _contig(dhk, torch.float32)
        dhv = None if dhv is None else _contig(dhv, torch.float32)
        dclock = None if dclock is None else _contig(dclock, torch.float32)
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        dg = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        ddelta = torch.empty_like(dg)
        dbeta = torch.empty_like(dg)
        dtable = torch.empty(H, 128, 128, device=dev, dtype=torch.float32)
        dqw = torch.empty(K, device=dev, dtype=torch.float32)
        dkw = torch.empty(K, device=dev, dtype=torch.float32)
        dhk0 = torch.empty(B, H, K, 128, device=dev, dtype=torch.float32)
        dhv0 = torch.empty(B, H, 128, V, device=dev, dtype=torch.float32)
        dclock0 = torch.empty(B, H, device=dev, dtype=torch.float32)
        nwork = _lib.lib().cyfa_chunk_work_bytes(B, T, H, K, V)
        work = torch.empty(nwork, device=dev, dtype=torch.uint8)
        args = _BwdArgs(fwd, _p(do), _p(dhk), _p(dhv), _p(dclock), _p(dq), _p(dk), _p(dv),
                        _p(dg), _p(ddelta), _p(dbeta), _p(dtable), _p(dqw), _p(dkw),
                        _p(dhk0), _p(dhv0), _p(dclock0))
        _lib.call("cyfa_chunk_bwd", _c.byref(args), _lib.ptr(saved),
                  _c.c_size_t(saved.numel()), _lib.ptr(work), _c.c_size_t(nwork),
                  _lib.stream())
        has_hk0, has_hv0, has_c0 = ctx.has_init
        dreadout = readout_grad(dtable, ctx.readout_meta) if ctx.needs_input_grad[6] else None
        return (dq, dk, dv, dg, ddelta, dbeta, dreadout, dqw, dkw,
                dhk0 if has_hk0 else None, dhv0 if has_hv0 else None,
                dclock0 if has_c0 else None, None, None, None)


def _chunk_cyfa_f32(q, k, v, g, delta, beta, readout, qw, kw, q_eps, k_eps, scale, hk0, hv0,
                    clock0, output_final_state):
    """fp32 inputs: the reference computes these in fp32 throughout (its generic
    path, ops/chunk.py:136-161,300-331), so they run on cyfa_chunk_fwd_f32, an
    fp32 token recurrence, instead of the bf16 tensor-core kernels.  Inference
    only: the fp32 training path is not built, so tracked gradients raise."""
    tracked = (q, k, v, g, delta, beta, readout, qw, kw, hk0, hv0, clock0)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tracked):
        raise NotImplementedError(
            "chunk_cyfa: fp32 inputs run the fp32 inference path, which has no backward; "
            "pass bfloat16 q/k/v for training, or call under torch.no_grad()")
    B, T, H, K = q.shape
    V = v.shape[-1]
    dev = q.device
    f32 = torch.float32
    o = torch.empty(B, T, H, V, device=dev, dtype=f32)
    hk = torch.empty(B, H, K, 128, device=dev, dtype=f32)
    hv = torch.empty(B, H, 128, V, device=dev, dtype=f32)
    clock = torch.empty(B, H, device=dev, dtype=f32)
    with torch.no_grad():
        table = readout_table(readout.detach()).contiguous()
        ins = [_contig(t.detach(), f32) for t in (q, k, v, g, delta, beta)]
        qn, kn = (_contig(t.detach(), f32) for t in (qw, kw))
        _lib.call("cyfa_chunk_fwd_f32", *[_p(t) for t in ins], _p(table), _p(qn), _p(kn),
                  _p(hk0), _p(hv0), _p(clock0), _p(o), _p(hk), _p(hv), _p(clock),
                  B, T, H, K, V, float(q_eps), float(k_eps), float(scale), _lib.stream())
    return o, ((hk, hv, clock) if output_final_state else None)


def chunk_cyfa(
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
    checkpoint_level=0,
    chunk_size=64,
):
    """Chunkwise Cyclic Flow Attention.

    Inputs q and k use [batch, time, heads, K], v [batch, time, heads, V]; g,
    delta and beta use [batch, time, heads]. The readout has [heads, slots-1,
    slots-1].  Returns the output [batch, time, heads, V] and, when requested,
    the fp32 state (key_state [B,H,K,slots], value_state [B,H,slots,V],
    clock [B,H]).  Same contract as the reference (ops/chunk.py:164-189); the
    tensors must live on a CUDA device.  ``chunk_size`` keeps its meaning for
    padding semantics; the kernels tile time in blocks of 128 tokens, which
    gives the same result (the chunk size is a scheduling choice).

    bf16 q/k/v run the tcgen05 kernels (bf16 operands, fp32 accumulation) with
    gradients.  fp32 q/k/v run in fp32 throughout (``cyfa_chunk_fwd_f32``),
    inference only: with tracked gradients they raise NotImplementedError.
    """
    if cu_seqlens is not None:
        raise NotImplementedError("packed layout requires native segment dispatch")
    if checkpoint_level != 0:
        raise NotImplementedError("only saved-activation training is implemented")
    _lib.require_cuda(q, k, v, g, delta, beta, readout, q_norm_weight, k_norm_weight)
    B, T, H, K = q.shape
    V = v.shape[-1]
    M = readout.shape[-1] + 1
    if M != 128:
        raise ValueError("the B200 kernels need num_slots = 128 (127 active slots)")
    if K not in (128, 256) or V not in (128, 256):
        raise ValueError(f"head dims must be 128 or 256, got K={K} V={V}")
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    sc = K ** -0.5 if scale is None else float(scale)
    hk0 = hv0 = clock0 = None
    if initial_state is not None:
        hk0, hv0, clock0 = (_contig(x, torch.float32) for x in initial_state)
    if q.dtype == torch.float32:
        return _chunk_cyfa_f32(q, k, v, g, delta, beta, readout, q_norm_weight, k_norm_weight,
                               q_norm_eps, k_norm_eps, sc, hk0, hv0, clock0, output_final_state)
    if q.dtype != torch.bfloat16:
        raise ValueError(f"q/k/v must be bfloat16 or float32, got {q.dtype}")
    out_dtype = q.dtype
    o, hk, hv, clock = ChunkCyfaFunction.apply(
        _contig(q, torch.bfloat16), _contig(k, torch.bfloat16), _contig(v, torch.bfloat16),
        _contig(g, torch.float32), _contig(delta, torch.float32), _contig(beta, torch.float32),
        readout, _contig(q_norm_weight, torch.float32), _contig(k_norm_weight, torch.float32),
        hk0, hv0, clock0, float(q_norm_eps), float(k_norm_eps), sc)
    if out_dtype != torch.bfloat16:
        o = o.to(out_dtype)
    state = (hk, hv, clock) if output_final_state else None
    return o, state
