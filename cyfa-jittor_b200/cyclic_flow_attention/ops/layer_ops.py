"""Autograd wrappers of the layer glue kernels and of the chunk op on a packed
q|k|v projection, used by the layer's fused training/prefill path.

All compute runs in libcyfa.so; these wrappers allocate outputs and work
buffers and pass raw pointers.
"""

import contextlib
import ctypes

import torch

from .. import _lib
from .chunk import _BwdArgs, _FwdArgs, _p, basis_t, readout_grad, table_bf16


@contextlib.contextmanager
def _sm_carveout(n):
    """GEMMs issued inside run through cuBLASLt targeting n fewer SMs than the
    device has (CUBLASLT_MATMUL_DESC_SM_COUNT_TARGET), so that a collective
    already running beside them keeps its SMs instead of waiting for the GEMM
    to finish (n = 0: no change).  Split-K partial sums stay in fp32 (no bf16
    reduction), so the result is as precise as the default path's."""
    if not n:
        yield
        return
    mm = torch.backends.cuda.matmul
    prev = torch._C._get_sm_carveout_experimental()
    prev_lib = torch.backends.cuda.preferred_blas_library()
    prev_red = mm.allow_bf16_reduced_precision_reduction
    torch._C._set_sm_carveout_experimental(int(n))
    torch.backends.cuda.preferred_blas_library("cublaslt")
    mm.allow_bf16_reduced_precision_reduction = False
    try:
        yield
    finally:
        mm.allow_bf16_reduced_precision_reduction = prev_red
        torch.backends.cuda.preferred_blas_library(prev_lib)
        torch._C._set_sm_carveout_experimental(prev)

_c = ctypes


def _work(nbytes, dev):
    return torch.empty(max(int(nbytes), 1), device=dev, dtype=torch.uint8)


def _fits_pieces(tensors):
    """True if every tensor can be a libcyfa bucket piece (CUDA, f32 or bf16,
    contiguous, 16-byte aligned)."""
    return all(t.is_cuda and t.dtype in (torch.float32, torch.bfloat16) and t.is_contiguous()
               and t.data_ptr() % 16 == 0 for t in tensors)


def _pieces(tensors, offs):
    arr = (_lib.BucketPiece * len(tensors))()
    for k, (t, o) in enumerate(zip(tensors, offs)):
        arr[k] = _lib.BucketPiece(t.data_ptr(), t.numel(), o,
                                  0 if t.dtype == torch.float32 else 1)
    return arr


def flat_f32(sizes, device):
    """One fp32 buffer holding consecutive pieces of the given sizes, each
    starting at a multiple of 8 elements; returns (buffer, offsets)."""
    offs, total = [], 0
    for n in sizes:
        offs.append(total)
        total += (n + 7) // 8 * 8
    return torch.empty(max(total, 8), device=device, dtype=torch.float32), offs


def gather_f32(tensors, stream=None):
    """The tensors as fp32 views of one buffer, filled by one libcyfa launch
    (the per-step conversion of the small parameters).  The buffer belongs to
    the current stream; the launch goes to `stream` if given (the caller then
    makes the current stream wait for it before the views are read)."""
    tensors = [t.detach() for t in tensors]
    flat, offs = flat_f32([t.numel() for t in tensors], tensors[0].device)
    if not _fits_pieces(tensors):
        return [t.float().contiguous() for t in tensors]
    with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
        _lib.call("cyfa_bucket_gather", _pieces(tensors, offs), len(tensors), _p(flat),
                  _lib.stream())
    return [flat[o:o + t.numel()].view(t.shape) for t, o in zip(tensors, offs)]


def scatter_from(flat, offs, like, stream=None):
    """Gradients held in fp32 at flat[offs[i]:] converted to the dtype and shape
    of like[i] by one libcyfa launch (on `stream` if given; the outputs belong to
    the current stream); fp32 targets are views of `flat`."""
    outs, pieces, poffs = [], [], []
    for o, t in zip(offs, like):
        if t.dtype == torch.float32:
            outs.append(flat[o:o + t.numel()].view(t.shape))
        else:
            outs.append(torch.empty(t.shape, device=flat.device, dtype=t.dtype))
            pieces.append(outs[-1])
            poffs.append(o)
    if pieces and _fits_pieces(pieces):
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
            _lib.call("cyfa_bucket_scatter", _pieces(pieces, poffs), len(pieces), _p(flat),
                      _c.c_float(1.0), _lib.stream())
    elif pieces:
        if stream is not None:
            torch.cuda.current_stream().wait_stream(stream)
        for i, (o, t) in enumerate(zip(offs, like)):
            if t.dtype != torch.float32:
                outs[i] = flat[o:o + t.numel()].view(t.shape).to(t.dtype)
    return outs


class ShortConvFunction(torch.autograd.Function):
    """Causal depthwise conv (no activation) of x [B,T,C] bf16 with weight [C,1,W]."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        B, T, C = x.shape
        W = weight.shape[-1]
        w = weight.detach().float().reshape(C, W).contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        y = torch.empty(B, T, C, device=x.device, dtype=torch.bfloat16)
        _lib.call("cyfa_short_conv_fwd", _p(x), _c.c_longlong(x.stride(1)), None, _p(w), _p(b),
                  _p(y), B, T, C, W, _lib.stream())
        ctx.save_for_backward(x, w)
        ctx.meta = (W, weight.dtype, bias is not None, None if bias is None else bias.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        W, wdt, has_bias, bdt = ctx.meta
        B, T, C = x.shape
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty(B, T, C, device=x.device, dtype=torch.bfloat16)
        dw = torch.empty(C, W, device=x.device, dtype=torch.float32)
        db = torch.empty(C, device=x.device, dtype=torch.float32) if has_bias else None
        nbytes = _lib.lib().cyfa_short_conv_work_bytes(B, T, C, W)
        work = _work(nbytes, x.device)
        _lib.call("cyfa_short_conv_bwd", _p(x), _c.c_longlong(x.stride(1)), _p(w), _p(dy), _p(dx),
                  _c.c_longlong(C), _p(dw), _p(db), B, T, C, W, _p(work), _c.c_size_t(nbytes),
                  _lib.stream())
        return dx, dw.reshape(C, 1, W).to(wdt), None if db is None else db.to(bdt)


class GateActFunction(torch.autograd.Function):
    """(g, delta, beta) from the packed auxiliary projection `aux` (a at column
    a_col, b at b_col, H columns each; no bias) and the d projection `dlin`
    [B,T,H] (no bias); the b and d biases are applied here so their gradients
    come from the kernel's fixed-order partial sums."""

    @staticmethod
    def forward(ctx, aux, dlin, A_log, dt_bias, b_bias, d_bias, a_col, b_col, H):
        B, T, _ = aux.shape
        rows = B * T
        dev = aux.device
        A = A_log.detach().float().contiguous()
        dt = dt_bias.detach().float().contiguous()
        bb = b_bias.detach().float().contiguous()
        db = d_bias.detach().float().contiguous()
        g = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        delta = torch.empty_like(g)
        beta = torch.empty_like(g)
        st = _c.c_longlong(aux.stride(1))
        _lib.call("cyfa_gate_act_fwd", _c.c_void_p(aux.data_ptr() + 2 * a_col), st,
                  _c.c_void_p(aux.data_ptr() + 2 * b_col), st, _p(dlin),
                  _c.c_longlong(dlin.stride(1)), _p(A), _p(dt), _p(bb), _p(db), _p(g),
                  _p(delta), _p(beta), rows, H, _lib.stream())
        ctx.save_for_backward(aux, dlin, A, dt, bb, db)
        ctx.meta = (a_col, b_col, H, A_log.dtype, dt_bias.dtype, b_bias.dtype, d_bias.dtype)
        return g, delta, beta

    @staticmethod
    def backward(ctx, dg, ddelta, dbeta):
        aux, dlin, A, dt, bb, db_ = ctx.saved_tensors
        a_col, b_col, H, adt, ddt, bdt, dbt = ctx.meta
        B, T, width = aux.shape
        rows = B * T
        dev = aux.device
        zeros = lambda: torch.zeros(B, T, H, device=dev, dtype=torch.float32)
        dg = zeros() if dg is None else dg.float().contiguous()
        ddelta = zeros() if ddelta is None else ddelta.float().contiguous()
        dbeta = zeros() if dbeta is None else dbeta.float().contiguous()
        daux = torch.zeros(B, T, width, device=dev, dtype=torch.bfloat16)
        dd = torch.empty(B, T, H, device=dev, dtype=torch.bfloat16)
        dA = torch.empty(H, device=dev, dtype=torch.float32)
        ddtb = torch.empty(H, device=dev, dtype=torch.float32)
        dbb = torch.empty(H, device=dev, dtype=torch.float32)
        ddb = torch.empty(H, device=dev, dtype=torch.float32)
        nbytes = _lib.lib().cyfa_gate_act_work_bytes(rows, H)
        work = _work(nbytes, dev)
        st = _c.c_longlong(aux.stride(1))
        _lib.call("cyfa_gate_act_bwd", _c.c_void_p(aux.data_ptr() + 2 * a_col), st,
                  _c.c_void_p(aux.data_ptr() + 2 * b_col), st, _p(dlin),
                  _c.c_longlong(dlin.stride(1)), _p(A), _p(dt), _p(bb), _p(db_), _p(dg),
                  _p(ddelta), _p(dbeta), _c.c_void_p(daux.data_ptr() + 2 * a_col),
                  _c.c_longlong(width), _c.c_void_p(daux.data_ptr() + 2 * b_col),
                  _c.c_longlong(width), _p(dd), _c.c_longlong(H), _p(dA), _p(ddtb), _p(dbb),
                  _p(ddb), rows, H, _p(work), _c.c_size_t(nbytes), _lib.stream())
        return (daux, dd, dA.to(adt), ddtb.to(ddt), dbb.to(bdt), ddb.to(dbt), None, None, None)


def _gate_rows_stride(gate_in, gate_w, D):
    """Row stride (elements) of gate_in [B,T,Kg] when the fused gate + norm
    kernel can read it (bf16, unit column stride, tokens uniformly strided,
    16-byte aligned rows, Kg a multiple of 64), else None."""
    if (gate_in.dtype != torch.bfloat16 or gate_w.dtype != torch.bfloat16 or gate_in.dim() != 3
            or D not in (128, 256) or gate_in.shape[-1] % 64 or not gate_w.is_contiguous()):
        return None
    B, T, Kg = gate_in.shape
    s0, s1, s2 = gate_in.stride()
    if s2 != 1 or (B > 1 and s0 != T * s1) or s1 < Kg or s1 % 8 or gate_in.data_ptr() % 16:
        return None
    return s1


def gated_norm_infer(x, gate_in, gate_w, gate_b, weight, eps, scale):
    """GatedNormFunction's forward without autograd (inference): the gate's
    second linear runs inside the norm kernel (cyfa_gated_norm_gate_fwd: tcgen05
    per 128-token tile and head, the gate rounded to bf16 as a bf16 linear's
    output is), so the gate never goes to memory.  Returns None for inputs the
    kernel does not take (the caller then uses GatedNormFunction)."""
    B, T, H, D = x.shape
    stride = _gate_rows_stride(gate_in, gate_w, D)
    if stride is None or x.dtype != torch.bfloat16 or not x.is_contiguous():
        return None
    w = weight.detach().float().contiguous()
    b = None if gate_b is None else gate_b.detach().to(torch.bfloat16).contiguous()
    y = torch.empty(B, T, H * D, device=x.device, dtype=torch.bfloat16)
    rstd = torch.empty(B * T * H, device=x.device, dtype=torch.float32)
    _lib.call("cyfa_gated_norm_gate_fwd", _p(x), _p(gate_in), _c.c_longlong(stride),
              _p(gate_w.detach()), _p(b), H, gate_in.shape[-1], _p(w), float(eps), float(scale),
              _p(y), _p(rstd), None, B * T, D, _lib.stream())
    return y


class GatedNormFunction(torch.autograd.Function):
    """y = RMSNorm(scale * x) * w * sigmoid(gate) over the last dim D of
    x [B,T,H,D], with gate = gate_in @ W^T + b (the output gate's second linear,
    [B,T,H*D]); returns [B,T,H*D] bf16.  The linear runs on cuBLAS without its
    bias and the gate is kept for the backward (writing it from the fused
    kernel of gated_norm_infer measured slower than the separate linear); the
    kernels add b and return its gradient (fixed-order sums)."""

    @staticmethod
    def forward(ctx, x, gate_in, gate_w, gate_b, weight, eps, scale, slot=None, gate_param=None):
        B, T, H, D = x.shape
        rows = B * T * H
        x = x.to(torch.bfloat16).contiguous()
        w = weight.detach().float().contiguous()
        y = torch.empty(B, T, H * D, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        b = None
        if gate_b is not None:
            b = gate_b.detach().to(torch.bfloat16).contiguous()
        gate = torch.nn.functional.linear(gate_in, gate_w).contiguous()
        if b is not None:
            _lib.call("cyfa_gated_norm_bias_fwd", _p(x), _p(gate), _p(b), H, _p(w), float(eps),
                      float(scale), _p(y), _p(rstd), rows, D, _lib.stream())
        else:
            _lib.call("cyfa_gated_norm_fwd", _p(x), _p(gate), _p(w), float(eps), float(scale),
                      _p(y), _p(rstd), rows, D, _lib.stream())
        ctx.save_for_backward(x, gate, gate_in, gate_w, w, rstd, b)
        ctx.meta = (scale, weight.dtype, None if gate_b is None else gate_b.dtype)
        ctx.slot = slot
        # (the Parameter behind gate_w,) as a plain object, for a deferred gradient
        ctx.gate_param = gate_param[0] if gate_param else None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gate, gate_in, gate_w, w, rstd, b = ctx.saved_tensors
        scale, wdt, bdt = ctx.meta
        B, T, H, D = x.shape
        rows = B * T * H
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x)
        dgate = torch.empty_like(gate)
        dw = torch.empty(D, device=x.device, dtype=torch.float32)
        d_gate_b = None
        if b is not None:
            db = torch.empty(H * D, device=x.device, dtype=torch.float32)
            nbytes = _lib.lib().cyfa_gated_norm_bias_work_bytes(rows, D, H)
            work = _work(nbytes, x.device)
            with _lib.deferred(_aux_stream(x.device)):
                _lib.call("cyfa_gated_norm_bias_bwd", _p(x), _p(gate), _p(b), H, _p(w),
                          float(scale), _p(rstd), _p(dy), _p(dx), _p(dgate), _p(dw), _p(db), rows,
                          D, _p(work), _c.c_size_t(nbytes), _lib.stream())
        else:
            nbytes = _lib.lib().cyfa_gated_norm_work_bytes(rows, D)
            work = _work(nbytes, x.device)
            with _lib.deferred(_aux_stream(x.device)):
                _lib.call("cyfa_gated_norm_bwd", _p(x), _p(gate), _p(w), float(scale), _p(rstd),
                          _p(dy), _p(dx), _p(dgate), _p(dw), rows, D, _p(work),
                          _c.c_size_t(nbytes), _lib.stream())
        dg2 = dgate.reshape(-1, H * D)
        gin2 = gate_in.reshape(-1, gate_in.shape[-1])
        slot = ctx.slot
        d_gate_w = None
        if slot is not None and ctx.gate_param is not None:
            d_gate_w = slot.defer_wgrad(ctx.gate_param, dg2, gin2)
        if d_gate_w is None:
            d_gate_w = dg2.t() @ gin2
        if slot is not None:
            # the producer of gate_in collects its gradient in a packed buffer:
            # write this part there directly and pass no separate gradient
            view = slot.claim(gate_in.device)
            torch.matmul(dg2, gate_w, out=view.reshape(-1, view.shape[-1]))
            d_gate_in = None
        else:
            d_gate_in = (dg2 @ gate_w).reshape(gate_in.shape)
        _join(x.device)  # the norm-weight (and gate-bias) sums ran on the aux stream
        if b is not None:
            d_gate_b = db.to(bdt)
        return dx, d_gate_in, d_gate_w, d_gate_b, dw.to(wdt), None, None, None, None


_SIDE = {}
_AUX = {}


def _side_stream(device):
    """Stream of the deferred weight-gradient GEMMs (joined in the front's backward)."""
    key = str(device)
    if key not in _SIDE:
        _SIDE[key] = torch.cuda.Stream(device=device)
    return _SIDE[key]


def _aux_stream(device):
    """Stream of the small parameter kernels (parameter conversions, the readout
    table, parameter-gradient reductions), each joined by the Function that
    forks it."""
    key = str(device)
    if key not in _AUX:
        _AUX[key] = torch.cuda.Stream(device=device)
    return _AUX[key]


def _fork(device):
    """The aux stream, ordered after the work issued so far on the current stream."""
    aux = _aux_stream(device)
    aux.wait_stream(torch.cuda.current_stream(device))
    return aux


def _join(device):
    torch.cuda.current_stream(device).wait_stream(_aux_stream(device))


class LinearFunction(torch.autograd.Function):
    """y = x W^T (no bias) whose weight gradient may be deferred to the layer's
    side stream through a PackedGradSlot (the layer's o_proj)."""

    @staticmethod
    def forward(ctx, x, weight, param, slot):
        # param: (the Parameter behind weight,), passed as a plain object
        ctx.save_for_backward(x, weight)
        ctx.param, ctx.slot = param[0], slot
        return torch.nn.functional.linear(x, weight)

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        dx = dy @ weight if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
            dw = ctx.slot.defer_wgrad(ctx.param, dy2, x2) if ctx.slot is not None else None
            if dw is None:
                dw = dy2.t() @ x2
        return dx, dw, None, None


class PackedGradSlot:
    """Hand-over of a packed gradient buffer between two autograd Functions.

    LayerFrontFunction returns the output-gate input as a column view of its
    packed projection; its consumer (GatedNormFunction, whose backward runs
    first) writes that gradient straight into the matching columns of a packed
    gradient buffer of the projection's layout instead of returning a separate
    tensor, and LayerFrontFunction's backward picks the buffer up.  This saves a
    strided copy of the gradient per step.  Without a consumer backward the buffer
    is allocated (and those columns zeroed) by LayerFrontFunction itself."""

    def __init__(self):
        self.shape = None  # (B, T, NB), column range of the gate input
        self.cols = None
        self.buf = None
        self.pending = []  # operands of deferred weight-gradient GEMMs, until join()
        self.front_backward = False  # LayerFrontFunction's backward will run (and join)

    def defer_wgrad(self, param, dy2, x2):
        """Weight gradient dy2^T x2 of `param` on the layer's side stream, so that
        these long-reduction GEMMs (few output tiles) run beside the attention
        backward instead of before it; LayerFrontFunction's backward joins them.
        Only when nothing can read the gradient before the join: the parameter
        has no gradient yet (autograd then stores the tensor without a kernel) and
        no hook of its own.  Returns the gradient tensor, or None to compute it now."""
        if (not self.front_backward or param.grad is not None or param._backward_hooks
                or not dy2.is_cuda or getattr(param, "_post_accumulate_grad_hooks", None)):
            return None
        out = torch.empty(dy2.shape[1], x2.shape[1], device=dy2.device, dtype=param.dtype)
        side = _side_stream(dy2.device)
        side.wait_stream(torch.cuda.current_stream(dy2.device))
        with torch.cuda.stream(side):
            torch.matmul(dy2.t(), x2, out=out)
        # the operands stay alive until the join; the result is held only by
        # autograd, which then stores it as the gradient without a copy
        self.pending.append((dy2, x2))
        return out

    def join(self):
        if self.pending:
            dev = self.pending[0][0].device
            torch.cuda.current_stream(dev).wait_stream(_side_stream(dev))
            self.pending.clear()

    def claim(self, device):
        if self.buf is None:
            self.buf = torch.empty(self.shape, device=device, dtype=torch.bfloat16)
        c0, c1 = self.cols
        return self.buf[..., c0:c1]

    def take(self):
        buf, self.buf = self.buf, None
        return buf


def packed_rows(ws):
    """[rows, cols] view over the 2-D tensors `ws` when they are consecutive row
    blocks of one buffer that extends to a multiple of 8 rows (the packed
    projection), else None."""
    w0 = ws[0]
    if not all(w.dim() == 2 and w.is_contiguous() and w.dtype == w0.dtype
               and w.shape[1] == w0.shape[1] for w in ws):
        return None
    end = w0.data_ptr()
    for w in ws:
        if w.data_ptr() != end:
            return None
        end += w.numel() * w.element_size()
    n = sum(w.shape[0] for w in ws)
    rows = (n + 7) // 8 * 8
    avail = w0.untyped_storage().nbytes() - w0.storage_offset() * w0.element_size()
    if avail < rows * w0.shape[1] * w0.element_size():
        return None
    return torch.as_strided(w0, (rows, w0.shape[1]), (w0.shape[1], 1))


class LayerFrontFunction(torch.autograd.Function):
    """The layer's input side as one op: a single projection of x onto
    [W_q; W_k; W_v; W_g0; W_a; W_b; W_d] (one GEMM, one read of x), the short
    convolution of the q|k|v columns, and the gate activations of the a, b, d
    columns.  Returns the convolved q|k|v [B,T,3C], the output-gate input
    (a column view of the projection) and g, delta, beta [B,T,H].

    Backward: every consumer's gradient lands in one packed buffer of the
    projection's layout (the conv and gate kernels write their columns with
    strides), so dx is one GEMM over the packed gradient and the weight gradients
    one more; d is projected from x.detach() in the reference
    (layers/cyfa.py:323-326), so its columns enter the weight gradient but not dx.
    """

    @staticmethod
    def forward(ctx, x, w_q, w_k, w_v, w_g0, w_a, w_b, w_d, cw_q, cw_k, cw_v, A_log, dt_bias,
                b_bias, d_bias, H, slot=None, grad_ready=None):
        # unused outputs get no gradient tensor (no zero fills, no adds of zeros)
        ctx.set_materialize_grads(False)
        B, T, hid = x.shape
        rows = B * T
        dev = x.device
        n_qkv = w_q.shape[0] + w_k.shape[0] + w_v.shape[0]
        c_g, n_g = n_qkv, w_g0.shape[0]
        c_a = c_g + n_g
        c_b, c_d = c_a + H, c_a + 2 * H
        n_used = c_d + H
        NB = (n_used + 7) // 8 * 8  # 16-byte rows
        parts = [w_q, w_k, w_v, w_g0, w_a, w_b, w_d]
        # conv weights (one [n_qkv, Wc] block when the q, k, v pieces are adjacent)
        # and gate parameters as fp32, one launch on the aux stream beside the
        # projection (joined before the convolution)
        aux = _fork(dev)
        cwq, cwk, cwv, A, dt, bb, db = gather_f32(
            [cw_q, cw_k, cw_v, A_log, dt_bias, b_bias, d_bias], aux)
        params_ready = aux.record_event()
        # the packed projection: a view when the weights already are consecutive
        # blocks of one buffer (the layer packs them once), else a concatenation;
        # the padding rows stay uninitialised: the columns they produce are never read
        W_big = packed_rows(parts)
        if W_big is None:
            W_big = torch.empty(NB, hid, device=dev, dtype=w_q.dtype)
            torch.cat(parts, out=W_big[:n_used])
        big = torch.nn.functional.linear(x, W_big)  # [B, T, NB]
        Wc = cw_q.shape[-1]
        # the gate activations (a | b | d columns) run on the aux stream beside the
        # convolution (q | k | v columns); the convolution waits only for its weights
        g = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        delta = torch.empty_like(g)
        beta = torch.empty_like(g)
        torch.cuda.current_stream(dev).wait_event(params_ready)
        aux.wait_stream(torch.cuda.current_stream(dev))
        base, st = big.data_ptr(), _c.c_longlong(NB)
        with torch.cuda.stream(aux):
            _lib.call("cyfa_gate_act_fwd", _c.c_void_p(base + 2 * c_a), st,
                      _c.c_void_p(base + 2 * c_b), st, _c.c_void_p(base + 2 * c_d), st, _p(A),
                      _p(dt), _p(bb), _p(db), _p(g), _p(delta), _p(beta), rows, H,
                      _lib.stream())
        if (cwk.data_ptr() == cwq.data_ptr() + 4 * cwq.numel()
                and cwv.data_ptr() == cwk.data_ptr() + 4 * cwk.numel()):
            cw = torch.as_strided(cwq, (n_qkv, Wc), (Wc, 1))
        else:
            cw = torch.cat([cwq.reshape(-1, Wc), cwk.reshape(-1, Wc), cwv.reshape(-1, Wc)])
        qkv = torch.empty(B, T, n_qkv, device=dev, dtype=torch.bfloat16)
        _lib.call("cyfa_short_conv_fwd", _p(big), _c.c_longlong(NB), None, _p(cw), None, _p(qkv),
                  B, T, n_qkv, Wc, _lib.stream())
        _join(dev)
        gate_in = big[..., c_g:c_g + n_g]
        if slot is not None:
            slot.shape, slot.cols, slot.buf = (B, T, NB), (c_g, c_g + n_g), None
        ctx.slot = slot
        # optional hand-over of the weight gradients as soon as they exist (before
        # dx), e.g. to start their data-parallel all-reduce early
        ctx.grad_ready = grad_ready
        ctx.params = (w_q, w_k, w_v, w_g0, w_a, w_b, w_d, cw_q, cw_k, cw_v, A_log, dt_bias,
                      b_bias, d_bias) if grad_ready is not None else None
        ctx.save_for_backward(x, W_big, big, cw, A, dt, bb, db)
        ctx.meta = (H, NB, n_qkv, c_g, n_g, c_a, c_b, c_d, n_used, Wc,
                    [w.shape[0] for w in parts[:7]], cw_q.dtype,
                    (A_log.dtype, dt_bias.dtype, b_bias.dtype, d_bias.dtype))
        # shapes and dtypes of the small parameters' gradients (zero-size stand-ins)
        ctx.small_like = [torch.empty(t.shape, device="meta", dtype=t.dtype)
                          for t in (cw_q, cw_k, cw_v, A_log, dt_bias, b_bias, d_bias)]
        return qkv, gate_in, g, delta, beta

    @staticmethod
    def backward(ctx, dqkv, dgate_in, dg, ddelta, dbeta):
        x, W_big, big, cw, A, dt, bb, db_ = ctx.saved_tensors
        (H, NB, n_qkv, c_g, n_g, c_a, c_b, c_d, n_used, Wc, sizes, cdt, gdts) = ctx.meta
        B, T, hid = x.shape
        rows = B * T
        dev = x.device
        # the packed gradient: possibly already holding the gate-input columns
        dbig = ctx.slot.take() if ctx.slot is not None else None
        if ctx.slot is not None:
            ctx.slot.join()  # the deferred o_proj / output-gate weight gradients
        gate_done = dbig is not None
        if dbig is None:
            dbig = torch.empty(B, T, NB, device=dev, dtype=torch.bfloat16)
        base, dbase, st = big.data_ptr(), dbig.data_ptr(), _c.c_longlong(NB)
        # fp32 gradients of the small parameters in one buffer: conv weights, A_log,
        # dt_bias, b_bias, d_bias (converted to the parameters' dtypes in one launch)
        n_cw = sizes[0] * Wc
        gflat, goffs = flat_f32([n_cw, sizes[1] * Wc, sizes[2] * Wc, H, H, H, H], dev)
        dcw = torch.as_strided(gflat, (n_qkv, Wc), (Wc, 1))
        if goffs[1] != n_cw or goffs[2] != goffs[1] + sizes[1] * Wc:
            dcw = torch.empty(n_qkv, Wc, device=dev, dtype=torch.float32)
        dA, ddtb, dbb, ddb = (gflat[o:o + H] for o in goffs[3:])
        # the parameter-gradient reductions of the convolution and gate kernels and
        # the scatter into the parameters' dtypes run on the aux stream, joined
        # before the gradients leave this function; their workspaces live until then
        aux = _aux_stream(dev)
        keep = []
        if dqkv is None:
            dbig[..., :n_qkv].zero_()
            dcw.zero_()
        else:
            dqkv = dqkv.to(torch.bfloat16).contiguous()
            nbytes = _lib.lib().cyfa_short_conv_work_bytes(B, T, n_qkv, Wc)
            keep.append(_work(nbytes, dev))
            with _lib.deferred(aux):
                _lib.call("cyfa_short_conv_bwd", _p(big), st, _p(cw), _p(dqkv), _p(dbig), st,
                          _p(dcw), None, B, T, n_qkv, Wc, _p(keep[-1]), _c.c_size_t(nbytes),
                          _lib.stream())
        # gate activation adjoints -> the a, b, d columns
        zeros = lambda: torch.zeros(B, T, H, device=dev, dtype=torch.float32)
        dg = zeros() if dg is None else dg.float().contiguous()
        ddelta = zeros() if ddelta is None else ddelta.float().contiguous()
        dbeta = zeros() if dbeta is None else dbeta.float().contiguous()
        nbytes = _lib.lib().cyfa_gate_act_work_bytes(rows, H)
        keep.append(_work(nbytes, dev))
        with _lib.deferred(aux):
            _lib.call("cyfa_gate_act_bwd", _c.c_void_p(base + 2 * c_a), st,
                      _c.c_void_p(base + 2 * c_b), st, _c.c_void_p(base + 2 * c_d), st, _p(A),
                      _p(dt), _p(bb), _p(db_), _p(dg), _p(ddelta), _p(dbeta),
                      _c.c_void_p(dbase + 2 * c_a), st, _c.c_void_p(dbase + 2 * c_b), st,
                      _c.c_void_p(dbase + 2 * c_d), st, _p(dA), _p(ddtb), _p(dbb), _p(ddb), rows,
                      H, _p(keep[-1]), _c.c_size_t(nbytes), _lib.stream())
        # output-gate input gradient -> its columns (unless its consumer wrote them)
        if dgate_in is not None:
            if gate_done:
                dbig[..., c_g:c_g + n_g].add_(dgate_in)
            else:
                dbig[..., c_g:c_g + n_g].copy_(dgate_in)
        elif not gate_done:
            dbig[..., c_g:c_g + n_g].zero_()
        d2 = dbig.view(rows, NB)
        x2 = x.reshape(rows, hid)
        # weight gradients first, so that their hand-over overlaps the dx GEMM
        dW = torch.matmul(d2[:, :n_used].t(), x2)
        if dcw.data_ptr() != gflat.data_ptr():  # conv pieces not adjacent in gflat
            _join(dev)
            for (o, n), blk in zip(((goffs[0], sizes[0]), (goffs[1], sizes[1]), (goffs[2], sizes[2])),
                                   torch.split(dcw, sizes[:3])):
                gflat[o:o + n * Wc].copy_(blk.reshape(-1))
        small = scatter_from(gflat, goffs, ctx.small_like, _fork(dev))
        grads = (*torch.split(dW, sizes), *small)
        leave = 0  # SMs the dx GEMM leaves to a collective launched just now
        if ctx.grad_ready is not None:
            _join(dev)
            leave = ctx.grad_ready(ctx.params, grads) or 0
        # dx from every column except d (projected from x.detach()) and the padding
        dx = None
        if ctx.needs_input_grad[0]:
            with _sm_carveout(leave):
                dx = torch.matmul(d2[:, :c_d], W_big[:c_d]).view(B, T, hid)
        _join(dev)
        del keep
        return (dx, *grads, None, None, None)


class ChunkCyfaPackedFunction(torch.autograd.Function):
    """chunk_cyfa on q|k|v packed in one [B,T,H*K + H*K + H*V] bf16 tensor (the
    projection + short-conv output); the gradient comes back in the same
    packed layout."""

    @staticmethod
    def forward(ctx, qkv, H, K, V, g, delta, beta, readout, qw, kw, q_eps, k_eps, scale,
                tb=None, lengths=None):
        # tb: the readout table already computed from `readout` on the aux stream;
        # lengths: int32 [B] valid tokens per sequence (right padding), or None
        ctx.set_materialize_grads(False)  # the final states usually get no gradient
        B, T, width = qkv.shape
        if lengths is not None and (lengths.dtype != torch.int32 or lengths.shape != (B,)
                                    or not lengths.is_contiguous()):
            raise ValueError("lengths must be a contiguous int32 tensor of shape [B]")
        dev = qkv.device
        row = qkv.stride(1)
        base = qkv.data_ptr()
        if tb is None:
            tb = table_bf16(readout)
        else:
            _join(dev)
        o = torch.empty(B, T, H, V, device=dev, dtype=torch.bfloat16)
        hk = torch.empty(B, H, K, 128, device=dev, dtype=torch.float32)
        hv = torch.empty(B, H, 128, V, device=dev, dtype=torch.float32)
        clock = torch.empty(B, H, device=dev, dtype=torch.float32)
        nbytes = _lib.lib().cyfa_chunk_saved_bytes(B, T, H, K, V)
        if nbytes == 0:
            raise ValueError(f"unsupported chunk_cyfa shape B={B} T={T} H={H} K={K} V={V}")
        saved = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        qp, kp, vp = base, base + 2 * H * K, base + 4 * H * K
        args = _FwdArgs(B, T, H, K, V, q_eps, k_eps, scale, qp, kp, vp, _p(g), _p(delta),
                        _p(beta), _p(qw), _p(kw), _p(tb), None, None, None, _p(o), _p(hk),
                        _p(hv), _p(clock), row, row, row, _p(lengths))
        _lib.call("cyfa_chunk_fwd", _c.byref(args), _lib.ptr(saved), _c.c_size_t(nbytes),
                  _lib.stream())
        ctx.save_for_backward(qkv, g, delta, beta, qw, kw, tb, hk, hv, clock, saved, lengths)
        ctx.readout_meta = readout.detach()[:0]
        ctx.meta = (H, K, V, q_eps, k_eps, scale)
        return o, hk, hv, clock

    @staticmethod
    def backward(ctx, do, dhk, dhv, dclock):
        qkv, g, delta, beta, qw, kw, tb, hk, hv, clock, saved, lengths = ctx.saved_tensors
        H, K, V, q_eps, k_eps, scale = ctx.meta
        B, T, width = qkv.shape
        dev = qkv.device
        row = qkv.stride(1)
        base = qkv.data_ptr()
        qp, kp, vp = base, base + 2 * H * K, base + 4 * H * K
        fwd = _FwdArgs(B, T, H, K, V, q_eps, k_eps, scale, qp, kp, vp, _p(g), _p(delta),
                       _p(beta), _p(qw), _p(kw), _p(tb), None, None, None, None, _p(hk), _p(hv),
                       _p(clock), row, row, row, _p(lengths))
        do = torch.zeros(B, T, H, V, device=dev, dtype=torch.bfloat16) if do is None \
            else do.to(torch.bfloat16).contiguous()
        dhk = None if dhk is None else dhk.float().contiguous()
        dhv = None if dhv is None else dhv.float().contiguous()
        dclock = None if dclock is None else dclock.float().contiguous()
        dqkv = torch.empty(B, T, width, device=dev, dtype=torch.bfloat16)
        db_ = dqkv.data_ptr()
        dg = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        ddelta = torch.empty_like(dg)
        dbeta = torch.empty_like(dg)
        dtable = torch.empty(H, 128, 128, device=dev, dtype=torch.float32)
        dqw = torch.empty(K, device=dev, dtype=torch.float32)
        dkw = torch.empty(K, device=dev, dtype=torch.float32)
        nwork = _lib.lib().cyfa_chunk_work_bytes(B, T, H, K, V)
        work = _work(nwork, dev)
        # the readout gradient comes from the table-gradient reduction's launch;
        # that launch and the norm-weight sums run on the aux stream, beside the
        # rest of the backward, and are joined before returning
        dr = torch.empty(H, 127, 127, device=dev, dtype=torch.float32) \
            if ctx.needs_input_grad[7] else None
        args = _BwdArgs(fwd, _p(do), _p(dhk), _p(dhv), _p(dclock), db_, db_ + 2 * H * K,
                        db_ + 4 * H * K, _p(dg), _p(ddelta), _p(dbeta), _p(dtable), _p(dqw),
                        _p(dkw), None, None, None, width, width, width,
                        _p(basis_t(128, dev)) if dr is not None else None, _p(dr))
        with _lib.deferred(_aux_stream(dev)):
            _lib.call("cyfa_chunk_bwd", _c.byref(args), _lib.ptr(saved),
                      _c.c_size_t(saved.numel()), _lib.ptr(work), _c.c_size_t(nwork),
                      _lib.stream())
        _join(dev)
        dreadout = None
        if dr is not None:
            rd = ctx.readout_meta.dtype
            dreadout = dr if rd == torch.float32 else dr.to(rd)
        return (dqkv, None, None, None, dg, ddelta, dbeta, dreadout, dqw, dkw, None, None, None,
                None, None)
