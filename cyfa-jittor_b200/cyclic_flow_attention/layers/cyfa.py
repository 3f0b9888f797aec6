"""Cyclic Flow Attention layer (PyTorch host, B200 kernels underneath).

Mirror of the reference layer (cyclic_flow_attention/layers/cyfa.py:236-357):
identical parameter names, shapes and default initialisation, so checkpoints
saved by the reference (PyTorch-compatible safetensors) load with
``load_state_dict``.

On bf16 weights and CUDA inputs (training and prefill) the fused path runs: one
packed projection GEMM (cuBLAS), the short convolutions and gate activations on
its columns, the attention core, and the gated output norm are libcyfa.so
kernels; only the GEMMs are library calls.  A right-padding attention mask runs
the fused path when no gradient is taken (per-row lengths).  T == 1 decode with a
cache runs ``cyfa_decode_layer`` (convolutions, gate activations, decode step
and gated norm in one launch) between the cuBLAS projections.  Other cases (fp32
weights, a mask with gradients, a cache during prefill) run torch glue around
``chunk_cyfa`` / ``fused_recurrent_cyfa``, whose core is libcyfa.so as well.
"""

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import chunk_cyfa, fused_recurrent_cyfa
from .. import _lib
from ..ops.chunk import readout_table, table_bf16
from ..ops.layer_ops import (
    ChunkCyfaPackedFunction,
    GatedNormFunction,
    gated_norm_infer,
    LayerFrontFunction,
    LinearFunction,
    PackedGradSlot,
    _fork,
    packed_rows,
)


class RMSNorm(nn.Module):
    """RMSNorm with an optional sigmoid gate, computed in fp32 and cast back
    (reference layers/cyfa.py:62-84)."""

    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x, gate=None):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()
        if gate is not None:
            y = y * torch.sigmoid(gate.float())
        return y.to(x.dtype)


class ShortConvolution(nn.Module):
    """Causal depthwise convolution without activation, with a decode cache
    (reference layers/cyfa.py:138-181).  weight [dim, 1, width]."""

    def __init__(self, dim, width, bias=False):
        super().__init__()
        self.width = width
        self.weight = nn.Parameter(torch.randn(dim, 1, width) * 0.02)
        self.bias = nn.Parameter(torch.zeros(dim)) if bias else None

    def forward(self, x, cache=None, lengths=None):
        B, T, D = x.shape
        history = x if cache is None else torch.cat([cache.to(x.dtype), x], dim=1)
        offset = self.width - 1 if cache is None else 0
        # y_t = sum_i w_i h_{t+i} over the left-padded history, as W shifted fp32
        # multiply-adds (exact fp32 products: no TF32 convolution algorithm)
        h = F.pad(history.float(), (0, 0, offset, 0))
        n = h.shape[1] - (self.width - 1)
        w = self.weight.float()[:, 0]
        y = h[:, :n] * w[:, 0]
        for i in range(1, self.width):
            y = y + h[:, i:i + n] * w[:, i]
        if self.bias is not None:
            y = y + self.bias.float()
        y = y[:, n - T:]
        if self.width == 1:
            new_cache = history[:, :0]
        elif lengths is None and history.shape[1] >= self.width - 1:
            new_cache = history[:, -(self.width - 1):]
        else:
            ends = torch.full((B,), T, dtype=torch.long, device=x.device) if lengths is None \
                else lengths.long()
            positions = ends.unsqueeze(1) - offset + torch.arange(self.width - 1, device=x.device)
            idx = positions.clamp_min(0)
            new_cache = history[torch.arange(B, device=x.device).unsqueeze(1), idx]
            new_cache = torch.where((positions >= 0).unsqueeze(-1), new_cache,
                                    torch.zeros((), dtype=new_cache.dtype, device=x.device))
        return y.to(x.dtype), new_cache


class CyclicFlowAttention(nn.Module):
    """CyFA attention with projections, short convolutions and a gated readout.

    forward returns (hidden_states, cache).  The cache contains recurrent
    states and the short-convolution histories when use_cache is enabled.
    """

    def __init__(
        self,
        hidden_size=1024,
        num_heads=4,
        head_dim=256,
        expand_k=1.0,
        expand_v=1.0,
        num_slots=128,
        use_short_conv=True,
        conv_size=4,
        conv_bias=False,
        norm_eps=1e-6,
        chunk_size=64,
        **kwargs,
    ):
        super().__init__()
        self.num_heads = num_heads
        self.head_k_dim = int(head_dim * expand_k)
        self.head_v_dim = int(head_dim * expand_v)
        self.key_dim = num_heads * self.head_k_dim
        self.value_dim = num_heads * self.head_v_dim
        self.num_slots, self.chunk_size = num_slots, chunk_size
        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.a_proj = nn.Linear(hidden_size, num_heads, bias=False)
        self.b_proj = nn.Linear(hidden_size, num_heads, bias=True)
        self.d_proj = nn.Linear(hidden_size, num_heads, bias=True)
        # dt_bias / A_log / readout as the reference initialises them (:274-284)
        dt = (torch.rand(num_heads) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)).exp()
        self.dt_bias = nn.Parameter(dt + torch.log(1.0 - torch.exp(-dt)))
        self.A_log = nn.Parameter(torch.log(torch.rand(num_heads) * 16.0 + 1e-3))
        self.readout = nn.Parameter(
            torch.eye(num_slots - 1).expand(num_heads, -1, -1).clone())
        self.q_norm = RMSNorm(self.head_k_dim, norm_eps)
        self.k_norm = RMSNorm(self.head_k_dim, norm_eps)
        self.use_short_conv = use_short_conv
        if use_short_conv:
            self.q_conv1d = ShortConvolution(self.key_dim, conv_size, conv_bias)
            self.k_conv1d = ShortConvolution(self.key_dim, conv_size, conv_bias)
            self.v_conv1d = ShortConvolution(self.value_dim, conv_size, conv_bias)
        self.g_proj = nn.Sequential(
            nn.Linear(hidden_size, self.head_v_dim, bias=False),
            nn.Linear(self.head_v_dim, self.value_dim, bias=True),
        )
        self.o_norm = RMSNorm(self.head_v_dim, norm_eps)
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)

    # Optional callable(params, grads) -> int: receives the input-side weight
    # gradients as soon as the fused backward has formed them (before the input
    # gradient), e.g. GradientBuckets.early to start their all-reduce early; it
    # returns how many SMs the input-gradient GEMM should leave free (0: none).
    grad_ready = None

    def grad_groups(self):
        """Parameters grouped in the order the fused backward produces their
        gradients (output side first, input side last); the last group is the
        one the fused backward hands to `grad_ready`."""
        front = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                 self.g_proj[0].weight, self.a_proj.weight, self.b_proj.weight,
                 self.d_proj.weight, self.q_conv1d.weight, self.k_conv1d.weight,
                 self.v_conv1d.weight, self.A_log, self.dt_bias, self.b_proj.bias,
                 self.d_proj.bias]
        g1 = self.g_proj[1]
        back = [p for p in (g1.weight, g1.bias, self.o_norm.weight) if p is not None]
        core = [self.readout, self.q_norm.weight, self.k_norm.weight]
        return [[self.o_proj.weight], back, core, front]

    def keep_fp32(self):
        """Casts to bf16 except the parameters the reference keeps in fp32
        (norm weights, readout, A_log, dt_bias; models/cyfa/modeling_cyfa.py:110-116)."""
        for name, p in self.named_parameters():
            keep = name.endswith("norm.weight") or name in ("readout", "A_log", "dt_bias")
            p.data = p.data.float() if keep else p.data.bfloat16()
        return self

    def _front_weights(self):
        return [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.g_proj[0].weight,
                self.a_proj.weight, self.b_proj.weight, self.d_proj.weight]

    def _pack_front(self):
        """Places the seven input-side projection weights as consecutive row blocks
        of one buffer (padded to a multiple of 8 rows), re-pointing each
        parameter's data at its block, so that the fused path multiplies by that
        buffer instead of concatenating the weights every step.  Done once, and
        again only if something (a device move, a cast, a load) replaced the
        parameters' storage."""
        ws = self._front_weights()
        if packed_rows(ws) is not None or torch.cuda.is_current_stream_capturing():
            return
        if any(w.dtype != ws[0].dtype or w.device != ws[0].device for w in ws):
            return
        n = sum(w.shape[0] for w in ws)
        buf = torch.empty((n + 7) // 8 * 8, ws[0].shape[1], device=ws[0].device, dtype=ws[0].dtype)
        with torch.no_grad():
            r = 0
            for w in ws:
                buf[r:r + w.shape[0]].copy_(w)
                w.data = buf[r:r + w.shape[0]]
                r += w.shape[0]

    def _fused_ok(self, x, cache, attention_mask):
        # a right-padding mask runs fused when no gradient is taken (prefill):
        # the masked gates make the padding neutral for the states and the
        # clock; with gradients it runs the reference's masking on torch glue
        return (
            cache is None
            and (attention_mask is None or not torch.is_grad_enabled())
            and x.is_cuda
            and x.dtype == torch.bfloat16
            and self.q_proj.weight.dtype == torch.bfloat16
            and self.use_short_conv
            and self.q_conv1d.width <= 4
            and self.q_conv1d.bias is None
            and self.num_slots == 128
            and self.head_k_dim in (128, 256)
            and self.head_v_dim in (128, 256)
            and (self.training or x.shape[1] > 1 or torch.is_grad_enabled())
        )

    def _forward_fused(self, x, use_cache, attention_mask=None, project=True):
        """One packed q|k|v|g0|a|b|d projection with the short convolution and the
        gate activations on its columns (LayerFrontFunction), the CyFA op on the
        convolved q|k|v, the gated output norm with the gate's second linear, and
        o_proj; the same math as the reference execute().

        A right-padding ``attention_mask`` (1 for the first lengths[b] tokens of
        row b) becomes per-row lengths for the op, which treats the later tokens
        as neutral padding (g = delta = beta = 0, reference layers/cyfa.py:304-308,
        326-328), and the convolution histories of the cache end at each row's
        length (the reference's ShortConvolution with lengths, :144-181).  The
        outputs at padded positions are not defined.  With ``project=False`` the
        result is the gated norm's output [B, T, H*V], before o_proj (the
        head-parallel layer gathers it across ranks first)."""
        B, T, _ = x.shape
        lengths = None
        if attention_mask is not None:
            lengths = attention_mask.sum(1).to(torch.int32).contiguous()  # int32 [B]
        H, K, V = self.num_heads, self.head_k_dim, self.head_v_dim
        g0 = self.g_proj[0]
        self._pack_front()
        slot = PackedGradSlot()
        # LayerFrontFunction's backward runs (and joins deferred side-stream work)
        # iff one of its differentiable inputs needs a gradient
        slot.front_backward = torch.is_grad_enabled() and any(
            t.requires_grad for t in (x, self.q_proj.weight, self.k_proj.weight,
                                      self.v_proj.weight, g0.weight, self.a_proj.weight,
                                      self.b_proj.weight, self.d_proj.weight))
        # the readout table on the aux stream, beside the projection (joined with
        # the parameter conversions before the convolution)
        tb = torch.empty(H, 128, 128, device=x.device, dtype=torch.bfloat16)
        with torch.cuda.stream(_fork(x.device)):
            table_bf16(self.readout, out=tb)
        qkv, gate_in, g, delta, beta = LayerFrontFunction.apply(
            x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, g0.weight,
            self.a_proj.weight, self.b_proj.weight, self.d_proj.weight, self.q_conv1d.weight,
            self.k_conv1d.weight, self.v_conv1d.weight, self.A_log, self.dt_bias,
            self.b_proj.bias, self.d_proj.bias, H, slot, self.grad_ready)
        o, hk, hv, clock = ChunkCyfaPackedFunction.apply(
            qkv, H, K, V, g, delta, beta, self.readout, self.q_norm.weight.float(),
            self.k_norm.weight.float(), float(self.q_norm.eps), float(self.k_norm.eps), K ** -0.5,
            tb, lengths)
        g1 = self.g_proj[1]
        y = None
        if not torch.is_grad_enabled():
            y = gated_norm_infer(o, gate_in, g1.weight, g1.bias, self.o_norm.weight,
                                 self.o_norm.eps, float(self.num_slots - 1))
        if y is None:
            y = GatedNormFunction.apply(o, gate_in, g1.weight, g1.bias, self.o_norm.weight,
                                        self.o_norm.eps, float(self.num_slots - 1), slot,
                                        (g1.weight,))
        if project:
            y = LinearFunction.apply(y, self.o_proj.weight, (self.o_proj.weight,), slot) \
                if self.o_proj.bias is None else self.o_proj(y)
        new_cache = None
        if use_cache:
            W = self.q_conv1d.width
            w_qkv = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight])
            # conv histories: the last W-1 projected (pre-conv) rows of q, k and v
            # before each row's end (zeros before the sequence start)
            if W > 1 and lengths is None and T >= W - 1:
                pre = F.linear(x[:, -(W - 1):], w_qkv)
            elif W > 1:
                ends = torch.full((B,), T, device=x.device, dtype=torch.long) \
                    if lengths is None else lengths.long()
                pos = ends.unsqueeze(1) - (W - 1) + torch.arange(W - 1, device=x.device)
                rows = x[torch.arange(B, device=x.device).unsqueeze(1), pos.clamp_min(0)]
                pre = F.linear(rows, w_qkv) * (pos >= 0).unsqueeze(-1).to(x.dtype)
            else:
                pre = x[:, :0]
            cq, ck, cv = (pre[..., :H * K], pre[..., H * K:2 * H * K], pre[..., 2 * H * K:]) \
                if W > 1 else (pre, pre, pre)
            new_cache = {"recurrent_state": (hk, hv, clock), "conv_state": (cq, ck, cv)}
        return y, new_cache

    def _decode_ok(self, x, cache, attention_mask):
        """T = 1 inference step with a full cache (recurrent state and the three
        convolution histories) on bf16 weights: the libcyfa decode glue path."""
        if (cache is None or attention_mask is not None or not x.is_cuda
                or x.dtype != torch.bfloat16 or x.shape[1] != 1 or self.training
                or torch.is_grad_enabled() or not self.use_short_conv):
            return False
        conv, state = cache.get("conv_state"), cache.get("recurrent_state")
        W = self.q_conv1d.width
        return (state is not None and conv is not None and all(c is not None for c in conv)
                and 2 <= W <= 4 and all(c.shape[1] == W - 1 for c in conv)
                and self.q_conv1d.bias is None and self.o_proj.bias is None
                and self.q_proj.weight.dtype == torch.bfloat16 and self.num_slots == 128
                and self.head_k_dim in (128, 256) and self.head_v_dim in (128, 256)
                and self.key_dim % 8 == 0 and self.value_dim % 8 == 0)

    def _decode_constants(self):
        """fp32/bf16 copies of the small parameters the decode kernels read (the
        readout table R.Phi, conv weights, norm weights, gate parameters), made
        once and remade only when one of those parameters changes."""
        g1 = self.g_proj[1]
        ps = (self.readout, self.q_conv1d.weight, self.k_conv1d.weight, self.v_conv1d.weight,
              self.q_norm.weight, self.k_norm.weight, self.A_log, self.dt_bias,
              self.b_proj.bias, self.d_proj.bias, self.o_norm.weight, g1.bias)
        key = tuple((p.data_ptr(), p._version) for p in ps)
        cached = getattr(self, "_decode_cached", None)
        if cached is None or cached[0] != key:
            W = self.q_conv1d.width

            def f32(t):
                return t.detach().float().contiguous()

            consts = dict(
                table=readout_table(self.readout.detach()).contiguous(),
                wq=f32(self.q_conv1d.weight).reshape(-1, W),
                wk=f32(self.k_conv1d.weight).reshape(-1, W),
                wv=f32(self.v_conv1d.weight).reshape(-1, W),
                q_norm=f32(self.q_norm.weight), k_norm=f32(self.k_norm.weight),
                A_log=f32(self.A_log), dt_bias=f32(self.dt_bias),
                b_bias=f32(self.b_proj.bias), d_bias=f32(self.d_proj.bias),
                o_norm=f32(self.o_norm.weight),
                g_bias=g1.bias.detach().to(torch.bfloat16).contiguous())
            self._decode_cached = (key, consts)
        return self._decode_cached[1]

    def _forward_decode(self, x, cache, inplace=False):
        """One token per sequence (reference layers/cyfa.py:299-357 at T = 1 with
        a cache): the packed q|k|v|g0|a|b|d projection and the gate's second
        linear (cuBLAS), then one cyfa_decode_layer launch for everything between
        them and o_proj: the three short convolutions with their histories, the
        gate activations, the recurrent step and the gated output norm with its
        bias.  With ``inplace`` the cache tensors are updated in place (the
        graphed decoder's static buffers); otherwise a new cache is returned and
        the caller's is left untouched, as the reference does."""
        B = x.shape[0]
        H, K, V = self.num_heads, self.head_k_dim, self.head_v_dim
        HK, HV = self.key_dim, self.value_dim
        c = self._decode_constants()
        self._pack_front()
        ws = self._front_weights()
        wf = packed_rows(ws)
        if wf is None:
            n = sum(w.shape[0] for w in ws)
            wf = torch.cat(ws + [ws[0].new_zeros((n + 7) // 8 * 8 - n, ws[0].shape[1])])
        P = torch.mm(x.reshape(B, -1), wf.t())  # [B, q|k|v|g0|a|b|d (+pad)]
        gate = torch.mm(P[:, 2 * HK + HV:2 * HK + HV + V], self.g_proj[1].weight.t())
        hk, hv, clock = cache["recurrent_state"]
        cq, ck, cv = cache["conv_state"]
        dev = x.device
        if inplace:
            hk_o, hv_o, clock_o = hk, hv, clock
        else:
            cq, ck, cv = (t.to(torch.bfloat16).contiguous().clone() for t in (cq, ck, cv))
            hk_o, hv_o = torch.empty_like(hk), torch.empty_like(hv)
            clock_o = torch.empty_like(clock)
        y = torch.empty(B, HV, device=dev, dtype=torch.bfloat16)
        p = _lib.ptr
        a = _lib.DecodeLayerArgs(
            B=B, H=H, K=K, V=V, W=self.q_conv1d.width, a_col=2 * HK + HV + V,
            P_stride=P.stride(0), P=p(P), cache_q=p(cq), cache_k=p(ck), cache_v=p(cv),
            wconv_q=p(c["wq"]), wconv_k=p(c["wk"]), wconv_v=p(c["wv"]), A_log=p(c["A_log"]),
            dt_bias=p(c["dt_bias"]), b_bias=p(c["b_bias"]), d_bias=p(c["d_bias"]),
            table=p(c["table"]), q_norm_weight=p(c["q_norm"]), k_norm_weight=p(c["k_norm"]),
            hk_in=p(hk), hv_in=p(hv), clock_in=p(clock), hk_out=p(hk_o), hv_out=p(hv_o),
            clock_out=p(clock_o), gate=p(gate), gate_bias=p(c["g_bias"]),
            o_norm_weight=p(c["o_norm"]), y=p(y), q_eps=float(self.q_norm.eps),
            k_eps=float(self.k_norm.eps), scale=K ** -0.5, o_eps=float(self.o_norm.eps),
            o_scale=float(self.num_slots - 1))
        _lib.call("cyfa_decode_layer", _lib.ctypes.byref(a), _lib.stream())
        out = torch.mm(y, self.o_proj.weight.t()).reshape(B, 1, -1)
        return out, {"recurrent_state": (hk_o, hv_o, clock_o), "conv_state": (cq, ck, cv)}

    def forward(self, x, cache=None, use_cache=False, attention_mask=None):
        if self._fused_ok(x, cache, attention_mask):
            return self._forward_fused(x, use_cache, attention_mask)
        if self._decode_ok(x, cache, attention_mask):
            y, new_cache = self._forward_decode(x, cache)
            return y, new_cache if use_cache else None
        B, T, _ = x.shape
        H = self.num_heads
        q, k, v = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        lengths = None
        if attention_mask is not None:
            # right padding is neutral for the recurrence and the convolution
            mask = attention_mask.unsqueeze(-1)
            q, k, v = (t * mask.to(t.dtype) for t in (q, k, v))
            lengths = attention_mask.long().sum(1)
        conv_cache = (None, None, None) if cache is None else cache.get("conv_state",
                                                                       (None, None, None))
        if self.use_short_conv:
            q, cq = self.q_conv1d(q, conv_cache[0], lengths)
            k, ck = self.k_conv1d(k, conv_cache[1], lengths)
            v, cv = self.v_conv1d(v, conv_cache[2], lengths)
        else:
            cq = ck = cv = None
        q = q.reshape(B, T, H, self.head_k_dim)
        k = k.reshape(B, T, H, self.head_k_dim)
        v = v.reshape(B, T, H, self.head_v_dim)
        a = self.a_proj(x).float() + self.dt_bias.float()
        g = -self.A_log.float().exp() * F.softplus(a)
        delta = torch.sigmoid(self.d_proj(x.detach()).float())
        beta = torch.sigmoid(self.b_proj(x).float())
        if attention_mask is not None:
            valid = attention_mask.unsqueeze(-1).bool()
            zero = torch.zeros((), device=x.device)
            g, delta, beta = (torch.where(valid, t, zero) for t in (g, delta, beta))
        kwargs = dict(
            q=q, k=k, v=v, g=g, delta=delta, beta=beta, readout=self.readout,
            q_norm_weight=self.q_norm.weight.float(), k_norm_weight=self.k_norm.weight.float(),
            q_norm_eps=self.q_norm.eps, k_norm_eps=self.k_norm.eps,
            initial_state=None if cache is None else cache["recurrent_state"],
            output_final_state=use_cache,
        )
        if not self.training and T == 1 and not torch.is_grad_enabled():
            o, state = fused_recurrent_cyfa(**kwargs)
        else:
            o, state = chunk_cyfa(**kwargs, chunk_size=self.chunk_size)
        gate = self.g_proj(x).reshape(B, T, H, self.head_v_dim)
        o = self.o_norm(o * (self.num_slots - 1), gate).reshape(B, T, self.value_dim)
        o = self.o_proj(o)
        new_cache = {"recurrent_state": state, "conv_state": (cq, ck, cv)} if use_cache else None
        return o, new_cache
