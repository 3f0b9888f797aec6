"""CyFA decoder blocks and causal language model (PyTorch host, libcyfa kernels).

Mirror of the reference's models/cyfa/modeling_cyfa.py: the same classes,
module tree and parameter names (``model.embeddings``, ``model.layers.N.attn``,
``attn_norm``, ``mlp_norm``, ``mlp.{gate,up,down}_proj``, ``model.norm``,
``lm_head``), so the reference's safetensors checkpoints load unchanged
(``cyclic_flow_attention.utils.load_model``).

Two execution paths:
* ``forward`` over a sequence: with gradients (training) the attention layer's
  fused path with the block norms and the gated MLP in PyTorch as the reference
  computes them (fp32 math, bf16 results); without (prefill) the same glue
  launches as the decode step below.
* ``decode_step`` for one token per sequence with a cache: every piece of glue
  is one libcyfa launch (``cyfa_add_rmsnorm`` for residual + norm,
  ``cyfa_swiglu`` for the MLP activation) around cuBLAS GEMMs on packed
  weights and the attention layer's decode path.  With ``inplace=True`` it
  updates the cache tensors in place, which is what
  ``generation.GraphedDecoder`` captures into one CUDA graph per step.
"""

import math

import torch
import torch.nn.functional as F
from torch import nn

from ... import _lib
from ...layers.cyfa import CyclicFlowAttention, RMSNorm
from ...ops.layer_ops import packed_rows
from .configuration_cyfa import CyclicFlowAttentionConfig

# Parameters the reference keeps in fp32 when it casts a model to bf16
# (models/cyfa/modeling_cyfa.py:110-116).
_FP32_NAMES = ("norm.weight", "readout", "A_log", "dt_bias")


def _pack_rows(ws):
    """Re-points the 2-D weights ``ws`` at consecutive row blocks of one buffer
    (rows padded to a multiple of 8) so that one GEMM multiplies by all of
    them; a no-op when they already are, or while a CUDA graph is captured."""
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


def _f32(t):
    return t.detach().float().contiguous()


class GatedMLP(nn.Module):
    """SwiGLU MLP (reference modeling_cyfa.py:13-27)."""

    def __init__(self, config):
        super().__init__()
        mid = config.intermediate_size or 256 * math.ceil(
            int(config.hidden_size * config.hidden_ratio * 2 / 3) / 256)
        self.intermediate_size = mid
        self.gate_proj = nn.Linear(config.hidden_size, mid, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, mid, bias=False)
        self.down_proj = nn.Linear(mid, config.hidden_size, bias=False)

    def forward(self, x):
        g = self.gate_proj(x).float()
        u = self.up_proj(x).float()
        return self.down_proj((g * torch.sigmoid(g) * u).to(x.dtype))

    def decode(self, h):
        """h [B, hidden] bf16 -> [B, hidden]: one GEMM on the packed gate|up
        weights, cyfa_swiglu, down_proj."""
        ws = [self.gate_proj.weight, self.up_proj.weight]
        _pack_rows(ws)
        wf = packed_rows(ws)
        if wf is None:
            wf = torch.cat(ws)
        mid = self.intermediate_size
        gu = torch.mm(h, wf.t())
        act = torch.empty(h.shape[0], mid, device=h.device, dtype=h.dtype)
        _lib.call("cyfa_swiglu", _lib.ptr(gu), _lib.ptr(act), h.shape[0], mid, _lib.stream())
        return torch.mm(act, self.down_proj.weight.t())


class CyFABlock(nn.Module):
    """attn_norm -> attention -> residual, mlp_norm -> MLP -> residual
    (reference modeling_cyfa.py:30-55)."""

    def __init__(self, config):
        super().__init__()
        self.attn_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.attn = CyclicFlowAttention(
            hidden_size=config.hidden_size, num_heads=config.num_heads,
            head_dim=config.head_dim, expand_k=config.expand_k, expand_v=config.expand_v,
            num_slots=config.num_slots, use_short_conv=config.use_short_conv,
            conv_size=config.conv_size, conv_bias=config.conv_bias, norm_eps=config.norm_eps,
            chunk_size=config.chunk_size)
        self.mlp_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.mlp = GatedMLP(config)

    def forward(self, x, cache=None, use_cache=False, attention_mask=None):
        y, cache = self.attn(self.attn_norm(x), cache, use_cache, attention_mask)
        residual = x + y
        return residual + self.mlp(self.mlp_norm(residual)), cache


class CyclicFlowAttentionModel(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.embeddings = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([CyFABlock(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.norm_eps)

    def _glue_ok(self, input_ids):
        w = self.embeddings.weight
        D = w.shape[1]
        return (not torch.is_grad_enabled() and w.is_cuda and w.dtype == torch.bfloat16
                and input_ids.is_cuda and D % 8 == 0 and D <= 8192
                and all(l.mlp.intermediate_size % 8 == 0 for l in self.layers))

    def forward(self, input_ids, cache=None, use_cache=False, attention_mask=None):
        if self._glue_ok(input_ids):
            return self._forward_glue(input_ids, cache, use_cache, attention_mask)
        x = self.embeddings(input_ids)
        new = []
        for i, layer in enumerate(self.layers):
            x, s = layer(x, None if cache is None else cache[i], use_cache, attention_mask)
            new.append(s)
        return self.norm(x), new if use_cache else None

    def _forward_glue(self, input_ids, cache, use_cache, attention_mask):
        """Inference over a sequence (prefill): the blocks of ``forward`` with
        their glue as libcyfa launches, as ``decode_step`` runs it.  The residual
        stream stays in one bf16 buffer: each cyfa_add_rmsnorm adds the previous
        branch output into it (rounded to bf16 as the reference's ``x + y``) and
        normalises it for the next branch; the MLP is one GEMM on the packed
        gate|up weights, cyfa_swiglu and down_proj."""
        x = self.embeddings(input_ids).contiguous()
        B, T, D = x.shape
        rows = B * T
        h = torch.empty_like(x)
        p, st = _lib.ptr, _lib.stream()
        prev = None
        new = []
        for i, layer in enumerate(self.layers):
            _lib.call("cyfa_add_rmsnorm", p(x), p(prev), p(_f32(layer.attn_norm.weight)),
                      float(layer.attn_norm.eps), p(h), rows, D, st)
            y, s = layer.attn(h, None if cache is None else cache[i], use_cache, attention_mask)
            new.append(s)
            _lib.call("cyfa_add_rmsnorm", p(x), p(y.contiguous()),
                      p(_f32(layer.mlp_norm.weight)), float(layer.mlp_norm.eps), p(h), rows, D,
                      st)
            prev = layer.mlp.decode(h.view(rows, D))
        _lib.call("cyfa_add_rmsnorm", p(x), p(prev), p(_f32(self.norm.weight)),
                  float(self.norm.eps), p(h), rows, D, st)
        return h, new if use_cache else None


class CyclicFlowAttentionForCausalLM(nn.Module):
    """CyFA causal language model with the reference's parameter names
    (reference modeling_cyfa.py:72-133)."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.model = CyclicFlowAttentionModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embeddings.weight

    @classmethod
    def from_pretrained(cls, path):
        from ...utils import load_model

        model, _ = load_model(path)
        return model

    def save_pretrained(self, directory, tokenizer=None):
        from ...utils import save_model

        save_model(self, directory, tokenizer)

    def _decode_ok(self, input_ids, cache, attention_mask):
        w = self.lm_head.weight
        return (cache is not None and attention_mask is None and input_ids.dim() == 2
                and input_ids.shape[1] == 1 and input_ids.is_cuda and w.is_cuda
                and w.dtype == torch.bfloat16 and not self.training
                and not torch.is_grad_enabled() and self.config.hidden_size % 8 == 0
                and self.model.layers[0].mlp.intermediate_size % 8 == 0)

    def forward(self, input_ids, labels=None, cache=None, use_cache=False, attention_mask=None):
        if labels is None and self._decode_ok(input_ids, cache, attention_mask):
            logits, new = self.decode_step(input_ids, cache)
            return {"logits": logits.unsqueeze(1), "loss": None,
                    "cache": new if use_cache else None}
        hidden, cache = self.model(input_ids, cache, use_cache, attention_mask)
        logits = self.lm_head(hidden)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(
                logits[:, :-1].float().reshape(-1, self.config.vocab_size),
                labels[:, 1:].reshape(-1), ignore_index=-100)
        return {"logits": logits, "loss": loss, "cache": cache}

    def decode_step(self, input_ids, cache, inplace=False):
        """One token per sequence: input_ids [B, 1] -> (logits [B, vocab], cache).

        The residual stream stays in one bf16 buffer: each cyfa_add_rmsnorm adds
        the previous branch output into it and normalises it for the next branch,
        the sums rounded to bf16 as the reference's ``x + y`` does."""
        B, D = input_ids.shape[0], self.config.hidden_size
        x = F.embedding(input_ids[:, 0], self.model.embeddings.weight).contiguous()
        h = torch.empty_like(x)
        p, st = _lib.ptr, _lib.stream()
        prev = None
        new = []
        for layer, c in zip(self.model.layers, cache):
            _lib.call("cyfa_add_rmsnorm", p(x), p(prev), p(_f32(layer.attn_norm.weight)),
                      float(layer.attn_norm.eps), p(h), B, D, st)
            if layer.attn._decode_ok(h.unsqueeze(1), c, None):
                y, c = layer.attn._forward_decode(h.unsqueeze(1), c, inplace)
            elif inplace:
                raise ValueError("in-place decoding needs every layer on the libcyfa decode "
                                 "path (bf16 weights, short convolutions without bias, full cache)")
            else:
                y, c = layer.attn(h.unsqueeze(1), c, True)
            y = y.reshape(B, D)
            _lib.call("cyfa_add_rmsnorm", p(x), p(y), p(_f32(layer.mlp_norm.weight)),
                      float(layer.mlp_norm.eps), p(h), B, D, st)
            prev = layer.mlp.decode(h)
            new.append(c)
        norm = self.model.norm
        _lib.call("cyfa_add_rmsnorm", p(x), p(prev), p(_f32(norm.weight)), float(norm.eps), p(h),
                  B, D, st)
        return torch.mm(h, self.lm_head.weight.t()), new

    def to_bfloat16(self):
        """bf16 except the parameters the reference keeps in fp32."""
        for name, p in self.named_parameters():
            keep = any(s in name for s in _FP32_NAMES)
            p.data = p.data.float() if keep else p.data.bfloat16()
        return self

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=32, eos_token_id=None):
        """Greedy generation (reference modeling_cyfa.py:118-133): prefill, then
        one decode step per token; stops early when every row emitted eos."""
        self.eval()
        hidden, cache = self.model(input_ids, use_cache=True)
        current = self.lm_head(hidden[:, -1]).argmax(-1, keepdim=True)
        tokens = [input_ids, current]
        for _ in range(max_new_tokens - 1):
            if eos_token_id is not None and bool((current == eos_token_id).all()):
                break
            logits, cache = self.decode_step(current, cache)
            current = logits.argmax(-1, keepdim=True)
            tokens.append(current)
        return torch.cat(tokens, dim=1)


__all__ = ["CyclicFlowAttentionConfig", "CyclicFlowAttentionForCausalLM",
           "CyclicFlowAttentionModel", "CyFABlock", "GatedMLP"]
