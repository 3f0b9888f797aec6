"""GPU checks of the CyFA language model's decode path: the three decode glue
kernels against plain fp32 PyTorch / the oracle, the model's logits against
the oracle LM, decoding after a prefill against the full-sequence forward at
every step (the reference's own pin, tests/test_inference.py:20-34: rel-RMS <
0.02), and the CUDA-graph decoder against eager decoding."""

import pytest
import torch

from gpu_util import rel_l2, seeded
from oracle import cyfa_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention import _lib
    from cyclic_flow_attention.models.cyfa import CyclicFlowAttentionConfig
    from cyclic_flow_attention.utils import initialize_model

    cfg = CyclicFlowAttentionConfig(hidden_size=256, num_heads=2, head_dim=128,
                                    num_hidden_layers=2, vocab_size=512)
    m = initialize_model(cfg, generator=seeded(0))
    with torch.no_grad():
        for blk in m.model.layers:  # break the readout's identity init
            blk.attn.readout.add_(0.05 * torch.randn(blk.attn.readout.shape, generator=seeded(1)))
    return _lib, cfg, m.cuda().eval()


def test_add_rmsnorm_kernel(lm):
    _lib, _, _ = lm
    rows, D = 37, 2048
    x = torch.randn(rows, D, generator=seeded(3)).bfloat16().cuda()
    y = torch.randn(rows, D, generator=seeded(4)).bfloat16().cuda()
    w = (1 + 0.1 * torch.randn(D, generator=seeded(5))).cuda()
    for res in (None, y):
        x0 = x.clone()
        out = torch.empty_like(x)
        _lib.call("cyfa_add_rmsnorm", _lib.ptr(x0), _lib.ptr(res), _lib.ptr(w), 1e-6,
                  _lib.ptr(out), rows, D, _lib.stream())
        s = x.float() if res is None else (x.float() + y.float()).bfloat16().float()
        ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        assert torch.equal(x0.float(), s)
        assert rel_l2(out, ref) < 1e-2


@pytest.mark.parametrize("W", [2, 4])
def test_decode_conv_kernel(lm, W):
    _lib, _, _ = lm
    B, Cq, Cv = 5, 256, 512
    P = torch.randn(B, 2 * Cq + Cv + 24, generator=seeded(6)).bfloat16().cuda()
    caches = [torch.randn(B, W - 1, c, generator=seeded(7 + i)).bfloat16().cuda()
              for i, c in enumerate((Cq, Cq, Cv))]
    ws = [torch.randn(c, 1, W, generator=seeded(10 + i)).cuda() * 0.3
          for i, c in enumerate((Cq, Cq, Cv))]
    ys = [torch.empty(B, c, device="cuda", dtype=torch.bfloat16) for c in (Cq, Cq, Cv)]
    before = [c.clone() for c in caches]
    p = _lib.ptr
    _lib.call("cyfa_decode_conv", p(P), P.stride(0), *(p(c) for c in caches),
              *(p(w.reshape(-1, W)) for w in ws), *(p(y) for y in ys), B, Cq, Cq, Cv, W,
              _lib.stream())
    cols = [P[:, :Cq], P[:, Cq:2 * Cq], P[:, 2 * Cq:2 * Cq + Cv]]
    for x, c0, c1, w, y in zip(cols, before, caches, ws, ys):
        ref, new = O.short_convolution(x[:, None].float().cpu(), w.cpu(), cache=c0.float().cpu())
        assert rel_l2(y[:, None], ref) < 1e-2
        assert torch.equal(c1.float().cpu(), new)


def test_swiglu_kernel(lm):
    _lib, _, _ = lm
    rows, mid = 19, 1024
    gu = torch.randn(rows, 2 * mid, generator=seeded(12)).bfloat16().cuda()
    out = torch.empty(rows, mid, device="cuda", dtype=torch.bfloat16)
    _lib.call("cyfa_swiglu", _lib.ptr(gu), _lib.ptr(out), rows, mid, _lib.stream())
    g, u = gu[:, :mid].float(), gu[:, mid:].float()
    assert rel_l2(out, g * torch.sigmoid(g) * u) < 1e-2


def _oracle_logits(cfg, m, ids):
    params = {n: t.float().cpu() for n, t in m.state_dict().items()}
    return O.cyfa_lm(params, ids.cpu(), cfg.num_hidden_layers, cfg.num_heads, cfg.head_dim,
                     cfg.head_dim)


def test_lm_matches_oracle(lm):
    _, cfg, m = lm
    ids = torch.randint(0, cfg.vocab_size, (2, 96), generator=seeded(13)).cuda()
    with torch.no_grad():
        logits = m(ids)["logits"]
    assert rel_l2(logits, _oracle_logits(cfg, m, ids)) < 1e-2


def test_lm_decode_matches_forward(lm):
    _, cfg, m = lm
    ids = torch.randint(0, cfg.vocab_size, (3, 72), generator=seeded(14)).cuda()
    with torch.no_grad():
        full = m(ids)["logits"]
        cache = m(ids[:, :64], use_cache=True)["cache"]
        for t in range(64, 72):
            snap = [t_.clone() for c in cache for t_ in c["recurrent_state"] + c["conv_state"]]
            out = m(ids[:, t:t + 1], cache=cache, use_cache=True)
            after = [t_ for c in cache for t_ in c["recurrent_state"] + c["conv_state"]]
            assert all(torch.equal(a, b) for a, b in zip(snap, after))  # caller's cache kept
            cache = out["cache"]
            err = rel_l2(out["logits"][:, 0], full[:, t])
            print("decode vs forward logits", t, round(err, 5))
            assert err < 1e-2, t


def test_graphed_decoder_matches_eager(lm):
    from cyclic_flow_attention.generation import GraphedDecoder

    _, cfg, m = lm
    ids = torch.randint(0, cfg.vocab_size, (4, 64), generator=seeded(15)).cuda()
    eager = m.generate(ids, max_new_tokens=8)[:, 64:]
    dec = GraphedDecoder(m)
    graphed = dec.generate(ids, 8)
    assert torch.equal(graphed, eager)
    # a second prefill re-captures over new state and gives the same tokens
    assert torch.equal(dec.generate(ids, 8), eager)


def _right_padded(prompts, width):
    ids = torch.zeros(len(prompts), width, dtype=torch.long)
    mask = torch.zeros_like(ids)
    for r, p in enumerate(prompts):
        ids[r, :len(p)] = torch.tensor(p)
        mask[r, :len(p)] = 1
    return ids.cuda(), mask.cuda()


def test_masked_prefill_matches_rows(lm):
    """A right-padded batch prefilled with its attention mask (the fused layer
    path with per-row lengths, as generate_batch runs it) gives each row the
    hidden states, recurrent state and convolution histories of that row run
    alone, and its last-token logits match the oracle LM on the row
    (reference layers/cyfa.py:304-328: padding is neutral)."""
    _, cfg, m = lm
    gen = seeded(16)
    lens = [5, 70, 33, 1]
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in lens]
    ids, mask = _right_padded(prompts, 128)
    with torch.no_grad():
        hidden, cache = m.model(ids, use_cache=True, attention_mask=mask)
        for r, p in enumerate(prompts):
            row_ids = torch.tensor([p], device="cuda")
            h1, c1 = m.model(row_ids, use_cache=True)
            assert rel_l2(hidden[r, :len(p)], h1[0]) < 1e-2, r
            for layer, (cb, cr) in enumerate(zip(cache, c1)):
                for a, b in zip(cb["recurrent_state"], cr["recurrent_state"]):
                    assert rel_l2(a[r], b[0]) < 1e-2, (r, layer)
                for a, b in zip(cb["conv_state"], cr["conv_state"]):
                    assert rel_l2(a[r], b[0]) < 1e-2, (r, layer)
        last = torch.stack([hidden[r, len(p) - 1] for r, p in enumerate(prompts)])
        logits = m.lm_head(last)
    ref = torch.stack([_oracle_logits(cfg, m, torch.tensor([p]))[0, -1] for p in prompts])
    assert rel_l2(logits, ref) < 1e-2


def test_generate_batch_is_greedy_per_row():
    """generate_batch (one masked prefill, batched decode steps, independent
    stopping; reference generation.py:64-102) gives every prompt a greedy
    continuation: each token is the arg-max, up to bf16 near-ties, of the
    logits of that prompt and its earlier tokens run alone through the model.
    A row stops at its own end-of-sequence token."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from cyclic_flow_attention.generation import generate_batch
    from cyclic_flow_attention.models.cyfa import CyclicFlowAttentionConfig
    from cyclic_flow_attention.utils import initialize_model

    cfg = CyclicFlowAttentionConfig(hidden_size=256, num_heads=2, head_dim=128,
                                    num_hidden_layers=2, vocab_size=256)
    m = initialize_model(cfg, generator=seeded(20)).cuda().eval()
    gen = seeded(21)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist()
               for n in (3, 67, 20)]
    got = generate_batch(m, prompts, max_new_tokens=6)
    with torch.no_grad():
        for p, toks in zip(prompts, got):
            assert len(toks) == 6
            for i, tok in enumerate(toks):
                logits = m(torch.tensor([p + toks[:i]], device="cuda"))["logits"][0, -1].float()
                top = logits.max()
                # greedy up to a near-tie: within 1e-2 of the logits' scale of the maximum
                assert logits[tok] >= top - 1e-2 * logits.abs().max(), (i, tok)
    eos = got[1][2]
    stopped = generate_batch(m, prompts, max_new_tokens=6, eos_token_id=eos)
    for g, w in zip(stopped, got):
        assert g == (w[:w.index(eos) + 1] if eos in w else w)
    with pytest.raises(ValueError):
        generate_batch(m, [[]])
