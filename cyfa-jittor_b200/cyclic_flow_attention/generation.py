"""Autoregressive generation with the constant-size recurrent state.

``generate`` and ``generate_batch`` mirror the reference's functions
(cyclic_flow_attention/generation.py:23-102): same arguments, validation and
results.  ``GraphedDecoder`` is the throughput path: the whole decode step of
the model (embedding, every layer, final norm, lm_head, greedy argmax) captured
once into a CUDA graph that updates the cache in place and feeds its argmax back
as the next step's input, so a step costs one graph launch and no host
round trip.
"""

import torch


def _validate(ids, max_new_tokens, temperature=0.0, top_p=1.0):
    if not ids or max_new_tokens < 0 or temperature < 0 or not 0 < top_p <= 1:
        raise ValueError("Invalid prompt or sampling options")


@torch.no_grad()
def generate(model, ids, max_new_tokens=64, eos_token_id=None, temperature=0.0, top_p=1.0,
             seed=42, on_token=None):
    """One prompt (list of ids) -> list of new ids; greedy at temperature 0,
    else nucleus sampling from a seeded host generator (reference :23-61)."""
    _validate(ids, max_new_tokens, temperature, top_p)
    model.eval()
    dev = model.lm_head.weight.device
    rng = torch.Generator().manual_seed(seed)
    current, cache, generated = list(ids), None, []
    for _ in range(max_new_tokens):
        out = model(torch.tensor([current], device=dev), cache=cache, use_cache=True)
        logits = out["logits"][0, -1].double().cpu()
        cache = out["cache"]
        if temperature == 0:
            token = int(logits.argmax())
        else:
            probs = torch.softmax(logits / temperature, -1)
            order = torch.argsort(-probs)
            sorted_p = probs[order]
            keep = torch.cumsum(sorted_p, 0) - sorted_p < top_p
            order = order[keep]
            weights = probs[order] / probs[order].sum()
            token = int(order[torch.multinomial(weights, 1, generator=rng)])
        generated.append(token)
        if on_token is not None and on_token(generated):
            break
        if token == eos_token_id:
            break
        current = [token]
    return generated


@torch.no_grad()
def generate_batch(model, prompts, max_new_tokens=48, eos_token_id=None, on_token=None):
    """Greedy generation for right-padded prompts with independent stopping
    (reference :64-102): one masked prefill, then one decode step per token."""
    if not prompts or any(not ids for ids in prompts) or max_new_tokens < 0:
        raise ValueError("Expected nonempty prompts and a nonnegative generation length")
    model.eval()
    dev = model.lm_head.weight.device
    lengths = torch.tensor([len(p) for p in prompts])
    width = int((lengths.max() + 63) // 64 * 64)
    ids = torch.zeros(len(prompts), width, dtype=torch.long)
    mask = torch.zeros_like(ids)
    for row, tokens in enumerate(prompts):
        ids[row, :len(tokens)] = torch.tensor(tokens)
        mask[row, :len(tokens)] = 1
    generated = [[] for _ in prompts]
    finished = [False] * len(prompts)
    hidden, cache = model.model(ids.to(dev), use_cache=True, attention_mask=mask.to(dev))
    last = hidden[torch.arange(len(prompts), device=dev), (lengths - 1).to(dev)]
    logits = model.lm_head(last)
    for step in range(max_new_tokens):
        tokens = logits.argmax(-1).cpu().tolist()
        for row, token in enumerate(tokens):
            if finished[row]:
                continue
            generated[row].append(token)
            finished[row] = token == eos_token_id or bool(on_token and on_token(generated[row]))
        if all(finished) or step + 1 == max_new_tokens:
            break
        out = model(torch.tensor(tokens, device=dev)[:, None], cache=cache, use_cache=True)
        cache = out["cache"]
        logits = out["logits"][:, -1]
    return generated


class GraphedDecoder:
    """Greedy decoding of a batch of equal-length prompts, one CUDA graph replay
    per token.

    ``prefill(input_ids)`` runs the prompt through the model (chunkwise path),
    keeps its cache as the decoder's state (conv histories made contiguous) and
    captures the decode step over it: an eager warm-up step that leaves the
    cache untouched, then the in-place step with the argmax written back into
    the graph's input.  ``step()`` replays it; ``generate(input_ids, n)``
    returns the prompt's n greedy continuation tokens [B, n] on the device.
    The captured graph holds the cache tensors' addresses: a new prefill
    captures a new graph.
    """

    def __init__(self, model):
        self.model = model.eval()
        self.graph = None

    @torch.no_grad()
    def prefill(self, input_ids):
        m = self.model
        self.graph = None
        hidden, cache = m.model(input_ids, use_cache=True)
        first = m.lm_head(hidden[:, -1]).argmax(-1, keepdim=True)
        del hidden
        for c in cache:
            c["conv_state"] = tuple(t.contiguous() for t in c["conv_state"])
            c["recurrent_state"] = tuple(t.contiguous() for t in c["recurrent_state"])
        self.cache = cache
        self.ids = first.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            m.decode_step(self.ids, self.cache, inplace=False)  # packs weights, constants
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            logits, _ = m.decode_step(self.ids, self.cache, inplace=True)
            self.ids.copy_(logits.argmax(-1, keepdim=True))
        return first

    def step(self):
        """Consumes the current token of every row, returns the next [B, 1]."""
        self.graph.replay()
        return self.ids

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens):
        B = input_ids.shape[0]
        out = torch.empty(B, max_new_tokens, dtype=torch.long, device=input_ids.device)
        if max_new_tokens == 0:
            return out
        out[:, :1] = self.prefill(input_ids)
        for i in range(1, max_new_tokens):
            out[:, i:i + 1] = self.step()
        return out


__all__ = ["generate", "generate_batch", "GraphedDecoder"]
