"""CPU oracle for the CyFA hot path -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker of the repository.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` / reference arm
may import it, and only to check or to time the reference algorithm on host
cores.  The product path (``cyclic_flow_attention`` under ``cyfa-jittor_b200``)
never imports it and fails loudly when its CUDA library is missing.

It restates, in plain PyTorch-CPU arithmetic (float64 for the known-answer
tests, float32 as the reference's fp32 path), the algorithm of the reference
package ``cyclic_flow_attention`` (Chyxx/CyFA-Jittor).  Every function cites the
reference file:line it follows.  Gradients come from torch autograd through the
restatement.

Parity pin: the reference needs Jittor plus a CUDA GPU and has no CPU path, and
it ships no golden vectors.  Its kernels are CUDA source strings, though:
``oracle/ref_build.py`` builds its decode kernel (ops/fused_recurrent.py:55-188)
and Fourier-basis kernel (ops/chunk.py:82-103) from the reference's own source
for sm_100a, and ``tests/golden/make_golden.py`` ran them on a B200 over seeded
sequences.  ``tests/test_golden.py`` pins this restatement to those outputs: the
decode step and the chunkwise forward reproduce the reference's token-by-token
results to 1e-4 in fp32 (measured 4e-6) and 1e-2 in bf16.  The restatement is
also checked against the paper's own definition (the relative-time recurrence
of README.md:32-106) and internal identities (chunkwise == token recurrence,
clock wrap invariance) in ``tests/test_oracle.py``.  Gradients come from
autograd through the pinned forward.
"""

import math

import torch

__all__ = [
    "basis",
    "readout_table",
    "clock_scan",
    "phase_cos_sin",
    "write_vector",
    "rotate",
    "head_rmsnorm",
    "scalar_la_chunk",
    "scalar_la_recurrent",
    "modal_readout",
    "chunk_cyfa",
    "fused_recurrent_cyfa",
    "relative_time_reference",
    "short_convolution",
    "gated_rmsnorm",
    "cyfa_layer",
    "cyfa_lm",
]


def basis(M, dtype=torch.float64):
    """Real Fourier basis Phi [M-1, M] (ops/chunk.py:82-103).

    Row r, column c: pair = c // 2, phase = r * 2*pi*pair/(M-1); even columns
    hold cos, odd columns sin; column 1 is identically zero; scale
    (M-1)^-1/2 for the first pair, (2/(M-1))^1/2 otherwise.
    """
    period = M - 1
    row = torch.arange(period, dtype=dtype).unsqueeze(1)
    col = torch.arange(M)
    pair = (col // 2).to(dtype)
    phase = row * (pair * (2 * math.pi / period)).unsqueeze(0)
    z = torch.where((col % 2 == 1).unsqueeze(0), torch.sin(phase), torch.cos(phase))
    scale = torch.full((M,), (2.0 / period) ** 0.5, dtype=dtype)
    scale[:2] = period ** -0.5
    out = z * scale.unsqueeze(0)
    out[:, 1] = 0.0
    return out


def readout_table(readout, dtype=torch.float64):
    """Table_h = R_h . Phi, [H, M-1, M] (ops/chunk.py:281)."""
    M = readout.shape[-1] + 1
    return readout.to(dtype) @ basis(M, dtype)


def clock_scan(delta, clock=None):
    """lambda_t = clock_0 + sum_{s<=t} delta_s over T, delta [B,H,T]
    (ops/utils.py:229-302 ClockScan; ops/chunk.py:254-256 clock offset)."""
    lam = torch.cumsum(delta, dim=-1)
    if clock is not None:
        lam = lam + clock.unsqueeze(-1)
    return lam


def phase_cos_sin(lam, M):
    """Per-pair cos/sin of the write/readout phase (ops/chunk.py:268-274).

    coord_p = ((floor(lam) mod (M-1)) * p mod (M-1)) + frac(lam) * p, wrapped to
    (-(M-1)/2, (M-1)/2]; phi = coord * 2*pi/(M-1).  The integer part is taken
    exactly (int64), so the phase is the exact angle 2*pi*p*lam/(M-1) mod 2*pi
    evaluated without losing precision for large lam.  The floor has zero
    derivative, so d phi/d lam = 2*pi*p/(M-1) (ops/utils.py:613-615).
    """
    R = M - 1
    pair = torch.arange(M // 2, dtype=torch.int64)
    whole = torch.floor(lam.detach())
    wi = torch.remainder(whole.to(torch.int64), R).unsqueeze(-1)
    frac = (lam - whole).unsqueeze(-1)
    coord = torch.remainder(wi * pair, R).to(lam.dtype) + frac * pair.to(lam.dtype)
    coord = torch.where(coord > R * 0.5, coord - R, coord)
    phase = coord * (2 * math.pi / R)
    return torch.cos(phase), torch.sin(phase)


def write_vector(lam, beta, M):
    """w_t = beta_t U(-lam_t) b, [.., M] (ops/chunk.py:275-279; compact kernel
    ops/utils.py:554-577): w[2p] = beta s_p cos(phi_p), w[2p+1] = -beta s_p sin(phi_p)."""
    c, s = phase_cos_sin(lam, M)
    R = M - 1
    pair = torch.arange(M // 2)
    atom_scale = torch.where(pair == 0, 1.0, 2.0).to(lam.dtype).div(R).sqrt()
    atom = torch.stack([atom_scale * c, -atom_scale * s], dim=-1)
    return beta.unsqueeze(-1) * atom.reshape(lam.shape + (M,)), c, s


def rotate(x, c, s, negative=False):
    """Per-pair 2x2 rotation U(+-lam) (ops/chunk.py:115-124)."""
    pairs = x.reshape(x.shape[:-1] + (x.shape[-1] // 2, 2))
    e, o = pairs[..., 0], pairs[..., 1]
    if negative:
        y0, y1 = c * e + s * o, -s * e + c * o
    else:
        y0, y1 = c * e - s * o, s * e + c * o
    return torch.stack([y0, y1], dim=-1).reshape(x.shape)


def head_rmsnorm(x, w, eps):
    """Per-head RMSNorm of [B,T,H,D] -> [B,H,T,D] (ops/qk_norm.py:206-239)."""
    xf = x.to(w.dtype) if w.dtype.is_floating_point else x
    rs = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * rs * w).permute(0, 2, 1, 3)


def scalar_la_chunk(q, k, v, g, initial, C, scale=1.0, bf16_points=False):
    """Chunkwise scalar-gated linear attention (ops/chunk.py:136-161).

    q,k [B,H,T,K], v [B,H,T,V], g [B,H,T] (natural-log decay), initial
    [B,H,K,V].  Returns (out [B,H,T,V], final [B,H,K,V]).  T % C == 0.
    ``bf16_points`` rounds what the reference's bf16 path rounds here: the
    decayed values of the state update (``v_tail``, :147), the chunk states read
    by the inter-chunk term (``states.cast``, :150) and the masked scores (:155).
    """
    B, H, T, K = q.shape
    V = v.shape[-1]
    N = T // C
    qc = q.reshape(B, H, N, C, K)
    kc = k.reshape(B, H, N, C, K)
    vc = v.reshape(B, H, N, C, V)
    gc = g.reshape(B, H, N, C).cumsum(-1)
    last = gc[..., -1]
    tails = (last.unsqueeze(-1) - gc).exp()
    updates = kc.transpose(-1, -2) @ _rp(vc * tails.unsqueeze(-1), bf16_points)
    decays = last.exp()
    states = []
    h = initial
    for n in range(N):  # affine scan, ops/utils.py:145-176
        states.append(h)
        h = h * decays[:, :, n, None, None] + updates[:, :, n]
    states = torch.stack(states, dim=2)
    inter = (qc @ _rp(states, bf16_points)) * gc.exp().unsqueeze(-1)
    scores = qc @ kc.transpose(-1, -2)
    i = torch.arange(C)
    mask = i.reshape(C, 1) >= i.reshape(1, C)
    decay = (gc.unsqueeze(-1) - gc.unsqueeze(-2)).masked_fill(~mask, 0.0).exp()
    scores = _rp(torch.where(mask, scores * decay, torch.zeros((), dtype=scores.dtype)),
                 bf16_points)
    intra = scores @ vc
    out = (inter + intra) * scale
    return out.reshape(B, H, T, V), h


def scalar_la_recurrent(q, k, v, g, initial, scale=1.0):
    """Token-by-token form of the same recurrence: S_t = a_t S_{t-1} + k_t v_t^T,
    o_t = scale q_t S_t.  Used only as a known-answer check of the chunk form."""
    B, H, T, K = q.shape
    h = initial
    outs = []
    for t in range(T):
        h = h * g[:, :, t, None, None].exp() + k[:, :, t, :, None] * v[:, :, t, None, :]
        outs.append(torch.einsum("bhk,bhkv->bhv", q[:, :, t], h) * scale)
    return torch.stack(outs, dim=2), h


def modal_readout(raw, c, s, table):
    """Middle readout (ops/chunk.py:320-331): z = U(lam) raw, logits = z Table^T
    over the M-1 active rows, p = softmax, coeff = p Table, weights = U(-lam) coeff.
    raw [B,H,T,M], table [H,M-1,M]."""
    z = rotate(raw, c, s)
    logits = torch.einsum("bhtm,hrm->bhtr", z, table)
    probs = torch.softmax(logits, dim=-1)
    coeff = torch.einsum("bhtr,hrm->bhtm", probs, table)
    return rotate(coeff, c, s, negative=True)


class _RoundBf16(torch.autograd.Function):
    """Rounds to bf16 in the forward and passes the gradient straight through:
    the value a bf16 tensor stored by the reference's bf16 path holds, with the
    gradient its backward formulas use."""

    @staticmethod
    def forward(ctx, x):
        return x.to(torch.bfloat16).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        return g


def _rp(x, on):
    return _RoundBf16.apply(x) if on else x


def _pad_time(x, padding):
    if not padding:
        return x
    shape = list(x.shape)
    shape[1] = padding
    return torch.cat([x, torch.zeros(shape, dtype=x.dtype)], dim=1)


def chunk_cyfa(
    q, k, v, g, delta, beta, readout, q_norm_weight, k_norm_weight,
    q_norm_eps=1e-6, k_norm_eps=1e-6, scale=None, initial_state=None,
    output_final_state=False, chunk_size=64, dtype=None, bf16_points=False,
):
    """Chunkwise CyFA, generic path (ops/chunk.py:164-353).

    q,k [B,T,H,K], v [B,T,H,V], g/delta/beta [B,T,H], readout [H,M-1,M-1].
    Computes in ``dtype`` (default: q's floating dtype).  Returns (o [B,T,H,V],
    (hk [B,H,K,M], hv [B,H,M,V], clock [B,H]) or None).

    ``bf16_points`` rounds to bf16 (straight-through gradient) the tensors the
    reference's bf16 path stores in bf16: the normalised q/k (qk_norm.py output
    dtype), the write vector (ops/chunk.py:279, ops/utils.py:575), the pass-1
    output raw (``round_output``, chunk.py:316-319), the rotated z, the table,
    the probabilities and the weights (utils.py:804-853, chunk.py:324-331), the
    decayed values, chunk states and scores of both passes (``scalar_la_chunk``),
    and the output.  It measures how far those rounding points alone move a result:
    the conditioning of each gradient under bf16 storage.
    """
    rp = bf16_points
    dt = dtype or (q.dtype if q.dtype in (torch.float32, torch.float64) else torch.float32)
    q, k, v, g, delta, beta = (x.to(dt) for x in (q, k, v, g, delta, beta))
    B, T, H, K = q.shape
    V = v.shape[-1]
    M = readout.shape[-1] + 1
    C = chunk_size
    padding = (-T) % C  # ops/chunk.py:198-207
    q, k, v, g, delta, beta = (_pad_time(x, padding) for x in (q, k, v, g, delta, beta))
    q = _rp(head_rmsnorm(q, q_norm_weight.to(dt), q_norm_eps), rp)  # chunk.py:226
    k = _rp(head_rmsnorm(k, k_norm_weight.to(dt), k_norm_eps), rp)  # chunk.py:227
    v = v.permute(0, 2, 1, 3)
    g, d, beta = (x.permute(0, 2, 1) for x in (g, delta, beta))  # head_gates, chunk.py:243
    if initial_state is None:
        hk = torch.zeros(B, H, K, M, dtype=dt)
        hv = torch.zeros(B, H, M, V, dtype=dt)
        clock = None
    else:
        hk, hv, clock = (x.to(dt) for x in initial_state)
    lam = clock_scan(d, clock)  # chunk.py:254-256
    write, c, s = write_vector(lam, beta, M)  # chunk.py:265-279
    write = _rp(write, rp)
    sc = K ** -0.5 if scale is None else scale
    raw, hkt = scalar_la_chunk(q, k, write, g, hk, C, sc, rp)  # pass 1, chunk.py:316-319
    table = readout_table(readout, dt)  # chunk.py:320
    if rp:
        z = _rp(rotate(_rp(raw, rp), c, s), rp)
        tb = _rp(table, rp)
        probs = _rp(torch.softmax(torch.einsum("bhtm,hrm->bhtr", z, tb), dim=-1), rp)
        weights = _rp(rotate(torch.einsum("bhtr,hrm->bhtm", probs, tb), c, s, negative=True), rp)
    else:
        weights = modal_readout(raw, c, s, table)  # chunk.py:324-331
    out, hvt = scalar_la_chunk(weights, write, v, g, hv, C, 1.0, rp)  # pass 2, chunk.py:338
    out = _rp(out.permute(0, 2, 1, 3)[:, :T], rp)
    state = None
    if output_final_state:  # chunk.py:347-352
        final_clock = d.sum(-1)
        if clock is not None:
            final_clock = final_clock + clock
        state = (hkt, hvt, final_clock)
    return out, state


def fused_recurrent_cyfa(
    q, k, v, g, delta, beta, readout, q_norm_weight, k_norm_weight,
    q_norm_eps=1e-6, k_norm_eps=1e-6, scale=None, initial_state=None,
    output_final_state=False, dtype=torch.float32, bf16_points=False,
):
    """One decode step, T=1 (ops/fused_recurrent.py:10-200, kernel :55-188).

    Same math as chunk_cyfa for one token: q/k RMSNorm, lam = clock + delta,
    hk = a hk + k w^T, raw = scale hk^T q, readout, hv = a hv + w v^T,
    o = hv^T weights.  Returns (o [B,1,H,V], (hk, hv, clock) or None).
    ``bf16_points`` rounds to bf16 where the reference's kernel casts to the
    bf16 input type: the normalised q and k (:84-85), the write vector (:97,
    :172), the rotated raw vector (:118), the table in both products (:126,
    :150), the probabilities (:150), the weights (:170) and the output (:187).
    """
    rp = bf16_points
    B, T, H, K = q.shape
    if T != 1:
        raise NotImplementedError("decode step needs T=1")
    V = v.shape[-1]
    M = readout.shape[-1] + 1
    q, k, v, g, delta, beta = (x.to(dtype) for x in (q, k, v, g, delta, beta))
    if initial_state is None:
        hk = torch.zeros(B, H, K, M, dtype=dtype)
        hv = torch.zeros(B, H, M, V, dtype=dtype)
        clock = torch.zeros(B, H, dtype=dtype)
    else:
        hk, hv, clock = (x.to(dtype) for x in initial_state)
    sc = K ** -0.5 if scale is None else scale
    qn = _rp(head_rmsnorm(q, q_norm_weight.to(dtype), q_norm_eps)[:, :, 0], rp)  # [B,H,K]
    kn = _rp(head_rmsnorm(k, k_norm_weight.to(dtype), k_norm_eps)[:, :, 0], rp)
    lam = clock + delta[:, 0]  # fused_recurrent.py:91
    alpha = g[:, 0].exp()
    w, c, s = write_vector(lam, beta[:, 0], M)
    w = _rp(w, rp)
    hk = hk * alpha[..., None, None] + kn[..., :, None] * w[..., None, :]  # :105-109
    raw = torch.einsum("bhkm,bhk->bhm", hk, qn * sc)
    table = readout_table(readout, dtype)
    if rp:
        z = _rp(rotate(raw, c, s), rp)
        tb = _rp(table, rp)
        probs = _rp(torch.softmax(torch.einsum("bhm,hrm->bhr", z, tb), dim=-1), rp)
        weights = _rp(rotate(torch.einsum("bhr,hrm->bhm", probs, tb), c, s, negative=True), rp)
    else:
        weights = modal_readout(raw.unsqueeze(2), c.unsqueeze(2), s.unsqueeze(2), table)[:, :, 0]
    hv = hv * alpha[..., None, None] + w[..., :, None] * v[:, 0][..., None, :]  # :177-184
    o = _rp(torch.einsum("bhmv,bhm->bhv", hv, weights).unsqueeze(1), rp)
    return o, ((hk, hv, lam) if output_final_state else None)


def relative_time_reference(q, k, v, g, delta, beta, readout, scale, M):
    """The paper's relative-time recurrence (README.md:32-56), float64.

    K_t = a_t P(delta_t) K_{t-1} + beta_t e_0 k_t^T, V_t likewise, with the
    fractional cyclic shift P(d) = Phi U(d) Phi^T; o_t = (R V_t)^T softmax(R K_t
    q_t).  q,k [B,H,T,K] already normalised, v [B,H,T,V], g/delta/beta [B,H,T].
    Independent of the absolute-clock two-pass form, so it pins that form.
    """
    B, H, T, K = q.shape
    V = v.shape[-1]
    R = M - 1
    phi = basis(M)  # [R, M]
    pair = torch.arange(M // 2, dtype=torch.float64)
    Kst = torch.zeros(B, H, R, K, dtype=torch.float64)
    Vst = torch.zeros(B, H, R, V, dtype=torch.float64)
    outs = []
    for t in range(T):
        ang = 2 * math.pi * pair * delta[:, :, t, None] / R  # exact additive phase
        c, s = torch.cos(ang), torch.sin(ang)
        # U(d) as a [B,H,M,M] block-diagonal matrix acting on column vectors
        U = torch.zeros(B, H, M, M, dtype=torch.float64)
        idx = torch.arange(M // 2)
        U[:, :, 2 * idx, 2 * idx] = c
        U[:, :, 2 * idx, 2 * idx + 1] = -s
        U[:, :, 2 * idx + 1, 2 * idx] = s
        U[:, :, 2 * idx + 1, 2 * idx + 1] = c
        P = phi @ U @ phi.T  # [B,H,R,R]
        a = g[:, :, t].exp()[..., None, None]
        e0 = torch.zeros(R, dtype=torch.float64)
        e0[0] = 1.0
        Kst = a * (P @ Kst) + beta[:, :, t, None, None] * e0[:, None] * k[:, :, t, None, :]
        Vst = a * (P @ Vst) + beta[:, :, t, None, None] * e0[:, None] * v[:, :, t, None, :]
        logits = torch.einsum("hrs,bhsk,bhk->bhr", readout, Kst, q[:, :, t]) * scale
        p = torch.softmax(logits, dim=-1)
        outs.append(torch.einsum("hrs,bhsv,bhr->bhv", readout, Vst, p))
    return torch.stack(outs, dim=2)


def short_convolution(x, weight, bias=None, cache=None):
    """Causal depthwise conv, no activation (layers/cyfa.py:144-181).

    x [B,T,D], weight [D,1,W]; y_t = sum_i w_i x_{t-(W-1)+i}; with a cache the
    history is concat(cache, x).  Returns (y, new_cache = last W-1 rows)."""
    B, T, D = x.shape
    W = weight.shape[-1]
    history = x if cache is None else torch.cat([cache.to(x.dtype), x], dim=1)
    offset = W - 1 if cache is None else 0
    padded = torch.cat([torch.zeros(B, offset, D, dtype=x.dtype), history], dim=1)
    y = torch.zeros(B, T, D, dtype=x.dtype)
    for i in range(W):
        y = y + padded[:, i:i + T] * weight[:, 0, i].to(x.dtype)
    if bias is not None:
        y = y + bias.to(x.dtype)
    return y, history[:, -(W - 1):] if W > 1 else history[:, :0]


def gated_rmsnorm(x, weight, eps, gate=None):
    """RMSNorm with optional sigmoid gate (layers/cyfa.py:62-84)."""
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight.to(x.dtype)
    if gate is not None:
        y = y * torch.sigmoid(gate.to(x.dtype))
    return y


def cyfa_layer(params, x, H, head_k_dim, head_v_dim, num_slots=128, eps=1e-6,
               chunk_size=64, conv=True, bf16_points=False, taps=None):
    """CyclicFlowAttention.execute training path (layers/cyfa.py:299-357).

    ``params`` maps the reference's parameter names (q_proj.weight, ...) to
    tensors.  x [B,T,hidden].  Returns y [B,T,hidden].  ``bf16_points`` as in
    ``chunk_cyfa``, plus the bf16 activations between the layer's GEMMs
    (projection outputs, convolution outputs, gate input).  ``taps``, a dict,
    receives the gate tensors g, delta, beta and the gate pre-activations
    (a + dt_bias, the d and b projections), with their gradients retained.
    """
    rp = bf16_points
    dt = x.dtype
    P = {n: t.to(dt) for n, t in params.items()}
    B, T, _ = x.shape
    q = _rp(x @ P["q_proj.weight"].T, rp)
    k = _rp(x @ P["k_proj.weight"].T, rp)
    v = _rp(x @ P["v_proj.weight"].T, rp)
    if conv:
        q = _rp(short_convolution(q, P["q_conv1d.weight"])[0], rp)
        k = _rp(short_convolution(k, P["k_conv1d.weight"])[0], rp)
        v = _rp(short_convolution(v, P["v_conv1d.weight"])[0], rp)
    q = q.reshape(B, T, H, head_k_dim)
    k = k.reshape(B, T, H, head_k_dim)
    v = v.reshape(B, T, H, head_v_dim)
    a = x @ P["a_proj.weight"].T + P["dt_bias"]
    g = -P["A_log"].exp() * torch.nn.functional.softplus(a)
    dpre = x.detach() @ P["d_proj.weight"].T + P["d_proj.bias"]
    bpre = x @ P["b_proj.weight"].T + P["b_proj.bias"]
    delta = torch.sigmoid(dpre)
    beta = torch.sigmoid(bpre)
    if taps is not None:
        for name, t in (("a", a), ("g", g), ("dpre", dpre), ("bpre", bpre), ("delta", delta),
                        ("beta", beta)):
            if t.requires_grad:
                t.retain_grad()
            taps[name] = t
    o, _ = chunk_cyfa(q, k, v, g, delta, beta, P["readout"], P["q_norm.weight"],
                      P["k_norm.weight"], eps, eps, chunk_size=chunk_size, dtype=dt,
                      bf16_points=rp)
    gate = _rp(x @ P["g_proj.0.weight"].T, rp) @ P["g_proj.1.weight"].T + P["g_proj.1.bias"]
    gate = gate.reshape(B, T, H, head_v_dim)
    o = gated_rmsnorm(o * (num_slots - 1), P["o_norm.weight"], eps, gate)
    return o.reshape(B, T, H * head_v_dim) @ P["o_proj.weight"].T


def cyfa_lm(params, ids, num_layers, H, head_k_dim, head_v_dim, num_slots=128, eps=1e-6,
            chunk_size=64, dtype=torch.float32):
    """CyclicFlowAttentionForCausalLM.execute without cache: embedding, blocks of
    attn_norm -> attention -> residual, mlp_norm -> SwiGLU MLP -> residual, final
    norm, lm_head (models/cyfa/modeling_cyfa.py:13-116).  ``params`` maps the
    reference's state-dict names to tensors; ids [B,T] -> logits [B,T,vocab]."""
    P = {n: t.to(dtype) for n, t in params.items()}
    x = P["model.embeddings.weight"][ids]
    for i in range(num_layers):
        pre = f"model.layers.{i}."
        attn = {n[len(pre) + 5:]: t for n, t in P.items() if n.startswith(pre + "attn.")}
        h = gated_rmsnorm(x, P[pre + "attn_norm.weight"], eps)
        x = x + cyfa_layer(attn, h, H, head_k_dim, head_v_dim, num_slots, eps, chunk_size)
        h = gated_rmsnorm(x, P[pre + "mlp_norm.weight"], eps)
        g = h @ P[pre + "mlp.gate_proj.weight"].T
        u = h @ P[pre + "mlp.up_proj.weight"].T
        x = x + (g * torch.sigmoid(g) * u) @ P[pre + "mlp.down_proj.weight"].T
    x = gated_rmsnorm(x, P["model.norm.weight"], eps)
    return x @ P["lm_head.weight"].T
