"""Helpers shared by the GPU parity tests."""

import torch


def rel_l2(a, b):
    """Relative L2 error ||a - b|| / ||b|| in float64."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def bf16_cpu(x):
    """Rounds to bf16 and returns fp32 on the CPU (the values the GPU sees)."""
    return x.to(torch.bfloat16).float()


def seeded(seed):
    return torch.Generator().manual_seed(seed)


def suffix_terms(x, group=None):
    """Per-term form of a suffix (reverse) cumulative sum along the last dim:
    t_i = x_i - x_{i+1}, restarting every `group` elements (the last element of
    each group is its own term).  x = reverse cumsum of t within each group."""
    x = x.detach().double().cpu()
    n = x.shape[-1]
    nxt = torch.zeros_like(x)
    nxt[..., :-1] = x[..., 1:]
    if group:
        nxt[..., group - 1::group] = 0.0
    return x - nxt


def suffix_condition(terms, group=None):
    """Condition number of the suffix sums of `terms` (last dim, restarting every
    `group`): ||suffix sums of |terms| || / ||suffix sums of terms||.  If every
    term is accurate to a relative error e, the sums are accurate to e times this
    (the forward error bound of summation)."""
    t = terms.detach().double().cpu()
    n = t.shape[-1]
    g = group or n
    pad = (-n) % g
    tp = torch.nn.functional.pad(t, (0, pad)).reshape(*t.shape[:-1], -1, g)
    s = tp.flip(-1).cumsum(-1).flip(-1).reshape(*t.shape[:-1], -1)[..., :n]
    a = tp.abs().flip(-1).cumsum(-1).flip(-1).reshape(*t.shape[:-1], -1)[..., :n]
    return (a.norm() / s.norm().clamp_min(1e-300)).item()


def sum_condition(terms, dims):
    """||sum of |terms| over dims|| / ||sum of terms over dims||: the condition
    number of a parameter gradient that is a token sum of per-token terms."""
    t = terms.detach().double().cpu()
    return (t.abs().sum(dims).norm() / t.sum(dims).norm().clamp_min(1e-300)).item()


def _prefix(y, group=None):
    """Prefix (inclusive) sums along dim 2 of [B, H, T, ...], restarting every
    `group` steps."""
    T = y.shape[2]
    if not group:
        return y.cumsum(2)
    out = y.clone()
    for s in range(0, T, group):
        out[:, :, s:s + group] = y[:, :, s:s + group].cumsum(2)
    return out


def gate_param_tolerances(taps, x, params, tol=1e-2):
    """Bounds for the layer's gate/clock parameter gradients, which are token
    sums of the op's per-token gate terms.  dg is an in-tile suffix sum of terms
    dG_u (128-token tiles) and ddelta a suffix sum over the sequence of the clock
    terms dlam_s, so, exchanging the sums,
        dA_log  = sum_u dG_u  P(g)_u,        dt_bias = sum_u dG_u P(s)_u,
        a_proj  = sum_u dG_u  P(s x)_u,      s = dg/d(a + dt_bias),
        d_proj  = sum_s dlam_s Q(d' [x])_s,  d' = delta (1 - delta),
        b_proj  = sum_t dbeta_t b' [x]_t,    b' = beta (1 - beta),
    with P the in-tile and Q the whole-sequence prefix sums.  The op-level tests
    hold the terms dG, dlam and dbeta to `tol`; a sum of terms each within
    `tol` is within `tol` times its condition number (sum of |terms| over
    |sum|), computed here from the oracle's own terms."""
    perm = (0, 2, 1)
    g = taps["g"].detach().double().permute(*perm)
    dg = taps["g"].grad.double().permute(*perm)
    a = taps["a"].detach().double().permute(*perm)
    d = taps["delta"].detach().double().permute(*perm)
    dd = taps["delta"].grad.double().permute(*perm)
    gb = taps["bpre"].grad.double().permute(*perm)
    xs = x.detach().double().unsqueeze(1)                      # [B, 1, T, hidden]
    A = params["A_log"].detach().double().view(1, -1, 1)
    s = -A.exp() * torch.sigmoid(a)
    dG = suffix_terms(dg, 128)
    dlam = suffix_terms(dd)
    dp = d * (1 - d)
    bt = (0, 2)
    terms = {
        "A_log": dG * _prefix(g, 128),
        "dt_bias": dG * _prefix(s, 128),
        "a_proj.weight": dG.unsqueeze(-1) * _prefix(s.unsqueeze(-1) * xs, 128),
        "d_proj.bias": dlam * _prefix(dp),
        "d_proj.weight": dlam.unsqueeze(-1) * _prefix(dp.unsqueeze(-1) * xs),
        "b_proj.bias": gb,
        "b_proj.weight": gb.unsqueeze(-1) * xs,
    }
    return {n: tol * max(1.0, sum_condition(t, bt)) for n, t in terms.items()}
