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


def gate_param_tolerances(taps, x, params, tol=1e-2):
    """The gate/clock parameters' gradients are token sums of per-token terms
    (dL/dA_log = sum g dg; dt_bias, a_proj: the gradient at a + dt_bias; d_proj,
    b_proj: at their pre-activations, times x for the weights).  Those terms are
    held to `tol` by the op-level tests; a sum of terms each within `tol` is
    within `tol` times its condition number (sum of |terms| over |sum|), taken
    here from the oracle's own terms."""
    ga = taps["a"].grad.double()
    gd = taps["dpre"].grad.double()
    gb = taps["bpre"].grad.double()
    xs = x.double()
    bt = (0, 1)
    terms = {
        "A_log": taps["g"].grad.double() * taps["g"].detach().double(),
        "dt_bias": ga, "d_proj.bias": gd, "b_proj.bias": gb,
        "a_proj.weight": ga.unsqueeze(-1) * xs.unsqueeze(-2),
        "d_proj.weight": gd.unsqueeze(-1) * xs.unsqueeze(-2),
        "b_proj.weight": gb.unsqueeze(-1) * xs.unsqueeze(-2),
    }
    return {n: tol * max(1.0, sum_condition(t, bt)) for n, t in terms.items()}
