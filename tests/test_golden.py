"""Pins the oracle to outputs of the reference's OWN kernels (CPU test).

tests/golden/ref_decode.npz holds what the reference's decode kernel
(cyclic_flow_attention/ops/fused_recurrent.py:55-188) and its Fourier-basis
kernel (ops/chunk.py:82-103) computed on a B200, built from the reference's
source by oracle/ref_build.py and run by tests/golden/make_golden.py: for each
seeded case, every token's output of a sequence decoded step by step from a
seeded state, the final clock and a fingerprint of the final states.

The oracle's decode step must reproduce them: fp32 cases to 1e-4 (the
reference computes in fp32 there); bf16 cases to 1e-2, with the oracle rounding
where the reference's kernel rounds (``bf16_points``: measured 0.1-0.2 % on the
outputs) and without (0.3-0.4 %).
The oracle's chunkwise forward over the whole sequence must reproduce the
reference's token-by-token decode at every token: fp32 to 1e-4, bf16 to 1e-2
(final-state checks on sampled entries: sums over the slot dimension cancel,
which magnifies the reference's bf16 rounding of the write vector).  The
reference's own test pins decode to the chunkwise forward the same way
(tests/test_inference.py:20-34)."""

import os
import sys

import numpy as np
import pytest
import torch

from gpu_util import rel_l2
from oracle import cyfa_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from golden_cases import CASES, EPS, case_inputs, summarize_state  # noqa: E402

GOLDEN = os.path.join(HERE, "golden", "ref_decode.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def _tol(case):
    return 1e-4 if case[5] == torch.float32 else 1e-2


def _table(gold, readout):
    return readout.double() @ torch.from_numpy(gold["basis"]).double()


def test_basis_matches_reference_kernel(gold):
    # the reference forms the phase in fp32 (ops/chunk.py:88-93); the oracle in fp64
    assert rel_l2(O.basis(128), torch.from_numpy(gold["basis"])) < 1e-5


def _check(case, gold, o, hk, hv, clock, tol, sums=True):
    name = case[0]
    assert rel_l2(o, torch.from_numpy(gold[f"{name}.o"])) < tol, name
    assert rel_l2(clock, torch.from_numpy(gold[f"{name}.clock"])) < 1e-6, name
    for k, v in summarize_state(case, hk, hv).items():
        if sums or k.endswith("sample"):
            assert rel_l2(v, torch.from_numpy(gold[f"{name}.{k}"])) < tol, (name, k)


def _decode(case, rounding):
    x = case_inputs(case)
    f = torch.float64
    state = (x["hk0"].to(f), x["hv0"].to(f), x["clock0"].to(f))
    outs = []
    for t in range(case[7]):
        sl = [x[n][:, t:t + 1].to(f) for n in ("q", "k", "v", "g", "delta", "beta")]
        o, state = O.fused_recurrent_cyfa(*sl, x["readout"].to(f), x["qw"].to(f),
                                          x["kw"].to(f), EPS, EPS, initial_state=state,
                                          output_final_state=True, dtype=f,
                                          bf16_points=rounding)
        outs.append(o)
    return torch.cat(outs, 1), state


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_decode_matches_reference_kernel(case, gold):
    bf16 = case[5] == torch.bfloat16
    o, state = _decode(case, False)
    _check(case, gold, o, *state, _tol(case), sums=not bf16)
    if bf16:  # rounding where the reference's kernel rounds: the slot sums agree too
        o, state = _decode(case, True)
        _check(case, gold, o, *state, 1e-2)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_chunk_forward_matches_reference_kernel(case, gold):
    """The chunkwise two-pass form over the whole sequence equals the
    reference's token-by-token decode at every token."""
    x = case_inputs(case)
    f = torch.float64
    ins = [x[n].to(f) for n in ("q", "k", "v", "g", "delta", "beta", "readout", "qw", "kw")]
    o, (hk, hv, clock) = O.chunk_cyfa(*ins, EPS, EPS, initial_state=(
        x["hk0"].to(f), x["hv0"].to(f), x["clock0"].to(f)), output_final_state=True, dtype=f)
    _check(case, gold, o, hk, hv, clock, _tol(case), sums=case[5] == torch.float32)
