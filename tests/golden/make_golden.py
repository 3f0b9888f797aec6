"""Generates the golden vectors of tests/golden/ from the reference's OWN
kernels, on a GPU box.

oracle/ref_build.py (run where the reference tree is present) compiles the
reference's decode kernel (cyclic_flow_attention/ops/fused_recurrent.py:55-188)
and its Fourier-basis kernel (ops/chunk.py:82-103) into oracle/_ref/; this
script loads them and runs, per case of golden_cases.CASES, the reference's
decode step token by token over a seeded sequence from a seeded initial
state: the reference's recurrent result for every token.  The readout table
is the reference's: its basis kernel's Phi times the readout, in fp32
(ops/fused_recurrent.py:51, jt.matmul).  It writes ref_decode.npz: the basis,
every token's output, the final clock and a fingerprint of the final states.

Run: python tests/golden/make_golden.py [output.npz]
"""

import ctypes
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from golden_cases import CASES, EPS, case_inputs, summarize_state  # noqa: E402

REF = os.path.join(ROOT, "oracle", "_ref")


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def reference_basis():
    lib = ctypes.CDLL(os.path.join(REF, "ref_basis.so"))
    out = torch.empty(127, 128, device="cuda")
    rc = lib.ref_basis(None, _ptrs([out]), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    if rc:
        raise RuntimeError(f"ref_basis failed: {rc}")
    return out


def run_case(case, basis):
    name, B, H, K, V, dtype, seed, T, _ = case
    lib = ctypes.CDLL(os.path.join(REF, f"ref_decode_{name}.so"))
    x = {n: t.cuda() for n, t in case_inputs(case).items()}
    table = torch.matmul(x["readout"].float(), basis).contiguous()  # [H, 127, 128]
    hk, hv, clock = x["hk0"].clone(), x["hv0"].clone(), x["clock0"].clone()
    outs = []
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for t in range(T):
        sl = lambda n: x[n][:, t:t + 1].contiguous()
        o = torch.empty(B, 1, H, V, device="cuda", dtype=dtype)
        hk2, hv2, clock2 = torch.empty_like(hk), torch.empty_like(hv), torch.empty_like(clock)
        ins = [sl("q"), sl("k"), sl("v"), sl("g"), sl("delta"), sl("beta"), table,
               x["qw"], x["kw"], hk, hv, clock]
        rc = lib.ref_decode(_ptrs(ins), _ptrs([o, hk2, hv2, clock2]), stream)
        if rc:
            raise RuntimeError(f"ref_decode {name} failed: {rc}")
        outs.append(o.float())
        hk, hv, clock = hk2, hv2, clock2
    torch.cuda.synchronize()
    res = {"o": torch.cat(outs, 1).cpu().numpy(), "clock": clock.double().cpu().numpy()}
    res.update({k: v.numpy() for k, v in summarize_state(case, hk, hv).items()})
    return res


def main(path):
    torch.backends.cuda.matmul.allow_tf32 = False
    basis = reference_basis()
    data = {"basis": basis.cpu().numpy()}
    for case in CASES:
        for k, v in run_case(case, basis).items():
            data[f"{case[0]}.{k}"] = v
    data["eps"] = np.array(EPS)
    np.savez_compressed(path, **data)
    print("wrote", path, sum(v.nbytes for v in data.values()), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_decode.npz"))
