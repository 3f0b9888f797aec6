"""Builds the reference's own decode kernel for the GPU box -- TEST INFRASTRUCTURE.

The reference (Chyxx/CyFA-Jittor) generates its CUDA kernels as Python
f-strings and compiles them through Jittor's ``jt.code`` (its decode kernel:
cyclic_flow_attention/ops/fused_recurrent.py:55-188).  Jittor is not installed
here, so this script runs the reference's own ``fused_recurrent_cyfa`` from its
source file under the reference tree with a minimal stand-in for the few
``jittor`` calls it makes (``jt.flags``, ``jt.matmul``, ``jt.code``), captures
the CUDA source string it builds for a given shape, expands Jittor's
``@ARGS_DEF`` / ``@PRECALC`` / ``@ARGS`` macros and ``inN_p`` / ``inN_type``
names, and compiles it with nvcc for sm_100a into ``oracle/_ref/`` (git-ignored;
it travels to the GPU box like the library).  The kernel source is the
reference's, unmodified; only the host wrapper around it is written here.

Outputs, per configuration name:
    oracle/_ref/ref_decode_<name>.cu / .so   extern "C" int ref_decode(void** ins,
                                             void** outs, void* stream)
    oracle/_ref/ref_basis.cu / .so           extern "C" int ref_basis(...): the
                                             Fourier basis Phi [127, 128] f32
with ins = q, k, v, g, delta, beta, table [H,127,128] f32, q_norm_weight,
k_norm_weight, hk, hv, clock and outs = o, hk', hv', clock' (the reference's
jt.code input / output order).

Nothing in the product imports this file; ``tests/golden/make_golden.py`` runs
the built kernels on the GPU box to produce the golden vectors committed under
``tests/golden/``, and ``tests/test_gpu_ref_decode_c4.py`` runs the
configs[3]-shape build beside the library's decode step.  Run: ``python oracle/ref_build.py [reference_root]``.
"""

import importlib.util
import os
import subprocess
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF_ROOT = "/root/reference"
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "-cudart", "static"]

# configurations: (name, B, H, K, V, dtype) -- those of the golden vectors, and
# BASELINE configs[3]'s decode shape (batch 256, 8 heads of 256) for the
# full-size parity and timing comparison of tests/test_gpu_ref_decode_c4.py
CONFIGS = [
    ("bf16_k128", 1, 2, 128, 128, "bfloat16"),
    ("f32_k128", 1, 2, 128, 128, "float32"),
    ("bf16_k256", 1, 2, 256, 256, "bfloat16"),
    ("bf16_c4", 256, 8, 256, 256, "bfloat16"),
]
EPS = 1e-6


class _Var:
    """Shape/dtype stand-in for a jittor Var as fused_recurrent_cyfa uses it."""

    def __init__(self, shape, dtype="float32"):
        self.shape = tuple(shape)
        self.dtype = dtype

    def is_stop_grad(self):
        return True

    def stop_grad(self):
        return self

    def float32(self):
        return _Var(self.shape, "float32")


class _AnyModule(types.ModuleType):
    """Stand-in for a reference sibling module a captured file imports names
    from (``from .utils import bmm``); none of them is called."""

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return lambda *a, **k: None


def _fake_jittor(captured):
    jt = types.ModuleType("jittor")
    jt.flags = types.SimpleNamespace(no_grad=True, use_cuda=1)
    jt.Function = type("Function", (), {})

    def zeros(shape, dtype="float32"):
        return _Var(shape, dtype)

    def matmul(a, b):
        return _Var(a.shape[:-1] + (b.shape[-1],), "float32")

    def code(shapes, dtypes, inputs, cuda_src="", cuda_header=""):
        single = isinstance(dtypes, str)
        if single:
            shapes, dtypes = [shapes], [dtypes]
        captured.append(dict(shapes=shapes, dtypes=dtypes, inputs=inputs, src=cuda_src,
                             header=cuda_header))
        outs = [_Var(s, d) for s, d in zip(shapes, dtypes)]
        return outs[0] if single else outs

    jt.zeros, jt.matmul, jt.code = zeros, matmul, code
    return jt


def capture_decode_source(ref_root, B, H, K, V, dtype):
    """Runs the reference's fused_recurrent_cyfa for one shape and returns the
    jt.code call it makes (source, input and output dtypes)."""
    captured = []
    saved = {n: sys.modules.get(n) for n in ("jittor", "_cyfa_ref_ops", "_cyfa_ref_ops.chunk")}
    try:
        sys.modules["jittor"] = _fake_jittor(captured)
        pkg = types.ModuleType("_cyfa_ref_ops")
        pkg.__path__ = []
        chunk = types.ModuleType("_cyfa_ref_ops.chunk")
        chunk._basis = lambda M: _Var((M - 1, M), "float32")
        sys.modules["_cyfa_ref_ops"] = pkg
        sys.modules["_cyfa_ref_ops.chunk"] = chunk
        path = os.path.join(ref_root, "cyclic_flow_attention", "ops", "fused_recurrent.py")
        spec = importlib.util.spec_from_file_location("_cyfa_ref_ops.fused_recurrent", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        M = 128
        q = _Var((B, 1, H, K), dtype)
        k = _Var((B, 1, H, K), dtype)
        v = _Var((B, 1, H, V), dtype)
        g = _Var((B, 1, H))
        state = (_Var((B, H, K, M)), _Var((B, H, M, V)), _Var((B, H)))
        mod.fused_recurrent_cyfa(q, k, v, g, g, g, _Var((H, M - 1, M - 1)), _Var((K,)),
                                 _Var((K,)), EPS, EPS, None, state, True)
    finally:
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m
    if len(captured) != 1:
        raise RuntimeError(f"expected one jt.code call, got {len(captured)}")
    return captured[0]


def capture_basis_source(ref_root, M=128):
    """Runs the reference's ``_basis`` (ops/chunk.py:82-103), the kernel that
    builds the Fourier basis Phi [M-1, M], and returns its jt.code call."""
    captured = []
    names = ["jittor", "_cyfa_ref_ops"] + [f"_cyfa_ref_ops.{m}" for m in
                                           ("chunk_bwd", "chunk_h", "chunk_o", "chunk_readout",
                                            "qk_norm", "utils")]
    saved = {n: sys.modules.get(n) for n in names}
    try:
        sys.modules["jittor"] = _fake_jittor(captured)
        pkg = types.ModuleType("_cyfa_ref_ops")
        pkg.__path__ = []
        sys.modules["_cyfa_ref_ops"] = pkg
        for n in names[2:]:
            sys.modules[n] = _AnyModule(n)
        path = os.path.join(ref_root, "cyclic_flow_attention", "ops", "chunk.py")
        spec = importlib.util.spec_from_file_location("_cyfa_ref_ops.chunk", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod._basis(M)
    finally:
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m
    if len(captured) != 1:
        raise RuntimeError(f"expected one jt.code call, got {len(captured)}")
    return captured[0]


_CTYPES = {"float32": "float", "bfloat16": "__nv_bfloat16"}


def expand(call, entry="ref_decode"):
    """Turns a captured jt.code call into a standalone .cu file: the kernel as
    the reference wrote it, Jittor's argument macros expanded, and an extern "C"
    host wrapper that makes the reference's launch on a given stream."""
    src = call["src"]
    n_in, n_out = len(call["inputs"]), len(call["shapes"])
    types_in = [_CTYPES[x.dtype] for x in call["inputs"]]
    types_out = [_CTYPES[d] for d in call["dtypes"]]
    args_def = ", ".join([f"in{i}_type* in{i}_p" for i in range(n_in)] +
                         [f"out{i}_type* out{i}_p" for i in range(n_out)])
    args = ", ".join([f"in{i}_p" for i in range(n_in)] + [f"out{i}_p" for i in range(n_out)])
    lines = src.strip("\n").split("\n")
    launch = [i for i, line in enumerate(lines) if "<<<" in line]
    if len(launch) != 1:
        raise RuntimeError("expected exactly one kernel launch in the captured source")
    kernel = "\n".join(lines[:launch[0]]).replace("@ARGS_DEF", args_def).replace("@PRECALC", "")
    call_line = lines[launch[0]].strip().replace("@ARGS", args)
    # the reference launches on Jittor's stream; the wrapper passes the caller's
    name, rest = call_line.split("<<<", 1)
    config, tail = rest.split(">>>", 1)
    call_line = f"{name}<<<{config}, 0, (cudaStream_t)stream>>>{tail}"
    typedefs = "\n".join([f"typedef {t} in{i}_type;" for i, t in enumerate(types_in)] +
                         [f"typedef {t} out{i}_type;" for i, t in enumerate(types_out)])
    unpack = "\n".join([f"  in{i}_type* in{i}_p = (in{i}_type*)ins[{i}];" for i in range(n_in)] +
                       [f"  out{i}_type* out{i}_p = (out{i}_type*)outs[{i}];"
                        for i in range(n_out)])
    return (
        "// Generated by oracle/ref_build.py from the reference's own kernel source\n"
        "// (cyclic_flow_attention/ops/fused_recurrent.py:55-188, ops/chunk.py:82-103),\n"
        "// Jittor's argument macros expanded.  Test infrastructure.\n"
        "#include <cuda_bf16.h>\n#include <cuda_runtime.h>\n" + call.get("header", "") + "\n" +
        typedefs + "\n" + kernel + "\n\n"
        f'extern "C" int {entry}(void** ins, void** outs, void* stream) {{\n' + unpack + "\n  " +
        call_line + "\n  return (int)cudaGetLastError();\n}\n")


def build(ref_root=REF_ROOT, nvcc="nvcc"):
    """Captures and compiles every configuration into oracle/_ref/."""
    if not os.path.isdir(os.path.join(ref_root, "cyclic_flow_attention")):
        raise FileNotFoundError(f"reference tree not found under {ref_root}")
    os.makedirs(OUT, exist_ok=True)
    jobs = [("ref_basis", expand(capture_basis_source(ref_root), "ref_basis"))]
    for name, B, H, K, V, dtype in CONFIGS:
        jobs.append((f"ref_decode_{name}",
                     expand(capture_decode_source(ref_root, B, H, K, V, dtype))))
    built = []
    for stem, text in jobs:
        cu = os.path.join(OUT, stem + ".cu")
        so = os.path.join(OUT, stem + ".so")
        old = open(cu).read() if os.path.exists(cu) else None
        if old != text or not os.path.exists(so):
            with open(cu, "w") as f:
                f.write(text)
            subprocess.run([nvcc, *NVCC_FLAGS, "-o", so, cu], check=True)
        built.append(so)
    return built


if __name__ == "__main__":
    for path in build(sys.argv[1] if len(sys.argv) > 1 else REF_ROOT):
        print(path)
