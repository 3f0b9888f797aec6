"""ctypes binding of libcyfa.so, the sm_100a CUDA library behind the ops.

The library is built in-tree (``python __graft_entry__.py`` or ``make -C
cyfa-jittor_b200/csrc``).  There is no CPU fallback: if the library or a CUDA
device is missing, every op raises.
"""

import contextlib
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# CYFA_LIB selects another build of the library (e.g. to compare two builds in
# one process environment); the default is the in-tree libcyfa.so.
LIB_PATH = os.environ.get("CYFA_LIB") or os.path.join(_HERE, "libcyfa.so")

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float

# name -> argtypes (restype is int for all)
_SIGNATURES = {
    "cyfa_version": [],
    "cyfa_device_error": [_i],
    "cyfa_selftest_umma": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "cyfa_decode_step": [_vp] * 16 + [_i] * 5 + [_f] * 3 + [_vp],
    "cyfa_chunk_fwd_f32": [_vp] * 16 + [_i] * 5 + [_f] * 3 + [_vp],
    "cyfa_decode_layer": [_vp, _vp],
    "cyfa_gates_fwd": [_vp] * 8 + [_i] * 3 + [_vp],
    "cyfa_token_fwd": [_vp] * 11 + [_i] * 4 + [_f] * 2 + [_vp],
    "cyfa_token_bwd": [_vp] * 17 + [_i] * 4 + [_vp],
    "cyfa_gates_bwd": [_vp] * 8 + [_i] * 3 + [_vp],
    "cyfa_chunk_fwd": [_vp, _vp, ctypes.c_size_t, _vp],
    "cyfa_short_conv_fwd": [_vp, ctypes.c_longlong, _vp, _vp, _vp, _vp] + [_i] * 4 + [_vp],
    "cyfa_short_conv_bwd": [_vp, ctypes.c_longlong, _vp, _vp, _vp, ctypes.c_longlong, _vp, _vp]
    + [_i] * 4 + [_vp, ctypes.c_size_t, _vp],
    "cyfa_gate_act_fwd": [_vp, ctypes.c_longlong] * 3 + [_vp] * 7 + [_i, _i, _vp],
    "cyfa_gate_act_bwd": [_vp, ctypes.c_longlong] * 3 + [_vp] * 7
    + [_vp, ctypes.c_longlong] * 3 + [_vp] * 4 + [_i, _i, _vp, ctypes.c_size_t, _vp],
    "cyfa_gated_norm_fwd": [_vp, _vp, _vp, _f, _f, _vp, _vp, _i, _i, _vp],
    "cyfa_gated_norm_bwd": [_vp, _vp, _vp, _f, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp,
                            ctypes.c_size_t, _vp],
    "cyfa_gated_norm_bwd_static": [_vp, _vp, _vp, _f, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp],
    "cyfa_gated_norm_bias_fwd": [_vp, _vp, _vp, _i, _vp, _f, _f, _vp, _vp, _i, _i, _vp],
    "cyfa_gated_norm_gate_fwd": [_vp, _vp, ctypes.c_longlong, _vp, _vp, _i, _i, _vp, _f, _f,
                                 _vp, _vp, _vp, _i, _i, _vp],
    "cyfa_gated_norm_bias_bwd": [_vp, _vp, _vp, _i, _vp, _f, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _i, _i, _vp, ctypes.c_size_t, _vp],
    "cyfa_chunk_bwd": [_vp, _vp, ctypes.c_size_t, _vp, ctypes.c_size_t, _vp],
    "cyfa_readout_table": [_vp, _vp, _vp, _i, _vp],
    "cyfa_readout_table_grad": [_vp, _vp, _vp, _i, _vp],
    "cyfa_bucket_gather": [_vp, _i, _vp, _vp],
    "cyfa_bucket_scatter": [_vp, _i, _vp, _f, _vp],
    "cyfa_adamw_step": [_vp, _i, _vp, _vp, _vp, _vp] + [_f] * 5 + [_i, _vp],
    "cyfa_grad_clip": [_vp, ctypes.c_longlong, _f, _vp, _vp, ctypes.c_size_t, _vp],
    "cyfa_add_rmsnorm": [_vp, _vp, _vp, _f, _vp, _i, _i, _vp],
    "cyfa_decode_conv": [_vp, ctypes.c_longlong] + [_vp] * 9 + [_i] * 5 + [_vp],
    "cyfa_swiglu": [_vp, _vp, _i, _i, _vp],
}

# size queries (restype size_t)
_SIZE_QUERIES = {
    "cyfa_chunk_saved_bytes": [_i] * 5,
    "cyfa_chunk_work_bytes": [_i] * 5,
    "cyfa_short_conv_work_bytes": [_i] * 4,
    "cyfa_gate_act_work_bytes": [_i] * 2,
    "cyfa_gated_norm_work_bytes": [_i] * 2,
    "cyfa_gated_norm_bias_work_bytes": [_i] * 3,
    "cyfa_grad_clip_work_bytes": [],
}


class DecodeLayerArgs(ctypes.Structure):
    """cyfa_decode_layer_args."""

    _fields_ = [(n, _i) for n in ("B", "H", "K", "V", "W", "a_col")] + \
        [("P_stride", ctypes.c_longlong)] + \
        [(n, _vp) for n in ("P", "cache_q", "cache_k", "cache_v", "wconv_q", "wconv_k",
                            "wconv_v", "A_log", "dt_bias", "b_bias", "d_bias", "table",
                            "q_norm_weight", "k_norm_weight", "hk_in", "hv_in", "clock_in",
                            "hk_out", "hv_out", "clock_out", "gate", "gate_bias",
                            "o_norm_weight", "y")] + \
        [(n, _f) for n in ("q_eps", "k_eps", "scale", "o_eps", "o_scale")]


class BucketPiece(ctypes.Structure):
    """cyfa_bucket_piece: one gradient tensor inside a flat fp32 bucket."""

    _fields_ = [("ptr", ctypes.c_void_p), ("n", ctypes.c_longlong),
                ("offset", ctypes.c_longlong), ("dtype", ctypes.c_int)]


class CyfaError(RuntimeError):
    """A libcyfa entry point returned a non-zero status."""


_lib = None


def lib():
    """Loads libcyfa.so once; raises if it is missing (no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"CyFA CUDA library not built: {LIB_PATH} is missing. "
                "Build it with `make -C cyfa-jittor_b200/csrc` (nvcc, sm_100a)."
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = ctypes.c_int
        for name, args in _SIZE_QUERIES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = ctypes.c_size_t
        handle.cyfa_launch_count.argtypes = []
        handle.cyfa_launch_count.restype = ctypes.c_longlong
        handle.cyfa_profile_enable.argtypes = [ctypes.c_int]
        handle.cyfa_profile_enable.restype = ctypes.c_int
        handle.cyfa_set_pdl.argtypes = [ctypes.c_int]
        handle.cyfa_set_pdl.restype = ctypes.c_int
        handle.cyfa_set_scan_split.argtypes = [ctypes.c_int]
        handle.cyfa_set_scan_split.restype = ctypes.c_int
        handle.cyfa_set_aux_stream.argtypes = [ctypes.c_void_p]
        handle.cyfa_set_aux_stream.restype = ctypes.c_int
        handle.cyfa_profile_report.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                               ctypes.POINTER(ctypes.c_float),
                                               ctypes.POINTER(ctypes.c_int)]
        handle.cyfa_profile_report.restype = ctypes.c_int
        handle.cyfa_strerror.argtypes = [ctypes.c_int]
        handle.cyfa_strerror.restype = ctypes.c_char_p
        _lib = handle
    return _lib


def call(name, *args):
    """Calls an entry point and raises CyfaError on a non-zero status."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().cyfa_strerror(status).decode()
        raise CyfaError(f"{name} failed with status {status}: {msg}")


def ptr(t):
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream():
    """The current torch CUDA stream as a raw handle."""
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@contextlib.contextmanager
def deferred(aux):
    """Inside the block, the library's final parameter-gradient reductions run on
    the torch stream `aux`, after the work already issued on the current stream
    (cyfa_set_aux_stream).  The caller makes the current stream wait for `aux`
    before those gradients are read and keeps the calls' workspaces alive until
    then."""
    lib().cyfa_set_aux_stream(ctypes.c_void_p(aux.cuda_stream))
    try:
        yield
    finally:
        lib().cyfa_set_aux_stream(None)


def require_cuda(*tensors):
    """Raises unless every tensor lives on a CUDA device (no CPU fallback)."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "CyFA ops run only on CUDA tensors (sm_100a); there is no CPU path. "
                "The CPU restatement lives in oracle/ and is test infrastructure."
            )


def device_error(reset=True):
    """Returns the device error word (1 = a bounded wait timed out)."""
    return lib().cyfa_device_error(1 if reset else 0)


def launch_count():
    """Kernels libcyfa has launched in this process."""
    return lib().cyfa_launch_count()


def set_pdl(on=True):
    """Programmatic dependent launch of the library's kernels on/off; returns
    the previous setting."""
    return bool(lib().cyfa_set_pdl(1 if on else 0))


def set_scan_split(on=True):
    """Segmented state scans (more parallelism for few sequences x heads) on/off;
    returns the previous setting."""
    return bool(lib().cyfa_set_scan_split(1 if on else 0))


def profile_enable(on=True):
    """Per-kernel CUDA-event timing on/off (clears earlier records)."""
    lib().cyfa_profile_enable(1 if on else 0)


def profile_report(max_names=64):
    """{kernel name: (total ms, launches)} since profile_enable(True)."""
    names = (ctypes.c_char_p * max_names)()
    ms = (ctypes.c_float * max_names)()
    counts = (ctypes.c_int * max_names)()
    n = lib().cyfa_profile_report(max_names, names, ms, counts)
    if n < 0:
        raise CyfaError("cyfa_profile_report failed")
    return {names[i].decode(): (ms[i], counts[i]) for i in range(n)}
