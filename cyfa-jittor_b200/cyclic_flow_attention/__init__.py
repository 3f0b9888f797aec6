"""Cyclic Flow Attention (CyFA) hot path for NVIDIA B200 (sm_100a).

Mirrors the reference package's public API (cyclic_flow_attention/__init__.py,
ops/__init__.py, layers/__init__.py): ``chunk_cyfa``, ``fused_recurrent_cyfa``
and the ``CyclicFlowAttention`` layer.  All attention math runs in libcyfa.so.
"""

from .layers import CyclicFlowAttention
from .ops import chunk_cyfa, fused_recurrent_cyfa

__version__ = "0.1.0"

__all__ = ["CyclicFlowAttention", "chunk_cyfa", "fused_recurrent_cyfa"]
