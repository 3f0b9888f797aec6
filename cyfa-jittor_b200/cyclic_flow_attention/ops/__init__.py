from .chunk import chunk_cyfa
from .fused_recurrent import fused_recurrent_cyfa

__all__ = ["chunk_cyfa", "fused_recurrent_cyfa"]
