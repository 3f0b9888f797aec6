from .cyfa import CyclicFlowAttention, RMSNorm, ShortConvolution

__all__ = ["CyclicFlowAttention", "RMSNorm", "ShortConvolution"]
