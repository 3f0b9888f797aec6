from .configuration_cyfa import CyclicFlowAttentionConfig
from .modeling_cyfa import (
    CyclicFlowAttentionForCausalLM,
    CyclicFlowAttentionModel,
    CyFABlock,
    GatedMLP,
)

__all__ = ["CyclicFlowAttentionConfig", "CyclicFlowAttentionForCausalLM",
           "CyclicFlowAttentionModel", "CyFABlock", "GatedMLP"]
