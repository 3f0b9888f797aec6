from .cyfa import CyclicFlowAttentionConfig, CyclicFlowAttentionForCausalLM

__all__ = ["CyclicFlowAttentionConfig", "CyclicFlowAttentionForCausalLM"]
