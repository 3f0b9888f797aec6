"""Configuration of the CyFA language models.

Same fields and defaults as the reference's CyclicFlowAttentionConfig
(models/cyfa/configuration_cyfa.py:9-27), so its config.json files load.
"""

import json
from dataclasses import asdict, dataclass, fields
from pathlib import Path


@dataclass
class CyclicFlowAttentionConfig:
    hidden_size: int = 1024
    num_heads: int = 4
    head_dim: int = 256
    expand_k: float = 1.0
    expand_v: float = 1.0
    num_slots: int = 128
    num_hidden_layers: int = 24
    vocab_size: int = 32000
    hidden_ratio: float = 4.0
    intermediate_size: int | None = None
    use_short_conv: bool = True
    conv_size: int = 4
    conv_bias: bool = False
    norm_eps: float = 1e-6
    tie_word_embeddings: bool = False
    chunk_size: int = 64

    @classmethod
    def from_dict(cls, data):
        """Known fields only, with the reference's checks (utils.py:97-112):
        positive sizes and the SwiGLU MLP."""
        names = {f.name for f in fields(cls)}
        config = cls(**{k: v for k, v in data.items() if k in names})
        if config.hidden_size <= 0 or config.num_hidden_layers <= 0 or config.vocab_size <= 1:
            raise ValueError("Invalid model dimensions")
        if data.get("hidden_act", "swish") not in ("swish", "silu"):
            raise ValueError("Only the released SwiGLU model architecture is supported")
        return config

    @classmethod
    def from_pretrained(cls, path):
        """Reads ``config.json`` from a checkpoint directory (or the file itself)."""
        path = Path(path)
        if path.is_dir():
            path = path / "config.json"
        return cls.from_dict(json.loads(path.read_text()))

    def to_dict(self):
        data = asdict(self)
        data.update(model_type="cyclic_flow_attention",
                    architectures=["CyclicFlowAttentionForCausalLM"])
        return data
