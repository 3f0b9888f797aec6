"""Host-side checks of the CyFA language model mirror (no GPU): parameter
names and dtypes as the reference's checkpoints hold them
(models/cyfa/modeling_cyfa.py:13-116, utils.py:115-176), config parsing, the
safetensors writer/reader, and a causality check of the oracle LM."""

import pytest
import torch

from cyclic_flow_attention.models.cyfa import CyclicFlowAttentionConfig, CyclicFlowAttentionForCausalLM
from cyclic_flow_attention.utils import (initialize_model, load_model, load_safetensors,
                                         save_model, save_safetensors)
from oracle import cyfa_oracle as O

ATTN = ["q_proj.weight", "k_proj.weight", "v_proj.weight", "a_proj.weight", "b_proj.weight",
        "b_proj.bias", "d_proj.weight", "d_proj.bias", "dt_bias", "A_log", "readout",
        "q_norm.weight", "k_norm.weight", "q_conv1d.weight", "k_conv1d.weight",
        "v_conv1d.weight", "g_proj.0.weight", "g_proj.1.weight", "g_proj.1.bias",
        "o_norm.weight", "o_proj.weight"]


def _tiny(layers=1, **kw):
    # the reference's configs/tiny.json, with optional overrides
    base = dict(hidden_size=256, head_dim=256, num_heads=1, num_hidden_layers=layers,
                vocab_size=256, intermediate_size=512, num_slots=128, use_short_conv=True,
                conv_size=4)
    base.update(kw)
    return CyclicFlowAttentionConfig.from_dict(base)


def test_state_dict_names_and_shapes_match_reference():
    cfg = _tiny(layers=2)
    m = CyclicFlowAttentionForCausalLM(cfg)
    expected = {"model.embeddings.weight", "model.norm.weight", "lm_head.weight"}
    for i in range(2):
        pre = f"model.layers.{i}."
        expected |= {pre + "attn_norm.weight", pre + "mlp_norm.weight"}
        expected |= {pre + "attn." + n for n in ATTN}
        expected |= {pre + f"mlp.{n}_proj.weight" for n in ("gate", "up", "down")}
    sd = m.state_dict()
    assert set(sd) == expected
    assert sd["model.layers.0.attn.readout"].shape == (1, 127, 127)
    assert sd["model.layers.0.attn.q_conv1d.weight"].shape == (256, 1, 4)
    assert sd["model.layers.0.attn.g_proj.0.weight"].shape == (256, 256)
    assert sd["model.layers.0.mlp.gate_proj.weight"].shape == (512, 256)


def test_mlp_width_rule():
    # 256 * ceil(int(hidden * ratio * 2 / 3) / 256) when intermediate_size is unset
    cfg = CyclicFlowAttentionConfig(hidden_size=2048, num_heads=8, num_hidden_layers=1)
    assert CyclicFlowAttentionForCausalLM(cfg).model.layers[0].mlp.intermediate_size == 5632


def test_bf16_policy():
    m = CyclicFlowAttentionForCausalLM(_tiny()).to_bfloat16()
    for name, p in m.named_parameters():
        keep = any(s in name for s in ("norm.weight", "readout", "A_log", "dt_bias"))
        assert p.dtype == (torch.float32 if keep else torch.bfloat16), name


def test_config_validation():
    with pytest.raises(ValueError):
        CyclicFlowAttentionConfig.from_dict({"hidden_act": "gelu"})
    with pytest.raises(ValueError):
        CyclicFlowAttentionConfig.from_dict({"hidden_size": 0})
    cfg = CyclicFlowAttentionConfig.from_dict({"hidden_size": 512, "unknown_key": 1})
    assert cfg.hidden_size == 512


def test_safetensors_roundtrip(tmp_path):
    tensors = {"a": torch.randn(3, 5).bfloat16(), "b": torch.randn(7), "c": torch.arange(4),
               "e": torch.zeros(0)}
    save_safetensors(tensors, tmp_path / "x.safetensors")
    back = load_safetensors(tmp_path / "x.safetensors")
    assert set(back) == set(tensors)
    for n, t in tensors.items():
        assert back[n].dtype == t.dtype and torch.equal(back[n], t), n
    raw = (tmp_path / "x.safetensors").read_bytes()
    assert int.from_bytes(raw[:8], "little") % 8 == 0


def test_model_save_load(tmp_path):
    m = initialize_model(_tiny(), generator=torch.Generator().manual_seed(0))
    save_model(m, tmp_path)
    loaded, directory = load_model(tmp_path)
    assert directory == tmp_path and loaded.config == m.config
    a, b = m.state_dict(), loaded.state_dict()
    for n in a:
        assert a[n].dtype == b[n].dtype and torch.equal(a[n], b[n]), n


def test_oracle_lm_is_causal():
    torch.manual_seed(0)
    m = initialize_model(_tiny(layers=2, head_dim=128, num_heads=2),
                         generator=torch.Generator().manual_seed(1))
    params = {n: t.float() for n, t in m.state_dict().items()}
    ids = torch.randint(0, 256, (1, 80), generator=torch.Generator().manual_seed(2))
    full = O.cyfa_lm(params, ids, 2, 2, 128, 128)
    ids2 = ids.clone()
    ids2[:, 70:] = (ids2[:, 70:] + 1) % 256
    part = O.cyfa_lm(params, ids2, 2, 2, 128, 128)
    assert torch.allclose(full[:, :70], part[:, :70], atol=1e-5)
    assert not torch.allclose(full[:, 70:], part[:, 70:], atol=1e-3)
