"""Checkpoint format of the CyFA language models: ``config.json`` plus
``model.safetensors`` with the reference's parameter names and dtype policy
(reference cyclic_flow_attention/utils.py:26-176).  The safetensors container
(8-byte little-endian header length, JSON header of name -> dtype, shape and
byte range, raw little-endian data) is read and written here directly, without
the ``safetensors`` package."""

import json
import os
import struct
from pathlib import Path

import torch

from .models.cyfa import CyclicFlowAttentionConfig, CyclicFlowAttentionForCausalLM

_CODES = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16",
          torch.int64: "I64", torch.int32: "I32", torch.uint8: "U8", torch.bool: "BOOL"}
_TYPES = {v: k for k, v in _CODES.items()}


def save_safetensors(tensors, path):
    """Writes {name: tensor} keeping each tensor's dtype (header padded to 8 bytes)."""
    path = Path(path)
    header, offset, blobs = {}, 0, []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        data = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _CODES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [offset, offset + len(data)]}
        offset += len(data)
        blobs.append(data)
    encoded = json.dumps(header, separators=(",", ":")).encode()
    encoded += b" " * (-len(encoded) % 8)
    tmp = path.with_name(path.name + ".tmp")
    with tmp.open("wb") as f:
        f.write(struct.pack("<Q", len(encoded)))
        f.write(encoded)
        for data in blobs:
            f.write(data)
    os.replace(tmp, path)


def load_safetensors(path):
    """{name: CPU tensor} in the file's dtypes."""
    with open(path, "rb") as f:
        size = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(size))
        raw = f.read()
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        begin, end = meta["data_offsets"]
        dtype = _TYPES[meta["dtype"]]
        buf = bytearray(raw[begin:end])
        t = torch.frombuffer(buf, dtype=torch.uint8) if buf else torch.empty(0, dtype=torch.uint8)
        out[name] = t.view(dtype).reshape(meta["shape"]).clone()
    return out


def read_config(directory):
    return CyclicFlowAttentionConfig.from_pretrained(directory)


def initialize_model(config, std=0.02, generator=None, device=None):
    """Random init as the reference's initialize_model (utils.py:122-129):
    every non-norm ``.weight`` ~ N(0, std), biases zero, then the bf16 cast
    that keeps norms, readout, A_log and dt_bias in fp32."""
    with torch.device(device if device is not None else "cpu"):
        model = CyclicFlowAttentionForCausalLM(config)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith(".weight") and "norm" not in name:
                p.copy_(torch.randn(p.shape, generator=generator, device=p.device) * std
                        if generator is not None and generator.device == p.device
                        else (torch.randn(p.shape, generator=generator) * std).to(p.device))
            elif name.endswith(".bias"):
                p.zero_()
    return model.to_bfloat16()


def save_model(model, directory, tokenizer=None):
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    config = model.config.to_dict()
    if tokenizer is not None:
        config.update(eos_token_id=tokenizer.eos_id, bos_token_id=tokenizer.bos_id)
    (directory / "config.json").write_text(json.dumps(config, indent=2) + "\n")
    save_safetensors(model.state_dict(), directory / "model.safetensors")


def load_model(path, device=None):
    """(model, directory): the reference's load_model (utils.py:115-119):
    bf16 model with the fp32 exceptions, weights from every *.safetensors file,
    cast to each parameter's dtype; missing or unexpected names raise."""
    directory = Path(path)
    model = CyclicFlowAttentionForCausalLM(read_config(directory)).to_bfloat16()
    weights = {}
    files = sorted(directory.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError("No safetensors weights under " + str(directory))
    for f in files:
        weights.update(load_safetensors(f))
    state = model.state_dict()
    missing = [n for n in state if n not in weights]
    unexpected = [n for n in weights if n not in state]
    if missing or unexpected:
        raise KeyError(f"checkpoint mismatch: missing {missing[:5]}, unexpected {unexpected[:5]}")
    with torch.no_grad():
        for name, t in state.items():
            t.copy_(weights[name].to(t.dtype))
    if device is not None:
        model = model.to(device)
    return model, directory
