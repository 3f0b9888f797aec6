"""Resumable training checkpoints, using safetensors and JSON only.

Counterpart of the reference's training/checkpoint.py:13-63, with the same
directory layout, so a run can stop and resume on the same number of ranks:

    <dir>/config.json, <dir>/model.safetensors     the model (save_model)
    <dir>/training_state/optimizer.safetensors     "{group}.{master|m|v}.{i}" fp32
    <dir>/training.json                            step, update_step, rng state,
                                                   arguments, parameter_names,
                                                   world_size

The directory is written as "<dir>.incomplete" and renamed in one step, so a
crash never leaves a half-written checkpoint under the final name.
"""

import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

from cyclic_flow_attention.utils import load_safetensors, save_model, save_safetensors


def _world_size():
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size()
    return 1


def _names(optimizer):
    return [list(group["names"]) for group in optimizer.param_groups]


def save_training(model, optimizer, tokenizer, directory, step, rng, arguments):
    """Writes the model, the optimizer's fp32 masters and moments, and the
    run's counters and host RNG state (reference training/checkpoint.py:13-38).
    `rng` is a numpy Generator; `arguments` a JSON-serialisable dict."""
    directory = Path(directory)
    temporary = directory.with_name(directory.name + ".incomplete")
    if directory.exists() or temporary.exists():
        raise FileExistsError(str(directory))
    temporary.mkdir(parents=True)
    save_model(model, temporary, tokenizer)
    tensors = {}
    for g, group in enumerate(optimizer.param_groups):
        for kind in ("master", "m", "v"):
            tensors.update({f"{g}.{kind}.{i}": value for i, value in enumerate(group[kind])})
    (temporary / "training_state").mkdir()
    save_safetensors(tensors, temporary / "training_state" / "optimizer.safetensors")
    state = dict(
        step=step,
        update_step=optimizer.update_step,
        rng=rng.bit_generator.state,
        arguments=arguments,
        parameter_names=_names(optimizer),
        world_size=_world_size(),
    )
    (temporary / "training.json").write_text(json.dumps(state, indent=2) + "\n")
    os.replace(temporary, directory)


def restore_training(optimizer, directory, rng):
    """Loads the optimizer state saved by ``save_training`` into `optimizer`
    and the RNG state into `rng`; returns the saved training state dict
    (reference training/checkpoint.py:41-63).  The world size, the parameter
    names and order and every tensor shape must match."""
    directory = Path(directory)
    state = json.loads((directory / "training.json").read_text())
    if state["world_size"] != _world_size():
        raise ValueError("Resume requires the same number of data-parallel ranks")
    if state["parameter_names"] != _names(optimizer):
        raise ValueError("Optimizer parameter names/order differ")
    tensors = load_safetensors(directory / "training_state" / "optimizer.safetensors")
    with torch.no_grad():
        for g, group in enumerate(optimizer.param_groups):
            for kind in ("master", "m", "v"):
                for i, value in enumerate(group[kind]):
                    array = tensors.pop(f"{g}.{kind}.{i}")
                    if tuple(array.shape) != tuple(value.shape):
                        raise ValueError("Optimizer parameter shape mismatch")
                    value.copy_(array.to(value.dtype))
    if tensors:
        raise ValueError("Unexpected optimizer tensors")
    optimizer.update_step = state["update_step"]
    optimizer.n_step = state["step"] * state["arguments"]["gradient_accumulation_steps"]
    rng.bit_generator.state = state["rng"]
    return state
