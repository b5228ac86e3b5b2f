"""Checkpoint loading (``ultils/loader.py:12-33``) for AWQ checkpoints.

Names are routed exactly as the reference does: a tensor name without the ``model.``
prefix gets it; a name containing a ``packed_modules_mapping`` key (``q_proj`` ->
``qkv_proj`` shard ``"q"``, ``gate_proj`` -> ``gate_up_proj`` shard 0, ...) goes to the
packed parameter's ``weight_loader(param, tensor, shard_id)``; every other tensor to
``weight_loader(param, tensor)``.  AWQ tensors (``qweight``, ``qzeros``, ``scales``) take
the same route as the reference's dense ``weight``.  After loading, every AWQ layer is
repacked into the kernel layout.
"""
from __future__ import annotations

import os
from glob import glob
from typing import Iterable

import torch
from torch import nn


def default_weight_loader(param: nn.Parameter, loaded_weight: torch.Tensor):
    param.data.copy_(loaded_weight)


def _load_one(model: nn.Module, weight_name: str, tensor: torch.Tensor, mapping: dict):
    param_name = weight_name if weight_name.startswith("model.") else f"model.{weight_name}"
    for k, (v, shard_id) in mapping.items():
        if k in weight_name:
            param = model.get_parameter(param_name.replace(k, v))
            param.weight_loader(param, tensor, shard_id)
            return
    try:
        param = model.get_parameter(param_name)
    except AttributeError:
        if param_name.endswith("rotary_emb.inv_freq"):
            return
        raise
    getattr(param, "weight_loader", default_weight_loader)(param, tensor)


def load_weights(model: nn.Module, weights: Iterable[tuple[str, torch.Tensor]] | dict):
    """Load ``(name, tensor)`` pairs (checkpoint names) into ``model``."""
    mapping = getattr(model, "packed_modules_mapping", {})
    items = weights.items() if isinstance(weights, dict) else weights
    for name, tensor in items:
        _load_one(model, name, tensor, mapping)
    # Repack for the kernels now when the model lives on a GPU (otherwise it happens on
    # the layer's first forward, after the model is moved to its device).
    on_gpu = any(p.is_cuda for p in model.parameters())
    if on_gpu and hasattr(model, "process_weights_after_loading"):
        model.process_weights_after_loading()


def load_model(model: nn.Module, path: str):
    """Load every ``*.safetensors`` file of a checkpoint directory (``loader.py:12-33``)."""
    from safetensors import safe_open

    def gen():
        for file in sorted(glob(os.path.join(path, "*.safetensors"))):
            with safe_open(file, "pt", "cpu") as f:
                for name in f.keys():
                    yield name, f.get_tensor(name)
    load_weights(model, gen())
