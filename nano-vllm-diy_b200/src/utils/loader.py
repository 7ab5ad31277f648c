"""Checkpoint loading through the modules' weight loaders.

load_model(model, path) reads every *.safetensors file under `path` (the
reference's src/utils/loader.py:12-28 behaviour, including leaving weights
untouched when there is none); load_weights(model, items) applies the same
dispatch to an iterable of (checkpoint name, tensor): names containing a key
of model.packed_modules_mapping go to the packed parameter with their shard
id, everything else to the parameter of the same name.
"""
from __future__ import annotations

import os
from glob import glob
from typing import Iterable

import torch
from torch import nn


def default_weight_loader(param: nn.Parameter, loaded_weight: torch.Tensor):
    param.data.copy_(loaded_weight)


def load_weights(model: nn.Module, items: Iterable[tuple[str, torch.Tensor]]) -> None:
    packed = getattr(model, "packed_modules_mapping", {})
    for name, tensor in items:
        for key, (target, shard_id) in packed.items():
            if key in name:
                param = model.get_parameter(name.replace(key, target))
                param.weight_loader(param, tensor, shard_id)
                break
        else:
            param = model.get_parameter(name)
            getattr(param, "weight_loader", default_weight_loader)(param, tensor)


def load_model(model: nn.Module, path: str) -> None:
    from safetensors import safe_open

    def items():
        for file in sorted(glob(os.path.join(path, "*.safetensors"))):
            with safe_open(file, "pt", "cpu") as f:
                for name in f.keys():
                    yield name, f.get_tensor(name)

    load_weights(model, items())
