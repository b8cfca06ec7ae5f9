"""Hugging Face GPT-OSS models with this library's expert layer.

`replace_experts_with_cutlass` restates the reference's model-level integration
(test_cutlass_model.py:48-117, `replace_experts_with_cutlass`): every `GptOssExperts` /
`Mxfp4GptOssExperts` module of the model becomes a `CutlassGptOssExperts`, its MXFP4 blocks,
UE8M0 scales and biases read from the checkpoint through `get_tensor(name)` under the
module's own name (`model.layers.<i>.mlp.experts.gate_up_proj_blocks`, ...), exactly as the
reference reads them.

`replace_mlp_with_fused_layer` goes one step further (no counterpart in the reference): the
whole `GptOssMLP` (router + experts) becomes one `gptoss_moe_layer_forward` call, the router
fused in front of the experts; the module keeps HF's `(hidden_states, router_scores)` return.

`checkpoint_getter(path)` opens a safetensors checkpoint directory (with its
`model.safetensors.index.json`) lazily, as the reference's loader does.
"""
from __future__ import annotations

import json
import os

import torch
from torch import nn

from .cutlass_experts import CutlassGptOssExperts, load_cutlass_weights
from .layer import GptOssMoELayer

_EXPERT_CLASSES = ("GptOssExperts", "Mxfp4GptOssExperts")


def checkpoint_getter(checkpoint_path: str):
    """name -> tensor over the safetensors files of a checkpoint directory (files opened on
    first use)."""
    from safetensors import safe_open

    with open(os.path.join(checkpoint_path, "model.safetensors.index.json")) as f:
        weight_map = json.load(f)["weight_map"]
    files = {}

    def get_tensor(name: str) -> torch.Tensor:
        fname = weight_map[name]
        if fname not in files:
            files[fname] = safe_open(os.path.join(checkpoint_path, fname), framework="pt")
        return files[fname].get_tensor(name)

    return get_tensor


def _experts_module(config, prefix: str, get_tensor, device) -> CutlassGptOssExperts:
    mod = CutlassGptOssExperts(config).to(device)
    mod.gate_up_proj_bias.data.copy_(get_tensor(f"{prefix}.gate_up_proj_bias").to(device))
    mod.down_proj_bias.data.copy_(get_tensor(f"{prefix}.down_proj_bias").to(device))
    load_cutlass_weights(mod, get_tensor(f"{prefix}.gate_up_proj_blocks"), get_tensor(f"{prefix}.gate_up_proj_scales"),
                         get_tensor(f"{prefix}.down_proj_blocks"), get_tensor(f"{prefix}.down_proj_scales"), device)
    return mod


def replace_experts_with_cutlass(model: nn.Module, get_tensor, config=None, device="cuda") -> int:
    """Replace every GPT-OSS expert module of `model` by a CutlassGptOssExperts loaded from
    `get_tensor`; returns the number of modules replaced."""
    config = config if config is not None else model.config
    n = 0
    for name, module in list(model.named_modules()):
        if module.__class__.__name__ not in _EXPERT_CLASSES:
            continue
        model.set_submodule(name, _experts_module(config, name, get_tensor, device))
        n += 1
    return n


class FusedGptOssMLP(nn.Module):
    """HF `GptOssMLP` drop-in: router + experts in one library call. forward(hidden_states
    [B, S, H]) -> (hidden_states [B, S, H], router_scores [B*S, k]) like HF's module."""

    def __init__(self, layer: GptOssMoELayer):
        super().__init__()
        self.layer = layer

    def forward(self, hidden_states: torch.Tensor):
        out, scores, _ = self.layer(hidden_states)
        return out, scores


def replace_mlp_with_fused_layer(model: nn.Module, get_tensor, config=None, device="cuda") -> int:
    """Replace every `GptOssMLP` (its router's weight and bias taken from the model, the
    experts from `get_tensor`) by a FusedGptOssMLP; returns the number replaced."""
    config = config if config is not None else model.config
    n = 0
    for name, module in list(model.named_modules()):
        if module.__class__.__name__ != "GptOssMLP":
            continue
        layer = GptOssMoELayer(config).to(device)
        layer.router_weight.data.copy_(module.router.weight.data.to(device, torch.bfloat16))
        layer.router_bias.data.copy_(module.router.bias.data.to(device, torch.bfloat16))
        layer.experts = _experts_module(config, f"{name}.experts", get_tensor, device)
        model.set_submodule(name, FusedGptOssMLP(layer))
        n += 1
    return n


__all__ = ["checkpoint_getter", "replace_experts_with_cutlass", "replace_mlp_with_fused_layer", "FusedGptOssMLP"]
