"""Shared helpers for the tests (not part of the product)."""
from __future__ import annotations

import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class Cfg:
    def __init__(self, E, H, I, k=4, limit=7.0):
        self.num_local_experts = E
        self.hidden_size = H
        self.intermediate_size = I
        self.num_experts_per_tok = k
        self.swiglu_limit = limit


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def build_experts(pkg, d: dict, device, E: int, H: int, I: int):
    m = pkg.CutlassGptOssExperts(Cfg(E, H, I)).to(device)
    m.gate_up_proj_bias.data.copy_(d["gu_bias"])
    m.down_proj_bias.data.copy_(d["dn_bias"])
    pkg.load_cutlass_weights(m, d["gu_blocks"], d["gu_scales"], d["dn_blocks"], d["dn_scales"], device)
    return m


def build_layer(pkg, d: dict, device, E: int, H: int, I: int, k: int):
    layer = pkg.GptOssMoELayer(Cfg(E, H, I, k)).to(device)
    layer.router_weight.data.copy_(d["router_w"])
    layer.router_bias.data.copy_(d["router_b"])
    layer.experts.gate_up_proj_bias.data.copy_(d["gu_bias"])
    layer.experts.down_proj_bias.data.copy_(d["dn_bias"])
    pkg.load_cutlass_weights(layer.experts, d["gu_blocks"], d["gu_scales"], d["dn_blocks"], d["dn_scales"], device)
    return layer


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.float().cpu()
    b = b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def max_abs_over_rms(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.float().cpu()
    b = b.float().cpu()
    return ((a - b).abs().max() / b.pow(2).mean().sqrt().clamp_min(1e-30)).item()


def assert_output_tolerance(out: torch.Tensor, ref: torch.Tensor, what: str = ""):
    """North-star output gate: rel-L2 <= 1e-2 and max-abs <= 5e-2 * rms(ref)."""
    r = rel_l2(out, ref)
    m = max_abs_over_rms(out, ref)
    assert r <= 1e-2 and m <= 5e-2, f"{what}: rel-L2 {r:.3e} (<=1e-2), max-abs/rms {m:.3e} (<=5e-2)"
    return r, m


def bf16_from_int16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
