"""Router + experts as one module: the GptOssMLP shape of the MoE block.

HF's GptOssMLP.forward (transformers models/gpt_oss/modeling_gpt_oss.py) runs
GptOssTopKRouter (F.linear -> topk -> softmax over the k logits) and then the experts
module with (hidden, router_indices, router_scores). The reference swaps only the experts
for CutlassGptOssExperts; here the router is fused in front of them
(gptoss::moe_layer_forward: router kernel, counting sort, quantiser, two GEMMs).
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops as _ops
from .cutlass_experts import CutlassGptOssExperts, ensure_custom_op_registered


class GptOssMoELayer(nn.Module):
    """router.weight [E, H] bf16, router.bias [E] bf16, experts: CutlassGptOssExperts."""

    def __init__(self, config):
        super().__init__()
        self.top_k = getattr(config, "num_experts_per_tok", 4)
        self.num_experts = config.num_local_experts
        self.hidden_size = config.hidden_size
        self.router_weight = nn.Parameter(torch.zeros(self.num_experts, self.hidden_size, dtype=torch.bfloat16),
                                          requires_grad=False)
        self.router_bias = nn.Parameter(torch.zeros(self.num_experts, dtype=torch.bfloat16), requires_grad=False)
        self.experts = CutlassGptOssExperts(config)

    def forward(self, hidden_states: torch.Tensor):
        """hidden_states [..., H] bf16 -> (out [..., H] bf16, router_scores [T, k] bf16,
        router_indices [T, k] int64)."""
        ensure_custom_op_registered()
        ex = self.experts
        shape = hidden_states.shape
        h = hidden_states.reshape(-1, self.hidden_size).contiguous()
        # plain tensors in eager mode call the implementation directly (the dispatcher of a
        # Python custom op costs ~30 us of host time per call); tracing goes through the op
        fn = _ops.moe_layer_forward_impl if _ops.eager_call(h) else torch.ops.gptoss.moe_layer_forward
        out, scores, idx = fn(h, self.router_weight, self.router_bias, int(self.top_k),
                              ex.gate_up_proj_data, ex.gate_up_proj_scales, ex.gate_up_proj_bias,
                              ex.down_proj_data, ex.down_proj_scales, ex.down_proj_bias,
                              float(ex.alpha), float(ex.limit), int(ex.gemm_mode))
        return out.view(shape), scores, idx

    def forward_block(self, hidden_states: torch.Tensor, norm_weight: torch.Tensor, norm_eps: float = 1e-5):
        """The decoder block's MoE half: hidden + self(RMSNorm(hidden)) (the model's
        residual + mlp(post_attention_layernorm(hidden))), as the MoE kernels alone: the norm
        and the residual copy are one kernel and GEMM2 adds into the residual rows
        (gptoss::moe_block_forward). -> (out [..., H] bf16, router_scores, router_indices)."""
        ensure_custom_op_registered()
        ex = self.experts
        shape = hidden_states.shape
        h = hidden_states.reshape(-1, self.hidden_size).contiguous()
        fn = _ops.moe_block_forward_impl if _ops.eager_call(h) else torch.ops.gptoss.moe_block_forward
        out, scores, idx = fn(h, norm_weight, float(norm_eps), self.router_weight, self.router_bias, int(self.top_k),
                              ex.gate_up_proj_data, ex.gate_up_proj_scales, ex.gate_up_proj_bias,
                              ex.down_proj_data, ex.down_proj_scales, ex.down_proj_bias,
                              float(ex.alpha), float(ex.limit), int(ex.gemm_mode))
        return out.view(shape), scores, idx

    def route(self, hidden_states: torch.Tensor):
        """Router only: (logits [T, E] bf16, scores [T, k] bf16, indices [T, k] int64)."""
        ensure_custom_op_registered()
        h = hidden_states.reshape(-1, self.hidden_size).contiguous()
        return torch.ops.gptoss.router_topk(h, self.router_weight.data, self.router_bias.data, int(self.top_k))


__all__ = ["GptOssMoELayer"]
