"""Drop-in replacement for the reference's ``kernels/cutlass_experts.py`` on B200 (sm_100a).

Same public names, constructor, forward signature, parameters/buffers and weight format:

  MXFP_BLOCK_SIZE, MMA_TILE_K, pad_k_to_tile, pad_fp4_weights, pad_fp8_activations
  get_cutlass_extension()        object with the six functions of the reference's pybind
                                 module (kernels/matmul_mxfp4_cutlass.cu:1173-1186)
  ensure_custom_op_registered()  registers cutlass::fp4_group_mm, cutlass::fused_moe_routing
                                 (+ the fused gptoss::* ops)
  quantize_activations_to_fp8    bit-exact FP8 e4m3 + UE8M0 (cutlass_experts.py:197-251)
  swiglu                         (cutlass_experts.py:258-276)
  CutlassGptOssExperts           (cutlass_experts.py:283-452)
  load_cutlass_weights           (cutlass_experts.py:455-530)

Differences a caller can observe:
  * Every op runs on CUDA (sm_100a) only; CPU tensors raise instead of computing.
  * forward() is one fused op (gptoss::moe_experts_forward): routing, quantisation,
    both GEMMs and their epilogues run as five kernels with no host synchronisation,
    so the module traces under torch.compile(fullgraph=True) and can be graph-captured.
  * The routing permutation is deterministic (stable, like torch.argsort(stable=True)).
  * Weight scales are converted to the blocked layout on the GPU at load time.

This file can be loaded either as a member of the package or on its own with
importlib.util.spec_from_file_location (the way the reference's tests load it).
"""
from __future__ import annotations

import os
import sys

import torch
from torch import nn

if __package__:
    from . import ops as _ops
else:  # loaded by file path: bring in the sibling package
    import importlib.util as _ilu

    _pkg_dir = os.path.dirname(os.path.abspath(__file__))
    _name = "gpt_oss_mxfp4_compile_b200"
    if _name not in sys.modules:
        _spec = _ilu.spec_from_file_location(_name, os.path.join(_pkg_dir, "__init__.py"),
                                             submodule_search_locations=[_pkg_dir])
        _mod = _ilu.module_from_spec(_spec)
        sys.modules[_name] = _mod
        _spec.loader.exec_module(_mod)
    _ops = sys.modules[_name + ".ops"]

# ---------------------------------------------------------------------------
# Constants and K padding (cutlass_experts.py:24-89)
# ---------------------------------------------------------------------------

MXFP_BLOCK_SIZE = 32  # elements per scale factor group
MMA_TILE_K = 128      # K of one staged MMA block; K must be a multiple of this


def pad_k_to_tile(K):
    """Return K padded to the next multiple of MMA_TILE_K."""
    return ((K + MMA_TILE_K - 1) // MMA_TILE_K) * MMA_TILE_K


def pad_fp4_weights(data, scales, K_orig):
    """Pad packed FP4 weights [N, K/2] and UE8M0 scales [N, K/32] along K to the tile
    boundary with zero data and zero scales. Returns (data, scales, K_padded)."""
    K_padded = pad_k_to_tile(K_orig)
    if K_padded == K_orig:
        return data, scales, K_orig
    data_padded = torch.nn.functional.pad(data, (0, (K_padded - K_orig) // 2), value=0)
    scales_padded = torch.nn.functional.pad(scales, (0, (K_padded - K_orig) // MXFP_BLOCK_SIZE), value=0)
    return data_padded, scales_padded, K_padded


def pad_fp8_activations(fp8_data, scales, K_orig):
    """Pad FP8 activations [M, K] and scales [M, K/32] along K to the tile boundary.
    Returns (data, scales, K_padded). (The fused path never calls this: the TMA unit
    reads the columns past K as zeros.)"""
    K_padded = pad_k_to_tile(K_orig)
    if K_padded == K_orig:
        return fp8_data, scales, K_orig
    data_padded = torch.nn.functional.pad(fp8_data.view(torch.uint8), (0, K_padded - K_orig), value=0)
    data_padded = data_padded.view(torch.float8_e4m3fn)
    scales_padded = torch.nn.functional.pad(scales, (0, (K_padded - K_orig) // MXFP_BLOCK_SIZE), value=0)
    return data_padded, scales_padded, K_padded


# ---------------------------------------------------------------------------
# Extension object (the reference's pybind module surface)
# ---------------------------------------------------------------------------

class _Extension:
    """Same function names as the reference's pybind module; all run on the GPU."""

    @staticmethod
    def cutlass_fp4_group_mm(output, a, b, a_blockscale, b_blockscales, alphas, problem_sizes, expert_offsets,
                             sf_offsets):
        _ops.fp4_group_mm_impl(output, a, b, a_blockscale, b_blockscales, alphas, problem_sizes, expert_offsets,
                               sf_offsets)

    @staticmethod
    def convert_a_scales_for_w4a8(scales, M, N, K):
        return _ops.convert_scales_blocked(scales.contiguous(), int(M), int(K))

    @staticmethod
    def convert_b_scales_for_w4a8(scales, M, N, K):
        return _ops.convert_scales_blocked(scales.contiguous(), int(N), int(K))

    @staticmethod
    def batch_convert_a_scales_for_w4a8(scales, expert_counts, expert_offsets, N, K):
        return _ops.batch_convert_a_scales(scales.contiguous(), expert_counts, expert_offsets, int(K))

    @staticmethod
    def batch_convert_a_scales_for_w4a8_gpu(scales, expert_counts, expert_offsets, N, K):
        return _ops.batch_convert_a_scales(scales.contiguous(), expert_counts, expert_offsets, int(K))

    @staticmethod
    def fused_moe_routing(router_indices, routing_weights, num_experts):
        return _ops.fused_moe_routing_impl(router_indices.contiguous(), routing_weights.float().contiguous(),
                                           int(num_experts))


_EXT = _Extension()


def get_cutlass_extension():
    """Return the (already built) extension object; raises if libgptoss_moe.so is missing."""
    _ops._lib.load()
    return _EXT


def ensure_custom_op_registered():
    """Register the custom ops for torch.compile (idempotent)."""
    _ops.register_ops()


# ---------------------------------------------------------------------------
# Building blocks
# ---------------------------------------------------------------------------

def quantize_activations_to_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """BF16/FP32 [M, K] -> float8_e4m3fn [M, K] + UE8M0 uint8 [M, K // 32] (row-major),
    bit-identical to the reference's eager quantiser."""
    assert x.dim() == 2, f"Expected 2D tensor, got {x.dim()}D"
    assert x.shape[1] % MXFP_BLOCK_SIZE == 0, f"K={x.shape[1]} must be divisible by {MXFP_BLOCK_SIZE}"
    ensure_custom_op_registered()
    return torch.ops.gptoss.quantize_fp8(x.contiguous())


def swiglu(gate_up: torch.Tensor, alpha: float = 1.702, limit: float = 7.0) -> torch.Tensor:
    """gate (even columns) * sigmoid(alpha * gate) * (up (odd columns) + 1), with
    gate <= limit and |up| <= limit."""
    ensure_custom_op_registered()
    return torch.ops.gptoss.swiglu(gate_up.contiguous(), float(alpha), float(limit))


# ---------------------------------------------------------------------------
# Expert module
# ---------------------------------------------------------------------------

class CutlassGptOssExperts(nn.Module):
    """MXFP4-weight, FP8-activation (W4A8) GPT-OSS expert layer for sm_100a.

    Parameters and buffers match the reference exactly:
      gate_up_proj_bias [E, 2I] f32, down_proj_bias [E, H] f32 (Parameters, frozen)
      gate_up_proj_data [E, 2I, Kh/2] u8, gate_up_proj_scales [E, cosize] u8 (blocked)
      down_proj_data [E, H, Ki/2] u8, down_proj_scales [E, cosize] u8 (blocked)
    Buffers are None until load_cutlass_weights() runs.
    """

    def __init__(self, config):
        super().__init__()
        self.num_experts = config.num_local_experts
        self.intermediate_size = config.intermediate_size
        self.hidden_size = config.hidden_size
        self.alpha = 1.702
        limit = getattr(config, "swiglu_limit", 7.0)
        self.limit = 7.0 if limit is None else limit   # HF configs may carry swiglu_limit=None
        self.gemm_mode = _ops.GEMM_AUTO

        self.gate_up_proj_bias = nn.Parameter(
            torch.zeros(self.num_experts, 2 * self.intermediate_size, dtype=torch.float32), requires_grad=False)
        self.down_proj_bias = nn.Parameter(
            torch.zeros(self.num_experts, self.hidden_size, dtype=torch.float32), requires_grad=False)

        self.register_buffer("gate_up_proj_data", None)
        self.register_buffer("gate_up_proj_scales", None)
        self.register_buffer("down_proj_data", None)
        self.register_buffer("down_proj_scales", None)

    def _run_cutlass_gemm(self, activations, act_scales_rowmajor, weights, weight_scales, expert_token_counts,
                          expert_offsets, N, K, K_padded):
        """One grouped GEMM with the reference's signature (kept for subclasses such as the
        reference's benchmark variants); forward() does not use it."""
        ensure_custom_op_registered()
        total_tokens = activations.shape[0]
        num_experts = expert_token_counts.shape[0]
        device = activations.device
        output = torch.zeros((total_tokens, N), device=device, dtype=torch.bfloat16)
        if K_padded > K:
            activations, act_scales_rowmajor, _ = pad_fp8_activations(activations, act_scales_rowmajor, K)
        act_scales_blocked, sf_offsets = _ops.batch_convert_a_scales(
            act_scales_rowmajor.contiguous(), expert_token_counts, expert_offsets, K_padded, exact_size=False)
        problem_sizes = torch.zeros((num_experts, 3), device=device, dtype=torch.int32)
        problem_sizes[:, 0] = expert_token_counts
        problem_sizes[:, 1] = N
        problem_sizes[:, 2] = K_padded
        alphas = torch.ones((num_experts,), device=device, dtype=torch.float32)
        torch.ops.cutlass.fp4_group_mm(output, activations.contiguous(), weights, act_scales_blocked, weight_scales,
                                       alphas, problem_sizes, expert_offsets, sf_offsets)
        return output

    def forward(self, hidden_states: torch.Tensor, router_indices: torch.Tensor,
                routing_weights: torch.Tensor) -> torch.Tensor:
        """hidden_states [..., H] bf16, router_indices [T, k] int64, routing_weights [T, k]
        -> same shape and dtype as hidden_states."""
        if self.gate_up_proj_data is None:
            raise RuntimeError("CutlassGptOssExperts: weights not loaded (call load_cutlass_weights)")
        ensure_custom_op_registered()
        input_shape = hidden_states.shape
        hidden = hidden_states.reshape(-1, self.hidden_size).contiguous()
        # eager calls on plain tensors skip the custom-op dispatcher (~30 us of host time)
        fn = _ops.moe_experts_forward_impl if _ops.eager_call(hidden) else torch.ops.gptoss.moe_experts_forward
        out = fn(hidden, router_indices.contiguous(), routing_weights.float().contiguous(),
                 self.gate_up_proj_data, self.gate_up_proj_scales, self.gate_up_proj_bias,
                 self.down_proj_data, self.down_proj_scales, self.down_proj_bias,
                 float(self.alpha), float(self.limit), int(self.gemm_mode))
        return out.view(input_shape)


def load_cutlass_weights(module: CutlassGptOssExperts, gate_up_blocks: torch.Tensor, gate_up_scales: torch.Tensor,
                         down_blocks: torch.Tensor, down_scales: torch.Tensor, device):
    """Load checkpoint MXFP4 weights into the module.

    gate_up_blocks [E, 2I, H/32, 16] (or [E, 2I, H/2]) u8, gate_up_scales [E, 2I, H/32] u8,
    down_blocks [E, H, I/32, 16] (or [E, H, I/2]) u8, down_scales [E, H, I/32] u8.
    K is zero-padded to a multiple of 128 and the scales are converted to the blocked
    layout on the GPU (one kernel per expert, no host round trip).
    """
    E = module.num_experts
    hidden = module.hidden_size
    inter = module.intermediate_size
    K_hidden_padded = pad_k_to_tile(hidden)
    K_inter_padded = pad_k_to_tile(inter)
    module.K_hidden_padded = K_hidden_padded
    module.K_inter_padded = K_inter_padded

    gu_data = gate_up_blocks.reshape(E, 2 * inter, hidden // 2).to(device).contiguous()
    dn_data = down_blocks.reshape(E, hidden, inter // 2).to(device).contiguous()
    gu_sc = gate_up_scales.reshape(E, 2 * inter, hidden // 32).to(device).contiguous()
    dn_sc = down_scales.reshape(E, hidden, inter // 32).to(device).contiguous()

    if K_hidden_padded > hidden:
        gu_data = torch.nn.functional.pad(gu_data, (0, (K_hidden_padded - hidden) // 2), value=0)
        gu_sc = torch.nn.functional.pad(gu_sc, (0, (K_hidden_padded - hidden) // MXFP_BLOCK_SIZE), value=0)
    if K_inter_padded > inter:
        dn_data = torch.nn.functional.pad(dn_data, (0, (K_inter_padded - inter) // 2), value=0)
        dn_sc = torch.nn.functional.pad(dn_sc, (0, (K_inter_padded - inter) // MXFP_BLOCK_SIZE), value=0)

    gu_conv = torch.stack([_ops.convert_scales_blocked(gu_sc[e].contiguous(), 2 * inter, K_hidden_padded)
                           for e in range(E)], dim=0)
    dn_conv = torch.stack([_ops.convert_scales_blocked(dn_sc[e].contiguous(), hidden, K_inter_padded)
                           for e in range(E)], dim=0)

    module.gate_up_proj_data = gu_data.contiguous()
    module.gate_up_proj_scales = gu_conv
    module.down_proj_data = dn_data.contiguous()
    module.down_proj_scales = dn_conv
