"""The allocation-free expert forward (gptoss_moe_experts_forward_noalloc).

Callers that cannot give the library a workspace — runtimes that pre-reserve all device
memory behind their own pool, FFI hosts without a device allocator, loops that cannot
afford cudaMalloc's device synchronisation — use this entry point; its workspace is a
static device array inside the library. This file is collected last so a failure here
never hides the other tests' results; it also passes when run alone.
"""
import ctypes

import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, build_experts

pytestmark = pytest.mark.gpu


def _noalloc(pkg, m, hidden, idx, w):
    lib = pkg._lib.load()
    out = torch.empty_like(hidden)
    E, H, I = m.num_experts, m.hidden_size, m.intermediate_size
    T, k = idx.shape
    rc = lib.gptoss_moe_experts_forward_noalloc(
        hidden.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k, E, H, I,
        m.gate_up_proj_data.data_ptr(), m.gate_up_proj_scales.data_ptr(), m.gate_up_proj_scales.numel() // E,
        m.gate_up_proj_bias.data.data_ptr(), m.down_proj_data.data_ptr(), m.down_proj_scales.data_ptr(),
        m.down_proj_scales.numel() // E, m.down_proj_bias.data.data_ptr(), ctypes.c_float(m.alpha),
        ctypes.c_float(m.limit), out.data_ptr(), 0, pkg.ops.status_tensor(hidden.device).data_ptr(),
        torch.cuda.current_stream(hidden.device).cuda_stream)
    assert rc == 0, lib.gptoss_last_error().decode()
    return out


def test_noalloc_matches_workspace_forward_on_consecutive_calls(pkg, dev):
    E, H, I = 32, 2880, 2880
    d = O.synth_layer(31, E=E, H=H, I=I, T=1)
    m = build_experts(pkg, d, dev, E, H, I)
    g = torch.Generator().manual_seed(7)
    for T in (48, 32):   # two calls in a row reuse the same static scratch
        hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        wv, ix = torch.topk(torch.randn(T, E, generator=g), 4, dim=-1)
        wv = torch.softmax(wv, -1).to(dev)
        ix = ix.to(dev)
        got = _noalloc(pkg, m, hidden, ix, wv)
        ref = m(hidden, ix, wv)            # gptoss_moe_experts_forward with a torch workspace
        torch.cuda.synchronize()
        assert pkg.ops.read_status(dev) == 0
        assert_output_tolerance(got.cpu(), ref.cpu(), f"noalloc T={T}")


def test_noalloc_rejects_batches_beyond_the_scratch(pkg, dev):
    E, H, I = 4, 2880, 2880
    d = O.synth_layer(32, E=E, H=H, I=I, T=1)
    m = build_experts(pkg, d, dev, E, H, I)
    lib = pkg._lib.load()
    T, k = 4096, 4
    small = torch.zeros(8, H, dtype=torch.bfloat16, device=dev)
    idx = torch.zeros(8, k, dtype=torch.int64, device=dev)
    w = torch.zeros(8, k, device=dev)
    rc = lib.gptoss_moe_experts_forward_noalloc(
        small.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k, E, H, I,
        m.gate_up_proj_data.data_ptr(), m.gate_up_proj_scales.data_ptr(), m.gate_up_proj_scales.numel() // E,
        m.gate_up_proj_bias.data.data_ptr(), m.down_proj_data.data_ptr(), m.down_proj_scales.data_ptr(),
        m.down_proj_scales.numel() // E, m.down_proj_bias.data.data_ptr(), ctypes.c_float(1.702),
        ctypes.c_float(7.0), small.data_ptr(), 0, None, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 1 and b"GPTOSS_NOALLOC_SCRATCH_BYTES" in lib.gptoss_last_error()
