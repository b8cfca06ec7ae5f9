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


def _noalloc(pkg, m, hidden, idx, w, out, mode=0):
    lib = pkg._lib.load()
    E, H, I = m.num_experts, m.hidden_size, m.intermediate_size
    T, k = idx.shape
    rc = lib.gptoss_moe_experts_forward_noalloc(
        hidden.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k, E, H, I,
        m.gate_up_proj_data.data_ptr(), m.gate_up_proj_scales.data_ptr(), m.gate_up_proj_scales.numel() // E,
        m.gate_up_proj_bias.data.data_ptr(), m.down_proj_data.data_ptr(), m.down_proj_scales.data_ptr(),
        m.down_proj_scales.numel() // E, m.down_proj_bias.data.data_ptr(), ctypes.c_float(m.alpha),
        ctypes.c_float(m.limit), out.data_ptr(), int(mode), pkg.ops.status_tensor(hidden.device).data_ptr(),
        torch.cuda.current_stream(hidden.device).cuda_stream)
    assert rc == 0, lib.gptoss_last_error().decode()
    return out


def _batch(g, T, E, H, dev):
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    wv, ix = torch.topk(torch.randn(T, E, generator=g), 4, dim=-1)
    return hidden, ix, torch.softmax(wv, -1)


@pytest.mark.parametrize("mode", [0, 1, 2, 3])   # GPTOSS_GEMM_AUTO / TOKENS_M / SWAP / SWAP_WIDE
def test_noalloc_matches_workspace_forward_on_consecutive_calls(pkg, dev, mode):
    E, H, I = 32, 2880, 2880
    d = O.synth_layer(31, E=E, H=H, I=I, T=1)
    m = build_experts(pkg, d, dev, E, H, I)
    g = torch.Generator().manual_seed(7)
    prev_mode = m.gemm_mode
    try:
        for T in (48, 32):   # two calls in a row reuse the same static scratch
            hidden, ix, wv = _batch(g, T, E, H, dev)
            hd, ixd, wvd = hidden.to(dev), ix.to(dev), wv.to(dev)
            got = _noalloc(pkg, m, hd, ixd, wvd, torch.empty_like(hd), mode)
            m.gemm_mode = mode
            ref = m(hd, ixd, wvd)          # gptoss_moe_experts_forward with a torch workspace
            torch.cuda.synchronize()
            assert pkg.ops.read_status(dev) == 0
            assert_output_tolerance(got.cpu(), ref.cpu(), f"noalloc T={T} mode={mode}")
            if mode == 0:                  # and the oracle's W4A8 forward on the same routing
                want = O.w4a8_experts_forward(hidden, ix.numpy(), wv.numpy(), O.numpy_weights(d))
                assert_output_tolerance(got.cpu(), want, f"noalloc vs oracle T={T}")
    finally:
        m.gemm_mode = prev_mode


def test_noalloc_allocates_nothing(pkg, dev):
    # a batch near the scratch limit (64-row chunks: 70 rows per expert on average); after
    # a warm-up call, a second call changes neither the device's free memory nor torch's
    E, H, I = 32, 2880, 2880
    d = O.synth_layer(33, E=E, H=H, I=I, T=1)
    m = build_experts(pkg, d, dev, E, H, I)
    g = torch.Generator().manual_seed(8)
    hidden, ix, wv = _batch(g, 560, E, H, dev)
    hd, ixd, wvd = hidden.to(dev), ix.to(dev), wv.to(dev)
    got, again = torch.empty_like(hd), torch.empty_like(hd)
    _noalloc(pkg, m, hd, ixd, wvd, got)
    torch.cuda.synchronize()
    free0, alloc0, res0 = torch.cuda.mem_get_info(dev)[0], torch.cuda.memory_allocated(dev), \
        torch.cuda.memory_reserved(dev)
    _noalloc(pkg, m, hd, ixd, wvd, again)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert torch.cuda.memory_allocated(dev) == alloc0 and torch.cuda.memory_reserved(dev) == res0
    assert pkg.ops.read_status(dev) == 0
    ref = m(hd, ixd, wvd)
    torch.cuda.synchronize()
    assert_output_tolerance(got.cpu(), ref.cpu(), "noalloc T=560")
    assert_output_tolerance(again.cpu(), ref.cpu(), "noalloc T=560, second call")


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
