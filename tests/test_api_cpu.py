"""Drop-in API surface checks that run without a GPU (module state, helpers, op schemas
and fake kernels, and the refusal to compute on CPU tensors)."""
import pytest
import torch

from helpers import Cfg


def test_module_state_matches_reference(pkg):
    m = pkg.CutlassGptOssExperts(Cfg(32, 2880, 2880))
    assert m.num_experts == 32 and m.hidden_size == 2880 and m.intermediate_size == 2880
    assert m.alpha == 1.702 and m.limit == 7.0
    assert m.gate_up_proj_bias.shape == (32, 5760) and m.gate_up_proj_bias.dtype == torch.float32
    assert m.down_proj_bias.shape == (32, 2880) and m.down_proj_bias.dtype == torch.float32
    assert not m.gate_up_proj_bias.requires_grad and not m.down_proj_bias.requires_grad
    for b in ("gate_up_proj_data", "gate_up_proj_scales", "down_proj_data", "down_proj_scales"):
        assert getattr(m, b) is None
    c = Cfg(4, 512, 256)
    del c.swiglu_limit
    assert pkg.CutlassGptOssExperts(c).limit == 7.0


def test_padding_helpers(pkg):
    assert pkg.pad_k_to_tile(2880) == 2944 and pkg.pad_k_to_tile(288) == 384 and pkg.pad_k_to_tile(512) == 512
    a = torch.zeros(3, 2880, dtype=torch.float8_e4m3fn)
    s = torch.ones(3, 90, dtype=torch.uint8)
    a2, s2, k = pkg.pad_fp8_activations(a, s, 2880)
    assert a2.shape == (3, 2944) and s2.shape == (3, 92) and k == 2944 and a2.dtype == torch.float8_e4m3fn
    assert int(s2[:, 90:].sum()) == 0
    d = torch.ones(5, 1440, dtype=torch.uint8)
    d2, s3, k = pkg.pad_fp4_weights(d, torch.ones(5, 90, dtype=torch.uint8), 2880)
    assert d2.shape == (5, 1472) and s3.shape == (5, 92) and int(d2[:, 1440:].sum()) == 0


def test_extension_object_surface(pkg):
    ext = pkg.get_cutlass_extension()
    for name in ("cutlass_fp4_group_mm", "convert_a_scales_for_w4a8", "convert_b_scales_for_w4a8",
                 "batch_convert_a_scales_for_w4a8", "batch_convert_a_scales_for_w4a8_gpu", "fused_moe_routing"):
        assert callable(getattr(ext, name))


def test_ops_registered_with_reference_qualnames(pkg):
    pkg.ensure_custom_op_registered()
    pkg.ensure_custom_op_registered()   # idempotent
    assert hasattr(torch.ops.cutlass, "fp4_group_mm")
    assert hasattr(torch.ops.cutlass, "fused_moe_routing")
    for n in ("moe_experts_forward", "moe_layer_forward", "moe_block_forward", "quantize_fp8", "swiglu",
              "router_topk", "route_quant", "gemm1", "gemm2", "ep_dispatch", "ep_expert_forward", "ep_combine"):
        assert hasattr(torch.ops.gptoss, n)


def test_fake_kernels_give_static_shapes(pkg):
    pkg.ensure_custom_op_registered()
    meta = torch.device("meta")
    idx = torch.empty(7, 4, dtype=torch.int64, device=meta)
    w = torch.empty(7, 4, dtype=torch.float32, device=meta)
    outs = torch.ops.cutlass.fused_moe_routing(idx, w, 32)
    assert [tuple(o.shape) for o in outs] == [(28,), (28,), (28,), (32,), (32,)]
    assert [o.dtype for o in outs] == [torch.int64, torch.int64, torch.float32, torch.int32, torch.int32]
    h = torch.empty(7, 512, dtype=torch.bfloat16, device=meta)
    y = torch.ops.gptoss.moe_experts_forward(
        h, idx, w, torch.empty(4, 512, 256, dtype=torch.uint8, device=meta),
        torch.empty(4, 16384, dtype=torch.uint8, device=meta), torch.empty(4, 512, device=meta),
        torch.empty(4, 512, 128, dtype=torch.uint8, device=meta), torch.empty(4, 8192, dtype=torch.uint8, device=meta),
        torch.empty(4, 512, device=meta), 1.702, 7.0, 0)
    assert y.shape == (7, 512) and y.dtype == torch.bfloat16
    q, s = torch.ops.gptoss.quantize_fp8(torch.empty(5, 64, dtype=torch.bfloat16, device=meta))
    assert q.shape == (5, 64) and q.dtype == torch.float8_e4m3fn and s.shape == (5, 2)
    # expert parallelism: static shapes from the arguments alone
    rb = pkg.ops.ep_row_bytes(512)
    rows, counts, pos = torch.ops.gptoss.ep_dispatch(h, idx, w, 32, 4, 40)
    assert rows.shape == (160, rb) and rows.dtype == torch.uint8 and counts.shape == (4,) and pos.shape == (28,)
    rows, _, _ = torch.ops.gptoss.ep_dispatch(h, idx, w, 32, 4, 0)
    assert rows.shape == (28, rb)
    back = torch.ops.gptoss.ep_expert_forward(
        torch.empty(28, rb, dtype=torch.uint8, device=meta), torch.empty(8, 512, 256, dtype=torch.uint8, device=meta),
        torch.empty(8, 16384, dtype=torch.uint8, device=meta), torch.empty(8, 512, device=meta),
        torch.empty(8, 512, 128, dtype=torch.uint8, device=meta), torch.empty(8, 8192, dtype=torch.uint8, device=meta),
        torch.empty(8, 512, device=meta), 1.702, 7.0, 0)
    assert back.shape == (28, 512) and back.dtype == torch.bfloat16
    out = torch.ops.gptoss.ep_combine(back, pos, idx)
    assert out.shape == (7, 512) and out.dtype == torch.bfloat16
    # the decoder block op: out, scores, indices
    o, sc, ix = torch.ops.gptoss.moe_block_forward(
        h, torch.empty(512, dtype=torch.bfloat16, device=meta), 1e-5, torch.empty(4, 512, dtype=torch.bfloat16, device=meta),
        torch.empty(4, dtype=torch.bfloat16, device=meta), 2, torch.empty(4, 512, 256, dtype=torch.uint8, device=meta),
        torch.empty(4, 16384, dtype=torch.uint8, device=meta), torch.empty(4, 512, device=meta),
        torch.empty(4, 512, 128, dtype=torch.uint8, device=meta), torch.empty(4, 8192, dtype=torch.uint8, device=meta),
        torch.empty(4, 512, device=meta), 1.702, 7.0, 0)
    assert o.shape == (7, 512) and sc.shape == (7, 2) and ix.shape == (7, 2) and ix.dtype == torch.int64


def test_one_launch_expert_parallel_gate(pkg):
    # when a decode-sized expert-parallel step runs as one launch per rank (a pure function of
    # the group's common sizes, so every rank decides alike): tokens, received rows, rows per
    # local expert, capacity; and the process-wide switch
    fits = pkg.ops.ep_p2p_layer_fits
    assert fits(32, 4, 32, 8, 2880, 2880, 128) and fits(32, 4, 32, 2, 2880, 2880, 128)
    assert fits(0, 4, 32, 2, 2880, 2880, 128)                  # a rank without tokens takes part
    assert not fits(65, 4, 32, 1, 2880, 2880, 260)             # > 64 tokens
    assert not fits(32, 4, 32, 8, 2880, 2880, 160)             # 8 x 160 > 1024 received rows
    assert not fits(32, 4, 32, 2, 2880, 2880, 100)             # capacity < T x k
    assert fits(64, 4, 8, 2, 512, 512, 256)                    # 64 rows per local expert
    assert not fits(64, 4, 8, 2, 512, 512, 272)                # 68
    assert not fits(32, 4, 30, 4, 2880, 2880, 128)             # E not a multiple of W
    prev = pkg.ops.set_ep_layer_kernel(False)
    try:
        assert not fits(32, 4, 32, 8, 2880, 2880, 128)
    finally:
        pkg.ops.set_ep_layer_kernel(prev)


def test_cpu_tensors_are_refused(pkg):
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        pkg.ops.quantize_fp8(x)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        pkg.ops.fused_moe_routing_impl(torch.zeros(2, 2, dtype=torch.int64), torch.zeros(2, 2), 4)


def test_forward_requires_loaded_weights(pkg):
    m = pkg.CutlassGptOssExperts(Cfg(4, 512, 256))
    with pytest.raises(RuntimeError, match="not loaded"):
        m(torch.zeros(2, 512, dtype=torch.bfloat16), torch.zeros(2, 2, dtype=torch.int64), torch.zeros(2, 2))


def test_standalone_file_load_like_reference_tests():
    # The reference's tests load cutlass_experts.py by path (kernels/test_cutlass_experts.py:28-31).
    import importlib.util
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpt-oss-mxfp4-compile_b200",
                        "cutlass_experts.py")
    spec = importlib.util.spec_from_file_location("cutlass_experts", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.pad_k_to_tile(2880) == 2944 and hasattr(mod, "CutlassGptOssExperts")
