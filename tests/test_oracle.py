"""Pins the CPU oracle to the reference: golden vectors produced by the reference's own
Python (tests/golden/make_golden.py) and CuTe's blocked layout (cute_sf_layout.cu)."""
import hashlib
import os

import numpy as np
import pytest
import torch

import oracle as O
from golden import make_golden as MG
from helpers import GOLDEN, bf16_from_int16, golden


def _sha(*arrays):
    return MG.sha(*arrays)


def test_quantizer_matches_reference_golden():
    g = golden("quant.npz")
    for name, x in MG.quant_inputs():
        assert bytes(g[f"{name}__sha"]).decode() == _sha(x), f"{name}: input generator drifted"
        codes, sf = O.quantize_fp8_ue8m0(x)
        assert np.array_equal(codes, g[f"{name}__codes"]), name
        assert np.array_equal(sf, g[f"{name}__scales"]), name


def test_e4m3_encoder_matches_torch_cast_and_roundtrips():
    codes = np.arange(256, dtype=np.uint8)
    finite = ~np.isnan(O.e4m3_decode(codes))
    vals = O.e4m3_decode(codes)[finite]
    assert np.array_equal(O.e4m3_encode(vals), codes[finite])
    v = torch.linspace(-448, 448, 100001)
    assert np.array_equal(O.e4m3_encode(v.numpy()), v.to(torch.float8_e4m3fn).view(torch.uint8).numpy())


def test_swiglu_matches_reference_golden():
    g = golden("swiglu.npz")
    for name, x in MG.swiglu_inputs():
        assert bytes(g[f"{name}__sha"]).decode() == _sha(x)
        y = O.swiglu_fp32(x)
        ref = g[f"{name}__out"]
        got = y.view(torch.int16).numpy() if y.dtype == torch.bfloat16 else y.numpy()
        assert np.array_equal(got, ref), name


def _cute_shapes(name="cute_sf_layout.txt"):
    path = os.path.join(GOLDEN, name)
    lines = open(path).read().strip().splitlines()
    i = 0
    out = []
    while i < len(lines):
        rows, K, cos_a, cos_b = map(int, lines[i].split())
        offs = np.array([list(map(int, lines[i + 1 + r].split())) for r in range(rows)], dtype=np.int64)
        out.append((rows, K, cos_a, cos_b, offs))
        i += 1 + rows
    return out


def test_blocked_layout_matches_cute():
    shapes = _cute_shapes()
    assert len(shapes) >= 5
    for rows, K, cos_a, cos_b, offs in shapes:
        G = K // 32
        assert O.blocked_sf_cosize(rows, G) == cos_a == cos_b
        r, g = np.meshgrid(np.arange(rows), np.arange(G), indexing="ij")
        assert np.array_equal(O.blocked_sf_offset(r, g, (G + 3) // 4), offs), (rows, K)


def test_blocked_layout_16_matches_cute():
    # the NVFP4 mode's layout (Sm1xxBlockScaledConfig<16>): the same closed form with one
    # group per 16 codes, so an atom spans 64 codes
    shapes = _cute_shapes("cute_sf_layout16.txt")
    assert len(shapes) >= 5
    for rows, K, cos_a, cos_b, offs in shapes:
        G = K // 16
        assert O.blocked_sf_cosize(rows, G) == cos_a == cos_b
        r, g = np.meshgrid(np.arange(rows), np.arange(G), indexing="ij")
        assert np.array_equal(O.blocked_sf_offset(r, g, (G + 3) // 4), offs), (rows, K)
        sf = np.random.default_rng(rows).integers(0, 256, (rows, G), dtype=np.uint8)
        assert np.array_equal(O.unblock_scales(O.convert_scales_blocked(sf), rows, G), sf)


def test_nvfp4_oracle_small_case():
    # one row, one weight row, K = 64: the dot product by hand
    a = np.zeros((1, 32), np.uint8)
    b = np.zeros((1, 1, 32), np.uint8)
    a[0, 0] = 0x2F        # codes k=0: -6 (0xF), k=1: 1.0 (0x2)
    b[0, 0, 0] = 0x37     # k=0: 6.0, k=1: 1.5
    a[0, 8] = 0x05        # k=16: 3.0 (second 16-group)
    b[0, 0, 8] = 0x02     # k=16: 1.0
    a_sf = np.array([[0x38, 0x40, 0x38, 0x38]], np.uint8)      # 1, 2, 1, 1
    b_sf = np.array([[[0x30, 0x38, 0x38, 0x38]]], np.uint8)    # 0.5, 1, 1, 1
    sfa = O.convert_scales_blocked(a_sf)
    sfb = O.convert_scales_blocked(b_sf[0])[None]
    out = O.nvfp4_group_mm(a, b, sfa, sfb, np.array([2.0], np.float32), [1], [0], [0])
    # (-6*6 + 1*1.5) * 1 * 0.5 + 3 * 1 * 2 * 1 = -17.25 + 6 = -11.25; x alpha 2
    assert out.float().item() == -22.5


def test_documented_cosize():
    # cutlass_matmul_investigations.md:155-157: N=2880, K=2880 -> 270,848 bytes
    assert O.blocked_sf_cosize(2880, 2880 // 32) == 270848
    assert O.blocked_sf_cosize(5760, 2944 // 32) == 529920


def test_routing_matches_reference_golden():
    g = golden("routing.npz")
    st, se, sw, counts, offsets = O.route_stable(g["router_indices"], g["routing_weights"], 32)
    assert np.array_equal(counts, g["counts"])
    assert np.array_equal(offsets, g["offsets"])
    assert np.array_equal(st, g["sorted_token"])
    assert np.array_equal(se, g["router_indices"].reshape(-1)[np.argsort(g["router_indices"].reshape(-1), kind="stable")])


def test_batch_convert_equals_per_expert_convert():
    # kernels/test_cutlass_experts.py:789-840 (m = [64, 0, 128, 32], K = 512)
    rng = np.random.default_rng(42)
    m = [64, 0, 128, 32]
    scales = rng.integers(0, 256, size=(sum(m), 16), dtype=np.uint8)
    counts = np.array(m, dtype=np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    flat, sf = O.batch_convert_a_scales(scales, counts, offsets)
    parts, ref_sf, cur, o = [], [], 0, 0
    for mi in m:
        ref_sf.append(cur)
        if mi:
            blk = O.convert_scales_blocked(scales[o:o + mi])
            parts.append(blk)
            cur += blk.size
            o += mi
    assert np.array_equal(flat, np.concatenate(parts))
    assert np.array_equal(sf, np.array(ref_sf, dtype=np.int32))


@pytest.mark.parametrize("name", ["small", "kpad", "decode", "cpu_ref"])
def test_layer_matches_reference_golden(name):
    g = golden(f"layer_{name}.npz")
    d, idx, w = MG.layer_inputs(name)
    assert bytes(g["inputs_sha"]).decode() == _sha(d["hidden"], d["gu_blocks"], d["gu_scales"], d["dn_blocks"],
                                                   d["dn_scales"], d["gu_bias"], d["dn_bias"])
    assert np.array_equal(idx.numpy(), g["router_indices"])
    torch.set_num_threads(os.cpu_count() or 1)
    out, im = O.w4a8_experts_forward(d["hidden"], idx.numpy(), w.numpy(), O.numpy_weights(d),
                                     return_intermediates=True)
    assert np.array_equal(im["counts"], g["counts"])
    assert hashlib.sha256(im["act_codes"].tobytes()).hexdigest() == bytes(g["act_codes_sha"]).decode()
    assert hashlib.sha256(im["act_scales"].tobytes()).hexdigest() == bytes(g["act_scales_sha"]).decode()
    assert torch.equal(out.view(torch.int16), bf16_from_int16(g["out"]).view(torch.int16)), name


def test_dequant_reference_distance():
    # kernels/test_cutlass_experts.py:457-471 accepts mean-abs rel < 0.15 for W4A8 vs
    # the dequantised reference; the README reports 0.044.
    d, idx, w = MG.layer_inputs("small")
    wn = O.numpy_weights(d)
    out = O.w4a8_experts_forward(d["hidden"], idx.numpy(), w.numpy(), wn)
    ref = O.dequant_fp32_reference(d["hidden"], idx.numpy(), w.numpy(), wn)
    rel = ((out.float() - ref.float()).abs().mean() / ref.float().abs().mean()).item()
    assert rel < 0.15


def test_round_bf16_exact_rounds_once():
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 (ties to even -> 1); just above the tie
    # rounds up, although float32(1 + 2^-8 + 2^-40) is the tie itself (a float32
    # intermediate would double-round it down)
    v = np.array([1.0 + 2.0 ** -8, 1.0 + 2.0 ** -8 + 2.0 ** -40, -(1.0 + 3 * 2.0 ** -8), 3.0, -0.15625])
    r = O.round_bf16_exact(v).float().numpy()
    assert r.tolist() == [1.0, 1.0 + 2.0 ** -7, -(1.0 + 2.0 ** -6), 3.0, -0.15625]


def test_router_logits_exact_matches_fp32_router_almost_everywhere():
    d = O.synth_layer(0, E=32, H=2880, I=64, T=32)
    ex = O.router_logits_exact(d["hidden"], d["router_w"], d["router_b"])
    f32 = O.router_logits_fp32(d["hidden"], d["router_w"], d["router_b"])
    # both round the same real number; they can only differ where fp32 accumulation error
    # crosses a bf16 rounding boundary (a handful of the 1024 logits at most)
    assert (ex != f32).sum().item() <= 8
    assert ((ex.float() - f32.float()).abs() <= ex.float().abs() * 2 ** -7 + 1e-30).all()


def test_rmsnorm_restatement_matches_hf_module():
    # the block op's norm is held to this restatement on the GPU; here it is pinned to the
    # transformers module the reference's model runs (bf16 model, weight in bf16)
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssRMSNorm
    g = torch.Generator().manual_seed(4)
    for H in (64, 2880):
        norm = GptOssRMSNorm(H, eps=1e-5).to(torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16))
        x = (3 * torch.randn(17, H, generator=g)).to(torch.bfloat16)
        with torch.no_grad():
            ref = norm(x)
        assert torch.equal(O.rmsnorm_hf(x, norm.weight.data, 1e-5), ref)
