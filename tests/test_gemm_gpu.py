"""W4A8 grouped GEMM (cutlass::fp4_group_mm) parity with the oracle's dequantised
semantics, both MMA orientations. The reference's criterion is mean-abs relative error
< 1e-3 (kernels/test_cutlass_experts.py:159-329); the accumulation here is fp32 on both
sides, so most outputs agree bit-for-bit after bf16 rounding."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

MODES = {"tokens_m": 1, "swap": 2}


def _problem(m_list, N, K, seed, a_cols=None):
    g = torch.Generator().manual_seed(seed)
    E = len(m_list)
    M = sum(m_list)
    a_cols = a_cols or K
    x = torch.randn(M, a_cols, generator=g).to(torch.bfloat16)
    a_codes, a_sf = O.quantize_fp8_ue8m0(x)
    wb = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.uint8)
    ws = torch.randint(118, 126, (E, N, K // 32), generator=g, dtype=torch.uint8)
    counts = np.array(m_list, dtype=np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    return a_codes, a_sf, wb, ws, counts, offsets


def _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, K, mode, out_rows=None):
    E, N = wb.shape[0], wb.shape[1]
    M = a_codes.shape[0]
    a = torch.from_numpy(a_codes).view(torch.float8_e4m3fn).to(dev)
    if a.shape[1] < K:   # the op takes padded activations like the reference
        a = torch.nn.functional.pad(a.view(torch.uint8), (0, K - a.shape[1])).view(torch.float8_e4m3fn)
        a_sf = np.pad(a_sf, ((0, 0), (0, K // 32 - a_sf.shape[1])))
    sfa, sfo = O.batch_convert_a_scales(a_sf, counts, offsets)
    sfb = np.stack([O.convert_scales_blocked(ws[e].numpy()) for e in range(E)])
    ps = np.stack([counts, np.full(E, N), np.full(E, K)], axis=1).astype(np.int32)
    out = torch.full((out_rows or M, N), 7.0, dtype=torch.bfloat16, device=dev)
    pkg.ops.fp4_group_mm_impl(out, a, wb.to(dev), torch.from_numpy(np.ascontiguousarray(sfa) if sfa.size else
                                                                  np.zeros(16, np.uint8)).to(dev),
                              torch.from_numpy(sfb).to(dev), torch.ones(E, device=dev),
                              torch.from_numpy(ps).to(dev), torch.from_numpy(offsets).to(dev),
                              torch.from_numpy(sfo).to(dev), gemm_mode=mode)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    return out.cpu()


def _check(out, ref, what):
    o = out.float()
    r = ref.float()
    rel = ((o - r).abs().mean() / r.abs().mean().clamp_min(1e-30)).item()
    exact = (out.view(torch.int16) == ref.view(torch.int16)).float().mean().item()
    assert rel < 1e-3, f"{what}: mean-abs rel {rel:.2e}"
    assert exact > 0.97, f"{what}: only {exact:.3f} of outputs bit-exact"
    return rel, exact


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (64, 128, 256), (256, 512, 1024)])
def test_single_expert(pkg, dev, mode, M, N, K):
    a_codes, a_sf, wb, ws, counts, offsets = _problem([M], N, K, seed=M + N)
    out = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, K, MODES[mode])
    ref = O.group_mm_bf16(a_codes, a_sf, wb.numpy(), ws.numpy(), counts, offsets)
    _check(out, ref, f"{mode} {M}x{N}x{K}")


@pytest.mark.parametrize("mode", list(MODES))
def test_multi_expert(pkg, dev, mode):
    a_codes, a_sf, wb, ws, counts, offsets = _problem([64, 32, 128, 64], 256, 512, seed=42)
    out = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 512, MODES[mode])
    ref = O.group_mm_bf16(a_codes, a_sf, wb.numpy(), ws.numpy(), counts, offsets)
    _check(out, ref, mode)


@pytest.mark.parametrize("mode", list(MODES))
def test_ragged_with_empty_experts_and_padded_k(pkg, dev, mode):
    # rows not multiples of 32/128, 0-token experts, K = 2880 padded to 2944, N = 2880
    m = [300, 0, 7, 129, 0, 33]
    a_codes, a_sf, wb, ws, counts, offsets = _problem(m, 2880, 2944, seed=5, a_cols=2880)
    out = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 2944, MODES[mode])
    ref = O.group_mm_bf16(a_codes, a_sf, wb[:, :, :1440].contiguous().numpy(), ws[:, :, :90].contiguous().numpy(),
                          counts, offsets)
    _check(out, ref, mode)


@pytest.mark.parametrize("mode", list(MODES))
def test_gate_up_shape(pkg, dev, mode):
    a_codes, a_sf, wb, ws, counts, offsets = _problem([5, 70], 5760, 2944, seed=9)
    out = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 2944, MODES[mode])
    ref = O.group_mm_bf16(a_codes, a_sf, wb.numpy(), ws.numpy(), counts, offsets)
    _check(out, ref, mode)


def test_rows_owned_by_no_expert_untouched(pkg, dev):
    a_codes, a_sf, wb, ws, counts, offsets = _problem([16, 16], 256, 512, seed=3)
    out = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 512, 0, out_rows=40)
    assert torch.all(out[32:] == 7.0)


def test_orientations_agree(pkg, dev):
    a_codes, a_sf, wb, ws, counts, offsets = _problem([40, 3, 90], 576, 384, seed=8)
    o1 = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 384, 1)
    o2 = _run(pkg, dev, a_codes, a_sf, wb, ws, counts, offsets, 384, 2)
    assert (o1.float() - o2.float()).abs().max().item() <= (o1.float().abs().max().item() * 2 ** -7)


@pytest.mark.parametrize("m_list,H,I", [([5, 0, 17, 40], 512, 256), ([3, 9], 288, 288)])
def test_run_cutlass_gemm_reference_signature(pkg, dev, m_list, H, I):
    # CutlassGptOssExperts._run_cutlass_gemm keeps the reference's signature
    # (kernels/cutlass_experts.py:329-374) for subclasses such as the reference's benchmark
    # variants: unpadded FP8 activations with row-major scales in, K padded inside,
    # blocked scales built on the GPU, fp4_group_mm on the module's gate_up weights
    from helpers import build_experts
    E = len(m_list)
    d = O.synth_layer(41, E=E, H=H, I=I, T=1)
    m = build_experts(pkg, d, dev, E, H, I)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(sum(m_list), H, generator=g).to(torch.bfloat16)
    a_codes, a_sf = O.quantize_fp8_ue8m0(x)
    counts = torch.tensor(m_list, dtype=torch.int32)
    offsets = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(counts, 0)[:-1].to(torch.int32)])
    out = m._run_cutlass_gemm(torch.from_numpy(a_codes).view(torch.float8_e4m3fn).to(dev),
                              torch.from_numpy(a_sf).to(dev), m.gate_up_proj_data, m.gate_up_proj_scales,
                              counts.to(dev), offsets.to(dev), 2 * I, H, m.K_hidden_padded)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    ref = O.group_mm_bf16(a_codes, a_sf, d["gu_blocks"].numpy(), d["gu_scales"].numpy(), counts.numpy(),
                          offsets.numpy())
    _check(out.cpu(), ref, f"_run_cutlass_gemm m={m_list} H={H}")
