"""W4A4 (NVFP4 x NVFP4) mode of cutlass::fp4_group_mm: packed E2M1 activations and weights,
UE4M3 scales per 16 codes in the blocked layout, tcgen05 kind::mxf4nvf4. The reference has
no numeric check of this mode (its test compares torch.compile with eager,
test_mxfp4_matmul.py:157-182); here the oracle is the dequantise-and-multiply restatement
(oracle.nvfp4_group_mm). Products are exact and both sides accumulate in at least fp32, so
the bar is the W4A8 tests': mean-abs relative error < 1e-3, > 97 % of outputs bit-exact
after bf16 rounding, and every output within 2^-7 of the largest |output| of its row
block."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

MODES = {"tokens_m": 1, "swap": 2}


def _scale_bytes(g, shape, lo=0x30, hi=0x41):
    # UE4M3 scales (sign bit clear) between 0.5 and 2.25
    return torch.randint(lo, hi, shape, generator=g, dtype=torch.uint8).numpy()


def _problem(m_list, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    E = len(m_list)
    M = sum(m_list)
    G = K // 16
    a = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.uint8).numpy()
    b = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.uint8).numpy()
    a_sf = _scale_bytes(g, (M, G))
    b_sf = _scale_bytes(g, (E, N, G))
    counts = np.array(m_list, dtype=np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    # expert e's activation scales: a blocked buffer of pad128(m_e) rows, laid end to end;
    # sf_offsets count ROWS (the reference multiplies them by K/16)
    parts, sf_rows, cur = [], [], 0
    for m, o in zip(counts.tolist(), offsets.tolist()):
        sf_rows.append(cur)
        if m:
            parts.append(O.convert_scales_blocked(a_sf[o:o + m]))
            cur += (m + 127) // 128 * 128
    sfa = np.concatenate(parts) if parts else np.zeros(512, np.uint8)
    sfb = np.stack([O.convert_scales_blocked(b_sf[e]) for e in range(E)])
    alphas = (0.5 + torch.rand(E, generator=g)).numpy().astype(np.float32)
    return a, b, sfa, sfb, alphas, counts, offsets, np.array(sf_rows, dtype=np.int32)


def _inputs(dev, a, b, sfa, sfb, alphas, counts, offsets, sf_rows, N, K, sf_dtype=torch.uint8):
    E = b.shape[0]
    ps = np.stack([counts, np.full(E, N), np.full(E, K)], axis=1).astype(np.int32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)   # noqa: E731
    return (t(a), t(b), t(sfa).view(sf_dtype), t(sfb).view(sf_dtype), t(alphas), t(ps), t(offsets), t(sf_rows))


def _run(pkg, dev, prob, N, K, mode, out_rows=None):
    a, b, sfa, sfb, alphas, counts, offsets, sf_rows = prob
    ins = _inputs(dev, *prob, N, K)
    out = torch.full((out_rows or a.shape[0], N), 7.0, dtype=torch.bfloat16, device=dev)
    pkg.ops.fp4_group_mm_impl(out, *ins, gemm_mode=mode)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    return out.cpu()


def _check(out, ref, what):
    o, r = out.float(), ref.float()
    rel = ((o - r).abs().mean() / r.abs().mean().clamp_min(1e-30)).item()
    exact = (out.view(torch.int16) == ref.view(torch.int16)).float().mean().item()
    worst = ((o - r).abs() / r.abs().amax(dim=1, keepdim=True).clamp_min(1e-30)).max().item()
    assert rel < 1e-3, f"{what}: mean-abs rel {rel:.2e}"
    assert exact > 0.97, f"{what}: only {exact:.3f} of outputs bit-exact"
    assert worst <= 2 ** -7, f"{what}: worst error {worst:.2e} of the row's largest output"


def _ref(prob):
    a, b, sfa, sfb, alphas, counts, offsets, sf_rows = prob
    return O.nvfp4_group_mm(a, b, sfa, sfb, alphas, counts, offsets, sf_rows)


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (64, 128, 256), (256, 512, 1024)])
def test_single_expert(pkg, dev, mode, M, N, K):
    prob = _problem([M], N, K, seed=M + N + K)
    _check(_run(pkg, dev, prob, N, K, MODES[mode]), _ref(prob), f"{mode} {M}x{N}x{K}")


@pytest.mark.parametrize("mode", list(MODES))
def test_ragged_experts_partial_k_block(pkg, dev, mode):
    # rows not multiples of 16/64/128, empty experts, K = 2880 (11 full 256-code k blocks
    # and one of 64 codes), N = 2880 (a 192-row tile and a 128-row block that straddle)
    m = [300, 0, 7, 129, 0, 33]
    prob = _problem(m, 2880, 2880, seed=5)
    _check(_run(pkg, dev, prob, 2880, 2880, MODES[mode]), _ref(prob), f"{mode} ragged")


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("K", [64, 320])
def test_short_k(pkg, dev, mode, K):
    prob = _problem([40, 3, 90], 576, K, seed=K)
    _check(_run(pkg, dev, prob, 576, K, MODES[mode]), _ref(prob), f"{mode} K={K}")


def test_orientations_agree(pkg, dev):
    prob = _problem([40, 3, 90], 576, 768, seed=8)
    o1 = _run(pkg, dev, prob, 576, 768, 1)
    o2 = _run(pkg, dev, prob, 576, 768, 2)
    assert (o1.float() - o2.float()).abs().max().item() <= o1.float().abs().max().item() * 2 ** -7


def test_rows_owned_by_no_expert_untouched(pkg, dev):
    prob = _problem([16, 16], 256, 512, seed=3)
    out = _run(pkg, dev, prob, 256, 512, 0, out_rows=40)
    assert torch.all(out[32:] == 7.0)


def test_float8_scale_dtype_and_compile_match_eager(pkg, dev):
    # the reference's W4A4 test (test_mxfp4_matmul.py:157-182): M, N, K = 128, 256, 512, one
    # expert, alphas 1, float8_e4m3fn scale tensors; the op under torch.compile matches eager
    M, N, K = 128, 256, 512
    prob = list(_problem([M], N, K, seed=11))
    prob[4] = np.ones(1, np.float32)
    ins = _inputs(dev, *prob, N, K, sf_dtype=torch.float8_e4m3fn)
    eager = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    torch.ops.cutlass.fp4_group_mm(eager, *ins)
    torch.cuda.synchronize()

    def fn(output, a, b, a_bs, b_bs, alphas, ps, eo, so):
        torch.ops.cutlass.fp4_group_mm(output, a, b, a_bs, b_bs, alphas, ps, eo, so)

    compiled = torch.compile(fn, backend="inductor", fullgraph=True)
    out2 = torch.empty_like(eager)
    compiled(out2, *ins)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    assert torch.equal(out2, eager)
    _check(eager.cpu(), _ref(prob), "reference shape")


def test_bad_shapes_rejected(pkg, dev):
    prob = _problem([8], 128, 512, seed=1)
    a, b, sfa, sfb, alphas, ps, offs, sfo = _inputs(dev, *prob, 128, 512)
    out = torch.empty((8, 128), dtype=torch.bfloat16, device=dev)
    with pytest.raises(RuntimeError, match="K/2"):      # activations not [M, K/2]
        pkg.ops.fp4_group_mm_impl(out, a[:, :128].contiguous(), b, sfa, sfb, alphas, ps, offs, sfo)
    bk = torch.zeros(1, 128, 48, dtype=torch.uint8, device=dev)   # K = 96: not a multiple of 64
    with pytest.raises(RuntimeError, match="multiple of 64"):
        pkg.ops.fp4_group_mm_impl(out, torch.zeros(8, 48, dtype=torch.uint8, device=dev), bk, sfa, sfb, alphas,
                                  ps, offs, sfo)


def test_mma_peak_probe_both_kinds(pkg, dev):
    # the tensor-pipe probes behind the roofline denominators run to completion for both
    # block-scaled kinds and both CTA shapes
    for kind in ("mxf8f6f4", "mxf4nvf4"):
        for pair in (False, True):
            r = pkg.ops.mma_peak(dev, pair=pair, n=192, iters=200, repeats=1, kind=kind)
            assert r["tflops"] > 0.0
    assert pkg.ops.read_status(dev) == 0
