"""Parity of the individual sm_100a kernels with the oracle and the reference goldens:
quantiser and SwiGLU (bit-exact), blocked scale conversion (byte-exact), routing
(exact, including the permutation)."""
import numpy as np
import pytest
import torch

import oracle as O
from golden import make_golden as MG
from helpers import golden

pytestmark = pytest.mark.gpu


def test_quantize_matches_reference_golden(pkg, dev):
    g = golden("quant.npz")
    for name, x in MG.quant_inputs():
        q, s = pkg.quantize_activations_to_fp8(x.to(dev))
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g[f"{name}__codes"]), name
        assert np.array_equal(s.cpu().numpy(), g[f"{name}__scales"]), name
    assert pkg.ops.read_status(dev) == 0


@pytest.mark.parametrize("shape,dtype", [((1024, 2880), torch.bfloat16), ((33, 2880), torch.float32),
                                         ((1, 32), torch.bfloat16), ((4096, 512), torch.float32)])
def test_quantize_matches_oracle(pkg, dev, shape, dtype):
    g = torch.Generator().manual_seed(shape[0])
    x = (torch.randn(*shape, generator=g) * torch.logspace(-3, 3, shape[0]).unsqueeze(1)).to(dtype)
    q, s = pkg.quantize_activations_to_fp8(x.to(dev))
    c, sf = O.quantize_fp8_ue8m0(x)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), c)
    assert np.array_equal(s.cpu().numpy(), sf)


def _special_rows(H=2880):
    # groups holding NaN (both signs), +-inf, values near the bf16 maximum, bf16
    # subnormals, an all-zero group, and exact powers of two times 448
    g = torch.Generator().manual_seed(7)
    x = torch.randn(8, H, generator=g)
    x[0, 5] = float("nan")
    x[0, 40] = -float("nan")
    x[1, 70] = float("inf")
    x[1, 100] = -float("inf")
    x[2, :] *= 3.0e38 / 4.0
    x[3, :] *= 1e-39
    x[4, 32:64] = 0.0
    x[5, :32] = 448.0 * 2.0 ** torch.arange(-8, 24).float()
    x[6, 64:96] = 7.0 * 2.0 ** -130
    return x.to(torch.bfloat16)


def test_quantize_special_values_match_oracle(pkg, dev):
    # the plain quantiser and the fused gather path agree with the oracle on NaN / inf /
    # saturating / subnormal / zero groups, byte for byte
    # (a NaN code is compared as NaN: the sign of the NaN that inf / inf yields is the
    # platform's choice, positive on the GPU and negative on x86)
    def canon(codes):
        codes = codes.copy()
        codes[(codes & 0x7F) == 0x7F] = 0x7F
        return codes

    x = _special_rows()
    c, sf = O.quantize_fp8_ue8m0(x)
    c = canon(c)
    q, s = pkg.quantize_activations_to_fp8(x.to(dev))
    assert np.array_equal(s.cpu().numpy(), sf)
    assert np.array_equal(canon(q.view(torch.uint8).cpu().numpy()), c)
    T, E = x.shape[0], 4
    idx = (torch.arange(T) % E).reshape(T, 1)
    ws = pkg.ops.ExpertsWorkspace(T, 1, E, x.shape[1], 512, dev)
    pkg.ops.route_quant(ws, x.to(dev), idx.to(dev), torch.ones(T, 1, device=dev), 1)
    torch.cuda.synchronize()
    st = ws.sorted_token.cpu().numpy()
    assert np.array_equal(canon(ws.act_codes.cpu().numpy()), c[st])


def test_quantize_empty(pkg, dev):
    q, s = pkg.quantize_activations_to_fp8(torch.empty(0, 64, dtype=torch.bfloat16, device=dev))
    assert q.shape == (0, 64) and s.shape == (0, 2)


def test_swiglu_matches_reference_golden(pkg, dev):
    g = golden("swiglu.npz")
    for name, x in MG.swiglu_inputs():
        y = pkg.swiglu(x.to(dev), 1.702, 7.0).cpu()
        ref = g[f"{name}__out"]
        if y.dtype == torch.bfloat16:
            got = y.view(torch.int16).numpy().astype(np.int32)
            ulp = np.abs(got - ref.astype(np.int32))
            assert ulp.max() <= 1 and (ulp == 0).mean() > 0.99, name
        else:
            np.testing.assert_allclose(y.numpy(), ref, rtol=2e-6, atol=1e-30)


@pytest.mark.parametrize("rows,k", [(1, 256), (200, 2944), (5760, 2944), (2880, 2944), (129, 384), (64, 512)])
def test_convert_scales_matches_oracle(pkg, dev, rows, k):
    rng = np.random.default_rng(rows)
    s = rng.integers(0, 256, size=(rows, k // 32), dtype=np.uint8)
    ext = pkg.get_cutlass_extension()
    a = ext.convert_a_scales_for_w4a8(torch.from_numpy(s).to(dev), rows, 128, k).cpu().numpy()
    b = ext.convert_b_scales_for_w4a8(torch.from_numpy(s).to(dev), 128, rows, k).cpu().numpy()
    ref = O.convert_scales_blocked(s)
    assert np.array_equal(a, ref) and np.array_equal(b, ref)


def test_batch_convert_matches_per_expert(pkg, dev):
    # kernels/test_cutlass_experts.py:789-885 (tests 10 and 11)
    m = [64, 0, 128, 32]
    torch.manual_seed(42)
    scales = torch.randint(0, 256, (sum(m), 16), dtype=torch.uint8)
    counts = torch.tensor(m, dtype=torch.int32)
    offsets = torch.zeros(4, dtype=torch.int32)
    torch.cumsum(counts[:-1], 0, out=offsets[1:])
    ext = pkg.get_cutlass_extension()
    flat, sf = ext.batch_convert_a_scales_for_w4a8_gpu(scales.to(dev), counts.to(dev), offsets.to(dev), 256, 512)
    ref_flat, ref_sf = O.batch_convert_a_scales(scales.numpy(), counts.numpy(), offsets.numpy())
    assert np.array_equal(flat.cpu().numpy(), ref_flat) and np.array_equal(sf.cpu().numpy(), ref_sf)
    flat2, sf2 = ext.batch_convert_a_scales_for_w4a8(scales.to(dev), counts.to(dev), offsets.to(dev), 256, 512)
    assert torch.equal(flat2, flat) and torch.equal(sf2, sf)
    parts = [ext.convert_a_scales_for_w4a8(scales[o:o + mi].to(dev), mi, 256, 512)
             for mi, o in zip(m, offsets.tolist()) if mi]
    assert torch.equal(torch.cat(parts), flat)


def test_batch_convert_all_empty(pkg, dev):
    ext = pkg.get_cutlass_extension()
    flat, sf = ext.batch_convert_a_scales_for_w4a8_gpu(torch.zeros(0, 16, dtype=torch.uint8, device=dev),
                                                       torch.zeros(3, dtype=torch.int32, device=dev),
                                                       torch.zeros(3, dtype=torch.int32, device=dev), 256, 512)
    assert flat.numel() == 0 and sf.tolist() == [0, 0, 0]


def _check_routing(pkg, dev, idx, w, E):
    ext = pkg.get_cutlass_extension()
    st, se, sw, counts, offsets = ext.fused_moe_routing(idx.to(dev), w.to(dev), E)
    rst, rse, rsw, rc, ro = O.route_stable(idx.numpy(), w.numpy(), E)
    assert np.array_equal(counts.cpu().numpy(), rc) and np.array_equal(offsets.cpu().numpy(), ro)
    assert np.array_equal(st.cpu().numpy(), rst), "permutation differs from stable argsort"
    assert np.array_equal(se.cpu().numpy(), rse)
    assert np.array_equal(sw.cpu().numpy(), rsw)
    assert st.dtype == torch.int64 and se.dtype == torch.int64 and sw.dtype == torch.float32
    assert counts.dtype == torch.int32 and offsets.dtype == torch.int32


def test_routing_matches_reference_golden(pkg, dev):
    # kernels/test_cutlass_experts.py:892-958, but the permutation is checked exactly.
    g = golden("routing.npz")
    ext = pkg.get_cutlass_extension()
    idx = torch.from_numpy(g["router_indices"])
    w = torch.from_numpy(g["routing_weights"])
    st, se, sw, counts, offsets = ext.fused_moe_routing(idx.to(dev), w.to(dev), 32)
    assert np.array_equal(counts.cpu().numpy(), g["counts"])
    assert np.array_equal(offsets.cpu().numpy(), g["offsets"])
    assert np.array_equal(st.cpu().numpy(), g["sorted_token"])
    _check_routing(pkg, dev, idx, w, 32)


@pytest.mark.parametrize("T,E,k", [(1, 4, 2), (32, 32, 4), (8192, 32, 4), (16384, 128, 4), (3, 8, 8)])
def test_routing_random(pkg, dev, T, E, k):
    g = torch.Generator().manual_seed(T + E)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    _check_routing(pkg, dev, idx, w, E)


def test_routing_all_to_one_expert(pkg, dev):
    T = 300
    idx = torch.zeros(T, 2, dtype=torch.int64)
    idx[:, 1] = 1
    _check_routing(pkg, dev, idx, torch.full((T, 2), 0.5), 4)


def test_routing_bad_index_sets_status(pkg, dev):
    # Host-side fault injection: an out-of-range expert id is skipped by the kernel and
    # reported through the status word; nothing faults.
    pkg.ops.read_status(dev)
    idx = torch.tensor([[0, 1], [7, 2]], dtype=torch.int64, device=dev)
    pkg.get_cutlass_extension().fused_moe_routing(idx, torch.ones(2, 2, device=dev), 4)
    assert pkg.ops.read_status(dev) == 0x201
    assert pkg.ops.read_status(dev) == 0


# the four benchmark workloads' router shapes: decode, prefill (skewed loads), one layer of
# the T=4096 stack, the E=128 Zipf layer
ROUTER_SHAPES = [(32, 32, 0, None), (8192, 32, 0, "prefill"), (4096, 32, 3, None), (16384, 128, 0, "zipf")]


def _router_inputs(T, E, seed, skew):
    d = O.synth_layer(seed, E=E, H=2880, I=32, T=T, skew=skew)   # I small: only the router inputs matter
    return d["hidden"], d["router_w"], d["router_b"]


@pytest.mark.parametrize("T,E,seed,skew", ROUTER_SHAPES)
def test_router_topk_bit_exact_on_given_logits(pkg, dev, T, E, seed, skew):
    # the top-k + softmax half of the router is exact: fed the oracle's bf16 logits
    # (F.linear on the CPU) it returns the oracle's indices, in the same order (ties by lower
    # expert id), and bit-identical bf16 scores
    x, w, b = _router_inputs(T, E, seed, skew)
    logits = O.router_topk_hf(x, w, b, 4)[0]
    scores, idx = pkg.ops.router_topk_from_logits(logits.to(dev), 4)
    ref_scores, ref_idx = O.router_topk_from_logits(logits, 4)
    assert torch.equal(idx.cpu(), ref_idx)
    assert torch.equal(scores.cpu().view(torch.int16), ref_scores.view(torch.int16))


@pytest.mark.parametrize("T,E,seed,skew", ROUTER_SHAPES)
def test_router_logits_counted_exceptions(pkg, dev, T, E, seed, skew):
    # The router kernel's logits are an fp32-accumulated dot product rounded once to bf16,
    # as F.linear's are; the two sum in different orders, so they can land on neighbouring
    # bf16 values where the real sum is close to a rounding boundary (counted here, one ulp
    # at most). Its top-k is then exact on its own logits, and its routing differs from the
    # CPU router's only on tokens where a logit differs.
    x, w, b = _router_inputs(T, E, seed, skew)
    lg, sc, ix = torch.ops.gptoss.router_topk(x.to(dev), w.to(dev), b.to(dev), 4)
    lg, sc, ix = lg.cpu(), sc.cpu(), ix.cpu()
    exact = O.router_logits_exact(x, w, b)
    hf = O.router_topk_hf(x, w, b, 4)[0]

    # the fp32 accumulation of H products errs by at most H * 2^-24 * sum |x_i w_i|
    # (a bound, seldom approached); a mismatch is that error carried across a bf16 rounding
    # boundary, so it lies within the bound plus one bf16 ulp of the exact value
    sum_abs = torch.from_numpy(x.abs().double().numpy() @ w.abs().double().numpy().T)
    ulp = torch.ldexp(torch.ones_like(exact.double()), torch.frexp(exact.double())[1] - 8)
    bound = ulp + x.shape[1] * 2.0 ** -24 * sum_abs
    assert ((lg.double() - exact.double()).abs() <= bound).all()
    assert ((hf.double() - exact.double()).abs() <= bound).all()
    n_exact = int((lg.view(torch.int16) != exact.view(torch.int16)).sum())
    n_hf = int((lg.view(torch.int16) != hf.view(torch.int16)).sum())
    assert n_exact <= max(4, T * E // 500), (n_exact, T * E)
    print(f"router logits T={T} E={E}: {n_exact} of {T * E} differ from the exactly rounded value, "
          f"{n_hf} from the CPU F.linear")
    # top-k on the kernel's own logits: bit-exact
    rs, ri = O.router_topk_from_logits(lg, 4)
    assert torch.equal(ix, ri) and torch.equal(sc.view(torch.int16), rs.view(torch.int16))
    # against the CPU router: differences only where a logit differs
    hs, hi = O.router_topk_from_logits(hf, 4)
    diff_tok = (ix != hi).any(dim=1) | (sc.view(torch.int16) != hs.view(torch.int16)).any(dim=1)
    mism_tok = (lg.view(torch.int16) != hf.view(torch.int16)).any(dim=1)
    assert not (diff_tok & ~mism_tok).any()
    print(f"router routing T={T} E={E}: {int(diff_tok.sum())} of {T} tokens differ from the CPU router")
