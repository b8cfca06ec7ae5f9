"""The one-launch decode layer (decode_layer_kernel): router, sort, quantisation and both
GEMMs in one persistent kernel, against the oracle and against the three-launch path.

Routing: the kernel's router logits are the exactly rounded F.linear value (exact bf16
products summed in float64, one rounding), so its top-k indices and bf16 scores must equal
the oracle's top-k + softmax applied to oracle.router_logits_exact bit for bit. Outputs:
the north-star tolerance against the oracle's W4A8 forward on the kernel's routing."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, build_experts, build_layer

pytestmark = pytest.mark.gpu

# (T, E, H, I, top_k, seed, skew): GPT-OSS-20B and 120B decode shapes, single tokens,
# K padding (288 -> 384), experts past 16 rows (several 16-row chunks per expert)
SHAPES = [
    (32, 32, 2880, 2880, 4, 0, None),
    (1, 32, 2880, 2880, 4, 1, None),
    (7, 128, 2880, 2880, 4, 2, None),
    (5, 8, 512, 512, 2, 3, None),
    (16, 4, 288, 288, 2, 4, None),
    (64, 32, 512, 256, 4, 5, "zipf"),
    (48, 64, 512, 512, 1, 6, None),
]


def _sorted_pairs(idx: torch.Tensor, scores: torch.Tensor):
    """Per-token (expert, score) rows sorted by expert id (torch.topk leaves the order of
    equal logits unspecified; the routed result does not depend on it)."""
    o = torch.argsort(idx, dim=1)
    return torch.gather(idx, 1, o), torch.gather(scores, 1, o)


@pytest.fixture
def one_launch(pkg):
    prev = pkg.ops.set_decode_layer_kernel(True)
    yield
    pkg.ops.set_decode_layer_kernel(prev)


def _run_layer(pkg, dev, layer, x, one_launch: bool):
    prev = pkg.ops.set_decode_layer_kernel(one_launch)
    try:
        launches0 = pkg._lib.query("gptoss_kernel_launch_count")
        out, scores, idx = layer(x)
        torch.cuda.synchronize()
        n = int(pkg._lib.query("gptoss_kernel_launch_count") - launches0)
    finally:
        pkg.ops.set_decode_layer_kernel(prev)
    assert pkg.ops.read_status(dev) == 0
    return out, scores, idx, n


@pytest.mark.parametrize("T,E,H,I,k,seed,skew", SHAPES)
def test_decode_kernel_layer_matches_oracle(pkg, dev, T, E, H, I, k, seed, skew):
    d = O.synth_layer(seed, E=E, H=H, I=I, T=T, skew=skew)
    layer = build_layer(pkg, d, dev, E, H, I, k)
    x = d["hidden"].to(dev)
    out, scores, idx, n = _run_layer(pkg, dev, layer, x, True)
    layout = pkg._lib.query("gptoss_moe_gemm_layout", 0, T * k, E)
    if layout == pkg.ops.GEMM_SWAP:
        assert n == 2, f"{n} launches: the decode kernel (+ its reset) should have run"
    # routing: bit-exact against top-k + softmax of the exactly rounded logits
    ref_logits = O.router_logits_exact(d["hidden"], d["router_w"], d["router_b"])
    ref_scores, ref_idx = O.router_topk_from_logits(ref_logits, k)
    i1, s1 = _sorted_pairs(idx.cpu(), scores.cpu())
    i2, s2 = _sorted_pairs(ref_idx, ref_scores)
    assert torch.equal(i1, i2), "top-k experts differ from the exactly rounded router"
    assert torch.equal(s1, s2), "softmax scores differ from the exactly rounded router"
    # outputs: the oracle's W4A8 forward on the same routing
    ref = O.w4a8_experts_forward(d["hidden"], idx.cpu().numpy(), scores.cpu().float().numpy(), O.numpy_weights(d))
    assert_output_tolerance(out.cpu(), ref, f"decode kernel T={T} E={E} H={H} I={I} k={k}")


@pytest.mark.parametrize("T,E,H,I,k,seed,skew", SHAPES[:5])
def test_decode_kernel_agrees_with_three_launch_path(pkg, dev, T, E, H, I, k, seed, skew):
    d = O.synth_layer(seed, E=E, H=H, I=I, T=T, skew=skew)
    layer = build_experts(pkg, d, dev, E, H, I)
    x = d["hidden"].to(dev)
    logits = O.router_logits_exact(d["hidden"], d["router_w"], d["router_b"])
    sc, ix = O.router_topk_from_logits(logits, k)
    ixd, wd = ix.to(dev), sc.float().to(dev)
    prev = pkg.ops.set_decode_layer_kernel(True)
    try:
        a = layer(x, ixd, wd)
        torch.cuda.synchronize()
        pkg.ops.set_decode_layer_kernel(False)
        b = layer(x, ixd, wd)
        torch.cuda.synchronize()
    finally:
        pkg.ops.set_decode_layer_kernel(prev)
    assert pkg.ops.read_status(dev) == 0
    # same FP8 codes, same GEMMs; only the order of the combine's bf16 atomics differs
    diff = (a.float() - b.float()).abs().max().item()
    assert diff <= 2 ** -7 * max(b.float().abs().max().item(), 1e-6), f"max |diff| {diff}"
    ref = O.w4a8_experts_forward(d["hidden"], ix.numpy(), sc.float().numpy(), O.numpy_weights(d))
    assert_output_tolerance(a.cpu(), ref, "decode kernel, routing given")


def test_decode_kernel_repeated_calls_reuse_workspace(pkg, dev, one_launch):
    # back-to-back launches on one stream share the workspace and its synchronisation
    # words; every call must see its own routing, not the previous call's
    E, H, I, k = 32, 1024, 1024, 4
    ds = [O.synth_layer(s, E=E, H=H, I=I, T=T) for s, T in ((20, 32), (21, 9), (22, 32))]
    layer = build_layer(pkg, ds[0], dev, E, H, I, k)
    xs = [d["hidden"].to(dev) for d in ds]
    outs = [layer(x) for x in xs * 2]
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    for j, (out, scores, idx) in enumerate(outs):
        x_cpu = ds[j % 3]["hidden"]
        ref = O.w4a8_experts_forward(x_cpu, idx.cpu().numpy(), scores.cpu().float().numpy(),
                                     O.numpy_weights(ds[0]))
        assert_output_tolerance(out.cpu(), ref, f"call {j}")
    for j in range(3):
        assert torch.equal(outs[j][2], outs[j + 3][2])
