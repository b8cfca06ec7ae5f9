"""Router + experts (GptOssMoELayer) at the benchmark workloads.

Decode (T=32) is compared with the reference's own output (golden); prefill (T=8192,
skewed loads) and the 120B-shaped layer (E=128, Zipf, T=16384) are too large for the CPU
oracle as a whole, so a fixed sample of tokens is recomputed on the CPU (each token's
output depends only on its own hidden state and routing)."""
import numpy as np
import pytest
import torch

import oracle as O
from golden import make_golden as MG
from helpers import assert_output_tolerance, bf16_from_int16, build_layer, golden

pytestmark = pytest.mark.gpu


def test_decode_layer_matches_reference_golden(pkg, dev):
    g = golden("layer_decode.npz")
    seed, E, H, I, T, k = MG.LAYERS["decode"]
    d = O.synth_layer(seed, E=E, H=H, I=I, T=T)
    layer = build_layer(pkg, d, dev, E, H, I, k)
    out, scores, idx = layer(d["hidden"].to(dev))
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    # same (expert, score) set per token; equal logits may be listed in another order
    # (torch.topk leaves tie order unspecified)
    ix, sc = idx.cpu(), scores.float().cpu()
    rix, rsc = torch.from_numpy(g["router_indices"]), torch.from_numpy(g["routing_weights"])
    o1, o2 = torch.argsort(ix, dim=1), torch.argsort(rix, dim=1)
    assert torch.equal(torch.gather(ix, 1, o1), torch.gather(rix, 1, o2)), "router top-4 differs"
    assert torch.equal(torch.gather(sc, 1, o1), torch.gather(rsc, 1, o2)), "router softmax differs"
    assert_output_tolerance(out.cpu(), bf16_from_int16(g["out"]), "decode layer")


@pytest.mark.parametrize("T,E,skew,seed", [(8192, 32, "prefill", 0), (16384, 128, "zipf", 0), (1024, 32, None, 4)])
def test_large_layer_sampled_tokens(pkg, dev, T, E, skew, seed):
    H = I = 2880
    d = O.synth_layer(seed, E=E, H=H, I=I, T=T, skew=skew)
    layer = build_layer(pkg, d, dev, E, H, I, 4)
    out, scores, idx = layer(d["hidden"].to(dev))
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    counts = np.bincount(idx.cpu().numpy().reshape(-1), minlength=E)
    if skew == "prefill":
        assert counts.min() > 1024 * 0.4 and counts.max() < 1024 * 1.7
    if skew == "zipf":
        assert (counts == 0).any() and counts.max() > 10 * counts.mean()
    sample = torch.randperm(T, generator=torch.Generator().manual_seed(T))[:48]
    ref = O.w4a8_experts_forward(d["hidden"][sample], idx.cpu()[sample].numpy(),
                                 scores.cpu()[sample].float().numpy(), O.numpy_weights(d))
    assert_output_tolerance(out.cpu()[sample], ref, f"T={T} E={E}")


def test_layer_router_outputs_feed_experts(pkg, dev):
    # layer(x) == experts(x, router(x)) for the same inputs
    d = O.synth_layer(3, E=8, H=512, I=512, T=64)
    layer = build_layer(pkg, d, dev, 8, 512, 512, 4)
    x = d["hidden"].to(dev)
    out, scores, idx = layer(x)
    lg, sc, ix = layer.route(x)
    assert torch.equal(ix, idx) and torch.equal(sc, scores)
    out2 = layer.experts(x, ix, sc.float())
    assert (out.float() - out2.float()).abs().max().item() <= 2 ** -7 * out.float().abs().max().item()
