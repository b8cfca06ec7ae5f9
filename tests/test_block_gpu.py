"""The decoder block around the MoE layer (gptoss_moe_block_forward): out = hidden +
layer(RMSNorm(hidden)) with the norm and the residual copy in one kernel and GEMM2 adding into
the residual rows. The norm is checked against the oracle's GptOssRMSNorm restatement (fp32 on
the CPU, pinned to the transformers module; within one bf16 ulp: the sum of squares runs in a
different order and rsqrt is the hardware's); the block against the same layer on the same
normalised rows plus a separate add, and against the oracle's experts, within a few bf16 ulps
of the residual; a CUDA graph of two blocks replays each block's eager result."""
import pytest
import torch

import oracle as O
from helpers import build_layer

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _assert_block_close(out, ref, what):
    # the block adds the k expert rows into the residual one bf16 rounding at a time, the
    # reference adds their bf16 sum once: equal up to a few bf16 ulps of the residual's size
    o, r = out.float().cpu(), ref.float().cpu()
    rms = r.pow(2).mean().sqrt().item()
    rel = ((o - r).norm() / r.norm()).item()
    ulp = torch.exp2(torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - 7)
    worst = ((o - r).abs() - 4 * ulp).max().item()
    assert rel <= 1e-2, f"{what}: rel-L2 {rel:.3e}"
    assert worst <= 5e-2 * rms, f"{what}: {worst:.3e} beyond 4 bf16 ulps (rms {rms:.3e})"


def _rms_ref(x, w):
    # the oracle's GptOssRMSNorm restatement (pinned to the transformers module on the CPU)
    return O.rmsnorm_hf(x.cpu(), w.cpu(), EPS).to(x.device)


@pytest.mark.parametrize("T,H", [(1, 2880), (37, 512), (4096, 2880)])
def test_rmsnorm_residual_kernel(pkg, dev, T, H):
    g = torch.Generator().manual_seed(T)
    x = (3 * torch.randn(T, H, generator=g)).to(torch.bfloat16).to(dev)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(dev)
    xn, res = pkg.ops.rmsnorm_residual(x, w, EPS)
    torch.cuda.synchronize()
    assert torch.equal(res, x)
    ref = _rms_ref(x, w)
    ulp = (xn.view(torch.int16).int() - ref.view(torch.int16).int()).abs()
    assert ulp.max().item() <= 1, "more than one bf16 ulp from the fp32 restatement"
    assert (ulp == 0).float().mean().item() > 0.99


@pytest.mark.parametrize("T", [32, 200, 4096])
def test_block_forward(pkg, dev, T):
    # T = 32: the one-launch decode kernel adding into the residual rows; 200 and 4096: the
    # router / sort / quantiser / two-GEMM path
    E, H, I, k = 32, 2880, 2880, 4
    d = O.synth_layer(80 + T, E=E, H=H, I=I, T=T)
    layer = build_layer(pkg, d, dev, E, H, I, k)
    g = torch.Generator().manual_seed(T)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(dev)
    t = d["hidden"].to(dev)
    out, scores, idx = layer.forward_block(t, w, EPS)
    # the same layer on the same normalised rows, then the residual add as its own op (the
    # routing is then the block's bit for bit; torch's RMSNorm can differ by an ulp and flip
    # a near-tie, which is the norm test's business)
    xn, _ = pkg.ops.rmsnorm_residual(t, w, EPS)
    moe, sc2, ix2 = layer(xn)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    assert torch.equal(idx, ix2) and torch.equal(scores, sc2), "routing"
    ref = (t.float() + moe.float()).to(torch.bfloat16)
    _assert_block_close(out, ref, f"block vs norm + layer + add, T={T}")
    # and against the oracle on the block's routing
    o_ref = O.w4a8_experts_forward(xn.cpu(), idx.cpu().numpy(), scores.float().cpu().numpy(), O.numpy_weights(d))
    _assert_block_close(out, (t.cpu().float() + o_ref.float()).to(torch.bfloat16), f"oracle, T={T}")


def test_block_stack_in_a_cuda_graph(pkg, dev):
    # two blocks captured in one CUDA graph; each replayed block is checked against the eager
    # block on the same input (the graph's own input of that block), so a near-tie in layer
    # 2's routing cannot amplify layer 1's bf16 scatter-add ordering into the comparison
    E, H, I, k, T = 32, 512, 512, 4, 256
    layers = [build_layer(pkg, O.synth_layer(90 + i, E=E, H=H, I=I, T=1), dev, E, H, I, k) for i in range(2)]
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(dev)
    for lay in layers:                                   # warm-up outside the capture
        lay.forward_block(x, w, EPS)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        t1, _, i1 = layers[0].forward_block(x, w, EPS)
        t2, _, i2 = layers[1].forward_block(t1, w, EPS)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    for lay, inp, got, idx, what in ((layers[0], x, t1, i1, "block 1"), (layers[1], t1.clone(), t2, i2, "block 2")):
        ref, _, idx_ref = lay.forward_block(inp, w, EPS)
        torch.cuda.synchronize()
        assert torch.equal(idx, idx_ref), f"{what}: routing"
        _assert_block_close(got, ref, f"{what}: graph replay vs eager")
