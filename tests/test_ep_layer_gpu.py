"""The one-launch expert-parallel step (decode_layer_kernel<true>, gptoss_ep_p2p_layer_forward)
on one GPU as a world of one rank: the kernel dispatches into its own receive rows, waits for
its own flags, runs the experts, returns the rows to itself and combines. (Several ranks of
this kernel wait on one another, so they only run as processes on several GPUs:
tests/test_ep_multi_gpu.py.) Checks: bit-exact against the five-launch peer-memory path
(route-dispatch, receive prologue, GEMM1, GEMM2 with the return stores, combine) on the same
buffers, the routing bit-exact against the router op, the output within the north-star gate
of the oracle, send counts and row positions equal to the dispatch's, and buffer reuse over
epochs."""
import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, build_experts

pytestmark = pytest.mark.gpu


def _chain(pkg, x, h, rw, rbias, ix, wv, k, E, cap, base, peer_bases, epoch, ws, dev):
    H = h.shape[1]
    if rw is not None:
        sc, ix, cnt, pos = pkg.ops.ep_p2p_route_dispatch(h, rw, rbias, k, 1, 0, cap, base, peer_bases, epoch)
    else:
        sc = None
        cnt, pos = pkg.ops.ep_p2p_dispatch(h, ix, wv, E, 1, 0, cap, base, peer_bases, epoch)
    back = torch.empty((cap, H), dtype=torch.bfloat16, device=dev)
    pkg.ops.ep_p2p_expert_forward(base, 1, 0, cap, epoch, x.gate_up_proj_data, x.gate_up_proj_scales,
                                  x.gate_up_proj_bias, x.down_proj_data, x.down_proj_scales, x.down_proj_bias, back, ws,
                                  peer_bases)
    out = pkg.ops.ep_p2p_combine(base, 1, cap, epoch, pos, ix, H, dev)
    return out, sc, ix, cnt, pos


@pytest.mark.parametrize("T,E,H,I,router", [(32, 32, 2880, 2880, True), (32, 32, 2880, 2880, False),
                                            (7, 16, 512, 256, True), (64, 32, 512, 512, True)])
def test_one_launch_matches_five_launch_path(pkg, dev, T, E, H, I, router):
    k = 4
    d = O.synth_layer(60 + T, E=E, H=H, I=I, T=T)
    x = build_experts(pkg, d, dev, E, H, I)
    cap = T * k
    assert pkg.ops.ep_p2p_layer_fits(T, k, E, 1, H, I, cap)
    base, _ = pkg.ops.ipc_alloc(pkg.ops.ep_p2p_buffer_bytes(1, cap, H))
    peer_bases = torch.tensor([base], dtype=torch.int64, device=dev)
    ws = torch.empty(pkg.ops.workspace_bytes(cap, 1, E, H, I), dtype=torch.uint8, device=dev)
    rw, rbias = d["router_w"].to(dev), d["router_b"].to(dev)
    g = torch.Generator().manual_seed(T)
    wv, ix = torch.topk(torch.randn(T, E, generator=g), k, dim=-1)
    wv = torch.softmax(wv, dim=-1).float().to(dev)
    ix = ix.to(dev)
    try:
        epoch = 0
        for rep in range(2):                               # buffers and counters reused across epochs
            h = (d["hidden"] if rep == 0 else torch.randn(T, H, generator=g).to(torch.bfloat16)).to(dev)
            epoch += 1
            one, sc1, ix1, cnt1, pos1 = pkg.ops.ep_p2p_layer_forward(
                h, rw if router else None, rbias if router else None, None if router else ix,
                None if router else wv, k, E, 1, 0, x.gate_up_proj_data, x.gate_up_proj_scales, x.gate_up_proj_bias,
                x.down_proj_data, x.down_proj_scales, x.down_proj_bias, cap, base, peer_bases, epoch, ws)
            torch.cuda.synchronize()
            assert pkg.ops.read_status(dev) == 0
            epoch += 1
            five, sc5, ix5, cnt5, pos5 = _chain(pkg, x, h, rw if router else None, rbias, ix, wv, k, E, cap, base,
                                                peer_bases, epoch, ws, dev)
            torch.cuda.synchronize()
            assert pkg.ops.read_status(dev) == 0
            assert torch.equal(ix1, ix5), "routing"
            if router:
                assert torch.equal(sc1, sc5), "scores"
                _, sc_ref, ix_ref = pkg.ops.router_topk_impl(h, rw, rbias, k)
                assert torch.equal(ix1, ix_ref) and torch.equal(sc1, sc_ref), "routing vs the router op"
            assert torch.equal(cnt1, cnt5) and torch.equal(pos1[:T * k], pos5), "send counts / row positions"
            assert torch.equal(one, five), "one launch vs five launches"
            wts = sc1.float().cpu() if router else wv.cpu()
            ref = O.w4a8_experts_forward(h.cpu(), ix1.cpu().numpy(), wts.numpy(), O.numpy_weights(d))
            assert_output_tolerance(one.cpu(), ref, f"T={T} E={E} H={H} rep {rep}")
    finally:
        torch.cuda.synchronize()
        pkg.ops.ipc_free(base)
