"""Guard bytes around the caller's buffers, in place of a device memory checker: the experts
forward and the router-included layer forward, on every GEMM layout and on both decode paths
(one persistent launch, three launches), write nothing outside `out`, the router outputs and
the workspace they are given, and leave their inputs as they were. Each buffer sits between
two 4 KB guards filled with a canary byte; the workspace itself starts full of the canary
too (the kernels may not depend on its contents). The outputs are then held to the output
gate against the module's own forward on the same layout. (The grouped GEMM op's rows beyond
its problem are covered by tests/test_gemm_gpu.py::test_rows_owned_by_no_expert_untouched.)"""
import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, build_layer

pytestmark = pytest.mark.gpu

GUARD = 4096
CANARY = 0xA5


class Guarded:
    """`nbytes` of device memory between two canary-filled guards."""

    def __init__(self, nbytes: int, dev):
        self.nbytes = nbytes
        self.buf = torch.full((GUARD + nbytes + GUARD,), CANARY, dtype=torch.uint8, device=dev)
        self.inner = self.buf[GUARD:GUARD + nbytes]

    def view(self, dtype, shape):
        return self.inner.view(dtype).view(shape)

    def check(self, what: str):
        head, tail = self.buf[:GUARD].cpu(), self.buf[GUARD + self.nbytes:].cpu()
        bad_h = (head != CANARY).nonzero().flatten()
        bad_t = (tail != CANARY).nonzero().flatten()
        assert bad_h.numel() == 0, \
            f"{what}: {bad_h.numel()} bytes written before the buffer (first at -{GUARD - int(bad_h[0])})"
        assert bad_t.numel() == 0, \
            f"{what}: {bad_t.numel()} bytes written past the buffer (first at +{int(bad_t[0])})"


# (T, E, H, I, gemm_mode, one-launch decode kernel): AUTO at decode size takes the one-launch
# kernel (or, switched off, the prologue + two GEMMs); 1 = tokens-on-M CTA pairs, 2 = SWAP with
# 16-row chunks, 3 = SWAP with 64-row chunks
# (H = I = 512 gives GEMM1 a partial last 192-row weight tile)
CASES = [(32, 32, 2880, 2880, 0, True), (32, 32, 2880, 2880, 0, False), (7, 16, 512, 256, 0, True),
         (48, 32, 512, 512, 2, True), (200, 32, 512, 512, 3, True), (600, 32, 512, 512, 1, True),
         (1000, 32, 512, 512, 0, True)]


@pytest.mark.parametrize("T,E,H,I,mode,one_launch", CASES)
def test_forwards_write_only_their_buffers(pkg, dev, T, E, H, I, mode, one_launch):
    k = 4
    d = O.synth_layer(120 + T, E=E, H=H, I=I, T=T)
    layer = build_layer(pkg, d, dev, E, H, I, k)
    ex = layer.experts
    hidden = d["hidden"].to(dev)
    hidden_copy = hidden.clone()
    g = torch.Generator().manual_seed(T)
    wv, ix = torch.topk(torch.randn(T, E, generator=g), k, dim=-1)
    wv, ix = torch.softmax(wv, -1).float().to(dev), ix.to(dev)
    ix_copy, wv_copy = ix.clone(), wv.clone()
    ws_bytes = pkg.ops.workspace_bytes(T, k, E, H, I)
    st = torch.cuda.current_stream(dev).cuda_stream
    status = pkg.ops.status_tensor(dev).data_ptr()
    wargs = (ex.gate_up_proj_data.data_ptr(), ex.gate_up_proj_scales.data_ptr(), ex.gate_up_proj_scales.numel() // E,
             ex.gate_up_proj_bias.data.data_ptr(), ex.down_proj_data.data_ptr(), ex.down_proj_scales.data_ptr(),
             ex.down_proj_scales.numel() // E, ex.down_proj_bias.data.data_ptr(), float(ex.alpha), float(ex.limit))
    prev_kernel = pkg.ops.set_decode_layer_kernel(one_launch)
    prev_mode = ex.gemm_mode
    try:
        # experts forward on given routing
        out = Guarded(T * H * 2, dev)
        ws = Guarded(ws_bytes, dev)
        pkg._lib.call("gptoss_moe_experts_forward", hidden.data_ptr(), ix.data_ptr(), wv.data_ptr(), T, k, E, H, I,
                      *wargs, out.inner.data_ptr(), ws.inner.data_ptr(), ws_bytes, mode, status, st)
        # router-included layer forward
        lout, lidx, lsc = Guarded(T * H * 2, dev), Guarded(T * k * 8, dev), Guarded(T * k * 2, dev)
        lws = Guarded(ws_bytes, dev)
        pkg._lib.call("gptoss_moe_layer_forward", hidden.data_ptr(), layer.router_weight.data_ptr(),
                      layer.router_bias.data_ptr(), T, k, E, H, I, *wargs, lout.inner.data_ptr(),
                      lidx.inner.data_ptr(), lsc.inner.data_ptr(), lws.inner.data_ptr(), ws_bytes, mode, status, st)
        torch.cuda.synchronize()
        assert pkg.ops.read_status(dev) == 0
        what = f"T={T} E={E} H={H} I={I} mode={mode} one_launch={one_launch}"
        for buf, name in ((out, "experts out"), (ws, "experts workspace"), (lout, "layer out"),
                          (lidx, "layer indices"), (lsc, "layer scores"), (lws, "layer workspace")):
            buf.check(f"{what}: {name}")
        assert torch.equal(hidden, hidden_copy) and torch.equal(ix, ix_copy) and torch.equal(wv, wv_copy), \
            f"{what}: an input changed"
        # the outputs in the guarded buffers are the forward's outputs
        ex.gemm_mode = mode
        ref = ex(hidden, ix, wv)
        lref, lsc_ref, lidx_ref = layer(hidden)
        torch.cuda.synchronize()
        assert_output_tolerance(out.view(torch.bfloat16, (T, H)).cpu(), ref.cpu(), f"{what}: experts")
        assert torch.equal(lidx.view(torch.int64, (T, k)), lidx_ref), f"{what}: routing"
        assert torch.equal(lsc.view(torch.bfloat16, (T, k)), lsc_ref), f"{what}: scores"
        assert_output_tolerance(lout.view(torch.bfloat16, (T, H)).cpu(), lref.cpu(), f"{what}: layer")
    finally:
        ex.gemm_mode = prev_mode
        pkg.ops.set_decode_layer_kernel(prev_kernel)
