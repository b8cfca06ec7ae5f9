"""Expert-parallel kernels on one GPU: dispatch rows bit-exact with the oracle, the local
expert forward within the output tolerance, the combine bit-exact, and a W-rank chain
emulated on one device (the all-to-alls done by slicing) against the oracle and the
single-GPU forward."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, build_experts

pytestmark = pytest.mark.gpu


def _inputs(seed, T, E, H, k=4):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(T, H, generator=g).to(torch.bfloat16)
    wv, ix = torch.topk(torch.randn(T, E, generator=g), k, dim=-1)
    return h, ix, torch.softmax(wv, dim=-1).float()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("H", [512, 2880])
def test_dispatch_rows_bit_exact(pkg, dev, world, H):
    E = 32
    h, ix, wv = _inputs(world + H, 37, E, H)
    rows, counts, pos = pkg.ops.ep_dispatch(h.to(dev), ix.to(dev), wv.to(dev), E, world)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    r_o, c_o, p_o = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, world)
    assert rows.shape == r_o.shape and rows.shape[1] == pkg.ops.ep_row_bytes(H) == O.ep_row_bytes(H)
    assert np.array_equal(counts.cpu().numpy(), c_o)
    assert np.array_equal(pos.cpu().numpy(), p_o)
    assert np.array_equal(rows.cpu().numpy(), r_o)


def test_dispatch_empty_and_bad_index(pkg, dev):
    H, E = 512, 8
    rows, counts, pos = pkg.ops.ep_dispatch(torch.empty(0, H, dtype=torch.bfloat16, device=dev),
                                            torch.empty(0, 4, dtype=torch.int64, device=dev),
                                            torch.empty(0, 4, device=dev), E, 2)
    assert rows.shape == (0, pkg.ops.ep_row_bytes(H)) and counts.tolist() == [0, 0]
    # an expert id outside [0, E) sets the status word; the other rows are still packed
    h, ix, wv = _inputs(3, 8, E, H)
    ix[2, 1] = E + 5
    rows, counts, pos = pkg.ops.ep_dispatch(h.to(dev), ix.to(dev), wv.to(dev), E, 2)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0x201
    assert int(counts.sum()) == 8 * 4 - 1


def test_expert_rows_and_combine(pkg, dev):
    E, H, I = 8, 512, 512
    d = O.synth_layer(21, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    m = build_experts(pkg, d, dev, E, H, I)
    h, ix, wv = _inputs(4, 48, E, H)
    rows, counts, pos = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 2)
    c0 = int(counts[0])
    for q, (lo, hi) in enumerate(((0, c0), (c0, rows.shape[0]))):
        loc = pkg.ep.shard_experts(m, q, 2)
        for mode in (1, 2, 3):
            loc.gemm_mode = mode
            back = pkg.ep.CudaKernels.expert_forward(torch.from_numpy(rows[lo:hi]).to(dev), loc)
            torch.cuda.synchronize()
            assert pkg.ops.read_status(dev) == 0
            ref = O.ep_expert_rows(rows[lo:hi], H, O.slice_experts(wn, q * E // 2, (q + 1) * E // 2))
            assert_output_tolerance(back.cpu(), ref, f"expert rows rank {q} mode {mode}")
    # combine is bit-exact for the same returned rows
    back = torch.randn(48 * 4, H).to(torch.bfloat16)
    out = pkg.ops.ep_combine(back.to(dev), torch.from_numpy(pos).to(dev), ix.to(dev))
    assert torch.equal(out.cpu(), O.ep_combine(back, pos, ix.numpy()))


@pytest.mark.parametrize("world", [2, 4])
def test_emulated_ranks_chain(pkg, dev, world):
    # dispatch on every "rank", all-to-all by slicing, local experts, all-to-all back,
    # combine: equals the oracle within tolerance and the single-GPU forward closely.
    E, H, I = 8, 512, 512
    d = O.synth_layer(5, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    m = build_experts(pkg, d, dev, E, H, I)
    ins = [_inputs(100 + r, 24 + 8 * r, E, H) for r in range(world)]
    disp = [pkg.ops.ep_dispatch(h.to(dev), ix.to(dev), wv.to(dev), E, world) for h, ix, wv in ins]
    seg = []  # seg[r][q] = rows of rank r for rank q
    for rows, counts, pos in disp:
        c = counts.cpu().tolist()
        o = np.concatenate([[0], np.cumsum(c)]).tolist()
        seg.append([rows[o[q]:o[q + 1]] for q in range(world)])
    backs = []
    for q in range(world):
        recv = torch.cat([seg[r][q] for r in range(world)])
        back = pkg.ep.CudaKernels.expert_forward(recv, pkg.ep.shard_experts(m, q, world))
        sizes = [seg[r][q].shape[0] for r in range(world)]
        backs.append(list(torch.split(back, sizes)))
    for r, (h, ix, wv) in enumerate(ins):
        ret = torch.cat([backs[q][r] for q in range(world)])
        out = pkg.ops.ep_combine(ret, disp[r][2], ix.to(dev))
        torch.cuda.synchronize()
        assert pkg.ops.read_status(dev) == 0
        ref = O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn)
        assert_output_tolerance(out.cpu(), ref, f"rank {r}")
        single = m(h.to(dev), ix.to(dev), wv.to(dev))
        diff = (out.float() - single.float()).abs().max().item()
        assert diff <= 2 ** -7 * single.float().abs().max().item(), diff


@pytest.mark.parametrize("world", [2, 8])
def test_dispatch_capacity_layout_bit_exact(pkg, dev, world):
    E, H, T = 32, 2880, 19
    h, ix, wv = _inputs(77 + world, T, E, H)
    cap = T * 4 + 3
    rows, counts, pos = pkg.ops.ep_dispatch(h.to(dev), ix.to(dev), wv.to(dev), E, world, cap)
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    r_o, c_o, p_o = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, world, cap)
    rows = rows.cpu().numpy()
    rb = O.ep_row_bytes(H)
    assert rows.shape == r_o.shape == (world * cap, rb)
    assert np.array_equal(counts.cpu().numpy(), c_o) and np.array_equal(pos.cpu().numpy(), p_o)
    used = np.zeros(world * cap, dtype=bool)
    used[p_o] = True
    assert np.array_equal(rows[used], r_o[used])                       # every byte of a used row
    assert np.array_equal(rows[~used, rb - 8:], r_o[~used, rb - 8:])   # empty marker + zero weight


def test_emulated_ranks_chain_capacity(pkg, dev):
    E, H, I, world = 8, 512, 512, 4
    d = O.synth_layer(6, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    m = build_experts(pkg, d, dev, E, H, I)
    cap_tokens = 20
    cap = cap_tokens * 4
    ins = [_inputs(200 + r, 12 + 2 * r, E, H) for r in range(world)]
    disp = [pkg.ops.ep_dispatch(h.to(dev), ix.to(dev), wv.to(dev), E, world, cap) for h, ix, wv in ins]
    # equal splits: rank q receives segment q of every rank, in rank order
    backs = []
    for q in range(world):
        recv = torch.cat([disp[r][0][q * cap:(q + 1) * cap] for r in range(world)])
        backs.append(pkg.ep.CudaKernels.expert_forward(recv, pkg.ep.shard_experts(m, q, world)))
    for r, (h, ix, wv) in enumerate(ins):
        ret = torch.cat([backs[q][r * cap:(r + 1) * cap] for q in range(world)])
        out = pkg.ops.ep_combine(ret, disp[r][2], ix.to(dev))
        torch.cuda.synchronize()
        assert pkg.ops.read_status(dev) == 0
        assert_output_tolerance(out.cpu(), O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn), f"rank {r}")


def test_p2p_wait_gives_up_with_status(pkg, dev):
    # A flag nothing raises: the combine's bounded wait runs out after ~1 s, records
    # 0x301 in the status word and the kernel returns; the device stays usable.
    import time
    world, cap, H = 1, 8, 512
    base, _ = pkg.ops.ipc_alloc(pkg.ops.ep_p2p_buffer_bytes(world, cap, H))
    try:
        idx = torch.zeros(2, 4, dtype=torch.int64, device=dev)
        pos = torch.zeros(8, dtype=torch.int32, device=dev)
        t0 = time.time()
        out = pkg.ops.ep_p2p_combine(base, world, cap, 7, pos, idx, H, dev)
        torch.cuda.synchronize()
        assert time.time() - t0 >= 0.9
        assert pkg.ops.read_status(dev) == 0x301
        assert out.shape == (2, H)
        x = torch.ones(4, device=dev)
        assert float((x * 2).sum()) == 8.0          # the context is healthy
    finally:
        pkg.ops.ipc_free(base)


def _device_bytes(addr: int, n: int) -> np.ndarray:
    """n bytes of device memory at a raw address (the exchange buffers are not tensors)."""
    from cuda.bindings import runtime as rt
    out = np.empty(n, dtype=np.uint8)
    err, = rt.cudaMemcpy(out.ctypes.data, addr, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess, err
    return out


@pytest.mark.parametrize("world,T,router", [(1, 24, False), (2, 24, True), (4, 24, False), (4, 24, True),
                                            (4, 8, True), (2, 80, False), (2, 80, True)])
def test_p2p_emulated_ranks(pkg, dev, world, T, router):
    # The peer-memory protocol with every rank's exchange buffer on this one GPU: all
    # dispatches, then every owner's expert forward, then every combine, in stream order
    # (each wait finds its flags already raised). T = 24 runs the one-launch dispatch
    # (router and quantiser fused into a cluster kernel), T = 80 the separate kernels; the
    # owners' GEMM2 stores its rows straight into the sources' return rows (16-row chunks
    # at T = 8, 64-row chunks otherwise).
    E, H, I, k = 8 * world if world > 1 else 8, 512, 512, 4
    d = O.synth_layer(40 + world, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    full = build_experts(pkg, d, dev, E, H, I)
    locs = [pkg.ep.shard_experts(full, q, world) for q in range(world)]
    cap = (T + 4 * world) * k
    rb = pkg.ops.ep_row_bytes(H)
    bases = [pkg.ops.ipc_alloc(pkg.ops.ep_p2p_buffer_bytes(world, cap, H))[0] for _ in range(world)]
    peer_bases = torch.tensor(bases, dtype=torch.int64, device=dev)
    rw, rbias = d["router_w"].to(dev), d["router_b"].to(dev)
    try:
        for epoch in (1, 2):                             # the second call reuses the buffers
            ins, disp = [], []
            for r in range(world):
                h, ix, wv = _inputs(100 * epoch + r, T + 4 * r, E, H, k)
                hd = h.to(dev)
                if router:
                    sc, ixd, cnt, pos = pkg.ops.ep_p2p_route_dispatch(hd, rw, rbias, k, world, r, cap, bases[r],
                                                                      peer_bases, epoch)
                    _, sc_ref, ix_ref = pkg.ops.router_topk_impl(hd, rw, rbias, k)
                    assert torch.equal(ixd, ix_ref) and torch.equal(sc, sc_ref), f"routing, rank {r}"
                    ix, wv = ixd.cpu(), sc.float().cpu()
                else:
                    ixd = ix.to(dev)
                    cnt, pos = pkg.ops.ep_p2p_dispatch(hd, ixd, wv.to(dev), E, world, r, cap, bases[r], peer_bases,
                                                       epoch)
                ins.append((h, ix, wv, ixd, pos, cnt))
            backs = []
            for q in range(world):
                x = locs[q]
                back = torch.empty((world * cap, H), dtype=torch.bfloat16, device=dev)
                ws = torch.empty(pkg.ops.workspace_bytes(world * cap, 1, E // world, H, I), dtype=torch.uint8,
                                 device=dev)
                pkg.ops.ep_p2p_expert_forward(bases[q], world, q, cap, epoch, x.gate_up_proj_data,
                                              x.gate_up_proj_scales, x.gate_up_proj_bias, x.down_proj_data,
                                              x.down_proj_scales, x.down_proj_bias, back, ws, peer_bases)
                backs.append((back, ws))
            for r, (h, ix, wv, ixd, pos, cnt) in enumerate(ins):
                out = pkg.ops.ep_p2p_combine(bases[r], world, cap, epoch, pos, ixd, H, dev)
                torch.cuda.synchronize()
                assert pkg.ops.read_status(dev) == 0
                # the dispatch rows equal the packed send rows of the fixed-capacity layout
                rows, counts, pos_ref = pkg.ops.ep_dispatch(h.to(dev), ixd, wv.to(dev), E, world, cap)
                assert torch.equal(cnt, counts) and torch.equal(pos, pos_ref), f"layout, rank {r}"
                rows = rows.cpu().numpy()
                for q in range(world):
                    seg = _device_bytes(bases[q] + 4 * 64 * 4 + r * cap * rb, cap * rb).reshape(cap, rb)
                    c = int(counts[q])
                    assert np.array_equal(seg[:c], rows[q * cap:q * cap + c]), f"rows {r}->{q}"
                    assert np.array_equal(seg[c:, rb - 8:], rows[q * cap + c:(q + 1) * cap, rb - 8:]), "markers"
                assert_output_tolerance(out.cpu(), O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn),
                                        f"world {world} rank {r} epoch {epoch}")
    finally:
        torch.cuda.synchronize()
        for b in bases:
            pkg.ops.ipc_free(b)
