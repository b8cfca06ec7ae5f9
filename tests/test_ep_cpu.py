"""Expert parallelism without a GPU: the oracle's EP restatement and the host logic of
ExpertParallelExperts (count exchange, split bookkeeping, all-to-alls in both directions,
return positions) on gloo ranks, world sizes 2 and 4."""
import numpy as np
import pytest
import torch

import oracle as O
from ep_harness import E, H, I, K, SEED, cpu_layer_worker, cpu_worker, dead_peer_worker, routing_case, run_ranks


def test_oracle_ep_chain_equals_single_device_forward():
    # dispatch -> (identity all-to-all, one rank) -> expert rows -> combine reproduces
    # w4a8_experts_forward bit for bit, also when the experts are split in two halves
    # whose rows are exchanged by hand.
    d = O.synth_layer(SEED, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    h, ix, wv = routing_case("random", 0, 2, 24)
    ref = O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn)
    rows, counts, pos = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 1)
    back = O.ep_expert_rows(rows, H, O.slice_experts(wn, 0, E))
    assert torch.equal(O.ep_combine(back, pos, ix.numpy()), ref)
    rows, counts, pos = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 2)
    assert counts.sum() == rows.shape[0] == 24 * K
    c0 = int(counts[0])
    b0 = O.ep_expert_rows(rows[:c0], H, O.slice_experts(wn, 0, E // 2))
    b1 = O.ep_expert_rows(rows[c0:], H, O.slice_experts(wn, E // 2, E))
    assert torch.equal(O.ep_combine(torch.cat([b0, b1]), pos, ix.numpy()), ref)


def test_oracle_ep_rows_carry_single_device_codes():
    # the dispatched codes and scales equal the single-device quantiser's for the token row
    h, ix, wv = routing_case("random", 0, 2, 8)
    rows, counts, pos = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 4)
    codes, sf = O.quantize_fp8_ue8m0(h)
    rb = O.ep_row_bytes(H)
    assert rows.shape == (8 * K, rb) and rb % 16 == 0
    for i in range(8 * K):
        t, p = i // K, pos[i]
        assert np.array_equal(rows[p, :H], codes[t]) and np.array_equal(rows[p, H:H + H // 32], sf[t])
        assert rows[p, rb - 8:rb - 4].view(np.int32)[0] == ix.numpy().reshape(-1)[i] % (E // 4)
        assert rows[p, rb - 4:].view(np.float32)[0] == wv.numpy().reshape(-1)[i]
    # destination-rank order, stable
    dest = ix.numpy().reshape(-1) // (E // 4)
    assert np.array_equal(np.argsort(pos), np.argsort(dest, kind="stable"))
    assert np.array_equal(counts, np.bincount(dest, minlength=4))


def test_gloo_two_ranks_match_single_device_oracle():
    res = run_ranks(cpu_worker, 2, ["random", "rank0", "empty"])
    for rank, (out, err) in enumerate(res):
        assert err is None, f"rank {rank}: {err}"
        by_case = {c: (shape, eq, splits) for c, shape, eq, splits in out}
        for case, (shape, eq, splits) in by_case.items():
            assert eq, f"rank {rank} case {case}: output differs from the oracle"
        # every assignment of 'rank0' goes to rank 0; rank 1 receives nothing
        s_send, s_recv = by_case["rank0"][2]
        assert s_send[1] == 0 and (rank == 0 or sum(s_recv) == 0)
        # 'empty': rank 1 has no tokens, sends nothing and still serves rank 0's rows
        shape, _, (s_send, s_recv) = by_case["empty"]
        if rank == 1:
            assert shape == (0, H) and sum(s_send) == 0
    # the splits agree across ranks: what r sends to q is what q receives from r
    for case_i in range(3):
        s0 = res[0][0][case_i][3]
        s1 = res[1][0][case_i][3]
        assert s0[0][1] == s1[1][0] and s1[0][0] == s0[1][1]


def test_gloo_four_ranks_match_single_device_oracle():
    # the same host logic with four ranks (two experts each): every rank's output equals the
    # single-device oracle in both layouts, and the split bookkeeping is consistent across
    # every pair -- what rank r sends to q is what q receives from r
    world = 4
    res = run_ranks(cpu_worker, world, ["random", "rank0", "empty"])
    for rank, (out, err) in enumerate(res):
        assert err is None, f"rank {rank}: {err}"
        for case, shape, eq, _ in out:
            assert eq, f"rank {rank} case {case}: output differs from the oracle"
    for ci, case in enumerate(("random", "rank0", "empty")):
        sends = [res[r][0][ci][3][0] for r in range(world)]
        recvs = [res[r][0][ci][3][1] for r in range(world)]
        for r in range(world):
            for q in range(world):
                assert sends[r][q] == recvs[q][r], f"{case}: rank {r} -> {q}"
        if case == "rank0":   # rank 0 owns the only two unpenalised experts: every token's top two
            assert all(sends[r][0] == 2 * 16 for r in range(world))
        if case == "empty":   # rank 1 holds no tokens and sends nothing
            assert sum(sends[1]) == 0 and res[1][0][ci][1] == (0, H)


def test_oracle_capacity_layout():
    # fixed-capacity segments: same rows as the compact layout, moved to q*cap, the rest
    # marked empty; the chain through them still equals the single-device forward.
    d = O.synth_layer(SEED, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    h, ix, wv = routing_case("random", 1, 2, 12)
    ref = O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn)
    rows_c, counts, pos_c = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 2)
    cap = 12 * K
    rows, counts2, pos = O.ep_dispatch(h, ix.numpy(), wv.numpy(), E, 2, cap)
    rb = O.ep_row_bytes(H)
    assert rows.shape == (2 * cap, rb) and np.array_equal(counts, counts2)
    c0, c1 = int(counts[0]), int(counts[1])
    assert np.array_equal(rows[:c0], rows_c[:c0]) and np.array_equal(rows[cap:cap + c1], rows_c[c0:])
    empty = np.concatenate([np.arange(c0, cap), np.arange(cap + c1, 2 * cap)])
    assert (rows[empty, rb - 8:rb - 4].view(np.int32) == -1).all()
    assert np.array_equal(rows[pos], rows_c[pos_c])
    b0 = O.ep_expert_rows(rows[:cap], H, O.slice_experts(wn, 0, E // 2))
    b1 = O.ep_expert_rows(rows[cap:], H, O.slice_experts(wn, E // 2, E))
    assert torch.equal(O.ep_combine(torch.cat([b0, b1]), pos, ix.numpy()), ref)


def test_dead_peer_ends_with_an_error_not_a_hang():
    # A rank that exits between steps: the surviving rank's next exchange raises (gloo
    # reports the closed connection or its 5 s timeout) instead of waiting forever.
    res = run_ranks(dead_peer_worker, 2, timeout=120)
    (r0, e0), (r1, e1) = res
    assert e0 is None and e1 is None and r1 == "left"
    status, kind, elapsed = r0
    assert status == "error", r0
    assert elapsed < 60, r0


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_router_and_experts_match_single_device(world):
    # ExpertParallelMoELayer end to end on gloo ranks: each rank routes its own tokens (the
    # CPU router stands in for the fused router op) and gets the single-device routing and
    # the single-device oracle output
    res = run_ranks(cpu_layer_worker, world)
    for rank, (out, err) in enumerate(res):
        assert err is None, f"rank {rank}: {err}"
        same_routing, same_out = out
        assert same_routing, f"rank {rank}: routing differs from the single-device router"
        assert same_out, f"rank {rank}: output differs from the single-device oracle"
