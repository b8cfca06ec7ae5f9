"""Expert parallelism over NCCL: one process per GPU (2 or more GPUs; skipped on a
1-GPU machine). Every rank's output must meet the output gate against the oracle on its
own tokens and agree closely with the single-GPU forward; the layer's routing must equal
the single-GPU layer's bit for bit."""
import pytest
import torch

from ep_harness import nccl_worker, run_ranks

pytestmark = pytest.mark.gpu


def _world():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    return min(n, 8)


@pytest.mark.parametrize("world_cap", [2, 8])
def test_nccl_expert_parallel(world_cap):
    world = min(_world(), world_cap)
    if world_cap == 8 and world < 4:
        pytest.skip("covered by the 2-rank case")
    shapes = [(8, 512, 512, 24), (32, 2880, 2880, 40)]
    res = run_ranks(nccl_worker, world, shapes, timeout=600)
    for rank, (out, err) in enumerate(res):
        assert err is None, f"rank {rank}: {err}"
        for row in out:
            if row[0] == "experts":
                _, e_tot, hs, st, r, mx, vs_single, splits = row
                assert st == 0, (rank, e_tot, st)
                assert r <= 1e-2 and mx <= 5e-2, (rank, e_tot, r, mx)
                assert vs_single <= 2 ** -7, (rank, e_tot, vs_single)
                assert sum(splits[0]) == (24 if e_tot == 8 else 40) * 4 + 8 * rank * 4
            else:
                _, e_tot, hs, st, same_idx, same_scores, r, _ = row
                assert st == 0 and same_idx and same_scores and r <= 1e-2, (rank, row)
