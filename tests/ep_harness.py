"""Expert-parallel test harness (not part of the product): the oracle's restatement of
the three local EP steps behind the kernel interface of ExpertParallelExperts, the
routing cases, and a per-rank worker used by the gloo (CPU) and NCCL (GPU) tests."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import torch
import torch.distributed as dist

import oracle as O
from helpers import Cfg

E, H, I, K = 8, 256, 256, 4
SEED = 11


class OracleKernels:
    """dispatch / expert_forward / combine on the CPU with the oracle."""

    def __init__(self, w_local: dict, hidden_size: int):
        self.w_local = w_local
        self.H = hidden_size

    def dispatch(self, hidden, router_indices, routing_weights, num_experts, world_size, capacity=0):
        rows, counts, pos = O.ep_dispatch(hidden, router_indices.numpy(), routing_weights.numpy(), num_experts,
                                          world_size, capacity)
        return torch.from_numpy(rows), torch.from_numpy(counts), torch.from_numpy(pos)

    def expert_forward(self, recv_rows, experts):
        return O.ep_expert_rows(recv_rows.numpy(), self.H, self.w_local)

    def combine(self, back_rows, pos_of, router_indices):
        return O.ep_combine(back_rows, pos_of.numpy(), router_indices.numpy())


def routing_case(case: str, rank: int, world: int, T: int, num_experts: int = E, k: int = K):
    """(hidden bf16 [T, H], router_indices i64 [T, k], routing_weights f32 [T, k]) of a
    rank: 'random' top-k of random logits, 'rank0' every assignment on rank 0's experts,
    'empty' rank 1 holds no tokens."""
    g = torch.Generator().manual_seed(1000 + 17 * rank + 101 * ("random", "rank0", "empty").index(case))
    if case == "empty" and rank == 1:
        T = 0
    h = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, num_experts, generator=g)
    if case == "rank0":
        logits[:, num_experts // world:] -= 100.0
    wv, ix = torch.topk(logits, k, dim=-1)
    return h, ix, torch.softmax(wv, dim=-1).float()


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_worker(rank: int, world: int, port: int, cases, q):
    """One gloo rank: ExpertParallelExperts with OracleKernels vs the single-process oracle."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import __graft_entry__ as ge

        pkg = ge.load_package()
        from gpt_oss_mxfp4_compile_b200 import ep as EP

        d = O.synth_layer(SEED, E=E, H=H, I=I, T=1)
        wn = O.numpy_weights(d)
        e_loc = E // world
        local = pkg.CutlassGptOssExperts(Cfg(e_loc, H, I))
        kern = OracleKernels(O.slice_experts(wn, rank * e_loc, (rank + 1) * e_loc), H)
        mod = EP.ExpertParallelExperts(local, E, kernels=kern)
        fixed = EP.ExpertParallelExperts(local, E, kernels=kern, capacity_tokens=16)
        results = []
        for case in cases:
            h, ix, wv = routing_case(case, rank, world, 16)
            out = mod(h, ix, wv)
            out_fixed = fixed(h, ix, wv)
            ref = O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn)
            results.append((case, tuple(out.shape), bool(torch.equal(out, ref) and torch.equal(out_fixed, ref)),
                            mod.last_splits))
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def cpu_layer_worker(rank: int, world: int, port: int, q):
    """One gloo rank: router + expert-parallel experts (ExpertParallelMoELayer with the CPU
    router and OracleKernels) on this rank's own tokens vs the single-process oracle."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import __graft_entry__ as ge

        pkg = ge.load_package()
        from gpt_oss_mxfp4_compile_b200 import ep as EP

        d = O.synth_layer(SEED, E=E, H=H, I=I, T=1)
        wn = O.numpy_weights(d)
        e_loc = E // world
        local = pkg.CutlassGptOssExperts(Cfg(e_loc, H, I))
        kern = OracleKernels(O.slice_experts(wn, rank * e_loc, (rank + 1) * e_loc), H)
        experts = EP.ExpertParallelExperts(local, E, kernels=kern)
        layer = EP.ExpertParallelMoELayer(d["router_w"], d["router_b"], K, experts, router=O.router_topk_hf)
        g = torch.Generator().manual_seed(500 + rank)
        h = torch.randn(24 + 8 * rank, H, generator=g).to(torch.bfloat16)
        out, scores, idx = layer(h)
        _, rsc, rix = O.router_topk_hf(h, d["router_w"], d["router_b"], K)
        ref = O.w4a8_experts_forward(h, rix.numpy(), rsc.float().numpy(), wn)
        q.put((rank, (bool(torch.equal(idx, rix) and torch.equal(scores, rsc)), bool(torch.equal(out, ref))), None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def run_ranks(target, world: int, *args, timeout: float = 240.0):
    """Runs `target(rank, world, port, *args, q)` in `world` spawned processes; returns
    the per-rank results in rank order."""
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=timeout)
            got[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [got[r] for r in range(world)]


_ = np


def nccl_worker(rank: int, world: int, port: int, shapes, q):
    """One NCCL rank on cuda:rank: ExpertParallelExperts (CUDA kernels, NCCL all-to-alls)
    vs the oracle on this rank's tokens and vs the single-GPU forward; then the layer
    (router + EP experts) vs the single-GPU GptOssMoELayer."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import __graft_entry__ as ge
        from helpers import build_experts, build_layer, max_abs_over_rms, rel_l2

        pkg = ge.load_package()
        pkg.ensure_custom_op_registered()
        EP = pkg.ep
        results = []
        for (e_tot, hs, isz, T) in shapes:
            d = O.synth_layer(SEED, E=e_tot, H=hs, I=isz, T=1)
            wn = O.numpy_weights(d)
            full = build_experts(pkg, d, dev, e_tot, hs, isz)
            local = EP.shard_experts(full, rank, world)
            mod = EP.ExpertParallelExperts(local, e_tot)
            fixed = EP.ExpertParallelExperts(local, e_tot, capacity_tokens=T + 8 * world)
            g = torch.Generator().manual_seed(500 + rank)
            h = torch.randn(T + 8 * rank, hs, generator=g).to(torch.bfloat16)
            wv, ix = torch.topk(torch.randn(h.shape[0], e_tot, generator=g), K, dim=-1)
            wv = torch.softmax(wv, -1).float()
            p2p = EP.ExpertParallelExperts(local, e_tot, capacity_tokens=T + 8 * world, transport="p2p", top_k=K)
            out = mod(h.to(dev), ix.to(dev), wv.to(dev))
            out_fixed = fixed(h.to(dev), ix.to(dev), wv.to(dev))
            out_p2p = [p2p(h.to(dev), ix.to(dev), wv.to(dev)) for _ in range(3)]   # buffer reuse over epochs
            torch.cuda.synchronize()
            st = pkg.ops.read_status(dev)
            p2p.close()
            ref = O.w4a8_experts_forward(h, ix.numpy(), wv.numpy(), wn)
            single = full(h.to(dev), ix.to(dev), wv.to(dev))
            for o in (out, out_fixed, *out_p2p):
                results.append(("experts", e_tot, hs, st, rel_l2(o.cpu(), ref), max_abs_over_rms(o.cpu(), ref),
                                (o.float() - single.float()).abs().max().item() / single.float().abs().max().item(),
                                mod.last_splits))
            # the layer: router on local tokens + EP experts vs the single-GPU layer
            single_layer = build_layer(pkg, d, dev, e_tot, hs, isz, K)
            ep_layer = EP.ExpertParallelMoELayer(d["router_w"].to(dev), d["router_b"].to(dev), K, mod)
            o1, s1, i1 = ep_layer(h.to(dev))
            o2, s2, i2 = single_layer(h.to(dev))
            torch.cuda.synchronize()
            results.append(("layer", e_tot, hs, pkg.ops.read_status(dev), bool(torch.equal(i1, i2)),
                            bool(torch.equal(s1, s2)), rel_l2(o1.cpu(), o2.cpu()), None))
            # the same layer over peer memory: router and dispatch in one call
            p2p_l = EP.ExpertParallelExperts(local, e_tot, capacity_tokens=T + 8 * world, transport="p2p", top_k=K)
            ep_layer_p2p = EP.ExpertParallelMoELayer(d["router_w"].to(dev), d["router_b"].to(dev), K, p2p_l)
            for _ in range(2):
                o3, s3, i3 = ep_layer_p2p(h.to(dev))
            torch.cuda.synchronize()
            st3 = pkg.ops.read_status(dev)
            p2p_l.close()
            results.append(("layer", e_tot, hs, st3, bool(torch.equal(i3, i2)), bool(torch.equal(s3, s2)),
                            rel_l2(o3.cpu(), o2.cpu()), None))
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback

        q.put((rank, None, repr(e) + traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def p2p_layer_worker(rank: int, world: int, port: int, steps: int, q):
    """One rank on cuda:rank running decode-sized expert-parallel layer steps over peer
    memory (T = 32 tokens per rank, E = 32, H = I = 2880, capacity T x k): each step once in
    one launch (decode_layer_kernel<true>) and once in five launches, on the same inputs,
    and the single-GPU layer on the same tokens. Every rank toggles the path in the same
    step (all ranks must take the same one)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import __graft_entry__ as ge
        from helpers import build_experts, build_layer, rel_l2

        pkg = ge.load_package()
        pkg.ensure_custom_op_registered()
        EP = pkg.ep
        e_tot, hs, isz, T, k = 32, 2880, 2880, 32, 4
        d = O.synth_layer(SEED, E=e_tot, H=hs, I=isz, T=1)
        wn = O.numpy_weights(d)
        full = build_experts(pkg, d, dev, e_tot, hs, isz)
        local = EP.shard_experts(full, rank, world)
        epx = EP.ExpertParallelExperts(local, e_tot, capacity_tokens=T, transport="p2p", top_k=k)
        layer = EP.ExpertParallelMoELayer(d["router_w"].to(dev), d["router_b"].to(dev), k, epx)
        single = build_layer(pkg, d, dev, e_tot, hs, isz, k)
        fits = pkg.ops.ep_p2p_layer_fits(T, k, e_tot, world, hs, isz, T * k)
        results = []
        g = torch.Generator().manual_seed(700 + rank)
        for step in range(steps):
            # the last step: rank 1 holds no tokens (it still takes part in the exchange)
            Tr = 0 if (step == steps - 1 and rank == 1) else T
            h = torch.randn(Tr, hs, generator=g).to(torch.bfloat16).to(dev)
            o1, s1, i1 = layer(h)                     # one launch
            prev = pkg.ops.set_ep_layer_kernel(False)
            o5, s5, i5 = layer(h)                     # five launches
            pkg.ops.set_ep_layer_kernel(prev)
            o_s, s_s, i_s = single(h)
            torch.cuda.synchronize()
            st = pkg.ops.read_status(dev)
            if Tr == 0:
                results.append((fits, st, o1.numel() == 0 and o5.numel() == 0, True, True, 0.0, 0.0))
                continue
            ref = O.w4a8_experts_forward(h.cpu(), i1.cpu().numpy(), s1.float().cpu().numpy(), wn)
            results.append((fits, st, bool(torch.equal(o1, o5)), bool(torch.equal(i1, i5) and torch.equal(s1, s5)),
                            bool(torch.equal(i1, i_s) and torch.equal(s1, s_s)), rel_l2(o1.cpu(), o_s.cpu()),
                            rel_l2(o1.cpu(), ref)))
        epx.close()
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback

        q.put((rank, None, repr(e) + traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def dead_peer_worker(rank: int, world: int, port: int, q):
    """Failure detection on the host: both ranks run one expert-parallel step, then rank 1
    leaves without joining the next one (it exits between steps, nothing in flight). Rank 0's
    next step must end with an error from the process group (peer gone, or the short
    timeout), not hang."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    import __graft_entry__ as ge

    pkg = ge.load_package()
    from gpt_oss_mxfp4_compile_b200 import ep as EP

    d = O.synth_layer(SEED, E=E, H=H, I=I, T=1)
    wn = O.numpy_weights(d)
    e_loc = E // world
    local = pkg.CutlassGptOssExperts(Cfg(e_loc, H, I))
    mod = EP.ExpertParallelExperts(local, E, kernels=OracleKernels(O.slice_experts(wn, rank * e_loc,
                                                                                  (rank + 1) * e_loc), H))
    h, ix, wv = routing_case("random", rank, world, 8)
    mod(h, ix, wv)                                  # one good step on both ranks
    if rank == 1:
        q.put((rank, "left", None))
        q.close()
        q.join_thread()                             # the message is out before the process goes
        os._exit(0)                                 # gone between steps
    t0 = time.time()
    try:
        mod(h, ix, wv)
        q.put((rank, ("no error", None, time.time() - t0), None))
    except Exception as e:  # the expected outcome
        q.put((rank, ("error", type(e).__name__, time.time() - t0), None))
    q.close()
    q.join_thread()
    os._exit(0)                                     # the group is broken; skip its teardown
