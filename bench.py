#!/usr/bin/env python
"""GPT-OSS-20B MoE layer benchmark on B200 (router + W4A8 experts, one step = one layer
forward over one batch of synthetic tokens).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config decode|prefill|stack|zipf]
  python bench.py --impl reference ...     CPU baseline arm (rank 0 only)

Workload at N=1: one GPT-OSS-20B MoE layer at decode (T=32 tokens, E=32, H=I=2880,
top-4, seeded synthetic weights/inputs). Under torchrun (N>1) the layer runs expert-parallel:
rank r holds experts [r*E/N, (r+1)*E/N) and its own batch of T tokens (weak scaling);
dispatch and combine move rows over NVLink (stores into peer-mapped buffers for
fixed-capacity exchanges, NCCL all-to-alls for exact splits). The reported value is the whole-job tokens/s
over the max-over-ranks device time.

Timing: W warm-up steps, then exactly K steps, each bracketed by CUDA events on the
launching stream; barrier + synchronize on both sides of the timed region. L2: every
configuration streams more input than L2 holds (424 MB of expert weights per layer step
against 126 MB of L2), so by default nothing is flushed between steps; `--l2 write`
writes a 256 MiB buffer before every timed step instead (its dirty lines are written back
to HBM inside the next step, so that number also carries the flush's write-back). The
JSON line reports the no-flush number and, for comparison, the write-flush one.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "GPT-OSS-20B MoE layer tokens/s; %HBM roofline (decode), %MMA peak (prefill)"

CONFIGS = {
    # name: (T, E, H, I, top_k, skew, description)
    "decode": (32, 32, 2880, 2880, 4, None, "GPT-OSS-20B MoE layer decode, T=32"),
    "prefill": (8192, 32, 2880, 2880, 4, "prefill", "GPT-OSS-20B MoE layer prefill, T=8192, loads +-50%"),
    "stack": (4096, 32, 2880, 2880, 4, None,
              "GPT-OSS-20B-shaped 24-layer stack (RMSNorm -> MoE -> residual), T=4096"),
    "zipf": (16384, 128, 2880, 2880, 4, "zipf",
             "GPT-OSS-120B-shaped MoE layer, 1.5 log-Zipf(1.1) router bias, T=16384"),
}
STACK_LAYERS = 24
CPU_BASELINE_CONFIGS = ("decode", "prefill")   # the others are minutes of CPU work per step

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from one
# ncu capture of that kernel on this workload (None until captured for this kernel/config).
NCU_TRAFFIC_BYTES = {"decode": 439_218_944,     # decode_layer_kernel, T = 32
                     "prefill": 769_571_328}    # GEMM1, tokens-on-M CTA-pair tiles, T = 8192



def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=list(CONFIGS), default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=45.0,
                    help="reference arm: CPU seconds the whole --warmup + --steps run may take; each step "
                         "times a token sample of the workload sized to fit")
    ap.add_argument("--mma-peak", action="store_true",
                    help="only measure the block-scaled FP8 x FP4 MMA peak (gptoss_mma_peak) and print it")
    ap.add_argument("--w4a4", action="store_true",
                    help="only measure the W4A4 (NVFP4) mode of fp4_group_mm: the reference's micro-bench "
                         "shape and a prefill-sized grouped shape, against the measured kind::mxf4nvf4 peak")
    ap.add_argument("--l2", choices=["none", "write"], default="none",
                    help="between timed steps: nothing (inputs larger than L2) or write a 256 MiB buffer")
    ap.add_argument("--ep-transport", choices=["auto", "p2p", "nccl"], default="auto",
                    help="N>1 exchange: stores into peer-mapped buffers (p2p, fixed capacity) or NCCL "
                         "all-to-alls; auto = p2p with the capacity layout, NCCL with exact splits")
    ap.add_argument("--ep-layout", choices=["auto", "capacity", "exact"], default="auto",
                    help="N>1 exchange layout: fixed-capacity segments (no host sync) or exact splits; "
                         "auto = capacity when W*T*k <= 8192 rows")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def alg_bytes(counts, T, k, H, I, E):
    """Algorithmic HBM bytes of one layer step (unpadded K): weights + scales + fp32
    biases of every touched expert, router weights, activations in/out and the FP8
    intermediates written and read once."""
    touched = sum(1 for c in counts if c > 0)
    A = T * k
    gu = touched * (2 * I * (H // 2) + 2 * I * (H // 32) + 2 * I * 4)
    dn = touched * (H * (I // 2) + H * (I // 32) + H * 4)
    act = A * H + A * (H // 32)           # FP8 rows + scales (GEMM1 A operand)
    inter = A * I + A * (I // 32)         # FP8 intermediate (written by GEMM1, read by GEMM2)
    g1 = gu + act + inter
    g2 = dn + inter + 2 * T * H           # output rows (read-modify-write counted once)
    layer = g1 + g2 + E * H * 2 + E * 2 + 2 * T * H   # + router weight and bias, hidden in
    return g1, g2, layer, touched


def clock_sampler_start(dev_index: int):
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        return subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100",
                                 "-i", str(dev_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except Exception:
        return None


def clock_sampler_stop(proc):
    if proc is None:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    time.sleep(0.25)
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except Exception:
        proc.kill()
        out = ""
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            mx.append(float(f[2]))
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower().startswith("active"):
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def cpu_baseline(cfg_name: str, steps: int, warmup: int, budget_s: float):
    """The reference's dequantised PyTorch CPU path (oracle.DequantCPULayer) on the host
    cores: `warmup` untimed and `steps` timed calls, each on the workload's first n
    tokens, n chosen (from one trial call) so that the whole run takes about budget_s."""
    import torch
    import oracle as O
    T, E, H, I, k, skew, _ = CONFIGS[cfg_name]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    d = O.synth_layer(0, E=E, H=H, I=I, T=T, skew=skew)
    t0 = time.perf_counter()
    layer = O.DequantCPULayer(d, top_k=k)
    dequant_s = time.perf_counter() - t0
    h = d["hidden"]
    n_try = min(T, 512)
    tw = time.perf_counter()
    layer(h[:n_try])
    per_tok = max(time.perf_counter() - tw, 1e-4) / n_try     # an upper bound for larger samples
    n = int(max(1, min(T, budget_s / max(1, steps + warmup) / per_tok)))
    sample = h[:n]
    for _ in range(warmup):
        layer(sample)
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        layer(sample)
        times.append(time.perf_counter() - t)
    per = statistics.mean(times)
    what = f"{steps} timed steps of {n} of the workload's {T} tokens"
    if cfg_name == "stack":   # one MoE layer timed; the stack is STACK_LAYERS of them (norms not counted)
        per *= STACK_LAYERS
        what += f" (one MoE layer, x {STACK_LAYERS} layers)"
    return {"value": n / per, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{what} through the dequantised bf16 expert path + HF router, "
                      f"mean {per * 1e3:.1f} ms/step; weights dequantised once beforehand ({dequant_s:.1f} s)",
            "ms_per_step": per * 1e3, "steps_run": steps, "tokens_per_step": n}


def workload_config(args, world: int) -> dict:
    """The `config` object both arms print (same keys and values for the same command line)."""
    T, E, H, I, k, _, desc = CONFIGS[args.config]
    if world > 1:
        layout, transport = ep_choice(args, world, T, k)
        par = (f"ep{world} (E/{world} experts per GPU, "
               f"{'peer-memory stores' if transport == 'p2p' else 'NCCL all-to-all'})")
    else:
        par = "single GPU"
    l2 = ("none between steps: inputs larger than L2 (each layer step streams 424 MB of expert weights; "
          "L2 is 126 MB)" if args.l2 == "none" else "256 MiB written before every timed step")
    return {"workload": desc, "T": T, "T_per_rank": T, "E": E, "hidden": H, "intermediate": I, "top_k": k,
            "parallelism": par, "l2": l2}


def ep_choice(args, world: int, T: int, k: int):
    """Expert-parallel exchange layout and transport for N > 1."""
    layout = args.ep_layout
    if layout == "auto":
        layout = "capacity" if world * T * k <= 8192 else "exact"
    transport = args.ep_transport
    if transport == "auto":
        transport = "p2p" if layout == "capacity" else "nccl"
    return layout, transport


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cb = cpu_baseline(args.config, max(1, args.steps), max(0, args.warmup), args.cpu_budget_s)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (dequantised weights), fp32 accumulate",
            "data": "synthetic (seeded: random MXFP4 weights, N(0,1) bf16 hidden)",
            "config": workload_config(args, world),
            "reference_note": f"the reference's CPU expert path on {cb['cores']} host cores, rank 0 only; "
                              f"{cb['tokens_per_step']} tokens per step",
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def device_layer_weights(E, H, I, seed, dev):
    """One layer's random weights with the synthetic recipe's distributions, drawn on the
    device (the 24-layer stack's 10 GB would take minutes on the host)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    d = {"router_w": (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16),
         "router_b": (torch.randn(E, generator=g, device=dev) * 0.01).to(torch.bfloat16)}
    for pre, n, kk in (("gu", 2 * I, H), ("dn", H, I)):
        d[f"{pre}_blocks"] = torch.randint(0, 256, (E, n, kk // 2), generator=g, device=dev, dtype=torch.uint8)
        d[f"{pre}_scales"] = torch.randint(119, 124, (E, n, kk // 32), generator=g, device=dev, dtype=torch.uint8)
        d[f"{pre}_bias"] = (torch.randn(E, n, generator=g, device=dev) * 0.01).to(torch.bfloat16).float()
    return d


def build_stack(pkg, Cfg, world, rank, dev, args, T, E, H, I, k):
    """The stack workload: STACK_LAYERS layers of RMSNorm -> MoE layer -> residual, fresh
    weights per layer (identical on every rank); under torchrun each rank keeps its E/N
    experts of every layer (NCCL all-to-alls with exact splits)."""
    import torch
    layers = []
    e_loc = E // world
    lo, hi = rank * e_loc, (rank + 1) * e_loc

    class LocalCfg(Cfg):
        num_local_experts = e_loc

    for li in range(STACK_LAYERS):
        d = device_layer_weights(E, H, I, 7000 + li, dev)
        ex = pkg.CutlassGptOssExperts(LocalCfg()).to(dev)
        ex.gate_up_proj_bias.data.copy_(d["gu_bias"][lo:hi])
        ex.down_proj_bias.data.copy_(d["dn_bias"][lo:hi])
        pkg.load_cutlass_weights(ex, d["gu_blocks"][lo:hi], d["gu_scales"][lo:hi], d["dn_blocks"][lo:hi],
                                 d["dn_scales"][lo:hi], dev)
        if world == 1:
            lay = pkg.GptOssMoELayer(Cfg()).to(dev)
            lay.experts = ex
            lay.router_weight.data.copy_(d["router_w"])
            lay.router_bias.data.copy_(d["router_b"])
        else:
            ep_ex = pkg.ep.ExpertParallelExperts(ex, E, top_k=k)
            lay = pkg.ep.ExpertParallelMoELayer(d["router_w"], d["router_b"], k, ep_ex)
        layers.append(lay)
        del d
    return layers, torch.ones(H, dtype=torch.bfloat16, device=dev)


def run_ours(args):
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    import oracle as O

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pkg = ge.load_package()
    pkg.ensure_custom_op_registered()
    T, E, H, I, k, skew, desc = CONFIGS[args.config]

    class Cfg:
        num_local_experts = E
        hidden_size = H
        intermediate_size = I
        num_experts_per_tok = k
        swiglu_limit = 7.0

    stack = args.config == "stack"
    if stack:
        layers, norm_w = build_stack(pkg, Cfg, world, rank, dev, args, T, E, H, I, k)
        g = torch.Generator().manual_seed(1000 + rank)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        layer, ex = layers[0], None

        if world == 1:
            # RMSNorm, the residual copy and the MoE layer as the block op (the norm kernel, then
            # the MoE kernels adding into the residual rows)
            def forward(t):
                for lay in layers:
                    t = lay.forward_block(t, norm_w, 1e-5)[0]
                return t
        else:
            def forward(t):
                for lay in layers:
                    t = t + lay(torch.nn.functional.rms_norm(t, (H,), norm_w, 1e-5))[0]
                return t
    elif world == 1:
        d = O.synth_layer(rank, E=E, H=H, I=I, T=T, skew=skew)
        layer = pkg.GptOssMoELayer(Cfg()).to(dev)
        layer.router_weight.data.copy_(d["router_w"])
        layer.router_bias.data.copy_(d["router_b"])
        ex = layer.experts
        ex.gate_up_proj_bias.data.copy_(d["gu_bias"])
        ex.down_proj_bias.data.copy_(d["dn_bias"])
        pkg.load_cutlass_weights(ex, d["gu_blocks"], d["gu_scales"], d["dn_blocks"], d["dn_scales"], dev)
        x = d["hidden"].to(dev)
    else:
        # one layer's weights, identical on every rank (seed 0); each rank keeps its
        # E/N experts and routes its own tokens
        d = O.synth_layer(0, E=E, H=H, I=I, T=T, skew=skew, with_hidden=False)
        e_loc = E // world
        lo, hi = rank * e_loc, (rank + 1) * e_loc

        class LocalCfg(Cfg):
            num_local_experts = e_loc

        ex = pkg.CutlassGptOssExperts(LocalCfg()).to(dev)
        ex.gate_up_proj_bias.data.copy_(d["gu_bias"][lo:hi])
        ex.down_proj_bias.data.copy_(d["dn_bias"][lo:hi])
        pkg.load_cutlass_weights(ex, d["gu_blocks"][lo:hi], d["gu_scales"][lo:hi], d["dn_blocks"][lo:hi],
                                 d["dn_scales"][lo:hi], dev)
        layout, transport = ep_choice(args, world, T, k)
        ep_experts = pkg.ep.ExpertParallelExperts(ex, E, capacity_tokens=T if layout == "capacity" else None,
                                                  transport=transport, top_k=k)
        layer = pkg.ep.ExpertParallelMoELayer(d["router_w"].to(dev), d["router_b"].to(dev), k, ep_experts)
        g = torch.Generator().manual_seed(1000 + rank)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    if not stack:
        del d

        def forward(t):
            return layer(t)[0]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def step():
        return forward(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    assert pkg.ops.read_status(dev) == 0
    graph_launches = None
    if stack and world == 1:
        # the 24-layer step as one CUDA graph: one host call per step; the library's launches
        # are counted once, at capture
        graph = torch.cuda.CUDAGraph()
        n0 = pkg._lib.query("gptoss_kernel_launch_count")
        with torch.cuda.graph(graph):
            graph_out = forward(x)
        graph_launches = int(pkg._lib.query("gptoss_kernel_launch_count") - n0)
        eager_forward = forward

        def step():
            graph.replay()
            return graph_out

        def forward(t):
            if t is not x:
                x.copy_(t, non_blocking=True)
            graph.replay()
            return graph_out

        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        assert pkg.ops.read_status(dev) == 0
        _ = eager_forward

    # ---------------------------------------------------------------- headline
    K = args.steps

    def timed_loop(l2_mode: str):
        """K steps back to back (consecutive launches overlap as programmatic dependent
        launches let them) between one pair of CUDA events; with the write flush every step
        is bracketed by its own pair instead (the flush itself stays outside)."""
        barrier()
        torch.cuda.synchronize(dev)
        sampler = clock_sampler_start(dev.index)
        time.sleep(0.3)
        launches0 = pkg._lib.query("gptoss_kernel_launch_count")
        if l2_mode == "write":
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
            for i in range(K):
                flush.zero_()
                ev[i][0].record(stream)
                step()
                ev[i][1].record(stream)
        else:
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))]
            ev[0][0].record(stream)
            for i in range(K):
                step()
            ev[0][1].record(stream)
        n_launch = int(pkg._lib.query("gptoss_kernel_launch_count") - launches0)   # this library's kernels
        if graph_launches is not None:        # replays launch the captured kernels
            n_launch = graph_launches * K
        torch.cuda.synchronize(dev)
        clk = clock_sampler_stop(sampler)
        barrier()
        t_ms = sum(s.elapsed_time(e) for s, e in ev) / K
        if world > 1:
            t = torch.tensor([t_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms, n_launch, clk

    ms, launches, clocks = timed_loop(args.l2)
    value = T * world / (ms / 1e3)
    other = "write" if args.l2 == "none" else "none"
    ms_other, _, _ = timed_loop(other)

    # ---------------------------------------------------------------- per-stage (roofline)
    stages = (stage_roofline(pkg, layer, ex, x, flush if args.l2 == "write" else None, stream, T, k, E, H, I, K,
                             ms, dev, args.config, launches / K)
              if world == 1 and not stack else None)

    # ---------------------------------------------------------------- end to end
    # Every step: its input copied host -> device from pinned memory, the layer, its output
    # copied device -> host into pinned memory. The copies run on two copy streams, so step
    # i+1's input lands while step i computes and step i's output drains while step i+1
    # computes (two device input buffers; events order every reuse). A graph replay writes
    # one static output tensor, so there the next step also waits for the previous output's
    # copy. One host synchronisation at the end; the events bracket the first input copy and
    # the last output copy.
    xh = x.cpu().pin_memory()
    ohs = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xds = [torch.empty_like(x) for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    static_out = graph_launches is not None
    Ke = min(K, 500)

    def e2e_steps(n: int, start: torch.cuda.Event):
        landed = [torch.cuda.Event(), torch.cuda.Event()]   # input j is on the device
        read = [None, None]                                 # the step that read input j is done
        copied = None                                       # the previous output is on the host
        h2d.wait_event(start)
        for i in range(n):
            j = i & 1
            with torch.cuda.stream(h2d):
                if read[j] is not None:
                    h2d.wait_event(read[j])
                xds[j].copy_(xh, non_blocking=True)
                landed[j].record(h2d)
            stream.wait_event(landed[j])
            if static_out and copied is not None:
                stream.wait_event(copied)
            y = forward(xds[j])
            read[j] = torch.cuda.Event()
            read[j].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(read[j])
                ohs[j].copy_(y, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(d2h)
            if not static_out:
                y.record_stream(d2h)             # the allocator keeps y until its copy is done
        stream.wait_stream(h2d)
        stream.wait_stream(d2h)

    barrier()
    w0 = torch.cuda.Event()
    w0.record(stream)
    e2e_steps(3, w0)                             # warm-up of the copy path
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    e2e_steps(Ke, a)
    b.record(stream)
    b.synchronize()
    e2e_ms = a.elapsed_time(b) / Ke
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    assert pkg.ops.read_status(dev) == 0

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config in CPU_BASELINE_CONFIGS:
        cb = cpu_baseline(args.config, 50, 2, min(args.cpu_budget_s, 30.0))
        cpu = {k2: cb[k2] for k2 in ("value", "unit", "cores", "kind", "sample")}

    ep_info = None
    if world > 1:
        rb = pkg.ops.ep_row_bytes(H)
        epx = layer.experts
        if epx.capacity_tokens:
            cap = epx.capacity_tokens * k
            sent = epx.last_send_counts.cpu().tolist()
            if epx.transport == "p2p":
                moved = (sum(sent) - sent[rank]) * (rb + 2 * H)
            else:
                moved = (world - 1) * cap * (rb + 2 * H)
            ep_info = {"layout": "fixed capacity", "transport": epx.transport, "capacity_rows_per_peer": cap,
                       "rank0_rows_used": sent, "rank0_nvlink_bytes_per_step": moved, "host_syncs_per_step": 0}
            if epx.transport == "p2p":
                ep_info["kernels"] = ("one persistent launch per rank and step (decode_layer_kernel<true>) behind a "
                                      "one-CTA reset" if epx._p2p_one_launch(x, cap) else
                                      "five launches per step (route-dispatch, receive, GEMM1, GEMM2 + return, "
                                      "combine)")
        else:
            s_send, s_recv = epx.last_splits
            ep_info = {"layout": "exact splits", "transport": "nccl", "rank0_rows_sent": s_send,
                       "rank0_rows_received": s_recv,
                       "rank0_nvlink_bytes_per_step": (sum(s_send) - s_send[rank] + sum(s_recv) - s_recv[rank])
                       * (rb + 2 * H), "host_syncs_per_step": STACK_LAYERS if stack else 1}
        ep_info.update({"experts_per_rank": E // world, "row_bytes_dispatch": rb, "row_bytes_combine": H * 2})

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8 e4m3 x fp4 e2m1 (UE8M0 1x32 scales), fp32 accumulate",
            "data": "synthetic (seeded: random MXFP4 weights, N(0,1) bf16 hidden)",
            "config": workload_config(args, world),
            "l2_comparison": {"l2": other, "ms_per_step": ms_other, "value": T * world / (ms_other / 1e3)},
            "roofline": stages["roofline"] if stages else None,
            "clocks": clocks,
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2 + (2 * world * 4 * ep_info["host_syncs_per_step"]
                                                       if ep_info else 0),
                    "copies": ("pinned host buffers; input and output copies on two copy streams, "
                               "overlapping the neighbouring steps' compute" +
                               ("; each graph replay waits for the previous output's copy" if static_out else ""))},
            "gpu_launches": launches,
            "cpu_baseline": cpu,
        }
        if stages:
            line["experts_touched"] = stages["touched"]
            line["layer_hbm"] = stages["layer_hbm"]
            line["mma"] = stages["mma"]
        if ep_info:
            line["ep"] = ep_info
            line["roofline_note"] = "per-kernel roofline is reported by the N=1 run"
        print(json.dumps(line), flush=True)
    if world > 1:
        for lay in (layers if stack else [layer]):
            lay.experts.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def stage_roofline(pkg, layer, ex, x, flush, stream, T, k, E, H, I, K, ms, dev, cfg_name, launches_per_step):
    """Times router+route+quant, GEMM1 and GEMM2 separately (single GPU, the staged API)
    and returns the roofline of the dominant kernel plus layer-level HBM and MMA figures.
    Decode-sized layers run as one persistent launch (decode_layer_kernel, plus a one-CTA
    reset of its synchronisation words): that kernel is the dominant one, its algorithmic
    bytes are the whole layer's and its time per launch is the timed loop's ms per step.
    Larger layers run router, sort, quantiser and the two GEMMs as separate kernels; GEMM1
    is the dominant one."""
    import torch
    ws = pkg.ops.ExpertsWorkspace(T, k, E, H, I, dev)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    Ks = min(K, 500)
    g1_ms, g2_ms, pre_ms = [], [], []
    for i in range(Ks + 3):
        # hold the stream so every launch of this step is queued before the GPU reaches
        # it (the staged calls go through Python; no host gap may land inside an event pair)
        torch.cuda._sleep(2_000_000)
        if flush is not None:
            flush.zero_()
        e0, e1, e2, e3 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
        e0.record(stream)
        _, sc, ix = layer.route(x)
        pkg.ops.route_quant(ws, x, ix, sc.float())
        out.zero_()
        e1.record(stream)
        pkg.ops.gemm1(ws, ex.gate_up_proj_data, ex.gate_up_proj_scales, ex.gate_up_proj_bias.data)
        e2.record(stream)
        pkg.ops.gemm2(ws, ex.down_proj_data, ex.down_proj_scales, ex.down_proj_bias.data, out)
        e3.record(stream)
        if i >= 3:
            pre_ms.append((e0, e1))
            g1_ms.append((e1, e2))
            g2_ms.append((e2, e3))
    torch.cuda.synchronize(dev)
    t_pre = statistics.mean(a.elapsed_time(b) for a, b in pre_ms)
    t_g1 = statistics.mean(a.elapsed_time(b) for a, b in g1_ms)
    t_g2 = statistics.mean(a.elapsed_time(b) for a, b in g2_ms)
    counts = ws.counts.cpu().tolist()
    b_g1, b_g2, b_layer, touched = alg_bytes(counts, T, k, H, I, E)
    hbm_peak, bf16_peak, peak_kind = measured_peaks()
    g1_gbs = b_g1 / (t_g1 / 1e3) / 1e9
    layer_gbs = b_layer / (ms / 1e3) / 1e9
    flops = 2 * T * k * (H * 2 * I + I * H)
    mma_peak = None
    if cfg_name in ("prefill", "zipf"):
        # dense block-scaled FP8 x FP4 contraction: the tensor pipe bounds it; the peak is
        # this GPU's own kind::mxf8f6f4 rate, measured here (MMA-only probe, CTA pairs, N = 192:
        # the GEMM's instruction shape)
        mma_peak = pkg.ops.mma_peak(dev, pair=True, n=192, iters=4000)["tflops"]
        g1_flops = 2 * T * k * H * 2 * I
        g1_tf = g1_flops / (t_g1 / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": "moe_gemm_kernel (GEMM1 gate_up + SwiGLU + requant, CTA pairs)",
                "achieved": g1_tf, "peak": mma_peak, "unit": "TFLOP/s", "frac": g1_tf / mma_peak,
                "traffic": NCU_TRAFFIC_BYTES.get(cfg_name),
                "peak_kind": "measured in this run: gptoss_mma_peak, kind::mxf8f6f4, CTA pairs, N = 192",
                "alg_flops_per_launch": g1_flops, "ms_per_launch": t_g1}
    elif launches_per_step <= 2.5:
        roof = {"bound": "hbm",
                "kernel": "decode_layer_kernel (router, top-k, sort, FP8 quantisation, GEMM1 + SwiGLU + requant, "
                          "GEMM2 + combine: one persistent launch)",
                "achieved": layer_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": layer_gbs / hbm_peak,
                "traffic": NCU_TRAFFIC_BYTES.get(cfg_name), "peak_kind": peak_kind, "alg_bytes_per_launch": b_layer,
                "ms_per_launch": ms, "launches_per_step": launches_per_step}
    else:
        roof = {"bound": "hbm", "kernel": "moe_gemm_kernel (GEMM1 gate_up + SwiGLU + requant)",
                "achieved": g1_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": g1_gbs / hbm_peak,
                "traffic": NCU_TRAFFIC_BYTES.get(cfg_name), "peak_kind": peak_kind, "alg_bytes_per_launch": b_g1,
                "ms_per_launch": t_g1}
    return {
        "touched": touched,
        "roofline": roof,
        "layer_hbm": {"alg_bytes": b_layer, "achieved_gbs": layer_gbs, "frac": layer_gbs / hbm_peak,
                      "staged_path_ms": {"router+route+quant": t_pre, "gemm1": t_g1, "gemm2": t_g2},
                      "staged_gemm1_gbs": g1_gbs, "staged_gemm2_gbs": b_g2 / (t_g2 / 1e3) / 1e9},
        "mma": {"flops_per_step": flops, "tflops": flops / (ms / 1e3) / 1e12,
                "frac_of_mxf8f6f4_peak": flops / (ms / 1e3) / 1e12 / mma_peak if mma_peak else None,
                "peak_tflops": mma_peak},
    }


def run_mma_peak(args):
    """One JSON line: the measured dense block-scaled FP8 x FP4 MMA throughput (the
    tensor-bound roofline denominator) for CTA pairs and single CTAs at N = 256/192/128."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    dev = torch.device("cuda", 0)
    sampler = clock_sampler_start(0)
    time.sleep(0.3)
    res = [pkg.ops.mma_peak(dev, pair=pair, n=n, iters=4000, kind=kind) for kind in ("mxf8f6f4", "mxf4nvf4")
           for pair in (True, False) for n in (256, 192, 128)]
    clocks = clock_sampler_stop(sampler)
    print(json.dumps({"metric": "block-scaled MMA peak (tcgen05.mma kind::mxf8f6f4 / kind::mxf4nvf4)",
                      "unit": "TFLOP/s",
                      "value": max(r["tflops"] for r in res if r["kind"] == "mxf8f6f4"),
                      "value_mxf4nvf4": max(r["tflops"] for r in res if r["kind"] == "mxf4nvf4"),
                      "results": res, "clocks": clocks}), flush=True)
    return 0


W4A4_SHAPES = {
    # kernels/benchmark_matmul_mxfp4_cutlass.py:51 (one expert)
    "reference_microbench": ([256], 4096, 4096),
    # a prefill-sized gate_up projection: 32 experts x 1024 rows, N = 2 x 2880, K = 2880
    "grouped_prefill": ([1024] * 32, 5760, 2880),
}


def run_w4a4(args):
    """One JSON line: W4A4 (NVFP4 x NVFP4) grouped GEMM throughput per shape and tile
    orientation (CUDA events around `--steps` back-to-back launches after `--warmup`),
    against the measured kind::mxf4nvf4 peak of single CTAs at N = 192 (the tile the
    tokens-on-M kernel issues). Random packed codes and sign-clear UE4M3 scale bytes; the
    scale buffers are filled directly in their blocked layout."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    pkg.ensure_custom_op_registered()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    peak = pkg.ops.mma_peak(dev, pair=False, n=192, iters=4000, kind="mxf4nvf4")["tflops"]
    out_lines = {}
    sampler = clock_sampler_start(0)
    time.sleep(0.3)
    for name, (m_list, N, K) in W4A4_SHAPES.items():
        E, M, G = len(m_list), sum(m_list), K // 16
        a = torch.randint(0, 256, (M, K // 2), device=dev, dtype=torch.uint8, generator=g)
        b = torch.randint(0, 256, (E, N, K // 2), device=dev, dtype=torch.uint8, generator=g)
        blk = lambda rows: ((rows + 127) // 128) * ((G + 3) // 4) * 512   # noqa: E731
        sf_rows = [0]
        for m in m_list[:-1]:
            sf_rows.append(sf_rows[-1] + (m + 127) // 128 * 128)
        sfa = torch.randint(0x30, 0x41, (sum(blk(m) for m in m_list),), device=dev, dtype=torch.uint8, generator=g)
        sfb = torch.randint(0x30, 0x41, (E, blk(N)), device=dev, dtype=torch.uint8, generator=g)
        counts = torch.tensor(m_list, dtype=torch.int32)
        ps = torch.stack([counts, torch.full((E,), N, dtype=torch.int32), torch.full((E,), K, dtype=torch.int32)],
                         1).to(dev)
        offs = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(counts, 0)[:-1].to(torch.int32)]).to(dev)
        sfo = torch.tensor(sf_rows, dtype=torch.int32, device=dev)
        alphas = torch.ones(E, device=dev)
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        flops = 2.0 * M * N * K
        res = {}
        for mode_name, mode in (("tokens_m", 1), ("swap", 2)):
            def call():
                pkg.ops.fp4_group_mm_impl(out, a, b, sfa, sfb, alphas, ps, offs, sfo, gemm_mode=mode)
            for _ in range(max(args.warmup, 3)):
                call()
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(args.steps):
                call()
            ev1.record()
            ev1.synchronize()
            ms = ev0.elapsed_time(ev1) / args.steps
            tf = flops / (ms / 1e3) / 1e12
            res[mode_name] = {"ms_per_call": ms, "tflops": tf, "frac_of_mxf4nvf4_peak": tf / peak}
        assert pkg.ops.read_status(dev) == 0
        out_lines[name] = {"experts": E, "M": M, "N": N, "K": K, "flops": flops, **res}
    clocks = clock_sampler_stop(sampler)
    print(json.dumps({"metric": "W4A4 (NVFP4) grouped GEMM throughput", "unit": "TFLOP/s",
                      "peak_mxf4nvf4_tflops": peak, "steps": args.steps, "warmup": args.warmup,
                      "shapes": out_lines, "clocks": clocks}), flush=True)
    return 0


def main():
    args = parse_args()
    if args.mma_peak:
        return run_mma_peak(args)
    if args.w4a4:
        return run_w4a4(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
