"""Generates the golden fixtures in this directory from the REFERENCE's own Python.

Run where a checkout of evil0sheep/gpt-oss-mxfp4-compile is available, with the
environment variable GPTOSS_REFERENCE pointing at it; the GPU box never runs this.

What runs, unmodified, from the reference:
  * kernels/cutlass_experts.py: quantize_activations_to_fp8 (:197-251), swiglu (:258-276)
  * benchmark_optimizations.py: CutlassExpertsPythonRouting.forward (:163-237) -- stable
    argsort routing, gather, quantise, bias, SwiGLU, requantise, bias, routing weight,
    bf16 scatter_add_ -- with only _run_cutlass_gemm replaced (the CUTLASS SM120 kernel
    cannot run on CPU). The replacement is the reference tests' own GEMM oracle
    (kernels/test_cutlass_experts.py:313-320): bf16(fp32(upcast(A)) @ fp32(upcast(B))^T)
    with triton_kernels' upcast_from_mxfp_torch (the local copy shipped in vllm).

Fixtures (numpy .npz): quant.npz, swiglu.npz, routing.npz, layer_<name>.npz. Inputs are
regenerated from seeds by the tests (the recipes are below and in oracle.synth_layer);
each fixture stores a sha256 of its inputs so a generator drift is detected.
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("GPTOSS_REFERENCE", "")
sys.path.insert(0, REPO)

import oracle as O  # noqa: E402  (only synth_layer: the seeded input recipe)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.contiguous().view(torch.uint8).numpy() if a.dtype == torch.bfloat16 else a.contiguous().numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "kernels")):
        raise SystemExit("set GPTOSS_REFERENCE to a checkout of evil0sheep/gpt-oss-mxfp4-compile")
    spec = importlib.util.spec_from_file_location("cutlass_experts", os.path.join(REF, "kernels", "cutlass_experts.py"))
    ce = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ce)
    sys.modules["cutlass_experts"] = ce
    spec = importlib.util.spec_from_file_location("benchmark_optimizations", os.path.join(REF, "benchmark_optimizations.py"))
    bo = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bo)
    return ce, bo


def quant_inputs():
    """Shapes of kernels/test_cutlass_experts.py:56-59 (seed 42) plus edge-value cases."""
    cases = []
    for M, K in [(128, 256), (64, 512), (256, 1024)]:
        torch.manual_seed(42)
        cases.append((f"bf16_{M}x{K}", torch.randn(M, K, dtype=torch.bfloat16)))
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, 256, generator=g) * torch.logspace(-30, 30, 64).unsqueeze(1)
    x[0] = 0.0
    x[1, :32] = -0.0
    x[2, :32] = 1e-42
    x[3, 5] = 448.0
    x[4, :32] = torch.linspace(-1, 1, 32) * 3.0e38
    cases.append(("f32_edges", x.float()))
    cases.append(("bf16_edges", x.clamp(-3e38, 3e38).to(torch.bfloat16)))
    return cases


def make_quant(ce):
    out = {}
    for name, x in quant_inputs():
        q, s = ce.quantize_activations_to_fp8(x)
        out[f"{name}__codes"] = q.view(torch.uint8).numpy()
        out[f"{name}__scales"] = s.numpy()
        out[f"{name}__sha"] = np.frombuffer(sha(x).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)


def swiglu_inputs():
    torch.manual_seed(42)
    a = torch.randn(64, 200, dtype=torch.bfloat16)          # test_cutlass_experts.py:116
    g = torch.Generator().manual_seed(6)
    b = torch.randn(96, 384, generator=g) * 6.0
    return [("bf16_64x200", a), ("f32_96x384", b)]


def make_swiglu(ce):
    out = {}
    for name, x in swiglu_inputs():
        y = ce.swiglu(x, 1.702, 7.0)
        out[f"{name}__out"] = y.view(torch.int16).numpy() if y.dtype == torch.bfloat16 else y.numpy()
        out[f"{name}__sha"] = np.frombuffer(sha(x).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "swiglu.npz"), **out)


def routing_inputs():
    """kernels/test_cutlass_experts.py:561-568 (T=128, E=32, top-4, seed 42)."""
    torch.manual_seed(42)
    logits = torch.randn(128, 32)
    w, idx = torch.topk(logits, 4, dim=-1)
    return idx, torch.softmax(w, dim=-1)


class _Cfg:
    def __init__(self, E, H, I):
        self.num_local_experts = E
        self.hidden_size = H
        self.intermediate_size = I
        self.swiglu_limit = 7.0


def run_reference_layer(bo, ce, d, router_indices, routing_weights, E, H, I):
    """CutlassExpertsPythonRouting.forward with the dequant GEMM oracle; returns output and
    the GEMM inputs the reference produced."""
    from vllm.third_party.triton_kernels.numerics_details.mxfp import upcast_from_mxfp_torch as upcast

    captured = []

    class GoldenExperts(bo.CutlassExpertsPythonRouting):
        def _run_cutlass_gemm(self, activations, act_scales_rowmajor, weights, weight_scales,
                              expert_token_counts, expert_offsets, N, K, K_padded):
            # forward() calls the gate_up GEMM first and the down GEMM second
            wb, ws = (self._gu_blocks, self._gu_scales) if len(captured) % 2 == 0 else (
                self._dn_blocks, self._dn_scales)
            captured.append(dict(codes=activations.view(torch.uint8).clone(), scales=act_scales_rowmajor.clone(),
                                 counts=expert_token_counts.clone(), offsets=expert_offsets.clone()))
            out = torch.zeros((activations.shape[0], N), dtype=torch.bfloat16)
            for e in range(self.num_experts):
                m = int(expert_token_counts[e])
                o = int(expert_offsets[e])
                if m == 0:
                    continue
                x_deq = upcast(activations[o:o + m], act_scales_rowmajor[o:o + m], torch.bfloat16, axis=1)
                w_deq = upcast(wb[e], ws[e], torch.bfloat16, axis=1)
                out[o:o + m] = (x_deq.float() @ w_deq.float().T).to(torch.bfloat16)
            return out

    m = GoldenExperts(_Cfg(E, H, I))
    m.gate_up_proj_bias.data.copy_(d["gu_bias"])
    m.down_proj_bias.data.copy_(d["dn_bias"])
    m._gu_blocks, m._gu_scales = d["gu_blocks"], d["gu_scales"]
    m._dn_blocks, m._dn_scales = d["dn_blocks"], d["dn_scales"]
    m.gate_up_proj_data = d["gu_blocks"]
    m.down_proj_data = d["dn_blocks"]
    m.K_hidden_padded = ce.pad_k_to_tile(H)
    m.K_inter_padded = ce.pad_k_to_tile(I)
    with torch.no_grad():
        y = m(d["hidden"], router_indices, routing_weights)
    return y, captured


LAYERS = {
    # name: (seed, E, H, I, T, top_k)
    "small": (11, 4, 512, 256, 32, 2),
    "kpad": (12, 4, 288, 288, 32, 2),
    "decode": (0, 32, 2880, 2880, 32, 4),     # GPT-OSS-20B layer, decode batch
    "cpu_ref": (0, 32, 2880, 2880, 128, 4),   # GPT-OSS-20B layer, the CPU baseline batch
}


def layer_inputs(name):
    seed, E, H, I, T, k = LAYERS[name]
    d = O.synth_layer(seed, E=E, H=H, I=I, T=T)
    logits, scores, idx = O.router_topk_hf(d["hidden"], d["router_w"], d["router_b"], k)
    return d, idx, scores.float()


def make_layers(ce, bo):
    for name, (seed, E, H, I, T, k) in LAYERS.items():
        d, idx, w = layer_inputs(name)
        y, cap = run_reference_layer(bo, ce, d, idx, w, E, H, I)
        g1, g2 = cap
        out = dict(
            out=y.view(torch.int16).numpy(),
            router_indices=idx.numpy(), routing_weights=w.numpy(),
            counts=g1["counts"].numpy(), offsets=g1["offsets"].numpy(),
            act_codes_sha=np.frombuffer(sha(g1["codes"]).encode(), dtype=np.uint8),
            act_scales_sha=np.frombuffer(sha(g1["scales"]).encode(), dtype=np.uint8),
            inter_codes_sha=np.frombuffer(sha(g2["codes"]).encode(), dtype=np.uint8),
            inputs_sha=np.frombuffer(sha(d["hidden"], d["gu_blocks"], d["gu_scales"], d["dn_blocks"],
                                         d["dn_scales"], d["gu_bias"], d["dn_bias"]).encode(), dtype=np.uint8),
        )
        if T * k <= 128 and H <= 512:
            out.update(act_codes=g1["codes"].numpy(), act_scales=g1["scales"].numpy(),
                       inter_codes=g2["codes"].numpy(), inter_scales=g2["scales"].numpy())
        np.savez_compressed(os.path.join(HERE, f"layer_{name}.npz"), **out)
        print(name, "done", y.float().abs().mean().item())


def make_routing():
    ce, bo = load_reference()
    idx, w = routing_inputs()
    # The reference's stable-argsort routing lines (benchmark_optimizations.py:170-187),
    # executed through a tiny CutlassExpertsPythonRouting forward whose GEMM hook records
    # the counts / offsets and the sorted activation rows.
    E, H = 32, 64
    g = torch.Generator().manual_seed(3)
    hidden = torch.randn(128, H, generator=g).to(torch.bfloat16)
    d = dict(hidden=hidden,
             gu_blocks=torch.zeros(E, 2 * H, H // 2, dtype=torch.uint8), gu_scales=torch.full((E, 2 * H, H // 32), 127, dtype=torch.uint8),
             dn_blocks=torch.zeros(E, H, H // 2, dtype=torch.uint8), dn_scales=torch.full((E, H, H // 32), 127, dtype=torch.uint8),
             gu_bias=torch.zeros(E, 2 * H), dn_bias=torch.zeros(E, H))
    _, cap = run_reference_layer(bo, ce, d, idx, w, E, H, H)
    q_hidden, _ = ce.quantize_activations_to_fp8(hidden)
    rows = q_hidden.view(torch.uint8)
    codes = cap[0]["codes"]
    # recover the permutation: each sorted row equals the quantised row of its token
    perm = []
    for r in range(codes.shape[0]):
        match = (rows == codes[r]).all(dim=1).nonzero().flatten().tolist()
        assert len(match) == 1
        perm.append(match[0])
    np.savez_compressed(os.path.join(HERE, "routing.npz"), router_indices=idx.numpy(), routing_weights=w.numpy(),
                        counts=cap[0]["counts"].numpy(), offsets=cap[0]["offsets"].numpy(),
                        sorted_token=np.asarray(perm, dtype=np.int64))


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    ce, bo = load_reference()
    make_quant(ce)
    make_swiglu(ce)
    make_routing()
    make_layers(ce, bo)


if __name__ == "__main__":
    main()
