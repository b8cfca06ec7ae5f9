"""Hugging Face GPT-OSS model with this library's experts: a two-layer GptOssForCausalLM
(random attention weights, seeded MXFP4 expert weights) after replace_experts_with_cutlass
(the reference's test_cutlass_model.py:48-117 swap) and after replace_mlp_with_fused_layer
(router + experts in one call), against the same model whose experts run the oracle's
restatement of the reference's W4A8 forward. Every layer's experts are held to the output
gate against the oracle on the inputs (and routing) that layer saw. Whole-model logits are
only held to a loose bound: one-ulp differences of one layer flip FP8 roundings (3 mantissa
bits) and near-tied routings in the next, and this small random model amplifies them. The
model's own eager experts, holding the dequantised MXFP4 weights in bf16, are a sanity bound:
W4A8 itself moves this model's logits by ~12 %."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_output_tolerance, rel_l2

pytestmark = pytest.mark.gpu

E, H, I, K, LAYERS, VOCAB = 8, 512, 512, 4, 2, 512


def _model_and_checkpoint(dev):
    from transformers import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig(hidden_size=H, intermediate_size=I, num_local_experts=E, num_experts_per_tok=K,
                       num_hidden_layers=LAYERS, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                       vocab_size=VOCAB, sliding_window=32,
                       layer_types=["sliding_attention", "full_attention"], swiglu_limit=7.0,
                       attn_implementation="eager", use_cache=False)
    torch.manual_seed(0)
    model = GptOssForCausalLM(cfg).to(torch.bfloat16).to(dev).eval()
    ckpt = {}
    for i in range(LAYERS):
        d = O.synth_layer(300 + i, E=E, H=H, I=I, T=1, with_hidden=False)
        p = f"model.layers.{i}.mlp.experts"
        ckpt[f"{p}.gate_up_proj_blocks"] = d["gu_blocks"]
        ckpt[f"{p}.gate_up_proj_scales"] = d["gu_scales"]
        ckpt[f"{p}.gate_up_proj_bias"] = d["gu_bias"]
        ckpt[f"{p}.down_proj_blocks"] = d["dn_blocks"]
        ckpt[f"{p}.down_proj_scales"] = d["dn_scales"]
        ckpt[f"{p}.down_proj_bias"] = d["dn_bias"]
        gu = np.stack([O.mxfp4_dequant(d["gu_blocks"][e].numpy(), d["gu_scales"][e].numpy()) for e in range(E)])
        dn = np.stack([O.mxfp4_dequant(d["dn_blocks"][e].numpy(), d["dn_scales"][e].numpy()) for e in range(E)])
        mlp = model.model.layers[i].mlp
        with torch.no_grad():      # HF keeps input-major weights: [E, H, 2I] and [E, I, H]
            mlp.experts.gate_up_proj.copy_(torch.from_numpy(gu).transpose(1, 2).to(torch.bfloat16))
            mlp.experts.down_proj.copy_(torch.from_numpy(dn).transpose(1, 2).to(torch.bfloat16))
            mlp.experts.gate_up_proj_bias.copy_(d["gu_bias"].to(torch.bfloat16))
            mlp.experts.down_proj_bias.copy_(d["dn_bias"].to(torch.bfloat16))
            mlp.router.weight.copy_(d["router_w"])
            mlp.router.bias.copy_(d["router_b"])
    return model, ckpt


class OracleExperts(torch.nn.Module):
    """The oracle's W4A8 expert forward (CPU) behind the HF experts interface."""

    def __init__(self, ckpt: dict, prefix: str):
        super().__init__()
        g = lambda n: ckpt[f"{prefix}.{n}"]   # noqa: E731
        self.w = O.numpy_weights({"gu_blocks": g("gate_up_proj_blocks"), "gu_scales": g("gate_up_proj_scales"),
                                  "gu_bias": g("gate_up_proj_bias"), "dn_blocks": g("down_proj_blocks"),
                                  "dn_scales": g("down_proj_scales"), "dn_bias": g("down_proj_bias")})

    def forward(self, hidden_states, router_indices, routing_weights):
        out = O.w4a8_experts_forward(hidden_states.cpu(), router_indices.cpu().numpy(),
                                     routing_weights.float().cpu().numpy(), self.w)
        return out.to(hidden_states.device, hidden_states.dtype)


def _capture(modules):
    """Forward hooks keeping each module's first (args, output); the output is left as is."""
    seen = {}

    def hook(name):
        def keep(module, args, output):
            seen.setdefault(name, (args, output))
        return keep

    for name, m in modules:
        m.register_forward_hook(hook(name))
    return seen


def test_hf_model_with_cutlass_experts(pkg, dev):
    ids = torch.randint(0, VOCAB, (2, 24), generator=torch.Generator().manual_seed(1)).to(dev)
    model, ckpt = _model_and_checkpoint(dev)
    with torch.no_grad():
        bf16_ref = model(ids).logits.float()
        for i in range(LAYERS):
            model.model.layers[i].mlp.experts = OracleExperts(ckpt, f"model.layers.{i}.mlp.experts")
        ref = model(ids).logits.float()
    oracles = [OracleExperts(ckpt, f"model.layers.{i}.mlp.experts") for i in range(LAYERS)]

    # (1) the reference's swap: every layer's experts against the oracle on that layer's inputs
    model, _ = _model_and_checkpoint(dev)
    assert pkg.hf.replace_experts_with_cutlass(model, ckpt.__getitem__) == LAYERS
    assert all(isinstance(model.model.layers[i].mlp.experts, pkg.CutlassGptOssExperts) for i in range(LAYERS))
    seen = _capture([(i, model.model.layers[i].mlp.experts) for i in range(LAYERS)])
    with torch.no_grad():
        out = model(ids).logits.float()
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    for i in range(LAYERS):
        (h, idx, w), o = seen[i]
        assert_output_tolerance(o.cpu(), oracles[i](h, idx, w).cpu(), f"layer {i} experts")
    r, r_bf16 = rel_l2(out.cpu(), ref.cpu()), rel_l2(out.cpu(), bf16_ref.cpu())
    print(f"experts swap: logits rel-L2 {r:.2e} vs the oracle W4A8 model, {r_bf16:.2e} vs the bf16 eager experts")
    assert r <= 0.15 and r_bf16 <= 0.25

    # (2) router + experts fused: each layer against the oracle experts under the layer's routing
    model2, _ = _model_and_checkpoint(dev)
    assert pkg.hf.replace_mlp_with_fused_layer(model2, ckpt.__getitem__) == LAYERS
    seen2 = _capture([(i, model2.model.layers[i].mlp.layer) for i in range(LAYERS)])
    with torch.no_grad():
        out2 = model2(ids).logits.float()
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    for i in range(LAYERS):
        (hs,), (o, scores, ix) = seen2[i]
        ref_o = oracles[i](hs.reshape(-1, H), ix, scores)
        assert_output_tolerance(o.reshape(-1, H).cpu(), ref_o.cpu(), f"layer {i} fused MLP")
    r2 = rel_l2(out2.cpu(), ref.cpu())
    print(f"fused router + experts: logits rel-L2 {r2:.2e} vs the oracle W4A8 model")
    assert r2 <= 0.15


def test_hf_model_compiled_like_the_reference(pkg, dev):
    # the reference's whole-model run (repro_compile_hftf.py:103-107): the GPT-OSS model with
    # the swapped experts under torch.compile(backend="inductor", mode="reduce-overhead") --
    # inductor traces the experts' custom ops through their fake kernels and replays the
    # model as CUDA graphs, and the experts' kernels run. Inductor's own kernels for the rest of
    # the model (norms, attention, the router) round differently from eager torch, and this
    # small random model amplifies every rounding (compiled vs eager measured 0.08-0.09 rel-L2,
    # two eager runs 0.02-0.05), so the logits are held to the whole-model bounds of the eager
    # tests: within the eager bound of the eager model, and within the bf16 sanity bound of
    # the oracle-experts model. A broken compiled path lands near 1.
    ids = torch.randint(0, VOCAB, (2, 24), generator=torch.Generator().manual_seed(2)).to(dev)
    model, ckpt = _model_and_checkpoint(dev)
    with torch.no_grad():
        for i in range(LAYERS):
            model.model.layers[i].mlp.experts = OracleExperts(ckpt, f"model.layers.{i}.mlp.experts")
        ref = model(ids).logits.float()
    model, _ = _model_and_checkpoint(dev)
    assert pkg.hf.replace_experts_with_cutlass(model, ckpt.__getitem__) == LAYERS
    with torch.no_grad():
        eager = model(ids).logits.float()
        eager2 = model(ids).logits.float()
        compiled = torch.compile(model, backend="inductor", mode="reduce-overhead")
        n0 = pkg._lib.query("gptoss_kernel_launch_count")
        for _ in range(3):                        # warm-up, recording, replays
            out = compiled(ids).logits.float().clone()
        n1 = pkg._lib.query("gptoss_kernel_launch_count")
    torch.cuda.synchronize()
    assert pkg.ops.read_status(dev) == 0
    assert n1 > n0, "the compiled model launched none of this library's kernels"
    r_ref, r_eager = rel_l2(out.cpu(), ref.cpu()), rel_l2(eager.cpu(), ref.cpu())
    r_ce, r_ee = rel_l2(out.cpu(), eager.cpu()), rel_l2(eager2.cpu(), eager.cpu())
    print(f"logits rel-L2 vs the oracle W4A8 model: compiled {r_ref:.2e}, eager {r_eager:.2e}; "
          f"compiled vs eager {r_ce:.2e}, two eager runs {r_ee:.2e}")
    assert r_ce <= 0.15 and r_ref <= 0.25
