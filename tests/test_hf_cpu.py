"""Hugging Face integration, host side: the checkpoint reader resolves tensor names through
the safetensors index the way the reference's loader does (test_cutlass_model.py:55-75)."""
import json
import os

import torch


def test_checkpoint_getter_reads_sharded_safetensors(pkg, tmp_path):
    from safetensors.torch import save_file
    a = {"model.layers.0.mlp.experts.gate_up_proj_bias": torch.arange(6, dtype=torch.float32).reshape(2, 3)}
    b = {"model.layers.1.mlp.experts.down_proj_scales": torch.full((2, 4, 1), 121, dtype=torch.uint8)}
    save_file(a, os.path.join(tmp_path, "model-00001-of-00002.safetensors"))
    save_file(b, os.path.join(tmp_path, "model-00002-of-00002.safetensors"))
    index = {"weight_map": {**{k: "model-00001-of-00002.safetensors" for k in a},
                            **{k: "model-00002-of-00002.safetensors" for k in b}}}
    with open(os.path.join(tmp_path, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f)
    get = pkg.hf.checkpoint_getter(str(tmp_path))
    for k, v in {**a, **b}.items():
        assert torch.equal(get(k), v)


def test_none_swiglu_limit_means_seven(pkg):
    class C:
        num_local_experts, hidden_size, intermediate_size, num_experts_per_tok = 4, 64, 64, 2
        swiglu_limit = None
    assert pkg.CutlassGptOssExperts(C()).limit == 7.0
