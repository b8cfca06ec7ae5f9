"""CPU oracle for the GPT-OSS MXFP4 W4A8 expert path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
``--impl reference``) may import this package, and only as the checker or the timed CPU
baseline. The product package (gpt-oss-mxfp4-compile_b200/) never imports it.

What it restates (citations are path:line in evil0sheep/gpt-oss-mxfp4-compile):
  * quantize_fp8_ue8m0       kernels/cutlass_experts.py:197-251
  * swiglu_fp32              kernels/cutlass_experts.py:258-276
  * blocked_sf_offset/...    the blocked scale layout the reference builds with CuTe
                             (kernels/matmul_mxfp4_cutlass.cu:666-759, :763-873)
  * route_stable             benchmark_optimizations.py:170-187 (stable argsort routing)
  * group_mm_bf16            the W4A8 grouped GEMM semantics (matmul_mxfp4_cutlass.cu:
                             471-655), as the reference validates it: bf16 of the fp32
                             product of dequantised operands (test_mxfp4_matmul.py:245-248,
                             kernels/test_cutlass_experts.py:313-320)
  * w4a8_experts_forward     CutlassGptOssExperts.forward, kernels/cutlass_experts.py:376-452
  * dequant_fp32_reference   kernels/test_cutlass_experts.py:422-455 (per-token loop)
  * router_topk_hf           HF GptOssTopKRouter (F.linear -> topk -> softmax(bf16))

Pinning: tests/golden/ holds outputs of the reference's own Python run in the build
container (tests/golden/make_golden.py) and offsets from CuTe's
Sm1xxBlockScaledConfig<32> (tests/golden/cute_sf_layout.cu); tests/test_oracle.py checks
this package against both.
"""
from .moe_oracle import *  # noqa: F401,F403
