"""B200-native (sm_100a) GPT-OSS MXFP4 W4A8 mixture-of-experts expert path.

The directory name is not a Python identifier; load it with :func:`load_package` in the
repository's ``__graft_entry__.py`` (which registers it as ``gpt_oss_mxfp4_compile_b200``)
or with importlib.util.spec_from_file_location.

Public surface (mirrors kernels/cutlass_experts.py of the reference):
  CutlassGptOssExperts, load_cutlass_weights, quantize_activations_to_fp8, swiglu,
  pad_k_to_tile, pad_fp4_weights, pad_fp8_activations, get_cutlass_extension,
  ensure_custom_op_registered, MXFP_BLOCK_SIZE, MMA_TILE_K
plus the fused layer (router + experts): :class:`GptOssMoELayer`, expert parallelism
(peer memory or NCCL) in :mod:`.ep`, and Hugging Face model integration in :mod:`.hf`.
"""
from . import _lib, ops  # noqa: F401
from .cutlass_experts import (  # noqa: F401
    MMA_TILE_K,
    MXFP_BLOCK_SIZE,
    CutlassGptOssExperts,
    ensure_custom_op_registered,
    get_cutlass_extension,
    load_cutlass_weights,
    pad_fp4_weights,
    pad_fp8_activations,
    pad_k_to_tile,
    quantize_activations_to_fp8,
    swiglu,
)
from .layer import GptOssMoELayer  # noqa: F401
from . import ep  # noqa: F401,E402
from . import hf  # noqa: F401,E402
