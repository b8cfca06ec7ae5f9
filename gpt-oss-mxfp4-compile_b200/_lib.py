"""ctypes binding of libgptoss_moe.so (the C ABI in include/gptoss_moe.h).

This is the only place the shared object is loaded. There is no fallback: if the
library is missing or cannot be loaded every call raises, so a run can never silently
take another code path.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_int64 = ctypes.c_int64
_c_int32 = ctypes.c_int32
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
_SIGNATURES = {
    "gptoss_last_error": (ctypes.c_char_p, []),
    "gptoss_abi_version": (_i, []),
    "gptoss_kernel_launch_count": (ctypes.c_uint64, []),
    "gptoss_set_decode_layer_kernel": (_i, [_i]),
    "gptoss_moe_gemm_layout": (_i, [_i, _c_int64, _i]),
    "gptoss_read_status": (_i, [_vp, _vp, _vp]),
    "gptoss_fused_moe_routing": (_i, [_vp, _vp, _c_int64, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gptoss_router_topk": (_i, [_vp, _vp, _vp, _c_int64, _c_int64, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "gptoss_router_topk_from_logits": (_i, [_vp, _c_int64, _i, _i, _vp, _vp, _vp, _vp]),
    "gptoss_mma_peak": (_i, [_i, _i, _i, _i, _vp, _vp]),
    "gptoss_quantize_fp8": (_i, [_vp, _i, _c_int64, _c_int64, _vp, _vp, _vp]),
    "gptoss_swiglu": (_i, [_vp, _i, _c_int64, _c_int64, _vp, _f, _f, _vp]),
    "gptoss_convert_scales_blocked": (_i, [_vp, _c_int64, _c_int64, _vp, _c_int64, _vp]),
    "gptoss_blocked_scales_bytes": (_c_int64, [_c_int64, _c_int64]),
    "gptoss_batch_convert_a_scales": (_i, [_vp, _vp, _vp, _i, _c_int64, _vp, _c_int64, _vp, _vp]),
    "gptoss_batch_blocked_scales_capacity": (_c_int64, [_c_int64, _i, _c_int64]),
    "gptoss_fp4_group_mm": (_i, [_vp, _vp, _c_int64, _c_int64, _vp, _i, _c_int64, _c_int64, _vp, _vp,
                                 _c_int64, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "gptoss_fp4_group_mm_w4a4": (_i, [_vp, _vp, _c_int64, _c_int64, _vp, _i, _c_int64, _c_int64, _vp, _vp,
                                      _c_int64, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "gptoss_moe_workspace_bytes": (_sz, [_c_int64, _i, _i, _c_int64, _c_int64]),
    "gptoss_moe_block_workspace_bytes": (_sz, [_c_int64, _i, _i, _c_int64, _c_int64]),
    "gptoss_moe_block_forward": (_i, [_vp, _vp, _f, _vp, _vp, _c_int64, _i, _i, _c_int64, _c_int64,
                                      _vp, _vp, _c_int64, _vp, _vp, _vp, _c_int64, _vp,
                                      _f, _f, _vp, _vp, _vp, _vp, _sz, _i, _vp, _vp]),
    "gptoss_rmsnorm_residual": (_i, [_vp, _vp, _f, _c_int64, _c_int64, _vp, _vp, _vp]),
    "gptoss_moe_experts_forward": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _c_int64, _c_int64,
                                        _vp, _vp, _c_int64, _vp, _vp, _vp, _c_int64, _vp,
                                        _f, _f, _vp, _vp, _sz, _i, _vp, _vp]),
    "gptoss_moe_layer_forward": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _c_int64, _c_int64,
                                      _vp, _vp, _c_int64, _vp, _vp, _vp, _c_int64, _vp,
                                      _f, _f, _vp, _vp, _vp, _vp, _sz, _i, _vp, _vp]),
    "gptoss_moe_experts_forward_noalloc": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _c_int64, _c_int64,
                                                _vp, _vp, _c_int64, _vp, _vp, _vp, _c_int64, _vp,
                                                _f, _f, _vp, _i, _vp, _vp]),
    "gptoss_moe_workspace_layout": (_i, [_c_int64, _i, _i, _c_int64, _c_int64, _vp]),
    "gptoss_ep_row_bytes": (_c_int64, [_c_int64]),
    "gptoss_ep_dispatch_workspace_bytes": (_sz, [_c_int64, _i, _i]),
    "gptoss_ep_dispatch": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _i, _c_int64, _c_int64, _vp, _vp, _vp, _vp, _sz,
                                _vp, _vp]),
    "gptoss_ep_expert_forward": (_i, [_vp, _c_int64, _i, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, _vp,
                                      _c_int64, _vp, _f, _f, _vp, _vp, _sz, _i, _vp, _vp]),
    "gptoss_ep_combine": (_i, [_vp, _c_int64, _vp, _vp, _c_int64, _i, _c_int64, _vp, _vp]),
    "gptoss_ipc_handle_bytes": (_i, []),
    "gptoss_ipc_alloc": (_i, [_sz, _vp, _vp]),
    "gptoss_ipc_open": (_i, [_vp, _vp]),
    "gptoss_ipc_close": (_i, [_vp]),
    "gptoss_ipc_free": (_i, [_vp]),
    "gptoss_ep_p2p_buffer_bytes": (_sz, [_i, _c_int64, _c_int64]),
    "gptoss_ep_p2p_dispatch": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _i, _i, _c_int64, _c_int64, _vp, _vp,
                                    _c_int32, _vp, _vp, _vp, _sz, _vp, _vp]),
    "gptoss_ep_p2p_route_dispatch": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _i, _i, _c_int64, _c_int64, _vp, _vp,
                                          _c_int32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "gptoss_ep_p2p_expert_forward": (_i, [_vp, _i, _i, _c_int64, _c_int32, _i, _c_int64, _c_int64, _vp, _vp,
                                          _c_int64, _vp, _vp, _vp, _c_int64, _vp, _f, _f, _vp, _vp, _vp, _sz, _i,
                                          _vp, _vp]),
    "gptoss_ep_p2p_combine": (_i, [_vp, _i, _c_int64, _c_int32, _vp, _vp, _c_int64, _i, _c_int64, _vp, _vp, _vp]),
    "gptoss_set_ep_layer_kernel": (_i, [_i]),
    "gptoss_ep_p2p_layer_fits": (_i, [_c_int64, _i, _i, _i, _c_int64, _c_int64, _c_int64]),
    "gptoss_ep_p2p_layer_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _c_int64, _i, _i, _i, _i, _c_int64, _c_int64,
                                         _vp, _vp, _c_int64, _vp, _vp, _vp, _c_int64, _vp, _f, _f, _c_int64, _vp,
                                         _vp, _c_int32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "gptoss_moe_route_quant": (_i, [_vp, _vp, _vp, _c_int64, _i, _i, _c_int64, _c_int64, _vp, _sz, _i, _vp, _vp]),
    "gptoss_moe_gemm1": (_i, [_c_int64, _i, _i, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _f, _f, _vp, _sz,
                              _i, _vp, _vp]),
    "gptoss_moe_gemm2": (_i, [_c_int64, _i, _i, _c_int64, _c_int64, _vp, _vp, _c_int64, _vp, _vp, _vp, _sz,
                              _i, _vp, _vp]),
}

ABI_VERSION = 2

_lock = threading.Lock()
_lib = None


class GptossError(RuntimeError):
    """Raised when a libgptoss_moe call returns a non-zero status."""


def lib_path() -> str:
    return os.environ.get("GPTOSS_MOE_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise GptossError(
                f"libgptoss_moe.so not found at {path}; build it with "
                "`python gpt-oss-mxfp4-compile_b200/build.py` (or __graft_entry__.build())")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.gptoss_abi_version()
        if ver != ABI_VERSION:
            raise GptossError(f"libgptoss_moe ABI {ver} != expected {ABI_VERSION}; rebuild the library")
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def call(name: str, *args) -> int:
    """Invoke an entry point and raise GptossError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.gptoss_last_error().decode(errors="replace")
        raise GptossError(f"{name} failed (status {rc}): {msg}")
    return rc


def query(name: str, *args):
    """Invoke a host-only query (sizes) and return its value."""
    return getattr(load(), name)(*args)
