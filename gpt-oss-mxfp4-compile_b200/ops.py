"""Tensor-level wrappers over the C ABI and their torch.library registrations.

Every function takes CUDA tensors, validates them the way the reference's CHECK_*
macros do (kernels/matmul_mxfp4_cutlass.cu:1107-1116: "must be a CUDA tensor", "must be
contiguous", dtype checks -> RuntimeError) and enqueues work on the current stream.
No function here computes anything on the host.

Registered ops (all with register_fake, static output shapes, no host sync unless noted):
  cutlass::fp4_group_mm        same schema as kernels/cutlass_experts.py:147-166
  cutlass::fused_moe_routing   same schema as kernels/cutlass_experts.py:168-188
  gptoss::quantize_fp8, gptoss::swiglu, gptoss::router_topk,
  gptoss::moe_experts_forward  (the whole CutlassGptOssExperts.forward)
  gptoss::moe_layer_forward    (router + experts)
  gptoss::route_quant, gptoss::gemm1, gptoss::gemm2   (its three stages on a workspace)
  gptoss::ep_dispatch, gptoss::ep_expert_forward, gptoss::ep_combine   (expert parallelism)
"""
from __future__ import annotations

import ctypes
import contextlib
import threading

import torch

from . import _lib

GEMM_AUTO, GEMM_TOKENS_M, GEMM_SWAP, GEMM_SWAP_WIDE = 0, 1, 2, 3
DTYPE_BF16, DTYPE_F32 = 0, 1

_status = {}
_status_lock = threading.Lock()


def _stream(dev: torch.device) -> int:
    """Raw handle of the current stream of `dev` (the fast path skips the Stream object)."""
    try:
        return torch._C._cuda_getCurrentRawStream(dev.index if dev.index is not None else torch.cuda.current_device())
    except AttributeError:
        return torch.cuda.current_stream(dev).cuda_stream


# Per (device, stream) scratch of the fused forwards, reused across calls: calls on one
# stream run in order on the GPU, so one buffer per stream is never used twice at once. A
# buffer outgrown by a larger call is kept alive, not freed: a CUDA graph captured earlier
# may still address it. During stream capture every call gets its own buffer from the
# graph's memory pool.
_ws_cache = {}
_ws_retired = []
_ws_bytes = {}


_tls = threading.local()


@contextlib.contextmanager
def _fresh_workspace():
    """Calls through the registered torch ops (traced and compiled code) take a fresh
    workspace from the caching allocator instead of the per-stream cache: under
    torch.compile(mode="reduce-overhead") the compiled model runs in CUDA-graph memory pools,
    and a workspace cached from such a run would keep that pool's memory alive."""
    prev = getattr(_tls, "fresh", False)
    _tls.fresh = True
    try:
        yield
    finally:
        _tls.fresh = prev


def _scratch(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    if torch.cuda.is_current_stream_capturing() or getattr(_tls, "fresh", False):
        return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    key = (dev.index, stream)
    t = _ws_cache.get(key)
    if t is None or t.numel() < nbytes:
        if t is not None:
            _ws_retired.append(t)
        t = torch.empty(max(nbytes, 256, 2 * t.numel() if t is not None else 0), dtype=torch.uint8, device=dev)
        _ws_cache[key] = t
    return t


def eager_call(t) -> bool:
    """True when an op can run its implementation directly (a plain CUDA tensor outside
    torch.compile tracing), skipping the dispatcher; fake, meta or traced tensors go
    through the registered torch.library op."""
    return type(t) is torch.Tensor and not torch.compiler.is_compiling()


def _p(t):
    return None if t is None else t.data_ptr()


def _cuda(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name}: must be a CUDA tensor.")
    if not t.is_contiguous():
        raise RuntimeError(f"{name}: must be contiguous.")


def _dtype(t: torch.Tensor, allowed, name: str):
    if t.dtype not in allowed:
        raise RuntimeError(f"{name}: Inconsistency of Tensor type: got {t.dtype}, expected one of {allowed}")


def status_tensor(device) -> torch.Tensor:
    """Per-device int32 word the kernels set on a timed-out wait or a bad index."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(key)
    if t is not None:
        return t
    with _status_lock:
        t = _status.get(key)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
            _status[key] = t
        return t


def set_decode_layer_kernel(enable: bool) -> bool:
    """Process-wide: decode-sized fused forwards as one persistent launch (True, the
    default) or as the three-launch path (False). Returns the previous setting."""
    return bool(_lib.query("gptoss_set_decode_layer_kernel", 1 if enable else 0))


def read_status(device) -> int:
    """Returns and clears the device status word (synchronises the current stream)."""
    t = status_tensor(device)
    out = ctypes.c_int32(0)
    _lib.call("gptoss_read_status", t.data_ptr(), ctypes.addressof(out), _stream(t.device))
    return int(out.value)


# ------------------------------------------------------------------ plain ops
def quantize_fp8(x: torch.Tensor):
    """BF16/FP32 [M, K] -> (float8_e4m3fn [M, K], uint8 UE8M0 [M, K/32]), bit-exact with
    quantize_activations_to_fp8 (kernels/cutlass_experts.py:197-251)."""
    if x.dim() != 2:
        raise RuntimeError(f"Expected 2D tensor, got {x.dim()}D")
    _cuda(x, "x")
    _dtype(x, (torch.bfloat16, torch.float32), "x")
    M, K = x.shape
    if K % 32 != 0:
        raise RuntimeError(f"K={K} must be divisible by 32")
    codes = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    scales = torch.empty((M, K // 32), dtype=torch.uint8, device=x.device)
    _lib.call("gptoss_quantize_fp8", x.data_ptr(), DTYPE_BF16 if x.dtype == torch.bfloat16 else DTYPE_F32,
              M, K, codes.data_ptr(), scales.data_ptr(), _stream(x.device))
    return codes, scales


def swiglu(gate_up: torch.Tensor, alpha: float = 1.702, limit: float = 7.0) -> torch.Tensor:
    """SwiGLU over interleaved gate (even) / up (odd) columns (cutlass_experts.py:258-276)."""
    _cuda(gate_up, "gate_up")
    _dtype(gate_up, (torch.bfloat16, torch.float32), "gate_up")
    if gate_up.shape[-1] % 2:
        raise RuntimeError("swiglu: last dimension must be even")
    rows = gate_up.numel() // gate_up.shape[-1]
    out = torch.empty((*gate_up.shape[:-1], gate_up.shape[-1] // 2), dtype=gate_up.dtype, device=gate_up.device)
    _lib.call("gptoss_swiglu", gate_up.data_ptr(), DTYPE_BF16 if gate_up.dtype == torch.bfloat16 else DTYPE_F32,
              rows, gate_up.shape[-1], out.data_ptr(), float(alpha), float(limit), _stream(gate_up.device))
    return out


def blocked_scales_bytes(rows: int, k: int) -> int:
    return int(_lib.query("gptoss_blocked_scales_bytes", rows, k))


def convert_scales_blocked(scales: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Row-major [rows, k/32] UE8M0 -> flat blocked buffer (convert_a/b_scales_for_w4a8,
    kernels/matmul_mxfp4_cutlass.cu:666-759), on the scales' device."""
    _cuda(scales, "scales")
    _dtype(scales, (torch.uint8,), "scales")
    if scales.numel() != rows * (k // 32):
        raise RuntimeError(f"scales has {scales.numel()} entries, expected rows*K/32 = {rows * (k // 32)}")
    nbytes = blocked_scales_bytes(rows, k)
    out = torch.empty(nbytes, dtype=torch.uint8, device=scales.device)
    if nbytes:
        _lib.call("gptoss_convert_scales_blocked", scales.data_ptr(), rows, k, out.data_ptr(), nbytes,
                  _stream(scales.device))
    return out


def batch_convert_a_scales(scales: torch.Tensor, counts: torch.Tensor, offsets: torch.Tensor, k: int,
                           exact_size: bool = True):
    """Per-expert blocked activation scales (batch_convert_a_scales_for_w4a8_gpu,
    kernels/matmul_mxfp4_cutlass.cu:912-1004). With exact_size=True the result is trimmed to
    the bytes actually used, which (like the reference) needs the counts on the host; with
    exact_size=False it returns the static-capacity buffer and never syncs."""
    _cuda(scales, "scales")
    _cuda(counts, "expert_counts")
    _cuda(offsets, "expert_offsets")
    _dtype(counts, (torch.int32,), "expert_counts")
    _dtype(offsets, (torch.int32,), "expert_offsets")
    E = counts.numel()
    rows = scales.shape[0] if scales.dim() else 0
    cap = int(_lib.query("gptoss_batch_blocked_scales_capacity", rows, E, k))
    out = torch.empty(max(cap, 1), dtype=torch.uint8, device=scales.device)
    sf_offsets = torch.empty(E, dtype=torch.int32, device=scales.device)
    _lib.call("gptoss_batch_convert_a_scales", scales.data_ptr(), counts.data_ptr(), offsets.data_ptr(), E, k,
              out.data_ptr(), cap, sf_offsets.data_ptr(), _stream(scales.device))
    if not exact_size:
        return out[:cap], sf_offsets
    c = counts.cpu().long()
    g4 = (k // 32 + 3) // 4
    total = int((((c + 127) // 128) * g4 * 512).sum())
    if total == 0:
        return torch.zeros(0, dtype=torch.uint8, device=scales.device), torch.zeros_like(sf_offsets)
    return out[:total], sf_offsets


def fused_moe_routing_impl(router_indices: torch.Tensor, routing_weights: torch.Tensor, num_experts: int):
    _cuda(router_indices, "router_indices")
    _cuda(routing_weights, "routing_weights")
    _dtype(router_indices, (torch.int64,), "router_indices")
    _dtype(routing_weights, (torch.float32,), "routing_weights")
    T, k = router_indices.shape
    dev = router_indices.device
    A = T * k
    st = torch.empty(A, dtype=torch.int64, device=dev)
    se = torch.empty(A, dtype=torch.int64, device=dev)
    sw = torch.empty(A, dtype=torch.float32, device=dev)
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts, dtype=torch.int32, device=dev)
    _lib.call("gptoss_fused_moe_routing", router_indices.data_ptr(), routing_weights.data_ptr(), T, k, num_experts,
              st.data_ptr(), se.data_ptr(), sw.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
              status_tensor(dev).data_ptr(), _stream(dev))
    return st, se, sw, counts, offsets


_FP4X2 = getattr(torch, "float4_e2m1fn_x2", None)
_SF_DTYPES = (torch.uint8, torch.float8_e4m3fn)


def fp4_group_mm_impl(output, a, b, a_blockscale, b_blockscales, alphas, problem_sizes, expert_offsets,
                      sf_offsets, gemm_mode: int = GEMM_AUTO):
    """Grouped GEMM into `output` (cutlass_fp4_group_mm, matmul_mxfp4_cutlass.cu:1118-1171).
    The dtype of `a` picks the mode as in the reference (:1157-1166): float8_e4m3fn [M, K]
    -> W4A8 (UE8M0 1x32 scales, sf_offsets in bytes); packed E2M1 bytes [M, K/2] (uint8) ->
    W4A4 / NVFP4 (UE4M3 1x16 scales, sf_offsets in rows). Scale tensors may be uint8 or
    float8_e4m3fn (their bytes are used either way)."""
    _cuda(a, "a")
    w4a4 = a.dtype == torch.uint8 or (_FP4X2 is not None and a.dtype == _FP4X2)
    if not w4a4:
        _dtype(a, (torch.float8_e4m3fn,), "a")
    _cuda(b, "b")
    _dtype(b, (torch.uint8,) + ((_FP4X2,) if _FP4X2 is not None else ()), "b")
    _cuda(a_blockscale, "a_blockscale")
    _dtype(a_blockscale, _SF_DTYPES, "a_blockscale")
    _cuda(b_blockscales, "b_blockscales")
    _dtype(b_blockscales, _SF_DTYPES, "b_blockscales")
    _cuda(alphas, "alphas")
    _dtype(alphas, (torch.float32,), "alphas")
    _cuda(output, "output")
    _dtype(output, (torch.bfloat16,), "output")
    for t, n in ((problem_sizes, "problem_sizes"), (expert_offsets, "expert_offsets"), (sf_offsets, "sf_offsets")):
        _cuda(t, n)
        _dtype(t, (torch.int32,), n)
    if b.dim() != 3:
        raise RuntimeError("b must be [E, N, K/2]")
    if b_blockscales.dim() not in (2, 3):
        raise RuntimeError("Invalid b_blockscales dim (expected 2D [E, converted_size] or 3D [E, N, K_groups])")
    if problem_sizes.dim() != 2:
        raise RuntimeError("problem_sizes must be 2D")
    E, N, K = b.shape[0], b.shape[1], 2 * b.shape[2]
    M = a.shape[0]
    if output.shape[0] < M or output.shape[1] != N:
        raise RuntimeError(f"output must be [M={M}, N={N}], got {tuple(output.shape)}")
    ldb = b_blockscales.numel() // E
    fn = "gptoss_fp4_group_mm_w4a4" if w4a4 else "gptoss_fp4_group_mm"
    _lib.call(fn, output.data_ptr(), a.data_ptr(), M, a.shape[1], b.data_ptr(), E, N, K,
              a_blockscale.data_ptr(), b_blockscales.data_ptr(), ldb, alphas.data_ptr(), problem_sizes.data_ptr(),
              expert_offsets.data_ptr(), sf_offsets.data_ptr(), int(gemm_mode), status_tensor(a.device).data_ptr(),
              _stream(a.device))


def mma_peak(device, pair: bool = True, n: int = 256, iters: int = 4000, repeats: int = 5,
             kind: str = "mxf8f6f4") -> dict:
    """Measured dense throughput (TFLOP/s, best of `repeats`) of a block-scaled MMA
    (gptoss_mma_peak): kind "mxf8f6f4" (FP8 x FP4, the W4A8 GEMMs) or "mxf4nvf4" (NVFP4 x
    NVFP4, the W4A4 mode); CTA pairs (M = 256) or single CTAs (M = 128), N = n."""
    kinds = {"mxf8f6f4": (0, 128), "mxf4nvf4": (1, 256)}
    if kind not in kinds:
        raise ValueError(f"kind must be one of {sorted(kinds)}")
    code, kb = kinds[kind]
    dev = torch.device(device)
    st = _stream(dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    units, M = (sms // 2, 256) if pair else (sms, 128)
    flops = float(units) * iters * 2 * M * n * kb
    best = 0.0
    _lib.call("gptoss_mma_peak", code, int(pair), int(n), 16, status_tensor(dev).data_ptr(), st)   # warm-up
    for _ in range(repeats):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _lib.call("gptoss_mma_peak", code, int(pair), int(n), int(iters), status_tensor(dev).data_ptr(), st)
        b.record()
        b.synchronize()
        best = max(best, flops / (a.elapsed_time(b) / 1e3) / 1e12)
    if read_status(dev) != 0:
        raise RuntimeError("mma_peak: a bounded wait gave up")
    return {"tflops": best, "kind": kind, "pair": bool(pair), "M": M, "N": n, "k_blocks": iters, "units": units}


def router_topk_from_logits(logits: torch.Tensor, top_k: int):
    """Top-k + softmax on given bf16 logits [T, E] (the router's second half) ->
    (scores bf16 [T, k], indices int64 [T, k])."""
    _cuda(logits, "logits")
    _dtype(logits, (torch.bfloat16,), "logits")
    logits = logits.contiguous()
    T, E = logits.shape
    idx = torch.empty((T, top_k), dtype=torch.int64, device=logits.device)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=logits.device)
    _lib.call("gptoss_router_topk_from_logits", logits.data_ptr(), T, E, int(top_k), idx.data_ptr(),
              scores.data_ptr(), None, _stream(logits.device))
    return scores, idx


def router_topk_impl(hidden, weight, bias, top_k: int):
    _cuda(hidden, "hidden_states")
    _cuda(weight, "router weight")
    _cuda(bias, "router bias")
    for t, n in ((hidden, "hidden_states"), (weight, "router weight"), (bias, "router bias")):
        _dtype(t, (torch.bfloat16,), n)
    T, H = hidden.shape
    E = weight.shape[0]
    dev = hidden.device
    idx = torch.empty((T, top_k), dtype=torch.int64, device=dev)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
    logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    _lib.call("gptoss_router_topk", hidden.data_ptr(), weight.data_ptr(), bias.data_ptr(), T, H, E, top_k,
              idx.data_ptr(), scores.data_ptr(), None, logits.data_ptr(), _stream(dev))
    return logits, scores, idx


def workspace_bytes(T, k, E, H, I) -> int:
    key = (T, k, E, H, I)
    n = _ws_bytes.get(key)
    if n is None:
        n = int(_lib.query("gptoss_moe_workspace_bytes", T, k, E, H, I))
        _ws_bytes[key] = n
    return n


def _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias):
    for t, n in ((gu_data, "gate_up_proj_data"), (gu_scales, "gate_up_proj_scales"),
                 (dn_data, "down_proj_data"), (dn_scales, "down_proj_scales")):
        _cuda(t, n)
        _dtype(t, (torch.uint8,), n)
    for t, n in ((gu_bias, "gate_up_proj_bias"), (dn_bias, "down_proj_bias")):
        _cuda(t, n)
        _dtype(t, (torch.float32,), n)


def moe_experts_forward_impl(hidden, router_indices, routing_weights, gu_data, gu_scales, gu_bias, dn_data,
                             dn_scales, dn_bias, alpha: float, limit: float, gemm_mode: int = GEMM_AUTO):
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(router_indices, "router_indices")
    _dtype(router_indices, (torch.int64,), "router_indices")
    _cuda(routing_weights, "routing_weights")
    _dtype(routing_weights, (torch.float32,), "routing_weights")
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    T, H = hidden.shape
    k = router_indices.shape[1]
    E = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    dev = hidden.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    st = _stream(dev)
    ws = _scratch(dev, st, workspace_bytes(T, k, E, H, I))
    _lib.call("gptoss_moe_experts_forward", hidden.data_ptr(), router_indices.data_ptr(), routing_weights.data_ptr(),
              T, k, E, H, I, gu_data.data_ptr(), gu_scales.data_ptr(), gu_scales.numel() // E, gu_bias.data_ptr(),
              dn_data.data_ptr(), dn_scales.data_ptr(), dn_scales.numel() // E, dn_bias.data_ptr(), float(alpha),
              float(limit), out.data_ptr(), ws.data_ptr(), ws.numel(), int(gemm_mode),
              status_tensor(dev).data_ptr(), st)
    return out


def moe_layer_forward_impl(hidden, router_weight, router_bias, top_k: int, gu_data, gu_scales, gu_bias, dn_data,
                           dn_scales, dn_bias, alpha: float, limit: float, gemm_mode: int = GEMM_AUTO):
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(router_weight, "router weight")
    _cuda(router_bias, "router bias")
    _dtype(router_weight, (torch.bfloat16,), "router weight")
    _dtype(router_bias, (torch.bfloat16,), "router bias")
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    T, H = hidden.shape
    E = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    dev = hidden.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=dev)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
    st = _stream(dev)
    ws = _scratch(dev, st, workspace_bytes(T, top_k, E, H, I))
    _lib.call("gptoss_moe_layer_forward", hidden.data_ptr(), router_weight.data_ptr(), router_bias.data_ptr(), T,
              top_k, E, H, I, gu_data.data_ptr(), gu_scales.data_ptr(), gu_scales.numel() // E, gu_bias.data_ptr(),
              dn_data.data_ptr(), dn_scales.data_ptr(), dn_scales.numel() // E, dn_bias.data_ptr(), float(alpha),
              float(limit), out.data_ptr(), idx.data_ptr(), scores.data_ptr(), ws.data_ptr(), ws.numel(),
              int(gemm_mode), status_tensor(dev).data_ptr(), st)
    return out, scores, idx


def moe_block_forward_impl(hidden, norm_weight, norm_eps: float, router_weight, router_bias, top_k: int, gu_data,
                           gu_scales, gu_bias, dn_data, dn_scales, dn_bias, alpha: float, limit: float,
                           gemm_mode: int = GEMM_AUTO):
    """hidden + layer(RMSNorm(hidden)) (gptoss_moe_block_forward) -> (out, scores, indices)."""
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(norm_weight, "norm weight")
    _dtype(norm_weight, (torch.bfloat16,), "norm weight")
    _cuda(router_weight, "router weight")
    _dtype(router_weight, (torch.bfloat16,), "router weight")
    _dtype(router_bias, (torch.bfloat16,), "router bias")
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    T, H = hidden.shape
    E = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    dev = hidden.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=dev)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
    st = _stream(dev)
    ws = _scratch(dev, st, int(_lib.query("gptoss_moe_block_workspace_bytes", T, top_k, E, H, I)))
    _lib.call("gptoss_moe_block_forward", hidden.data_ptr(), norm_weight.data_ptr(), float(norm_eps),
              router_weight.data_ptr(), router_bias.data_ptr(), T, top_k, E, H, I, gu_data.data_ptr(),
              gu_scales.data_ptr(), gu_scales.numel() // E, gu_bias.data_ptr(), dn_data.data_ptr(),
              dn_scales.data_ptr(), dn_scales.numel() // E, dn_bias.data_ptr(), float(alpha), float(limit),
              out.data_ptr(), idx.data_ptr(), scores.data_ptr(), ws.data_ptr(), ws.numel(), int(gemm_mode),
              status_tensor(dev).data_ptr(), st)
    return out, scores, idx


def rmsnorm_residual(x, weight, eps: float):
    """(RMSNorm(x) bf16, copy of x) from one kernel (gptoss_rmsnorm_residual)."""
    _cuda(x, "x")
    _dtype(x, (torch.bfloat16,), "x")
    T, H = x.shape
    xn = torch.empty_like(x)
    res = torch.empty_like(x)
    _lib.call("gptoss_rmsnorm_residual", x.data_ptr(), weight.data_ptr(), float(eps), T, H, xn.data_ptr(),
              res.data_ptr(), _stream(x.device))
    return xn, res


# ------------------------------------------------------------------ registration
_registered = False
_reg_lock = threading.Lock()


def register_ops() -> None:
    """Register every op with torch.library (idempotent)."""
    global _registered
    if _registered:
        return
    with _reg_lock:
        if _registered:
            return
        _lib.load()   # fail loudly before anything is registered

        @torch.library.custom_op("cutlass::fp4_group_mm", mutates_args=("output",))
        def fp4_group_mm(output: torch.Tensor, a: torch.Tensor, b: torch.Tensor, a_blockscale: torch.Tensor,
                         b_blockscales: torch.Tensor, alphas: torch.Tensor, problem_sizes: torch.Tensor,
                         expert_offsets: torch.Tensor, sf_offsets: torch.Tensor) -> None:
            fp4_group_mm_impl(output, a, b, a_blockscale, b_blockscales, alphas, problem_sizes, expert_offsets,
                              sf_offsets)

        @fp4_group_mm.register_fake
        def _(output, a, b, a_blockscale, b_blockscales, alphas, problem_sizes, expert_offsets, sf_offsets):
            return None

        @torch.library.custom_op("cutlass::fused_moe_routing", mutates_args=())
        def fused_moe_routing(router_indices: torch.Tensor, routing_weights: torch.Tensor, num_experts: int
                              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
            return fused_moe_routing_impl(router_indices, routing_weights, num_experts)

        @fused_moe_routing.register_fake
        def _(router_indices, routing_weights, num_experts):
            total = router_indices.shape[0] * router_indices.shape[1]
            dev = router_indices.device
            return (torch.empty(total, dtype=torch.int64, device=dev),
                    torch.empty(total, dtype=torch.int64, device=dev),
                    torch.empty(total, dtype=torch.float32, device=dev),
                    torch.empty(num_experts, dtype=torch.int32, device=dev),
                    torch.empty(num_experts, dtype=torch.int32, device=dev))

        @torch.library.custom_op("gptoss::quantize_fp8", mutates_args=())
        def quantize_fp8_op(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
            return quantize_fp8(x)

        @quantize_fp8_op.register_fake
        def _(x):
            M, K = x.shape
            return (torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device),
                    torch.empty((M, K // 32), dtype=torch.uint8, device=x.device))

        @torch.library.custom_op("gptoss::swiglu", mutates_args=())
        def swiglu_op(gate_up: torch.Tensor, alpha: float, limit: float) -> torch.Tensor:
            return swiglu(gate_up, alpha, limit)

        @swiglu_op.register_fake
        def _(gate_up, alpha, limit):
            return gate_up.new_empty((*gate_up.shape[:-1], gate_up.shape[-1] // 2))

        @torch.library.custom_op("gptoss::router_topk", mutates_args=())
        def router_topk_op(hidden: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, top_k: int
                           ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
            return router_topk_impl(hidden, weight, bias, top_k)

        @router_topk_op.register_fake
        def _(hidden, weight, bias, top_k):
            T = hidden.shape[0]
            return (hidden.new_empty((T, weight.shape[0])), hidden.new_empty((T, top_k)),
                    torch.empty((T, top_k), dtype=torch.int64, device=hidden.device))

        @torch.library.custom_op("gptoss::moe_experts_forward", mutates_args=())
        def moe_experts_forward(hidden: torch.Tensor, router_indices: torch.Tensor, routing_weights: torch.Tensor,
                                gate_up_data: torch.Tensor, gate_up_scales: torch.Tensor, gate_up_bias: torch.Tensor,
                                down_data: torch.Tensor, down_scales: torch.Tensor, down_bias: torch.Tensor,
                                alpha: float, limit: float, gemm_mode: int) -> torch.Tensor:
            with _fresh_workspace():
                return moe_experts_forward_impl(hidden, router_indices, routing_weights, gate_up_data, gate_up_scales,
                                                gate_up_bias, down_data, down_scales, down_bias, alpha, limit, gemm_mode)

        @moe_experts_forward.register_fake
        def _(hidden, router_indices, routing_weights, gate_up_data, gate_up_scales, gate_up_bias, down_data,
              down_scales, down_bias, alpha, limit, gemm_mode):
            return torch.empty_like(hidden)

        @torch.library.custom_op("gptoss::moe_layer_forward", mutates_args=())
        def moe_layer_forward(hidden: torch.Tensor, router_weight: torch.Tensor, router_bias: torch.Tensor,
                              top_k: int, gate_up_data: torch.Tensor, gate_up_scales: torch.Tensor,
                              gate_up_bias: torch.Tensor, down_data: torch.Tensor, down_scales: torch.Tensor,
                              down_bias: torch.Tensor, alpha: float, limit: float, gemm_mode: int
                              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
            with _fresh_workspace():
                return moe_layer_forward_impl(hidden, router_weight, router_bias, top_k, gate_up_data, gate_up_scales,
                                              gate_up_bias, down_data, down_scales, down_bias, alpha, limit, gemm_mode)

        @moe_layer_forward.register_fake
        def _(hidden, router_weight, router_bias, top_k, gate_up_data, gate_up_scales, gate_up_bias, down_data,
              down_scales, down_bias, alpha, limit, gemm_mode):
            T = hidden.shape[0]
            return (torch.empty_like(hidden), hidden.new_empty((T, top_k)),
                    torch.empty((T, top_k), dtype=torch.int64, device=hidden.device))

        @torch.library.custom_op("gptoss::moe_block_forward", mutates_args=())
        def moe_block_forward(hidden: torch.Tensor, norm_weight: torch.Tensor, norm_eps: float,
                              router_weight: torch.Tensor, router_bias: torch.Tensor, top_k: int,
                              gate_up_data: torch.Tensor, gate_up_scales: torch.Tensor, gate_up_bias: torch.Tensor,
                              down_data: torch.Tensor, down_scales: torch.Tensor, down_bias: torch.Tensor,
                              alpha: float, limit: float, gemm_mode: int
                              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
            with _fresh_workspace():
                return moe_block_forward_impl(hidden, norm_weight, norm_eps, router_weight, router_bias, top_k,
                                              gate_up_data, gate_up_scales, gate_up_bias, down_data, down_scales,
                                              down_bias, alpha, limit, gemm_mode)

        @moe_block_forward.register_fake
        def _(hidden, norm_weight, norm_eps, router_weight, router_bias, top_k, gate_up_data, gate_up_scales,
              gate_up_bias, down_data, down_scales, down_bias, alpha, limit, gemm_mode):
            T = hidden.shape[0]
            return (torch.empty_like(hidden), hidden.new_empty((T, top_k)),
                    torch.empty((T, top_k), dtype=torch.int64, device=hidden.device))

        # the staged forward on a caller-owned workspace (the three fused stages)
        @torch.library.custom_op("gptoss::route_quant", mutates_args=("workspace",))
        def route_quant_op(workspace: torch.Tensor, hidden: torch.Tensor, router_indices: torch.Tensor,
                           routing_weights: torch.Tensor, num_experts: int, intermediate_size: int,
                           gemm_mode: int) -> None:
            route_quant_ws(workspace, hidden, router_indices, routing_weights, num_experts, intermediate_size,
                           gemm_mode)

        @route_quant_op.register_fake
        def _(workspace, hidden, router_indices, routing_weights, num_experts, intermediate_size, gemm_mode):
            return None

        @torch.library.custom_op("gptoss::gemm1", mutates_args=("workspace",))
        def gemm1_op(workspace: torch.Tensor, num_tokens: int, top_k: int, num_experts: int, hidden_size: int,
                     intermediate_size: int, gate_up_data: torch.Tensor, gate_up_scales: torch.Tensor,
                     gate_up_bias: torch.Tensor, alpha: float, limit: float, gemm_mode: int) -> None:
            gemm1_ws(workspace, num_tokens, top_k, num_experts, hidden_size, intermediate_size, gate_up_data,
                     gate_up_scales, gate_up_bias, alpha, limit, gemm_mode)

        @gemm1_op.register_fake
        def _(workspace, num_tokens, top_k, num_experts, hidden_size, intermediate_size, gate_up_data,
              gate_up_scales, gate_up_bias, alpha, limit, gemm_mode):
            return None

        @torch.library.custom_op("gptoss::gemm2", mutates_args=("workspace", "out"))
        def gemm2_op(workspace: torch.Tensor, out: torch.Tensor, num_tokens: int, top_k: int, num_experts: int,
                     hidden_size: int, intermediate_size: int, down_data: torch.Tensor, down_scales: torch.Tensor,
                     down_bias: torch.Tensor, gemm_mode: int) -> None:
            gemm2_ws(workspace, out, num_tokens, top_k, num_experts, hidden_size, intermediate_size, down_data,
                     down_scales, down_bias, gemm_mode)

        @gemm2_op.register_fake
        def _(workspace, out, num_tokens, top_k, num_experts, hidden_size, intermediate_size, down_data,
              down_scales, down_bias, gemm_mode):
            return None

        # expert parallelism: dispatch / local experts / combine around the caller's exchange
        @torch.library.custom_op("gptoss::ep_dispatch", mutates_args=())
        def ep_dispatch_op(hidden: torch.Tensor, router_indices: torch.Tensor, routing_weights: torch.Tensor,
                           num_experts: int, world_size: int, capacity: int
                           ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
            return ep_dispatch(hidden, router_indices, routing_weights, num_experts, world_size, capacity)

        @ep_dispatch_op.register_fake
        def _(hidden, router_indices, routing_weights, num_experts, world_size, capacity):
            A = router_indices.shape[0] * router_indices.shape[1]
            dev = hidden.device
            return (torch.empty((world_size * capacity if capacity else A, ep_row_bytes(hidden.shape[1])),
                                dtype=torch.uint8, device=dev),
                    torch.empty(world_size, dtype=torch.int32, device=dev),
                    torch.empty(A, dtype=torch.int32, device=dev))

        @torch.library.custom_op("gptoss::ep_expert_forward", mutates_args=())
        def ep_expert_forward_op(recv_rows: torch.Tensor, gate_up_data: torch.Tensor, gate_up_scales: torch.Tensor,
                                 gate_up_bias: torch.Tensor, down_data: torch.Tensor, down_scales: torch.Tensor,
                                 down_bias: torch.Tensor, alpha: float, limit: float, gemm_mode: int
                                 ) -> torch.Tensor:
            return ep_expert_forward(recv_rows, gate_up_data, gate_up_scales, gate_up_bias, down_data, down_scales,
                                     down_bias, alpha, limit, gemm_mode)

        @ep_expert_forward_op.register_fake
        def _(recv_rows, gate_up_data, gate_up_scales, gate_up_bias, down_data, down_scales, down_bias, alpha,
              limit, gemm_mode):
            return torch.empty((recv_rows.shape[0], down_data.shape[1]), dtype=torch.bfloat16,
                               device=recv_rows.device)

        @torch.library.custom_op("gptoss::ep_combine", mutates_args=())
        def ep_combine_op(back_rows: torch.Tensor, pos_of: torch.Tensor, router_indices: torch.Tensor
                          ) -> torch.Tensor:
            return ep_combine(back_rows, pos_of, router_indices)

        @ep_combine_op.register_fake
        def _(back_rows, pos_of, router_indices):
            return torch.empty((router_indices.shape[0], back_rows.shape[1]), dtype=torch.bfloat16,
                               device=back_rows.device)

        _registered = True


# ------------------------------------------------------------------ staged forward
WS_REGIONS = ("sorted_token", "sorted_expert", "sorted_weight", "counts", "offsets", "act_sf_offsets",
              "inter_sf_offsets", "act_codes", "act_scales", "inter_codes", "inter_scales", "router_idx",
              "router_weights", "total")


class ExpertsWorkspace:
    """Device workspace of the staged expert forward (route_quant -> gemm1 -> gemm2) with
    typed views of its regions; the layout comes from gptoss_moe_workspace_layout."""

    def __init__(self, T: int, k: int, E: int, H: int, I: int, device):
        self.T, self.k, self.E, self.H, self.I = T, k, E, H, I
        offs = (ctypes.c_int64 * len(WS_REGIONS))()
        _lib.call("gptoss_moe_workspace_layout", T, k, E, H, I, ctypes.addressof(offs))
        self.offsets = dict(zip(WS_REGIONS, list(offs)))
        self.nbytes = int(self.offsets["total"])
        self.buf = torch.empty(max(self.nbytes, 256), dtype=torch.uint8, device=device)
        A = T * k
        o = self.offsets

        def view(name, dtype, n):
            nb = n * torch.empty((), dtype=dtype).element_size()
            return self.buf[o[name]:o[name] + nb].view(dtype)

        self.sorted_token = view("sorted_token", torch.int64, A)
        self.sorted_expert = view("sorted_expert", torch.int64, A)
        self.sorted_weight = view("sorted_weight", torch.float32, A)
        self.counts = view("counts", torch.int32, E)
        self.expert_offsets = view("offsets", torch.int32, E)
        self.act_sf_offsets = view("act_sf_offsets", torch.int32, E)
        self.inter_sf_offsets = view("inter_sf_offsets", torch.int32, E)
        self.act_codes = view("act_codes", torch.uint8, A * H).view(A, H)
        self.act_scales = self.buf[o["act_scales"]:o["inter_codes"]]
        self.inter_codes = view("inter_codes", torch.uint8, A * I).view(A, I)
        self.inter_scales = self.buf[o["inter_scales"]:o["router_idx"]]

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()


def route_quant(ws: ExpertsWorkspace, hidden, router_indices, routing_weights, gemm_mode: int = GEMM_AUTO):
    if tuple(router_indices.shape) != (ws.T, ws.k) or tuple(hidden.shape) != (ws.T, ws.H):
        raise RuntimeError("route_quant: inputs do not match the workspace's (T, k, H)")
    route_quant_ws(ws.buf, hidden, router_indices, routing_weights, ws.E, ws.I, gemm_mode)


def gemm1(ws: ExpertsWorkspace, gu_data, gu_scales, gu_bias, alpha: float = 1.702, limit: float = 7.0,
          gemm_mode: int = GEMM_AUTO):
    gemm1_ws(ws.buf, ws.T, ws.k, ws.E, ws.H, ws.I, gu_data, gu_scales, gu_bias, alpha, limit, gemm_mode)


def gemm2(ws: ExpertsWorkspace, dn_data, dn_scales, dn_bias, out, gemm_mode: int = GEMM_AUTO):
    gemm2_ws(ws.buf, out, ws.T, ws.k, ws.E, ws.H, ws.I, dn_data, dn_scales, dn_bias, gemm_mode)


def route_quant_ws(workspace, hidden, router_indices, routing_weights, num_experts: int, intermediate_size: int,
                   gemm_mode: int = GEMM_AUTO):
    """route_quant on a raw workspace tensor (u8, at least workspace_bytes(T, k, E, H, I))."""
    _cuda(workspace, "workspace")
    _cuda(hidden, "hidden_states")
    T, H = hidden.shape
    k = router_indices.shape[1]
    _lib.call("gptoss_moe_route_quant", hidden.data_ptr(), router_indices.data_ptr(), routing_weights.data_ptr(),
              T, k, int(num_experts), H, int(intermediate_size), workspace.data_ptr(), workspace.numel(),
              int(gemm_mode), status_tensor(hidden.device).data_ptr(), _stream(hidden.device))


def gemm1_ws(workspace, T: int, k: int, E: int, H: int, I: int, gu_data, gu_scales, gu_bias, alpha: float = 1.702,
             limit: float = 7.0, gemm_mode: int = GEMM_AUTO):
    """gemm1 on a raw workspace tensor."""
    _cuda(workspace, "workspace")
    _lib.call("gptoss_moe_gemm1", T, k, E, H, I, gu_data.data_ptr(), gu_scales.data_ptr(), gu_scales.numel() // E,
              gu_bias.data_ptr(), float(alpha), float(limit), workspace.data_ptr(), workspace.numel(),
              int(gemm_mode), status_tensor(gu_data.device).data_ptr(), _stream(gu_data.device))


def gemm2_ws(workspace, out, T: int, k: int, E: int, H: int, I: int, dn_data, dn_scales, dn_bias,
             gemm_mode: int = GEMM_AUTO):
    """gemm2 on a raw workspace tensor; adds into `out` [T, H] bf16."""
    _cuda(workspace, "workspace")
    _cuda(out, "out")
    _lib.call("gptoss_moe_gemm2", T, k, E, H, I, dn_data.data_ptr(), dn_scales.data_ptr(), dn_scales.numel() // E,
              dn_bias.data_ptr(), out.data_ptr(), workspace.data_ptr(), workspace.numel(), int(gemm_mode),
              status_tensor(dn_data.device).data_ptr(), _stream(dn_data.device))


# ------------------------------------------------------------------ expert parallelism
def ep_row_bytes(hidden_size: int) -> int:
    """Bytes of one dispatched row: FP8 codes, UE8M0 scales, padding, int32 local expert,
    f32 routing weight (16-byte multiple)."""
    rb = int(_lib.query("gptoss_ep_row_bytes", int(hidden_size)))
    if rb <= 0:
        raise RuntimeError(f"ep_row_bytes: hidden size {hidden_size} must be a positive multiple of 32")
    return rb


def ep_dispatch(hidden, router_indices, routing_weights, num_experts: int, world_size: int, capacity: int = 0):
    """Sorts the T*k assignments by destination rank (experts [r*E/W, (r+1)*E/W) live on
    rank r) and quantises each assignment's hidden row into a packed send row.
    Returns (send_rows u8 [rows, row_bytes], send_counts i32 [W], pos_of i32 [T*k]) with
    rows = T*k (capacity 0: compact) or W*capacity (fixed segments, empty rows marked)."""
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(router_indices, "router_indices")
    _dtype(router_indices, (torch.int64,), "router_indices")
    _cuda(routing_weights, "routing_weights")
    _dtype(routing_weights, (torch.float32,), "routing_weights")
    T, H = hidden.shape
    k = router_indices.shape[1]
    dev = hidden.device
    A = T * k
    if capacity and capacity < A:
        raise RuntimeError(f"ep_dispatch: capacity {capacity} < T*k = {A}")
    send_rows = torch.empty((world_size * capacity if capacity else A, ep_row_bytes(H)), dtype=torch.uint8,
                            device=dev)
    send_counts = torch.empty(world_size, dtype=torch.int32, device=dev)
    pos_of = torch.empty(A, dtype=torch.int32, device=dev)
    nbytes = int(_lib.query("gptoss_ep_dispatch_workspace_bytes", T, k, world_size))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    _lib.call("gptoss_ep_dispatch", hidden.data_ptr(), router_indices.data_ptr(), routing_weights.data_ptr(), T, k,
              int(num_experts), int(world_size), H, int(capacity), send_rows.data_ptr(), send_counts.data_ptr(),
              pos_of.data_ptr(),
              ws.data_ptr(), ws.numel(), status_tensor(dev).data_ptr(), _stream(dev))
    return send_rows, send_counts, pos_of


def ep_expert_forward(recv_rows, gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias, alpha: float = 1.702,
                      limit: float = 7.0, gemm_mode: int = GEMM_AUTO):
    """Received rows [R, row_bytes] -> routing-weighted expert outputs [R, H] bf16 on this
    rank's local experts (the weights' leading dimension)."""
    _cuda(recv_rows, "recv_rows")
    _dtype(recv_rows, (torch.uint8,), "recv_rows")
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    E_loc = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    H = dn_data.shape[1]
    R = recv_rows.shape[0]
    if recv_rows.dim() != 2 or (R and recv_rows.shape[1] != ep_row_bytes(H)):
        raise RuntimeError(f"recv_rows: expected [R, {ep_row_bytes(H)}], got {tuple(recv_rows.shape)}")
    dev = gu_data.device
    back = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
    ws = torch.empty(max(workspace_bytes(R, 1, E_loc, H, I) if R else 0, 256), dtype=torch.uint8, device=dev)
    _lib.call("gptoss_ep_expert_forward", recv_rows.data_ptr() if R else None, R, E_loc, H, I, gu_data.data_ptr(),
              gu_scales.data_ptr(), gu_scales.numel() // E_loc, gu_bias.data_ptr(), dn_data.data_ptr(),
              dn_scales.data_ptr(), dn_scales.numel() // E_loc, dn_bias.data_ptr(), float(alpha), float(limit),
              back.data_ptr() if R else None, ws.data_ptr(), ws.numel(), int(gemm_mode),
              status_tensor(dev).data_ptr(), _stream(dev))
    return back


def ep_combine(back_rows, pos_of, router_indices):
    """Returned rows [T*k, H] -> out [T, H]: each token's k rows summed in fp32 in
    ascending expert order, rounded to bf16 once."""
    _cuda(back_rows, "back_rows")
    _dtype(back_rows, (torch.bfloat16,), "back_rows")
    _cuda(pos_of, "pos_of")
    _cuda(router_indices, "router_indices")
    T, k = router_indices.shape
    H = back_rows.shape[1]
    dev = back_rows.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    if T == 0:
        return out
    _lib.call("gptoss_ep_combine", back_rows.data_ptr(), back_rows.shape[0], pos_of.data_ptr(),
              router_indices.data_ptr(), T, k, H, out.data_ptr(), _stream(dev))
    return out


# ------------------------------------------------------------------ peer-memory expert parallelism
def ipc_alloc(nbytes: int):
    """Zeroed device buffer of the current device plus its IPC handle -> (address, handle bytes)."""
    hb = int(_lib.query("gptoss_ipc_handle_bytes"))
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * hb)()
    _lib.call("gptoss_ipc_alloc", int(nbytes), ctypes.byref(ptr), handle)
    return int(ptr.value), bytes(handle)


def ipc_open(handle: bytes) -> int:
    buf = (ctypes.c_uint8 * len(handle)).from_buffer_copy(handle)
    ptr = ctypes.c_void_p()
    _lib.call("gptoss_ipc_open", buf, ctypes.byref(ptr))
    return int(ptr.value)


def ipc_close(ptr: int):
    _lib.call("gptoss_ipc_close", ptr)


def ipc_free(ptr: int):
    _lib.call("gptoss_ipc_free", ptr)


def ep_p2p_buffer_bytes(world_size: int, capacity: int, hidden_size: int) -> int:
    return int(_lib.query("gptoss_ep_p2p_buffer_bytes", int(world_size), int(capacity), int(hidden_size)))


def ep_p2p_route_dispatch(hidden, router_weight, router_bias, top_k: int, world_size: int, rank: int,
                          capacity: int, local_base: int, peer_bases, epoch: int):
    """Router + dispatch in one call (one launch at decode sizes). Returns
    (scores bf16 [T, k], router_indices i64 [T, k], send_counts i32 [W], pos_of i32 [T*k])."""
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(router_weight, "router weight")
    _dtype(router_weight, (torch.bfloat16,), "router weight")
    _dtype(router_bias, (torch.bfloat16,), "router bias")
    T, H = hidden.shape
    E = router_weight.shape[0]
    dev = hidden.device
    idx = torch.empty((T, top_k), dtype=torch.int64, device=dev)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
    wf = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    send_counts = torch.empty(world_size, dtype=torch.int32, device=dev)
    pos_of = torch.empty(T * top_k, dtype=torch.int32, device=dev)
    st = _stream(dev)
    ws = _scratch(dev, st, int(_lib.query("gptoss_ep_dispatch_workspace_bytes", T, top_k, world_size)))
    _lib.call("gptoss_ep_p2p_route_dispatch", _p(hidden) if T else None, router_weight.data_ptr(),
              router_bias.data_ptr(), T, int(top_k), int(E), int(world_size), int(rank), H, int(capacity),
              int(local_base), peer_bases.data_ptr(), int(epoch), idx.data_ptr() if T else None,
              scores.data_ptr() if T else None, wf.data_ptr() if T else None, send_counts.data_ptr(),
              pos_of.data_ptr() if T else None, ws.data_ptr(), ws.numel(), status_tensor(dev).data_ptr(), st)
    return scores, idx, send_counts, pos_of


def ep_p2p_dispatch(hidden, router_indices, routing_weights, num_experts: int, world_size: int, rank: int,
                    capacity: int, local_base: int, peer_bases, epoch: int):
    """Quantised rows straight into the owners' receive rows + dispatch flags.
    Returns (send_counts i32 [W], pos_of i32 [T*k])."""
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _cuda(router_indices, "router_indices")
    _dtype(router_indices, (torch.int64,), "router_indices")
    _cuda(routing_weights, "routing_weights")
    _dtype(routing_weights, (torch.float32,), "routing_weights")
    T, H = hidden.shape
    k = router_indices.shape[1]
    dev = hidden.device
    send_counts = torch.empty(world_size, dtype=torch.int32, device=dev)
    pos_of = torch.empty(T * k, dtype=torch.int32, device=dev)
    nbytes = int(_lib.query("gptoss_ep_dispatch_workspace_bytes", T, k, world_size))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    _lib.call("gptoss_ep_p2p_dispatch", _p(hidden) if T else None, _p(router_indices) if T else None,
              _p(routing_weights) if T else None, T, k, int(num_experts), int(world_size), int(rank), H,
              int(capacity), int(local_base), peer_bases.data_ptr(), int(epoch), send_counts.data_ptr(),
              pos_of.data_ptr() if T else None, ws.data_ptr(), ws.numel(), status_tensor(dev).data_ptr(),
              _stream(dev))
    return send_counts, pos_of


def ep_p2p_expert_forward(local_base: int, world_size: int, rank: int, capacity: int, epoch: int, gu_data,
                          gu_scales, gu_bias, dn_data, dn_scales, dn_bias, back_rows, workspace, peer_bases,
                          alpha: float = 1.702, limit: float = 7.0, gemm_mode: int = GEMM_AUTO):
    """Local experts on this rank's receive rows; outputs stored into the source ranks'
    return rows + return flags. `back_rows` [W*cap, H] bf16 and `workspace` (u8, at least
    workspace_bytes(W*cap, 1, E/W, H, I)) are this rank's scratch."""
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    E_loc = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    H = dn_data.shape[1]
    dev = gu_data.device
    _lib.call("gptoss_ep_p2p_expert_forward", int(local_base), int(world_size), int(rank), int(capacity), int(epoch),
              E_loc, H, I, gu_data.data_ptr(), gu_scales.data_ptr(), gu_scales.numel() // E_loc, gu_bias.data_ptr(),
              dn_data.data_ptr(), dn_scales.data_ptr(), dn_scales.numel() // E_loc, dn_bias.data_ptr(),
              float(alpha), float(limit), back_rows.data_ptr(), peer_bases.data_ptr(), workspace.data_ptr(),
              workspace.numel(), int(gemm_mode), status_tensor(dev).data_ptr(), _stream(dev))


def set_ep_layer_kernel(enable: bool) -> bool:
    """Process-wide: decode-sized expert-parallel steps over peer memory as one persistent
    launch (True, the default) or as the five-launch path (False). Returns the previous
    setting."""
    return bool(_lib.query("gptoss_set_ep_layer_kernel", 1 if enable else 0))


def ep_p2p_layer_fits(num_tokens: int, top_k: int, num_experts: int, world_size: int, hidden_size: int,
                      intermediate_size: int, capacity: int) -> bool:
    """Whether gptoss_ep_p2p_layer_forward serves this step (and is turned on)."""
    return bool(_lib.query("gptoss_ep_p2p_layer_fits", int(num_tokens), int(top_k), int(num_experts),
                           int(world_size), int(hidden_size), int(intermediate_size), int(capacity)))


def ep_p2p_layer_forward(hidden, router_weight, router_bias, router_indices, routing_weights, top_k: int,
                         num_experts: int, world_size: int, rank: int, gu_data, gu_scales, gu_bias, dn_data,
                         dn_scales, dn_bias, capacity: int, local_base: int, peer_bases, epoch: int, workspace,
                         alpha: float = 1.702, limit: float = 7.0):
    """One expert-parallel step in one launch (router, or the given routing when
    `router_weight` is None; dispatch, local experts, return, combine). Returns
    (out bf16 [T, H], scores bf16 [T, k] or None, router_indices i64 [T, k], send_counts i32 [W],
    pos_of i32 [T*k]). `workspace` (u8) holds at least workspace_bytes(W*cap, 1, E/W, H, I)."""
    _cuda(hidden, "hidden_states")
    _dtype(hidden, (torch.bfloat16,), "hidden_states")
    _check_weights(gu_data, gu_scales, gu_bias, dn_data, dn_scales, dn_bias)
    T, H = hidden.shape
    E_loc = gu_data.shape[0]
    I = gu_data.shape[1] // 2
    dev = hidden.device
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    send_counts = torch.empty(world_size, dtype=torch.int32, device=dev)
    pos_of = torch.empty(max(T * top_k, 1), dtype=torch.int32, device=dev)
    scores = None
    if router_weight is not None:
        _dtype(router_weight, (torch.bfloat16,), "router weight")
        _dtype(router_bias, (torch.bfloat16,), "router bias")
        router_indices = torch.empty((T, top_k), dtype=torch.int64, device=dev)
        scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
        wf = torch.empty((T, top_k), dtype=torch.float32, device=dev)
        args = (router_weight.data_ptr(), router_bias.data_ptr(), None, None)
        outs = (router_indices.data_ptr(), scores.data_ptr(), wf.data_ptr())
    else:
        _dtype(router_indices, (torch.int64,), "router_indices")
        _dtype(routing_weights, (torch.float32,), "routing_weights")
        args = (None, None, router_indices.data_ptr(), routing_weights.data_ptr())
        outs = (None, None, None)
    _lib.call("gptoss_ep_p2p_layer_forward", _p(hidden) if T else None, *args, T, int(top_k), int(num_experts),
              int(world_size), int(rank), H, I, gu_data.data_ptr(), gu_scales.data_ptr(), gu_scales.numel() // E_loc,
              gu_bias.data_ptr(), dn_data.data_ptr(), dn_scales.data_ptr(), dn_scales.numel() // E_loc,
              dn_bias.data_ptr(), float(alpha), float(limit), int(capacity), int(local_base), peer_bases.data_ptr(),
              int(epoch), _p(out) if T else None, *outs, send_counts.data_ptr(), pos_of.data_ptr(), workspace.data_ptr(),
              workspace.numel(), status_tensor(dev).data_ptr(), _stream(dev))
    return out, scores, router_indices, send_counts, pos_of


def ep_p2p_combine(local_base: int, world_size: int, capacity: int, epoch: int, pos_of, router_indices,
                   hidden_size: int, device):
    T, k = router_indices.shape
    out = torch.empty((T, hidden_size), dtype=torch.bfloat16, device=device)
    _lib.call("gptoss_ep_p2p_combine", int(local_base), int(world_size), int(capacity), int(epoch),
              pos_of.data_ptr() if T else None, router_indices.data_ptr() if T else None, T, k, int(hidden_size),
              out.data_ptr() if T else None, status_tensor(device).data_ptr(), _stream(device))
    return out
