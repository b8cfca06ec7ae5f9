"""C-ABI checks that need no GPU: the library loads, exports every symbol the header
declares, answers host-only size queries and rejects bad arguments before touching a
device."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "gptoss_moe.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gptoss_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for must in ("gptoss_fused_moe_routing", "gptoss_fp4_group_mm", "gptoss_moe_experts_forward",
                 "gptoss_moe_layer_forward", "gptoss_quantize_fp8", "gptoss_router_topk", "gptoss_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in gptoss_moe.h but not exported"
        assert name in pkg._lib._SIGNATURES, f"{name} has no ctypes signature"
    raw = ctypes.CDLL(pkg._lib.lib_path())
    for name in _declared():
        getattr(raw, name)


def test_abi_version(pkg):
    assert pkg._lib.load().gptoss_abi_version() == pkg._lib.ABI_VERSION


def test_host_size_queries(pkg):
    q = pkg._lib.query
    assert q("gptoss_blocked_scales_bytes", 2880, 2944) == 270848
    assert q("gptoss_blocked_scales_bytes", 5760, 2944) == 529920
    assert q("gptoss_blocked_scales_bytes", 0, 2944) == 0
    assert q("gptoss_batch_blocked_scales_capacity", 128, 32, 2944) >= 33 * 23 * 512
    w1 = q("gptoss_moe_workspace_bytes", 32, 4, 32, 2880, 2880)
    w2 = q("gptoss_moe_workspace_bytes", 8192, 4, 32, 2880, 2880)
    assert 0 < w1 < w2
    assert q("gptoss_moe_workspace_bytes", -1, 4, 32, 2880, 2880) == 0


def test_argument_errors_before_device_access(pkg):
    lib = pkg._lib.load()
    rc = lib.gptoss_quantize_fp8(None, 0, 4, 31, None, None, None)
    assert rc == 1 and b"multiple of 32" in lib.gptoss_last_error()
    rc = lib.gptoss_fp4_group_mm(None, None, 4, 512, None, 1, 256, 500, None, None, 0, None, None, None, None, 0,
                                 None, None)
    assert rc == 1 and b"multiple of 128" in lib.gptoss_last_error()
    rc = lib.gptoss_moe_experts_forward(None, None, None, 4, 9, 4, 512, 256, None, None, 0, None, None, None, 0,
                                        None, 1.702, 7.0, None, None, 0, 0, None, None)
    assert rc == 1 and b"top_k" in lib.gptoss_last_error()


def test_later_entry_points_check_arguments_first(pkg):
    # the MMA probe, the W4A4 grouped GEMM, the norm kernel, the block op and the one-launch
    # expert-parallel step validate their sizes on the host and fail with a message
    lib = pkg._lib.load()

    def fails(rc, text):
        assert rc == 1 and text in lib.gptoss_last_error(), lib.gptoss_last_error()

    fails(lib.gptoss_mma_peak(2, 1, 256, 10, None, None), b"kind must be")
    fails(lib.gptoss_mma_peak(0, 1, 200, 10, None, None), b"multiple of 16")
    fails(lib.gptoss_mma_peak(1, 0, 128, 0, None, None), b"iters")
    fails(lib.gptoss_fp4_group_mm_w4a4(None, None, 4, 50, None, 1, 256, 100, None, None, 0, None, None, None, None, 0,
                                       None, None), b"multiple of 64")
    fails(lib.gptoss_fp4_group_mm_w4a4(None, None, 4, 64, None, 1, 100, 128, None, None, 0, None, None, None, None, 0,
                                       None, None), b"multiple of 8")
    fails(lib.gptoss_fp4_group_mm_w4a4(None, None, 4, 128, None, 1, 256, 128, None, None, 0, None, None, None, None, 0,
                                       None, None), b"[M, K/2]")
    fails(lib.gptoss_rmsnorm_residual(None, None, 1e-5, 4, 2884, None, None, None), b"multiple of 8")
    fails(lib.gptoss_rmsnorm_residual(None, None, 1e-5, -1, 2880, None, None, None), b"num_tokens")
    assert lib.gptoss_rmsnorm_residual(None, None, 1e-5, 0, 2880, None, None, None) == 0   # nothing to do
    fails(lib.gptoss_moe_block_forward(None, None, 1e-5, None, None, 4, 9, 4, 512, 256, None, None, 0, None, None,
                                       None, 0, None, 1.702, 7.0, None, None, None, None, 0, 0, None, None),
          b"top_k")
    fails(lib.gptoss_ep_p2p_layer_forward(None, None, None, None, None, 4, 4, 32, 3, 0, 512, 256, None, None, 0, None,
                                          None, None, 0, None, 1.702, 7.0, 16, None, None, 1, None, None, None, None,
                                          None, None, None, 0, None, None), b"multiple of world_size")
    fails(lib.gptoss_ep_p2p_layer_forward(None, None, None, None, None, 4, 4, 32, 2, 2, 512, 256, None, None, 0, None,
                                          None, None, 0, None, 1.702, 7.0, 16, None, None, 1, None, None, None, None,
                                          None, None, None, 0, None, None), b"world_size / rank")
    # host-only size answers
    q = pkg._lib.query
    e = q("gptoss_moe_workspace_bytes", 32, 4, 32, 2880, 2880)
    assert q("gptoss_moe_block_workspace_bytes", 32, 4, 32, 2880, 2880) >= e + 32 * 2880 * 2
    assert q("gptoss_moe_block_workspace_bytes", -1, 4, 32, 2880, 2880) == 0


def test_wrapper_raises_on_failure(pkg):
    with pytest.raises(pkg._lib.GptossError, match="multiple of 32"):
        pkg._lib.call("gptoss_quantize_fp8", None, 0, 4, 31, None, None, None)


def test_header_is_plain_c():
    # FFI hosts (cgo, JNI, N-API, ctypes) consume the header as C: it must compile as C99
    # on its own, with no CUDA or C++ headers.
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    r = subprocess.run([cc, "-fsyntax-only", "-std=c99", "-Wall", "-Werror", "-x", "c", HEADER],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_c_program_links_and_calls_host_queries(pkg, tmp_path):
    # What a C / cgo / JNI host does: include the header, link the library, call entry
    # points. Only host-side queries run here (no GPU on this machine).
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = pkg._lib.lib_path()
    src = tmp_path / "probe.c"
    src.write_text(r"""
#include <stdio.h>
#include "gptoss_moe.h"
int main(void) {
  if (gptoss_abi_version() != 2) return 1;
  size_t ws = gptoss_moe_workspace_bytes(32, 4, 32, 2880, 2880);
  long long rb = (long long)gptoss_ep_row_bytes(2880);
  printf("%zu %lld\n", ws, rb);
  return ws > 0 && rb == 2992 ? 0 : 2;
}
""")
    exe = tmp_path / "probe"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe),
                        lib, "-Wl,-rpath," + os.path.dirname(lib)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.stdout, r.stderr)
    assert int(r.stdout.split()[0]) == pkg.ops.workspace_bytes(32, 4, 32, 2880, 2880)


def test_gemm_layout_choice(pkg):
    # AUTO: 16-row chunks up to 12 rows per expert on average, 64-row chunks up to 80,
    # tokens on M above (crossovers measured on B200 for H = I = 2880)
    q = lambda mode, rows, e: pkg._lib.query("gptoss_moe_gemm_layout", mode, rows, e)   # noqa: E731
    AUTO, TOK, SWAP, WIDE = pkg.ops.GEMM_AUTO, pkg.ops.GEMM_TOKENS_M, pkg.ops.GEMM_SWAP, pkg.ops.GEMM_SWAP_WIDE
    assert q(AUTO, 32 * 4, 32) == SWAP                     # decode, T = 32
    assert q(AUTO, 12 * 32, 32) == SWAP and q(AUTO, 12 * 32 + 1, 32) == WIDE
    assert q(AUTO, 80 * 32, 32) == WIDE and q(AUTO, 80 * 32 + 1, 32) == TOK
    assert q(AUTO, 8192 * 4, 32) == TOK                    # prefill
    for m in (TOK, SWAP, WIDE):
        assert q(m, 8192 * 4, 32) == m and q(m, 4, 32) == m
    assert q(7, 4, 32) == -1 and q(AUTO, 4, 0) == -1
