"""The C-ABI library loads and exports every symbol include/mirai_b200.h declares (no GPU needed)."""

import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            with open(os.path.join(inc, fn)) as f:
                text = f.read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"^[A-Za-z_][\w \*]*?\b(mirai_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("mirai_route_topk", "mirai_dispatch_plan", "mirai_permute_rows_bf16",
                     "mirai_moe_gateup_swiglu_bf16", "mirai_moe_down_bf16", "mirai_moe_combine"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from mirai_b200 import _lib
    from mirai_b200.build import build

    build()
    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert lib.mirai_b200_version() >= 100


def test_host_side_validation_without_gpu():
    """Argument checks run on the host before any launch and report clean errors."""
    from mirai_b200 import _lib

    lib = _lib.load()
    rc = lib.mirai_route_topk(None, 4, 8, 9, 0, None, 1, 1.0, None, None, None)
    assert rc == 1 and b"k <=" in lib.mirai_b200_last_error()
    rc = lib.mirai_moe_gateup_swiglu_bf16(None, None, 4, 128, 100, 128, None, None, None, None, None)
    assert rc == 2 and b"K % 64" in lib.mirai_b200_last_error()
    rc = lib.mirai_moe_down_bf16(None, None, 4, 128, 128, 200, None, None, None)
    assert rc == 2
    assert lib.mirai_dispatch_plan_workspace_bytes(1000, 2, 8) == 8 * 4  # one 2048-route chunk
    with pytest.raises(_lib.MiraiError):
        _lib.call("mirai_moe_combine", None, None, None, 4, 0, 8, None, 0, None)


def test_exchange_entry_points_validate_on_the_host():
    """The expert-parallel exchange helpers reject bad arguments before any CUDA call."""
    import ctypes

    from mirai_b200 import _lib

    lib = _lib.load()
    off = ctypes.c_uint64(0)
    handle = (ctypes.c_uint8 * 64)()
    assert lib.mirai_ipc_export(None, handle, ctypes.byref(off)) == 1
    assert lib.mirai_ipc_import(None, 0, None, None) == 1
    assert lib.mirai_ipc_release(None) == 0                     # nothing to release
    assert lib.mirai_copy_async(None, None, 0, None) == 0        # zero bytes: no copy
    assert lib.mirai_copy_async(None, None, 16, None) == 1
    addrs = (ctypes.c_uint64 * 2)(0, 4096)
    sizes = (ctypes.c_uint64 * 2)(0, 0)
    assert lib.mirai_copy_blocks(0, None, None, None, None) == 0        # empty list
    assert lib.mirai_copy_blocks(-1, addrs, addrs, sizes, None) == 1
    assert lib.mirai_copy_blocks(2, None, addrs, sizes, None) == 1      # missing array
    assert lib.mirai_copy_blocks(2, addrs, addrs, sizes, None) == 0     # zero-byte blocks are skipped
    sizes[1] = 16
    assert lib.mirai_copy_blocks(2, addrs, (ctypes.c_uint64 * 2)(0, 0), sizes, None) == 1  # null source
    assert b"block 1" in lib.mirai_b200_last_error()
    slots = (_lib.c_vp * 2)()
    assert lib.mirai_ep_signal(slots, 0, 1, None) == 1           # no slots
    assert lib.mirai_ep_signal(slots, 65, 1, None) == 1          # more peers than supported
    assert lib.mirai_ep_wait(None, 2, 0, 1, None) == 1
    assert lib.mirai_ep_wait(_lib.c_vp(8 * 1024 + 4), 2, 0, 1, None) == 1  # flags not 8-byte aligned
    assert lib.mirai_b200_set_gemm_sm_limit(1) == 1
    assert lib.mirai_b200_set_gemm_sm_limit(-2) == 1
    assert lib.mirai_b200_set_gemm_sm_limit(0) == 0
    rc = lib.mirai_moe_gateup_swiglu_src_bf16(None, None, 0, 4, 128, 256, 256, None, None, None, None, None)
    assert rc == 1 and b"sources" in lib.mirai_b200_last_error()
