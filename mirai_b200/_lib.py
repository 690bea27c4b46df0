"""ctypes binding of ``libmirai_b200.so`` (the C ABI in include/mirai_b200.h).

There is no fallback: if the library is missing or a CUDA device is needed and
absent, calls raise.  Every wrapper passes raw device pointers and the current
torch CUDA stream, checks the returned status and raises ``MiraiError`` with
the library's message.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmirai_b200.so")

c_vp = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_size = ctypes.c_size_t

MIRAI_OK = 0
ERROR_NAMES = {
    1: "invalid argument",
    2: "unsupported shape",
    3: "CUDA error",
    4: "device wait timed out",
    5: "device index check failed",
    6: "workspace too small",
}


class MiraiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"libmirai_b200: {ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


class Nf4Weight(ctypes.Structure):
    _fields_ = [
        ("packed", c_vp), ("absmax", c_vp), ("nested_absmax", c_vp), ("offset", c_vp),
        ("code", c_vp), ("nested_code", c_vp), ("blocksize", c_i32), ("nested_blocksize", c_i32),
    ]


class Int8Weight(ctypes.Structure):
    _fields_ = [("q", c_vp), ("scale", c_vp)]


# name -> (restype, argtypes)
SIGNATURES = {
    "mirai_b200_last_error": (ctypes.c_char_p, []),
    "mirai_b200_version": (ctypes.c_int, []),
    "mirai_b200_launch_count": (ctypes.c_uint64, []),
    "mirai_b200_device_status": (ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "mirai_route_topk": (ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_i32, c_f32, c_vp, c_vp, c_vp]),
    "mirai_b200_set_gemm_sm_limit": (ctypes.c_int, [c_i32]),
    "mirai_ipc_export": (ctypes.c_int, [c_vp, c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "mirai_ipc_import": (ctypes.c_int, [c_vp, ctypes.c_uint64, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp)]),
    "mirai_ipc_release": (ctypes.c_int, [c_vp]),
    "mirai_copy_async": (ctypes.c_int, [c_vp, c_vp, ctypes.c_uint64, c_vp]),
    "mirai_copy_blocks": (ctypes.c_int, [c_i32, c_vp, c_vp, c_vp, c_vp]),
    "mirai_ep_signal": (ctypes.c_int, [ctypes.POINTER(c_vp), c_i32, ctypes.c_uint64, c_vp]),
    "mirai_ep_wait": (ctypes.c_int, [c_vp, c_i32, c_i32, ctypes.c_uint64, c_vp]),
    "mirai_dispatch_plan_workspace_bytes": (c_size, [c_i64, c_i32, c_i32]),
    "mirai_dispatch_plan_static_scratch_bytes": (c_size, []),
    "mirai_dispatch_plan_static": (ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                                  c_vp]),
    "mirai_dispatch_plan": (ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                           c_size, c_vp]),
    "mirai_permute_rows_bf16": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_i32, c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp,
                                                    c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                   ctypes.POINTER(Nf4Weight), ctypes.POINTER(Nf4Weight), c_vp,
                                                   c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                    ctypes.POINTER(Int8Weight), ctypes.POINTER(Int8Weight), c_vp,
                                                    c_vp, c_vp]),
    "mirai_moe_down_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "mirai_moe_down_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Nf4Weight),
                                          c_vp, c_vp]),
    "mirai_moe_down_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Int8Weight),
                                           c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_src_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, c_vp,
                                                        c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_src_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32,
                                                       ctypes.POINTER(Nf4Weight), ctypes.POINTER(Nf4Weight), c_vp,
                                                       c_vp, c_vp]),
    "mirai_moe_gateup_swiglu_src_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32,
                                                        ctypes.POINTER(Int8Weight), ctypes.POINTER(Int8Weight), c_vp,
                                                        c_vp, c_vp]),
    "mirai_moe_down_src_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "mirai_moe_down_src_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32,
                                              ctypes.POINTER(Nf4Weight), c_vp, c_vp]),
    "mirai_moe_down_src_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32,
                                               ctypes.POINTER(Int8Weight), c_vp, c_vp]),
    "mirai_moe_combine": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_i32, c_vp]),
    "mirai_moe_combine_backward": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "mirai_moe_down_dx_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_down_dx_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Nf4Weight),
                                             c_vp, c_vp, c_vp]),
    "mirai_moe_down_dx_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Int8Weight),
                                              c_vp, c_vp, c_vp]),
    "mirai_moe_gateup_dx_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_gateup_dx_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Nf4Weight),
                                               ctypes.POINTER(Nf4Weight), c_vp, c_vp]),
    "mirai_moe_gateup_dx_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                ctypes.POINTER(Int8Weight), ctypes.POINTER(Int8Weight), c_vp,
                                                c_vp]),
    "mirai_moe_lora_project": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_vp, c_i32, c_i32, c_f32, c_vp,
                                              c_vp]),
    "mirai_moe_lora_grad": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_i64, c_i64, c_i64,
                                           c_vp]),
    "mirai_moe_down_lora_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp,
                                                c_vp]),
    "mirai_moe_down_lora_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Nf4Weight),
                                               c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_down_lora_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Int8Weight),
                                                c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_down_dx_lora_bf16": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp,
                                                   c_vp, c_vp]),
    "mirai_moe_down_dx_lora_nf4": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                  ctypes.POINTER(Nf4Weight), c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mirai_moe_down_dx_lora_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                   ctypes.POINTER(Int8Weight), c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mirai_nf4_quantize_workspace_bytes": (c_size, [c_i32, c_i64, c_i64]),
    "mirai_nf4_dequantize": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i64, c_i64, c_i32, c_i32,
                                            c_vp, c_vp]),
    "mirai_nf4_quantize": (ctypes.c_int, [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp,
                                          c_vp, c_vp, c_size, c_vp]),
    "mirai_int8_quantize_rows": (ctypes.c_int, [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "mirai_rotate_rows": (ctypes.c_int, [c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_i32, c_vp]),
    "mirai_moe_lora_project_src": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_vp, c_i32, c_i32,
                                                  c_f32, c_vp, c_vp]),
    "mirai_moe_lora_grad_src": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, c_vp, c_i64,
                                               c_i64, c_i64, c_vp]),
    **{f"mirai_moe_down_lora_src_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, t, c_vp, c_vp,
                                                       c_vp, c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)), ("int8", ctypes.POINTER(Int8Weight)))},
    **{f"mirai_moe_down_dx_lora_src_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, t, c_vp,
                                                          c_vp, c_vp, c_vp, c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)), ("int8", ctypes.POINTER(Int8Weight)))},
    **{f"mirai_moe_down_dx_src_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, t, c_vp, c_vp,
                                                     c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)), ("int8", ctypes.POINTER(Int8Weight)))},
    **{f"mirai_moe_gateup_dx_src_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_i32, t, t, c_vp,
                                                       c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)), ("int8", ctypes.POINTER(Int8Weight)))},
    "mirai_route_topk_rows": (ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_i64, c_i32, c_f32, c_vp,
                                             c_vp, c_vp]),
    **{f"mirai_moe_gateup_ex_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, t, t, c_i32, c_i32, c_vp,
                                                   c_vp, c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)))},
    **{f"mirai_moe_down_ex_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, t, c_i32, c_vp, c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)))},
    **{f"mirai_moe_down_dx_ex_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, t, c_i32, c_i32, c_vp,
                                                    c_vp, c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)))},
    **{f"mirai_moe_gateup_dx_ex_{f}": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, t, t, c_i32, c_vp,
                                                      c_vp])
       for f, t in (("bf16", c_vp), ("nf4", ctypes.POINTER(Nf4Weight)))},
    "mirai_swiglu_backward_rotated": (ctypes.c_int, [c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_vp]),
    "mirai_moe_down_dh_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(Int8Weight),
                                              c_vp, c_vp]),
    "mirai_moe_down_dh_lora_int8": (ctypes.c_int, [c_vp, c_vp, c_i32, c_i64, c_i32, c_i32,
                                                   ctypes.POINTER(Int8Weight), c_vp, c_vp, c_vp, c_vp]),
}

_lib = None


def load(required: bool = True):
    """Load the library (once).  Raises if it is missing and ``required``."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if not required:
            return None
        raise MiraiError(3, f"{LIB_PATH} is not built; run `python -m mirai_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported(name: str) -> bool:
    return hasattr(load(), name)


def call(name: str, *args) -> None:
    lib = load()
    fn = getattr(lib, name, None)
    if fn is None:
        raise MiraiError(2, f"{name} is not exported by {LIB_PATH}")
    rc = fn(*args)
    if rc != MIRAI_OK:
        msg = lib.mirai_b200_last_error()
        raise MiraiError(rc, msg.decode() if msg else "")


def launch_count() -> int:
    return int(load().mirai_b200_launch_count())


def device_status(stream_handle: int) -> tuple[int, int]:
    lib = load()
    code = ctypes.c_int(0)
    info = ctypes.c_int(0)
    rc = lib.mirai_b200_device_status(c_vp(stream_handle), ctypes.byref(code), ctypes.byref(info))
    if rc != MIRAI_OK:
        raise MiraiError(rc, lib.mirai_b200_last_error().decode())
    return code.value, info.value
