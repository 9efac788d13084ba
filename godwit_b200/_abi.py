"""ctypes binding of include/godwit_cuda.h.

The product path is the CUDA library `libgodwit_cuda.so` next to this file.
There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgodwit_cuda.so")

GW_OK = 0
GW_E_ARG = -1
GW_E_CUDA = -2
GW_E_OOM = -3
GW_E_TIMEOUT = -4
GW_E_STATE = -5
GW_E_UNSUPPORTED = -6

GW_DTYPE_F16 = 0
GW_DTYPE_BF16 = 1
GW_DTYPE_F32 = 2  # int8 projection outputs only
GW_ACT_GPTOSS_CLAMPED = 0
GW_ACT_SILU = 1

SECTIONS = ("gate_up_blocks", "gate_up_scales", "down_blocks", "down_scales",
            "gate_up_bias", "down_bias")

_STATUS_NAMES = {GW_E_ARG: "GW_E_ARG", GW_E_CUDA: "GW_E_CUDA", GW_E_OOM: "GW_E_OOM",
                 GW_E_TIMEOUT: "GW_E_TIMEOUT", GW_E_STATE: "GW_E_STATE",
                 GW_E_UNSUPPORTED: "GW_E_UNSUPPORTED"}


class GodwitCUDAError(RuntimeError):
    """A non-zero gw_status, with the library's thread-local message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")


class BankDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32), ("intermediate", C.c_int32), ("experts", C.c_int32),
        ("layers", C.c_int32), ("top_k", C.c_int32), ("activation", C.c_int32),
        ("limit", C.c_float), ("alpha", C.c_float), ("has_router_bias", C.c_int32),
        ("shard_rank", C.c_int32), ("shard_count", C.c_int32), ("reserved0", C.c_int32),
        ("expert_stride", C.c_int64), ("section_offset", C.c_int64 * 6),
        ("section_length", C.c_int64 * 6),
    ]


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
ST = C.c_int32

# name -> (restype, argtypes); every entry of include/godwit_cuda.h
SIGNATURES = {
    "gw_last_error": (C.c_char_p, []),
    "gw_version": (I32, []),
    "gw_init": (ST, [I32, C.POINTER(P)]),
    "gw_shutdown": (ST, [P]),
    "gw_ctx_set_stream": (ST, [P, P]),
    "gw_sync": (ST, [P]),
    "gw_selftest_wait_timeout": (ST, [P, I64]),
    "gw_set_tensor_core_min_tokens": (ST, [P, I32]),
    "gw_set_block_scaled": (ST, [P, I32]),
    "gw_layout_default": (ST, [I32, I32, I32, I32, I32, I32, C.POINTER(BankDesc)]),
    "gw_bank_create": (ST, [P, C.POINTER(BankDesc), C.POINTER(P)]),
    "gw_bank_destroy": (ST, [P]),
    "gw_bank_upload_expert": (ST, [P, I32, I32, P, C.c_size_t]),
    "gw_bank_upload_router": (ST, [P, I32, P, P]),
    "gw_bank_fill_synthetic": (ST, [P, C.c_uint64]),
    "gw_bank_download_expert": (ST, [P, I32, I32, P, C.c_size_t]),
    "gw_bank_bytes": (ST, [P, C.POINTER(I64)]),
    "gw_router_logits": (ST, [P, P, I32, P, I32, I32, P]),
    "gw_route": (ST, [P, P, I32, P, I32, I32, P, P]),
    "gw_expert_apply": (ST, [P, P, I32, I32, P, I32, P]),
    "gw_expert_apply_batch": (ST, [P, P, I32, P, I32, I32, P, P, P]),
    "gw_moe_forward": (ST, [P, P, I32, P, I32, I32, P, P, P, P, P]),
    "gw_mxfp4_gemv": (ST, [P, P, P, P, P, I32, P, I32, I32]),
    "gw_int8_affine_gemv": (ST, [P, P, P, P, P, I32, I32, I32, P, I32]),
    "gw_ep_dispatch_async": (ST, [P, P, P, I32, I32, P, P, I32, I32, P, P, P]),
    "gw_ep_combine_async": (ST, [P, P, P, P, I32, P]),
    "gw_int8_affine_gemv_async": (ST, [P, P, P, P, P, I32, I32, I32, P, I32]),
    "gw_mxfp4_dequant": (ST, [P, P, P, I32, I32, P]),
    "gw_mxfp4_gemv_batched_async": (ST, [P, I32, P, I64, P, I64, P, I64, P, I64, I32, P, I64,
                                         I32, I32]),
    "gw_moe_forward_async": (ST, [P, P, I32, P, I32, I32, P, P, P]),
    "gw_moe_stack_forward_async": (ST, [P, P, P, I32, I32, P]),
    "gw_moe_apply_async": (ST, [P, P, I32, P, I32, I32, P, P, P, I32]),
    "gw_residual_round_async": (ST, [P, P, P, P, I32, I64]),
    "gw_last_launch_count": (ST, [P, C.POINTER(I64)]),
    "gw_rmsnorm_async": (ST, [P, P, P, C.c_float, I32, I32, P]),
    "gw_route_async": (ST, [P, P, I32, P, I32, I32, P, P]),
    "gw_moe_block": (ST, [P, P, I32, P, P, C.c_float, I32, P, P]),
    "gw_moe_block_async": (ST, [P, P, I32, P, P, C.c_float, I32, P, P]),
}

class Profile(C.Structure):
    _fields_ = [("gateup_launches", C.c_int64), ("down_launches", C.c_int64),
                ("gemv_launches", C.c_int64), ("gateup_ms", C.c_double), ("down_ms", C.c_double),
                ("gemv_ms", C.c_double), ("expert_passes", C.c_int64),
                ("gemv_matrices", C.c_int64), ("router_launches", C.c_int64),
                ("combine_launches", C.c_int64), ("router_ms", C.c_double),
                ("combine_ms", C.c_double)]


SIGNATURES["gw_moe_forward_noalloc_async"] = (ST, [P, P, I32, P, I32, I32, P, P, P])
SIGNATURES["gw_profile_enable"] = (ST, [P, I32])
SIGNATURES["gw_profile_read"] = (ST, [P, C.POINTER(Profile)])

_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> C.CDLL:
    """Loads the CUDA library (building it first if its sources are newer)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise GodwitCUDAError(GW_E_STATE, f"CUDA library {p} is not built; run "
                                  "`python -m godwit_b200.build` (no CPU fallback exists)")
        lib = C.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != GW_OK:
        msg = load().gw_last_error()
        raise GodwitCUDAError(status, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
