"""ctypes binding of the in-tree CUDA library (``libaipu_q4k.so``, C ABI in include/aipu_q4k.h).

There is no fallback: if the library is missing or fails to load, importing the bindings raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaipu_q4k.so")

# status codes (include/aipu_q4k.h)
AIPU_OK, AIPU_EINVAL, AIPU_ECUDA, AIPU_ETIMEOUT, AIPU_ENCCL, AIPU_ENOMEM = 0, -1, -2, -3, -4, -5
# weight types
Q4_K, Q6_K, Q8_0, F16, F32 = 0, 1, 2, 3, 4
DT_F32, DT_BF16 = 0, 1
MODE_FAST, MODE_STRICT = 0, 1
FLAG_PDL = 1
FLAG_STRICT = 2
FLAG_TC_DECODE = 4
FLAG_FAST_DOWN = 8

c_void_p, c_int, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float


class AipuError(RuntimeError):
    """A C entry point returned a non-zero status; carries the code and the library's text."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"aipu error {code}: {msg}")
        self.code = code


class MoeWeights(ctypes.Structure):
    """aipu_moe_weights (include/aipu_q4k.h)."""

    _fields_ = [
        ("hidden", c_int64), ("ffn", c_int64), ("n_experts", c_int64), ("topk", ctypes.c_int32),
        ("scale", c_float), ("router_wtype", ctypes.c_int32), ("router_w", c_void_p), ("router_bias", c_void_p),
        ("gate_wtype", ctypes.c_int32), ("up_wtype", ctypes.c_int32), ("down_wtype", ctypes.c_int32),
        ("gate_w", c_void_p), ("up_w", c_void_p), ("down_w", c_void_p),
        ("shared_gate_w", c_void_p), ("shared_up_w", c_void_p), ("shared_down_w", c_void_p),
    ]


# name -> (restype, argtypes); every function the header declares
SIGNATURES = {
    "aipu_version": (c_int, []),
    "aipu_last_error": (ctypes.c_char_p, []),
    "aipu_row_bytes": (c_int64, [c_int, c_int64]),
    "aipu_ctx_create": (c_int, [ctypes.POINTER(c_void_p), c_int]),
    "aipu_ctx_destroy": (c_int, [c_void_p]),
    "aipu_ctx_status": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "aipu_ctx_set_flags": (c_int, [c_void_p, c_int]),
    "aipu_ctx_set_wait_limit": (c_int, [c_void_p, c_int64]),
    "aipu_selftest_wait": (c_int, [c_void_p, c_void_p]),
    "aipu_q4k_dequant": (c_int, [c_int, c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p]),
    "aipu_act_eval": (c_int, [c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "aipu_q4k_gemm": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p,
                              c_void_p, c_int, c_void_p]),
    "aipu_q4k_gemm_noalloc": (c_int, [c_int, c_void_p, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p,
                                      c_void_p]),
    "aipu_q4k_gemm_noalloc_status": (c_int, [ctypes.POINTER(c_int)]),
    "aipu_q4k_gemm_tc": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                                 c_void_p]),
    "aipu_bf16_dot_gemv": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p]),
    "aipu_q4k_gemm_grouped": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                      c_int, c_int64, c_void_p, c_void_p]),
    "aipu_moe_router": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                                c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "aipu_moe_layer": (c_int, [c_void_p, ctypes.POINTER(MoeWeights), c_void_p, c_int64, c_void_p, c_void_p,
                               c_void_p, c_void_p]),
    "aipu_swiglu_expert": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int64, c_int64,
                                   c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "aipu_moe_experts": (c_int, [c_void_p, ctypes.POINTER(MoeWeights), c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                                 c_int64, c_int64, c_void_p, c_void_p]),
    "aipu_moe_combine": (c_int, [c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_void_p]),
    "aipu_ep_create": (c_int, [c_void_p, c_int, c_int, c_int64, c_int64, c_int, ctypes.POINTER(c_void_p), c_void_p]),
    "aipu_ep_connect": (c_int, [c_void_p, c_void_p]),
    "aipu_ep_moe_layer": (c_int, [c_void_p, ctypes.POINTER(MoeWeights), c_int64, c_void_p, c_int64, c_void_p, c_void_p]),
    "aipu_ep_destroy": (c_int, [c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m aipu_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != AIPU_OK:
        raise AipuError(rc, lib().aipu_last_error().decode(errors="replace"))
