"""ctypes wrapper of oracle/build/liboracle.so (TEST INFRASTRUCTURE ONLY: checker and CPU baseline).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "build", "liboracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        L.oracle_gemm.restype = ctypes.c_int
        L.oracle_gemm.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]
        L.oracle_dequant_row.restype = None
        L.oracle_dequant_row.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        _lib = L
    return _lib


def gemm(wtype: int, w: np.ndarray, N: int, K: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """bf16-valued fp32 [M, N]: the sequential-contract GEMM in C, split over threads."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0]
    y = np.empty((M, N), np.uint16)
    nt = nthreads or (os.cpu_count() or 1)
    rc = lib().oracle_gemm(wtype, w.ctypes.data, N, K, x.ctypes.data, M, y.ctypes.data, nt)
    if rc:
        raise RuntimeError("oracle_gemm failed")
    return (y.astype(np.uint32) << 16).view(np.float32)


def dequant_row(wtype: int, row: np.ndarray, K: int) -> np.ndarray:
    out = np.empty(K, np.float32)
    lib().oracle_dequant_row(wtype, np.ascontiguousarray(row, np.uint8).ctypes.data, K, out.ctypes.data)
    return out
