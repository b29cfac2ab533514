"""CPU checks of the C-ABI boundary: the library loads and exports every declared entry point."""
import ctypes
import os
import re

import pytest

from aipu_b200 import _lib
from aipu_b200 import formats as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names |= set(re.findall(r"\b(aipu_\w+)\s*\(", txt))
    return names


def test_library_loads_and_exports_all_declared_symbols():
    L = _lib.lib()
    names = declared()
    assert names, "no declarations found"
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(_lib.SIGNATURES) >= names, f"no ctypes signature for {names - set(_lib.SIGNATURES)}"


def test_version_and_row_bytes():
    L = _lib.lib()
    assert L.aipu_version() >= 100
    for wt in (F.Q4_K, F.Q6_K, F.Q8_0, F.F16, F.F32):
        for K in (256, 2048, 6144):
            assert L.aipu_row_bytes(wt, K) == F.row_bytes(wt, K)
    assert L.aipu_row_bytes(F.Q4_K, 100) == 0
    assert L.aipu_row_bytes(9, 256) == 0


def test_errors_do_not_need_a_gpu():
    L = _lib.lib()
    rc = L.aipu_q4k_dequant(F.Q4_K, None, 1, 256, None, 0, None)
    assert rc == _lib.AIPU_EINVAL
    assert b"bad arguments" in L.aipu_last_error()
    with pytest.raises(_lib.AipuError):
        _lib.check(rc)


def test_argument_errors_of_newer_entry_points_do_not_need_a_gpu():
    """Null contexts and bad shapes are rejected before any device work, with a message."""
    L = _lib.lib()
    assert L.aipu_bf16_dot_gemv(None, None, 16, 64, None, 1, None, None) == _lib.AIPU_EINVAL
    assert b"bf16_dot_gemv" in L.aipu_last_error()
    assert L.aipu_moe_layer(None, None, None, 1, None, None, None, None) == _lib.AIPU_EINVAL
    assert L.aipu_ep_moe_layer(None, None, 0, None, 1, None, None) != 0
