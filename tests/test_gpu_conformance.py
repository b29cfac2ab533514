"""Conformance: the reference's own self-tests run against the drop-in modules.

Where the reference tree is reachable (environment variable AIPU_REFERENCE = its root) and a CUDA
device is present, this loads the reference's tools/q4k_ref.py and tools/glm_model_q4k_ref.py unchanged
and runs their `_selftest` functions with the drop-in's functions in place of the reference's own:
  * q4k_ref._selftest (tools/q4k_ref.py:150-182) executes with aipu_b200.q4k_ref as its module
    namespace, so every dequant and scale-table call goes to the GPU drop-in;
  * glm_model_q4k_ref._selftest (tools/glm_model_q4k_ref.py:844-979) executes with the reference
    module's namespace in which the MoE/GEMM names this library covers (QW, _mk_qw, Weights,
    matmul_q4k, moe_router, swiglu_expert, glm_sigmoid, glm_silu, matmul_q4k_col) are replaced by the
    drop-in's; the attention and decoder-stack functions (outside this library's path) stay the
    reference's and call the drop-in's MoE operators.
Both must report all passed. Elsewhere (no reference tree, or no GPU) the test is skipped: the GPU
test environment carries no copy of the reference.
"""
import importlib.util
import os
import types

import pytest

pytestmark = pytest.mark.gpu
REF = os.environ.get("AIPU_REFERENCE", "")


def _need():
    import torch

    if not REF or not os.path.isdir(os.path.join(REF, "tools")):
        pytest.skip("reference tree not reachable (set AIPU_REFERENCE to its root)")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _load(name):
    import sys

    sys.path.insert(0, os.path.join(REF, "tools"))
    spec = importlib.util.spec_from_file_location(f"_ref_{name}", os.path.join(REF, "tools", name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_q4k_ref_selftest_with_dropin(capsys):
    _need()
    from aipu_b200 import q4k_ref as mine

    ref = _load("q4k_ref")
    ns = dict(vars(mine))
    ns.setdefault("np", __import__("numpy"))
    rc = types.FunctionType(ref._selftest.__code__, ns)()
    assert rc == 0 and "ALL" in capsys.readouterr().out


def test_glm_selftest_with_dropin(capsys):
    _need()
    from aipu_b200 import glm_model_q4k_ref as mine
    from aipu_b200 import q4k_ref as mine_q

    ref = _load("glm_model_q4k_ref")
    for n in ("QW", "_mk_qw", "Weights", "matmul_q4k", "moe_router", "swiglu_expert", "glm_sigmoid", "glm_silu"):
        setattr(ref, n, getattr(mine, n))
    ref.matmul_q4k_col = mine_q.matmul_q4k_col
    fails = ref._selftest()
    assert fails == 0 and "SELF-TEST ALL PASSED" in capsys.readouterr().out
