"""The bf16 dot GEMV (LM-head contract, tools/glm_model_q4k_ref.py:474-486) on the GPU: bit-exact
against the reference-generated fixture and against the oracle at LM-head-like sizes, ragged K
(K % 56 != 0) and 1-6 token rows."""
import numpy as np
import pytest
import torch

from aipu_b200 import ops
from oracle import moe_oracle as mo
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu
F32 = np.float32


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _to_bf16(bits_u16, d):
    return torch.from_numpy(np.ascontiguousarray(bits_u16).astype(np.uint16).view(np.int16)).to(d).view(torch.bfloat16)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().astype(np.uint16)


def test_bf16_dot_fixture_bitexact(golden):
    d = _dev()
    g = golden("lmhead_golden")
    for c in ("a", "b", "c"):
        y = ops.bf16_dot_gemv(_to_bf16(g[f"{c}_w"], d), _to_bf16(g[f"{c}_x"], d))
        assert np.array_equal(_bits(y), g[f"{c}_y"]), c


@pytest.mark.parametrize("V,K,M", [(3000, 6144, 1), (2500, 4096, 2), (1000, 6136, 3), (777, 1000, 5), (64, 8, 6)])
def test_bf16_dot_matches_oracle(V, K, M):
    d = _dev()
    rng = np.random.default_rng(V + K + M)
    x = qo.bf16_round(rng.standard_normal((M, K)).astype(F32))
    w = qo.bf16_round((rng.standard_normal((V, K)) * 0.02).astype(F32))
    y = ops.bf16_dot_gemv(_to_bf16(w.view(np.uint32) >> 16, d), _to_bf16(x.view(np.uint32) >> 16, d))
    ref = mo.bf16_dot7(x, w)
    assert np.array_equal(_bits(y), (ref.view(np.uint32) >> 16).astype(np.uint16))
