"""GPU parity of the tcgen05 prefill GEMM (aipu_q4k_gemm_tc) against the oracle.

Bar: >= 99.9 % of outputs within 1 bf16 ulp of the sequential reference and max relative error
<= 1e-2 (denominator floored at 2^-8 * rms of the reference row), as for the fast decode GEMV.
"""
import numpy as np
import pytest
import torch

from aipu_b200 import formats as F
from aipu_b200 import ops
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu
F32 = np.float32


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bf16_dev(x):
    bits = (np.asarray(x, F32).view(np.uint32) >> 16).astype(np.uint16)
    return torch.from_numpy(bits.view(np.int16)).to(_dev()).view(torch.bfloat16)


def _bf16_np(t):
    return (t.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(F32)


@pytest.mark.parametrize("wt", [F.Q4_K, F.Q6_K])
@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (70, 300, 2048), (200, 256, 6144)])
def test_gemm_tc_matches_oracle(wt, M, N, K):
    d = _dev()
    w = F.random_rows_np(wt, N, K, seed=M + N + wt)
    x = qo.bf16_round(np.random.default_rng(M).standard_normal((M, K)).astype(F32))
    ref = qo.gemm(wt, w, N, K, x)
    y = ops.gemm_tc(wt, torch.from_numpy(w).to(d), N, K, _bf16_dev(x))
    torch.cuda.synchronize()
    st = qo.parity_stats(_bf16_np(y), ref)
    assert st["frac_within_1ulp"] >= 0.999 and st["max_rel"] <= 1e-2, st
