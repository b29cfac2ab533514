"""GPU parity of the bit-exact chain kernel (aipu_b200/csrc/chain.cu) through the C ABI.

Every output must equal the reference's sequential fp32 chain (tools/q4k_ref.py:86-92) bit for bit:
aipu_q4k_gemm in AIPU_MODE_STRICT runs the chain kernel for Q4_K/Q6_K rows (K a multiple of 256 and
16-byte rows) and the generic strict kernel otherwise; both are checked against the oracle at uint32
equality, for bf16 and fp32 activations, token counts that need several passes (M > 8), row counts
that leave a partial tile, and fp16 scale edge cases (zero, subnormal, max).
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


def _bf16_np(t):
    return (t.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(F32)


def _x(M, K, seed, f32):
    x = np.random.default_rng(seed).standard_normal((M, K)).astype(F32)
    return x if f32 else qo.bf16_round(x)


def _to_dev(x, f32, d):
    if f32:
        return torch.from_numpy(x).to(d)
    return torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(d).view(torch.bfloat16)


@pytest.mark.parametrize("wt,N,K,M,f32", [
    (F.Q4_K, 256, 256, 1, False), (F.Q4_K, 300, 2048, 3, False), (F.Q4_K, 2048, 6144, 1, False),
    (F.Q4_K, 520, 4096, 1, True), (F.Q4_K, 96, 1024, 19, False),
    (F.Q6_K, 6144, 2048, 1, False), (F.Q6_K, 700, 2048, 5, False), (F.Q6_K, 130, 4096, 9, True),
    (F.Q6_K, 64, 256, 2, False)])   # Q6_K K = 256: 210-byte rows, the generic strict kernel
def test_strict_gemm_bit_exact(wt, N, K, M, f32):
    d = _dev()
    w = F.random_rows_np(wt, N, K, seed=N + K + M)
    x = _x(M, K, M + 1, f32)
    y32 = torch.empty((M, N), dtype=torch.float32, device=d)
    y = ops.gemm(wt, torch.from_numpy(w).to(d), N, K, _to_dev(x, f32, d), mode="strict")
    torch.cuda.synchronize()
    ref = qo.gemm(wt, w, N, K, x)
    assert np.array_equal(_bf16_np(y).view(np.uint32), ref.view(np.uint32))


def test_strict_gemm_scale_edge_cases():
    """fp16 d / dmin of 0, the smallest subnormal, the largest finite value, and all-15 / all-0 codes."""
    d = _dev()
    N, K, M = 256, 512, 2
    w = F.random_rows_np(F.Q4_K, N, K, seed=5).reshape(N, K // 256, 144)
    vals = np.array([0x0000, 0x0001, 0x03FF, 0x7BFF, 0x3C00, 0x8001], np.uint16)
    for r in range(N):
        w[r, :, 0:2] = np.frombuffer(vals[r % 6].tobytes(), np.uint8)
        w[r, :, 2:4] = np.frombuffer(vals[(r // 6) % 6].tobytes(), np.uint8)
        if r % 7 == 0:
            w[r, :, 16:] = 0xFF
        if r % 11 == 0:
            w[r, :, 16:] = 0x00
    w = w.reshape(N, -1)
    x = _x(M, K, 3, False) * F32(1e-3)
    x = qo.bf16_round(x)
    y = ops.gemm(F.Q4_K, torch.from_numpy(w).to(d), N, K, _to_dev(x, False, d), mode="strict")
    torch.cuda.synchronize()
    ref = qo.gemm(F.Q4_K, w, N, K, x)
    assert np.array_equal(_bf16_np(y).view(np.uint32), ref.view(np.uint32))


def test_strict_gemm_f32_accumulators():
    """y_f32 receives the sequential fp32 chain itself (before bf16 rounding)."""
    d = _dev()
    N, K, M = 300, 1024, 2
    w = F.random_rows_np(F.Q4_K, N, K, seed=9)
    x = _x(M, K, 4, False)
    y32 = torch.empty((M, N), dtype=torch.float32, device=d)
    ops.gemm(F.Q4_K, torch.from_numpy(w).to(d), N, K, _to_dev(x, False, d), mode="strict", out_f32=y32)
    torch.cuda.synchronize()
    ref = qo.matmul_seq_f32(x, qo.dequant_rows(F.Q4_K, w, N, K))
    assert np.array_equal(y32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
