"""GPU test of aipu_q4k_gemm_noalloc, the GEMM entry point that never allocates device memory.

Some callers cannot call cudaMalloc: a serving engine whose own pool already holds the device
memory, a plug-in that must not keep a context object, or a latency-critical path that cannot
afford cudaMalloc's device-wide synchronisation. For them the library keeps the GEMM's scratch in
a static array of its own. This test calls that entry point straight through the C ABI (ctypes,
no context object) and checks, on two calls in a row, that its output matches the ordinary
context-based fast GEMM (aipu_q4k_gemm) within the fast-GEMM tolerance used by the other tests
(here: at most 1 bf16 ulp apart), and that the oracle bar holds. The second call checks that the
shared scratch left behind by the first call does not leak into the next result.

The file name makes pytest collect it last, so a run that stops at its first failure has already
run every other test; it passes alone in a fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from aipu_b200 import _lib
from aipu_b200 import formats as F
from aipu_b200 import ops
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu

F32 = np.float32


def _bf16_np(t):
    return (t.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(F32)


@pytest.mark.parametrize("wt,N,K,M,xdt", [(F.Q4_K, 2048, 6144, 1, "bf16"), (F.Q6_K, 300, 2048, 3, "bf16"),
                                          (F.Q4_K, 40, 512, 9, "bf16"), (F.Q4_K, 300, 512, 6, "f32"),
                                          (F.Q8_0, 260, 1024, 2, "bf16"), (F.F16, 130, 768, 5, "f32")])
def test_noalloc_gemm_matches_context_gemm_twice(wt, N, K, M, xdt):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    L = _lib.lib()
    w_np = F.random_rows_np(wt, N, K, seed=77 + N)
    x_np = np.random.default_rng(5 + M).standard_normal((M, K)).astype(F32)
    if xdt == "bf16":
        x_np = qo.bf16_round(x_np)
        x = torch.from_numpy((x_np.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(d).view(torch.bfloat16)
        dt = _lib.DT_BF16
    else:  # fp32 activations: the entry point splits M into blocks of 4 tokens of 4-byte elements
        x = torch.from_numpy(x_np).to(d)
        dt = _lib.DT_F32
    w = torch.from_numpy(w_np).to(d)
    ref_ctx = ops.gemm(wt, w, N, K, x)  # the existing entry point, with a context workspace
    ref = qo.gemm(wt, w_np, N, K, x_np)
    stream = ctypes.c_void_p(torch.cuda.current_stream(d).cuda_stream)
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=d)
        rc = L.aipu_q4k_gemm_noalloc(wt, ctypes.c_void_p(w.data_ptr()), N, K, ctypes.c_void_p(x.data_ptr()),
                                     dt, M, ctypes.c_void_p(y.data_ptr()), stream)
        _lib.check(rc)
        torch.cuda.synchronize()
        status = ctypes.c_int(-1)
        _lib.check(L.aipu_q4k_gemm_noalloc_status(ctypes.byref(status)))
        assert status.value == 0, "a bounded wait in the kernel gave up"
        got = _bf16_np(y)
        assert qo.ulp_diff_bf16(got, _bf16_np(ref_ctx)).max() <= 1
        st = qo.parity_stats(got, ref)
        assert st["frac_within_1ulp"] >= 0.999 and st["max_rel"] <= 1e-2, st


def test_noalloc_gemm_rejects_rows_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _lib.lib()
    d = torch.device("cuda", 0)
    buf = torch.zeros(16, dtype=torch.uint8, device=d)
    rc = L.aipu_q4k_gemm_noalloc(F.Q4_K, ctypes.c_void_p(buf.data_ptr()), 65537, 256, ctypes.c_void_p(buf.data_ptr()),
                                 _lib.DT_BF16, 1, ctypes.c_void_p(buf.data_ptr()), None)
    assert rc == _lib.AIPU_EINVAL
    assert b"65536" in L.aipu_last_error()
