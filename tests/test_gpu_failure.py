"""Failure detection without a GPU fault: a bounded device wait that nothing releases runs out at a
short, test-set limit; the kernel returns, the context's status word reports it through the C ABI
(aipu_ctx_status), and the same context keeps working afterwards."""
import numpy as np
import pytest
import torch

from aipu_b200 import formats as F
from aipu_b200 import ops
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    ctx = ops.Context(d)
    assert ctx.status() == 0
    ctx.set_wait_limit(2_000_000)  # about 1 ms of SM clock
    ctx.selftest_wait()
    torch.cuda.synchronize()
    assert ctx.status() == 1  # ST_TIMEOUT_FULL: a wait for data gave up
    assert ctx.status() == 0  # reading resets it
    # the context and the device stay usable: an exact GEMM on the same context
    w = F.random_rows_np(F.Q4_K, 256, 1024, seed=1)
    x = qo.bf16_round(np.random.default_rng(1).standard_normal((1, 1024)).astype(np.float32))
    xb = torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(d).view(torch.bfloat16)
    y = ops.gemm(F.Q4_K, torch.from_numpy(w).to(d), 256, 1024, xb, mode="strict", ctx=ctx)
    torch.cuda.synchronize()
    got = (y.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(got.view(np.uint32), qo.gemm(F.Q4_K, w, 256, 1024, x).view(np.uint32))
    assert ctx.status() == 0
    ctx.set_wait_limit(0)
    ctx.close()
