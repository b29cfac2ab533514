"""Two devices in one process: every kernel whose launcher sets a per-function attribute (the router's
and the GEMMs' dynamic shared memory, the SiLU table) must work on the second device too. Contexts on
devices 0 and 1 run the router (both the few-token and the many-token kernel), the tcgen05 GEMM, the
decode GEMV, the exact chain GEMV and the bf16 dot GEMV on the same inputs; the deterministic kernels
must give the same bits on both devices. Skipped with fewer than two devices."""
import numpy as np
import pytest
import torch

from aipu_b200 import formats as F
from aipu_b200 import ops

pytestmark = pytest.mark.gpu


def _devs():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    return torch.device("cuda", 0), torch.device("cuda", 1)


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


def _run(d, seed_w, x_cpu):
    with torch.cuda.device(d):
        ctx = ops.Context(d)
        out = {}
        g = torch.Generator().manual_seed(seed_w)
        H, E = 1024, 64
        wr = (torch.randn((H, E), generator=g) * 0.02).to(d)
        bias = (torch.randn((E,), generator=g) * 0.01).to(d)
        for M in (1, 40):
            x = x_cpu[:M].to(d)
            sel, sw, gate = ops.moe_router(F.F32, wr, x, E, 4, bias=bias, ctx=ctx)
            out[f"router{M}"] = (sel.cpu().numpy(), _bits(sw), _bits(gate))
        w = torch.from_numpy(F.random_rows_np(F.Q4_K, 256, H, seed=seed_w)).to(d)
        x1 = x_cpu[:1].to(d)
        out["gemv"] = _bits(ops.gemm(F.Q4_K, w, 256, H, x1, ctx=ctx))
        out["chain"] = _bits(ops.gemm(F.Q4_K, w, 256, H, x1, mode="strict", ctx=ctx))
        out["tc"] = _bits(ops.gemm_tc(F.Q4_K, w, 256, H, x_cpu[:96].to(d), ctx=ctx))
        wb = (torch.randn((512, H), generator=g)).to(torch.bfloat16).to(d)
        out["dot"] = _bits(ops.bf16_dot_gemv(wb, x_cpu[:2].to(d), ctx=ctx))
        torch.cuda.synchronize(d)
        ctx.close()
    return out


def test_kernels_on_two_devices_agree():
    d0, d1 = _devs()
    x = torch.randn((96, 1024), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    a = _run(d0, 11, x)
    b = _run(d1, 11, x)
    for k in a:
        if isinstance(a[k], tuple):
            for u, v in zip(a[k], b[k]):
                assert np.array_equal(u, v), k
        else:
            assert np.array_equal(a[k], b[k]), k
