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


@pytest.mark.parametrize("M,down_wt", [(96, F.Q6_K), (200, F.Q4_K)])
def test_moe_prefill_layer_matches_oracle(M, down_wt):
    """The many-token MoE path (router, per-expert token lists, tensor-core SwiGLU and down
    projections grouped by expert, shared expert, slot-order combine) against the oracle layer:
    routing bit-exact, outputs within the reference's SwiGLU tolerance (tools/swiglu_q4k_gen.py:91-95)."""
    from oracle import moe_oracle as mo

    d = _dev()
    H, Fd, E, T = 512, 512, 16, 4
    rng = np.random.default_rng(M)
    gate = F.random_rows_np(F.Q4_K, (E + 1) * Fd, H, seed=1).reshape(E + 1, Fd, -1)
    up = F.random_rows_np(F.Q4_K, (E + 1) * Fd, H, seed=2).reshape(E + 1, Fd, -1)
    down = F.random_rows_np(down_wt, (E + 1) * H, Fd, seed=3).reshape(E + 1, H, -1)
    wr = rng.normal(0, 0.02, (H, E)).astype(F32)
    bias = rng.normal(0, 0.01, E).astype(F32)
    x = qo.bf16_round(rng.standard_normal((M, H)).astype(F32))
    tod = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(d)  # noqa: E731
    W = ops.MoeLayerWeights(hidden=H, ffn=Fd, n_experts=E, topk=T, router_wtype=F.F32, router_w=tod(wr),
                            router_bias=tod(bias), gate_w=tod(gate[:E]), up_w=tod(up[:E]), down_w=tod(down[:E]),
                            gate_wtype=F.Q4_K, down_wtype=down_wt, shared_gate_w=tod(gate[E]),
                            shared_up_w=tod(up[E]), shared_down_w=tod(down[E]))
    y, sel, sw = ops.moe_layer(W, _bf16_dev(x), return_routing=True)
    torch.cuda.synchronize()

    def deq(e):
        return (qo.dequant_rows(F.Q4_K, gate[e], Fd, H), qo.dequant_rows(F.Q4_K, up[e], Fd, H),
                qo.dequant_rows(down_wt, down[e], H, Fd))

    y_ref, sel_ref, sw_ref, mag = mo.moe_layer(x, wr.T.copy(), deq, deq(E), T, bias=bias, want_mag=True)
    assert np.array_equal(sel.cpu().numpy(), sel_ref)
    assert np.array_equal(_bf16_np(sw).view(np.uint32), sw_ref.view(np.uint32))
    got = _bf16_np(y).astype(np.float64)
    ref = y_ref.astype(np.float64)
    tol = np.maximum(np.maximum(0.06 * np.abs(ref), 0.02 * mag), 0.03)
    st = qo.parity_stats(got.astype(F32), y_ref)
    assert not (np.abs(got - ref) > tol).any(), st
    assert st["frac_within_1ulp"] >= 0.97, st
