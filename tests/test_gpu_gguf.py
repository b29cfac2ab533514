"""GGUF checkpoints through the CUDA path: tensors of the reference-written file dequantise on the
GPU to the reference's fp32 values, and a MoE layer loaded from a GGUF equals the oracle layer
(strict mode bit for bit) built from the same file."""
import os

import numpy as np
import pytest
import torch

from aipu_b200 import gguf
from aipu_b200 import ops
from oracle import moe_oracle as mo
from oracle import q4k_oracle as qo

pytestmark = pytest.mark.gpu
F32 = np.float32
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def test_reference_gguf_dequant_on_gpu(golden):
    d = _dev()
    g = golden("gguf_golden")
    with gguf.GGUFFile(os.path.join(GOLDEN, "ref_synthetic.gguf")) as gf:
        for i, name in enumerate(str(n) for n in g["names"]):
            if f"t{i}_deq" not in g:
                continue
            t = gf.info(name)
            K, N = t.ne
            out = ops.dequant(t.wtype, gf.to_device(name, d), N, K)
            assert np.array_equal(out.cpu().numpy().view(np.uint32), g[f"t{i}_deq"]), name


@pytest.mark.parametrize("M", [1, 3])
def test_moe_layer_from_gguf_strict_matches_oracle(tmp_path, M):
    d = _dev()
    p = str(tmp_path / "moe.gguf")
    H, Fd, E, T = 512, 256, 16, 4
    gguf.synthetic_moe_gguf(p, layers=1, H=H, Fd=Fd, E=E, topk=T, seed=11)
    with gguf.GGUFFile(p) as gf:
        W = gguf.load_moe_layer(gf, 0, d)
        n = gguf.moe_names(0)
        gv = np.array(gf.raw(n["gate"])).reshape(E, Fd, -1)
        uv = np.array(gf.raw(n["up"])).reshape(E, Fd, -1)
        dv = np.array(gf.raw(n["down"])).reshape(E, H, -1)
        wr_t = np.array(gf.raw(n["router"])).view(F32).reshape(E, H)
        bias = np.array(gf.raw(n["bias"])).view(F32).reshape(E)
        shared = (qo.dequant_rows(W.gate_wtype, np.array(gf.raw(n["shared_gate"])), Fd, H),
                  qo.dequant_rows(W.gate_wtype, np.array(gf.raw(n["shared_up"])), Fd, H),
                  qo.dequant_rows(W.down_wtype, np.array(gf.raw(n["shared_down"])), H, Fd))

    def deq(e):
        return (qo.dequant_rows(W.gate_wtype, gv[e], Fd, H), qo.dequant_rows(W.gate_wtype, uv[e], Fd, H),
                qo.dequant_rows(W.down_wtype, dv[e], H, Fd))

    x = qo.bf16_round(np.random.default_rng(5 + M).standard_normal((M, H)).astype(F32))
    xd = torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(d).view(torch.bfloat16)
    ctx = ops.Context(d).set_flags(strict=True)
    y, sel, sw = ops.moe_layer(W, xd, ctx=ctx, return_routing=True)
    torch.cuda.synchronize()
    y_ref, sel_ref, sw_ref = mo.moe_layer(x, wr_t, deq, shared, T, bias=bias)
    assert np.array_equal(sel.cpu().numpy(), sel_ref)
    got = (y.view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16)
    assert np.array_equal(got, y_ref.view(np.uint32))
