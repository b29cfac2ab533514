"""The drop-in modules aipu_b200.q4k_ref and aipu_b200.glm_model_q4k_ref, called exactly like the
reference's tools/q4k_ref.py and tools/glm_model_q4k_ref.py, against the golden outputs those
reference modules produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from aipu_b200 import glm_model_q4k_ref as G
from aipu_b200 import q4k_ref as R
from oracle import q4k_oracle as qo

F32 = np.float32


def _f(bits):
    return np.asarray(bits, np.uint32).view(F32)


def _qw_from_rows(rows, nin):
    """GGUF Q4_K rows [nout, 144] (one block per column) -> a QW as the reference builds it."""
    nout = rows.shape[0]
    codes, d, dmin, scales = [], [], [], []
    for o in range(nout):
        b = rows[o]
        qs = b[16:144]
        c = np.zeros(256, np.int64)
        for g in range(4):
            c[64 * g:64 * g + 32] = qs[32 * g:32 * g + 32] & 0xF
            c[64 * g + 32:64 * g + 64] = qs[32 * g:32 * g + 32] >> 4
        codes.append([int(v) for v in c[:nin]])
        d.append(int(b[0]) | (int(b[1]) << 8))
        dmin.append(int(b[2]) | (int(b[3]) << 8))
        scales.append([int(v) for v in b[4:16]])
    return G.QW(nout, nin, codes, d, dmin, scales)


# ------------------------------------------------------------------ host-side helpers (CPU)
def test_host_helpers_match_oracle(golden):
    g = golden("dequant_golden")
    blk = g["q4k_blocks"][5]
    sc, mn = qo.scale_min_k4(blk[4:16])
    for j in range(8):
        assert R.get_scale_min_k4(j, [int(v) for v in blk[4:16]]) == (int(sc[j]), int(mn[j]))
    for v in (0.0, 1.0, -3.25e-3, 1e30, float("inf"), 7.0000005):
        assert R.bf16_round(v).view(np.uint32) == qo.bf16_round(np.array([v], F32))[0].view(np.uint32)
    scs, mns = [1, 63, 5, 0, 17, 33, 2, 60], [0, 7, 63, 8, 9, 31, 32, 1]
    packed = R._pack_6bit_scales(scs, mns)
    assert [R.get_scale_min_k4(j, packed) for j in range(8)] == list(zip(scs, mns))


def test_compute_calls_fail_loudly_without_cuda():
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    with pytest.raises(RuntimeError):
        R.dequantize_block_q8_0(0x3C00, [1] * 32)


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_dropin_dequant_blocks(golden):
    g = golden("dequant_golden")
    for i in range(0, 208, 37):
        b = g["q4k_blocks"][i]
        y = R.dequantize_block_q4_K(int(b[0]) | (int(b[1]) << 8), int(b[2]) | (int(b[3]) << 8), list(b[4:16]),
                                    list(b[16:]))
        assert np.array_equal(y.view(np.uint32), g["q4k_y"][i])
    rows = [(int(b[0]) | (int(b[1]) << 8), int(b[2]) | (int(b[3]) << 8), bytes(b[4:16]), bytes(b[16:]))
            for b in g["q4k_blocks"][:6]]
    assert np.array_equal(R.dequantize_row_q4_K(rows).view(np.uint32), g["q4k_y"][:6].reshape(-1))
    for i in range(0, 303, 61):
        b = g["q6k_blocks"][i]
        y = R.dequantize_block_q6_K(int(b[208]) | (int(b[209]) << 8), list(b[:128]), list(b[128:192]),
                                    [R._s8(int(v)) for v in b[192:208]])
        assert np.array_equal(y.view(np.uint32), g["q6k_y"][i])
    for i in range(0, 300, 59):
        b = g["q80_blocks"][i]
        y = R.dequantize_block_q8_0(int(b[0]) | (int(b[1]) << 8), [R._s8(int(v)) for v in b[2:]])
        assert np.array_equal(y.view(np.uint32), g["q80_y"][i])


@pytest.mark.gpu
def test_dropin_matmul_contract(golden):
    g = golden("gemm_golden")
    x = _f(g["c1_x"])
    wdeq = _f(g["c1_wdeq"])
    y = _f(g["c1_y"])
    for m in range(x.shape[0]):
        for n in range(wdeq.shape[0]):
            assert R.matmul_q4k_col(x[m], wdeq[n]).view(np.uint32) == y[m, n].view(np.uint32)
        got = np.array(G.matmul_q4k(list(x[m]), list(wdeq)), F32)
        assert np.array_equal(got.view(np.uint32), y[m].view(np.uint32))


@pytest.mark.gpu
def test_dropin_activations(golden):
    g = golden("act_golden")
    xs = (np.arange(0, 65536, 997, dtype=np.uint32) << 16).view(F32)
    sig = np.asarray(G.glm_sigmoid(xs), F32)
    silu = np.asarray(G.glm_silu(xs), F32)
    assert np.array_equal((sig.view(np.uint32) >> 16).astype(np.uint16), g["sigmoid"][::997])
    assert np.array_equal((silu.view(np.uint32) >> 16).astype(np.uint16), g["silu"][::997])
    assert (G.glm_silu(F32(0.5)).view(np.uint32) >> 16) == g["silu"][0x3F00]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["r8", "r256"])
def test_dropin_moe_router_fixture(golden, name):
    g = golden("moe_golden")
    E, T, D = (int(v) for v in g[f"{name}_meta"])
    cfg = G.Config(N_EXPERT=E, TOPK=T, MODEL_DIM=D)
    Wg = _qw_from_rows(g[f"{name}_w"], D)
    for t in range(0, 24, 5):
        x = list(_f(g[f"{name}_x"][t]))
        sel, sw, gate = G.moe_router(cfg, x, Wg)
        assert sel == [int(v) for v in g[f"{name}_sel"][t]]
        assert np.array_equal(np.array(sw, F32).view(np.uint32), g[f"{name}_sw"][t])
        assert np.array_equal(np.array(gate, F32).view(np.uint32), g[f"{name}_gate"][t])


@pytest.mark.gpu
def test_dropin_swiglu_expert_fixture(golden):
    g = golden("moe_golden")
    E, T, D, Fd = (int(v) for v in g["moe_meta"])
    cfg = G.Config(N_EXPERT=E, TOPK=T, MODEL_DIM=D, INTER_MOE=Fd)
    for t in range(3):
        x = list(_f(g["moe_x"][t]))
        experts = [int(v) for v in g["moe_sel"][t]] + [E]  # the selected experts, then the shared one
        for slot, e in enumerate(experts[:2] + [E]):
            idx = slot if e != E else T
            Wgate = _qw_from_rows(g["moe_gate_w"][e], D)
            Wup = _qw_from_rows(g["moe_up_w"][e], D)
            Wdown = _qw_from_rows(g["moe_down_w"][e][:D], Fd)
            y = G.swiglu_expert(cfg, x, Wgate, Wup, Wdown)
            assert np.array_equal(np.array(y, F32).view(np.uint32), g["moe_yslots"][t, idx])


@pytest.mark.gpu
def test_dropin_matmul_bf16_dot_fixture(golden):
    """matmul_bf16_dot(a_bf, w_bf) as the reference calls it (LM head), against its own outputs."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = golden("lmhead_golden")
    for c in ("b", "c"):
        x = (g[f"{c}_x"].astype(np.uint32) << 16).view(F32)
        w = (g[f"{c}_w"].astype(np.uint32) << 16).view(F32)
        y = (g[f"{c}_y"].astype(np.uint32) << 16).view(F32)
        for v in range(min(4, w.shape[0])):
            got = G.matmul_bf16_dot(list(x[0]), list(w[v]))
            assert np.float32(got).view(np.uint32) == y[0, v].view(np.uint32), (c, v)
