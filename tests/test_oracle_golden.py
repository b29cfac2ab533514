"""Pins the CPU oracle (oracle/) to the reference's own outputs stored in tests/golden/.

Every fixture was produced by running the reference's unchanged modules
(tools/q4k_ref.py, tools/glm_model_q4k_ref.py, tools/q4k_matmul_gen.py, tools/q4k_mixed_gen.py);
see tests/golden/make_golden.py. All comparisons are bit-exact.
"""
import numpy as np
import pytest

from oracle import moe_oracle as mo
from oracle import q4k_oracle as qo

F32 = np.float32


def bits(a):
    return np.asarray(a, F32).view(np.uint32)


def test_dequant_q4k_bitexact(golden):
    g = golden("dequant_golden")
    y = qo.dequant_q4k(g["q4k_blocks"])
    assert np.array_equal(bits(y), g["q4k_y"])


def test_dequant_q6k_bitexact(golden):
    g = golden("dequant_golden")
    assert np.array_equal(bits(qo.dequant_q6k(g["q6k_blocks"])), g["q6k_y"])


def test_dequant_q80_bitexact(golden):
    g = golden("dequant_golden")
    assert np.array_equal(bits(qo.dequant_q80(g["q80_blocks"])), g["q80_y"])


def test_dequant_f16_all_patterns(golden):
    g = golden("dequant_golden")
    y = qo.dequant_f16(g["f16_bits"].view(np.uint8))
    assert np.array_equal(bits(y), g["f16_y"])


def test_scale_pack_roundtrip():
    rng = np.random.default_rng(3)
    for _ in range(200):
        scs = [int(v) for v in rng.integers(0, 64, 8)]
        mns = [int(v) for v in rng.integers(0, 64, 8)]
        sc, m = qo.scale_min_k4(np.array(qo.pack_6bit_scales(scs, mns), np.uint8))
        assert list(sc) == scs and list(m) == mns


@pytest.mark.parametrize("ci", range(10))
def test_gemm_seq_bitexact(golden, ci):
    g = golden("gemm_golden")
    wt, N, K, M = g[f"c{ci}_meta"]
    wdeq = qo.dequant_rows(int(wt), g[f"c{ci}_w"], int(N), int(K))
    assert np.array_equal(bits(wdeq), g[f"c{ci}_wdeq"])
    x = g[f"c{ci}_x"].view(F32)
    y = qo.matmul_seq(x, wdeq)
    assert np.array_equal(bits(y), g[f"c{ci}_y"])


def test_gemm_fp32_activations(golden):
    g = golden("gemm_golden")
    wt, N, K, M = g["f32x_meta"]
    y = qo.gemm(int(wt), g["f32x_w"], int(N), int(K), g["f32x_x"].view(F32))
    assert np.array_equal(bits(y), g["f32x_y"])


def test_reference_matmul_generator_vectors(golden):
    """tools/q4k_matmul_gen.py's own seeded vectors (committed K list + real-dims list)."""
    g = golden("refvec_golden")
    for i in range(int(g["n_mm"])):
        wt, N, K, M, _ = g[f"mm{i}_meta"]
        x = qo.bf16_from_bits(g[f"mm{i}_a"])
        y = qo.gemm(0, g[f"mm{i}_w"], int(N), int(K), x)
        assert np.array_equal(qo.bf16_bits(y), g[f"mm{i}_c"]), f"vector {i}"


def test_reference_mixed_generator_vectors(golden):
    """tools/q4k_mixed_gen.py emit_mixed_gemm tiles (columns of all four types)."""
    g = golden("refvec_golden")
    for t in range(int(g["n_mx"])):
        K, PE_M, PE_N = (int(v) for v in g[f"mx{t}_meta"])
        x = qo.bf16_from_bits(g[f"mx{t}_a"])
        for pj, wt in enumerate(g[f"mx{t}_types"]):
            y = qo.gemm(int(wt), g[f"mx{t}_w{pj}"], 1, K, x)
            assert np.array_equal(qo.bf16_bits(y[:, 0]), g[f"mx{t}_c"][:, pj]), (t, pj)


def test_sigmoid_silu_all_bf16(golden):
    g = golden("act_golden")
    xs = qo.bf16_from_bits(np.arange(65536))
    assert np.array_equal(qo.bf16_bits(mo.glm_sigmoid(xs)), g["sigmoid"])
    assert np.array_equal(qo.bf16_bits(mo.glm_silu(xs)), g["silu"])


def test_rsqrt(golden):
    g = golden("act_golden")
    y = mo.fp32_rsqrt(g["rsqrt_in"].view(F32))
    assert np.array_equal(bits(y), g["rsqrt_out"])


@pytest.mark.parametrize("name", ["r8", "r256"])
def test_router_reference(golden, name):
    g = golden("moe_golden")
    E, T, D = (int(v) for v in g[f"{name}_meta"])
    wdeq = qo.dequant_rows(0, g[f"{name}_w"], E, 256)
    x = g[f"{name}_x"].view(F32)
    xp = np.zeros((x.shape[0], 256), F32)
    xp[:, :D] = x
    sel, sw, gate = mo.moe_router(xp, wdeq, T)
    assert np.array_equal(sel, g[f"{name}_sel"])
    assert np.array_equal(bits(sw), g[f"{name}_sw"])
    assert np.array_equal(bits(gate), g[f"{name}_gate"])


def test_moe_layer_reference(golden):
    g = golden("moe_golden")
    E, T, D, F = (int(v) for v in g["moe_meta"])
    x = g["moe_x"].view(F32)
    rdeq = qo.dequant_rows(0, g["moe_router_w"], E, 256)

    def deq(e):
        wg = qo.dequant_rows(0, g["moe_gate_w"][e], F, 256)
        wu = qo.dequant_rows(0, g["moe_up_w"][e], F, 256)
        wd = qo.dequant_rows(0, g["moe_down_w"][e], D, 256)[:, :F]
        return wg, wu, wd

    out, sel, sw = mo.moe_layer(x, rdeq, deq, deq(E), T)
    assert np.array_equal(sel, g["moe_sel"])
    assert np.array_equal(bits(sw), g["moe_sw"])
    assert np.array_equal(bits(out), g["moe_y"])


@pytest.mark.parametrize("ci", range(10))
def test_c_oracle_matches_reference_fixtures(golden, ci):
    """The C restatement (CPU baseline) is bit-exact to the reference too, for any thread count."""
    from oracle import cpu

    g = golden("gemm_golden")
    wt, N, K, M = (int(v) for v in g[f"c{ci}_meta"])
    x = g[f"c{ci}_x"].view(F32)
    for nt in (1, 3):
        y = cpu.gemm(wt, g[f"c{ci}_w"], N, K, x, nthreads=nt)
        assert np.array_equal(bits(y), g[f"c{ci}_y"])
    row = cpu.dequant_row(wt, g[f"c{ci}_w"][0], K)
    assert np.array_equal(bits(row), g[f"c{ci}_wdeq"][0])


def test_c_oracle_dequant_edge_blocks(golden):
    from oracle import cpu

    g = golden("dequant_golden")
    for name, wt, bw in (("q4k", 0, 256), ("q6k", 1, 256), ("q80", 2, 32)):
        blocks = g[f"{name}_blocks"]
        y = np.stack([cpu.dequant_row(wt, b, bw) for b in blocks])
        assert np.array_equal(bits(y), g[f"{name}_y"])
    y = cpu.dequant_row(3, g["f16_bits"].view(np.uint8), g["f16_bits"].size)
    assert np.array_equal(bits(y), g["f16_y"])


def test_bf16_dot7_oracle_matches_reference_fixture(golden):
    """The vectorised bf16 dot (LM-head contract) equals the reference's matmul_bf16_dot."""
    g = golden("lmhead_golden")
    for c in ("a", "b", "c"):
        x = (g[f"{c}_x"].astype(np.uint32) << 16).view(np.float32)
        w = (g[f"{c}_w"].astype(np.uint32) << 16).view(np.float32)
        y = mo.bf16_dot7(x, w)
        assert np.array_equal((y.view(np.uint32) >> 16).astype(np.uint16), g[f"{c}_y"]), c


def test_moe_layer_packed_reference(golden):
    """The full-size oracle layer (C-restatement GEMMs on packed rows) equals the reference's MoE
    branch bit for bit (F padded to 256 with zero gate/up rows, which leave h and y unchanged)."""
    g = golden("moe_golden")
    E, T, D, Fd = (int(v) for v in g["moe_meta"])
    Fp = 256
    gate = np.zeros((E + 1, Fp, 144), np.uint8)
    up = np.zeros((E + 1, Fp, 144), np.uint8)
    gate[:, :Fd] = g["moe_gate_w"]
    up[:, :Fd] = g["moe_up_w"]
    down = g["moe_down_w"]
    x = g["moe_x"].view(F32)
    rrows = qo.dequant_rows(0, g["moe_router_w"], E, 256)
    out, sel, sw = mo.moe_layer_packed(x, rrows, lambda e: (gate[e], up[e], down[e]), (gate[E], up[E], down[E]), T,
                                       gate_wtype=0, down_wtype=0)
    assert np.array_equal(sel, g["moe_sel"])
    assert np.array_equal(bits(sw), g["moe_sw"])
    assert np.array_equal(bits(out), g["moe_y"])
