"""The parity comparators reject real bugs (the reference's rule that every "it passes" claim is paired
with an injected fault that a real bug fails, README.md:109-111).

Each case builds the output a plausible kernel bug would produce -- swapped nibble halves, a dropped
dmin term, an off-by-one sub-block scale index, a byte-swapped fp16 scale, outputs 2 bf16 ulps off --
and checks that the bar the GPU tests use rejects it: bit equality for dequant and strict paths, and
(>= 99.9 % within 1 bf16 ulp, max relative error <= 1e-2) for the tensor-core GEMM.
"""
import numpy as np
import pytest

from aipu_b200 import formats as F
from oracle import q4k_oracle as qo

F32 = np.float32
N, K = 256, 1024


def fast_bar(got, ref) -> bool:
    st = qo.parity_stats(got, ref)
    return st["frac_within_1ulp"] >= 0.999 and st["max_rel"] <= 1e-2


def exact(got, ref) -> bool:
    return np.array_equal(np.asarray(got, F32).view(np.uint32), np.asarray(ref, F32).view(np.uint32))


def _deq_q4k_mut(blocks, kind):
    """Q4_K dequant with one injected bug (a numpy rewrite of tools/q4k_ref.py:39-61 plus the bug)."""
    b = np.asarray(blocks, np.uint8).reshape(-1, 144)
    dh = b[:, 0:2].copy()
    if kind == "fp16_byteswap":
        dh = dh[:, ::-1].copy()
    d = dh.view(np.float16).astype(F32).reshape(-1)
    dm = b[:, 2:4].copy().view(np.float16).astype(F32).reshape(-1)
    sc, mn = qo.scale_min_k4(b[:, 4:16])
    if kind == "scale_index_off_by_one":
        sc = np.roll(sc, -1, axis=1)
    qs = b[:, 16:]
    y = np.empty((b.shape[0], 256), F32)
    with np.errstate(invalid="ignore", over="ignore"):
        _fill(y, d, dm, sc, mn, qs, kind)
    return y


def _fill(y, d, dm, sc, mn, qs, kind):
    for g in range(4):
        lo, hi = qs[:, 32 * g:32 * g + 32] & 0xF, qs[:, 32 * g:32 * g + 32] >> 4
        if kind == "swapped_nibbles":
            lo, hi = hi, lo
        for j, q in ((2 * g, lo), (2 * g + 1, hi)):
            d1 = d * sc[:, j].astype(F32)
            m1 = dm * mn[:, j].astype(F32)
            t = d1[:, None] * q.astype(F32)
            y[:, 32 * j:32 * j + 32] = t if kind == "dropped_dmin" else t - m1[:, None]


@pytest.fixture(scope="module")
def case():
    w = F.random_rows_np(F.Q4_K, N, K, seed=99)
    x = qo.bf16_round(np.random.default_rng(5).standard_normal((2, K)).astype(F32))
    ref_deq = qo.dequant_rows(F.Q4_K, w, N, K)
    ref_y = qo.matmul_seq(x, ref_deq)
    return w, x, ref_deq, ref_y


def test_unmutated_restatement_passes(case):
    w, x, ref_deq, ref_y = case
    deq = _deq_q4k_mut(w.reshape(-1, 144), "none").reshape(N, K)
    assert exact(deq, ref_deq)
    assert exact(qo.matmul_seq(x, deq), ref_y) and fast_bar(ref_y, ref_y)


@pytest.mark.parametrize("kind", ["swapped_nibbles", "dropped_dmin", "scale_index_off_by_one", "fp16_byteswap"])
def test_dequant_and_gemm_mutations_are_rejected(case, kind):
    w, x, ref_deq, ref_y = case
    deq = _deq_q4k_mut(w.reshape(-1, 144), kind).reshape(N, K)
    assert not exact(deq, ref_deq), kind
    y = qo.matmul_seq(x, deq)
    assert not exact(y, ref_y), kind
    assert not fast_bar(y, ref_y), kind


def test_two_ulp_perturbation_is_rejected(case):
    """2 bf16 ulps on 0.5 % of the outputs (more than the 0.1 % the bar allows beyond 1 ulp)."""
    _, _, _, ref_y = case
    u = (ref_y.view(np.uint32) >> 16).astype(np.int64)
    flat = u.reshape(-1).copy()
    idx = np.random.default_rng(3).choice(flat.size, flat.size // 200, replace=False)
    flat[idx] += np.where(flat[idx] & 0x8000, -2, 2)
    y = ((flat.reshape(u.shape).astype(np.uint32) & 0xFFFF) << 16).view(F32)
    assert qo.parity_stats(y, ref_y)["max_ulp"] == 2
    assert not fast_bar(y, ref_y)
    assert not exact(y, ref_y)


def test_one_ulp_noise_within_the_bar_is_accepted(case):
    """The bar is not vacuous the other way either: 1-ulp differences on 5 % of outputs pass it."""
    _, _, _, ref_y = case
    u = (ref_y.view(np.uint32) >> 16).astype(np.int64).reshape(-1).copy()
    idx = np.random.default_rng(4).choice(u.size, u.size // 20, replace=False)
    u[idx] += 1
    y = ((u.reshape(ref_y.shape).astype(np.uint32) & 0xFFFF) << 16).view(F32)
    assert fast_bar(y, ref_y) and not exact(y, ref_y)
