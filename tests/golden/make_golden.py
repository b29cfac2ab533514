#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own code.

Run once, in a checkout where the Wick-Lim/AIPU tree is available:

    AIPU_REFERENCE=/path/to/AIPU python tests/golden/make_golden.py

It imports the reference's ``tools/q4k_ref.py``, ``tools/glm_model_q4k_ref.py``,
``tools/q4k_matmul_gen.py`` and ``tools/q4k_mixed_gen.py`` unchanged, runs their seeded
generators and scalar goldens, and stores inputs and outputs as small .npz files. The tests and
the GPU parity checks read only these files (the reference tree is not needed at test time).

Weight bytes are stored in the GGUF block layout the library consumes (rows of super-blocks);
where a reference generator emits per-weight codes, they are packed back into ggml blocks by
``pack_q4k`` / ``pack_q6k`` here, and the test re-checks that the packed bytes dequantise to the
reference's own fp32 values.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("AIPU_REFERENCE")
if not REF:
    sys.exit("set AIPU_REFERENCE to the root of the Wick-Lim/AIPU tree")
sys.path.insert(0, os.path.join(REF, "tools"))

import q4k_ref as R            # noqa: E402  (reference module, unchanged)
import glm_model_q4k_ref as G  # noqa: E402
import q4k_matmul_gen as MG    # noqa: E402
import q4k_mixed_gen as XG     # noqa: E402

F32 = np.float32


def f32bits(a):
    return np.asarray(a, F32).view(np.uint32).copy()


def f16b(x):
    return R._f32_to_f16bits(x)


# --------------------------------------------------------------- ggml block packers
def pack_q4k(d_h, dm_h, scales12, codes256):
    """One Q4_K super-block from (fp16 d, fp16 dmin, 12 scale bytes, 256 codes in weight order).
    Weight k of the block lives in qs[32*(k//64) + k%32], low nibble if (k%64)<32 else high
    (the packing the reference self-test uses, glm_model_q4k_ref.py:856-862)."""
    b = np.zeros(144, np.uint8)
    b[0:2] = np.frombuffer(np.uint16(d_h).tobytes(), np.uint8)
    b[2:4] = np.frombuffer(np.uint16(dm_h).tobytes(), np.uint8)
    b[4:16] = np.asarray(scales12, np.uint8)
    qs = np.zeros(128, np.uint8)
    for k in range(256):
        byte = 32 * (k // 64) + (k % 32)
        if (k % 64) < 32:
            qs[byte] |= codes256[k] & 0xF
        else:
            qs[byte] |= (codes256[k] & 0xF) << 4
    b[16:144] = qs
    return b


def pack_q6k(d_h, sc16, codes256):
    """One Q6_K super-block from 256 six-bit codes in ggml y-position order (the inverse of the
    reference's q4k_mixed_gen.q6k_codes)."""
    ql = np.zeros(128, np.uint8)
    qh = np.zeros(64, np.uint8)
    for half in range(2):
        bq, bh, by = half * 64, half * 32, half * 128
        for l in range(32):
            c1, c2, c3, c4 = (codes256[by + l + o] for o in (0, 32, 64, 96))
            ql[bq + l] = (c1 & 0xF) | ((c3 & 0xF) << 4)
            ql[bq + l + 32] = (c2 & 0xF) | ((c4 & 0xF) << 4)
            qh[bh + l] = ((c1 >> 4) & 3) | (((c2 >> 4) & 3) << 2) | (((c3 >> 4) & 3) << 4) | (((c4 >> 4) & 3) << 6)
    b = np.zeros(210, np.uint8)
    b[0:128] = ql
    b[128:192] = qh
    b[192:208] = np.asarray([s & 0xFF for s in sc16], np.uint8)
    b[208:210] = np.frombuffer(np.uint16(d_h).tobytes(), np.uint8)
    return b


def pack_q80(d_h, qs32):
    b = np.zeros(34, np.uint8)
    b[0:2] = np.frombuffer(np.uint16(d_h).tobytes(), np.uint8)
    b[2:34] = np.asarray([q & 0xFF for q in qs32], np.uint8)
    return b


# --------------------------------------------------------------- 1. dequant goldens
def gen_dequant():
    out = {}
    # Q4_K: the reference self-test's distribution (q4k_ref.py:150-182, seed 0) plus edge blocks
    rng = np.random.default_rng(0)
    blocks, ys = [], []
    for t in range(200):
        scs = [int(v) for v in rng.integers(0, 64, 8)]
        mns = [int(v) for v in rng.integers(0, 64, 8)]
        scales = R._pack_6bit_scales(scs, mns)
        qs = [int(v) for v in rng.integers(0, 256, 128)]
        d_h = f16b(rng.uniform(0.001, 0.05))
        dm_h = f16b(rng.uniform(0.0, 0.02))
        b = np.zeros(144, np.uint8)
        b[0:2] = np.frombuffer(np.uint16(d_h).tobytes(), np.uint8)
        b[2:4] = np.frombuffer(np.uint16(dm_h).tobytes(), np.uint8)
        b[4:16] = scales
        b[16:] = qs
        blocks.append(b)
        ys.append(R.dequantize_block_q4_K(d_h, dm_h, scales, qs))
    # edge blocks: fp16 subnormal / zero / negative / max d, all-63 scales, all-15 codes
    edge_d = [0x0001, 0x03FF, 0x0000, 0x8001, 0x7BFF, 0xBC00, 0x3C00, 0x0400]
    for i, dh in enumerate(edge_d):
        dm = edge_d[(i + 3) % len(edge_d)]
        scs = [63 if (i + j) % 2 else (j * 9) % 64 for j in range(8)]
        mns = [(j * 7 + i) % 64 for j in range(8)]
        scales = R._pack_6bit_scales(scs, mns)
        qs = [(0xFF if (k + i) % 3 == 0 else (k * 37 + i) % 256) for k in range(128)]
        b = np.zeros(144, np.uint8)
        b[0:2] = np.frombuffer(np.uint16(dh).tobytes(), np.uint8)
        b[2:4] = np.frombuffer(np.uint16(dm).tobytes(), np.uint8)
        b[4:16] = scales
        b[16:] = qs
        blocks.append(b)
        ys.append(R.dequantize_block_q4_K(dh, dm, scales, qs))
    out["q4k_blocks"] = np.stack(blocks)
    out["q4k_y"] = f32bits(np.stack(ys))

    # Q6_K / Q8_0: the mixed generator's block samplers (q4k_mixed_gen.py:56-100, seed 0x6C0FFEE)
    rng = np.random.default_rng(0x6C0FFEE)
    b6, y6 = [], []
    for _ in range(300):
        ql, qh, sc, dh = XG.rand_q6k_block(rng)
        b = np.zeros(210, np.uint8)
        b[0:128] = ql
        b[128:192] = qh
        b[192:208] = [s & 0xFF for s in sc]
        b[208:210] = np.frombuffer(np.uint16(dh).tobytes(), np.uint8)
        b6.append(b)
        y6.append(R.dequantize_block_q6_K(dh, ql, qh, [s & 0xFF for s in sc]))
    for dh in (0x0001, 0x8400, 0x7BFF):               # edge d values
        ql = [(k * 29) % 256 for k in range(128)]
        qh = [(k * 53) % 256 for k in range(64)]
        sc = [(-128 + 17 * j) for j in range(16)]
        b = np.zeros(210, np.uint8)
        b[0:128] = ql
        b[128:192] = qh
        b[192:208] = [s & 0xFF for s in sc]
        b[208:210] = np.frombuffer(np.uint16(dh).tobytes(), np.uint8)
        b6.append(b)
        y6.append(R.dequantize_block_q6_K(dh, ql, qh, [s & 0xFF for s in sc]))
    out["q6k_blocks"] = np.stack(b6)
    out["q6k_y"] = f32bits(np.stack(y6))
    b8, y8 = [], []
    for _ in range(300):
        dh, qs = XG.rand_q8_block(rng)
        b8.append(pack_q80(dh, qs))
        y8.append(R.dequantize_block_q8_0(dh, [q & 0xFF for q in qs]))
    out["q80_blocks"] = np.stack(b8)
    out["q80_y"] = f32bits(np.stack(y8))
    # F16: every fp16 bit pattern except NaNs, through numpy's widen (the reference's rule)
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    fin = ((pats >> 10) & 0x1F) != 0x1F
    pats = pats[fin | ((pats & 0x3FF) == 0)]
    out["f16_bits"] = pats
    out["f16_y"] = f32bits(pats.view(np.float16).astype(F32))
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **out)


# --------------------------------------------------------------- 2. GEMM goldens
def _rand_q4k_row(rng, K):
    """A Q4_K row with the BASELINE distribution: d,dmin = fp16(|N(0,1)|*2^-8), 6-bit
    scales/mins uniform 0..63, quant bytes uniform."""
    blocks = []
    for _ in range(K // 256):
        scales = R._pack_6bit_scales([int(v) for v in rng.integers(0, 64, 8)],
                                     [int(v) for v in rng.integers(0, 64, 8)])
        b = np.zeros(144, np.uint8)
        b[0:2] = np.frombuffer(np.uint16(f16b(abs(rng.standard_normal()) * 2 ** -8)).tobytes(), np.uint8)
        b[2:4] = np.frombuffer(np.uint16(f16b(abs(rng.standard_normal()) * 2 ** -8)).tobytes(), np.uint8)
        b[4:16] = scales
        b[16:] = rng.integers(0, 256, 128)
        blocks.append(b)
    return np.concatenate(blocks)


def _rand_q6k_row(rng, K):
    blocks = []
    for _ in range(K // 256):
        b = np.zeros(210, np.uint8)
        b[0:192] = rng.integers(0, 256, 192)
        b[192:208] = (rng.integers(-32, 32, 16) & 0xFF)
        b[208:210] = np.frombuffer(np.uint16(f16b(abs(rng.standard_normal()) * 2 ** -8)).tobytes(), np.uint8)
        blocks.append(b)
    return np.concatenate(blocks)


def _rand_q80_row(rng, K):
    blocks = []
    for _ in range(K // 32):
        blocks.append(pack_q80(f16b(abs(rng.standard_normal()) * 2 ** -8),
                               [int(v) for v in rng.integers(-128, 128, 32)]))
    return np.concatenate(blocks)


def _rand_f16_row(rng, K):
    return rng.normal(0, 0.02, K).astype(np.float16).view(np.uint8)


def _ref_dequant_row(wtype, row, K):
    if wtype == 0:
        ys = []
        for sb in range(K // 256):
            b = row[sb * 144:(sb + 1) * 144]
            dh = int(np.frombuffer(b[0:2].tobytes(), np.uint16)[0])
            dm = int(np.frombuffer(b[2:4].tobytes(), np.uint16)[0])
            ys.append(R.dequantize_block_q4_K(dh, dm, [int(v) for v in b[4:16]], [int(v) for v in b[16:]]))
        return np.concatenate(ys)
    if wtype == 1:
        ys = []
        for sb in range(K // 256):
            b = row[sb * 210:(sb + 1) * 210]
            dh = int(np.frombuffer(b[208:210].tobytes(), np.uint16)[0])
            ys.append(R.dequantize_block_q6_K(dh, [int(v) for v in b[0:128]], [int(v) for v in b[128:192]],
                                              [int(v) for v in b[192:208]]))
        return np.concatenate(ys)
    if wtype == 2:
        ys = []
        for i in range(K // 32):
            b = row[i * 34:(i + 1) * 34]
            dh = int(np.frombuffer(b[0:2].tobytes(), np.uint16)[0])
            ys.append(R.dequantize_block_q8_0(dh, [int(v) for v in b[2:34]]))
        return np.concatenate(ys)
    return row.view(np.float16).astype(F32)


def gen_gemm():
    """Seeded small GEMMs of every weight type with BASELINE-shaped distributions; outputs from the
    reference's scalar q4k_ref.matmul_q4k_col (sequential fp32 MAC, bf16 RNE)."""
    out = {}
    makers = {0: _rand_q4k_row, 1: _rand_q6k_row, 2: _rand_q80_row, 3: _rand_f16_row}
    cases = [(0, 8, 256, 3), (0, 8, 768, 2), (0, 6, 6144, 4), (1, 8, 512, 2), (1, 6, 2048, 4),
             (1, 4, 6144, 1), (2, 8, 256, 3), (2, 6, 6144, 4), (3, 8, 256, 2), (3, 4, 6144, 4)]
    for ci, (wt, N, K, M) in enumerate(cases):
        rng = np.random.default_rng(1000 + ci)
        W = np.stack([makers[wt](rng, K) for _ in range(N)])
        xb = np.array([[R.bf16_round(F32(v)) for v in rng.standard_normal(K)] for _ in range(M)], F32)
        wdeq = [_ref_dequant_row(wt, W[n], K) for n in range(N)]
        y = np.array([[R.matmul_q4k_col(xb[m], wdeq[n]) for n in range(N)] for m in range(M)], F32)
        out[f"c{ci}_meta"] = np.array([wt, N, K, M], np.int64)
        out[f"c{ci}_w"] = W
        out[f"c{ci}_x"] = f32bits(xb)
        out[f"c{ci}_wdeq"] = f32bits(np.stack(wdeq))
        out[f"c{ci}_y"] = f32bits(y)
    # C1-style case: fp32 activations ~N(0,1), Q4_K, K = 4096
    rng = np.random.default_rng(77)
    N, K = 8, 4096
    W = np.stack([_rand_q4k_row(rng, K) for _ in range(N)])
    xf = rng.standard_normal((1, K)).astype(F32)
    wdeq = [_ref_dequant_row(0, W[n], K) for n in range(N)]
    y = np.array([[R.matmul_q4k_col(xf[0], wdeq[n]) for n in range(N)]], F32)
    out["f32x_meta"] = np.array([0, N, K, 1], np.int64)
    out["f32x_w"] = W
    out["f32x_x"] = f32bits(xf)
    out["f32x_y"] = f32bits(y)
    out["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **out)


# --------------------------------------------------------------- 3. reference generator vectors
def _parse_matmul_gen(text):
    """Parse tools/q4k_matmul_gen.py output (its layout docstring, q4k_matmul_gen.py:6-13)."""
    tok = text.split("\n")
    ntest, PE_M, PE_N = map(int, tok[0].split())
    p = 1
    tests = []
    for _ in range(ntest):
        K, NSB = map(int, tok[p].split()); p += 1
        d = [int(v, 16) for v in tok[p].split()]; p += 1
        dm = [int(v, 16) for v in tok[p].split()]; p += 1
        s96 = [int(v, 16) for v in tok[p].split()]; p += 1
        A = np.zeros((PE_M, K), np.uint16)
        Q = np.zeros((PE_N, K), np.uint8)
        for k in range(K):
            f = tok[p].split(); p += 1
            A[:, k] = [int(v, 16) for v in f[:PE_M]]
            Q[:, k] = [int(v, 16) for v in f[PE_M:]]
        C = np.array([int(v, 16) for v in tok[p].split()], np.uint16).reshape(PE_M, PE_N); p += 1
        tests.append((K, NSB, d, dm, s96, A, Q, C))
    return PE_M, PE_N, tests


def gen_refvectors():
    """The reference generators' own seeded vectors: q4k_matmul_gen (seed 0, both its committed
    K list and its real-dims list 512/2048/6144) and q4k_mixed_gen.emit_mixed_gemm (seed 11).
    K is padded to whole super-blocks with zero activations (adding +-0 leaves the sequential
    fp32 sum unchanged)."""
    out = {}
    idx = 0
    for (ntest, kch) in ((40, None), (6, [512, 2048, 6144])):
        PE_M, PE_N, tests = _parse_matmul_gen(MG.gen(ntest, 2, 2, seed=0, kchoices=kch))
        for (K, NSB, d, dm, s96, A, Q, C) in tests:
            Kp = NSB * 256
            W = np.zeros((PE_N, NSB * 144), np.uint8)
            for pj in range(PE_N):
                for sb in range(NSB):
                    codes = np.zeros(256, np.int64)
                    seg = Q[pj, sb * 256:min(K, (sb + 1) * 256)]
                    codes[:len(seg)] = seg
                    sc12 = [(s96[pj * NSB + sb] >> (8 * i)) & 0xFF for i in range(12)]
                    W[pj, sb * 144:(sb + 1) * 144] = pack_q4k(d[pj * NSB + sb], dm[pj * NSB + sb], sc12, codes)
            Ap = np.zeros((PE_M, Kp), np.uint16)
            Ap[:, :K] = A
            out[f"mm{idx}_w"] = W
            out[f"mm{idx}_a"] = Ap
            out[f"mm{idx}_c"] = C
            out[f"mm{idx}_meta"] = np.array([0, PE_N, Kp, PE_M, K], np.int64)
            idx += 1
    out["n_mm"] = np.array(idx)

    # mixed-type GEMM tiles (q4k_mixed_gen.emit_mixed_gemm layout, q4k_mixed_gen.py:274-296)
    path = os.path.join("/tmp", "aipu_mixed_vec.txt")
    XG.emit_mixed_gemm(path)
    tok = open(path).read().split("\n")
    ntest, PE_M, PE_N = map(int, tok[0].split())
    p = 1
    for t in range(ntest):
        K, NSB, NB8 = map(int, tok[p].split()); p += 1
        types = [int(v) for v in tok[p].split()]; p += 1
        wd = [int(v, 16) for v in tok[p].split()]; p += 1
        wdm = [int(v, 16) for v in tok[p].split()]; p += 1
        wsc = [int(v, 16) for v in tok[p].split()]; p += 1
        q6 = [int(v, 16) for v in tok[p].split()]; p += 1
        q8 = [int(v, 16) for v in tok[p].split()]; p += 1
        A = np.zeros((PE_M, K), np.uint16)
        WQ = np.zeros((PE_N, K), np.int64)
        HP = np.zeros((PE_N, K), np.int64)
        for k in range(K):
            f = tok[p].split(); p += 1
            A[:, k] = [int(v, 16) for v in f[:PE_M]]
            for pj in range(PE_N):
                WQ[pj, k] = int(f[PE_M + 2 * pj], 16)
                HP[pj, k] = int(f[PE_M + 2 * pj + 1], 16)
        C = np.array([int(v, 16) for v in tok[p].split()], np.uint16).reshape(PE_M, PE_N); p += 1
        for pj in range(PE_N):
            ty = types[pj]
            if ty == 0:
                row = np.concatenate([pack_q4k(wd[pj * NSB + sb], wdm[pj * NSB + sb],
                                               [(wsc[pj * NSB + sb] >> (8 * i)) & 0xFF for i in range(12)],
                                               WQ[pj, sb * 256:(sb + 1) * 256]) for sb in range(NSB)])
            elif ty == 1:
                row = np.concatenate([pack_q6k(wd[pj * NSB + sb],
                                               [v - 256 if v > 127 else v for v in q6[(pj * NSB + sb) * 16:(pj * NSB + sb + 1) * 16]],
                                               HP[pj, sb * 256:(sb + 1) * 256]) for sb in range(NSB)])
            elif ty == 2:
                row = np.concatenate([pack_q80(q8[pj * NB8 + b], HP[pj, b * 32:(b + 1) * 32]) for b in range(NB8)])
            else:
                row = HP[pj].astype(np.uint16).view(np.uint8)
            out[f"mx{t}_w{pj}"] = row
        out[f"mx{t}_types"] = np.array(types, np.int64)
        out[f"mx{t}_a"] = A
        out[f"mx{t}_c"] = C
        out[f"mx{t}_meta"] = np.array([K, PE_M, PE_N], np.int64)
    out["n_mx"] = np.array(ntest)
    np.savez_compressed(os.path.join(HERE, "refvec_golden.npz"), **out)


# --------------------------------------------------------------- 4. activations
def gen_act():
    """glm_sigmoid / glm_silu of the reference on EVERY bf16 bit pattern, plus fp32_rsqrt."""
    pats = np.arange(65536, dtype=np.uint32)
    xs = (pats << 16).view(F32)
    sig = np.array([G.bf16_bits(G.glm_sigmoid(F32(v))) for v in xs], np.uint16)
    silu = np.array([G.bf16_bits(G.glm_silu(F32(v))) for v in xs], np.uint16)
    rng = np.random.default_rng(5)
    r_in = np.concatenate([rng.uniform(1e-3, 1e3, 3000).astype(F32),
                           rng.uniform(0.1, 20.0, 2000).astype(F32),
                           np.array([0.0, -0.0, -1.0, np.inf, -np.inf, np.nan, 1e-40, 3.4e38, 1.0, 2.5], F32)])
    r_out = np.array([G.fp32_rsqrt(F32(v)) for v in r_in], F32)
    np.savez_compressed(os.path.join(HERE, "act_golden.npz"), sigmoid=sig, silu=silu,
                        rsqrt_in=f32bits(r_in), rsqrt_out=f32bits(r_out))


# --------------------------------------------------------------- 5. router / swiglu / MoE
def _qw_to_rows(qw):
    """Reference QW (nin <= 256, one super-block per column) -> GGUF Q4_K rows [nout, 144]."""
    rows = []
    for o in range(qw.nout):
        codes = np.zeros(256, np.int64)
        codes[:qw.nin] = qw.codes[o]
        rows.append(pack_q4k(qw.d[o], qw.dmin[o], qw.scales[o], codes))
    return np.stack(rows)


def gen_moe():
    out = {}
    # (a) the reference router at its committed slice (8 experts, top-2, Weights seed 7)
    #     and at GLM-like width (256 experts, top-8), MODEL_DIM 256; Q4_K router, no bias.
    for name, kw, seed in (("r8", dict(), 7), ("r256", dict(N_EXPERT=256, TOPK=8, MODEL_DIM=256), 11)):
        cfg = G.Config(**kw)
        rng = np.random.default_rng(seed)
        Wg = G._mk_qw(rng, cfg.N_EXPERT, cfg.MODEL_DIM)
        if name == "r256":
            # make experts 40..47 exact copies of expert 3 -> exact gate ties (lower index wins)
            for e in range(40, 48):
                Wg.codes[e] = list(Wg.codes[3]); Wg.d[e] = Wg.d[3]; Wg.dmin[e] = Wg.dmin[3]
                Wg.scales[e] = list(Wg.scales[3])
            Wg._deq = None
        X, SEL, SW, GATE = [], [], [], []
        for t in range(24):
            x = [G.bf16(F32(v)) for v in rng.uniform(-1.5, 1.5, cfg.MODEL_DIM)]
            sel, sw, gate = G.moe_router(cfg, x, Wg)
            X.append(f32bits(x)); SEL.append(sel); SW.append(f32bits(sw)); GATE.append(f32bits(gate))
        out[f"{name}_meta"] = np.array([cfg.N_EXPERT, cfg.TOPK, cfg.MODEL_DIM], np.int64)
        out[f"{name}_w"] = _qw_to_rows(Wg)
        out[f"{name}_x"] = np.stack(X)
        out[f"{name}_sel"] = np.array(SEL, np.int64)
        out[f"{name}_sw"] = np.stack(SW)
        out[f"{name}_gate"] = np.stack(GATE)

    # (b) swiglu_expert + the decoder-block MoE combine at MODEL_DIM 256, INTER 128,
    #     16 experts top-4 + shared; combine replicated from decoder_block (glm_model_q4k_ref.py:797-809)
    cfg = G.Config(N_EXPERT=16, TOPK=4, MODEL_DIM=256, INTER_MOE=128)
    rng = np.random.default_rng(2024)
    Wg = G._mk_qw(rng, cfg.N_EXPERT, cfg.MODEL_DIM)
    Mg = [G._mk_qw(rng, cfg.INTER_MOE, cfg.MODEL_DIM) for _ in range(cfg.N_EXPERT + 1)]
    Mu = [G._mk_qw(rng, cfg.INTER_MOE, cfg.MODEL_DIM) for _ in range(cfg.N_EXPERT + 1)]
    Md = [G._mk_qw(rng, cfg.MODEL_DIM, cfg.INTER_MOE) for _ in range(cfg.N_EXPERT + 1)]
    X, Y, SEL, SW, YE = [], [], [], [], []
    for t in range(3):
        x = [G.bf16(F32(v)) for v in rng.uniform(-1.5, 1.5, cfg.MODEL_DIM)]
        sel, sw, _ = G.moe_router(cfg, x, Wg)
        facc = [F32(0.0)] * cfg.MODEL_DIM
        yes = []
        for slot in range(cfg.TOPK):
            e = sel[slot]
            y_e = G.swiglu_expert(cfg, x, Mg[e], Mu[e], Md[e])
            yes.append(f32bits(y_e))
            g = G.b2f(sw[slot])
            for d in range(cfg.MODEL_DIM):
                facc[d] = G.fadd(facc[d], G.fmul(g, G.b2f(y_e[d])))
        y_sh = G.swiglu_expert(cfg, x, Mg[-1], Mu[-1], Md[-1])
        for d in range(cfg.MODEL_DIM):
            facc[d] = G.fadd(facc[d], G.b2f(y_sh[d]))
        fbuf = [G.bf16(facc[d]) for d in range(cfg.MODEL_DIM)]
        X.append(f32bits(x)); Y.append(f32bits(fbuf)); SEL.append(sel); SW.append(f32bits(sw))
        YE.append(np.stack(yes + [f32bits(y_sh)]))
    out["moe_meta"] = np.array([cfg.N_EXPERT, cfg.TOPK, cfg.MODEL_DIM, cfg.INTER_MOE], np.int64)
    out["moe_router_w"] = _qw_to_rows(Wg)
    # gate/up rows: nin = MODEL_DIM = 256 -> one super-block per row; down rows: nin = 128 -> padded
    out["moe_gate_w"] = np.stack([_qw_to_rows(q) for q in Mg])
    out["moe_up_w"] = np.stack([_qw_to_rows(q) for q in Mu])
    out["moe_down_w"] = np.stack([_qw_to_rows(q) for q in Md])
    out["moe_x"] = np.stack(X)
    out["moe_y"] = np.stack(Y)
    out["moe_sel"] = np.array(SEL, np.int64)
    out["moe_sw"] = np.stack(SW)
    out["moe_yslots"] = np.stack(YE)
    np.savez_compressed(os.path.join(HERE, "moe_golden.npz"), **out)


if __name__ == "__main__":
    steps = sys.argv[1:] or ["dequant", "gemm", "refvec", "act", "moe"]
    for s in steps:
        print("generating", s, flush=True)
        {"dequant": gen_dequant, "gemm": gen_gemm, "refvec": gen_refvectors,
         "act": gen_act, "moe": gen_moe}[s]()
    print("done")
