"""CPU oracle for the MoE operators on the dequant-GEMM path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this module;
the library never does.

Restates, vectorised with numpy, the reference's numpy golden of the MoE branch
(Wick-Lim/AIPU ``tools/glm_model_q4k_ref.py``):
  * fp32_rsqrt (Quake seed 0x5F3759DF + 2 Newton steps)      glm_model_q4k_ref.py:96-116
  * glm_act sigmoid / silu (Horner exp + rsqrt^2 reciprocal)  glm_model_q4k_ref.py:214-299
  * moe_router (sigmoid, top-K, renorm x SCALE)               glm_model_q4k_ref.py:663-681
  * f32_bits_key ordering, lower index wins ties              glm_model_q4k_ref.py:684-688
  * _sum_tree balanced fp32 add tree                          glm_model_q4k_ref.py:691-699
  * swiglu_expert                                              glm_model_q4k_ref.py:702-708
  * MoE combine inside decoder_block (slot order, then shared) glm_model_q4k_ref.py:797-809
  * matmul_bf16_dot (7 interleaved partial sums + add tree)   glm_model_q4k_ref.py:474-486

Router extension (not in the reference): a dense fp32 router W_r [K, E] plus a per-expert fp32
bias. Logits follow the same sequential fp32 MAC contract (fp32 weights instead of dequantised
Q4_K ones). The bias is added in fp32 to the bf16 gate for SELECTION ONLY; the routing weights
are renormalised from the unbiased gates. With bias = None this is exactly the reference router.

All fp32 arithmetic is one numpy float32 op per reference op (no fusion); bit manipulations use
uint32 views.
"""
from __future__ import annotations

import numpy as np

from . import q4k_oracle as qo

F32 = np.float32
U32 = np.uint32


def _bits(x):
    return np.asarray(x, F32).view(U32)


def _f32(u):
    return np.asarray(u, np.uint64).astype(U32).view(F32)


_ONE = F32(1.0)
_LOG2E = _f32(0x3FB8AA3B)
_LN2 = _f32(0x3F317218)
_XSAT_BITS = 0x41800000            # 16.0
_KMAX = 64
_P = [_f32(v) for v in (0x3C088889, 0x3D2AAAAB, 0x3E2AAAAB, 0x3F000000)]  # 1/120,1/24,1/6,1/2


def fp32_rsqrt(x) -> np.ndarray:
    """Quake seed + exactly 2 Newton iterations (glm_model_q4k_ref.py:96-116).
    NaN / negative / zero (exp==0 counts as zero) -> quiet NaN; +inf -> +0."""
    x = np.asarray(x, F32)
    u = _bits(x).astype(np.int64)
    e = (u >> 23) & 0xFF
    man = u & 0x7FFFFF
    sign = (u >> 31) & 1
    with np.errstate(over="ignore", invalid="ignore"):
        xhalf = F32(0.5) * x
        y = _f32((0x5F3759DF - (u >> 1)) & 0xFFFFFFFF)
        for _ in range(2):
            yy = y * y
            xyy = xhalf * yy
            t = F32(1.5) + (-xyy)
            y = y * t
    bad = ((e == 0xFF) & (man != 0)) | (sign == 1) | (e == 0)
    y = np.where((e == 0xFF) & (man == 0), F32(0.0), y)
    y = np.where(bad, _f32(0x7FC00000), y)
    return np.asarray(y, F32)


def _sanitize(xb):
    u = _bits(xb).astype(np.int64)
    sat = (u & 0x80000000) | _XSAT_BITS
    return np.where(((u >> 23) & 0xFF) == 0xFF, _f32(sat), np.asarray(xb, F32))


def _clamp(x):
    u = _bits(x).astype(np.int64)
    sat = (u & 0x80000000) | _XSAT_BITS
    return np.where((u & 0x7FFFFFFF) >= _XSAT_BITS, _f32(sat), np.asarray(x, F32))


def _round_to_int(f):
    """glm_act fp32_round_to_int (round half up on the magnitude); |f| <= ~23."""
    u = _bits(f).astype(np.int64)
    s = (u >> 31) & 1
    e = (u >> 23) & 0xFF
    m = 0x800000 | (u & 0x7FFFFF)
    rsh = np.clip(23 - (e - 127), 1, 63)
    shifted = m >> rsh
    mag = (shifted & 0xFF) + ((m >> (rsh - 1)) & 1)
    r = np.where(e < 127, np.where(e == 126, 1, 0), mag)
    return np.where(s == 1, -r, r)


def _scale_pow2(v, k):
    u = _bits(v).astype(np.int64)
    e_new = ((u >> 23) & 0xFF) + k
    sgn = u & 0x80000000
    out = sgn | ((e_new & 0xFF) << 23) | (u & 0x7FFFFF)
    out = np.where(e_new >= 255, sgn | (0xFE << 23) | (u & 0x7FFFFF), out)
    out = np.where(e_new <= 0, sgn, out)
    return _f32(out)


def sigmoid_f32(xbf) -> np.ndarray:
    """glm_act sigmoid core, fp32 result before rounding (glm_model_q4k_ref.py:279-291)."""
    xcl = _clamp(_sanitize(np.asarray(xbf, F32)))
    z = _f32(_bits(xcl) ^ np.uint32(0x80000000))
    kf = z * _LOG2E
    k = np.clip(_round_to_int(kf), -_KMAX, _KMAX)
    kfl = k.astype(F32)                                     # exact for |k| <= 64
    r = z + (-(kfl * _LN2))
    p = _P[1] + r * _P[0]
    p = _P[2] + r * p
    p = _P[3] + r * p
    p = _ONE + r * p
    p = _ONE + r * p
    ex = _scale_pow2(p, k)
    d = _ONE + ex
    t = fp32_rsqrt(d)
    return np.asarray(t * t, F32)


def glm_sigmoid(xbf) -> np.ndarray:
    """bf16(sigmoid) (glm_model_q4k_ref.py:293-294)."""
    return qo.bf16_round(sigmoid_f32(xbf))


def glm_silu(xbf) -> np.ndarray:
    """bf16(sigmoid(x) * sanitize(x)) (glm_model_q4k_ref.py:296-299)."""
    s = sigmoid_f32(xbf)
    return qo.bf16_round(s * _sanitize(np.asarray(xbf, F32)))


def f32_bits_key(x) -> np.ndarray:
    """Order-preserving uint32 key of an fp32 (glm_model_q4k_ref.py:684-688)."""
    u = _bits(x).astype(np.uint64)
    return np.where((u >> 31) == 0, u ^ 0x80000000, (~u) & 0xFFFFFFFF).astype(np.uint64)


def sum_tree(vals: np.ndarray) -> np.ndarray:
    """Balanced fp32 add tree over the last axis, +0.0 padded to a power of two
    (glm_model_q4k_ref.py:691-699)."""
    v = np.asarray(vals, F32)
    topk = v.shape[-1]
    lev = 1 if topk <= 1 else int(np.ceil(np.log2(topk)))
    n = 1 << lev
    node = np.zeros(v.shape[:-1] + (n,), F32)
    node[..., :topk] = v
    for _ in range(lev):
        node = node[..., 0::2] + node[..., 1::2]
    return node[..., 0]


RSCALE_DEFAULT = F32(2.5)       # Config.RSCALE_BITS = 0x40200000 (glm_model_q4k_ref.py:584)


def route_from_logits(logit_bf, topk: int, bias=None, scale=RSCALE_DEFAULT):
    """Sigmoid gates -> top-K selection -> renormalised routing weights.

    logit_bf: fp32 [M, E] bf16-valued logits. Returns (sel int32 [M, topk] in slot order,
    weight bf16-valued fp32 [M, topk], gate bf16-valued fp32 [M, E]).
    Restates glm_model_q4k_ref.py:669-681; selection key = gate, or fp32(gate + bias).
    """
    gate = glm_sigmoid(np.asarray(logit_bf, F32))
    M, E = gate.shape
    score = gate if bias is None else (gate + np.asarray(bias, F32)[None, :])
    key = (f32_bits_key(score) << np.uint64(16)) | (np.uint64(0xFFFF) - np.arange(E, dtype=np.uint64))[None, :]
    order = np.argsort(key, axis=1)[:, ::-1]                 # keys are unique
    sel = order[:, :topk].astype(np.int32)
    win = np.take_along_axis(gate, sel, axis=1)
    s = sum_tree(win)
    rr = fp32_rsqrt(s)
    rs = (rr * rr) * F32(scale)
    w = qo.bf16_round(win * rs[:, None])
    return sel, w, gate


def router_logits(x_bf, wr_t: np.ndarray) -> np.ndarray:
    """Sequential-fp32 router logits, bf16: x [M, K] x W^T where wr_t is [E, K] fp32
    (dequantised Q4_K router rows, or the fp32 router transposed)."""
    return qo.matmul_seq(np.asarray(x_bf, F32), wr_t)


def moe_router(x_bf, wr_t, topk: int, bias=None, scale=RSCALE_DEFAULT):
    """moe_router (glm_model_q4k_ref.py:663-681), batched over M token rows."""
    return route_from_logits(router_logits(x_bf, wr_t), topk, bias, scale)


def swiglu_expert(x_bf, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray) -> np.ndarray:
    """y = (silu(x@Wg) * (x@Wu)) @ Wd with bf16 rounding at each stage
    (glm_model_q4k_ref.py:702-708). wg/wu: fp32 [F, H]; wd: fp32 [H, F]; x: [M, H]."""
    g = qo.matmul_seq(x_bf, wg)
    u = qo.matmul_seq(x_bf, wu)
    h = qo.bf16_round(glm_silu(g) * u)
    return qo.matmul_seq(h, wd)


def swiglu_hidden(x_bf, wg, wu) -> np.ndarray:
    """The bf16 hidden activation h = bf16(silu(g) * u) of swiglu_expert."""
    g = qo.matmul_seq(x_bf, wg)
    u = qo.matmul_seq(x_bf, wu)
    return qo.bf16_round(glm_silu(g) * u)


def combine(sel_w: np.ndarray, y_slots: np.ndarray, y_shared) -> np.ndarray:
    """facc = sum over slots (slot order) of fp32(w_slot) * y_slot, + y_shared, then bf16
    (glm_model_q4k_ref.py:799-809). sel_w [M, T]; y_slots [M, T, H]; y_shared [M, H] or None."""
    M, T, H = y_slots.shape
    facc = np.zeros((M, H), F32)
    for s in range(T):
        facc = facc + np.asarray(sel_w[:, s:s + 1], F32) * y_slots[:, s, :]
    if y_shared is not None:
        facc = facc + np.asarray(y_shared, F32)
    return qo.bf16_round(facc)


def swiglu_magnitude(h_bf, wd) -> np.ndarray:
    """sum_k |h_k| * |w_d[n, k]| per output: the scale the reference's own SwiGLU tolerance uses
    (tools/swiglu_q4k_gen.py:91-95)."""
    return np.abs(np.asarray(h_bf, np.float64)) @ np.abs(np.asarray(wd, np.float64)).T


def moe_layer(x_bf, wr_t, experts_deq, shared_deq, topk: int, bias=None, scale=RSCALE_DEFAULT, want_mag=False):
    """The MoE branch of decoder_block (glm_model_q4k_ref.py:797-809) on M token rows.

    experts_deq: callable e -> (wg [F,H], wu [F,H], wd [H,F]) fp32 dequantised weights
    (called once per expert in the union of selections); shared_deq: same tuple or None.
    Returns (out bf16-valued fp32 [M, H], sel, sel_w), plus the per-output magnitude
    sum_slots |w| * sum_k |h||w_d| (+ shared) when want_mag.
    """
    x = np.asarray(x_bf, F32)
    sel, sel_w, _ = moe_router(x, wr_t, topk, bias, scale)
    M = x.shape[0]
    union = sorted(set(int(e) for e in sel.reshape(-1)))
    y_by_e, mag_by_e = {}, {}
    for e in union:
        wg, wu, wd = experts_deq(e)
        h = swiglu_hidden(x, wg, wu)
        y_by_e[e] = qo.matmul_seq(h, wd)                  # rows are independent
        if want_mag:
            mag_by_e[e] = swiglu_magnitude(h, wd)
    H = next(iter(y_by_e.values())).shape[1]
    y_slots = np.empty((M, topk, H), F32)
    mag = np.zeros((M, H), np.float64)
    for m in range(M):
        for s in range(topk):
            e = int(sel[m, s])
            y_slots[m, s] = y_by_e[e][m]
            if want_mag:
                mag[m] += abs(float(sel_w[m, s])) * mag_by_e[e][m]
    y_sh = None
    if shared_deq is not None:
        wg, wu, wd = shared_deq
        h = swiglu_hidden(x, wg, wu)
        y_sh = qo.matmul_seq(h, wd)
        if want_mag:
            mag += swiglu_magnitude(h, wd)
    out = combine(sel_w, y_slots, y_sh)
    return (out, sel, sel_w, mag) if want_mag else (out, sel, sel_w)


def bf16_dot7(x_bf: np.ndarray, w_bf: np.ndarray) -> np.ndarray:
    """matmul_bf16_dot (glm_model_q4k_ref.py:474-486) for every (token, row): x_bf [M, K], w_bf [V, K]
    bf16-valued fp32 -> bf16-valued fp32 [M, V]. Partial sum l (0..6) adds fl(x_k * w_k) for
    k = l, l + 7, ... in order; then a01 = p0 + p1, a23 = p2 + p3, a45 = p4 + p5, a6 = p6 + 0,
    b0 = a01 + a23, b1 = a45 + a6, out = bf16(b0 + b1)."""
    x = np.asarray(x_bf, F32)
    w = np.asarray(w_bf, F32)
    M, K = x.shape
    ps = np.zeros((7, M, w.shape[0]), F32)
    for k in range(K):
        ps[k % 7] = ps[k % 7] + x[:, k:k + 1] * w[None, :, k]
    z = F32(0.0)
    a01, a23, a45, a6 = ps[0] + ps[1], ps[2] + ps[3], ps[4] + ps[5], ps[6] + z
    return qo.bf16_round((a01 + a23) + (a45 + a6))


def moe_layer_packed(x_bf, router_rows_f32, experts, shared, topk: int, bias=None, scale=RSCALE_DEFAULT,
                     gate_wtype: int = 0, down_wtype: int = 1):
    """moe_layer on packed GGUF rows, with every GEMM done by the C restatement of the sequential
    contract (oracle/q4k_oracle.c; bit-identical to qo.matmul_seq), for full-size layers.
    x_bf [M, H] bf16-valued fp32; router_rows_f32 [E, H] fp32 (router rows); experts: callable
    e -> (gate rows, up rows, down rows) as uint8 [rows, row bytes]; shared: same tuple or None.
    Returns (out [M, H], sel, sel_w) exactly as moe_layer (glm_model_q4k_ref.py:797-809)."""
    from . import cpu

    x = np.ascontiguousarray(np.asarray(x_bf, F32))
    M, H = x.shape
    E = router_rows_f32.shape[0]
    logits = cpu.gemm(4, np.ascontiguousarray(router_rows_f32, F32).view(np.uint8), E, H, x)
    sel, sel_w, _ = route_from_logits(logits, topk, bias, scale)

    def expert_rows(wg, wu, wd, xr):
        Fd = wg.shape[0]
        g = cpu.gemm(gate_wtype, wg, Fd, H, xr)
        u = cpu.gemm(gate_wtype, wu, Fd, H, xr)
        h = qo.bf16_round(glm_silu(g) * u)
        return cpu.gemm(down_wtype, wd, H, Fd, h)

    y_slots = np.empty((M, topk, H), F32)
    for e in sorted(set(int(v) for v in sel.reshape(-1))):
        rows = np.nonzero((sel == e).any(axis=1))[0]
        ye = expert_rows(*experts(e), x[rows])
        for i, m in enumerate(rows):
            for s in range(topk):
                if sel[m, s] == e:
                    y_slots[m, s] = ye[i]
    y_sh = expert_rows(*shared, x) if shared is not None else None
    return combine(sel_w, y_slots, y_sh), sel, sel_w
