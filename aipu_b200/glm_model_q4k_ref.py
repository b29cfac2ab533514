"""Drop-in for the MoE/GEMM part of the reference's ``tools/glm_model_q4k_ref.py``: the same names,
arguments and return values, computed by the CUDA library.

    from aipu_b200 import glm_model_q4k_ref as ref     # instead of: import glm_model_q4k_ref as ref
    sel, sel_w, gates = ref.moe_router(cfg, x_bf, W.Wg[layer])
    y = ref.swiglu_expert(cfg, x_bf, W.Mg[layer][e], W.Mu[layer][e], W.Md[layer][e])

Covered: the fp32/bf16 bit helpers (host), ``glm_sigmoid`` / ``glm_silu`` (aipu_act_eval),
``matmul_q4k`` (strict GEMM), the ``QW`` Q4_K weight container (packed to GGUF Q4_K rows and
dequantised on the GPU), ``moe_router`` (aipu_moe_router), ``swiglu_expert`` (aipu_swiglu_expert
in strict mode), ``f32_bits_key`` and ``_sum_tree``. Results are bit-identical to the reference.
Attention, RoPE, RMSNorm and the decoder stack are outside this library's path.

A reference ``QW`` holds one super-block per output column (its 12 scale bytes serve the whole
reduction, so NIN <= 256); columns are packed into one 256-weight GGUF Q4_K block, the reduction
padded with zero activations and zero weights (unused sub-blocks get scale and min 0).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import formats as F
from . import ops
from .q4k_ref import _pack_6bit_scales, bf16_round, get_scale_min_k4

F32 = np.float32
U32 = np.uint32
U16 = np.uint16
QK_K = 256


def _dev() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("aipu_b200.glm_model_q4k_ref needs a CUDA device (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


_STRICT = {}


def _strict_ctx(d: torch.device) -> ops.Context:
    c = _STRICT.get(d.index)
    if c is None:
        c = ops.Context(d).set_flags(strict=True)
        _STRICT[d.index] = c
    return c


# ---------------------------------------------------------------- bit helpers (host)
def f32_bits(x):
    return int(F32(x).view(U32))


def bits_f32(u):
    return F32(np.uint32(u & 0xFFFFFFFF).view(np.float32))


def fp16_to_f32(h):
    return F32(np.frombuffer(U16(h & 0xFFFF).tobytes(), dtype=np.float16)[0])


def f32_to_f16bits(x):
    return int(np.frombuffer(np.float16(x).tobytes(), dtype=U16)[0])


def bf16_bits(x):
    return (f32_bits(bf16_round(x)) >> 16) & 0xFFFF


def bf16_from_bits(u16):
    return bits_f32((u16 & 0xFFFF) << 16)


def bf16(x):
    return bf16_round(x)


def b2f(x):
    return F32(x)


def fmul(a, b):
    return F32(F32(a) * F32(b))


def fadd(a, b):
    return F32(F32(a) + F32(b))


def fneg(x):
    return bits_f32(f32_bits(x) ^ 0x80000000)


QNAN = bits_f32(0x7FC00000)


def _bf16_dev(vals, n_pad: int | None = None) -> torch.Tensor:
    """bf16-valued fp32 values -> a bf16 device row (zero padded to n_pad)"""
    a = np.asarray([f32_bits(v) >> 16 for v in vals], dtype=np.uint32).astype(np.uint16)
    if n_pad is not None and n_pad > a.size:
        a = np.concatenate([a, np.zeros(n_pad - a.size, np.uint16)])
    return torch.from_numpy(a.view(np.int16)).to(_dev()).view(torch.bfloat16)


def _bf16_host(t: torch.Tensor) -> np.ndarray:
    u = t.contiguous().view(torch.int16).cpu().numpy().astype(np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


# ---------------------------------------------------------------- activations (GPU)
def _act(kind: str, xbf):
    scalar = np.ndim(xbf) == 0
    vals = [xbf] if scalar else list(np.asarray(xbf, F32).reshape(-1))
    out = _bf16_host(ops.act(kind, _bf16_dev(vals)))
    return F32(out[0]) if scalar else out.reshape(np.shape(xbf))


def glm_sigmoid(xbf):
    """bf16 glm sigmoid of a bf16 value (tools/glm_model_q4k_ref.py:293-294)."""
    return _act("sigmoid", xbf)


def glm_silu(xbf):
    """bf16 glm SiLU of a bf16 value (tools/glm_model_q4k_ref.py:296-299)."""
    return _act("silu", xbf)


# ---------------------------------------------------------------- matmul (GPU)
def matmul_q4k(a_row, wdeq_cols):
    """out[o] = bf16( sequential fp32 sum_k a[k] * wdeq_cols[o][k] ) (tools/glm_model_q4k_ref.py:470-472)."""
    w = np.ascontiguousarray(np.stack([np.asarray(c, F32) for c in wdeq_cols]))
    a = np.ascontiguousarray(np.asarray(a_row, F32).reshape(1, -1))
    d = _dev()
    y = ops.gemm(F.F32, torch.from_numpy(w.view(np.uint8)).to(d), w.shape[0], w.shape[1],
                 torch.from_numpy(a).to(d), mode="strict")
    return [F32(v) for v in _bf16_host(y)[0]]


def matmul_bf16_dot(a_bf, w_bf):
    """One bf16 dot product under the reference's 7-partial-sum contract
    (tools/glm_model_q4k_ref.py:474-486) on the GPU. Both vectors are zero padded to a multiple of 8
    (the padding adds +0 products, which leave every partial sum unchanged: a sum that starts at +0
    never becomes -0 under round-to-nearest)."""
    K = len(a_bf)
    kp = (K + 7) // 8 * 8
    x = _bf16_dev(list(np.asarray(a_bf, F32).reshape(-1)), kp).view(1, kp)
    w = _bf16_dev(list(np.asarray(w_bf, F32).reshape(-1)), kp).view(1, kp)
    return F32(_bf16_host(ops.bf16_dot_gemv(w, x))[0, 0])


# ---------------------------------------------------------------- Q4_K weight container
class QW:
    """Q4_K weight matrix: NOUT output columns x NIN reduction (tools/glm_model_q4k_ref.py:491-519),
    with the GGUF block bytes of every column kept on the device for the GPU kernels."""
    __slots__ = ("nout", "nin", "codes", "d", "dmin", "scales", "_deq", "_dev_rows")

    def __init__(self, nout, nin, codes, d, dmin, scales):
        if nin > QK_K:
            raise ValueError("a reference QW column is one super-block: NIN <= 256")
        self.nout = nout
        self.nin = nin
        self.codes = codes
        self.d = d
        self.dmin = dmin
        self.scales = scales
        self._deq = None
        self._dev_rows = None

    def gguf_rows(self) -> np.ndarray:
        """[nout, 144] GGUF Q4_K blocks; reduction padded to 256 with zero codes and zero
        scale/min for the sub-blocks the reference never reads."""
        nsub = (self.nin + 31) // 32
        out = np.zeros((self.nout, 144), np.uint8)
        for o in range(self.nout):
            sm = [get_scale_min_k4(j, self.scales[o]) for j in range(8)]
            scs = [sm[j][0] if j < nsub else 0 for j in range(8)]
            mns = [sm[j][1] if j < nsub else 0 for j in range(8)]
            codes = np.zeros(QK_K, np.uint8)
            codes[:self.nin] = np.asarray(self.codes[o], np.uint8)
            qs = np.zeros(128, np.uint8)
            for g in range(4):
                qs[32 * g:32 * g + 32] = codes[64 * g:64 * g + 32] | (codes[64 * g + 32:64 * g + 64] << 4)
            out[o, 0:2] = np.frombuffer(np.uint16(self.d[o] & 0xFFFF).tobytes(), np.uint8)
            out[o, 2:4] = np.frombuffer(np.uint16(self.dmin[o] & 0xFFFF).tobytes(), np.uint8)
            out[o, 4:16] = np.asarray(_pack_6bit_scales(scs, mns), np.uint8)
            out[o, 16:] = qs
        return out

    def device_rows(self) -> torch.Tensor:
        if self._dev_rows is None:
            self._dev_rows = torch.from_numpy(self.gguf_rows()).to(_dev())
        return self._dev_rows

    def dequant_col(self, o):
        return self.dequant()[o]

    def dequant(self):
        if self._deq is None:
            full = ops.dequant(F.Q4_K, self.device_rows(), self.nout, QK_K).cpu().numpy()
            self._deq = [np.ascontiguousarray(full[o, :self.nin]) for o in range(self.nout)]
        return self._deq


# ---------------------------------------------------------------- MoE operators (GPU)
def moe_router(cfg, x_bf, Wg):
    """logits = x @ W_g -> sigmoid -> top-K -> renorm * SCALE (tools/glm_model_q4k_ref.py:663-681).
    Returns (sel_idx list, sel_weight bf16 list, gate_bf list)."""
    E, T = cfg.N_EXPERT, cfg.TOPK
    x = _bf16_dev(x_bf, QK_K).view(1, QK_K)
    sel, sw, gate = ops.moe_router(F.Q4_K, Wg.device_rows(), x, E, T, scale=float(bits_f32(cfg.RSCALE_BITS)),
                                   ctx=_strict_ctx(x.device))
    return ([int(v) for v in sel.cpu().numpy()[0]], [F32(v) for v in _bf16_host(sw)[0]],
            [F32(v) for v in _bf16_host(gate)[0]])


def f32_bits_key(x):
    """order-preserving integer key of an fp32 (tools/glm_model_q4k_ref.py:684-688)"""
    u = f32_bits(x)
    return (u ^ 0x80000000) if (u >> 31) == 0 else (~u & 0xFFFFFFFF)


def _sum_tree(vals, topk):
    """balanced fp32 add tree of clog2(topk) levels, +0.0 pad (tools/glm_model_q4k_ref.py:691-699)"""
    sumlev = 1 if topk <= 1 else int(math.ceil(math.log2(topk)))
    node = [vals[i] if i < len(vals) else F32(0.0) for i in range(1 << sumlev)]
    for _ in range(sumlev):
        node = [fadd(node[2 * i], node[2 * i + 1]) for i in range(len(node) // 2)]
    return node[0]


def swiglu_expert(cfg, x_bf, Wgate, Wup, Wdown):
    """y = (silu(x @ W_gate) * (x @ W_up)) @ W_down (tools/glm_model_q4k_ref.py:702-708), bit-exact
    (strict mode). The hidden and FFN dims are padded to 256 with zero weights and activations."""
    H, Fd = Wdown.nout, Wgate.nout
    if Wgate.nin != H or Wup.nin != H or Wup.nout != Fd or Wdown.nin != Fd or H > QK_K or Fd > QK_K:
        raise ValueError("swiglu_expert: inconsistent or oversize weight shapes")
    d = _dev()
    gpad = torch.zeros((QK_K, 144), dtype=torch.uint8, device=d)
    upad = torch.zeros((QK_K, 144), dtype=torch.uint8, device=d)
    dpad = torch.zeros((QK_K, 144), dtype=torch.uint8, device=d)
    gpad[:Fd] = Wgate.device_rows()
    upad[:Fd] = Wup.device_rows()
    dpad[:H] = Wdown.device_rows()
    x = _bf16_dev(x_bf, QK_K).view(1, QK_K)
    y = ops.swiglu_expert(F.Q4_K, gpad, upad, F.Q4_K, dpad, QK_K, QK_K, x, ctx=_strict_ctx(d))
    return [F32(v) for v in _bf16_host(y)[0, :H]]


class Config:
    """The reference's model configuration object (tools/glm_model_q4k_ref.py:559-584): module
    defaults, overridable by keyword. Only the MoE fields are used by this module."""

    def __init__(self, **kw):
        self.MODEL_DIM = 128
        self.L = 6
        self.N_DENSE = 3
        self.VOCAB = 256
        self.H_HEADS = 4
        self.NOPE = 16
        self.ROPE = 16
        self.V_DIM = 32
        self.Q_LORA = 64
        self.KV_LORA = 32
        self.S_MAX = 8
        self.TOPK_ATTN = 8
        self.THETA = 8000000
        self.PE_N = 4
        self.POSW = 20
        self.N_EXPERT = 8
        self.TOPK = 2
        self.INTER_MOE = 64
        self.INTER_DENSE = 256
        self.RSCALE_BITS = 0x40200000
        self.TN = 4
        self.LM_TN = 4
        for k, v in kw.items():
            setattr(self, k, v)

    # derived dimensions (tools/glm_model_q4k_ref.py:586-606), used by Weights
    @property
    def QK_DIM(self):
        return self.NOPE + self.ROPE

    @property
    def HQK(self):
        return self.H_HEADS * self.QK_DIM

    @property
    def HNOPE(self):
        return self.H_HEADS * self.NOPE

    @property
    def HV(self):
        return self.H_HEADS * self.V_DIM

    @property
    def SWIN(self):
        return min(self.S_MAX, self.TOPK_ATTN)


# the spec-decode slice configuration of the reference's full-model test bench
# (tools/glm_model_q4k_ref.py:609-612)
SPEC_SLICE = dict(MODEL_DIM=16, L=2, N_DENSE=1, VOCAB=16, H_HEADS=2, NOPE=4, ROPE=4, V_DIM=4, Q_LORA=8, KV_LORA=8,
                  S_MAX=2, TOPK_ATTN=2, PE_N=2, N_EXPERT=4, TOPK=2, INTER_MOE=8, INTER_DENSE=32)


# ---------------------------------------------------------------- seeded weights
# These generators reproduce the reference's seeded weight draws (tools/glm_model_q4k_ref.py:522-544,
# 619-658): the same numpy Generator calls in the same order, so Weights(cfg, seed) holds exactly the
# reference's weights and tests written against the reference's seeds see the same numbers.
def _mk_qw(rng, nout, nin):
    """A QW of nout columns x nin: codes uniform 0..15; d = dmin = fp16(U(0.004, 0.012)) per column;
    6-bit scales U{1..4} per sub-block with mins round(7.5 sc) + U{-1, 0, 1} clamped to 0..63, which
    centres every sub-block's weights near zero."""
    codes = [[int(v) for v in rng.integers(0, 16, nin)] for _ in range(nout)]
    d = [f32_to_f16bits(rng.uniform(0.004, 0.012)) for _ in range(nout)]
    dmin = list(d)
    scales = []
    for _ in range(nout):
        sc = [int(v) for v in rng.integers(1, 5, 8)]
        mn = [min(63, max(0, int(round(7.5 * v)) + int(rng.integers(-1, 2)))) for v in sc]
        scales.append(list(_pack_6bit_scales(sc, mn)))
    return QW(nout, nin, codes, d, dmin, scales)


def _mk_bf16(rng, n, lo=-1.0, hi=1.0):
    """n bf16 values drawn uniform in [lo, hi)."""
    return [bf16(F32(v)) for v in rng.uniform(lo, hi, n)]


def _mk_gamma(rng, n):
    """RMSNorm scales: n bf16 values uniform in [0.6, 1.4)."""
    return [bf16(F32(v)) for v in rng.uniform(0.6, 1.4, n)]


class Weights:
    """Every weight of one model, per layer, drawn from `seed` in the reference's order
    (tools/glm_model_q4k_ref.py:619-658): embeddings, then per layer the two norm scales, the MLA
    projections (W_dq, W_uq, W_uk, W_uv, W_o) and KV-cache rows, the router (k-major, a QW of
    N_EXPERT columns), the dense FFN, the routed experts (gate, up, down) and the shared expert;
    then the final norm and the LM head. This library computes the MoE and GEMM parts; the
    attention weights are held for callers that run the rest of the block elsewhere."""

    def __init__(self, cfg, seed=424242):
        self.cfg = c = cfg
        rng = np.random.default_rng(seed)
        self.EMB = [_mk_bf16(rng, c.MODEL_DIM) for _ in range(c.VOCAB)]
        names = ("G1", "G2", "W_dq", "W_uq", "W_uk", "W_uv", "W_o", "CKV", "KRP", "Wg", "Dg", "Du", "Dd", "Mg",
                 "Mu", "Md", "SHg", "SHu", "SHd")
        for n in names:
            setattr(self, n, [])
        for _ in range(c.L):
            self.G1.append(_mk_gamma(rng, c.MODEL_DIM))
            self.G2.append(_mk_gamma(rng, c.MODEL_DIM))
            self.W_dq.append(_mk_qw(rng, c.Q_LORA, c.MODEL_DIM))
            self.W_uq.append(_mk_qw(rng, c.HQK, c.Q_LORA))
            self.W_uk.append(_mk_qw(rng, c.HNOPE, c.KV_LORA))
            self.W_uv.append(_mk_qw(rng, c.HV, c.KV_LORA))
            self.W_o.append(_mk_qw(rng, c.MODEL_DIM, c.HV))
            self.CKV.append([_mk_bf16(rng, c.KV_LORA) for _ in range(c.S_MAX)])
            self.KRP.append([_mk_bf16(rng, c.ROPE) for _ in range(c.S_MAX)])
            self.Wg.append(_mk_qw(rng, c.N_EXPERT, c.MODEL_DIM))
            self.Dg.append(_mk_qw(rng, c.INTER_DENSE, c.MODEL_DIM))
            self.Du.append(_mk_qw(rng, c.INTER_DENSE, c.MODEL_DIM))
            self.Dd.append(_mk_qw(rng, c.MODEL_DIM, c.INTER_DENSE))
            self.Mg.append([_mk_qw(rng, c.INTER_MOE, c.MODEL_DIM) for _ in range(c.N_EXPERT)])
            self.Mu.append([_mk_qw(rng, c.INTER_MOE, c.MODEL_DIM) for _ in range(c.N_EXPERT)])
            self.Md.append([_mk_qw(rng, c.MODEL_DIM, c.INTER_MOE) for _ in range(c.N_EXPERT)])
            self.SHg.append(_mk_qw(rng, c.INTER_MOE, c.MODEL_DIM))
            self.SHu.append(_mk_qw(rng, c.INTER_MOE, c.MODEL_DIM))
            self.SHd.append(_mk_qw(rng, c.MODEL_DIM, c.INTER_MOE))
        self.GF = _mk_gamma(rng, c.MODEL_DIM)
        self.Wlm = [_mk_bf16(rng, c.MODEL_DIM) for _ in range(c.VOCAB)]
