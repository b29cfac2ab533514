"""Torch-tensor front end of the C ABI. Tensors are only the boundary: every call goes straight to
``libaipu_q4k.so`` on the current CUDA stream. There is no CPU path; CPU tensors are rejected.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L
from ._lib import check, lib

_DTYPE = {torch.float32: L.DT_F32, torch.bfloat16: L.DT_BF16}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("aipu_b200 runs on CUDA tensors only (no CPU fallback)")
        if t is not None and not t.is_contiguous():
            raise ValueError("aipu_b200 needs contiguous tensors")


def row_bytes(wtype: int, K: int) -> int:
    n = lib().aipu_row_bytes(wtype, K)
    if n <= 0:
        raise ValueError(f"K={K} is not a whole number of blocks of type {wtype}")
    return n


class Context:
    """Per-device workspace (stream-K partials, MoE scratch, side stream) owned by the library."""

    _default: dict = {}

    def __init__(self, device: int | torch.device | None = None):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("Context needs a CUDA device")
        self.device = dev
        h = ctypes.c_void_p()
        check(lib().aipu_ctx_create(ctypes.byref(h), dev.index if dev.index is not None else 0))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().aipu_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_flags(self, pdl: bool = False, strict: bool = False, tc_decode: bool = False,
                  fast_down: bool = False) -> "Context":
        """pdl=True: fast GEMMs start streaming weights while the previous kernel drains (only when no
        kernel right before a GEMM writes its weights). strict=True: every MoE path (the many-token
        one included) is bit-exact (the reference's sequential fp32 chains). The decode MoE path is
        bit-exact by default (chain kernel); tc_decode=True runs it on the tensor-core GEMV instead
        (each GEMM within 1 bf16 ulp, the layer not bit-exact); fast_down=True keeps the exact chains
        for gate/up (h bit-exact) and runs only the down projection on the GEMV (1-ulp bar)."""
        flags = ((L.FLAG_PDL if pdl else 0) | (L.FLAG_STRICT if strict else 0)
                 | (L.FLAG_TC_DECODE if tc_decode else 0) | (L.FLAG_FAST_DOWN if fast_down else 0))
        check(lib().aipu_ctx_set_flags(self.handle, flags))
        return self

    def set_wait_limit(self, cycles: int) -> "Context":
        """Limit of every bounded device wait of this context's kernels in SM cycles (<= 0: default)."""
        check(lib().aipu_ctx_set_wait_limit(self.handle, int(cycles)))
        return self

    def selftest_wait(self) -> None:
        """Run one bounded wait that nothing releases (the failure-detection path); read status()."""
        check(lib().aipu_selftest_wait(self.handle, _stream(self.device)))

    def status(self) -> int:
        v = ctypes.c_int()
        check(lib().aipu_ctx_status(self.handle, ctypes.byref(v)))
        return v.value

    @classmethod
    def default(cls, device: torch.device) -> "Context":
        key = device.index if device.index is not None else torch.cuda.current_device()
        if key not in cls._default:
            cls._default[key] = Context(torch.device("cuda", key))
        return cls._default[key]


def dequant(wtype: int, w: torch.Tensor, nrows: int, K: int, out_dtype=torch.float32) -> torch.Tensor:
    """Exact dequantisation of ``nrows`` GGUF rows of K weights -> [nrows, K] fp32 (or bf16 RNE)."""
    _need_cuda(w)
    if w.numel() * w.element_size() < nrows * row_bytes(wtype, K):
        raise ValueError("weight buffer smaller than nrows * row_bytes")
    out = torch.empty((nrows, K), dtype=out_dtype, device=w.device)
    check(lib().aipu_q4k_dequant(wtype, _ptr(w), nrows, K, _ptr(out), _DTYPE[out_dtype], _stream(w.device)))
    return out


def act(kind: str, x: torch.Tensor) -> torch.Tensor:
    """bf16 glm sigmoid (kind "sigmoid") or SiLU (kind "silu") of a bf16 tensor."""
    _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("act needs bf16 input")
    out = torch.empty_like(x)
    check(lib().aipu_act_eval({"sigmoid": 0, "silu": 1}[kind], _ptr(x), x.numel(), _ptr(out), _stream(x.device)))
    return out


def gemm(wtype: int, w: torch.Tensor, N: int, K: int, x: torch.Tensor, mode: str = "fast",
         ctx: Optional[Context] = None, out: Optional[torch.Tensor] = None,
         out_f32: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[M, N] bf16 = x[M, K] (fp32 or bf16) x W^T, W = N GGUF rows of K weights."""
    _need_cuda(w, x, out, out_f32)
    if x.dim() != 2 or x.shape[1] != K:
        raise ValueError("x must be [M, K]")
    if w.numel() * w.element_size() < N * row_bytes(wtype, K):
        raise ValueError("weight buffer smaller than N * row_bytes")
    ctx = ctx or Context.default(w.device)
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=w.device)
    m = L.MODE_STRICT if mode == "strict" else L.MODE_FAST
    check(lib().aipu_q4k_gemm(ctx.handle, wtype, _ptr(w), N, K, _ptr(x), _DTYPE[x.dtype], M, _ptr(out),
                              _ptr(out_f32), m, _stream(w.device)))
    return out


def gemm_tc(wtype: int, w: torch.Tensor, N: int, K: int, x: torch.Tensor, ctx: Optional[Context] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Prefill GEMM on tcgen05: y[M, N] bf16 = x[M, K] (bf16) x W^T, Q4_K or Q6_K rows."""
    _need_cuda(w, x, out)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != K:
        raise ValueError("x must be bf16 [M, K]")
    ctx = ctx or Context.default(w.device)
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=w.device)
    check(lib().aipu_q4k_gemm_tc(ctx.handle, wtype, _ptr(w), N, K, _ptr(x), M, _ptr(out), _stream(w.device)))
    return out


def bf16_dot_gemv(w: torch.Tensor, x: torch.Tensor, ctx: Optional[Context] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LM-head style GEMV: y[M, V] bf16 = the reference's bf16 dot (7 interleaved fp32 partial sums
    and a fixed add tree) of every token row x[M, K] with every weight row w[V, K] (both bf16)."""
    _need_cuda(w, x, out)
    if w.dtype != torch.bfloat16 or x.dtype != torch.bfloat16 or w.dim() != 2 or x.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("w [V, K] and x [M, K] must be bf16 with the same K")
    ctx = ctx or Context.default(w.device)
    w, x = w.contiguous(), x.contiguous()  # held until the launch is queued
    V, K = w.shape
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, V), dtype=torch.bfloat16, device=w.device)
    check(lib().aipu_bf16_dot_gemv(ctx.handle, _ptr(w), V, K, _ptr(x), M, _ptr(out), _stream(w.device)))
    return out


def gemm_grouped(wtype: int, w: torch.Tensor, n_mats: int, N: int, K: int, x: torch.Tensor,
                 mat_stride: Optional[int] = None, ctx: Optional[Context] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[g, M, N] bf16 = x[M, K] x W_g^T for n_mats matrices stored back to back (stride in bytes)."""
    _need_cuda(w, x, out)
    stride = mat_stride or N * row_bytes(wtype, K)
    if w.numel() * w.element_size() < (n_mats - 1) * stride + N * row_bytes(wtype, K):
        raise ValueError("weight buffer too small for n_mats matrices")
    ctx = ctx or Context.default(w.device)
    M = x.shape[0]
    if out is None:
        out = torch.empty((n_mats, M, N), dtype=torch.bfloat16, device=w.device)
    check(lib().aipu_q4k_gemm_grouped(ctx.handle, wtype, _ptr(w), n_mats, stride, N, K, _ptr(x), _DTYPE[x.dtype],
                                      M, _ptr(out), _stream(w.device)))
    return out


def moe_router(router_wtype: int, w: torch.Tensor, x: torch.Tensor, n_experts: int, topk: int,
               bias: Optional[torch.Tensor] = None, scale: float = 2.5, ctx: Optional[Context] = None,
               want_logits: bool = False):
    """Strict router: returns (sel int32 [M, topk], sel_w bf16 [M, topk], gate bf16 [M, E][, logits])."""
    _need_cuda(w, x, bias)
    if x.dtype != torch.bfloat16:
        raise ValueError("router activations must be bf16")
    M, K = x.shape
    ctx = ctx or Context.default(x.device)
    sel = torch.empty((M, topk), dtype=torch.int32, device=x.device)
    sw = torch.empty((M, topk), dtype=torch.bfloat16, device=x.device)
    gate = torch.empty((M, n_experts), dtype=torch.bfloat16, device=x.device)
    logits = torch.empty((M, n_experts), dtype=torch.bfloat16, device=x.device) if want_logits else None
    # the C entry point takes up to 1024 tokens per call; rows are independent
    x = x.contiguous()
    for m0 in range(0, M, 1024):
        m1 = min(M, m0 + 1024)
        check(lib().aipu_moe_router(ctx.handle, router_wtype, _ptr(w), _ptr(bias), _ptr(x[m0:m1]), m1 - m0, K,
                                    n_experts, topk, scale, _ptr(sel[m0:m1]), _ptr(sw[m0:m1]), _ptr(gate[m0:m1]),
                                    _ptr(logits[m0:m1]) if logits is not None else None, _stream(x.device)))
    return (sel, sw, gate, logits) if want_logits else (sel, sw, gate)


@dataclass
class MoeLayerWeights:
    """Device weights of one MoE layer (experts back to back in one uint8 tensor per projection)."""

    hidden: int
    ffn: int
    n_experts: int
    topk: int
    router_wtype: int
    router_w: Optional[torch.Tensor]
    gate_w: torch.Tensor
    up_w: torch.Tensor
    down_w: torch.Tensor
    gate_wtype: int = L.Q4_K
    down_wtype: int = L.Q6_K
    router_bias: Optional[torch.Tensor] = None
    shared_gate_w: Optional[torch.Tensor] = None
    shared_up_w: Optional[torch.Tensor] = None
    shared_down_w: Optional[torch.Tensor] = None
    scale: float = 2.5

    def cstruct(self) -> L.MoeWeights:
        s = L.MoeWeights()
        s.hidden, s.ffn, s.n_experts, s.topk, s.scale = self.hidden, self.ffn, self.n_experts, self.topk, self.scale
        s.router_wtype = self.router_wtype
        s.router_w = self.router_w.data_ptr() if self.router_w is not None else None
        s.router_bias = self.router_bias.data_ptr() if self.router_bias is not None else None
        s.gate_wtype = s.up_wtype = self.gate_wtype
        s.down_wtype = self.down_wtype
        s.gate_w, s.up_w, s.down_w = self.gate_w.data_ptr(), self.up_w.data_ptr(), self.down_w.data_ptr()
        if self.shared_gate_w is not None:
            s.shared_gate_w = self.shared_gate_w.data_ptr()
            s.shared_up_w = self.shared_up_w.data_ptr()
            s.shared_down_w = self.shared_down_w.data_ptr()
        return s


def moe_layer(W: MoeLayerWeights, x: torch.Tensor, ctx: Optional[Context] = None, out: Optional[torch.Tensor] = None,
              return_routing: bool = False):
    """MoE branch on bf16 rows x[M, H] -> bf16 [M, H] (router, union of experts, SwiGLU, combine)."""
    _need_cuda(x, out)
    if x.dtype != torch.bfloat16:
        raise ValueError("MoE activations must be bf16")
    M = x.shape[0]
    ctx = ctx or Context.default(x.device)
    if out is None:
        out = torch.empty((M, W.hidden), dtype=torch.bfloat16, device=x.device)
    sel = sw = None
    if return_routing:
        sel = torch.empty((M, W.topk), dtype=torch.int32, device=x.device)
        sw = torch.empty((M, W.topk), dtype=torch.bfloat16, device=x.device)
    cs = W.cstruct()
    check(lib().aipu_moe_layer(ctx.handle, ctypes.byref(cs), _ptr(x), M, _ptr(out), _ptr(sel), _ptr(sw),
                               _stream(x.device)))
    return (out, sel, sw) if return_routing else out


def swiglu_expert(gate_wtype: int, gate_w: torch.Tensor, up_w: torch.Tensor, down_wtype: int, down_w: torch.Tensor,
                  H: int, F: int, x: torch.Tensor, ctx: Optional[Context] = None, return_hidden: bool = False):
    """One SwiGLU expert on bf16 rows x[M, H] -> y bf16 [M, H] (and h bf16 [M, F])."""
    _need_cuda(gate_w, up_w, down_w, x)
    M = x.shape[0]
    ctx = ctx or Context.default(x.device)
    h = torch.empty((M, F), dtype=torch.bfloat16, device=x.device)
    y = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    check(lib().aipu_swiglu_expert(ctx.handle, gate_wtype, _ptr(gate_w), gate_wtype, _ptr(up_w), down_wtype,
                                   _ptr(down_w), H, F, _ptr(x), M, _ptr(h), _ptr(y), _stream(x.device)))
    return (y, h) if return_hidden else y


def expert_slice(W: MoeLayerWeights, lo: int, n: int) -> MoeLayerWeights:
    """The weights of routed experts [lo, lo + n) of W (views, no copy), shared expert and router kept."""
    F_rb = row_bytes(W.gate_wtype, W.hidden)
    D_rb = row_bytes(W.down_wtype, W.ffn)
    g = W.gate_w.view(-1)[lo * W.ffn * F_rb:(lo + n) * W.ffn * F_rb]
    u = W.up_w.view(-1)[lo * W.ffn * F_rb:(lo + n) * W.ffn * F_rb]
    d = W.down_w.view(-1)[lo * W.hidden * D_rb:(lo + n) * W.hidden * D_rb]
    return MoeLayerWeights(hidden=W.hidden, ffn=W.ffn, n_experts=n, topk=W.topk, router_wtype=W.router_wtype,
                           router_w=W.router_w, gate_w=g, up_w=u, down_w=d, gate_wtype=W.gate_wtype,
                           down_wtype=W.down_wtype, router_bias=W.router_bias, shared_gate_w=W.shared_gate_w,
                           shared_up_w=W.shared_up_w, shared_down_w=W.shared_down_w, scale=W.scale)


def moe_experts(W_local: MoeLayerWeights, expert_lo: int, x: torch.Tensor, sel: torch.Tensor,
                y_slots: Optional[torch.Tensor] = None, shared_range: Optional[tuple] = None,
                ctx: Optional[Context] = None):
    """Expert computation of one expert-parallel rank: y_slots[m, s] for the slots whose expert is in
    [expert_lo, expert_lo + W_local.n_experts), and the shared expert of tokens shared_range=(t0, n).
    Returns (y_slots [M, topk, H], y_shared [n, H] or None)."""
    _need_cuda(x, sel, y_slots)
    if x.dtype != torch.bfloat16 or sel.dtype != torch.int32:
        raise ValueError("moe_experts: x must be bf16 and sel int32")
    M = x.shape[0]
    ctx = ctx or Context.default(x.device)
    if y_slots is None:
        y_slots = torch.empty((M, W_local.topk, W_local.hidden), dtype=torch.bfloat16, device=x.device)
    t0, n = shared_range if shared_range is not None else (0, 0)
    y_sh = torch.empty((n, W_local.hidden), dtype=torch.bfloat16, device=x.device) if n > 0 else None
    cs = W_local.cstruct()
    check(lib().aipu_moe_experts(ctx.handle, ctypes.byref(cs), expert_lo, _ptr(x), M, _ptr(sel), _ptr(y_slots), t0, n,
                                 _ptr(y_sh), _stream(x.device)))
    return y_slots, y_sh


def moe_combine(sel: torch.Tensor, sel_w: torch.Tensor, experts_per_piece: int, pieces: torch.Tensor,
                y_shared: Optional[torch.Tensor] = None, ctx: Optional[Context] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[m] = bf16( sum_s sel_w[m, s] * pieces[sel[m, s] // experts_per_piece][m, s] + y_shared[m] ),
    slot order; pieces [P, M, topk, H] bf16."""
    _need_cuda(sel, sel_w, pieces, y_shared, out)
    P, M, T, H = pieces.shape
    ctx = ctx or Context.default(pieces.device)
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=pieces.device)
    check(lib().aipu_moe_combine(ctx.handle, M, H, T, _ptr(sel), _ptr(sel_w), experts_per_piece, _ptr(pieces),
                                 _ptr(y_shared), _ptr(out), _stream(pieces.device)))
    return out
