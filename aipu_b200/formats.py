"""GGUF k-quant block formats and seeded synthetic weight generators.

Block layouts (ggml; rows of blocks along K, rows back to back):
  Q4_K 144 B: [fp16 d][fp16 dmin][12 B packed 6-bit scales/mins][128 B qs]   (256 weights)
  Q6_K 210 B: [128 B ql][64 B qh][16 x int8 scales][fp16 d]                    (256 weights)
  Q8_0  34 B: [fp16 d][32 x int8]                                              (32 weights)
  F16    2 B / weight, F32 4 B / weight

The generators follow the distributions of the benchmark configurations: d, dmin =
fp16(|N(0,1)| * 2^-8); Q4_K 6-bit scales and mins uniform 0..63; Q6_K int8 scales uniform
-32..31; quant bytes uniform; F16 ~ N(0, 0.02). ``*_np`` versions are numpy (host, seeded,
reproducible anywhere); ``*_dev`` versions draw on the GPU with a seeded torch generator (for
multi-GB benchmark weights).
"""
from __future__ import annotations

import numpy as np

Q4_K, Q6_K, Q8_0, F16, F32 = 0, 1, 2, 3, 4
NAMES = {Q4_K: "Q4_K", Q6_K: "Q6_K", Q8_0: "Q8_0", F16: "F16", F32: "F32"}
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34, F16: 2, F32: 4}
BLOCK_WEIGHTS = {Q4_K: 256, Q6_K: 256, Q8_0: 32, F16: 1, F32: 1}


def row_bytes(wtype: int, K: int) -> int:
    bw = BLOCK_WEIGHTS[wtype]
    if K % bw:
        raise ValueError(f"K={K} is not a multiple of the {NAMES[wtype]} block ({bw})")
    return (K // bw) * BLOCK_BYTES[wtype]


def pack_scales_np(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack 6-bit scales/mins [..., 8] into the 12-byte Q4_K table (inverse of get_scale_min_k4)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    q = np.empty(sc.shape[:-1] + (12,), np.uint8)
    q[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    q[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    q[..., 8:12] = (sc[..., 4:8] & 0xF) | ((mn[..., 4:8] & 0xF) << 4)
    return q


def _f16_scale_np(rng, n):
    return (np.abs(rng.standard_normal(n)) * 2.0 ** -8).astype(np.float16).view(np.uint8).reshape(n, 2)


def random_rows_np(wtype: int, N: int, K: int, seed: int = 0) -> np.ndarray:
    """N rows x K weights of type `wtype` as uint8 [N, row_bytes] (numpy, seeded)."""
    rng = np.random.default_rng(seed)
    rb = row_bytes(wtype, K)
    if wtype == F16:
        return rng.normal(0.0, 0.02, (N, K)).astype(np.float16).view(np.uint8).reshape(N, rb)
    if wtype == F32:
        return rng.normal(0.0, 0.02, (N, K)).astype(np.float32).view(np.uint8).reshape(N, rb)
    nb = N * K // BLOCK_WEIGHTS[wtype]
    b = rng.integers(0, 256, (nb, BLOCK_BYTES[wtype]), dtype=np.uint8)
    if wtype == Q4_K:
        b[:, 0:2] = _f16_scale_np(rng, nb)
        b[:, 2:4] = _f16_scale_np(rng, nb)
        b[:, 4:16] = pack_scales_np(rng.integers(0, 64, (nb, 8)), rng.integers(0, 64, (nb, 8)))
    elif wtype == Q6_K:
        b[:, 192:208] = rng.integers(-32, 32, (nb, 16)).astype(np.int8).view(np.uint8)
        b[:, 208:210] = _f16_scale_np(rng, nb)
    elif wtype == Q8_0:
        b[:, 0:2] = _f16_scale_np(rng, nb)
    return b.reshape(N, rb)


def random_rows_dev(wtype: int, N: int, K: int, seed: int = 0, device="cuda", out=None):
    """Like random_rows_np but drawn on the GPU (torch generator seeded with `seed`)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rb = row_bytes(wtype, K)
    if out is None:
        out = torch.empty((N, rb), dtype=torch.uint8, device=device)
    if wtype in (F16, F32):
        dt = torch.float16 if wtype == F16 else torch.float32
        v = out.view(-1).view(dt)
        v.normal_(0.0, 0.02, generator=g)
        return out
    nb = N * K // BLOCK_WEIGHTS[wtype]
    bb = BLOCK_BYTES[wtype]
    flat = out.view(-1)
    flat.random_(0, 256, generator=g)
    b = flat.view(nb, bb)

    def f16_scales():
        return (torch.randn(nb, device=device, generator=g).abs_() * 2.0 ** -8).to(torch.float16).view(torch.uint8)

    if wtype == Q4_K:
        b[:, 0:2] = f16_scales().view(nb, 2)
        b[:, 2:4] = f16_scales().view(nb, 2)
        sc = torch.randint(0, 64, (nb, 8), device=device, generator=g, dtype=torch.int32)
        mn = torch.randint(0, 64, (nb, 8), device=device, generator=g, dtype=torch.int32)
        q = torch.empty((nb, 12), dtype=torch.int32, device=device)
        q[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
        q[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
        q[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
        b[:, 4:16] = q.to(torch.uint8)
    elif wtype == Q6_K:
        b[:, 192:208] = torch.randint(-32, 32, (nb, 16), device=device, generator=g, dtype=torch.int8).view(torch.uint8)
        b[:, 208:210] = f16_scales().view(nb, 2)
    elif wtype == Q8_0:
        b[:, 0:2] = f16_scales().view(nb, 2)
    return out
