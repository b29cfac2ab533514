"""Drop-in for the reference's ``tools/q4k_ref.py``: the same names and arguments, computed by the
CUDA library (GGML k-quant dequantisation and the sequential-fp32 GEMM contract).

    from aipu_b200 import q4k_ref          # instead of: import q4k_ref
    y = q4k_ref.dequantize_block_q4_K(d_h, dmin_h, scales, qs)

Every dequantisation and dot product runs on the GPU through the C ABI (``aipu_q4k_dequant``,
``aipu_q4k_gemm`` in strict mode); results are bit-identical to the reference. The small format
helpers (6-bit scale packing, bf16 rounding of a scalar, signed-byte conversion) are host-side bit
manipulation, as in the reference. There is no CPU fallback: without the built library or a CUDA
device every compute call raises.

Batch forms for many blocks at once are ``dequantize_row_q4_K`` (one launch per row) and
``aipu_b200.ops.dequant`` / ``aipu_b200.ops.gemm`` on device tensors.
"""
from __future__ import annotations

import numpy as np
import torch

from . import formats as F
from . import ops

QK_K = 256

_DEV = None


def _dev() -> torch.device:
    global _DEV
    if _DEV is None:
        if not torch.cuda.is_available():
            raise RuntimeError("aipu_b200.q4k_ref needs a CUDA device (there is no CPU path)")
        _DEV = torch.device("cuda", torch.cuda.current_device())
    return _DEV


def _u8(seq) -> np.ndarray:
    """bytes / list of byte values (or int8 values) -> uint8 array"""
    if isinstance(seq, (bytes, bytearray)):
        return np.frombuffer(bytes(seq), dtype=np.uint8)
    return np.asarray([int(v) & 0xFF for v in seq], dtype=np.uint8)


def _dequant_bytes(wtype: int, raw: np.ndarray, nblocks: int, per_block: int) -> np.ndarray:
    w = torch.from_numpy(np.ascontiguousarray(raw)).to(_dev())
    out = ops.dequant(wtype, w, 1, nblocks * per_block)
    return out.cpu().numpy().reshape(-1)


# ---------------------------------------------------------------- format helpers (host)
def get_scale_min_k4(j, scales):
    """6-bit (scale, min) of sub-block j from the 12-byte table (tools/q4k_ref.py:27-37)."""
    q = scales
    if j < 4:
        return q[j] & 63, q[j + 4] & 63
    return (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4), (q[j + 4] >> 4) | ((q[j] >> 6) << 4)


def _s8(b):
    """Raw byte -> signed int8 value (tools/q4k_ref.py:99-103)."""
    return b - 256 if b > 127 else b


def _pack_6bit_scales(scs, mns):
    """8 six-bit scales + 8 six-bit mins -> the 12-byte table (tools/q4k_ref.py:132-145)."""
    assert len(scs) == 8 and len(mns) == 8 and all(0 <= v < 64 for v in list(scs) + list(mns))
    q = [0] * 12
    for j in range(4):
        q[j] = scs[j]
        q[j + 4] = mns[j]
    for j in range(4, 8):
        q[j + 4] = (scs[j] & 0xF) | ((mns[j] & 0xF) << 4)
        q[j - 4] |= ((scs[j] >> 4) & 0x3) << 6
        q[j] |= ((mns[j] >> 4) & 0x3) << 6
    return q


def _f32_to_f16bits(x):
    return int(np.frombuffer(np.float16(x).tobytes(), dtype=np.uint16)[0])


def bf16_round(x):
    """fp32 -> bf16-valued fp32, round-to-nearest-even; inf/nan truncated (tools/q4k_ref.py:76-84)."""
    u = int(np.frombuffer(np.float32(x).tobytes(), dtype=np.uint32)[0])
    if (u & 0x7F800000) == 0x7F800000:
        u2 = u & 0xFFFF0000
    else:
        u2 = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return np.float32(np.frombuffer(np.uint32(u2).tobytes(), dtype=np.float32)[0])


# ---------------------------------------------------------------- block packing
def pack_block_q4_K(d_h, dmin_h, scales, qs) -> np.ndarray:
    """GGUF Q4_K block bytes (144): fp16 d, fp16 dmin, 12 scale bytes, 128 quant bytes."""
    b = np.zeros(144, np.uint8)
    b[0:2] = np.frombuffer(np.uint16(d_h & 0xFFFF).tobytes(), np.uint8)
    b[2:4] = np.frombuffer(np.uint16(dmin_h & 0xFFFF).tobytes(), np.uint8)
    b[4:16] = _u8(scales)[:12]
    b[16:144] = _u8(qs)[:128]
    return b


def pack_block_q6_K(d_h, ql, qh, sc) -> np.ndarray:
    """GGUF Q6_K block bytes (210): ql[128], qh[64], int8 scales[16], fp16 d."""
    b = np.zeros(210, np.uint8)
    b[0:128] = _u8(ql)[:128]
    b[128:192] = _u8(qh)[:64]
    b[192:208] = _u8(sc)[:16]
    b[208:210] = np.frombuffer(np.uint16(d_h & 0xFFFF).tobytes(), np.uint8)
    return b


def pack_block_q8_0(d_h, qs) -> np.ndarray:
    """GGUF Q8_0 block bytes (34): fp16 d, 32 int8."""
    b = np.zeros(34, np.uint8)
    b[0:2] = np.frombuffer(np.uint16(d_h & 0xFFFF).tobytes(), np.uint8)
    b[2:34] = _u8(qs)[:32]
    return b


# ---------------------------------------------------------------- dequantisation (GPU)
def dequantize_block_q4_K(d_h, dmin_h, scales, qs):
    """ONE Q4_K super-block -> 256 fp32, exactly as ggml (tools/q4k_ref.py:39-61)."""
    return _dequant_bytes(F.Q4_K, pack_block_q4_K(d_h, dmin_h, scales, qs), 1, QK_K)


def dequantize_row_q4_K(blocks):
    """Iterable of (d_h, dmin_h, scales, qs) -> the concatenated fp32 row (tools/q4k_ref.py:63-65)."""
    raw = [pack_block_q4_K(*b) for b in blocks]
    if not raw:
        return np.zeros(0, np.float32)
    return _dequant_bytes(F.Q4_K, np.concatenate(raw), len(raw), QK_K)


def dequantize_block_q6_K(d_h, ql, qh, sc):
    """ONE Q6_K super-block -> 256 fp32 (tools/q4k_ref.py:105-124). ``sc`` holds raw bytes or int8."""
    return _dequant_bytes(F.Q6_K, pack_block_q6_K(d_h, ql, qh, sc), 1, QK_K)


def dequantize_block_q8_0(d_h, qs):
    """ONE Q8_0 block -> 32 fp32 (tools/q4k_ref.py:126-129)."""
    return _dequant_bytes(F.Q8_0, pack_block_q8_0(d_h, qs), 1, 32)


# ---------------------------------------------------------------- GEMM contract (GPU)
def matmul_q4k_col(a_row_f32, wdeq_col_f32):
    """bf16( sequential fp32 sum_k a[k] * w[k] ) of one bf16-valued activation row and one
    dequantised weight column (tools/q4k_ref.py:86-92), as the strict GEMM on the GPU."""
    a = np.ascontiguousarray(np.asarray(a_row_f32, np.float32).reshape(1, -1))
    w = np.ascontiguousarray(np.asarray(wdeq_col_f32, np.float32).reshape(1, -1))
    if a.shape[1] != w.shape[1]:
        raise ValueError("activation row and weight column differ in length")
    d = _dev()
    y = ops.gemm(F.F32, torch.from_numpy(w.view(np.uint8)).to(d), 1, a.shape[1], torch.from_numpy(a).to(d),
                 mode="strict")
    return np.float32(y.float().cpu().numpy()[0, 0])
