#!/usr/bin/env python3
"""Generate tests/golden/lmhead_golden.npz with the REFERENCE's own bf16 dot product.

    AIPU_REFERENCE=/path/to/AIPU python tests/golden/make_lmhead_golden.py

``tools/glm_model_q4k_ref.py`` (unchanged) provides ``matmul_bf16_dot`` (the LM-head / bf16 GEMV
contract: 7 interleaved fp32 partial sums, then a fixed 3-level add tree, bf16 out). Seeded
bf16-valued inputs; the npz stores inputs and outputs as bit patterns.
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

import glm_model_q4k_ref as G  # noqa: E402  (reference module, unchanged)
import q4k_ref as R            # noqa: E402

F32 = np.float32


def bf16_vals(rng, shape, scale):
    v = (rng.standard_normal(shape) * scale).astype(F32)
    return np.array([R.bf16_round(F32(t)) for t in v.reshape(-1)], F32).reshape(shape)


def case(rng, V, K, M, scale_w):
    x = bf16_vals(rng, (M, K), 1.0)
    w = bf16_vals(rng, (V, K), scale_w)
    w[0, :] = 0.0                  # an all-zero row
    w[1, ::7] = -w[1, ::7]          # sign pattern on one chain
    y = np.array([[G.matmul_bf16_dot(list(x[m]), list(w[v])) for v in range(V)] for m in range(M)], F32)
    return x, w, y


def main():
    rng = np.random.default_rng(20240611)
    out = {}
    for name, (V, K, M, s) in {"a": (12, 6144, 2, 0.02), "b": (10, 1000, 3, 1.0), "c": (7, 56, 1, 4.0)}.items():
        x, w, y = case(rng, V, K, M, s)
        out[f"{name}_x"] = x.view(np.uint32) >> 16
        out[f"{name}_w"] = w.view(np.uint32) >> 16
        out[f"{name}_y"] = y.view(np.uint32) >> 16
    np.savez_compressed(os.path.join(HERE, "lmhead_golden.npz"), **{k: v.astype(np.uint16) for k, v in out.items()})
    print("wrote lmhead_golden.npz")


if __name__ == "__main__":
    main()
