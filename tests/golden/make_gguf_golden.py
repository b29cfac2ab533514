#!/usr/bin/env python3
"""Generate tests/golden/ref_synthetic.gguf and gguf_golden.npz with the REFERENCE's own GGUF codec.

    AIPU_REFERENCE=/path/to/AIPU python tests/golden/make_gguf_golden.py

``tools/ckpt_pack_q4k.py`` (unchanged) writes its seeded synthetic mixed-type GGUF (Q4_K, Q6_K,
Q8_0, F16, F32 tensors) and parses it back with its own reader; ``tools/q4k_ref.py`` dequantises
every quantised tensor. The npz stores, per tensor, the reference reader's type, dims and raw bytes
and the reference dequantisation (fp32 bits, row-major [N, K]). The tests parse the .gguf with
aipu_b200.gguf and compare against these, without the reference tree.
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

import ckpt_pack_q4k as CP  # noqa: E402  (reference module, unchanged)
import q4k_ref as R          # noqa: E402


def ref_dequant(ttype, raw):
    if ttype == CP.GGML_Q4_K:
        out = [R.dequantize_block_q4_K(int.from_bytes(raw[o:o + 2], "little"), int.from_bytes(raw[o + 2:o + 4], "little"),
                                       raw[o + 4:o + 16], raw[o + 16:o + 144]) for o in range(0, len(raw), 144)]
    elif ttype == CP.GGML_Q6_K:
        out = [R.dequantize_block_q6_K(int.from_bytes(raw[o + 208:o + 210], "little"), raw[o:o + 128],
                                       raw[o + 128:o + 192], raw[o + 192:o + 208]) for o in range(0, len(raw), 210)]
    elif ttype == CP.GGML_Q8_0:
        out = [R.dequantize_block_q8_0(int.from_bytes(raw[o:o + 2], "little"),
                                       np.frombuffer(raw[o + 2:o + 34], dtype=np.int8)) for o in range(0, len(raw), 34)]
    else:
        return None
    return np.concatenate(out).astype(np.float32)


def main():
    buf = CP.gen_synthetic(None)
    with open(os.path.join(HERE, "ref_synthetic.gguf"), "wb") as f:
        f.write(buf)
    meta, tensors = CP.read_gguf(buf)
    out = {"names": np.array(sorted(tensors), dtype=object).astype(str)}
    for i, name in enumerate(sorted(tensors)):
        ttype, dims, raw = tensors[name]
        out[f"t{i}_type"] = np.array([ttype], np.int64)
        out[f"t{i}_dims"] = np.array(dims, np.int64)
        out[f"t{i}_raw"] = np.frombuffer(raw, np.uint8).copy()
        deq = ref_dequant(ttype, raw)
        if deq is not None:
            out[f"t{i}_deq"] = deq.view(np.uint32).reshape(dims[1], dims[0])
    out["alignment"] = np.array([meta.get("general.alignment", 32)], np.int64)
    np.savez_compressed(os.path.join(HERE, "gguf_golden.npz"), **out)
    print("wrote ref_synthetic.gguf", len(buf), "bytes;", len(tensors), "tensors")


if __name__ == "__main__":
    main()
