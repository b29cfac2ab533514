"""Generates tests/golden/weights_golden.npz: digests of the reference's seeded model weights
(tools/glm_model_q4k_ref.py Weights / _mk_qw), made by importing the reference module unchanged.

    python tests/golden/make_weights_golden.py /path/to/reference

The drop-in aipu_b200.glm_model_q4k_ref.Weights must reproduce them exactly (tests/test_dropin_weights.py).
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
FIELDS = ("EMB", "G1", "G2", "W_dq", "W_uq", "W_uk", "W_uv", "W_o", "CKV", "KRP", "Wg", "Dg", "Du", "Dd", "Mg", "Mu",
          "Md", "SHg", "SHu", "SHd", "GF", "Wlm")


def _feed(h, v):
    if hasattr(v, "codes"):  # a QW
        h.update(np.asarray(v.codes, np.uint8).tobytes())
        h.update(np.asarray(v.d, np.uint16).tobytes())
        h.update(np.asarray(v.dmin, np.uint16).tobytes())
        h.update(np.asarray(v.scales, np.uint8).tobytes())
        h.update(np.asarray([v.nout, v.nin], np.int64).tobytes())
    elif isinstance(v, (list, tuple)) and v and (isinstance(v[0], (list, tuple)) or hasattr(v[0], "codes")):
        for u in v:
            _feed(h, u)
    else:
        h.update(np.asarray(v, np.float32).tobytes())


def digest(W) -> str:
    h = hashlib.sha256()
    for f in FIELDS:
        h.update(f.encode())
        _feed(h, getattr(W, f))
    return h.hexdigest()


CASES = [("default_seed7", {}, 7), ("spec_slice_seed11", "SPEC_SLICE", 11), ("default_seed424242", {}, 424242)]


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import glm_model_q4k_ref as ref

    out = {}
    for name, kw, seed in CASES:
        cfg = ref.Config(**(ref.SPEC_SLICE if kw == "SPEC_SLICE" else kw))
        W = ref.Weights(cfg, seed=seed)
        out[name] = np.frombuffer(bytes.fromhex(digest(W)), np.uint8)
        if name == "spec_slice_seed11":
            out["spec_Mg00_codes"] = np.asarray(W.Mg[0][0].codes, np.uint8)
            out["spec_Mg00_scales"] = np.asarray(W.Mg[0][0].scales, np.uint8)
            out["spec_Mg00_d"] = np.asarray(W.Mg[0][0].d, np.uint16)
    np.savez_compressed(os.path.join(HERE, "weights_golden.npz"), **out)
    print("wrote", sorted(out))


if __name__ == "__main__":
    # the reference tree's root: first argument, else the AIPU_REFERENCE environment variable
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AIPU_REFERENCE", "")
    if not root:
        sys.exit("usage: make_weights_golden.py <reference tree root> (or set AIPU_REFERENCE)")
    main(root)
