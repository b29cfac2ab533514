"""The drop-in's seeded weight generators (aipu_b200.glm_model_q4k_ref Weights, _mk_qw) reproduce the
reference's weights exactly (digests made by tests/golden/make_weights_golden.py from the reference's
own tools/glm_model_q4k_ref.py). Host-only: building the weights needs no GPU."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from aipu_b200 import glm_model_q4k_ref as g  # noqa: E402
import make_weights_golden as mk  # noqa: E402


@pytest.mark.parametrize("name,kw,seed", mk.CASES)
def test_weights_match_reference(golden, name, kw, seed):
    ref = golden("weights_golden")
    cfg = g.Config(**(g.SPEC_SLICE if kw == "SPEC_SLICE" else kw))
    W = g.Weights(cfg, seed=seed)
    assert mk.digest(W) == bytes(ref[name]).hex()
    if name == "spec_slice_seed11":
        assert np.array_equal(np.asarray(W.Mg[0][0].codes, np.uint8), ref["spec_Mg00_codes"])
        assert np.array_equal(np.asarray(W.Mg[0][0].scales, np.uint8), ref["spec_Mg00_scales"])


def test_config_derived_dims():
    c = g.Config(**g.SPEC_SLICE)
    assert (c.QK_DIM, c.HQK, c.HNOPE, c.HV, c.SWIN) == (8, 16, 8, 8, 2)
