"""The aipu_dequant_dump CLI (aipu_b200/csrc/dequant_dump.cpp): the reference's ggml dump tool's command
line (tools/dequant_dump.c:16-39) over the library's exact GPU dequant.

CPU tests: the binary is built and rejects a bad command line, an unknown type and a file that is not a
whole number of blocks (all before touching the GPU). GPU test: it reproduces the reference's own
dequantised blocks (tests/golden/dequant_golden.npz, made by tools/q4k_ref.py) bit for bit.
"""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DUMP = os.path.join(ROOT, "aipu_b200", "aipu_dequant_dump")


@pytest.fixture(scope="module")
def dump():
    if not os.path.exists(DUMP):
        from aipu_b200 import build

        build.build()
    assert os.path.exists(DUMP)
    return DUMP


def test_usage_and_type_errors(dump, tmp_path):
    assert subprocess.run([dump], capture_output=True).returncode == 2
    r = subprocess.run([dump, "q5_k", "a", "b"], capture_output=True)
    assert r.returncode == 2 and b"unknown type" in r.stderr
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"\0" * 145)
    r = subprocess.run([dump, "q4_k", str(bad), str(tmp_path / "o.bin")], capture_output=True)
    assert r.returncode == 1 and b"multiple" in r.stderr
    r = subprocess.run([dump, "q6_k", str(tmp_path / "missing.bin"), str(tmp_path / "o.bin")], capture_output=True)
    assert r.returncode == 1


@pytest.mark.gpu
@pytest.mark.parametrize("kind,blocks,want", [("q4_k", "q4k_blocks", "q4k_y"), ("q6_k", "q6k_blocks", "q6k_y"),
                                              ("q8_0", "q80_blocks", "q80_y"), ("f16", "f16_bits", "f16_y")])
def test_dump_matches_reference_fixture(dump, tmp_path, golden, kind, blocks, want):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = golden("dequant_golden")
    src, out = tmp_path / "in.bin", tmp_path / "out.bin"
    src.write_bytes(np.ascontiguousarray(g[blocks]).tobytes())
    r = subprocess.run([dump, kind, str(src), str(out)], capture_output=True)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, dtype=np.uint32)
    assert np.array_equal(got, g[want].reshape(-1))
