"""GGUF v3 container (aipu_b200.gguf) on CPU: the reference-written synthetic checkpoint parses to
the reference reader's tensors byte for byte and dequantises (oracle) to the reference's own fp32
values; the writer round-trips; malformed files are rejected; MoE layers load with the right
layouts."""
import os
import struct

import numpy as np
import pytest
import torch

from aipu_b200 import formats as F
from aipu_b200 import gguf
from oracle import q4k_oracle as qo

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_reference_written_gguf_parses_bit_exact(golden):
    g = golden("gguf_golden")
    names = [str(n) for n in g["names"]]
    with gguf.GGUFFile(os.path.join(GOLDEN, "ref_synthetic.gguf")) as gf:
        assert sorted(gf.tensors) == names
        assert gf.alignment == int(g["alignment"][0])
        for i, name in enumerate(names):
            t = gf.info(name)
            assert t.ggml_type == int(g[f"t{i}_type"][0])
            assert list(t.ne) == list(g[f"t{i}_dims"])
            raw = gf.raw(name)
            assert np.array_equal(raw.reshape(-1), g[f"t{i}_raw"]), name
            if f"t{i}_deq" in g:  # quantised: rows of blocks, ne[0] = K per row
                K, N = t.ne
                deq = qo.dequant_rows(t.wtype, raw, N, K)
                assert np.array_equal(deq.view(np.uint32), g[f"t{i}_deq"]), name


def test_writer_round_trip(tmp_path):
    p = str(tmp_path / "rt.gguf")
    specs = [gguf.TensorSpec("a.q4k", gguf.GGML_Q4_K, (512, 3), F.random_rows_np(F.Q4_K, 3, 512, seed=1).tobytes()),
             gguf.TensorSpec("b.q6k", gguf.GGML_Q6_K, (256, 5, 2), F.random_rows_np(F.Q6_K, 10, 256, seed=2).tobytes()),
             gguf.TensorSpec("c.q80", gguf.GGML_Q8_0, (64, 7), F.random_rows_np(F.Q8_0, 7, 64, seed=3).tobytes()),
             gguf.TensorSpec("d.f16", gguf.GGML_F16, (33, 2), F.random_rows_np(F.F16, 2, 33, seed=4).tobytes()),
             gguf.TensorSpec("e.f32", gguf.GGML_F32, (9,), np.arange(9, dtype=np.float32).tobytes())]
    meta = {"general.architecture": "x", "x.block_count": 3, "x.expert_weights_scale": 2.5, "x.flag": True,
            "x.list": [1, 2, 3], "x.names": ["p", "qq"], "x.neg": -5}
    gguf.write_gguf(p, specs, meta, alignment=64)
    with gguf.GGUFFile(p) as gf:
        assert gf.alignment == 64 and gf.data_start % 64 == 0
        for s in specs:
            t = gf.info(s.name)
            assert t.ne == s.ne and t.ggml_type == s.ggml_type and t.offset % 64 == 0
            assert gf.raw(s.name).tobytes() == s.data
        assert gf.arch() == "x" and gf.arch_value("block_count") == 3
        assert gf.metadata["x.flag"] is True and gf.metadata["x.list"] == [1, 2, 3]
        assert gf.metadata["x.names"] == ["p", "qq"] and gf.metadata["x.neg"] == -5
        assert abs(gf.metadata["x.expert_weights_scale"] - 2.5) < 1e-7


def test_malformed_files_are_rejected(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(gguf.GGUFError, match="magic"):
        gguf.GGUFFile(str(p))
    p.write_bytes(struct.pack("<IIQQ", gguf.GGUF_MAGIC, 2, 0, 0))
    with pytest.raises(gguf.GGUFError, match="version"):
        gguf.GGUFFile(str(p))
    good = tmp_path / "good.gguf"
    gguf.write_gguf(str(good), [gguf.TensorSpec("w", gguf.GGML_Q4_K, (256, 4),
                                                F.random_rows_np(F.Q4_K, 4, 256, seed=5).tobytes())])
    data = good.read_bytes()
    p.write_bytes(data[:-100])
    with pytest.raises(gguf.GGUFError, match="past the end"):
        gguf.GGUFFile(str(p))
    p.write_bytes(data[:20])
    with pytest.raises(gguf.GGUFError, match="truncated"):
        gguf.GGUFFile(str(p))
    with pytest.raises(gguf.GGUFError, match="type"):
        gguf.write_gguf(str(p), [gguf.TensorSpec("w", 2, (32,), b"\0" * 18)])  # Q4_0: not handled


def test_moe_layer_loads_with_kernel_layouts(tmp_path):
    p = str(tmp_path / "moe.gguf")
    H, Fd, E = 512, 256, 8
    gguf.synthetic_moe_gguf(p, layers=2, H=H, Fd=Fd, E=E, topk=4, seed=3)
    with gguf.GGUFFile(p) as gf:
        assert gf.moe_layers() == [0, 1]
        W = gguf.load_moe_layer(gf, 1, "cpu")
        assert (W.hidden, W.ffn, W.n_experts, W.topk) == (H, Fd, E, 4) and abs(W.scale - 2.5) < 1e-7
        assert W.gate_wtype == F.Q4_K and W.down_wtype == F.Q6_K and W.router_wtype == F.F32
        # router: GGUF stores E rows of H; the fp32 router kernel reads [H, E]
        r = np.array(gf.raw("blk.1.ffn_gate_inp.weight")).view(np.float32).reshape(E, H)
        assert np.array_equal(W.router_w.numpy(), r.T)
        assert W.gate_w.shape == (E * Fd, F.row_bytes(F.Q4_K, H))
        assert W.down_w.shape == (E * H, F.row_bytes(F.Q6_K, Fd))
        assert torch.equal(W.up_w, torch.from_numpy(np.array(gf.raw("blk.1.ffn_up_exps.weight"))))
        assert W.shared_down_w.shape == (H, F.row_bytes(F.Q6_K, Fd)) and W.router_bias.shape == (E,)
        with pytest.raises(KeyError):
            gguf.load_moe_layer(gf, 2, "cpu")


def test_load_matrix_keeps_rows_and_type():
    with gguf.GGUFFile(os.path.join(GOLDEN, "ref_synthetic.gguf")) as gf:
        m = gguf.load_matrix(gf, "blk.0.ffn_down.weight", "cpu")
        assert (m.wtype, m.N, m.K) == (F.Q4_K, 8, 512)
        assert m.rows.shape == (8, F.row_bytes(F.Q4_K, 512))
        assert np.array_equal(m.rows.numpy(), np.array(gf.raw("blk.0.ffn_down.weight")))
        with pytest.raises(gguf.GGUFError):
            gguf.load_matrix(gf, "blk.0.attn_norm.weight", "cpu")


def test_load_matrix_rejects_non_gemm_tensors(tmp_path):
    """A 2-D F32 tensor, or one whose K is not a multiple of 256, is refused at load time with its name."""
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, [gguf.TensorSpec("f32w", gguf.GGML_F32, (256, 4), np.zeros(1024, np.float32).tobytes()),
                        gguf.TensorSpec("q8w", gguf.GGML_Q8_0, (96, 4), F.random_rows_np(F.Q8_0, 4, 96, seed=1).tobytes()),
                        gguf.TensorSpec("okw", gguf.GGML_Q8_0, (256, 4), F.random_rows_np(F.Q8_0, 4, 256, seed=2).tobytes())])
    with gguf.GGUFFile(p) as gf:
        with pytest.raises(gguf.GGUFError, match="f32w"):
            gguf.load_matrix(gf, "f32w", "cpu")
        with pytest.raises(gguf.GGUFError, match="q8w.*256"):
            gguf.load_matrix(gf, "q8w", "cpu")
        m = gguf.load_matrix(gf, "okw", "cpu")
        assert (m.wtype, m.N, m.K) == (F.Q8_0, 4, 256)


def test_manifest_round_trip_and_corruption(tmp_path):
    """The per-tensor integrity manifest (the reference provisioning manifest's per-tensor fields) of a
    reference-written GGUF verifies against it; a manifest in the reference's layout (extra image
    fields) is accepted; a flipped byte, a wrong shape or a missing tensor is reported."""
    import json

    with gguf.GGUFFile(os.path.join(GOLDEN, "ref_synthetic.gguf")) as gf:
        m = gguf.tensor_manifest(gf)
        assert m["tensor_count"] == len(gf.tensors) and gguf.verify_manifest(gf, m) == []
        ref_style = {"format_version": "provimg-1.0", "image_sha256": "0" * 64, "segments": [],
                     "tensors": [dict(t, offset=i * 4096, segment="resident_hot") for i, t in enumerate(m["tensors"])]}
        assert gguf.verify_manifest(gf, json.loads(json.dumps(ref_style))) == []
        bad = json.loads(json.dumps(m))
        bad["tensors"][0]["sha256"] = "f" * 64
        bad["tensors"][1]["shape"] = [1, 2]
        bad["tensors"].append({"name": "missing.weight", "sha256": "0" * 64})
        fails = gguf.verify_manifest(gf, bad)
        assert len(fails) == 3 and "sha256" in fails[0] and "shape" in fails[1] and "not present" in fails[2]
    # a corrupted copy of the file fails against the manifest of the original
    data = bytearray(open(os.path.join(GOLDEN, "ref_synthetic.gguf"), "rb").read())
    t0 = m["tensors"][0]
    data[t0["src_offset"] + 7] ^= 0x10
    p = tmp_path / "corrupt.gguf"
    p.write_bytes(bytes(data))
    with gguf.GGUFFile(str(p)) as gf:
        fails = gguf.verify_manifest(gf, m)
        assert len(fails) == 1 and t0["name"] in fails[0]
