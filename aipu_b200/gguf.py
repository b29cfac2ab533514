"""GGUF v3 checkpoints: a reader that maps tensors without copying, a writer (synthetic files and
fixtures), and a loader that builds MoE layer weights for this library's kernels.

The container format follows the layout the reference's packer reads and writes
(tools/ckpt_pack_q4k.py:70-170): little-endian header ``"GGUF"``, version 3, tensor count, metadata
count; metadata key/value pairs (typed values, arrays, strings as u64 length + UTF-8); tensor infos
(name, dims in ggml ``ne`` order — ne[0] is the fastest, i.e. the reduction length K — ggml type,
offset relative to the data section); the data section starts at the next multiple of
``general.alignment`` (default 32).

Tensor types handled (the reference's per-tensor type map, tools/ckpt_pack_q4k.py:58-67): F32 (0),
F16 (1), Q8_0 (8), Q4_K (12), Q6_K (14). Quantised rows are used exactly as stored: a tensor with
ne = [K, N] is N rows of K/block blocks, which is the row layout every kernel here consumes.

MoE tensor names follow llama.cpp's convention for routed-expert models:
``blk.{i}.ffn_gate_inp.weight`` (router, ne = [H, E]), ``blk.{i}.exp_probs_b.bias`` (selection bias,
[E]), ``blk.{i}.ffn_{gate,up}_exps.weight`` (ne = [H, F, E]), ``blk.{i}.ffn_down_exps.weight``
(ne = [F, H, E]) and the shared expert ``blk.{i}.ffn_{gate,up,down}_shexp.weight``.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import formats as F

GGUF_MAGIC = 0x46554747  # "GGUF"
GGUF_VERSION = 3

# ggml type id -> (format of this package, weights per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 8, 12, 14
GGML_TYPES = {
    GGML_F32: (F.F32, 1, 4),
    GGML_F16: (F.F16, 1, 2),
    GGML_Q8_0: (F.Q8_0, 32, 34),
    GGML_Q4_K: (F.Q4_K, 256, 144),
    GGML_Q6_K: (F.Q6_K, 256, 210),
}
FORMAT_TO_GGML = {v[0]: k for k, v in GGML_TYPES.items()}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_FIXED = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
          _U64: "<Q", _I64: "<q", _F64: "<d"}


class GGUFError(ValueError):
    pass


def tensor_nbytes(ggml_type: int, ne: Sequence[int]) -> int:
    if ggml_type not in GGML_TYPES:
        raise GGUFError(f"unsupported ggml tensor type {ggml_type}")
    _, bw, bb = GGML_TYPES[ggml_type]
    n = int(np.prod(ne, dtype=np.int64))
    if ne[0] % bw:
        raise GGUFError(f"ne[0]={ne[0]} is not a multiple of the block ({bw} weights)")
    return n // bw * bb


@dataclass
class TensorInfo:
    name: str
    ggml_type: int
    ne: Tuple[int, ...]  # ggml order: ne[0] fastest
    offset: int          # absolute file offset of the first byte
    nbytes: int

    @property
    def wtype(self) -> int:
        return GGML_TYPES[self.ggml_type][0]

    @property
    def rows(self) -> int:
        return int(np.prod(self.ne[1:], dtype=np.int64)) if len(self.ne) > 1 else 1


class GGUFFile:
    """A GGUF v3 file mapped read-only; tensor bytes are numpy views of the mapping."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:  # empty file
            self._f.close()
            raise GGUFError(f"{path}: not a GGUF file ({e})") from None
        self.metadata: Dict[str, object] = {}
        self.tensors: Dict[str, TensorInfo] = {}
        self._parse()

    # ---------------------------------------------------------------- parsing
    def _parse(self) -> None:
        buf, off = self._mm, 0
        size = len(buf)

        def take(fmt: str):
            nonlocal off
            n = struct.calcsize(fmt)
            if off + n > size:
                raise GGUFError(f"{self.path}: truncated header at byte {off}")
            v = struct.unpack_from(fmt, buf, off)
            off += n
            return v[0]

        def rstr() -> str:
            nonlocal off
            n = take("<Q")
            if off + n > size:
                raise GGUFError(f"{self.path}: truncated string at byte {off}")
            s = bytes(buf[off:off + n]).decode("utf-8")
            off += n
            return s

        def rval(vt: int):
            if vt in _FIXED:
                return take(_FIXED[vt])
            if vt == _STR:
                return rstr()
            if vt == _ARR:
                at, n = take("<I"), take("<Q")
                return [rval(at) for _ in range(n)]
            raise GGUFError(f"{self.path}: unknown metadata value type {vt}")

        if take("<I") != GGUF_MAGIC:
            raise GGUFError(f"{self.path}: bad magic (not a GGUF file)")
        version = take("<I")
        if version != GGUF_VERSION:
            raise GGUFError(f"{self.path}: GGUF version {version} (only version 3 is supported)")
        n_tensors, n_kv = take("<Q"), take("<Q")
        for _ in range(n_kv):
            key = rstr()
            self.metadata[key] = rval(take("<I"))
        infos = []
        for _ in range(n_tensors):
            name = rstr()
            nd = take("<I")
            ne = tuple(take("<Q") for _ in range(nd))
            infos.append((name, take("<I"), ne, take("<Q")))
        self.alignment = int(self.metadata.get("general.alignment", 32))
        self.data_start = off + (-off) % self.alignment
        for name, tt, ne, rel in infos:
            nb = tensor_nbytes(tt, ne)
            start = self.data_start + rel
            if start + nb > size:
                raise GGUFError(f"{self.path}: tensor {name} runs past the end of the file")
            self.tensors[name] = TensorInfo(name, tt, ne, start, nb)

    # ---------------------------------------------------------------- access
    def close(self) -> None:
        """Release the file. Views returned by raw() stay valid: the mapping is then unmapped when
        the last of them is gone."""
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # numpy views of the mapping are still alive
                pass
            self._f.close()
            self._mm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view [rows, row bytes] of the mapping."""
        if self._mm is None:
            raise GGUFError(f"{self.path}: file is closed")
        t = self.info(name)
        a = np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=t.offset)
        return a.reshape(t.rows, t.nbytes // t.rows)

    def info(self, name: str) -> TensorInfo:
        if name not in self.tensors:
            raise KeyError(f"{self.path}: no tensor {name!r}")
        return self.tensors[name]

    def to_device(self, name: str, device):
        """The tensor's bytes copied to a torch uint8 tensor [rows, row bytes] on `device`."""
        import torch
        return torch.from_numpy(np.array(self.raw(name))).to(device)

    def arch(self) -> Optional[str]:
        a = self.metadata.get("general.architecture")
        return a if isinstance(a, str) else None

    def arch_value(self, key: str, default=None):
        a = self.arch()
        return self.metadata.get(f"{a}.{key}", default) if a else default

    def moe_layers(self) -> List[int]:
        """Indices i of the blocks that hold routed experts (blk.i.ffn_gate_exps.weight)."""
        out = []
        for n in self.tensors:
            if n.startswith("blk.") and n.endswith(".ffn_gate_exps.weight"):
                out.append(int(n.split(".")[1]))
        return sorted(out)


# -------------------------------------------------------------------- writer
@dataclass
class TensorSpec:
    name: str
    ggml_type: int
    ne: Tuple[int, ...]
    data: bytes


def _wstr(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _wval(v) -> Tuple[int, bytes]:
    if isinstance(v, bool):
        return _BOOL, struct.pack("<?", v)
    if isinstance(v, int):
        return (_U32, struct.pack("<I", v)) if 0 <= v < 2 ** 32 else (_I64, struct.pack("<q", v))
    if isinstance(v, float):
        return _F32, struct.pack("<f", v)
    if isinstance(v, str):
        return _STR, _wstr(v)
    if isinstance(v, (list, tuple)):
        if not v:
            return _ARR, struct.pack("<I", _U32) + struct.pack("<Q", 0)
        items = [_wval(x) for x in v]
        t0 = items[0][0]
        if any(t != t0 for t, _ in items):
            raise GGUFError("metadata arrays must be homogeneous")
        return _ARR, struct.pack("<I", t0) + struct.pack("<Q", len(items)) + b"".join(b for _, b in items)
    raise GGUFError(f"unsupported metadata value {v!r}")


def write_gguf(path: str, tensors: Sequence[TensorSpec], metadata: Optional[Dict[str, object]] = None,
               alignment: int = 32) -> None:
    """Write a GGUF v3 file (tensor data aligned to `alignment`, in the order given)."""
    meta = dict(metadata or {})
    meta.setdefault("general.alignment", alignment)
    kv = b""
    for k, v in meta.items():
        t, b = _wval(v)
        kv += _wstr(k) + struct.pack("<I", t) + b
    info, blob = b"", bytearray()
    for t in tensors:
        nb = tensor_nbytes(t.ggml_type, t.ne)
        if len(t.data) != nb:
            raise GGUFError(f"{t.name}: {len(t.data)} bytes, expected {nb}")
        info += _wstr(t.name) + struct.pack("<I", len(t.ne)) + b"".join(struct.pack("<Q", d) for d in t.ne)
        info += struct.pack("<I", t.ggml_type) + struct.pack("<Q", len(blob))
        blob += t.data
        blob += b"\0" * ((-len(blob)) % alignment)
    head = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(meta)) + kv + info
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % alignment))
        f.write(bytes(blob))


# -------------------------------------------------------------------- matrices
@dataclass
class Matrix:
    """A 2-D GGUF weight on the device as the GEMV consumes it: N rows of K weights of `wtype`."""
    wtype: int
    N: int
    K: int
    rows: object  # torch uint8 [N, row bytes]


def load_matrix(gf: GGUFFile, name: str, device) -> Matrix:
    """A 2-D tensor (ne = [K, N]) for ops.gemm / ops.gemm_grouped: e.g. the attention projections
    blk.{i}.attn_{q_a,q_b,kv_a_mqa,kv_b,output}.weight, whatever their per-tensor type."""
    t = gf.info(name)
    if len(t.ne) != 2:
        raise GGUFError(f"{name}: expected a 2-D tensor, got ne = {list(t.ne)}")
    K, N = t.ne
    if t.wtype not in (F.Q4_K, F.Q6_K, F.Q8_0, F.F16):
        raise GGUFError(f"{name}: type {t.ggml_type} is not a GEMM weight type (Q4_K, Q6_K, Q8_0 or F16)")
    if K % 256:
        raise GGUFError(f"{name}: K = {K} is not a multiple of 256 (the fast GEMM streams 256-weight columns)")
    return Matrix(t.wtype, N, K, gf.to_device(name, device))


# -------------------------------------------------------------------- MoE layers
def moe_names(layer: int) -> Dict[str, str]:
    b = f"blk.{layer}."
    return {"router": b + "ffn_gate_inp.weight", "bias": b + "exp_probs_b.bias",
            "gate": b + "ffn_gate_exps.weight", "up": b + "ffn_up_exps.weight", "down": b + "ffn_down_exps.weight",
            "shared_gate": b + "ffn_gate_shexp.weight", "shared_up": b + "ffn_up_shexp.weight",
            "shared_down": b + "ffn_down_shexp.weight"}


def load_moe_layer(gf: GGUFFile, layer: int, device, topk: Optional[int] = None, scale: Optional[float] = None):
    """MoeLayerWeights of block `layer` on `device` (expert tensors copied as stored; an F32 router
    [E rows of H] is transposed once into the [H, E] layout of the fp32 router kernel)."""
    import torch

    from . import ops
    n = moe_names(layer)
    gi, ui, di = gf.info(n["gate"]), gf.info(n["up"]), gf.info(n["down"])
    if len(gi.ne) != 3 or gi.ne != ui.ne:
        raise GGUFError(f"layer {layer}: gate/up experts must be ne = [H, F, E] and equal")
    H, Fd, E = gi.ne
    if di.ne != (Fd, H, E):
        raise GGUFError(f"layer {layer}: down experts must be ne = [F, H, E] = [{Fd}, {H}, {E}], got {list(di.ne)}")
    if gi.ggml_type != ui.ggml_type:
        raise GGUFError(f"layer {layer}: gate and up must have one type")
    ri = gf.info(n["router"])
    if ri.ne != (H, E):
        raise GGUFError(f"layer {layer}: router must be ne = [H, E] = [{H}, {E}], got {list(ri.ne)}")
    if ri.ggml_type == GGML_F32:
        rw = torch.from_numpy(np.array(gf.raw(n["router"])).view(np.float32).reshape(E, H).T.copy()).to(device)
    else:
        rw = gf.to_device(n["router"], device)
    bias = None
    if n["bias"] in gf.tensors:
        bi = gf.info(n["bias"])
        if bi.ggml_type != GGML_F32 or bi.ne != (E,):
            raise GGUFError(f"layer {layer}: selection bias must be F32 [E]")
        bias = torch.from_numpy(np.array(gf.raw(n["bias"])).view(np.float32).reshape(E)).to(device)
    shared = {}
    if all(n[k] in gf.tensors for k in ("shared_gate", "shared_up", "shared_down")):
        sg, su, sd = gf.info(n["shared_gate"]), gf.info(n["shared_up"]), gf.info(n["shared_down"])
        if (sg.ne[:2] != (H, Fd) or su.ne[:2] != (H, Fd) or sd.ne[:2] != (Fd, H) or sg.ggml_type != gi.ggml_type
                or su.ggml_type != gi.ggml_type or sd.ggml_type != di.ggml_type):
            raise GGUFError(f"layer {layer}: shared expert shapes/types differ from the routed experts")
        shared = dict(shared_gate_w=gf.to_device(n["shared_gate"], device),
                      shared_up_w=gf.to_device(n["shared_up"], device),
                      shared_down_w=gf.to_device(n["shared_down"], device))
    k = topk if topk is not None else int(gf.arch_value("expert_used_count", 8))
    sc = scale if scale is not None else float(gf.arch_value("expert_weights_scale", 2.5))
    return ops.MoeLayerWeights(
        hidden=H, ffn=Fd, n_experts=E, topk=k, router_wtype=ri.wtype, router_w=rw, router_bias=bias,
        gate_w=gf.to_device(n["gate"], device), up_w=gf.to_device(n["up"], device),
        down_w=gf.to_device(n["down"], device), gate_wtype=gi.wtype, down_wtype=di.wtype, scale=sc, **shared)


def synthetic_moe_gguf(path: str, layers: int, H: int, Fd: int, E: int, topk: int = 8, seed: int = 0,
                       gate_type: int = GGML_Q4_K, down_type: int = GGML_Q6_K, shared: bool = True,
                       arch: str = "glm4moe") -> None:
    """A GGUF holding `layers` MoE blocks of seeded random weights with the benchmark distributions
    (router F32 ~N(0, 0.02), bias ~N(0, 0.01), expert blocks from formats.random_rows_np)."""
    rng = np.random.default_rng(seed)
    gt, dt = GGML_TYPES[gate_type][0], GGML_TYPES[down_type][0]
    specs: List[TensorSpec] = []
    for i in range(layers):
        n = moe_names(i)
        s = seed + 1000 * (i + 1)
        specs.append(TensorSpec(n["router"], GGML_F32, (H, E), rng.normal(0, 0.02, (E, H)).astype(np.float32).tobytes()))
        specs.append(TensorSpec(n["bias"], GGML_F32, (E,), rng.normal(0, 0.01, E).astype(np.float32).tobytes()))
        specs.append(TensorSpec(n["gate"], gate_type, (H, Fd, E), F.random_rows_np(gt, E * Fd, H, seed=s + 1).tobytes()))
        specs.append(TensorSpec(n["up"], gate_type, (H, Fd, E), F.random_rows_np(gt, E * Fd, H, seed=s + 2).tobytes()))
        specs.append(TensorSpec(n["down"], down_type, (Fd, H, E), F.random_rows_np(dt, E * H, Fd, seed=s + 3).tobytes()))
        if shared:
            specs.append(TensorSpec(n["shared_gate"], gate_type, (H, Fd), F.random_rows_np(gt, Fd, H, seed=s + 4).tobytes()))
            specs.append(TensorSpec(n["shared_up"], gate_type, (H, Fd), F.random_rows_np(gt, Fd, H, seed=s + 5).tobytes()))
            specs.append(TensorSpec(n["shared_down"], down_type, (Fd, H), F.random_rows_np(dt, H, Fd, seed=s + 6).tobytes()))
    write_gguf(path, specs, {"general.architecture": arch, f"{arch}.block_count": layers,
                             f"{arch}.expert_count": E, f"{arch}.expert_used_count": topk,
                             f"{arch}.expert_weights_scale": 2.5, "general.quantization_version": 2})


# -------------------------------------------------------------------- integrity manifest
GGML_TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K", GGML_Q6_K: "Q6_K"}


def tensor_manifest(gf: GGUFFile) -> Dict[str, object]:
    """Per-tensor integrity manifest of a GGUF: for every tensor its name, type name, ggml type id,
    shape (ne), absolute source offset, byte length and sha256 of its bytes. The per-tensor field
    names are those of the reference's provisioning manifest (tools/provision_image.py:295-340), so a
    manifest written by either side can be checked against a GGUF by verify_manifest; the
    reference's flash-image fields (image offsets, segments, image hash) belong to its FPGA boot
    image and are not produced here."""
    import hashlib

    out = []
    for name, t in sorted(gf.tensors.items(), key=lambda kv: kv[1].offset):
        out.append({"name": name, "type": GGML_TYPE_NAMES.get(t.ggml_type, str(t.ggml_type)),
                    "ggml_type": t.ggml_type, "shape": list(t.ne), "src_offset": t.offset, "length": t.nbytes,
                    "sha256": hashlib.sha256(bytes(gf.raw(name))).hexdigest()})
    import os

    return {"source_gguf": os.path.basename(gf.path), "tensor_count": len(out), "tensors": out}


def verify_manifest(gf: GGUFFile, manifest: Dict[str, object]) -> List[str]:
    """Check every tensor a manifest lists against the GGUF: present, same ggml type, shape and byte
    length, and the sha256 of its bytes equal to the manifest's (tools/provision_image.py:385-440 does
    the same for the reference's flash image). Returns the failures (empty when all match)."""
    import hashlib

    fails = []
    for t in manifest.get("tensors", []):
        name = t["name"]
        if name not in gf.tensors:
            fails.append(f"{name}: not present in the GGUF")
            continue
        info = gf.tensors[name]
        if "ggml_type" in t and int(t["ggml_type"]) != info.ggml_type:
            fails.append(f"{name}: ggml type {info.ggml_type} != manifest {t['ggml_type']}")
        if "shape" in t and [int(v) for v in t["shape"]] != list(info.ne):
            fails.append(f"{name}: shape {list(info.ne)} != manifest {t['shape']}")
        if "length" in t and int(t["length"]) != info.nbytes:
            fails.append(f"{name}: length {info.nbytes} != manifest {t['length']}")
            continue
        sha = hashlib.sha256(bytes(gf.raw(name))).hexdigest()
        if sha != t.get("sha256"):
            fails.append(f"{name}: sha256 {sha} != manifest {t.get('sha256')}")
    return fails
