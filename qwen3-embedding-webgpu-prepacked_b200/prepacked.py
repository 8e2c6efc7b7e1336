"""The ``.wgpack`` prepacked weight format (host side).

Follows src/prepacked/format.ts of the reference:

* ``pack_q40_tile32(name, parts)`` -- packQ40Tile32 (format.ts:65-99): GGML
  Q4_0 rows (18-byte blocks: f16 scale, 16 nibble bytes) of one or more parts
  stacked along n, regrouped into tiles of 32 rows; the record of (tile,
  k-block, row) sits at ((tile * kBlocks + kBlock) * 32 + row) * 20 and holds
  the scale bytes, two zero bytes and the 16 nibble bytes; rows past n in the
  last tile stay zero;
* ``build_prepacked_file`` / ``parse_prepacked_model`` -- format.ts:101-169:
  magic ``WGPACK02``, a little-endian u32 header length, the JSON header, and
  tensor data at 256-byte aligned offsets after the header.

Errors are raised with the reference's messages. ``random_q40_rows`` makes
seeded synthetic Q4_0 rows (no checkpoint is available).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

import numpy as np

MAGIC = b"WGPACK02"
PRELUDE_BYTES = 12
DATA_ALIGNMENT = 256
PREPACKED_LAYOUT = "q4_0-tile32-compact-v2"
TILE_ROWS = 32
BLOCK_VALUES = 32
BLOCK_BYTES = 20
Q40_BLOCK_BYTES = 18
STORAGE_COMPACT = "q4_0-tile32-compact"
STORAGE_RAW = "raw"
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 2, 12, 14  # src/gguf/types.ts:17-23


@dataclass
class Q40TensorPart:
    name: str
    k: int
    n: int
    bytes: np.ndarray  # uint8, n * (k / 32) * 18


@dataclass
class PackedTensorBytes:
    name: str
    dimensions: List[int]
    type: int
    storage: str
    bytes: np.ndarray


@dataclass
class PrepackedModel:
    header: dict
    tensors: Dict[str, dict] = field(default_factory=dict)  # header entry + "byteOffset"
    buffer: bytes = b""
    data_offset: int = 0

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return np.frombuffer(self.buffer, np.uint8, t["byteLength"], t["byteOffset"])


def _align(value: int, alignment: int) -> int:
    return -(-value // alignment) * alignment


def pack_q40_tile32(name: str, parts: Sequence[Q40TensorPart]) -> PackedTensorBytes:
    if not parts:
        raise ValueError(f"cannot pack {name} without tensor parts")
    k = parts[0].k
    if k % BLOCK_VALUES:
        raise ValueError(f"{name} K={k} is not divisible by 32")
    for p in parts:
        if p.k != k:
            raise ValueError(f"{name} has mismatched K dimensions")
        expected = p.n * (k // 32) * Q40_BLOCK_BYTES
        if np.asarray(p.bytes).nbytes != expected:
            raise ValueError(f"{p.name} has {np.asarray(p.bytes).nbytes} bytes; expected {expected}")
    n = sum(p.n for p in parts)
    kb = k // BLOCK_VALUES
    tiles = -(-n // TILE_ROWS)
    # all rows as [n_padded, kb, 18] blocks, then [tile, row, kb] -> [tile, kb, row]
    blocks = np.zeros((tiles * TILE_ROWS, kb, Q40_BLOCK_BYTES), np.uint8)
    row = 0
    for p in parts:
        blocks[row:row + p.n] = np.asarray(p.bytes, np.uint8).reshape(p.n, kb, Q40_BLOCK_BYTES)
        row += p.n
    by_tile = blocks.reshape(tiles, TILE_ROWS, kb, Q40_BLOCK_BYTES).swapaxes(1, 2)
    records = np.zeros((tiles, kb, TILE_ROWS, BLOCK_BYTES), np.uint8)
    records[..., 0:2] = by_tile[..., 0:2]    # f16 scale
    records[..., 4:20] = by_tile[..., 2:18]  # nibbles; bytes 2..3 stay zero
    return PackedTensorBytes(name, [k, n], GGML_Q4_0, STORAGE_COMPACT, records.reshape(-1))


def raw_tensor(name: str, dimensions: Sequence[int], type_: int,
               data: np.ndarray) -> PackedTensorBytes:
    return PackedTensorBytes(name, list(dimensions), type_, STORAGE_RAW,
                             np.frombuffer(np.ascontiguousarray(data).tobytes(), np.uint8))


def build_prepacked_file(source_sha256: str, source_bytes: int, metadata: dict,
                         tensors: Sequence[PackedTensorBytes]) -> bytes:
    entries, offset = [], 0
    for t in tensors:
        offset = _align(offset, DATA_ALIGNMENT)
        entries.append({"name": t.name, "dimensions": list(t.dimensions), "type": t.type,
                        "storage": t.storage, "offset": offset, "byteLength": int(t.bytes.nbytes)})
        offset += int(t.bytes.nbytes)
    header = {"version": 2, "sourceSha256": source_sha256, "sourceBytes": source_bytes,
              "layout": PREPACKED_LAYOUT, "tileRows": TILE_ROWS, "blockValues": BLOCK_VALUES,
              "blockBytes": BLOCK_BYTES, "metadata": metadata, "tensors": entries}
    hbytes = json.dumps(header, separators=(",", ":")).encode()
    data_offset = _align(PRELUDE_BYTES + len(hbytes), DATA_ALIGNMENT)
    out = bytearray(data_offset + offset)
    out[0:8] = MAGIC
    out[8:12] = struct.pack("<I", len(hbytes))
    out[PRELUDE_BYTES:PRELUDE_BYTES + len(hbytes)] = hbytes
    for t, e in zip(tensors, entries):
        start = data_offset + e["offset"]
        out[start:start + e["byteLength"]] = t.bytes.tobytes()
    return bytes(out)


def parse_prepacked_model(buffer: bytes) -> PrepackedModel:
    if len(buffer) < PRELUDE_BYTES:
        raise ValueError("prepacked model is shorter than its prelude")
    magic = bytes(buffer[0:8])
    if magic != MAGIC:
        raise ValueError(f"invalid prepacked model magic {json.dumps(magic.decode('latin-1'))}")
    (hlen,) = struct.unpack("<I", bytes(buffer[8:12]))
    if PRELUDE_BYTES + hlen > len(buffer):
        raise ValueError("prepacked model header extends past end of file")
    header = json.loads(bytes(buffer[PRELUDE_BYTES:PRELUDE_BYTES + hlen]).decode())
    if (header.get("version") != 2 or header.get("layout") != PREPACKED_LAYOUT
            or header.get("tileRows") != 32 or header.get("blockValues") != 32
            or header.get("blockBytes") != 20):
        raise ValueError(f"unsupported prepacked layout {header.get('layout')}")
    data_offset = _align(PRELUDE_BYTES + hlen, DATA_ALIGNMENT)
    model = PrepackedModel(header, {}, bytes(buffer), data_offset)
    for t in header["tensors"]:
        byte_offset = data_offset + t["offset"]
        if byte_offset + t["byteLength"] > len(buffer):
            raise ValueError(f"{t['name']} extends past end of prepacked file")
        if t["name"] in model.tensors:
            raise ValueError(f"duplicate prepacked tensor {t['name']}")
        if t["storage"] == STORAGE_COMPACT and (t["type"] != GGML_Q4_0 or len(t["dimensions"]) != 2):
            raise ValueError(f"{t['name']} has invalid compact Q4_0 metadata")
        if t["storage"] not in (STORAGE_COMPACT, STORAGE_RAW):
            raise ValueError(f"{t['name']} has unsupported storage {t['storage']}")
        model.tensors[t["name"]] = dict(t, byteOffset=byte_offset)
    return model


def random_q40_rows(rng: np.random.Generator, n: int, k: int,
                    scale: float = 0.02, centered: bool = False) -> np.ndarray:
    """Seeded synthetic GGML Q4_0 bytes of an [n, k] matrix (k/32 blocks per
    row): f16 scales |N(0, scale)|, nibbles uniform in [0, 16) -- or, with
    ``centered``, in [1, 16), so the values scale * (q - 8) have mean zero
    (a full model of such matrices keeps its residual stream unbiased)."""
    kb = k // 32
    out = np.empty((n, kb, Q40_BLOCK_BYTES), np.uint8)
    out[..., 0:2] = np.abs(rng.standard_normal((n, kb)) * scale).astype(np.float16) \
        .view(np.uint8).reshape(n, kb, 2)
    if centered:
        nib = rng.integers(1, 16, size=(n, kb, 32), dtype=np.uint8)
        out[..., 2:] = nib[..., :16] | (nib[..., 16:] << 4)
    else:
        out[..., 2:] = rng.integers(0, 256, size=(n, kb, 16), dtype=np.uint8)
    return out.reshape(n, kb * Q40_BLOCK_BYTES)


def random_q6k_rows(rng: np.random.Generator, vocab: int, width: int,
                    d_scale: float = 0.002) -> np.ndarray:
    """Seeded synthetic Q6_K bytes of a [vocab, width] matrix (210-byte blocks of
    256 values, src/gguf/quantization.ts:46-72): random 6-bit quants, int8
    scales in [-64, 64), d ~ |N(0, d_scale)| as f16."""
    nb = width // 256
    blk = rng.integers(0, 256, size=(vocab, nb, 210), dtype=np.uint8)
    blk[:, :, 192:208] = rng.integers(-64, 64, size=(vocab, nb, 16)).astype(np.int8) \
        .view(np.uint8)
    blk[:, :, 208:210] = np.abs(rng.standard_normal((vocab, nb)) * d_scale) \
        .astype(np.float16).view(np.uint8).reshape(vocab, nb, 2)
    return blk.reshape(-1)


def q40_part(name: str, rows: np.ndarray, k: int) -> Q40TensorPart:
    return Q40TensorPart(name, k, rows.shape[0], rows.reshape(-1))


def dimensions_kn(t: PackedTensorBytes) -> Tuple[int, int]:
    return t.dimensions[0], t.dimensions[1]


# ------------------------------------------------------------------ device load

ATTENTION_TENSORS = ("attn_norm", "attn_qkv", "attn_q_norm", "attn_k_norm", "attn_output")


class PrepackedWeights:
    """Tensors of a parsed .wgpack uploaded to one CUDA device, as the
    reference's Qwen3WebGPUModel does for a prepacked source
    (src/webgpu/model.ts:209-224): compact Q4_0 matrices stay packed (uint8;
    the matmul path dequantises each once), raw F32 / F16 tensors become
    float32 / float16 tensors, other raw types (the Q6_K token embedding) are
    kept as bytes. ``dims[name]`` is the reference's [k, n] / shape list."""

    def __init__(self, model: PrepackedModel, device=None):
        import torch
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        self.tensors: Dict[str, "torch.Tensor"] = {}
        self.dims: Dict[str, List[int]] = {}
        self.storage: Dict[str, str] = {}
        self.metadata = model.header.get("metadata", {})
        for name, t in model.tensors.items():
            raw = model.tensor_bytes(name)
            if t["storage"] == STORAGE_RAW and t["type"] == GGML_F32:
                host = np.frombuffer(raw.tobytes(), np.float32)
            elif t["storage"] == STORAGE_RAW and t["type"] == GGML_F16:
                host = np.frombuffer(raw.tobytes(), np.float16)
            else:
                host = np.array(raw, dtype=np.uint8)
            self.tensors[name] = torch.from_numpy(np.array(host)).to(self.device)
            self.dims[name] = list(t["dimensions"])
            self.storage[name] = t["storage"]

    @classmethod
    def from_file(cls, path: str, device=None) -> "PrepackedWeights":
        with open(path, "rb") as f:
            return cls(parse_prepacked_model(f.read()), device)

    def weight(self, name: str):
        """Model.weight (model.ts:250-254): the tensor, or an error naming it."""
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"missing tensor {name}")
        return t

    def layers(self) -> int:
        n = 0
        while f"blk.{n}.attn_qkv.weight" in self.tensors:
            n += 1
        return n

    def attention_layer(self, layer: int) -> Dict[str, "torch.Tensor"]:
        """The attention-half tensors of one block, by the reference's names
        (model.ts:89-100): attn_norm, attn_qkv (compact [1024, 4096]),
        attn_q_norm, attn_k_norm, attn_output (compact [2048, 1024])."""
        out = {}
        for key in ATTENTION_TENSORS:
            name = f"blk.{layer}.{key}.weight"
            out[key] = self.weight(name)
        for key, kn in (("attn_qkv", [1024, 4096]), ("attn_output", [2048, 1024])):
            name = f"blk.{layer}.{key}.weight"
            if self.storage[name] != STORAGE_COMPACT or self.dims[name] != kn:
                raise ValueError(f"{name} must be a compact Q4_0 matrix of dimensions {kn}")
        return out
