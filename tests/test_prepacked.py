"""The .wgpack format on the host (no GPU).

Restates tests/prepacked-format.test.ts of the reference through the
package's packer / file builder / parser, and checks the packer against the
oracle's independent restatement on random rows.
"""
import importlib

import numpy as np
import pytest

from oracle import q40

pp = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.prepacked")


def test_builds_self_contained_file_with_compact_and_raw_tensors():
    first = q40.q40_block(0x3C00, [i & 15 for i in range(32)])
    second = q40.q40_block(0x4000, [15 - (i & 15) for i in range(32)])
    packed = pp.pack_q40_tile32("fused", [pp.Q40TensorPart("first", 32, 1, first),
                                          pp.Q40TensorPart("second", 32, 1, second)])
    assert packed.dimensions == [32, 2]
    assert packed.bytes.nbytes == 32 * 20
    assert list(packed.bytes[0:8]) == [0x00, 0x3C, 0x00, 0x00, 0x00, 0x11, 0x22, 0x33]
    assert list(packed.bytes[20:28]) == [0x00, 0x40, 0x00, 0x00, 0xFF, 0xEE, 0xDD, 0xCC]

    raw = pp.raw_tensor("norm", [1], pp.GGML_F32, np.array([1, 2, 3, 4], np.uint8))
    data = pp.build_prepacked_file("abc123", 42, {"general.name": "test"}, [raw, packed])
    parsed = pp.parse_prepacked_model(data)
    assert parsed.header["sourceSha256"] == "abc123"
    assert parsed.header["sourceBytes"] == 42
    assert parsed.header["metadata"]["general.name"] == "test"
    norm = parsed.tensors["norm"]
    assert (norm["dimensions"], norm["type"], norm["storage"], norm["byteLength"]) == \
        ([1], pp.GGML_F32, "raw", 4)
    fused = parsed.tensors["fused"]
    assert (fused["dimensions"], fused["type"], fused["storage"], fused["byteLength"]) == \
        ([32, 2], pp.GGML_Q4_0, "q4_0-tile32-compact", 640)
    assert np.array_equal(parsed.tensor_bytes("fused"), packed.bytes)
    assert parsed.tensors["fused"]["byteOffset"] % 256 == 0


def test_packer_matches_oracle_on_random_parts():
    rng = np.random.default_rng(5)
    a, b = pp.random_q40_rows(rng, 45, 96), pp.random_q40_rows(rng, 30, 96)
    got = pp.pack_q40_tile32("x", [pp.q40_part("a", a, 96), pp.q40_part("b", b, 96)])
    ref, k, n = q40.pack_q40_tile32([(a, 45), (b, 30)])
    assert (k, n) == (96, 75) and got.dimensions == [96, 75]
    assert np.array_equal(got.bytes, ref)


def test_packer_and_parser_errors():
    with pytest.raises(ValueError, match="without tensor parts"):
        pp.pack_q40_tile32("x", [])
    with pytest.raises(ValueError, match="not divisible by 32"):
        pp.pack_q40_tile32("x", [pp.Q40TensorPart("p", 40, 1, np.zeros(18, np.uint8))])
    with pytest.raises(ValueError, match="mismatched K"):
        pp.pack_q40_tile32("x", [pp.Q40TensorPart("p", 32, 1, np.zeros(18, np.uint8)),
                                 pp.Q40TensorPart("q", 64, 1, np.zeros(36, np.uint8))])
    with pytest.raises(ValueError, match="expected 18"):
        pp.pack_q40_tile32("x", [pp.Q40TensorPart("p", 32, 1, np.zeros(17, np.uint8))])
    with pytest.raises(ValueError, match="shorter than its prelude"):
        pp.parse_prepacked_model(b"WGPACK")
    with pytest.raises(ValueError, match="invalid prepacked model magic"):
        pp.parse_prepacked_model(b"NOTAPACK" + bytes(8))
    good = pp.build_prepacked_file("s", 1, {}, [])
    bad = bytearray(good)
    bad[8:12] = (10 ** 6).to_bytes(4, "little")
    with pytest.raises(ValueError, match="extends past end of file"):
        pp.parse_prepacked_model(bytes(bad))
    t = pp.raw_tensor("t", [4], pp.GGML_F32, np.zeros(4, np.float32))
    data = pp.build_prepacked_file("s", 1, {}, [t, t])
    with pytest.raises(ValueError, match="duplicate prepacked tensor t"):
        pp.parse_prepacked_model(data)
