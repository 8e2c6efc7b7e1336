"""The Q4_0 tile32 oracle against the reference's own known answers.

Restates the byte expectations of tests/prepacked-format.test.ts and the
Q4_0 decode expectations of tests/quantization.test.ts (reference repo), then
checks the tile32 dequantisation against the GGML block decoder.
"""
import numpy as np

from oracle import q40


def test_packer_golden_bytes():
    # two rows of one block each: scale 1.0 (0x3c00) with quants index & 15,
    # scale 2.0 (0x4000) with quants 15 - (index & 15)
    first = q40.q40_block(0x3C00, [i & 15 for i in range(32)])
    second = q40.q40_block(0x4000, [15 - (i & 15) for i in range(32)])
    packed, k, n = q40.pack_q40_tile32([(first, 1), (second, 1)])
    assert (k, n) == (32, 2)
    assert packed.nbytes == 32 * 20
    assert list(packed[0:8]) == [0x00, 0x3C, 0x00, 0x00, 0x00, 0x11, 0x22, 0x33]
    assert list(packed[20:28]) == [0x00, 0x40, 0x00, 0x00, 0xFF, 0xEE, 0xDD, 0xCC]
    assert not packed[40:].any()  # rows 2..31 of the tile are zero records


def test_q40_block_decode_known_answer():
    block = np.zeros(18, np.uint8)
    block[0:2] = [0x00, 0x3C]  # d = 1
    block[2:] = 0xF0           # low nibble 0 -> -8, high nibble 15 -> 7
    v = q40.dequant_q40_block(block)
    assert v[0] == -8 and v[15] == -8 and v[16] == 7 and v[31] == 7


def test_tile32_dequant_matches_block_decoder():
    rng = np.random.default_rng(1)
    n, k = 70, 128  # three tiles, the last one partial
    rows = q40.random_q40_rows(rng, n, k)
    packed, kk, nn = q40.pack_q40_tile32([(rows[:40], 40), (rows[40:], 30)])
    assert (kk, nn) == (k, n)
    w = q40.dequant_tile32(packed, n, k)
    ref = np.stack([np.concatenate([q40.dequant_q40_block(rows[r, 18 * b:18 * b + 18])
                                    for b in range(k // 32)]) for r in range(n)])
    # the f16 product equals the f32 product rounded to f16
    assert np.array_equal(w, ref.astype(np.float16))


def test_matmul_oracle_is_exact_product():
    rng = np.random.default_rng(2)
    a = rng.standard_normal((5, 64)).astype(np.float16)
    w = rng.standard_normal((7, 64)).astype(np.float16)
    got = q40.matmul(a, w)
    ref = np.array([[sum(float(a[i, t]) * float(w[j, t]) for t in range(64)) for j in range(7)]
                    for i in range(5)])
    assert np.allclose(got, ref, rtol=0, atol=1e-9)
