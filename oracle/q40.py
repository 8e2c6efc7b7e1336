"""CPU oracle for the Q4_0 tile32 projection -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's baseline legs use this
module, as the checker. Restates, from the reference's TypeScript:

* ``q40_block`` / ``dequant_q40_block``: GGML Q4_0 blocks of 18 bytes (f16
  scale d, 16 bytes of nibbles; value j = d * (low nibble j - 8), value j+16 =
  d * (high nibble j - 8)), src/gguf/quantization.ts:40-44;
* ``pack_q40_tile32``: packQ40Tile32, src/prepacked/format.ts:65-99 (rows cut
  into tiles of 32; record ((tile * kBlocks + kBlock) * 32 + row) * 20 holds
  the scale, two zero bytes, then the 16 nibble bytes);
* ``dequant_tile32``: q40PrepackedDequant, src/webgpu/quant-matmul.ts:98-107
  (f16(scale) * (f16(q) - 8) in f16 arithmetic);
* ``matmul``: output[m, n] = sum_k input[m, k] * W[n, k] in fp64 (the
  reference accumulates in f16, quant-matmul.ts:395-428; fp64 is the exact
  value the tensor-core f32 accumulation is checked against).

Parity is pinned by the reference's golden bytes and known answers
(tests/prepacked-format.test.ts, tests/quantization.test.ts), restated in
tests/test_q40_oracle.py.
"""
from __future__ import annotations

import numpy as np

TILE_ROWS = 32
BLOCK_VALUES = 32
BLOCK_BYTES = 18
RECORD_BYTES = 20


def q40_block(scale_bits: int, quants) -> np.ndarray:
    """One 18-byte GGML Q4_0 block from an f16 scale bit pattern and 32 quants."""
    q = np.asarray(quants, dtype=np.uint8)
    assert q.shape == (32,) and q.max() < 16
    b = np.zeros(BLOCK_BYTES, np.uint8)
    b[0], b[1] = scale_bits & 0xFF, scale_bits >> 8
    b[2:] = q[:16] | (q[16:] << 4)
    return b


def dequant_q40_block(block: np.ndarray) -> np.ndarray:
    """quantization.ts:40-44 (float32 result)."""
    d = np.frombuffer(bytes(block[:2]), dtype="<f2")[0].astype(np.float32)
    p = np.asarray(block[2:18], np.uint8)
    out = np.empty(32, np.float32)
    out[:16] = d * ((p & 15).astype(np.float32) - 8)
    out[16:] = d * ((p >> 4).astype(np.float32) - 8)
    return out


def random_q40_rows(rng: np.random.Generator, n: int, k: int, scale: float = 0.02) -> np.ndarray:
    """GGML Q4_0 bytes of an [n, k] matrix: n rows of k/32 blocks (18 bytes each),
    scales ~ |N(0, scale)| as f16, quants uniform in [0, 16)."""
    assert k % 32 == 0
    kb = k // 32
    scales = np.abs(rng.standard_normal((n, kb)) * scale).astype(np.float16)
    quants = rng.integers(0, 16, size=(n, kb, 32), dtype=np.uint8)
    blocks = np.zeros((n, kb, BLOCK_BYTES), np.uint8)
    blocks[:, :, 0:2] = scales.view(np.uint8).reshape(n, kb, 2)
    blocks[:, :, 2:] = quants[:, :, :16] | (quants[:, :, 16:] << 4)
    return blocks.reshape(n, kb * BLOCK_BYTES)


def pack_q40_tile32(parts) -> tuple[np.ndarray, int, int]:
    """packQ40Tile32 over parts [(rows_bytes [n_i, k/32*18], n_i)] stacked along n.
    Returns (packed uint8, k, n)."""
    rows = np.concatenate([np.asarray(p, np.uint8).reshape(n_i, -1) for p, n_i in parts])
    n = rows.shape[0]
    kb = rows.shape[1] // BLOCK_BYTES
    k = kb * BLOCK_VALUES
    tiles = (n + TILE_ROWS - 1) // TILE_ROWS
    out = np.zeros((tiles, kb, TILE_ROWS, RECORD_BYTES), np.uint8)
    src = rows.reshape(n, kb, BLOCK_BYTES)
    padded = np.zeros((tiles * TILE_ROWS, kb, BLOCK_BYTES), np.uint8)
    padded[:n] = src
    padded = padded.reshape(tiles, TILE_ROWS, kb, BLOCK_BYTES).transpose(0, 2, 1, 3)
    out[:, :, :, 0:2] = padded[:, :, :, 0:2]
    out[:, :, :, 4:20] = padded[:, :, :, 2:18]
    # rows past n stay zero records
    return out.reshape(-1), k, n


def dequant_tile32(packed: np.ndarray, n: int, k: int) -> np.ndarray:
    """quant-matmul.ts:98-107 -> f16 W [n, k]."""
    kb = k // BLOCK_VALUES
    tiles = (n + TILE_ROWS - 1) // TILE_ROWS
    rec = np.asarray(packed, np.uint8).reshape(tiles, kb, TILE_ROWS, RECORD_BYTES)
    scale = rec[:, :, :, 0:2].copy().view(np.float16)  # [tiles, kb, 32, 1]
    q = rec[:, :, :, 4:20]
    vals = np.empty((tiles, kb, TILE_ROWS, 32), np.float16)
    eight = np.float16(8)
    vals[..., :16] = scale * ((q & 15).astype(np.float16) - eight)
    vals[..., 16:] = scale * ((q >> 4).astype(np.float16) - eight)
    w = vals.transpose(0, 2, 1, 3).reshape(tiles * TILE_ROWS, k)
    return w[:n]


def matmul(inp: np.ndarray, w: np.ndarray) -> np.ndarray:
    """fp64 output[m, n] = sum_k inp[m, k] * w[n, k]."""
    return np.asarray(inp, np.float64) @ np.asarray(w, np.float64).T
