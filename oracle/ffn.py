"""CPU oracle for the token-embedding lookup and the FFN's SwiGLU -- TEST
INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's baseline legs use it as
the checker; the product never imports it).

Restates, from the reference's TypeScript:

* ``dequant_q6k_block``: dequantizeQ6KBlock, src/gguf/quantization.ts:46-72
  (210-byte block: ql[128], qh[64], int8 scales[16], f16 d; 256 values
  d * scale * (q - 32), computed exactly in fp64);
* ``embedding_lookup_f16``: what embeddingShader (src/webgpu/ops.ts:381-413)
  writes: f16((d * scale) * q) with the two products in f32;
* ``swiglu``: swigluShader (ops.ts:74-88) math, g / (1 + exp(-g)) * u, in
  fp64 (the kernel's f32 result is checked against it within an f16 ulp).

Pinned by the reference's Q6_K known answer (tests/quantization.test.ts:
35-42), restated in tests/test_ffn_oracle.py.
"""
from __future__ import annotations

import numpy as np

Q6K_BLOCK_BYTES, Q6K_BLOCK_VALUES = 210, 256


def dequant_q6k_block(block) -> np.ndarray:
    """quantization.ts:46-72: fp64 [256]."""
    b = np.asarray(block, np.uint8)
    ql, qh = b[:128].astype(np.int64), b[128:192].astype(np.int64)
    scales = b[192:208].view(np.int8).astype(np.float64)
    d = float(b[208:210].view("<f2")[0])
    out = np.empty(256, np.float64)
    for half in range(2):
        lo, hi, so = half * 64, half * 32, half * 8
        for lane in range(32):
            pair = lane >> 4
            high = qh[hi + lane]
            a, bb = ql[lo + lane], ql[lo + lane + 32]
            q1 = (a & 15) | ((high & 3) << 4)
            q2 = (bb & 15) | (((high >> 2) & 3) << 4)
            q3 = (a >> 4) | (((high >> 4) & 3) << 4)
            q4 = (bb >> 4) | (((high >> 6) & 3) << 4)
            base = half * 128 + lane
            out[base] = d * scales[so + pair] * (q1 - 32)
            out[base + 32] = d * scales[so + pair + 2] * (q2 - 32)
            out[base + 64] = d * scales[so + pair + 4] * (q3 - 32)
            out[base + 96] = d * scales[so + pair + 6] * (q4 - 32)
    return out


def _fields(table: np.ndarray, vocab: int, width: int):
    """Vectorised block fields of a [vocab, width] Q6_K matrix."""
    nb = width // Q6K_BLOCK_VALUES
    blk = np.asarray(table, np.uint8).reshape(vocab, nb, Q6K_BLOCK_BYTES)
    i = np.arange(256)
    half, pos = i // 128, i % 128
    quad, lane = pos // 32, pos % 32
    low_b = blk[:, :, half * 64 + lane + (quad & 1) * 32].astype(np.int64)
    low = np.where(quad >= 2, low_b >> 4, low_b & 15)
    high = (blk[:, :, 128 + half * 32 + lane].astype(np.int64) >> (2 * quad)) & 3
    q = (low | (high << 4)) - 32
    scale = blk[:, :, 192 + half * 8 + lane // 16 + quad * 2].view(np.int8).astype(np.int64)
    d = blk[:, :, 208:210].copy().view("<f2")[..., 0]
    return d, scale, q


def dequant_q6k(table: np.ndarray, vocab: int, width: int) -> np.ndarray:
    """fp64 [vocab, width], exactly d * scale * (q - 32) per value."""
    d, scale, q = _fields(table, vocab, width)
    return (d.astype(np.float64)[..., None] * scale * q).reshape(vocab, width)


def embedding_lookup_f16(ids, table: np.ndarray, vocab: int, width: int) -> np.ndarray:
    """f16 [tokens, width] as embeddingShader writes it; ids >= vocab give 0."""
    d, scale, q = _fields(table, vocab, width)
    vals = ((d.astype(np.float32)[..., None] * scale.astype(np.float32)) *
            q.astype(np.float32)).astype(np.float16).reshape(vocab, width)
    ids = np.asarray(ids, np.int64)
    out = np.zeros((len(ids), width), np.float16)
    ok = ids < vocab
    out[ok] = vals[ids[ok]]
    return out


def swiglu(combined: np.ndarray, width: int) -> np.ndarray:
    """fp64 [rows, width]: silu(gate) * up from f16 combined [rows, 2*width]."""
    c = np.asarray(combined, np.float64)
    g, u = c[:, :width], c[:, width:2 * width]
    return g / (1.0 + np.exp(-g)) * u
