"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
``--impl reference`` legs import this module, and only as the checker.
The shipped library never calls it.

Two independent restatements of the math of the reference's WGSL shaders
(shihanqu/qwen3-embedding-webgpu-prepacked, src/webgpu/ops.ts):

* ``c_*``  -- the C/OpenMP restatement in oracle.c (fp64), used for large cases
  and as the timed CPU baseline;
* ``np_*`` -- a numpy twin (fp64), used to cross-check the C code.

Parity status: UNPINNED against the reference itself -- the reference has no
CPU implementation of this path and its WGSL runs only under a browser
WebGPU, which is unavailable on this box.  The f16 conversion
(src/math/f16.ts:4-25) and the halfToFloat known answers
(tests/quantization.test.ts:5-9) are pinned; the mask, RoPE and softmax
semantics are pinned by analytic known-answer tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

Q_HEADS, KV_HEADS, HEAD_DIM = 16, 8, 128
SCALE = 0.08838834764831845  # 1/sqrt(128), src/webgpu/ops.ts:224
PREFIX, WINDOW = 176, 432  # src/webgpu/ops.ts:206
SPARSE_MAX_SEQ = 8192  # src/webgpu/ops.ts:328
MODE_AUTO, MODE_FULL, MODE_SPARSE = 0, 1, 2

_lib = None


def build() -> str:
    """Compile oracle.c into liboracle.so (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        L.oracle_half_to_double.restype = ctypes.c_double
        L.oracle_half_to_double.argtypes = [ctypes.c_uint16]
        L.oracle_float_to_half.restype = ctypes.c_uint16
        L.oracle_float_to_half.argtypes = [ctypes.c_float]
        L.oracle_rope_table.argtypes = [ctypes.c_double, ctypes.c_int, P]
        L.oracle_qk_norm_rope.argtypes = [P, ctypes.c_int64, P, P, P, P, ctypes.c_int,
                                          ctypes.c_double, P, P]
        L.oracle_attention.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.oracle_attention_rows.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, P,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, P, ctypes.c_int64, P]
        L.oracle_keep.argtypes = [ctypes.c_int] * 5
        L.oracle_keep.restype = ctypes.c_int
        L.oracle_resolve_sparse.argtypes = [ctypes.c_int, ctypes.c_int]
        L.oracle_resolve_sparse.restype = ctypes.c_int
        L.oracle_kept_pairs.argtypes = [ctypes.c_int] * 4
        L.oracle_kept_pairs.restype = ctypes.c_int64
        L.oracle_last_token_pool.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P]
        L.oracle_float_to_half_rne.restype = ctypes.c_uint16
        L.oracle_float_to_half_rne.argtypes = [ctypes.c_float]
        L.oracle_rms_norm.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                      ctypes.c_int]
        L.oracle_attention_wgsl.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, P,
                                            ctypes.c_int, ctypes.c_int, P]
        L.oracle_threads.restype = ctypes.c_int
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _cu(cu_seqlens) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int32))


# ---------------------------------------------------------------- C oracle

def c_float_to_half(x: float) -> int:
    """floatToHalf of src/math/f16.ts:4-25 (bit pattern)."""
    return int(lib().oracle_float_to_half(ctypes.c_float(x)))


def c_half_to_float(bits: int) -> float:
    return float(lib().oracle_half_to_double(bits))


def c_rope_table(theta: float, positions: int) -> np.ndarray:
    """src/webgpu/model.ts:76-83 -> f32 [positions, 64, 2] (cos, sin)."""
    t = np.zeros((max(positions, 1), 64, 2), dtype=np.float32)
    lib().oracle_rope_table(theta, positions, _ptr(t))
    return t


def c_qk_norm_rope(qkv: np.ndarray, q_weight, k_weight, cu_seqlens, eps=1e-6, theta=1e6,
                   table: np.ndarray | None = None):
    """src/webgpu/ops.ts:104-150; returns fp64 q [T,16,128], k [T,8,128]."""
    qkv = np.ascontiguousarray(qkv)
    assert qkv.dtype == np.float16 and qkv.ndim == 2 and qkv.shape[1] >= 3072
    cu = _cu(cu_seqlens)
    batch = len(cu) - 1
    T = int(cu[-1])
    max_len = int(np.max(np.diff(cu))) if batch else 0
    if table is None:
        table = c_rope_table(theta, max_len)
    qw = np.ascontiguousarray(q_weight, dtype=np.float32)
    kw = np.ascontiguousarray(k_weight, dtype=np.float32)
    q = np.zeros((T, Q_HEADS, HEAD_DIM), dtype=np.float64)
    k = np.zeros((T, KV_HEADS, HEAD_DIM), dtype=np.float64)
    if T:
        lib().oracle_qk_norm_rope(_ptr(qkv), qkv.shape[1], _ptr(qw), _ptr(kw),
                                  _ptr(np.ascontiguousarray(table, dtype=np.float32)), _ptr(cu),
                                  batch, eps, _ptr(q), _ptr(k))
    return q, k


def c_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, v_stride: int, v_offset: int,
                cu_seqlens, mode=MODE_AUTO, prefix=PREFIX, window=WINDOW) -> np.ndarray:
    """src/webgpu/ops.ts:168-241 math; q/k/v f16; returns fp64 [T,16,128].

    ``v`` is a 2-D f16 array whose rows have ``v_stride`` elements; head g of
    token t is at v[t, v_offset + g*128 : ...] (ops.ts:215-216)."""
    q = np.ascontiguousarray(q, dtype=np.float16)
    k = np.ascontiguousarray(k, dtype=np.float16)
    v = np.ascontiguousarray(v, dtype=np.float16)
    assert v.shape[-1] == v_stride
    cu = _cu(cu_seqlens)
    T = int(cu[-1])
    out = np.zeros((T, Q_HEADS, HEAD_DIM), dtype=np.float64)
    if T:
        lib().oracle_attention(_ptr(q), _ptr(k), _ptr(v), v_stride, v_offset, _ptr(cu),
                               len(cu) - 1, mode, prefix, window, _ptr(out))
    return out


def c_attention_wgsl(q: np.ndarray, k: np.ndarray, v: np.ndarray, v_stride: int, v_offset: int,
                     cu_seqlens, fused: bool = True) -> np.ndarray:
    """The reference shader's own arithmetic (src/webgpu/ops.ts:168-241): f16
    dot products, f16 weights / denominators / accumulators, 16-key blocks,
    each request its own padded sequence (tiled path, S <= 8192). Returns the
    f16 values it would write, as fp64 [T,16,128]. ``fused``: f16 a*b+c
    rounded once (FMA contraction) or twice."""
    q = np.ascontiguousarray(q, dtype=np.float16)
    k = np.ascontiguousarray(k, dtype=np.float16)
    v = np.ascontiguousarray(v, dtype=np.float16)
    assert v.shape[-1] == v_stride
    cu = _cu(cu_seqlens)
    assert int(np.max(np.diff(cu), initial=0)) <= 8192, "tiled path only (S <= 8192)"
    T = int(cu[-1])
    out = np.zeros((T, Q_HEADS, HEAD_DIM), dtype=np.float64)
    if T:
        lib().oracle_attention_wgsl(_ptr(q), _ptr(k), _ptr(v), v_stride, v_offset, _ptr(cu),
                                    len(cu) - 1, 1 if fused else 0, _ptr(out))
    return out


def c_attention_rows(q, k, v, v_stride: int, v_offset: int, cu_seqlens, rows,
                     mode=MODE_AUTO, prefix=PREFIX, window=WINDOW) -> np.ndarray:
    """Oracle attention for selected output rows (row = token*16 + head)."""
    q = np.ascontiguousarray(q, dtype=np.float16)
    k = np.ascontiguousarray(k, dtype=np.float16)
    v = np.ascontiguousarray(v, dtype=np.float16)
    assert v.shape[-1] == v_stride
    cu = _cu(cu_seqlens)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.zeros((len(rows), HEAD_DIM), dtype=np.float64)
    if len(rows):
        lib().oracle_attention_rows(_ptr(q), _ptr(k), _ptr(v), v_stride, v_offset, _ptr(cu),
                                    len(cu) - 1, mode, prefix, window, _ptr(rows), len(rows),
                                    _ptr(out))
    return out


def c_last_token_pool(hidden: np.ndarray, cu_seqlens) -> np.ndarray:
    """src/webgpu/ops.ts:347-359; hidden f16 [T, width]; returns fp64 [B, width]."""
    hidden = np.ascontiguousarray(hidden)
    assert hidden.dtype == np.float16 and hidden.ndim == 2
    cu = _cu(cu_seqlens)
    batch = len(cu) - 1
    out = np.zeros((batch, hidden.shape[1]), dtype=np.float64)
    if batch:
        lib().oracle_last_token_pool(_ptr(hidden), hidden.shape[1], _ptr(cu), batch, _ptr(out))
    return out


def c_rms_norm(x: np.ndarray, residual, weight, eps=1e-6):
    """src/webgpu/ops.ts:21-57; x/residual f16 [rows, width], weight f32 [width].
    Returns (x updated by the residual, normalized), both f16."""
    x = np.array(x, dtype=np.float16, copy=True, order="C")
    rows, width = x.shape
    w = np.ascontiguousarray(weight, dtype=np.float32)
    normalized = np.zeros_like(x)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float16)
    if rows:
        lib().oracle_rms_norm(_ptr(x.view(np.uint16)), None if r is None else _ptr(r.view(np.uint16)),
                              _ptr(w), _ptr(normalized.view(np.uint16)), rows, width, eps,
                              0 if r is None else 1)
    return x, normalized


def c_kept_pairs(length: int, sparse: bool, prefix=PREFIX, window=WINDOW) -> int:
    return int(lib().oracle_kept_pairs(length, int(sparse), prefix, window))


def set_threads(n: int) -> None:
    """Number of OpenMP threads for later oracle calls."""
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_threads())


# ------------------------------------------------------------- numpy twin

def np_rope_table(theta: float, positions: int) -> np.ndarray:
    p = np.arange(positions, dtype=np.float64)[:, None]
    d = np.arange(64, dtype=np.float64)[None, :]
    ang = p * np.power(theta, -d / 64.0)
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def positions_of(cu_seqlens) -> np.ndarray:
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    T = int(cu[-1])
    t = np.arange(T)
    b = np.searchsorted(cu, t, side="right") - 1
    return t - cu[b]


def np_qk_norm_rope(qkv, q_weight, k_weight, cu_seqlens, eps=1e-6, theta=1e6):
    qkv = np.asarray(qkv, dtype=np.float16).astype(np.float64)
    T = qkv.shape[0]
    pos = positions_of(cu_seqlens)
    table = np_rope_table(theta, int(pos.max()) + 1 if T else 1).astype(np.float64)
    cos = table[pos, :, 0]
    sin = table[pos, :, 1]
    cos = np.concatenate([cos, cos], axis=1)[:, None, :]
    sin = np.concatenate([sin, sin], axis=1)[:, None, :]

    def one(x, w):
        inv = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) / 128.0 + eps)
        n = x * inv * np.asarray(w, dtype=np.float32).astype(np.float64)
        rot = np.concatenate([-n[..., 64:], n[..., :64]], axis=-1)
        return n * cos + rot * sin

    q = one(qkv[:, :2048].reshape(T, Q_HEADS, HEAD_DIM), q_weight)
    k = one(qkv[:, 2048:3072].reshape(T, KV_HEADS, HEAD_DIM), k_weight)
    return q, k


def resolve_sparse(mode: int, max_seqlen: int) -> bool:
    """Dispatch rule of src/webgpu/ops.ts:328 (AUTO) or a forced mode."""
    if mode == MODE_FULL:
        return False
    if mode == MODE_SPARSE:
        return True
    return max_seqlen <= SPARSE_MAX_SEQ


def keep_mask(length: int, sparse: bool, prefix=PREFIX, window=WINDOW) -> np.ndarray:
    """Kept (q,k) pairs, src/webgpu/ops.ts:220."""
    qi = np.arange(length)[:, None]
    ki = np.arange(length)[None, :]
    m = ki <= qi
    if sparse:
        m &= (ki < prefix) | (ki + window > qi)
    return m


def np_attention(q, k, v, v_stride, v_offset, cu_seqlens, mode=MODE_AUTO, prefix=PREFIX,
                 window=WINDOW):
    q = np.asarray(q, dtype=np.float16).astype(np.float64)
    k = np.asarray(k, dtype=np.float16).astype(np.float64)
    v = np.asarray(v, dtype=np.float16).astype(np.float64)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    T = int(cu[-1])
    lens = np.diff(cu)
    sparse = resolve_sparse(mode, int(lens.max()) if len(lens) else 0)
    out = np.zeros((T, Q_HEADS, HEAD_DIM))
    for b in range(len(lens)):
        s0, L = int(cu[b]), int(lens[b])
        if L == 0:
            continue
        m = keep_mask(L, sparse, prefix, window)
        for h in range(Q_HEADS):
            g = h // (Q_HEADS // KV_HEADS)
            qs = q[s0:s0 + L, h]
            ks = k[s0:s0 + L, g]
            vs = v[s0:s0 + L, v_offset + g * 128: v_offset + (g + 1) * 128]
            sc = qs @ ks.T * SCALE
            sc = np.where(m, sc, -np.inf)
            sc -= sc.max(axis=1, keepdims=True)
            p = np.exp(sc)
            out[s0:s0 + L, h] = (p @ vs) / p.sum(axis=1, keepdims=True)
    return out


def np_rms_norm(x, residual, weight, eps=1e-6):
    """numpy twin of c_rms_norm (float32 elementwise, numpy's RNE casts)."""
    v = np.asarray(x, dtype=np.float16).astype(np.float32)
    if residual is not None:
        v = v + np.asarray(residual, dtype=np.float16).astype(np.float32)
    xs = v.astype(np.float16)
    ss = np.sum(v.astype(np.float64) ** 2, axis=1, keepdims=True)
    inv = (1.0 / np.sqrt(ss / v.shape[1] + eps)).astype(np.float32)
    w = np.asarray(weight, dtype=np.float32)
    return xs, (xs.astype(np.float32) * inv * w).astype(np.float16)


def np_last_token_pool(hidden, cu_seqlens) -> np.ndarray:
    """numpy twin of c_last_token_pool (src/webgpu/ops.ts:347-359)."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    h = np.asarray(hidden).astype(np.float64)
    out = np.zeros((len(cu) - 1, h.shape[1]))
    for b in range(len(cu) - 1):
        if cu[b + 1] > cu[b]:
            x = h[cu[b + 1] - 1]
            out[b] = x / np.sqrt(np.sum(x * x))
    return out


def np_last_token_pool_padded(hidden, lengths, sequence: int) -> np.ndarray:
    """The reference's padded indexing, row b*sequence + lengths[b]-1
    (src/webgpu/ops.ts:351), as a twin for the padded entry point."""
    cu_rows = [b * sequence + int(n) for b, n in enumerate(lengths)]
    h = np.asarray(hidden).astype(np.float64)
    out = np.zeros((len(lengths), h.shape[1]))
    for b, n in enumerate(lengths):
        if n:
            x = h[cu_rows[b] - 1]
            out[b] = x / np.sqrt(np.sum(x * x))
    return out


def wgsl_block_skipped(key_base: int, query_tile_start: int, sequence: int) -> bool:
    """Literal transliteration of the tile-skip test, src/webgpu/ops.ts:206-209
    (16-key blocks, unsigned arithmetic)."""
    prefix_size = min(sequence, 176)
    local_window = min(sequence, 432)
    local_start = query_tile_start + 1 - local_window if query_tile_start + 1 > local_window else 0
    return key_base >= prefix_size and key_base + 15 < local_start


def wgsl_keep(q_pos: int, k_pos: int, sequence: int) -> bool:
    """Literal transliteration of the per-element test, src/webgpu/ops.ts:220."""
    prefix_size = min(sequence, 176)
    local_window = min(sequence, 432)
    return (q_pos < sequence and k_pos <= q_pos and k_pos < sequence
            and (k_pos < prefix_size or k_pos + local_window > q_pos))
