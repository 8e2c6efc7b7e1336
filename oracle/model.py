"""CPU oracle of the whole embedding forward -- TEST INFRASTRUCTURE ONLY.

Chains the oracle's restatements in the encode order of
Qwen3ExecutionPlan (src/webgpu/model.ts:90-136): Q6_K token embedding
(ops.ts:381-426), RMSNorm (ops.ts:21-64), per layer the attn_qkv projection
(Q4_0 tile32, quant-matmul.ts:98-107), the Q/K RMSNorm + RoPE prologue
(ops.ts:104-150), attention (ops.ts:168-241), attn_output, residual + RMSNorm,
ffn_gate_up, SwiGLU (ops.ts:74-88), ffn_down, residual + RMSNorm with the
next layer's attn_norm (output_norm after the last), then the last-token L2
pool (ops.ts:347-359).

Every product and sum is exact (fp64); values are rounded to f16 wherever
the device stores an f16 tensor (qkv, q, k, attention output, projection
outputs, the residual stream, normalized states, the SwiGLU output), so a
device run and this chain see the same rounding points and differ only by
the accumulation error inside each step.
"""
from __future__ import annotations

import numpy as np

from . import ffn, q40
from . import oracle as core

HIDDEN, INTERMEDIATE = 1024, 3072
COMPACT = {"attn_qkv": (4096, HIDDEN), "attn_output": (HIDDEN, 2048),
           "ffn_gate_up": (2 * INTERMEDIATE, HIDDEN), "ffn_down": (HIDDEN, INTERMEDIATE)}


def _proj(x16: np.ndarray, packed: np.ndarray, n: int, k: int) -> np.ndarray:
    w = q40.dequant_tile32(packed, n, k)
    return q40.matmul(x16, w).astype(np.float16)


def forward(model, ids, cu_seqlens, layers: int, trace: list | None = None) -> np.ndarray:
    """model: a parsed .wgpack (``prepacked.parse_prepacked_model``). Returns the
    final normalized f16 state [T, 1024]; ``trace`` receives the residual
    stream after every layer."""
    def raw(name, dtype):
        return np.frombuffer(model.tensor_bytes(name).tobytes(), dtype)

    vocab = model.tensors["token_embd.weight"]["dimensions"][1]
    x = ffn.embedding_lookup_f16(ids, np.array(model.tensor_bytes("token_embd.weight")), vocab,
                                 HIDDEN)
    x, normalized = core.c_rms_norm(x, None, raw("blk.0.attn_norm.weight", np.float32))
    cu = list(cu_seqlens)
    for l in range(layers):
        b = f"blk.{l}"
        mats = {name: np.array(model.tensor_bytes(f"{b}.{name}.weight")) for name in COMPACT}
        qkv = _proj(normalized, mats["attn_qkv"], *COMPACT["attn_qkv"])
        q, k = core.c_qk_norm_rope(qkv, raw(f"{b}.attn_q_norm.weight", np.float32),
                                   raw(f"{b}.attn_k_norm.weight", np.float32), cu)
        o = core.c_attention(q.astype(np.float16), k.astype(np.float16), qkv, 4096, 3072, cu)
        delta = _proj(o.astype(np.float16).reshape(-1, 2048), mats["attn_output"],
                      *COMPACT["attn_output"])
        x, normalized = core.c_rms_norm(x, delta, raw(f"{b}.ffn_norm.weight", np.float32))
        gate_up = _proj(normalized, mats["ffn_gate_up"], *COMPACT["ffn_gate_up"])
        hidden = ffn.swiglu(gate_up, INTERMEDIATE).astype(np.float16)
        delta = _proj(hidden, mats["ffn_down"], *COMPACT["ffn_down"])
        nxt = f"blk.{l + 1}.attn_norm.weight" if l + 1 < layers else "output_norm.weight"
        x, normalized = core.c_rms_norm(x, delta, raw(nxt, np.float32))
        if trace is not None:
            trace.append(x.copy())
    return normalized


def embed(model, ids, cu_seqlens, layers: int, trace: list | None = None) -> np.ndarray:
    """fp64 [batch, 1024] last-token embeddings."""
    return core.c_last_token_pool(forward(model, ids, cu_seqlens, layers, trace), cu_seqlens)
