"""B200-native (sm_100a) attention hot path for Qwen3-Embedding-0.6B-shaped layers.

Fused per-head Q/K RMSNorm + RoPE and causal / sparse GQA prefill attention
(16 q-heads, 8 kv-heads, head_dim 128) over ragged micro-batches, behind the
C ABI in include/qwa.h (libqwa.so). ``attention`` mirrors the reference's
QKNormRopeKernel / CausalAttentionKernel interface (src/webgpu/ops.ts).

The directory name is not a Python identifier; import it with
``importlib.import_module("qwen3-embedding-webgpu-prepacked_b200")``.
"""
from . import _lib, attention, engine, executor, ffn, matmul, model, norm, pooling, prepacked, sharding, workloads  # noqa: F401

__all__ = ["_lib", "attention", "engine", "executor", "ffn", "matmul", "model", "norm", "pooling", "prepacked", "sharding", "workloads"]
