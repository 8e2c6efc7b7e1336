"""The FFN's SwiGLU and the Q6_K token-embedding lookup.

Mirrors ``SwiGLUKernel.createRun(combined, output, rows, width)``
(src/webgpu/ops.ts:90-102) and ``EmbeddingLookupKernel.createRun(tokens,
weights, output, tokenCount, width=1024)`` (ops.ts:415-426); launches are the
CUDA kernels of csrc/ffn.cu through the C ABI.
"""
from __future__ import annotations

from typing import Optional

import torch

from .attention import Context, EncodableRun, _need, _ptr, encode_run


def _f16(t: torch.Tensor, name: str, n: int) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16
          and t.is_contiguous() and t.numel() >= n,
          f"{name} must be a contiguous CUDA float16 tensor of at least {n} elements")


def q6k_bytes(rows: int, width: int) -> int:
    """Size of a Q6_K matrix: rows * width/256 blocks of 210 bytes."""
    return rows * (width // 256) * 210


class SwiGLUKernel:
    """ops.ts:90-102 -- output[r, c] = silu(gate) * up of the gate_up output."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, combined: torch.Tensor, output: torch.Tensor, rows: int,
                   width: int) -> EncodableRun:
        _f16(combined, "combined", rows * 2 * width)
        _f16(output, "output", rows * width)
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(combined), _ptr(output), rows, width)
        return EncodableRun(lambda s: lib.qwa_swiglu(h, *args, s), self.ctx, "fused SwiGLU")


class EmbeddingLookupKernel:
    """ops.ts:415-426 -- rows of a Q6_K token-embedding matrix as f16."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, tokens: torch.Tensor, weights: torch.Tensor, output: torch.Tensor,
                   token_count: int, width: int = 1024, vocab: Optional[int] = None
                   ) -> EncodableRun:
        """``tokens``: CUDA int32/uint32 ids; ``weights``: the Q6_K bytes of a
        [vocab, width] matrix (``vocab`` defaults to what the buffer holds)."""
        _need(tokens.is_cuda and tokens.dtype in (torch.int32, torch.uint32)
              and tokens.is_contiguous() and tokens.numel() >= token_count,
              "tokens must be a contiguous CUDA int32/uint32 tensor of token_count ids")
        _need(weights.is_cuda and weights.dtype == torch.uint8 and weights.is_contiguous(),
              "weights must be a contiguous CUDA uint8 Q6_K buffer")
        row_bytes = q6k_bytes(1, width)
        vocab = weights.numel() // row_bytes if vocab is None else vocab
        _need(weights.numel() >= vocab * row_bytes, "weights smaller than vocab rows")
        _f16(output, "output", token_count * width)
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(tokens), _ptr(weights), vocab, _ptr(output), token_count, width)
        return EncodableRun(lambda s: lib.qwa_embedding_lookup_q6k(h, *args, s), self.ctx,
                            "Q6_K embedding lookup")


def swiglu(combined: torch.Tensor, width: int, out: Optional[torch.Tensor] = None,
           stream=None) -> torch.Tensor:
    rows = combined.shape[0]
    out = out if out is not None else torch.empty(rows, width, dtype=torch.float16,
                                                  device=combined.device)
    encode_run(stream, SwiGLUKernel(combined.device.index).create_run(combined, out, rows, width))
    return out


def embedding_lookup(ids: torch.Tensor, table: torch.Tensor, width: int = 1024,
                     vocab: Optional[int] = None, out: Optional[torch.Tensor] = None,
                     stream=None) -> torch.Tensor:
    n = ids.numel()
    out = out if out is not None else torch.empty(n, width, dtype=torch.float16, device=ids.device)
    encode_run(stream, EmbeddingLookupKernel(ids.device.index).create_run(ids, table, out, n,
                                                                           width, vocab))
    return out
