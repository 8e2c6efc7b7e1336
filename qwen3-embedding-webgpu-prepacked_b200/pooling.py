"""Last-token L2 pooling, the step after the last layer.

Mirrors ``LastTokenPoolKernel`` (src/webgpu/ops.ts:361-379): ``create_run(input,
lengths, output, batch, sequence, width=1024)`` pools row ``b*sequence +
lengths[b]-1`` of a padded f16 batch into an f32 ``[batch, width]`` embedding
scaled by ``1/sqrt(sum of squares)`` (poolShader, ops.ts:347-359).
``create_run_varlen`` does the same for a packed ragged batch (row
``cu_seqlens[b+1]-1``). Both launch the CUDA kernel of csrc/pool.cu through
the C ABI.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _lib
from .attention import Context, EncodableRun, _need, _ptr, encode_run

WIDTH = 1024  # hidden size of Qwen3-Embedding-0.6B, ops.ts:361 default


def _f16_rows(t: torch.Tensor, name: str) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16
          and t.is_contiguous(), f"{name} must be a contiguous CUDA float16 tensor")


def _f32_out(t: torch.Tensor, batch: int, width: int) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32
          and t.is_contiguous() and t.numel() >= batch * width,
          "output must be a contiguous CUDA float32 tensor of batch * width elements")


class LastTokenPoolKernel:
    """ops.ts:361-379 -- last-token L2 pool."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, input: torch.Tensor, lengths: torch.Tensor, output: torch.Tensor,
                   batch: int, sequence: int, width: int = WIDTH) -> EncodableRun:
        """Padded layout; ``lengths`` is a CUDA uint32/int32 tensor of ``batch``
        request lengths (the reference's lengths buffer)."""
        _f16_rows(input, "input")
        _need(lengths.is_cuda and lengths.dtype in (torch.int32, torch.uint32)
              and lengths.is_contiguous() and lengths.numel() >= batch,
              "lengths must be a contiguous CUDA int32/uint32 tensor of batch elements")
        _need(input.numel() >= batch * sequence * width, "input smaller than batch*sequence*width")
        _f32_out(output, batch, width)
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(input), _ptr(lengths), _ptr(output), batch, sequence, width)
        return EncodableRun(lambda s: lib.qwa_last_token_pool_padded(h, *args, s), self.ctx,
                            "last-token L2 pool")

    def create_run_varlen(self, input: torch.Tensor, cu_seqlens: Sequence[int],
                          output: torch.Tensor, width: int = WIDTH) -> EncodableRun:
        """Packed ragged batch: request b ends at row ``cu_seqlens[b+1]-1``."""
        _f16_rows(input, "input")
        cu = _lib.cu_array(cu_seqlens)
        batch = len(cu) - 1
        _need(input.numel() >= cu[batch] * width, "input smaller than tokens * width")
        _f32_out(output, batch, width)
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(input), width, _ptr(output), cu, batch)
        return EncodableRun(lambda s: lib.qwa_last_token_pool(h, *args, s), self.ctx,
                            "last-token L2 pool (varlen)")


def last_token_pool(hidden: torch.Tensor, cu_seqlens: Sequence[int],
                    out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """f32 [B, width] L2-normalised last-token rows of packed hidden [T, width]."""
    width = hidden.shape[-1]
    batch = len(cu_seqlens) - 1
    out = out if out is not None else torch.empty(batch, width, dtype=torch.float32,
                                                  device=hidden.device)
    kern = LastTokenPoolKernel(hidden.device.index)
    encode_run(stream, kern.create_run_varlen(hidden, cu_seqlens, out, width))
    return out
