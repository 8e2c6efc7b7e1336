"""Residual add + RMSNorm of the residual stream.

Mirrors ``RmsNormKernel.createRun(x, residual, weight, normalized, rows,
width, epsilon, hasResidual)`` (src/webgpu/ops.ts:57-64): with a residual,
``x`` is updated in place to ``f16(x + residual)``; ``normalized`` receives
``f16(x / sqrt(mean(x^2) + eps) * weight)`` (rmsNormShader, ops.ts:21-55).
The launch is the CUDA kernel of csrc/rmsnorm.cu through the C ABI.
"""
from __future__ import annotations

from typing import Optional

import torch

from .attention import EPSILON, Context, EncodableRun, _need, _ptr, encode_run


def _f16(t: torch.Tensor, name: str, n: int) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16
          and t.is_contiguous() and t.numel() >= n,
          f"{name} must be a contiguous CUDA float16 tensor of at least rows*width elements")


class RmsNormKernel:
    """ops.ts:57-64 -- residual + RMSNorm."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                   normalized: torch.Tensor, rows: int, width: int, epsilon: float = EPSILON,
                   has_residual: bool = True) -> EncodableRun:
        _f16(x, "x", rows * width)
        _f16(normalized, "normalized", rows * width)
        if has_residual:
            _need(residual is not None, "has_residual needs a residual tensor")
            _f16(residual, "residual", rows * width)
        _need(weight.is_cuda and weight.dtype == torch.float32 and weight.is_contiguous()
              and weight.numel() >= width, "weight must be a contiguous CUDA float32 [width]")
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(x), _ptr(residual) if has_residual else None, _ptr(weight),
                _ptr(normalized), rows, width, epsilon, 1 if has_residual else 0)
        return EncodableRun(lambda s: lib.qwa_rms_norm(h, *args, s), self.ctx,
                            "residual + RMSNorm")


def rms_norm(x: torch.Tensor, weight: torch.Tensor, residual: Optional[torch.Tensor] = None,
             eps: float = EPSILON, out: Optional[torch.Tensor] = None,
             stream=None) -> torch.Tensor:
    """normalized f16 [rows, width]; with ``residual``, x += residual in place."""
    rows, width = x.shape
    out = out if out is not None else torch.empty_like(x)
    kern = RmsNormKernel(x.device.index)
    encode_run(stream, kern.create_run(x, residual, weight, out, rows, width, eps,
                                       residual is not None))
    return out
