"""Projection matmuls: Q4_0 tile32 weights on the tensor cores.

Mirrors ``QuantMatmulKernel`` for the prepacked layout
(src/webgpu/quant-matmul.ts:453-540): ``create_run_from_buffers(input,
weights, m, n, k, output)`` binds a run computing ``output[m, n] = sum_k
input[m, k] * W[n, k]`` where W is the Q4_0 "q4_0-tile32-compact" matrix in
``weights`` (src/prepacked/format.ts:65-99), and ``encode(stream, run)``
issues it. On B200 the matrix is dequantised once to an f16 copy (bit-exact
with the reference's dequantised values) and every run is a tcgen05 GEMM with
f32 accumulation (csrc/gemm.cu); the reference accumulates in f16.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .attention import Context, _need, _ptr, _stream

LAYOUT_TILE32 = "q4_0-tile32-compact"


def packed_bytes(n: int, k: int) -> int:
    """Size of a tile32-compact matrix: ceil(n/32) * (k/32) * 32 records of 20 B."""
    return (n + 31) // 32 * (k // 32) * 32 * 20


_tracked: dict = {}  # (device, data_ptr) of packed tensors with a forget finalizer


def _track_packed(ctx: Context, packed: torch.Tensor) -> None:
    """The context caches an f16 copy of a packed matrix keyed by its device
    address; drop it when the tensor dies, before the allocator can hand the
    same address to another buffer."""
    key = (ctx.device, packed.data_ptr())
    if key in _tracked:
        return
    lib, handle, ptr = ctx.lib, ctx.handle, packed.data_ptr()

    def forget():
        _tracked.pop(key, None)
        if ctx.handle:
            lib.qwa_q40_forget(handle, ctypes.c_void_p(ptr))

    _tracked[key] = weakref.finalize(packed, forget)


def _f16(t: torch.Tensor, name: str, numel: int) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16
          and t.is_contiguous() and t.numel() >= numel,
          f"{name} must be a contiguous CUDA float16 tensor of at least {numel} elements")


@dataclass
class QuantMatmulRun:
    """quant-matmul.ts:442-451 (input, weights, output, m, n, k)."""
    input: torch.Tensor
    weights: torch.Tensor
    output: torch.Tensor
    m: int
    n: int
    k: int


class QuantMatmulKernel:
    """quant-matmul.ts:453 -- prepacked tile32 Q4_0 only (GGUF Q4_K/Q6_K are
    outside the attention path)."""

    def __init__(self, device=None, layout: str = LAYOUT_TILE32):
        if layout != LAYOUT_TILE32:
            raise ValueError("only the q4_0-tile32-compact layout is supported")
        self.ctx = Context.for_device(device)
        self.layout = layout

    def create_run_from_buffers(self, input: torch.Tensor, weights: torch.Tensor, m: int, n: int,
                                k: int, output: Optional[torch.Tensor] = None) -> QuantMatmulRun:
        _f16(input, "input", m * k)
        _need(weights.is_cuda and weights.dtype == torch.uint8 and weights.is_contiguous()
              and weights.numel() >= packed_bytes(n, k),
              "weights must be a contiguous CUDA uint8 tile32-compact buffer")
        if output is None:
            output = torch.empty(m, n, dtype=torch.float16, device=input.device)
        _f16(output, "output", m * n)
        return QuantMatmulRun(input, weights, output, m, n, k)

    def encode(self, stream, run: QuantMatmulRun) -> None:
        _track_packed(self.ctx, run.weights)
        st = self.ctx.lib.qwa_q40_matmul(self.ctx.handle, _ptr(run.input), _ptr(run.weights),
                                         _ptr(run.output), run.m, run.n, run.k, _stream(stream))
        _lib.check(st, self.ctx.handle)

    def forget(self, weights: torch.Tensor) -> None:
        """Drop the f16 copy made from ``weights`` (after rewriting it in place)."""
        _lib.check(self.ctx.lib.qwa_q40_forget(self.ctx.handle, _ptr(weights)), self.ctx.handle)
        f = _tracked.pop((self.ctx.device, weights.data_ptr()), None)
        if f is not None:
            f.detach()


def q40_dequantize(packed: torch.Tensor, n: int, k: int, out: Optional[torch.Tensor] = None,
                   stream=None) -> torch.Tensor:
    """f16 W [n, k] from a tile32-compact buffer."""
    _need(packed.is_cuda and packed.dtype == torch.uint8 and packed.numel() >= packed_bytes(n, k),
          "packed must be a CUDA uint8 tile32-compact buffer")
    out = out if out is not None else torch.empty(n, k, dtype=torch.float16, device=packed.device)
    _f16(out, "out", n * k)
    ctx = Context.for_device(packed.device.index)
    _lib.check(ctx.lib.qwa_q40_dequantize(ctx.handle, _ptr(packed), n, k, _ptr(out),
                                          _stream(stream)), ctx.handle)
    return out


def q40_matmul(input: torch.Tensor, packed: torch.Tensor, n: int, k: int,
               out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """f16 [m, n] = input [m, k] @ W^T with W the Q4_0 tile32 matrix ``packed``
    (quant-matmul.ts:495-540): m <= 64 rows on n <= 2048 read the records
    directly; other shapes use the context's cached f16 copy."""
    kern = QuantMatmulKernel(input.device.index)
    run = kern.create_run_from_buffers(input, packed, input.shape[0], n, k, out)
    kern.encode(stream, run)
    return run.output


def matmul(input: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None,
           stream=None) -> torch.Tensor:
    """f16 [m, n] = input [m, k] @ weight [n, k]^T on the tensor cores."""
    m, k = input.shape
    n = weight.shape[0]
    _f16(input, "input", m * k)
    _f16(weight, "weight", n * k)
    out = out if out is not None else torch.empty(m, n, dtype=torch.float16, device=input.device)
    _f16(out, "out", m * n)
    ctx = Context.for_device(input.device.index)
    _lib.check(ctx.lib.qwa_matmul(ctx.handle, _ptr(input), _ptr(weight), _ptr(out), m, n, k,
                                  _stream(stream)), ctx.handle)
    return out


def interleave_gate_up(weight: torch.Tensor) -> torch.Tensor:
    """The gate_up weight [2w, k] (gate rows, then up rows) with its rows
    interleaved in 128-row blocks, the layout ``matmul_swiglu`` reads."""
    n, k = weight.shape
    _need(n % 256 == 0, "gate_up rows must be a multiple of 256")
    return weight.view(2, n // 256, 128, k).transpose(0, 1).reshape(n, k).contiguous()


def matmul_swiglu(input: torch.Tensor, weight_interleaved: torch.Tensor,
                  out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """f16 [m, n/2] = SwiGLU of input [m, k] @ gate_up^T, the SwiGLU applied in
    the GEMM's epilogue (bit for bit ``swiglu(matmul(...))``); the weight is
    ``interleave_gate_up(gate_up)``."""
    m, k = input.shape
    n = weight_interleaved.shape[0]
    _f16(input, "input", m * k)
    _f16(weight_interleaved, "weight", n * k)
    out = out if out is not None else torch.empty(m, n // 2, dtype=torch.float16,
                                                  device=input.device)
    _f16(out, "out", m * (n // 2))
    ctx = Context.for_device(input.device.index)
    _lib.check(ctx.lib.qwa_matmul_swiglu(ctx.handle, _ptr(input), _ptr(weight_interleaved),
                                         _ptr(out), m, n, k, _stream(stream)), ctx.handle)
    return out


def qkv_projection(input: torch.Tensor, weight: torch.Tensor, q_weight: torch.Tensor,
                   k_weight: torch.Tensor, cu_seqlens, eps: float = 1e-6, theta: float = 1e6,
                   q_out: Optional[torch.Tensor] = None, k_out: Optional[torch.Tensor] = None,
                   v_out: Optional[torch.Tensor] = None, rope_table: Optional[torch.Tensor] = None,
                   stream=None):
    """attn_qkv projection fused with the per-head Q/K RMSNorm + RoPE
    (src/webgpu/model.ts:93-94). ``weight`` is f16 [4096, k] or a uint8 Q4_0
    tile32-compact buffer; returns (q [T,16,128], k [T,8,128], v [T,1024])."""
    T, k = input.shape
    _need(T == int(cu_seqlens[-1]), "input rows must equal cu_seqlens[-1]")
    _f16(input, "input", T * k)
    dev = input.device
    q_out = q_out if q_out is not None else torch.empty(T, 16, 128, dtype=torch.float16, device=dev)
    k_out = k_out if k_out is not None else torch.empty(T, 8, 128, dtype=torch.float16, device=dev)
    v_out = v_out if v_out is not None else torch.empty(T, 1024, dtype=torch.float16, device=dev)
    _f16(q_out, "q_out", T * 2048)
    _f16(k_out, "k_out", T * 1024)
    _f16(v_out, "v_out", T * 1024)
    for t, name in ((q_weight, "q_weight"), (k_weight, "k_weight")):
        _need(t.is_cuda and t.dtype == torch.float32 and t.numel() == 128 and t.is_contiguous(),
              f"{name} must be a contiguous CUDA float32 tensor of 128 elements")
    ctx = Context.for_device(dev.index)
    cu = _lib.cu_array(cu_seqlens)
    if weight.dtype == torch.uint8:
        _need(weight.is_cuda and weight.numel() >= packed_bytes(4096, k),
              "packed weight must be a CUDA tile32-compact buffer of [4096, k]")
        fn = ctx.lib.qwa_q40_qkv_projection
        _track_packed(ctx, weight)
    else:
        _f16(weight, "weight", 4096 * k)
        fn = ctx.lib.qwa_qkv_projection
    st = fn(ctx.handle, _ptr(input), _ptr(weight), k, _ptr(q_weight), _ptr(k_weight),
            _ptr(q_out), _ptr(k_out), _ptr(v_out), cu, len(cu) - 1, eps, theta,
            _ptr(rope_table), _stream(stream))
    _lib.check(st, ctx.handle)
    return q_out, k_out, v_out
