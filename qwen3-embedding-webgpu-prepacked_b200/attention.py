"""Host-side mirror of the reference's attention dispatch interface.

The reference (src/webgpu/ops.ts) exposes

* ``QKNormRopeKernel.createRun(input, qWeight, kWeight, qOutput, kOutput,
  tokens, sequence, epsilon, ropeTable, inputStride=3072) -> EncodableRun``
  (ops.ts:152-166),
* ``CausalAttentionKernel.createRun(q, k, v, output, batch, sequence,
  qHeads=16, kvHeads=8, valueStride=1024, valueOffset=0) -> AttentionRun``
  and ``encode(pass, run)`` (ops.ts:320-345),
* ``encodeRun(pass, run)`` (ops.ts:15-19),

and ``Qwen3ExecutionPlan`` calls them once per layer (model.ts:94-95) and
encodes them into one compute pass (model.ts:123). This module keeps those
names, argument meanings and error behaviour (invalid shapes raise, like the
reference's ``throw new Error``); a "pass" is a CUDA stream and a run is a
bound call into libqwa.so through its C ABI. Buffers are torch CUDA tensors
(caller-owned device memory). Varlen (cu_seqlens) variants are added next to
the padded ones.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import torch

from . import _lib

Q_HEADS, KV_HEADS, HEAD_DIM = 16, 8, 128
EPSILON, ROPE_THETA = 1e-6, 1e6  # src/webgpu/model.ts:22-23
PREFIX, WINDOW = 176, 432  # src/webgpu/ops.ts:206
MODE_AUTO, MODE_FULL, MODE_SPARSE = _lib.MODE_AUTO, _lib.MODE_FULL, _lib.MODE_SPARSE


class Context:
    """One qwa_ctx per CUDA device (the reference's GPUDevice handle)."""

    _by_device: dict = {}
    _lock = threading.Lock()

    def __init__(self, device: int):
        self.device = device
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        st = self.lib.qwa_create(device, ctypes.byref(h))
        _lib.check(st)
        self.handle = h

    @classmethod
    def for_device(cls, device=None) -> "Context":
        if device is None:
            device = torch.cuda.current_device()
        device = torch.device("cuda", device).index if not isinstance(device, int) else device
        with cls._lock:
            ctx = cls._by_device.get(device)
            if ctx is None:
                ctx = cls._by_device[device] = Context(device)
            return ctx

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Synchronise and raise if a kernel recorded a device-side timeout."""
        s = stream.cuda_stream if stream is not None else torch.cuda.current_stream(
            self.device).cuda_stream
        _lib.check(self.lib.qwa_check(self.handle, s), self.handle)

    def close(self) -> None:
        if self.handle:
            self.lib.qwa_destroy(self.handle)
            self.handle = None


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _f16_cuda(t: torch.Tensor, name: str) -> None:
    _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16,
          f"{name} must be a CUDA float16 tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def _f32_weight(t: torch.Tensor, name: str) -> None:
    _need(t.is_cuda and t.dtype == torch.float32 and t.numel() == HEAD_DIM and t.is_contiguous(),
          f"{name} must be a contiguous CUDA float32 tensor of 128 elements")


@dataclass
class EncodableRun:
    """A bound launch; ``encode_run(stream, run)`` issues it (ops.ts:9-19)."""
    launch: Callable[[int], int]
    ctx: Context
    label: str = ""


@dataclass
class AttentionRun:
    """ops.ts:318 -- commands plus buffers the run owns (none here: the
    context owns plans and tables)."""
    commands: List[EncodableRun]
    owned_buffers: List[torch.Tensor] = field(default_factory=list)


def encode_run(stream, run: EncodableRun) -> None:
    """encodeRun (ops.ts:15-19): issue the run on ``stream`` (None = current)."""
    _lib.check(run.launch(_stream(stream)), run.ctx.handle)


class QKNormRopeKernel:
    """ops.ts:152-166 -- fused per-head RMSNorm + RoPE."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, input: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                   q_output: torch.Tensor, k_output: torch.Tensor, tokens: int, sequence: int,
                   epsilon: float = EPSILON, rope_table: Optional[torch.Tensor] = None,
                   input_stride: int = 3072, theta: float = ROPE_THETA) -> EncodableRun:
        """Padded layout: ``tokens`` rows, position = row % sequence (ops.ts:146)."""
        _f16_cuda(input, "input")
        _f16_cuda(q_output, "q_output")
        _f16_cuda(k_output, "k_output")
        _f32_weight(q_weight, "q_weight")
        _f32_weight(k_weight, "k_weight")
        _need(input.numel() >= tokens * input_stride, "input smaller than tokens * input_stride")
        _need(q_output.numel() >= tokens * Q_HEADS * HEAD_DIM, "q_output too small")
        _need(k_output.numel() >= tokens * KV_HEADS * HEAD_DIM, "k_output too small")
        if rope_table is not None:
            _need(rope_table.is_cuda and rope_table.dtype == torch.float32
                  and rope_table.numel() >= min(sequence, tokens) * 128,
                  "rope_table must be CUDA float32 [sequence, 64, 2]")
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(input), input_stride, _ptr(q_weight), _ptr(k_weight), _ptr(q_output),
                _ptr(k_output), tokens, sequence, epsilon, theta, _ptr(rope_table))
        return EncodableRun(lambda s: lib.qwa_qk_norm_rope_padded(h, *args, s), self.ctx,
                            "QK norm + RoPE")

    def create_run_varlen(self, input: torch.Tensor, q_weight: torch.Tensor,
                          k_weight: torch.Tensor, q_output: torch.Tensor, k_output: torch.Tensor,
                          cu_seqlens: Sequence[int], epsilon: float = EPSILON,
                          input_stride: int = 3072, theta: float = ROPE_THETA,
                          rope_table: Optional[torch.Tensor] = None) -> EncodableRun:
        """Packed ragged batch: position = index inside the request."""
        _f16_cuda(input, "input")
        _f16_cuda(q_output, "q_output")
        _f16_cuda(k_output, "k_output")
        _f32_weight(q_weight, "q_weight")
        _f32_weight(k_weight, "k_weight")
        cu = _lib.cu_array(cu_seqlens)
        total = cu[len(cu) - 1]
        _need(input.numel() >= total * input_stride, "input smaller than tokens * input_stride")
        _need(q_output.numel() >= total * Q_HEADS * HEAD_DIM, "q_output too small")
        _need(k_output.numel() >= total * KV_HEADS * HEAD_DIM, "k_output too small")
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(input), input_stride, _ptr(q_weight), _ptr(k_weight), _ptr(q_output),
                _ptr(k_output), cu, len(cu) - 1, epsilon, theta, _ptr(rope_table))
        return EncodableRun(lambda s: lib.qwa_qk_norm_rope(h, *args, s), self.ctx,
                            "QK norm + RoPE (varlen)")


class CausalAttentionKernel:
    """ops.ts:320-345 -- causal GQA prefill (sparse prefix+window rule as AUTO)."""

    def __init__(self, device=None):
        self.ctx = Context.for_device(device)

    def create_run(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   output: torch.Tensor, batch: int, sequence: int, q_heads: int = Q_HEADS,
                   kv_heads: int = KV_HEADS, value_stride: int = 1024,
                   value_offset: int = 0) -> AttentionRun:
        for t, n in ((q, "q"), (k, "k"), (v, "v"), (output, "output")):
            _f16_cuda(t, n)
        tokens = batch * sequence
        _need(q.numel() >= tokens * q_heads * HEAD_DIM, "q too small")
        _need(k.numel() >= tokens * kv_heads * HEAD_DIM, "k too small")
        _need(v.numel() >= (tokens - 1) * value_stride + value_offset + kv_heads * HEAD_DIM,
              "v too small for value_stride/value_offset")
        _need(output.numel() >= tokens * q_heads * HEAD_DIM, "output too small")
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(q), _ptr(k), _ptr(v), _ptr(output), batch, sequence, q_heads, kv_heads,
                value_stride, value_offset)
        run = EncodableRun(lambda s: lib.qwa_attention_padded(h, *args, s), self.ctx,
                           "tiled flash attention")
        return AttentionRun([run])

    def create_run_varlen(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          output: torch.Tensor, cu_seqlens: Sequence[int],
                          value_stride: int = 1024, value_offset: int = 0,
                          mode: int = MODE_AUTO, prefix: int = PREFIX,
                          window: int = WINDOW) -> AttentionRun:
        for t, n in ((q, "q"), (k, "k"), (v, "v"), (output, "output")):
            _f16_cuda(t, n)
        cu = _lib.cu_array(cu_seqlens)
        total = cu[len(cu) - 1]
        _need(q.numel() >= total * Q_HEADS * HEAD_DIM, "q too small")
        _need(k.numel() >= total * KV_HEADS * HEAD_DIM, "k too small")
        _need(total == 0 or v.numel() >= (total - 1) * value_stride + value_offset + 1024,
              "v too small for value_stride/value_offset")
        _need(output.numel() >= total * Q_HEADS * HEAD_DIM, "output too small")
        lib, h = self.ctx.lib, self.ctx.handle
        args = (_ptr(q), _ptr(k), _ptr(v), value_stride, value_offset, _ptr(output), cu,
                len(cu) - 1, mode, prefix, window)
        run = EncodableRun(lambda s: lib.qwa_attention(h, *args, s), self.ctx,
                           "tiled flash attention (varlen)")
        return AttentionRun([run])

    def encode(self, stream, run: AttentionRun) -> None:
        for command in run.commands:
            encode_run(stream, command)


# ----------------------------------------------------------- functional API

def qk_norm_rope(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 cu_seqlens: Sequence[int], eps: float = EPSILON, theta: float = ROPE_THETA,
                 q_out: Optional[torch.Tensor] = None, k_out: Optional[torch.Tensor] = None,
                 stream=None):
    """Normed + roped q [T,16,128] and k [T,8,128] (f16) from qkv [T, stride]."""
    T = int(cu_seqlens[-1])
    q_out = q_out if q_out is not None else torch.empty(T, Q_HEADS, HEAD_DIM, dtype=torch.float16,
                                                        device=qkv.device)
    k_out = k_out if k_out is not None else torch.empty(T, KV_HEADS, HEAD_DIM, dtype=torch.float16,
                                                        device=qkv.device)
    kern = QKNormRopeKernel(qkv.device.index)
    encode_run(stream, kern.create_run_varlen(qkv, q_weight, k_weight, q_out, k_out, cu_seqlens,
                                              eps, qkv.shape[1], theta))
    return q_out, k_out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: Sequence[int],
              value_stride: int = 1024, value_offset: int = 0, mode: int = MODE_AUTO,
              prefix: int = PREFIX, window: int = WINDOW, out: Optional[torch.Tensor] = None,
              stream=None) -> torch.Tensor:
    T = int(cu_seqlens[-1])
    out = out if out is not None else torch.empty(T, Q_HEADS, HEAD_DIM, dtype=torch.float16,
                                                  device=q.device)
    kern = CausalAttentionKernel(q.device.index)
    kern.encode(stream, kern.create_run_varlen(q, k, v, out, cu_seqlens, value_stride,
                                               value_offset, mode, prefix, window))
    return out


def prefill_attention_layer(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                            cu_seqlens: Sequence[int], mode: int = MODE_AUTO,
                            prefix: int = PREFIX, window: int = WINDOW, eps: float = EPSILON,
                            theta: float = ROPE_THETA, q_buf=None, k_buf=None, out=None,
                            stream=None, ctx: Optional[Context] = None) -> torch.Tensor:
    """Prologue + attention of one layer (model.ts:94-95): qkv [T, 4096] f16.
    ``ctx``: the context to launch on (default: the device's shared one)."""
    _f16_cuda(qkv, "qkv")
    _f32_weight(q_weight, "q_weight")
    _f32_weight(k_weight, "k_weight")
    T = int(cu_seqlens[-1])
    dev = qkv.device
    q_buf = q_buf if q_buf is not None else torch.empty(T, Q_HEADS, HEAD_DIM, dtype=torch.float16,
                                                        device=dev)
    k_buf = k_buf if k_buf is not None else torch.empty(T, KV_HEADS, HEAD_DIM, dtype=torch.float16,
                                                        device=dev)
    out = out if out is not None else torch.empty(T, Q_HEADS, HEAD_DIM, dtype=torch.float16,
                                                  device=dev)
    ctx = ctx if ctx is not None else Context.for_device(dev.index)
    cu = _lib.cu_array(cu_seqlens)
    st = ctx.lib.qwa_prefill_attention_layer(ctx.handle, _ptr(qkv), qkv.shape[1], _ptr(q_weight),
                                             _ptr(k_weight), _ptr(q_buf), _ptr(k_buf), _ptr(out),
                                             cu, len(cu) - 1, mode, prefix, window, eps, theta,
                                             _stream(stream))
    _lib.check(st, ctx.handle)
    return out


def attention_work(cu_seqlens: Sequence[int], mode: int = MODE_AUTO, prefix: int = PREFIX,
                   window: int = WINDOW):
    """(kept pairs per q-head, key tiles visited per kv group) of one call."""
    cu = _lib.cu_array(cu_seqlens)
    pairs, tiles = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(_lib.load().qwa_attention_work(cu, len(cu) - 1, mode, prefix, window,
                                              ctypes.byref(pairs), ctypes.byref(tiles)))
    return pairs.value, tiles.value


def selftest_tile(a: torch.Tensor, b: torch.Tensor, vt: torch.Tensor):
    """Diagnostic single-tile tcgen05 check (see include/qwa.h)."""
    for t, n in ((a, "a"), (b, "b"), (vt, "vt")):
        _f16_cuda(t, n)
        _need(t.shape == (128, 128), f"{n} must be 128x128")
    ctx = Context.for_device(a.device.index)
    c = torch.empty(128, 128, dtype=torch.float32, device=a.device)
    d = torch.empty(128, 128, dtype=torch.float32, device=a.device)
    _lib.check(ctx.lib.qwa_selftest_tile(ctx.handle, _ptr(a), _ptr(b), _ptr(vt), _ptr(c), _ptr(d),
                                         _stream(None)), ctx.handle)
    return c, d
