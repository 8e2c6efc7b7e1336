"""Micro-batch scheduler for embedding requests, with varlen packing.

Mirrors ``Qwen3EmbeddingEngine`` (src/webgpu/embedding-engine.ts:21-87):

* ``embed(text)`` tokenizes, appends the EOS token (151643) unless the text
  already ends with it, queues the request and schedules a flush after
  ``batch_window_ms`` (embedding-engine.ts:39-55);
* a flush takes up to ``max_batch_size`` (1..16) queued requests at a time,
  runs them through one plan taken from a cache keyed by the batch shape, and
  resolves the requests in order, or rejects all of them with the plan's
  error (embedding-engine.ts:57-87); requests queued during a flush are
  picked up by the same flush loop, and a new flush is scheduled if any remain.

Two packings:

* ``"padded"`` -- the reference's: ids ``[batch * sequence]`` padded with EOS
  after each request's last token, ``lengths[batch]``, plan cache key
  ``(batch, sequence)``, ``runtime.create_plan(batch, sequence)`` and
  ``plan.run(ids, lengths)``;
* ``"varlen"`` -- no padding: ids are the requests' tokens back to back with
  ``cu_seqlens[batch + 1]`` offsets, the plan cache key is ``(batch,
  capacity)`` with capacity the total token count rounded up to a power of two
  (at least 256), ``runtime.create_varlen_plan(batch, capacity)`` and
  ``plan.run_varlen(ids, cu_seqlens)``. At the reference's 16 requests of
  15..5000 tokens the padded batch computes up to 16x the tokens (and far more
  attention pairs) of the packed one.

``AttentionStackRuntime`` is a device runtime for both packings that runs
libqwa's kernels (Q/K norm + RoPE, attention, residual + RMSNorm, last-token
pool) for every layer.
"""
from __future__ import annotations

import asyncio
import inspect
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

EOS_TOKEN = 151643  # embedding-engine.ts:33
MAX_BATCH = 16  # embedding-engine.ts:35


def _token_list(result: Any) -> List[int]:
    """First row of a tokenizer result: ``result.input_ids.tolist()[0]``
    (embedding-engine.ts:40), or a dict / nested list holding the same."""
    ids = result["input_ids"] if isinstance(result, dict) else getattr(result, "input_ids", result)
    rows = ids.tolist() if hasattr(ids, "tolist") else ids
    return [int(t) for t in rows[0]]


def capacity_for(tokens: int) -> int:
    """Varlen plan capacity: power of two >= tokens, at least 256."""
    cap = 256
    while cap < tokens:
        cap *= 2
    return cap


@dataclass
class _Pending:
    tokens: List[int]
    future: asyncio.Future


class EmbeddingEngine:
    """Coalesces concurrent ``embed`` calls into micro-batches on one runtime."""

    def __init__(self, runtime, tokenizer: Callable[[str], Any], max_batch_size: int = MAX_BATCH,
                 batch_window_ms: float = 0, eos_token: int = EOS_TOKEN,
                 packing: str = "padded"):
        if max_batch_size < 1 or max_batch_size > MAX_BATCH:
            raise ValueError("maxBatchSize must be between 1 and 16")
        if packing not in ("padded", "varlen"):
            raise ValueError("packing must be 'padded' or 'varlen'")
        self.runtime = runtime
        self.tokenizer = tokenizer
        self.max_batch_size = max_batch_size
        self.batch_window_ms = batch_window_ms
        self.eos_token = eos_token
        self.packing = packing
        self.pending: List[_Pending] = []
        self.plans: Dict[Tuple[int, int], Any] = {}
        self._scheduled = False
        self._flushing = False

    # -------------------------------------------------------------- public
    def embed(self, text: str) -> "asyncio.Future":
        """Queue one request; the future resolves to its embedding."""
        tokens = _token_list(self.tokenizer(text))
        if not tokens or tokens[-1] != self.eos_token:
            tokens.append(self.eos_token)
        return self.submit_tokens(tokens)

    def submit_tokens(self, tokens: Sequence[int]) -> "asyncio.Future":
        """Queue already-tokenized ids (EOS included) -- the part of ``embed``
        after the tokenizer."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self.pending.append(_Pending(list(tokens), fut))
        self._schedule()
        return fut

    # ----------------------------------------------------------- internals
    def _schedule(self) -> None:
        if self._scheduled or self._flushing:
            return
        self._scheduled = True
        loop = asyncio.get_running_loop()

        def fire():
            self._scheduled = False
            loop.create_task(self.flush())

        loop.call_later(self.batch_window_ms / 1000.0, fire)

    def _plan(self, key: Tuple[int, int], make: Callable[[], Any]):
        plan = self.plans.get(key)
        if plan is None:
            plan = self.plans[key] = make()
        return plan

    def assemble_padded(self, requests: Sequence[Sequence[int]]):
        """(ids, lengths, sequence) of embedding-engine.ts:61-68."""
        sequence = max(len(r) for r in requests)
        ids = np.full(len(requests) * sequence, self.eos_token, dtype=np.uint32)
        lengths = np.zeros(len(requests), dtype=np.uint32)
        for i, r in enumerate(requests):
            ids[i * sequence:i * sequence + len(r)] = r
            lengths[i] = len(r)
        return ids, lengths, sequence

    @staticmethod
    def assemble_varlen(requests: Sequence[Sequence[int]]):
        """(ids, cu_seqlens): tokens back to back, no padding."""
        cu = np.zeros(len(requests) + 1, dtype=np.int32)
        cu[1:] = np.cumsum([len(r) for r in requests])
        ids = np.zeros(int(cu[-1]), dtype=np.uint32)
        for i, r in enumerate(requests):
            ids[cu[i]:cu[i + 1]] = r
        return ids, cu

    async def _run_batch(self, requests: List[_Pending]):
        toks = [r.tokens for r in requests]
        batch = len(toks)
        if self.packing == "padded":
            ids, lengths, sequence = self.assemble_padded(toks)
            plan = self._plan((batch, sequence),
                              lambda: self.runtime.create_plan(batch, sequence))
            result = plan.run(ids, lengths)
        else:
            ids, cu = self.assemble_varlen(toks)
            cap = capacity_for(int(cu[-1]))
            plan = self._plan((batch, cap),
                              lambda: self.runtime.create_varlen_plan(batch, cap))
            result = plan.run_varlen(ids, cu)
        if inspect.isawaitable(result):
            result = await result
        return result

    async def flush(self) -> None:
        if self._flushing:
            return
        self._flushing = True
        try:
            while self.pending:
                requests = self.pending[:self.max_batch_size]
                del self.pending[:self.max_batch_size]
                try:
                    embeddings = await self._run_batch(requests)
                except Exception as error:  # reject the whole micro-batch
                    for r in requests:
                        if not r.future.done():
                            r.future.set_exception(error)
                    continue
                for r, e in zip(requests, embeddings):
                    if not r.future.done():
                        r.future.set_result(e)
        finally:
            self._flushing = False
            if self.pending:
                self._schedule()


# ------------------------------------------------------------------ runtime

class AttentionStackRuntime:
    """Device runtime for both packings: per layer, the attention half of a
    Qwen3 block with seeded synthetic weights, in the encode order of
    src/webgpu/model.ts:90-104 without the FFN -- QKV projection with the
    Q/K norm + RoPE fused into its epilogue, attention, output projection,
    residual add + RMSNorm with the next layer's weight -- then the last-token
    L2 pool. Every step is a libqwa kernel: the projections take Q4_0
    tile32-compact matrices (as the prepacked model stores attn_qkv /
    attn_output), dequantised once at construction, on the tcgen05 GEMM.

    Weights are seeded random (no checkpoint), so the embeddings are not the
    model's; what this runtime shows is that padded and packed batches give
    the same embedding per request, and what packing saves.
    """

    def __init__(self, layers: int = 28, vocab: int = 151669, hidden: int = 1024,
                 device: Optional[int] = None, seed: int = 0, weights=None):
        from . import attention as attn
        from . import matmul, norm, prepacked
        self._attn = attn
        self._norm = norm
        self._matmul = matmul
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        self.layers = layers
        self.vocab = vocab
        self.hidden = hidden
        g = torch.Generator(device=self.device).manual_seed(seed)
        rng = np.random.default_rng(seed)
        dev = self.device

        def packed(n: int, k: int, scale: float) -> torch.Tensor:
            rows = prepacked.random_q40_rows(rng, n, k, scale)
            t = prepacked.pack_q40_tile32("w", [prepacked.q40_part("w", rows, k)])
            return torch.from_numpy(t.bytes).to(dev)

        def gains(n: int) -> torch.Tensor:
            return (1 + 0.02 * torch.randn(n, generator=g, device=dev)).float()

        self.embed_table = torch.randn(vocab, hidden, generator=g, device=dev).half()
        # Q4_0 values are scale * (q - 8), q uniform: std ~ 4.6 * scale
        self.w_qkv = [packed(4096, hidden, 0.2 / hidden ** 0.5) for _ in range(layers)]
        self.w_o = [packed(hidden, 2048, 0.2 / 2048 ** 0.5) for _ in range(layers)]
        self.q_norm = [gains(128) for _ in range(layers)]
        self.k_norm = [gains(128) for _ in range(layers)]
        self.in_norm = [gains(hidden) for _ in range(layers)]
        self.final_norm = gains(hidden)
        if weights is not None:
            self._use_prepacked(weights)
        self._dequantize()

    def _use_prepacked(self, weights) -> None:
        """Take the attention-half tensors of a PrepackedWeights
        (blk.N.attn_qkv / attn_output compact Q4_0, attn_q_norm, attn_k_norm,
        attn_norm, output_norm). The token embedding stays seeded: the
        reference stores it as Q6_K, whose lookup is not part of this path."""
        n = weights.layers()
        if n < self.layers:
            raise ValueError(f"prepacked weights hold {n} layers; runtime needs {self.layers}")
        for l in range(self.layers):
            t = weights.attention_layer(l)
            self.w_qkv[l], self.w_o[l] = t["attn_qkv"], t["attn_output"]
            self.q_norm[l], self.k_norm[l] = t["attn_q_norm"].float(), t["attn_k_norm"].float()
            self.in_norm[l] = t["attn_norm"].float()
        if "output_norm.weight" in weights.tensors:
            self.final_norm = weights.weight("output_norm.weight").float()

    def _dequantize(self) -> None:
        """f16 copies of every projection, made once (bit-exact with the
        reference's dequantised values); the GEMMs then read them directly."""
        mm = self._matmul
        self.f_qkv = [mm.q40_dequantize(w, 4096, self.hidden) for w in self.w_qkv]
        self.f_o = [mm.q40_dequantize(w, self.hidden, 2048) for w in self.w_o]

    def forward(self, ids: torch.Tensor, cu_seqlens: Sequence[int]) -> torch.Tensor:
        """Final normalized hidden state f16 [T, hidden] for packed ``ids``."""
        norm = self._norm
        x = self.embed_table[ids.long()]  # residual stream, updated in place
        normalized = norm.rms_norm(x, self.in_norm[0])
        for l in range(self.layers):
            # attn_qkv projection fused with the Q/K norm + RoPE (one launch)
            q, k, v = self._matmul.qkv_projection(normalized, self.f_qkv[l], self.q_norm[l],
                                                  self.k_norm[l], cu_seqlens)
            o = self._attn.attention(q, k, v, cu_seqlens, value_stride=1024, value_offset=0)
            delta = self._matmul.matmul(o.view(-1, 2048), self.f_o[l])
            next_w = self.in_norm[l + 1] if l + 1 < self.layers else self.final_norm
            norm.rms_norm(x, next_w, residual=delta, out=normalized)
        return normalized

    def create_plan(self, batch: int, sequence: int) -> "_PaddedPlan":
        return _PaddedPlan(self, batch, sequence)

    def create_varlen_plan(self, batch: int, capacity: int) -> "_VarlenPlan":
        return _VarlenPlan(self, batch, capacity)


class _PaddedPlan:
    """The reference's plan shape: every request computed at ``sequence``."""

    def __init__(self, rt: AttentionStackRuntime, batch: int, sequence: int):
        self.rt, self.batch, self.sequence = rt, batch, sequence
        self.cu = [b * sequence for b in range(batch + 1)]

    def run(self, ids: np.ndarray, lengths: np.ndarray) -> List[np.ndarray]:
        from .pooling import LastTokenPoolKernel
        rt = self.rt
        d_ids = torch.from_numpy(ids.astype(np.int32)).to(rt.device)
        d_len = torch.from_numpy(lengths.astype(np.int32)).to(rt.device)
        h = rt.forward(d_ids, self.cu)
        out = torch.empty(self.batch, rt.hidden, dtype=torch.float32, device=rt.device)
        kern = LastTokenPoolKernel(rt.device.index)
        rt._attn.encode_run(None, kern.create_run(h, d_len, out, self.batch, self.sequence,
                                                  rt.hidden))
        return list(out.cpu().numpy())


class _VarlenPlan:
    """Packed plan: only the requests' own tokens are computed."""

    def __init__(self, rt: AttentionStackRuntime, batch: int, capacity: int):
        self.rt, self.batch, self.capacity = rt, batch, capacity

    def run_varlen(self, ids: np.ndarray, cu_seqlens: np.ndarray) -> List[np.ndarray]:
        from .pooling import last_token_pool
        rt = self.rt
        if int(cu_seqlens[-1]) > self.capacity:
            raise ValueError("micro-batch exceeds the plan's token capacity")
        cu = [int(c) for c in cu_seqlens]
        d_ids = torch.from_numpy(ids.astype(np.int32)).to(rt.device)
        h = rt.forward(d_ids, cu)
        return list(last_token_pool(h, cu).cpu().numpy())
