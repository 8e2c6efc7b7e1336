"""The whole Qwen3-Embedding-0.6B forward on one B200, from prepacked weights.

Follows ``Qwen3ExecutionPlan`` (src/webgpu/model.ts:60-136) step for step:

* Q6_K token-embedding lookup into the residual stream ``x`` (ops.ts:381-426)
  and the first RMSNorm with blk.0.attn_norm (no residual);
* per layer: the attn_qkv projection (Q4_0) with the per-head Q/K RMSNorm +
  RoPE fused into its epilogue, attention (sparse 176 + 432 rule up to 8192
  tokens), the attn_output projection, residual + RMSNorm with ffn_norm, the
  ffn_gate_up projection with the SwiGLU in its epilogue, the ffn_down
  projection, and residual + RMSNorm with the next layer's attn_norm
  (output_norm after the last);
* the last-token L2 pool of the final normalized state (ops.ts:347-379).

Every step is a libqwa kernel. Projections run on the tcgen05 GEMM from f16
copies of the Q4_0 tile32 matrices, dequantised once (bit-exact with the
reference's dequantised values). Requests are packed back to back
(``cu_seqlens``) or padded like the reference (``create_plan``); the
engine (engine.py) drives either.

``synthetic_model_file`` builds a complete ``.wgpack`` with seeded random
weights of the model's shapes: the 384 MiB release file is not available
here, so embeddings are not the trained model's.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np
import torch

from . import attention as attn
from . import ffn, matmul, norm, prepacked
from .pooling import last_token_pool

HIDDEN, INTERMEDIATE, Q_WIDTH, LAYERS = 1024, 3072, 2048, 28  # model.ts:18-21
EPSILON = 1e-6
# batches of at most this many tokens run the 1024-row projections (attn_output,
# ffn_down) straight from the Q4_0 records (qwa_q40_matmul's small-batch path)
SMALL_ROWS = 64

# name -> [k, n] of each compact Q4_0 matrix of a block (model.ts:89-101)
COMPACT = {"attn_qkv": [HIDDEN, 4096], "attn_output": [Q_WIDTH, HIDDEN],
           "ffn_gate_up": [HIDDEN, 2 * INTERMEDIATE], "ffn_down": [INTERMEDIATE, HIDDEN]}


def synthetic_model_file(layers: int = LAYERS, vocab: int = 4096, seed: int = 0) -> bytes:
    """A complete .wgpack (format.ts:101-169) with seeded weights: Q6_K
    token_embd [1024, vocab]; per block the four compact Q4_0 matrices,
    attn_norm, ffn_norm (F32 [1024]) and attn_q_norm / attn_k_norm (F32
    [128]); output_norm. Scales keep every projection's output near unit
    variance, so the residual stream stays in f16 range over 28 layers."""
    rng = np.random.default_rng(seed)
    pp = prepacked
    table = pp.random_q6k_rows(rng, vocab, HIDDEN)
    tensors = [pp.raw_tensor("token_embd.weight", [HIDDEN, vocab], pp.GGML_Q6_K, table)]

    def gains(n):
        return (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)

    for l in range(layers):
        b = f"blk.{l}"
        tensors.append(pp.raw_tensor(f"{b}.attn_norm.weight", [HIDDEN], pp.GGML_F32,
                                     gains(HIDDEN)))
        for name, (k, n) in COMPACT.items():
            rows = pp.random_q40_rows(rng, n, k, 0.25 / k ** 0.5, centered=True)
            tensors.append(pp.pack_q40_tile32(f"{b}.{name}.weight",
                                              [pp.q40_part(name, rows, k)]))
        tensors.append(pp.raw_tensor(f"{b}.attn_q_norm.weight", [128], pp.GGML_F32, gains(128)))
        tensors.append(pp.raw_tensor(f"{b}.attn_k_norm.weight", [128], pp.GGML_F32, gains(128)))
        tensors.append(pp.raw_tensor(f"{b}.ffn_norm.weight", [HIDDEN], pp.GGML_F32,
                                     gains(HIDDEN)))
    tensors.append(pp.raw_tensor("output_norm.weight", [HIDDEN], pp.GGML_F32, gains(HIDDEN)))
    meta = {"general.architecture": "qwen3", "general.name": "synthetic",
            "qwen3.block_count": layers}
    return pp.build_prepacked_file("0" * 64, 0, meta, tensors)


class Qwen3EmbeddingModel:
    """Qwen3WebGPUModel + Qwen3ExecutionPlan (model.ts:60-136, 189-274) for a
    prepacked source on one CUDA device."""

    def __init__(self, weights: "prepacked.PrepackedWeights", layers: Optional[int] = None):
        self.w = weights
        self.device = weights.device
        self._attn = attn
        n_layers = weights.layers()
        compact = sum(1 for s in weights.storage.values() if s == prepacked.STORAGE_COMPACT)
        if compact != n_layers * 4:
            # the reference's check (model.ts:222)
            raise ValueError(f"prepacked model has {compact} compact matrices; expected "
                             f"{n_layers * 4}")
        self.layers = n_layers if layers is None else layers
        if self.layers > n_layers:
            raise ValueError(f"prepacked weights hold {n_layers} layers; {self.layers} asked")
        emb_dims = weights.dims["token_embd.weight"]
        if weights.storage["token_embd.weight"] != prepacked.STORAGE_RAW or emb_dims[0] != HIDDEN:
            raise ValueError("token_embd.weight must be a raw Q6_K [1024, vocab] tensor")
        self.vocab = int(emb_dims[1])
        self.embed_table = weights.weight("token_embd.weight")
        self.f16 = []  # per layer: dequantised projections, f16 [n, k]
        self.packed = []  # per layer: the compact Q4_0 bytes of attn_output / ffn_down
        self.gains = []
        for l in range(self.layers):
            mats = {}
            for name, kn in COMPACT.items():
                full = f"blk.{l}.{name}.weight"
                if weights.storage[full] != prepacked.STORAGE_COMPACT or weights.dims[full] != kn:
                    raise ValueError(f"{full} must be a compact Q4_0 matrix of dimensions {kn}")
                k, n = kn
                mats[name] = matmul.q40_dequantize(weights.weight(full), n, k)
            # gate_up rows interleaved in 128-row blocks for the GEMM whose
            # epilogue applies the SwiGLU (no [T, 6144] intermediate)
            mats["ffn_gate_up"] = matmul.interleave_gate_up(mats["ffn_gate_up"])
            self.f16.append(mats)
            self.packed.append({name: weights.weight(f"blk.{l}.{name}.weight")
                                for name in ("attn_output", "ffn_down")})
            self.gains.append({key: weights.weight(f"blk.{l}.{key}.weight").float().contiguous()
                               for key in ("attn_norm", "attn_q_norm", "attn_k_norm",
                                           "ffn_norm")})
        self.output_norm = weights.weight("output_norm.weight").float().contiguous()

    def forward(self, ids: torch.Tensor, cu_seqlens: Sequence[int], mode: int = attn.MODE_AUTO,
                trace: Optional[List[torch.Tensor]] = None) -> torch.Tensor:
        """Final normalized hidden state f16 [T, 1024] for packed ``ids``
        (CUDA int32). ``trace``: if a list, receives a copy of the residual
        stream after every layer."""
        T = int(cu_seqlens[-1])
        dev = self.device
        f16 = dict(dtype=torch.float16, device=dev)
        x = ffn.embedding_lookup(ids, self.embed_table, HIDDEN, self.vocab)
        normalized = norm.rms_norm(x, self.gains[0]["attn_norm"])
        delta = torch.empty(T, HIDDEN, **f16)
        hidden = torch.empty(T, INTERMEDIATE, **f16)
        q = torch.empty(T, 16, 128, **f16)
        k = torch.empty(T, 8, 128, **f16)
        v = torch.empty(T, 1024, **f16)
        o = torch.empty(T, 16, 128, **f16)
        for l in range(self.layers):
            w, g = self.f16[l], self.gains[l]
            matmul.qkv_projection(normalized, w["attn_qkv"], g["attn_q_norm"], g["attn_k_norm"],
                                  cu_seqlens, EPSILON, q_out=q, k_out=k, v_out=v)
            attn.attention(q, k, v, cu_seqlens, value_stride=1024, value_offset=0, mode=mode,
                           out=o)
            if T <= SMALL_ROWS:  # few rows: read the Q4_0 records (less weight traffic)
                matmul.q40_matmul(o.view(T, Q_WIDTH), self.packed[l]["attn_output"], HIDDEN,
                                  Q_WIDTH, out=delta)
            else:
                matmul.matmul(o.view(T, Q_WIDTH), w["attn_output"], out=delta)
            norm.rms_norm(x, g["ffn_norm"], residual=delta, out=normalized)
            matmul.matmul_swiglu(normalized, w["ffn_gate_up"], out=hidden)
            if T <= SMALL_ROWS:
                matmul.q40_matmul(hidden, self.packed[l]["ffn_down"], HIDDEN, INTERMEDIATE,
                                  out=delta)
            else:
                matmul.matmul(hidden, w["ffn_down"], out=delta)
            nxt = self.gains[l + 1]["attn_norm"] if l + 1 < self.layers else self.output_norm
            norm.rms_norm(x, nxt, residual=delta, out=normalized)
            if trace is not None:
                trace.append(x.clone())
        return normalized

    def embed(self, ids: torch.Tensor, cu_seqlens: Sequence[int]) -> torch.Tensor:
        """L2-normalised last-token embeddings f32 [batch, 1024]."""
        return last_token_pool(self.forward(ids, cu_seqlens), cu_seqlens)

    # the engine's runtime interface (engine.py)
    hidden = HIDDEN

    def create_plan(self, batch: int, sequence: int):
        from .engine import _PaddedPlan
        return _PaddedPlan(self, batch, sequence)

    def create_varlen_plan(self, batch: int, capacity: int):
        from .engine import _VarlenPlan
        return _VarlenPlan(self, batch, capacity)


class MultiDeviceModel:
    """One micro-batch of embedding requests over several devices of a box:
    each device holds its own ``Qwen3EmbeddingModel`` (weights replicated),
    the requests are split by LPT on their attention work
    (``sharding.lpt_shard``), every device runs its share as one packed batch
    from one host thread, and the embeddings come back in request order. No
    collective is involved. AUTO attention is resolved on the whole
    micro-batch, as one device would (ops.ts:328).

    It offers the engine's runtime interface (``create_plan`` /
    ``create_varlen_plan``), so ``EmbeddingEngine`` can drive it unchanged."""

    hidden = HIDDEN

    def __init__(self, models: Sequence[Qwen3EmbeddingModel]):
        if not models:
            raise ValueError("models must not be empty")
        self.models = list(models)

    def embed_packed(self, ids: np.ndarray, cu_seqlens: Sequence[int],
                     mode: int = attn.MODE_AUTO) -> np.ndarray:
        """f32 [batch, 1024] embeddings of packed host ids (int)."""
        import threading

        from . import sharding
        cu = [int(c) for c in cu_seqlens]
        lengths = [cu[b + 1] - cu[b] for b in range(len(cu) - 1)]
        sparse = sharding.resolve_sparse(mode, lengths)
        rmode = attn.MODE_SPARSE if sparse else attn.MODE_FULL
        assignment = sharding.lpt_shard(lengths, len(self.models), rmode)
        out = np.zeros((len(lengths), HIDDEN), np.float32)
        errors: List[BaseException] = []

        def work(r: int) -> None:
            reqs = [b for b in assignment[r] if lengths[b] > 0]
            if not reqs:
                return
            try:
                m = self.models[r]
                local_ids = np.concatenate([ids[cu[b]:cu[b + 1]] for b in reqs])
                local_cu = [0] + np.cumsum([lengths[b] for b in reqs]).astype(int).tolist()
                with torch.cuda.device(m.device):
                    d_ids = torch.from_numpy(local_ids.astype(np.int32)).to(m.device)
                    emb = last_token_pool(m.forward(d_ids, local_cu, rmode), local_cu)
                    out[reqs] = emb.cpu().numpy()
            except BaseException as e:  # noqa: BLE001 -- re-raised on the caller's thread
                errors.append(e)

        threads = [threading.Thread(target=work, args=(r,)) for r in range(len(self.models))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return out

    def create_plan(self, batch: int, sequence: int):
        return _MultiPlan(self, batch, sequence)

    def create_varlen_plan(self, batch: int, capacity: int):
        return _MultiPlan(self, batch, capacity)


class _MultiPlan:
    """Both packings reduce to the packed batch of the requests' own tokens
    (a padded plan's EOS padding never changes a request's last-token
    embedding, since attention is causal)."""

    def __init__(self, rt: MultiDeviceModel, batch: int, size: int):
        self.rt, self.batch, self.size = rt, batch, size

    def run(self, ids: np.ndarray, lengths: np.ndarray) -> List[np.ndarray]:
        seq = self.size
        packed = np.concatenate([ids[b * seq:b * seq + int(n)] for b, n in enumerate(lengths)])
        cu = [0] + np.cumsum(np.asarray(lengths, int)).tolist()
        return list(self.rt.embed_packed(packed, cu))

    def run_varlen(self, ids: np.ndarray, cu_seqlens: np.ndarray) -> List[np.ndarray]:
        if int(cu_seqlens[-1]) > self.size:
            raise ValueError("micro-batch exceeds the plan's token capacity")
        return list(self.rt.embed_packed(np.asarray(ids), cu_seqlens))
