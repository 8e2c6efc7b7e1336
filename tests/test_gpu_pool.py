"""Last-token L2 pool kernel and the varlen engine runtime on the GPU.

The pool is f32 output from f16 rows; the tolerance is 1e-6 absolute per
element against the fp64 oracle (src/webgpu/ops.ts:347-359 sums in f32 too).
"""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
POOL_TOL = 1e-6


def _rows(rng, T, width):
    return rng.standard_normal((T, width)).astype(np.float16)


@pytest.mark.parametrize("lengths,width", [
    ([50], 1024),                       # config 1 shape
    ([1, 0, 300, 5000, 17], 1024),      # ragged, with an empty request
    ([128] * 16, 1024),                 # full micro-batch
    ([7, 9], 4096),                     # wider rows
    ([3], 8),                           # narrowest legal width
])
def test_pool_varlen_matches_oracle(pkg, oracle, cuda_dev, lengths, width):
    pool = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.pooling")
    rng = np.random.default_rng(sum(lengths) + width)
    cu = [0] + [int(c) for c in np.cumsum(lengths)]
    h = _rows(rng, cu[-1], width)
    got = pool.last_token_pool(torch.from_numpy(h).cuda(), cu).cpu().numpy()
    ref = oracle.c_last_token_pool(h, cu)
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= POOL_TOL


def test_pool_padded_matches_reference_indexing(pkg, oracle, cuda_dev):
    pool = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.pooling")
    rng = np.random.default_rng(5)
    S, lengths = 300, [1, 300, 0, 123]
    h = _rows(rng, len(lengths) * S, 1024)
    d_len = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    out = torch.full((len(lengths), 1024), float("nan"), device="cuda")
    kern = pool.LastTokenPoolKernel(0)
    pkg.attention.encode_run(None, kern.create_run(torch.from_numpy(h).cuda(), d_len, out,
                                                   len(lengths), S))
    ref = oracle.np_last_token_pool_padded(h, lengths, S)
    assert np.abs(out.cpu().numpy() - ref).max() <= POOL_TOL


def test_pool_rejects_bad_width(pkg, cuda_dev):
    pool = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.pooling")
    h = torch.zeros(4, 12, dtype=torch.float16, device="cuda")
    with pytest.raises(Exception):
        pool.last_token_pool(h, [0, 4])


def _requests(rng, lengths, vocab):
    return [list(rng.integers(0, vocab - 1, size=n - 1)) + [vocab - 1] for n in lengths]


def test_engine_varlen_equals_padded_and_single(pkg, cuda_dev):
    """Packed and padded micro-batches give each request the same embedding,
    and batching does not change it (the batch-vs-single gate of
    src/main.ts:314-316 asks cosine >= 0.999)."""
    import asyncio
    eng_mod = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.engine")
    vocab = 4096
    rt = eng_mod.AttentionStackRuntime(layers=3, vocab=vocab, seed=1)
    rng = np.random.default_rng(9)
    reqs = _requests(rng, [15, 700, 1, 150, 64, 999], vocab)

    async def embed_all(packing, batch_size):
        eng = eng_mod.EmbeddingEngine(rt, None, batch_size, 0, vocab - 1, packing=packing)
        return await asyncio.gather(*[eng.submit_tokens(r) for r in reqs])

    var = np.stack(asyncio.run(embed_all("varlen", 16)))
    pad = np.stack(asyncio.run(embed_all("padded", 16)))
    single = np.stack(asyncio.run(embed_all("varlen", 1)))
    assert np.isfinite(var).all()
    assert np.allclose(np.linalg.norm(var, axis=1), 1.0, atol=1e-5)
    for other in (pad, single):
        cos = np.sum(var * other, axis=1)
        assert cos.min() >= 0.9999, cos
