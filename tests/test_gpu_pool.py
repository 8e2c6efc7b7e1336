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


def test_engine_runtime_from_prepacked_file(pkg, cuda_dev, tmp_path):
    """A synthetic .wgpack with the reference's tensor names loads onto the
    device, and the runtime built from it embeds like the seeded one built from
    the same packed bytes."""
    import asyncio
    pp = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.prepacked")
    eng_mod = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.engine")
    rng = np.random.default_rng(4)
    layers, tensors = 2, []
    for l in range(layers):
        tensors.append(pp.pack_q40_tile32(f"blk.{l}.attn_qkv.weight", [
            pp.q40_part("q", pp.random_q40_rows(rng, 2048, 1024, 0.006), 1024),
            pp.q40_part("k", pp.random_q40_rows(rng, 1024, 1024, 0.006), 1024),
            pp.q40_part("v", pp.random_q40_rows(rng, 1024, 1024, 0.006), 1024)]))
        tensors.append(pp.pack_q40_tile32(f"blk.{l}.attn_output.weight", [
            pp.q40_part("o", pp.random_q40_rows(rng, 1024, 2048, 0.004), 2048)]))
        for key, n in (("attn_q_norm", 128), ("attn_k_norm", 128), ("attn_norm", 1024)):
            tensors.append(pp.raw_tensor(f"blk.{l}.{key}.weight", [n], pp.GGML_F32,
                                         (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)))
    tensors.append(pp.raw_tensor("output_norm.weight", [1024], pp.GGML_F32,
                                 np.ones(1024, np.float32)))
    path = tmp_path / "tiny.wgpack"
    path.write_bytes(pp.build_prepacked_file("0" * 64, 0, {"general.name": "tiny"}, tensors))
    weights = pp.PrepackedWeights.from_file(str(path), 0)
    assert weights.layers() == 2 and weights.metadata["general.name"] == "tiny"
    assert weights.weight("blk.1.attn_qkv.weight").dtype == torch.uint8
    assert weights.weight("blk.0.attn_q_norm.weight").dtype == torch.float32
    with pytest.raises(KeyError, match="missing tensor"):
        weights.weight("blk.9.attn_qkv.weight")
    rt = eng_mod.AttentionStackRuntime(layers=2, vocab=4096, seed=3, weights=weights)
    reqs = _requests(np.random.default_rng(1), [40, 300, 7], 4096)

    async def run():
        eng = eng_mod.EmbeddingEngine(rt, None, 16, 0, 4095, packing="varlen")
        return await asyncio.gather(*[eng.submit_tokens(r) for r in reqs])

    emb = np.stack(asyncio.run(run()))
    assert np.isfinite(emb).all() and np.allclose(np.linalg.norm(emb, axis=1), 1, atol=1e-5)
    # the same layers through matmul + attention, step by step, match
    mm, attn, norm = pkg.matmul, pkg.attention, pkg.norm
    cu = [0, 40, 340, 347]
    ids = torch.from_numpy(np.concatenate(reqs).astype(np.int64)).cuda()
    x = rt.embed_table[ids]
    h = norm.rms_norm(x, rt.in_norm[0])
    for l in range(2):
        qkv = mm.matmul(h, mm.q40_dequantize(rt.w_qkv[l], 4096, 1024))
        o = attn.prefill_attention_layer(qkv, rt.q_norm[l], rt.k_norm[l], cu)
        delta = mm.matmul(o.view(-1, 2048), mm.q40_dequantize(rt.w_o[l], 1024, 2048))
        nxt = rt.in_norm[l + 1] if l + 1 < 2 else rt.final_norm
        norm.rms_norm(x, nxt, residual=delta, out=h)
    ref = pkg.pooling.last_token_pool(h, cu).cpu().numpy()
    assert np.array_equal(ref, emb)
