"""Q4_0 tile32 dequantisation and the tcgen05 projection GEMM vs the oracle.

Dequantisation is bit-exact (f16 products, round to nearest even). The GEMM
accumulates in f32 and rounds once to f16; against the fp64 oracle each
element must satisfy |got - ref| <= 1e-3 * |ref| + 2e-3 * max|ref| (f16
output rounding plus f32 accumulation over up to 3072 terms), and every row
must have cosine >= 0.99999 with the oracle.
"""
import importlib

import numpy as np
import pytest
import torch

from oracle import q40

pytestmark = pytest.mark.gpu


def _check(got: np.ndarray, ref: np.ndarray):
    got = got.astype(np.float64)
    scale = np.abs(ref).max()
    assert np.all(np.abs(got - ref) <= 1e-3 * np.abs(ref) + 2e-3 * scale), \
        float(np.abs(got - ref).max() / scale)
    cos = np.sum(got * ref, 1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1) + 1e-30)
    assert cos.min() >= 0.99999


def _packed(rng, n, k):
    rows = q40.random_q40_rows(rng, n, k)
    packed, _, _ = q40.pack_q40_tile32([(rows, n)])
    return packed


@pytest.mark.parametrize("n,k", [(4096, 1024), (1000, 64), (31, 2048)])
def test_dequant_bit_exact(pkg, cuda_dev, n, k):
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(n + k)
    packed = _packed(rng, n, k)
    got = mm.q40_dequantize(torch.from_numpy(packed).cuda(), n, k).cpu().numpy()
    ref = q40.dequant_tile32(packed, n, k)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("m,n,k", [
    (1, 256, 64), (50, 1024, 1024), (128, 4096, 1024), (1000, 1024, 2048),
    (777, 512, 3072), (5000, 4096, 1024), (300, 6144, 1024),
    (4096, 256, 64), (9000, 1024, 2048),  # M >= 4096 runs on CTA pairs (cta_group::2)
])
def test_matmul_matches_oracle(pkg, cuda_dev, m, n, k):
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(m * 31 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * k ** -0.5).astype(np.float16)
    got = mm.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda())
    pkg.attention.Context.for_device(0).check()
    _check(got.cpu().numpy(), q40.matmul(a, w))


def test_q40_matmul_run_matches_oracle_and_caches(pkg, cuda_dev):
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(7)
    m, n, k = 640, 4096, 1024
    packed = _packed(rng, n, k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    kern = mm.QuantMatmulKernel(0)
    dp = torch.from_numpy(packed).cuda()
    run = kern.create_run_from_buffers(torch.from_numpy(a).cuda(), dp, m, n, k)
    kern.encode(None, run)
    first = run.output.clone()
    kern.encode(None, run)  # served from the cached f16 copy
    assert torch.equal(first, run.output)
    _check(run.output.cpu().numpy(), q40.matmul(a, q40.dequant_tile32(packed, n, k)))
    # rewriting the packed buffer needs forget(); then the new values are used
    dp.zero_()
    kern.forget(dp)
    kern.encode(None, run)
    assert not run.output.any()


def test_matmul_rejects_unsupported_shapes(pkg, cuda_dev):
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    a = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(Exception):
        mm.matmul(a, torch.zeros(100, 64, dtype=torch.float16, device="cuda"))
    with pytest.raises(Exception):
        mm.matmul(torch.zeros(4, 40, dtype=torch.float16, device="cuda"),
                  torch.zeros(256, 40, dtype=torch.float16, device="cuda"))


@pytest.mark.parametrize("m,n,k", [(197, 6144, 1024), (1, 512, 64), (4096, 6144, 1024),
                                   (5000, 1024, 128), (64, 6144, 1024)])
def test_gate_up_swiglu_equals_unfused_bits(pkg, cuda_dev, m, n, k):
    """gate_up GEMM with the SwiGLU in its epilogue (interleaved weight rows)
    must give the bits of the GEMM, its f16 output, then the SwiGLU kernel;
    m = 4096 and 5000 take the CTA-pair shape with TMA stores."""
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(m + n + k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float16)).cuda()
    w = torch.from_numpy((rng.standard_normal((n, k)) * 2 * k ** -0.5).astype(np.float16)).cuda()
    fused = mm.matmul_swiglu(x, mm.interleave_gate_up(w))
    ref = pkg.ffn.swiglu(mm.matmul(x, w), n // 2)
    pkg.attention.Context.for_device(0).check()
    assert fused.shape == (m, n // 2)
    assert torch.equal(fused.view(torch.int16), ref.view(torch.int16))


def test_interleave_gate_up_layout(pkg):
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    w = torch.arange(512 * 2, dtype=torch.float32).view(512, 2).half()
    il = mm.interleave_gate_up(w)
    assert torch.equal(il[0:128], w[0:128]) and torch.equal(il[128:256], w[256:384])
    assert torch.equal(il[256:384], w[128:256]) and torch.equal(il[384:512], w[384:512])


@pytest.mark.parametrize("lengths,k", [([50, 17, 130], 1024), ([1], 64), ([5000, 128, 1], 1024),
                                       ([300, 0, 257], 2048)])
def test_fused_qkv_projection_equals_unfused_bits(pkg, cuda_dev, lengths, k):
    """GEMM + rounding to f16 + prologue, fused, must give the unfused bits."""
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    attn = pkg.attention
    rng = np.random.default_rng(sum(lengths) + k)
    cu = [0] + [int(c) for c in np.cumsum(lengths)]
    T = cu[-1]
    x = torch.from_numpy(rng.standard_normal((T, k)).astype(np.float16)).cuda()
    w = torch.from_numpy((rng.standard_normal((4096, k)) * k ** -0.5).astype(np.float16)).cuda()
    qw = torch.from_numpy((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)).cuda()
    kw = torch.from_numpy((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)).cuda()
    q, kk, v = mm.qkv_projection(x, w, qw, kw, cu)
    qkv = mm.matmul(x, w)
    q_ref, k_ref = attn.qk_norm_rope(qkv, qw, kw, cu)
    attn.Context.for_device(0).check()
    assert torch.equal(q.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(kk.view(torch.int16), k_ref.view(torch.int16))
    assert torch.equal(v, qkv[:, 3072:])


def test_fused_qkv_projection_q40_matches_oracle(pkg, oracle, cuda_dev):
    """Q4_0 weights through the fused kernel vs the CPU oracle (dequantise,
    fp64 matmul rounded to f16, C prologue). The kernel's f32 accumulation can
    round a qkvRaw value to the neighbouring f16, so the bound per element is
    2e-3 plus one f16 ulp of the value (2^-10 |ref|); per-head cosine >= 0.9999."""
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(77)
    lengths = [50, 17, 130]
    cu = [0] + [int(c) for c in np.cumsum(lengths)]
    T, k = cu[-1], 1024
    packed = _packed(rng, 4096, k)
    x = rng.standard_normal((T, k)).astype(np.float16)
    qw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    q, kk, v = mm.qkv_projection(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(),
                                 torch.from_numpy(qw).cuda(), torch.from_numpy(kw).cuda(), cu)
    w = q40.dequant_tile32(packed, 4096, k)
    qkv = q40.matmul(x, w).astype(np.float16)
    q_ref, k_ref = oracle.c_qk_norm_rope(qkv, qw, kw, cu)
    for got, ref in ((q.cpu().numpy().astype(np.float64), q_ref),
                     (kk.cpu().numpy().astype(np.float64), k_ref)):
        assert np.all(np.abs(got - ref) <= 2e-3 + np.abs(ref) * 2.0 ** -10)
        cos = np.sum(got * ref, -1) / (np.linalg.norm(got, axis=-1) * np.linalg.norm(ref, axis=-1))
        assert cos.min() >= 0.9999
    _check(v.cpu().numpy(), q40.matmul(x, w)[:, 3072:])


def test_q40_cache_entry_dies_with_its_tensor(pkg, cuda_dev):
    """A new packed matrix placed at a freed one's address must not be served
    the old f16 copy (the wrapper forgets the copy when the tensor dies)."""
    import gc
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(8)
    m, n, k = 64, 256, 64
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float16)).cuda()
    kern = mm.QuantMatmulKernel(0)
    for trial in range(3):
        packed = _packed(rng, n, k)
        dp = torch.from_numpy(packed).cuda()
        run = kern.create_run_from_buffers(a, dp, m, n, k)
        kern.encode(None, run)
        _check(run.output.cpu().numpy(),
               q40.matmul(a.cpu().numpy(), q40.dequant_tile32(packed, n, k)))
        del run, dp
        gc.collect()


@pytest.mark.parametrize("m", [1, 7, 16, 33, 50, 64])
@pytest.mark.parametrize("n,k", [(1024, 2048), (1024, 3072), (256, 1024), (2048, 64)])
def test_q40_small_batch_reads_packed_records(pkg, cuda_dev, m, n, k):
    """m <= 64 rows on n <= 2048: the projection reads the Q4_0 records
    directly (K split over CTAs, partial sums added in a fixed order): oracle
    parity, identical bits on a repeat, and a rewritten packed buffer is used
    at once (no f16 copy is cached on this path)."""
    mm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.matmul")
    rng = np.random.default_rng(m * 7 + n + k)
    packed = _packed(rng, n, k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    kern = mm.QuantMatmulKernel(0)
    dp = torch.from_numpy(packed).cuda()
    run = kern.create_run_from_buffers(torch.from_numpy(a).cuda(), dp, m, n, k)
    kern.encode(None, run)
    first = run.output.clone()
    kern.encode(None, run)
    pkg.attention.Context.for_device(0).check()
    assert torch.equal(first, run.output)
    _check(first.cpu().numpy(), q40.matmul(a, q40.dequant_tile32(packed, n, k)))
    packed2 = _packed(rng, n, k)
    dp.copy_(torch.from_numpy(packed2))
    kern.encode(None, run)
    pkg.attention.Context.for_device(0).check()
    _check(run.output.cpu().numpy(), q40.matmul(a, q40.dequant_tile32(packed2, n, k)))
