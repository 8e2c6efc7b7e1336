"""Residual add + RMSNorm kernel vs the oracle (src/webgpu/ops.ts:21-64).

The in-place residual update x = f16(x + residual) is one f32 add and one
round-to-nearest-even, so it must be bit-exact. The normalized output may
differ from the oracle by one f16 ulp, because the oracle sums the squares in
fp64 where the kernel uses an f32 tree.
"""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulps(a: np.ndarray, b: np.ndarray) -> int:
    """Largest distance in f16 ulps (monotone integer mapping of the bits)."""
    def key(h):
        i = h.view(np.uint16).astype(np.int32)
        return np.where(i & 0x8000, 0x8000 - (i & 0x7fff), 0x8000 + i)
    return int(np.abs(key(a) - key(b)).max()) if a.size else 0


@pytest.mark.parametrize("rows,width,has_residual", [
    (1, 1024, True), (5000, 1024, True), (333, 1024, False),   # register path (Qwen3 width)
    (64, 256, True), (64, 2048, False),                          # other register widths
    (17, 40, True), (9, 1000, False), (3, 3072, True),           # generic row path
])
def test_rms_norm_matches_oracle(pkg, oracle, cuda_dev, rows, width, has_residual):
    norm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.norm")
    rng = np.random.default_rng(rows * 7 + width)
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float16)
    r = (rng.standard_normal((rows, width)) * 3).astype(np.float16) if has_residual else None
    w = (1 + 0.02 * rng.standard_normal(width)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dr = torch.from_numpy(r).cuda() if has_residual else None
    out = norm.rms_norm(dx, torch.from_numpy(w).cuda(), residual=dr)
    ref_x, ref_n = oracle.c_rms_norm(x, r, w)
    got_x, got_n = dx.cpu().numpy(), out.cpu().numpy()
    assert np.array_equal(got_x.view(np.uint16), ref_x.view(np.uint16))
    assert _ulps(got_n, ref_n) <= 1


def test_rms_norm_create_run_mirror(pkg, oracle, cuda_dev):
    norm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.norm")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((10, 1024)).astype(np.float16)
    r = rng.standard_normal((10, 1024)).astype(np.float16)
    w = np.ones(1024, np.float32)
    dx, dr = torch.from_numpy(x).cuda(), torch.from_numpy(r).cuda()
    out = torch.empty_like(dx)
    k = norm.RmsNormKernel(0)
    run = k.create_run(dx, dr, torch.from_numpy(w).cuda(), out, 10, 1024, 1e-6, True)
    pkg.attention.encode_run(None, run)
    pkg.attention.encode_run(None, run)  # a second encode adds the residual again
    xs = oracle.c_rms_norm(oracle.c_rms_norm(x, r, w)[0], r, w)
    assert np.array_equal(dx.cpu().numpy().view(np.uint16), xs[0].view(np.uint16))
    assert _ulps(out.cpu().numpy(), xs[1]) <= 1


def test_rms_norm_rejects_bad_width(pkg, cuda_dev):
    norm = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.norm")
    x = torch.zeros(2, 12, dtype=torch.float16, device="cuda")
    with pytest.raises(Exception):
        norm.rms_norm(x, torch.ones(12, device="cuda"))
