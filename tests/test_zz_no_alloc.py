"""qwa_attention_noalloc: attention for callers that cannot allocate device memory.

Some hosts (a serving runtime with a fixed, pre-planned memory arena, or a
process that holds no qwa_ctx) may not call cudaMalloc on their hot path.
This entry point keeps its work list in a fixed array inside the library; the
test checks, through the C ABI, that two calls in a row (different shapes, so
the second overwrites what the first left in that array) match the regular
qwa_attention within the same tolerance as the other parity tests, and that a
call too large for the array is rejected before launching.

This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3


def _noalloc(pkg, q, k, v, cu, v_stride, v_offset, mode, prefix=176, window=432):
    lib = pkg._lib.load()
    out = torch.empty_like(q)
    arr = pkg._lib.cu_array(cu)
    st = lib.qwa_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), v_stride, v_offset, ctypes.c_void_p(out.data_ptr()), arr,
        len(cu) - 1, mode, prefix, window, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == pkg._lib.QWA_OK, pkg._lib.status_string(st)
    return out


def test_noalloc_matches_attention_two_calls(pkg, cuda_dev):
    attn = pkg.attention
    cases = [([700, 33, 1300], 0), ([5000, 128, 1], 1)]
    for n, (lengths, mode) in enumerate(cases):
        rng = np.random.default_rng(100 + n)
        cu = [0] + [int(x) for x in np.cumsum(lengths)]
        T = cu[-1]
        q = torch.from_numpy(rng.standard_normal((T, 16, 128), dtype=np.float32)).half().cuda()
        k = torch.from_numpy(rng.standard_normal((T, 8, 128), dtype=np.float32)).half().cuda()
        v = torch.from_numpy(rng.standard_normal((T, 4096), dtype=np.float32)).half().cuda()
        got = _noalloc(pkg, q, k, v, cu, 4096, 3072, mode)
        ref = attn.attention(q, k, v, cu, 4096, 3072, mode)
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= MAX_ABS, f"call {n}: max-abs {err}"


def test_noalloc_rejects_oversized_batch(pkg, cuda_dev):
    lib = pkg._lib.load()
    # 9000 requests of 128 tokens need 72,000 work items (> 65,520 in the array)
    cu = [128 * i for i in range(9001)]
    dummy = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = ctypes.c_void_p(dummy.data_ptr())
    st = lib.qwa_attention_noalloc(p, p, p, 1024, 0, p, pkg._lib.cu_array(cu), 9000, 0, 176, 432,
                                   None)
    assert st == pkg._lib.QWA_ERR_INVALID_ARG
