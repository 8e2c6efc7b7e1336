"""qwa_attention_noalloc: attention for callers that cannot allocate device memory.

Some hosts (a serving runtime with a fixed, pre-planned memory arena, or a
process that holds no qwa_ctx) may not call cudaMalloc on their hot path.
This entry point keeps its work list in a fixed array inside the library.
The tests check, through the C ABI:

* two calls in a row, the larger first (so the second runs over what the
  first left in that array), each against the CPU oracle within the parity
  tolerance of the other tests;
* that calls after the first allocate nothing (free device memory and
  torch's allocator unchanged);
* a call of exactly the array's capacity (65,520 work items) is accepted and
  equals the regular qwa_attention, and one item more, or more than 4096
  requests, is rejected before launching;
* qwa_check(NULL, stream) reports the entry point's status word (clear here).

This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MAX_ITEMS = 65520


def _call(pkg, q, k, v, cu, v_stride, v_offset, mode, out=None, prefix=176, window=432):
    lib = pkg._lib.load()
    out = torch.empty_like(q) if out is None else out
    arr = pkg._lib.cu_array(cu)
    st = lib.qwa_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), v_stride, v_offset, ctypes.c_void_p(out.data_ptr()), arr,
        len(cu) - 1, mode, prefix, window, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == pkg._lib.QWA_OK, pkg._lib.status_string(st)
    return out


def _check_noalloc_status(pkg):
    lib = pkg._lib.load()
    st = lib.qwa_check(None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == pkg._lib.QWA_OK, pkg._lib.status_string(st)


def _inputs(lengths, seed):
    rng = np.random.default_rng(seed)
    cu = [0] + [int(x) for x in np.cumsum(lengths)]
    T = cu[-1]
    q = rng.standard_normal((T, 16, 128), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((T, 8, 128), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((T, 4096), dtype=np.float32).astype(np.float16)
    return cu, q, k, v


def test_noalloc_two_calls_match_oracle_and_allocate_nothing(pkg, oracle, cuda_dev):
    # larger call first, then a smaller one over the array's stale tail
    cases = [([5000, 128, 1], 1), ([700, 33, 1300], 0)]
    data = [_inputs(lengths, 100 + n) for n, (lengths, _) in enumerate(cases)]
    dev = [tuple(torch.from_numpy(a).cuda() for a in (q, k, v)) for _, q, k, v in data]
    outs = [torch.empty_like(d[0]) for d in dev]
    # warm-up: the first call on a device looks up the array's address and
    # loads the kernels
    _call(pkg, *dev[1], data[1][0], 4096, 3072, cases[1][1], out=outs[1])
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for n, (_, mode) in enumerate(cases):
        _call(pkg, *dev[n], data[n][0], 4096, 3072, mode, out=outs[n])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "device memory was allocated"
    assert torch.cuda.memory_allocated() == alloc0
    _check_noalloc_status(pkg)
    for n, (cu, q, k, v) in enumerate(data):
        ref = oracle.c_attention(q, k, v, 4096, 3072, cu, cases[n][1])
        err = np.abs(outs[n].cpu().numpy().astype(np.float64) - ref).max()
        assert err <= MAX_ABS, f"call {n}: max-abs {err}"


def test_noalloc_at_capacity_equals_attention(pkg, oracle, cuda_dev):
    # 2 requests x 4095 query tiles x 8 kv heads = 65,520 work items, sparse
    # rule (the kernel's cost stays linear in the length)
    lengths = [4095 * 128, 4095 * 128]
    cu = [0, lengths[0], lengths[0] + lengths[1]]
    T = cu[-1]
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    q = torch.randn(T, 16, 128, generator=g, device="cuda").half()
    k = torch.randn(T, 8, 128, generator=g, device="cuda").half()
    v = torch.randn(T, 1024, generator=g, device="cuda").half()
    got = _call(pkg, q, k, v, cu, 1024, 0, 2)
    ref = pkg.attention.attention(q, k, v, cu, 1024, 0, 2)
    torch.cuda.synchronize()
    _check_noalloc_status(pkg)
    assert torch.equal(got, ref)
    # sampled rows against the oracle (row = token * 16 + head)
    rng = np.random.default_rng(3)
    rows = np.concatenate([rng.integers(0, T * 16, 48), [0, 16 * (lengths[0] - 1) + 5,
                                                         16 * T - 1]])
    want = oracle.c_attention_rows(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), 1024, 0,
                                   cu, rows, 2)
    gotr = got.view(T * 16, 128)[torch.from_numpy(rows).cuda()].cpu().numpy().astype(np.float64)
    assert np.abs(gotr - want).max() <= MAX_ABS


def test_noalloc_rejects_oversized_calls(pkg, cuda_dev):
    lib = pkg._lib.load()
    dummy = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = ctypes.c_void_p(dummy.data_ptr())
    # one work item past the capacity: 8191 query tiles
    cu = [0, 8191 * 128]
    st = lib.qwa_attention_noalloc(p, p, p, 1024, 0, p, pkg._lib.cu_array(cu), 1, 2, 176, 432,
                                   None)
    assert st == pkg._lib.QWA_ERR_INVALID_ARG
    # more requests than the 4096 the call carries in its kernel parameters
    cu = list(range(4098))
    st = lib.qwa_attention_noalloc(p, p, p, 1024, 0, p, pkg._lib.cu_array(cu), 4097, 0, 176, 432,
                                   None)
    assert st == pkg._lib.QWA_ERR_INVALID_ARG
