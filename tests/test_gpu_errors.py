"""The device half of the error path: a bounded wait that runs out.

The reference's shaders cannot report errors; its engine rejects a whole
micro-batch when a plan fails (src/webgpu/embedding-engine.ts:76-81). Here
every pipeline wait of the attention kernel is bounded. The test shortens
the limit to 50 ms and makes the first CTA leave out one K (or V) load
(qwa_set_debug), so the MMA issuer's wait for it runs out: the kernel stops
that CTA cleanly (issued copies and MMAs complete, tensor memory is freed),
qwa_check reports QWA_ERR_TIMEOUT, and the next normal call on the same
context gives the same bits as before. Nothing here faults or hangs a GPU:
the missing load is a barrier that nothing completes, and the wait on it has
a limit."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(pkg, ctx, q, k, v, out, cu):
    arr = pkg._lib.cu_array(cu)
    P = ctypes.c_void_p
    st = ctx.lib.qwa_attention(ctx.handle, P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()),
                               1024, 0, P(out.data_ptr()), arr, len(cu) - 1, 0, 176, 432,
                               P(torch.cuda.current_stream().cuda_stream))
    pkg._lib.check(st, ctx.handle)


def _check_status(pkg, ctx):
    return ctx.lib.qwa_check(ctx.handle,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_timeout_is_reported_and_the_context_recovers(pkg, cuda_dev):
    ctx = pkg.attention.Context(0)
    try:
        rng = np.random.default_rng(12)
        cu = [0, 700, 1000]
        T = cu[-1]
        q = torch.from_numpy(rng.standard_normal((T, 16, 128), dtype=np.float32)).half().cuda()
        k = torch.from_numpy(rng.standard_normal((T, 8, 128), dtype=np.float32)).half().cuda()
        v = torch.from_numpy(rng.standard_normal((T, 1024), dtype=np.float32)).half().cuda()
        ref = torch.empty_like(q)
        _call(pkg, ctx, q, k, v, ref, cu)
        assert _check_status(pkg, ctx) == pkg._lib.QWA_OK
        out = torch.empty_like(q)
        # load 0 is the first K tile (no MMA issued yet when the wait runs
        # out); load 1 the first V tile (both heads' S MMAs are in flight)
        for skip in (0, 1):
            assert ctx.lib.qwa_set_debug(ctx.handle, 50_000_000, skip) == pkg._lib.QWA_OK
            _call(pkg, ctx, q, k, v, out, cu)
            st = _check_status(pkg, ctx)
            assert st == pkg._lib.QWA_ERR_TIMEOUT, pkg._lib.status_string(st)
            assert b"timed out" in ctx.lib.qwa_last_error(ctx.handle)
            # the status word was cleared by the check
            assert _check_status(pkg, ctx) == pkg._lib.QWA_OK
        assert ctx.lib.qwa_set_debug(ctx.handle, 0, -1) == pkg._lib.QWA_OK
        _call(pkg, ctx, q, k, v, out, cu)
        assert _check_status(pkg, ctx) == pkg._lib.QWA_OK
        assert torch.equal(out, ref)
        assert ctx.lib.qwa_set_debug(ctx.handle, 0, -2) == pkg._lib.QWA_ERR_INVALID_ARG
    finally:
        ctx.close()
