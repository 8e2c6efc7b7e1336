"""A micro-batch split by request across devices (executor.py) on the GPU.

Two shards share cuda:0 here (one host thread and one context each), which
exercises the same scatter -> prologue + attention -> gather path as two
devices; the kernels of the two shards never wait on each other."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(T, n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        x = rng.standard_normal((T, 4096)).astype(np.float16)
        qw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
        kw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
        out.append((x, qw, kw))
    return out


@pytest.mark.parametrize("lengths,shards", [([300, 17, 0, 130, 700, 64], 2),
                                            ([50, 1500, 9, 260], 3)])
def test_multi_device_executor_matches_single_call_and_oracle(pkg, oracle, cuda_dev, lengths,
                                                              shards):
    ex = pkg.executor
    L = 3
    cu = [0] + list(np.cumsum(lengths))
    T = cu[-1]
    layers = _layers(T, L, seed=21)
    host_in = [torch.from_numpy(x).pin_memory() for x, _, _ in layers]
    host_out = [torch.zeros(T, 16, 128, dtype=torch.float16).pin_memory() for _ in range(L)]
    m = ex.MultiDeviceExecutor(lengths, [0] * shards)
    try:
        m.set_weights([(qw, kw) for _, qw, kw in layers])
        m.run(host_in, host_out)
        assert sorted(i for r in m.plan.assignment for i in r) == list(range(len(lengths)))
    finally:
        m.close()
    for l, (x, qw, kw) in enumerate(layers):
        # the single-device call on the whole batch gives the same bits:
        # every request's rows are computed independently of the others
        one = pkg.attention.prefill_attention_layer(
            torch.from_numpy(x).to(cuda_dev), torch.from_numpy(qw).to(cuda_dev),
            torch.from_numpy(kw).to(cuda_dev), cu)
        torch.cuda.synchronize()
        assert torch.equal(one.cpu(), host_out[l]), f"layer {l}: sharded != single call"
        q, k = oracle.c_qk_norm_rope(x, qw, kw, cu)
        ref = oracle.c_attention(q.astype(np.float16), k.astype(np.float16), x, 4096, 3072, cu)
        got = host_out[l].numpy().astype(np.float64)
        assert np.abs(got - ref).max() <= 2e-3


def test_device_backend_rejects_nothing_for_an_idle_rank(pkg, cuda_dev):
    """A rank with no requests (4 requests over 8 devices) does no work."""
    ex = pkg.executor
    plan = ex.ShardPlan([40, 40, 40, 40], 8)
    idle = [r for r in range(8) if plan.local_tokens(r) == 0]
    assert len(idle) == 4
    be = ex.DeviceBackend(0, 0)
    try:
        shard = ex.ShardExecutor(plan, idle[0], be)
        shard.run([None], [None], [(None, None)])
        be.check()
    finally:
        be.close()


def test_multi_device_executor_on_two_gpus(pkg, oracle, cuda_dev):
    """The same split over two real devices (skipped on a one-GPU box)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ex = pkg.executor
    lengths = [700, 17, 1300, 64, 5]
    cu = [0] + list(np.cumsum(lengths))
    T = cu[-1]
    layers = _layers(T, 2, seed=3)
    host_in = [torch.from_numpy(x).pin_memory() for x, _, _ in layers]
    host_out = [torch.zeros(T, 16, 128, dtype=torch.float16).pin_memory() for _ in range(2)]
    m = ex.MultiDeviceExecutor(lengths, [0, 1])
    try:
        m.set_weights([(qw, kw) for _, qw, kw in layers])
        m.run(host_in, host_out)
    finally:
        m.close()
    for l, (x, qw, kw) in enumerate(layers):
        q, k = oracle.c_qk_norm_rope(x, qw, kw, cu)
        ref = oracle.c_attention(q.astype(np.float16), k.astype(np.float16), x, 4096, 3072, cu)
        assert np.abs(host_out[l].numpy().astype(np.float64) - ref).max() <= 2e-3


def test_auto_mode_is_resolved_on_the_whole_batch(pkg, oracle, cuda_dev):
    """A 9000-token request makes the reference's AUTO rule pick full causal for
    the whole batch (ops.ts:328). The shard that holds only the 1000-token
    request must run full causal too (on its own it would pick the sparse
    rule, which drops keys of rows past 608)."""
    ex = pkg.executor
    lengths = [9000, 1000]
    plan = ex.ShardPlan(lengths, 2)
    assert plan.resolved_mode == ex.MODE_FULL
    assert sorted(len(r) for r in plan.assignment) == [1, 1]
    cu = [0, 9000, 10000]
    layers = _layers(10000, 1, seed=9)
    host_in = [torch.from_numpy(layers[0][0]).pin_memory()]
    host_out = [torch.zeros(10000, 16, 128, dtype=torch.float16).pin_memory()]
    m = ex.MultiDeviceExecutor(lengths, [0, 0])
    try:
        m.set_weights([(layers[0][1], layers[0][2])])
        m.run(host_in, host_out)
    finally:
        m.close()
    x, qw, kw = layers[0]
    one = pkg.attention.prefill_attention_layer(torch.from_numpy(x).to(cuda_dev),
                                                torch.from_numpy(qw).to(cuda_dev),
                                                torch.from_numpy(kw).to(cuda_dev), cu)
    torch.cuda.synchronize()
    assert torch.equal(one.cpu(), host_out[0])
    # rows of the short request past 608 against the full-causal oracle
    q, k = oracle.c_qk_norm_rope(x, qw, kw, cu)
    rows = np.array([(9000 + t) * 16 + h for t in (0, 607, 608, 700, 999) for h in (0, 5, 15)])
    ref = oracle.c_attention_rows(q.astype(np.float16), k.astype(np.float16), x, 4096, 3072, cu,
                                  rows, 1)
    got = host_out[0].view(-1, 128)[torch.from_numpy(rows)].numpy().astype(np.float64)
    assert np.abs(got - ref).max() <= 2e-3
