"""Request sharding across ranks (host logic; world_size 2 over gloo on CPU)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def test_kept_pairs_closed_form_matches_mask(pkg, oracle):
    for L in (1, 100, 608, 609, 1500):
        for sparse in (False, True):
            assert pkg.sharding.kept_pairs(L, sparse) == int(oracle.keep_mask(L, sparse).sum())


def test_lpt_balances_and_covers(pkg):
    lengths = list(pkg.workloads.WORKLOADS["c2_ragged16"].lengths)
    for world in (1, 2, 4, 8):
        a = pkg.sharding.lpt_shard(lengths, world)
        assert sorted(i for r in a for i in r) == list(range(len(lengths)))
        loads = [sum(pkg.sharding.kept_pairs(lengths[i], True) for i in r) for r in a]
        assert max(loads) <= 1.5 * (sum(loads) / world) + max(
            pkg.sharding.kept_pairs(L, True) for L in lengths)
    even = pkg.sharding.lpt_shard([5000] * 16, 8)
    assert all(len(r) == 2 for r in even)


def test_gather_order_restores_batch(pkg):
    a = [[0, 3], [1], [2, 4]]
    flat = [i for r in a for i in r]
    order = pkg.sharding.gather_order(a)
    assert [flat[j] for j in order] == [0, 1, 2, 3, 4]


def test_shard_plan_rows_and_mode(pkg):
    ex = pkg.executor
    plan = ex.ShardPlan([7, 40, 0, 3, 25, 12], 3, mode=0)
    rows = []
    for r in range(3):
        local = 0
        for g, l0, n in plan.row_ranges(r):
            assert l0 == local
            rows.extend(range(g, g + n))
            local += n
        assert local == plan.local_tokens(r)
    assert sorted(rows) == list(range(plan.total_tokens))
    # one rank holds every request: its rows form a single run
    assert ex.ShardPlan([5, 6, 7], 1).row_ranges(0) == [(0, 0, 18)]
    # AUTO is resolved on the whole batch: a rank holding only a short request
    # still runs full causal when another request exceeds 8192 tokens
    p = ex.ShardPlan([9000, 20], 2, mode=0)
    assert p.resolved_mode == ex.MODE_FULL
    assert ex.ShardPlan([8192, 20], 2).resolved_mode == ex.MODE_SPARSE
    assert ex.ShardPlan([20], 4).local_tokens(3) == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _OracleBackend:
    """The CPU oracle in place of the device, for the executor's host logic."""
    buffers = 1

    def __init__(self, oracle, tokens):
        self.o = oracle
        self.x = np.zeros((tokens, 4096), np.float16)
        self.out = None

    def stage_in(self, b, ranges, host):
        for g, l0, n in ranges:
            self.x[l0:l0 + n] = host[g:g + n]

    def compute(self, b, cu, weights, mode, prefix, window):
        q, k = self.o.c_qk_norm_rope(self.x, weights[0], weights[1], cu)
        self.out = self.o.c_attention(q.astype(np.float16), k.astype(np.float16), self.x, 4096,
                                      3072, cu, mode, prefix, window).astype(np.float16)

    def stage_out(self, b, ranges, host):
        for g, l0, n in ranges:
            host[g:g + n] = self.out[l0:l0 + n]

    def finish(self):
        return None


LENGTHS, LAYERS = [7, 40, 3, 0, 25, 12], 2


def _rank_main(rank, world, port, tmp):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import oracle
    pkg = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200")
    ex = pkg.executor
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    plan = ex.ShardPlan(LENGTHS, world, mode=2)
    T = plan.total_tokens
    # host buffers shared by the ranks: rank 0 creates them, the others map them
    names = [f"{tmp}/in{l}" for l in range(LAYERS)] + [f"{tmp}/out{l}" for l in range(LAYERS)]
    shapes = [(T, 4096)] * LAYERS + [(T, 16, 128)] * LAYERS
    if rank == 0:
        bufs = [ex.SharedHostBuffer(n, s, create=True, pin=False) for n, s in zip(names, shapes)]
        rng = np.random.default_rng(99)
        for l in range(LAYERS):
            bufs[l].array[:] = rng.standard_normal((T, 4096)).astype(np.float16)
        dist.barrier()
    else:
        dist.barrier()
        bufs = [ex.SharedHostBuffer(n, s, pin=False) for n, s in zip(names, shapes)]
    wrng = np.random.default_rng(5)
    weights = [tuple((1 + 0.02 * wrng.standard_normal(128)).astype(np.float32) for _ in range(2))
               for _ in range(LAYERS)]
    # assign -> compute (oracle in place of the device) -> gather into the
    # shared host output at each request's rows
    executor = ex.ShardExecutor(plan, rank, _OracleBackend(oracle, plan.local_tokens(rank)),
                                prefix=5, window=11)
    executor.run([b.array for b in bufs[:LAYERS]], [b.array for b in bufs[LAYERS:]], weights)
    dist.barrier()
    if rank == 0:
        errs = []
        for l in range(LAYERS):
            x = bufs[l].array
            q, k = oracle.c_qk_norm_rope(x, weights[l][0], weights[l][1], plan.cu)
            ref = oracle.c_attention(q.astype(np.float16), k.astype(np.float16), x, 4096, 3072,
                                     plan.cu, 2, 5, 11).astype(np.float16)
            errs.append(float(np.abs(bufs[LAYERS + l].array.astype(np.float64) - ref).max()))
        np.save(f"{tmp}/err.npy", np.array(errs))
    dist.barrier()
    for b in bufs:
        b.close()
    dist.destroy_process_group()


def test_two_rank_executor_shards_and_gathers(tmp_path, pkg):
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    errs = np.load(str(tmp_path / "err.npy"))
    assert errs.shape == (LAYERS,) and float(errs.max()) == 0.0
