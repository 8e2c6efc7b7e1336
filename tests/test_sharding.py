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


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, result_path):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import oracle
    pkg = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lengths = [7, 40, 3, 25, 12]
    mode, prefix, window = 2, 5, 11
    rng = np.random.default_rng(99)  # same batch on every rank
    cu = [0] + list(np.cumsum(lengths))
    qkv = rng.standard_normal((cu[-1], 4096)).astype(np.float16)
    assignment = pkg.sharding.lpt_shard(lengths, world, mode)
    mine = assignment[rank]
    # each rank computes only its requests (here with the oracle standing in
    # for the device) and the host gathers per-rank outputs
    sub_cu = [0] + list(np.cumsum([lengths[i] for i in mine]))
    rows = np.concatenate([np.arange(cu[i], cu[i + 1]) for i in mine]) if mine else np.zeros(0, int)
    q = qkv[rows, :2048].reshape(-1, 16, 128).copy()
    k = qkv[rows, 2048:3072].reshape(-1, 8, 128).copy()
    out = oracle.c_attention(q, k, qkv[rows].copy(), 4096, 3072, sub_cu, mode, prefix, window)
    per_req = [out[sub_cu[n]:sub_cu[n + 1]] for n in range(len(mine))]
    gathered = [None] * world
    dist.all_gather_object(gathered, per_req)
    if rank == 0:
        flat = [r for part in gathered for r in part]
        order = pkg.sharding.gather_order(assignment)
        full = np.concatenate([flat[j] for j in order])
        ref = oracle.c_attention(qkv[:, :2048].reshape(-1, 16, 128).copy(),
                                 qkv[:, 2048:3072].reshape(-1, 8, 128).copy(), qkv, 4096, 3072,
                                 cu, mode, prefix, window)
        np.save(result_path, np.abs(full - ref).max())
    dist.destroy_process_group()


def test_two_rank_shard_and_host_gather(tmp_path, pkg):
    path = str(tmp_path / "err.npy")
    mp.spawn(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True)
    assert float(np.load(path)) < 1e-12
