"""The C oracle reproduces the committed golden fixtures (no GPU)."""
import glob
import os

import numpy as np
import pytest

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def test_fixtures_present():
    names = {os.path.basename(p) for p in GOLDEN}
    assert {"c1_single_50.npz", "ragged_sparse_small.npz"} <= names


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_oracle_reproduces_golden(oracle, path):
    g = np.load(path)
    cu = g["cu_seqlens"]
    q, k = oracle.c_qk_norm_rope(g["qkv"], g["q_weight"], g["k_weight"], cu)
    # stored q/k are the exact values rounded to f16: C oracle must round the same
    assert np.array_equal(q.astype(np.float16), g["q16"])
    assert np.array_equal(k.astype(np.float16), g["k16"])
    out = oracle.c_attention(g["q16"], g["k16"], g["qkv"], 4096, 3072, cu, int(g["mode"]),
                             int(g["prefix"]), int(g["window"]))
    assert np.abs(out - g["out"]).max() < 1e-6
