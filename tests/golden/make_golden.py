"""Generate the golden fixtures for the attention hot path.

Run from the repository root:  python tests/golden/make_golden.py

Inputs are seeded f16 ~N(0,1) qkv activations and 1+N(0,0.02) norm weights;
expected outputs come from the numpy restatement of the reference's shader
math (oracle/oracle.py np_* functions, fp64) and are stored as f16 (normed+roped q/k, the
layout the kernels must produce) and float32 (attention output).
The reference itself cannot produce them: its path exists only as WGSL for a
browser WebGPU, unavailable here. tests/test_golden.py checks that the C
oracle reproduces these files; the GPU tests compare the kernels to them.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # one request, 50 tokens, full causal (sparse rule no-op)
    "c1_single_50": dict(lengths=[50], mode=0, prefix=176, window=432, seed=11),
    # ragged micro-batch incl. an empty request; sparse with a small
    # prefix/window so prefix + window tiles and both mask edges are exercised
    "ragged_sparse_small": dict(lengths=[1, 30, 0, 13], mode=2, prefix=6, window=10, seed=12),
}


def make(name, lengths, mode, prefix, window, seed):
    rng = np.random.default_rng(seed)
    cu = np.array([0] + list(np.cumsum(lengths)), dtype=np.int32)
    T = int(cu[-1])
    qkv = rng.standard_normal((T, 4096), dtype=np.float32).astype(np.float16)
    qw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    q, k = oracle.np_qk_norm_rope(qkv, qw, kw, cu)
    q16, k16 = q.astype(np.float16), k.astype(np.float16)
    out = oracle.np_attention(q16, k16, qkv, 4096, 3072, cu, mode, prefix, window)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), qkv=qkv, q_weight=qw, k_weight=kw,
                        cu_seqlens=cu, mode=mode, prefix=prefix, window=window,
                        q16=q16, k16=k16, out=out.astype(np.float32))


if __name__ == "__main__":
    for n, c in CASES.items():
        make(n, **c)
        print("wrote", n)
