"""The C ABI from a C host program (tests/c/abi_layer.c): built with gcc against
include/qwa.h and libqwa.so, with no Python or torch in the process, its
prologue + attention layer is checked against the oracle."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_c_host_program(pkg, oracle, cuda_dev, tmp_path):
    libdir = os.path.dirname(pkg._lib.LIB_PATH)
    exe = str(tmp_path / "abi_layer")
    subprocess.run(["gcc", "-O2", "-std=c11", os.path.join(HERE, "c", "abi_layer.c"),
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
                    "-L", libdir, "-lqwa", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                    f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}",
                    "-o", exe], check=True)
    lengths = [700, 33, 1]
    cu = np.array([0] + list(np.cumsum(lengths)), np.int32)
    T = int(cu[-1])
    rng = np.random.default_rng(31)
    qkv = rng.standard_normal((T, 4096)).astype(np.float16)
    qw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    with open(tmp_path / "in.bin", "wb") as f:
        f.write(np.int32(len(lengths)).tobytes() + cu.tobytes() + qw.tobytes() + kw.tobytes()
                + qkv.tobytes())
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = np.fromfile(tmp_path / "out.bin", np.float16)
    q = out[:T * 2048].reshape(T, 16, 128)
    k = out[T * 2048:T * 3072].reshape(T, 8, 128)
    o = out[T * 3072:].reshape(T, 16, 128)
    q_ref, k_ref = oracle.c_qk_norm_rope(qkv, qw, kw, cu)
    assert np.abs(q.astype(np.float64) - q_ref).max() <= 2e-3
    assert np.abs(k.astype(np.float64) - k_ref).max() <= 2e-3
    o_ref = oracle.c_attention(q, k, qkv, 4096, 3072, cu)
    assert np.abs(o.astype(np.float64) - o_ref).max() <= 2e-3
