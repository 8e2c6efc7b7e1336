"""The C-ABI library loads without a GPU and exports what include/qwa.h declares."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "qwa.h")).read()
    return sorted(set(re.findall(r"QWA_API\s+[\w\s\*]*?\b(qwa_\w+)\s*\(", text)))


def test_header_declares_expected_surface():
    syms = declared_symbols()
    for s in ["qwa_create", "qwa_destroy", "qwa_qk_norm_rope", "qwa_attention",
              "qwa_attention_padded", "qwa_prefill_attention_layer", "qwa_last_error"]:
        assert s in syms


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(pkg._lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # and the python binding covers the same surface
    assert set(declared_symbols()) == set(pkg._lib.SIGNATURES)


def test_library_links_no_cuda_shared_runtime(pkg):
    # cudart is static and the driver is resolved at run time, so the .so
    # loads on a machine without a GPU driver
    import subprocess
    out = subprocess.run(["ldd", pkg._lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


def test_status_strings_and_version(pkg):
    lib = pkg._lib.load()
    assert lib.qwa_version().startswith(b"qwa")
    assert lib.qwa_status_string(0) == b"ok"
    assert lib.qwa_status_string(4) == b"device wait timed out"


def test_create_without_device_fails_cleanly(pkg):
    import torch
    if torch.cuda.is_available():
        return
    h = ctypes.c_void_p()
    st = pkg._lib.load().qwa_create(0, ctypes.byref(h))
    assert st == pkg._lib.QWA_ERR_NO_DEVICE and not h.value


def test_attention_work_matches_closed_form(pkg):
    from oracle import oracle
    cu = [0, 5000, 5500, 5501, 7000]
    lens = np.diff(cu)
    for mode in (0, 1, 2):
        pairs, tiles = pkg.attention.attention_work(cu, mode)
        sparse = pkg.sharding.resolve_sparse(mode, list(lens))
        assert pairs == sum(pkg.sharding.kept_pairs(int(L), sparse) for L in lens)
        assert pairs == sum(oracle.c_kept_pairs(int(L), sparse) for L in lens)
        assert tiles > 0


def test_attention_work_rejects_bad_cu(pkg):
    lib = pkg._lib.load()
    a, b = ctypes.c_int64(), ctypes.c_int64()
    bad = (ctypes.c_int32 * 3)(0, 10, 5)  # decreasing
    assert lib.qwa_attention_work(bad, 2, 0, 176, 432, ctypes.byref(a), ctypes.byref(b)) == 1
    bad0 = (ctypes.c_int32 * 2)(3, 10)  # cu[0] != 0
    assert lib.qwa_attention_work(bad0, 1, 0, 176, 432, ctypes.byref(a), ctypes.byref(b)) == 1
    good = (ctypes.c_int32 * 2)(0, 10)
    assert lib.qwa_attention_work(good, 1, 0, 176, 0, ctypes.byref(a), ctypes.byref(b)) == 1
