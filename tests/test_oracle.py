"""CPU oracle: pinned known answers and C-vs-numpy agreement (no GPU)."""
import numpy as np
import pytest


def test_half_kats(oracle):
    # tests/quantization.test.ts:5-9 of the reference (halfToFloat)
    assert oracle.c_half_to_float(0x3C00) == 1.0
    assert oracle.c_half_to_float(0xC000) == -2.0
    assert oracle.c_half_to_float(0x0000) == 0.0


def test_float_to_half_matches_numpy_rne(oracle):
    # floatToHalf (src/math/f16.ts:4-25) is round-to-nearest-even like numpy
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(2000) * 10.0 ** rng.integers(-6, 5, 2000),
                           [0.0, -0.0, 1.0, 65504.0, 65520.0, 1e-8, 6e-5, -3.14159]])
    vals = vals.astype(np.float32)
    ours = np.array([oracle.c_float_to_half(float(v)) for v in vals], dtype=np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_rope_table_c_vs_numpy(oracle):
    a = oracle.c_rope_table(1e6, 300)
    b = oracle.np_rope_table(1e6, 300)
    assert np.array_equal(a, b)
    assert np.all(a[0, :, 0] == 1.0) and np.all(a[0, :, 1] == 0.0)


def test_rope_position_zero_is_identity_and_rms_is_one(oracle):
    rng = np.random.default_rng(3)
    qkv = rng.standard_normal((1, 4096)).astype(np.float16)
    ones = np.ones(128, np.float32)
    q, k = oracle.c_qk_norm_rope(qkv, ones, ones, [0, 1])
    x = qkv[0, :2048].astype(np.float64).reshape(16, 128)
    n = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6)
    assert np.allclose(q[0], n, atol=1e-12)
    assert np.allclose((q[0] ** 2).mean(-1), 1.0, atol=1e-5)


@pytest.mark.parametrize("lengths", [[50], [3, 17, 40], [1, 129, 0, 64]])
def test_prologue_c_vs_numpy(oracle, lengths):
    rng = np.random.default_rng(len(lengths))
    cu = [0] + list(np.cumsum(lengths))
    qkv = rng.standard_normal((cu[-1], 4096)).astype(np.float16)
    qw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    q1, k1 = oracle.c_qk_norm_rope(qkv, qw, kw, cu)
    q2, k2 = oracle.np_qk_norm_rope(qkv, qw, kw, cu)
    assert np.abs(q1 - q2).max() < 1e-12 and np.abs(k1 - k2).max() < 1e-12


@pytest.mark.parametrize("lengths,mode,prefix,window", [
    ([50], 0, 176, 432), ([3, 17, 40], 1, 176, 432), ([200, 90], 2, 20, 40),
    ([700], 0, 176, 432), ([1, 0, 33], 2, 5, 9)])
def test_attention_c_vs_numpy(oracle, lengths, mode, prefix, window):
    rng = np.random.default_rng(sum(lengths))
    cu = [0] + list(np.cumsum(lengths))
    T = cu[-1]
    q = rng.standard_normal((T, 16, 128)).astype(np.float16)
    k = rng.standard_normal((T, 8, 128)).astype(np.float16)
    v = rng.standard_normal((T, 4096)).astype(np.float16)
    a = oracle.c_attention(q, k, v, 4096, 3072, cu, mode, prefix, window)
    b = oracle.np_attention(q, k, v, 4096, 3072, cu, mode, prefix, window)
    assert np.abs(a - b).max() < 1e-10
    rows = np.arange(0, T * 16, 7)
    c = oracle.c_attention_rows(q, k, v, 4096, 3072, cu, rows, mode, prefix, window)
    assert np.abs(c - a.reshape(T * 16, 128)[rows]).max() < 1e-12


def test_attention_known_answers(oracle):
    # identical keys -> uniform softmax -> mean of kept values
    T = 700
    rng = np.random.default_rng(5)
    q = rng.standard_normal((T, 16, 128)).astype(np.float16)
    k = np.tile(rng.standard_normal((1, 8, 128)).astype(np.float16), (T, 1, 1))
    v = rng.standard_normal((T, 1024)).astype(np.float16)
    out = oracle.c_attention(q, k, v, 1024, 0, [0, T], oracle.MODE_SPARSE)
    vf = v.astype(np.float64)
    for qpos in (0, 1, 175, 607, 608, 699):
        m = oracle.keep_mask(T, True)[qpos]
        expect = vf[m].reshape(-1, 8, 128).mean(0)
        assert np.allclose(out[qpos, 0], expect[0], atol=1e-12)
        assert np.allclose(out[qpos, 15], expect[7], atol=1e-12)
    # query row 0 attends only to key 0
    assert np.allclose(out[0].reshape(8, 2, 128)[:, 0], vf[0].reshape(8, 128), atol=1e-12)


@pytest.mark.parametrize("S", [1, 15, 16, 17, 176, 431, 432, 433, 607, 608, 609, 1500, 5000])
def test_mask_matches_wgsl_predicate_and_tile_skip(oracle, S):
    m = oracle.keep_mask(S, oracle.resolve_sparse(oracle.MODE_AUTO, S))
    qs = np.arange(S)
    for qp in sorted(set([0, S // 2, S - 1] + list(qs[:: max(1, S // 40)]))):
        lit = np.array([oracle.wgsl_keep(qp, kp, S) for kp in range(S)])
        assert np.array_equal(lit, m[qp])
    # the reference's 16-key block skip never drops a kept pair (ops.ts:209)
    for qt in range(0, S, 16):
        for kb in range(0, min(S, qt + 16), 16):
            if oracle.wgsl_block_skipped(kb, qt, S):
                assert not m[qt:qt + 16, kb:kb + 16].any()


def test_kept_pairs_counts(oracle):
    assert oracle.c_kept_pairs(500, True) == 500 * 501 // 2  # sparse is a no-op <= 608
    assert oracle.c_kept_pairs(5000, False) == 5000 * 5001 // 2
    assert 16 * oracle.c_kept_pairs(5000, True) == 45_687_552
    assert oracle.resolve_sparse(oracle.MODE_AUTO, 8192) and not oracle.resolve_sparse(0, 8193)


def test_last_token_pool_c_matches_numpy(oracle):
    rng = np.random.default_rng(11)
    h = rng.standard_normal((300, 1024)).astype(np.float16)
    cu = [0, 1, 1, 90, 300]
    a = oracle.c_last_token_pool(h, cu)
    b = oracle.np_last_token_pool(h, cu)
    assert np.abs(a - b).max() < 1e-12
    assert np.allclose(np.linalg.norm(a[[0, 2, 3]], axis=1), 1.0)
    assert not a[1].any()  # empty request -> zero row
    # the row pooled is the request's last one (ops.ts:351)
    x = h[89].astype(np.float64)
    assert np.allclose(a[2], x / np.linalg.norm(x))


def test_last_token_pool_padded_twin_matches_varlen(oracle):
    rng = np.random.default_rng(12)
    S, lengths = 40, [3, 40, 17]
    h = rng.standard_normal((len(lengths) * S, 64)).astype(np.float16)
    pad = oracle.np_last_token_pool_padded(h, lengths, S)
    rows = np.concatenate([h[b * S:b * S + n] for b, n in enumerate(lengths)])
    cu = np.concatenate([[0], np.cumsum(lengths)])
    assert np.abs(pad - oracle.c_last_token_pool(rows, cu)).max() < 1e-12


def test_rne_half_conversion_matches_numpy(oracle):
    import warnings
    rng = np.random.default_rng(21)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                           for s in (1e-8, 1e-6, 1e-4, 1.0, 100.0, 6e4)] +
                          [np.array([65504, 65519.99, 65520, 5.96e-8, 2.98e-8, 2.99e-8, 0.0,
                                     -0.0, np.inf, -np.inf], np.float32)])
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.lib().oracle_float_to_half_rne(float(v)) for v in vals], np.uint16)
    assert np.array_equal(ref, got)


@pytest.mark.parametrize("has_residual", [True, False])
def test_rms_norm_c_matches_numpy(oracle, has_residual):
    rng = np.random.default_rng(22)
    x = rng.standard_normal((40, 1024)).astype(np.float16)
    r = rng.standard_normal((40, 1024)).astype(np.float16) if has_residual else None
    w = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    cx, cn = oracle.c_rms_norm(x, r, w)
    nx, nn = oracle.np_rms_norm(x, r, w)
    assert np.array_equal(cx, nx) and np.array_equal(cn, nn)
    if not has_residual:
        assert np.array_equal(cx, x)
    # RMS of the normalized row (before the weight) is 1
    rms = np.sqrt(np.mean((cn.astype(np.float64) / w) ** 2, axis=1))
    assert np.allclose(rms, 1.0, atol=2e-3)


def _qkv(rng, lengths):
    cu = [0] + list(np.cumsum(lengths))
    T = cu[-1]
    q = rng.standard_normal((T, 16, 128)).astype(np.float16)
    k = rng.standard_normal((T, 8, 128)).astype(np.float16)
    v = rng.standard_normal((T, 1024)).astype(np.float16)
    return cu, q, k, v


@pytest.mark.parametrize("fused", [True, False])
def test_wgsl_mode_known_answers(oracle, fused):
    """The reference-arithmetic emulation (ops.ts:168-241 with its f16 rounding
    points): a one-token request returns its value row exactly; identical keys
    give the f16 mean of the kept values."""
    rng = np.random.default_rng(8)
    cu, q, k, v = _qkv(rng, [1, 40])
    out = oracle.c_attention_wgsl(q, k, v, 1024, 0, cu, fused)
    for h in range(16):
        assert np.array_equal(out[0, h], v[0, (h // 2) * 128:(h // 2 + 1) * 128].astype(np.float64))
    k[:] = k[0]
    out = oracle.c_attention_wgsl(q, k, v, 1024, 0, cu, fused)
    v2 = v[1:].astype(np.float64).reshape(40, 8, 128)
    for t in range(40):
        mean = v2[:t + 1].mean(0)
        for h in range(16):
            # f16 running sums of up to 40 values near N(0, 1)
            assert np.abs(out[1 + t, h] - mean[h // 2]).max() < 8e-3


@pytest.mark.parametrize("lengths", [[50], [16, 33, 130], [700]])
def test_wgsl_mode_is_close_to_exact_math(oracle, lengths):
    """The emulated reference stays within f16 accumulation error of the exact
    attention, including the sparse rule (700 > 608) and the block skip."""
    rng = np.random.default_rng(len(lengths))
    cu, q, k, v = _qkv(rng, lengths)
    ex = oracle.c_attention(q, k, v, 1024, 0, cu)
    for fused in (True, False):
        w = oracle.c_attention_wgsl(q, k, v, 1024, 0, cu, fused)
        assert np.abs(w - ex).max() < 1e-2
        a, b = w.reshape(-1, 128), ex.reshape(-1, 128)
        cos = (a * b).sum(1) / np.linalg.norm(a, axis=1) / np.linalg.norm(b, axis=1)
        assert cos.min() > 0.999
