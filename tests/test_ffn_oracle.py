"""The Q6_K / SwiGLU oracle (no GPU): the reference's known answer and the
vectorised form against the block-by-block restatement."""
import numpy as np

from oracle import ffn


def test_q6k_centered_block_known_answer():
    # tests/quantization.test.ts:35-42 of the reference
    block = np.zeros(210, np.uint8)
    block[192:208] = 1
    block[208:210] = np.array([0x3c00], "<u2").view(np.uint8)
    assert np.all(ffn.dequant_q6k_block(block) == -32.0)
    assert np.all(ffn.dequant_q6k(block, 1, 256) == -32.0)
    assert np.all(ffn.embedding_lookup_f16([0], block, 1, 256) == -32.0)


def test_q6k_vectorised_matches_block_restatement(pkg):
    rng = np.random.default_rng(2)
    table = pkg.prepacked.random_q6k_rows(rng, 3, 512)
    full = ffn.dequant_q6k(table, 3, 512)
    blocks = table.reshape(6, 210)
    for i in range(6):
        assert np.array_equal(full.reshape(6, 256)[i], ffn.dequant_q6k_block(blocks[i]))
    f16 = ffn.embedding_lookup_f16([2, 0, 7], table, 3, 512)
    assert np.array_equal(f16[0], f16[0])
    assert np.all(np.abs(f16[:2].astype(np.float64) - full[[2, 0]])
                  <= np.spacing(np.abs(full[[2, 0]]).astype(np.float16)).astype(np.float64))
    assert np.all(f16[2] == 0)  # out-of-range id


def test_swiglu_values():
    c = np.array([[0.0, 1.0, -2.0, 3.0, 5.0, 7.0]], np.float16)
    out = ffn.swiglu(c, 3)
    assert out[0, 0] == 0.0
    assert np.isclose(out[0, 1], 1.0 / (1 + np.exp(-1.0)) * 5.0)
