"""The CPU oracle against the reference's own test oracle (no GPU).

Pins: the committed golden vectors (tests/golden/make_golden.py: gguf-py 0.19.0 dequantize, and the numpy Q2_0
decoder of strata-mlx tests/test_gguf.py:33-38), and gguf-py itself on the reference's random_tensor shapes.
"""

import os

import numpy as np
import pytest

from oracle import blocks_ref as R
from tests.golden.make_golden import KINDS, gguf_reference, random_blocks

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz")


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_oracle_is_the_golden_vectors_bit_for_bit(kind):
    g = np.load(GOLDEN)
    rows, cols = int(g["rows"]), int(g["cols"])
    got = R.dequantize(g[f"{kind}_blocks"], kind, (rows, cols))
    want = g[f"{kind}_weights"]
    assert got.dtype == np.float32 and got.shape == want.shape
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_oracle_is_gguf_py_on_the_reference_test_shapes(kind):
    """strata-mlx tests/test_blocks.py:13-19 asks 1e-6 of the largest weight; the restatement gives every bit."""
    rows, cols = 6, 2560
    data = random_blocks(kind, seed=7, rows=rows, cols=cols)
    want = gguf_reference(kind, data, rows, cols)
    got = R.dequantize(data, kind, (rows, cols))
    assert np.abs(got - want).max() <= 1e-6 * np.abs(want).max()
    assert (got.view(np.uint32) != want.view(np.uint32)).sum() == 0


def test_block_table_is_the_references():
    assert R.BLOCK == {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
                       "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56),
                       "Q2_0": (64, 18), "Q3_K": (256, 110)}
    with pytest.raises(ValueError):
        R.row_bytes("IQ3_S", 640)  # a row of 640 does not end on a block of 256


def test_top_k_takes_the_lower_index_on_ties():
    logits = np.array([[1.0, 3.0, 3.0, 2.0, 3.0, 0.5]], dtype=np.float32)
    np.testing.assert_array_equal(R.top_k(logits, 4), [[1, 2, 4, 3]])


def test_softmax_over_the_chosen_logits_sums_to_one():
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((3, 64)).astype(np.float32)
    idx = R.top_k(lg, 10)
    w = R.softmax_topk(lg, idx)
    np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-6)
    assert (np.diff(w, axis=-1) <= 0).all()


def test_combine_adds_in_mlxs_order():
    """Eight partial sums (partial j takes k = j, j+8, ...) then in order: k = 10 makes the order visible."""
    y = np.zeros((1, 10, 1), dtype=np.float32)
    y[0, :, 0] = [1e8, 1, 1, 1, 1, 1, 1, 1, -1e8, 1]
    w = np.ones((1, 10), dtype=np.float32)
    out = R.moe_combine(y, w, np.full(1, -np.inf, np.float32), np.zeros((1, 1), np.float32), np.float32)
    # partial 0 = y0 + y8 = 0, partial 1 = y1 + y9 = 2, partials 2..7 = 1 each: 8 in all
    assert out[0, 0] == 8.0


def test_bfloat16_rounding_is_to_nearest_even():
    v = np.array([1.0 + 2**-8, 1.0 + 3 * 2**-8, -1.0 - 2**-8], dtype=np.float32)
    np.testing.assert_array_equal(R.round_to(v, "bfloat16"), np.array([1.0, 1.0 + 2**-6, -1.0], dtype=np.float32))


def test_swiglu_rounds_as_mlx_lm():
    g = np.array([0.5, -2.0, 3.0], dtype=np.float32)
    u = np.array([1.0, 0.25, -1.5], dtype=np.float32)
    got = R.swiglu(g, u, np.float32)
    np.testing.assert_allclose(got, g / (1 + np.exp(-g)) * u, rtol=1e-6)
