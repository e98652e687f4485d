"""The C form of the oracle against the numpy oracle (no GPU): the same weights bit for bit, the same block."""

import numpy as np
import pytest

from oracle import blocks_ref as R
from oracle import cref
from strata_mlx_b200.synthetic import layer_numpy
from tests.golden.make_golden import KINDS, random_blocks


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_c_decoders_are_the_numpy_oracles_bit_for_bit(kind):
    data = random_blocks(kind, seed=11, rows=6, cols=2560)
    want = R.dequantize(data, kind, (6, 2560))
    got = cref.dequantize(data, kind, (6, 2560))
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kinds", [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "Q2_0")])
def test_c_moe_block_is_the_numpy_oracles(kinds):
    rng = np.random.default_rng(5)
    H, I, E, K = 512, 128, 32, 10
    L = layer_numpy(rng, H, I, E, kinds, shared_inter=128)
    W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)),
        ("sgate", kinds[0], (128, H)), ("sup", kinds[1], (128, H)), ("sdown", kinds[2], (H, 128)))}
    x = R.round_to(rng.standard_normal((2, H)).astype(np.float32), "bfloat16")
    want, widx, _ = R.moe_layer(x, L["router"], L["shared_gate"], W["gate"], W["up"], W["down"], W["sgate"],
                                W["sup"], W["sdown"], K, "bfloat16")
    got, idx, w = cref.Layer(L, H, I, E, K, "bfloat16", shared_inter=128)(x)
    np.testing.assert_array_equal(np.sort(idx, -1), np.sort(widx, -1))
    np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-6)
    assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()
