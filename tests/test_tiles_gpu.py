"""Prefill: tiles_of and the tile product against the oracle (ported from strata-mlx tests/test_blocks.py:97-212)."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import blocks as B
from strata_mlx_b200.synthetic import blocks_numpy

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stack(kind, rng, experts, rows, cols):
    data = blocks_numpy(kind, experts, rows, cols, rng, uniform=0.01)
    return dev(data), R.dequantize(data, kind, (experts, rows, cols))


@pytest.mark.parametrize("tokens, k, experts", [(211, 3, 7), (5, 2, 40), (64, 10, 512), (1, 1, 3), (2048, 10, 512)])
def test_tiles_hold_every_pair_with_its_expert(cuda, tokens, k, experts):
    rng = np.random.default_rng(tokens)
    idx = rng.integers(0, experts, (1, tokens, k))
    idx[0, : tokens // 3] = 1
    if tokens >= 33 and experts > 4:
        idx[0, -33:, 0] = np.repeat([3, 4], [16, 17])
    te, token, where = (a.view(torch.int32).cpu().numpy() for a in B.tiles_of(dev(idx), experts))
    R.tiles_of_check(idx, experts, te, token, where)


@pytest.mark.parametrize("kind", sorted(B.BLOCK))
@pytest.mark.parametrize("dt, nd", [(torch.float16, np.float16), (torch.float32, np.float32), (torch.bfloat16, "bfloat16")])
def test_the_tile_product_is_the_product_with_the_weights(cuda, kind, dt, nd):
    rng = np.random.default_rng(0)
    shape = (4, 128, 512)
    blocks, w = stack(kind, rng, *shape)
    tiles = np.array([3, 0, 0, 2, 3])
    a32 = rng.standard_normal((16 * len(tiles), shape[2])).astype(np.float32)
    a = dev(a32).to(dt)
    got = B.tile_matmul(blocks, kind, shape, a, dev(tiles.astype(np.int32))).cpu().numpy()
    want = R.tile_matmul(w, a.float().cpu().numpy(), tiles, nd)
    assert got.shape == want.shape and got.dtype == np.float32
    assert np.abs(got - want).max() <= 2e-6 * np.abs(want).max()  # sums are float32


def test_a_tile_of_no_expert_is_left_out(cuda):
    rng = np.random.default_rng(3)
    blocks, w = stack("Q2_0", rng, 4, 128, 192)
    tiles = np.array([1, 4, 2, 9])
    a = rng.standard_normal((16 * len(tiles), 192)).astype(np.float16)
    out = torch.full((64, 128), 7.0, device="cuda")
    got = B.tile_matmul(blocks, "Q2_0", (4, 128, 192), dev(a), dev(tiles.astype(np.int32))).cpu().numpy()
    for t in (0, 2):
        want = a[16 * t : 16 * t + 16].astype(np.float64) @ R.round_to(w[tiles[t]], np.float16).astype(np.float64).T
        assert np.abs(got[16 * t : 16 * t + 16] - want).max() <= 2e-6 * np.abs(want).max()


def test_what_fits_in_tiles():
    assert B.tileable("Q2_0", 640, 2560) and B.tileable("IQ3_S", 640, 2560) and B.tileable("IQ4_NL", 2560, 640)
    assert not B.tileable("IQ3_S", 2560, 640)
    assert not B.tileable("Q2_0", 2, 2560)


@pytest.mark.parametrize("kinds", [("Q2_0", "Q2_0"), ("IQ3_S", "IQ4_NL"), ("IQ2_S", "Q2_0")])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_a_prompt_through_tiles_is_the_prompt_a_pair_at_a_time(cuda, monkeypatch, kinds, dt):
    """strata-mlx tests/test_blocks.py:112-174: switch_glu sends a chunk's pairs through the tiles, and what
    comes out is what a pair at a time gives."""
    rng = np.random.default_rng(1)
    experts, hidden, inner, k = 7, 256, 64, 3
    lins, ws = {}, {}
    for name, kind, (rows, cols) in (("gate", kinds[0], (inner, hidden)), ("up", kinds[0], (inner, hidden)),
                                     ("down", kinds[1], (hidden, inner * 4))):
        b, w = stack(kind, rng, experts, rows, cols)
        lins[name], ws[name] = B.BlockSwitchLinear(b, kind, (experts, rows, cols)), w
    rows_ = 211
    x = dev(rng.standard_normal((1, rows_, hidden)).astype(np.float32)).to(dt)
    idx = rng.integers(0, experts - 1, (1, rows_, k))
    idx[0, :40] = 2
    t, token, where = B.tiles_of(dev(idx), experts)
    a = x.reshape(-1, hidden).index_select(0, token.to(torch.int64))
    xs = x.float().cpu().numpy()[0].astype(np.float64)
    nd = {torch.float16: np.float16, torch.bfloat16: "bfloat16", torch.float32: np.float32}[dt]
    for name in ("gate", "up"):
        lin = lins[name]
        got = B.tile_matmul(lin.blocks, lin.kind, (experts, inner, hidden), a, t)
        got = got.index_select(0, where.to(torch.int64)).reshape(rows_, k, inner).cpu().numpy()
        # the weights rounded to the activations' type multiply (blocks.py:492): float32 sums of those
        rounded = np.einsum("tkoi,ti->tko", R.round_to(ws[name], nd).astype(np.float64)[idx[0]], xs)
        assert np.abs(got - rounded).max() <= 2e-5 * np.abs(rounded).max()
        # and against the exact weights, the rounding of the type (bfloat16 keeps 8 bits, float16 11)
        want = np.einsum("tkoi,ti->tko", ws[name][idx[0]], xs)
        tol = {torch.float16: 2e-3, torch.bfloat16: 1e-2, torch.float32: 2e-5}[dt]
        assert np.abs(got - want).max() <= tol * np.abs(want).max()
