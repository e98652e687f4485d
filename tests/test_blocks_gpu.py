"""The block kernels against the CPU oracle on the same seeded bytes (ported from strata-mlx tests/test_blocks.py)."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200.synthetic import blocks_numpy
from tests.golden.make_golden import KINDS, random_blocks

pytestmark = pytest.mark.gpu
EXPERTS, OUT = 3, 2  # the reference's test tensors: 6 rows of 2560, three experts of two rows


def dev(a, d="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(d)


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_dequant_is_the_oracle_bit_for_bit(cuda, kind):
    g = np.load("tests/golden/dequant_golden.npz")
    rows, cols = int(g["rows"]), int(g["cols"])
    got = B.dequantize(dev(g[f"{kind}_blocks"]), kind, (rows, cols)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), g[f"{kind}_weights"].view(np.uint32))
    data = random_blocks(kind, seed=3, rows=6, cols=2560)  # the reference's random_tensor shape
    want = R.dequantize(data, kind, (6, 2560))
    got = B.dequantize(dev(data), kind, (6, 2560)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    for dt, nd in ((torch.float16, np.float16), (torch.bfloat16, "bfloat16")):
        got = B.dequantize(dev(data), kind, (2, 3, 2560), dt).float().cpu().numpy().reshape(6, 2560)
        np.testing.assert_array_equal(got, R.round_to(want, nd))


def test_dequant_config1_expert(cuda):
    """Config 1: one IQ3_S SwiGLU expert, gate/up 2048->512, down 512->2048, d ~ N(0, 0.02)."""
    rng = np.random.default_rng(0)
    for rows, cols in ((512, 2048), (2048, 512)):
        data = blocks_numpy("IQ3_S", 1, rows, cols, rng)
        want = R.dequantize(data, "IQ3_S", (rows, cols))
        got = B.dequantize(dev(data), "IQ3_S", (1, rows, cols)).cpu().numpy()[0]
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def stack(kind, seed, experts, rows, cols, uniform=0.05):
    rng = np.random.default_rng(seed)
    data = blocks_numpy(kind, experts, rows, cols, rng, uniform=uniform)
    return data, R.dequantize(data, kind, (experts, rows, cols))


@pytest.mark.parametrize("kind", sorted(B.BLOCK))
@pytest.mark.parametrize("per_row", [1, 4, 16])
def test_products_on_blocks_are_products_on_the_weights(cuda, kind, per_row):
    """strata-mlx tests/test_blocks.py:22-39: both layouts, a row to each token (gate/up) and to each pair (down)."""
    data, w = stack(kind, 1, EXPERTS, OUT, 2560)
    layer = B.BlockSwitchLinear(dev(data), kind, w.shape, per_row=per_row)
    rng = np.random.default_rng(2)
    idx = np.array([[2, 0], [1, 1], [0, 2], [2, 2], [0, 1]])
    scale = np.abs(w).max() * np.sqrt(w.shape[-1])
    x = rng.standard_normal((5, 1, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx)).cpu().numpy()
    assert got.shape == (5, 2, 1, OUT)
    assert np.abs(got[:, :, 0] - np.einsum("tkoi,ti->tko", w[idx], x[:, 0, 0])).max() <= 1e-5 * scale
    x = rng.standard_normal((5, 2, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx)).cpu().numpy()
    assert np.abs(got[:, :, 0] - np.einsum("tkoi,tki->tko", w[idx], x[:, :, 0])).max() <= 1e-5 * scale
    _lib.check_device_errors()


@pytest.mark.parametrize("kind", ["IQ4_NL", "IQ2_S", "Q2_0", "IQ3_S"])
@pytest.mark.parametrize("unpacked", [False, True])
def test_a_prompt_gets_the_same_products_a_pair_at_a_time_and_from_unpacked_weights(cuda, kind, unpacked):
    data, w = stack(kind, 3, EXPERTS, OUT, 2560)
    layer = B.BlockSwitchLinear(dev(data), kind, w.shape)
    layer.unpack_from = 100 if unpacked else 1000
    rng = np.random.default_rng(4)
    idx = np.sort(rng.integers(0, EXPERTS, 200))
    x = rng.standard_normal((200, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx), sorted_indices=True).cpu().numpy()
    assert got.shape == (200, 1, OUT)
    scale = np.abs(w).max() * np.sqrt(w.shape[-1])
    assert np.abs(got[:, 0] - np.einsum("noi,ni->no", w[idx], x[:, 0])).max() <= 1e-5 * scale


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_half_precision_activations_come_back_as_half(cuda, dt):
    data, w = stack("IQ3_XXS", 5, EXPERTS, OUT, 2560)
    layer = B.BlockSwitchLinear(dev(data), "IQ3_XXS", w.shape)
    x = torch.randn((2, 1, 1, 2560), device="cuda").to(dt)
    idx = dev(np.array([[0, 1], [2, 0]]))
    out = layer(x, idx)
    assert out.dtype == dt and out.shape == (2, 2, 1, OUT)
    want = layer(x.float(), idx)
    assert (out.float() - want).abs().max().item() <= 2e-3 * want.abs().max().item() * (4 if dt == torch.bfloat16 else 1)


@pytest.mark.parametrize("kind, rows, cols", [("Q2_0", 512, 2048), ("IQ3_S", 512, 2048), ("IQ3_XXS", 2048, 512),
                                              ("IQ3_S", 2048, 512), ("Q2_0", 2048, 512), ("IQ4_XS", 640, 2560)])
def test_decode_shapes_of_the_benchmark(cuda, kind, rows, cols):
    """Config-2 shapes, 512 experts, top-10 for 1 and 5 tokens: within 2e-3 of float64 sums of the exact weights."""
    experts = 64
    rng = np.random.default_rng(rows + cols)
    data = blocks_numpy(kind, experts, rows, cols, rng)
    w = R.dequantize(data, kind, (experts, rows, cols))
    layer = B.BlockSwitchLinear(dev(data), kind, (experts, rows, cols))
    for tokens in (1, 5):
        idx = np.stack([rng.choice(experts, 10, replace=False) for _ in range(tokens)])
        x = rng.standard_normal((tokens, 1, 1, cols)).astype(np.float32)
        got = layer(dev(x), dev(idx)).cpu().numpy()[:, :, 0]
        want = np.einsum("tkoi,ti->tko", w[idx].astype(np.float64), x[:, 0, 0].astype(np.float64))
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()
        assert np.abs(got - want).max() <= 1e-5 * np.abs(w).max() * np.sqrt(cols)


def test_matvec_separate_and_window(cuda):
    data, w = stack("IQ3_S", 9, 4, 64, 512)
    per = 64 * 512 // 256 * 110
    experts = [dev(data[e * per : (e + 1) * per]) for e in (3, 1, 3)]
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 512)).astype(np.float32)
    got = B.matvec_separate(experts, "IQ3_S", 64, 512, dev(x), 3).cpu().numpy()
    want = np.stack([w[e] @ x[0] for e in (3, 1, 3)])
    assert np.abs(got - want).max() <= 1e-5 * np.abs(w).max() * np.sqrt(512)
    xs = rng.standard_normal((6, 512)).astype(np.float32)
    got = B.window_matvec(dev(data[:per]), "IQ3_S", 64, 512, dev(xs)).cpu().numpy()
    assert np.abs(got - xs @ w[0].T).max() <= 1e-5 * np.abs(w).max() * np.sqrt(512)
    alone = torch.cat([B.window_matvec(dev(data[:per]), "IQ3_S", 64, 512, dev(xs[t : t + 1])) for t in range(6)])
    assert torch.equal(alone.cpu(), torch.from_numpy(got))  # a token's sums do not depend on the window


@pytest.mark.parametrize("kind", ["IQ3_S", "IQ2_XS", "IQ4_NL", "Q2_0"])
@pytest.mark.parametrize("tokens", [1, 20])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_down_taking_swiglu_itself_and_unsorted_pairs_give_the_same_bits(cuda, monkeypatch, kind, tokens, dt):
    """strata-mlx tests/test_blocks.py:232-255, and the fused gate/up kernel against separate products."""
    monkeypatch.setattr(B, "MATVEC_GLU_UPTO", 1 << 20)
    monkeypatch.setattr(B, "LOOKUP_FROM", 1 << 62)
    rng = np.random.default_rng(tokens)

    def experts(rows, cols):
        return B.BlockSwitchLinear(dev(blocks_numpy(kind, 6, rows, cols, rng, uniform=0.05)), kind, (6, rows, cols))

    gate, up, down = experts(256, 512), experts(256, 512), experts(512, 256)
    x = dev((0.01 * rng.standard_normal((1, tokens, 512))).astype(np.float32)).to(dt)
    idx = dev(np.stack([rng.choice(6, 4, replace=False) for _ in range(tokens)])[None].astype(np.int32))
    got = B.switch_glu(x, idx, up, gate, down)  # fused gate/up kernel
    x5 = x.unsqueeze(-2).unsqueeze(-2)
    g, u = gate(x5, idx), up(x5, idx)
    flat = idx.reshape(-1)
    glu = B.matvec_glu(down, flat, g.reshape(flat.numel(), -1), u.reshape(flat.numel(), -1)).reshape(got.shape)
    monkeypatch.setattr(B, "BLOCK_GLU", False)
    want = B.switch_glu(x, idx, up, gate, down)
    assert got.shape == want.shape == glu.shape
    assert torch.equal(got, want) and torch.equal(glu, want)
    assert torch.isfinite(want.float()).float().mean().item() > 0.9


@pytest.mark.parametrize("pairs", [1, 10, 30])
@pytest.mark.parametrize("rows, cols", [(256, 640), (96, 128), (40, 2048)])
def test_the_glu_table_built_in_down_gives_the_bits_of_its_own_kernel(cuda, pairs, rows, cols):
    """strata-mlx tests/test_blocks.py:215-229."""
    rng = np.random.default_rng(pairs + rows)
    blocks = rng.integers(0, 256, (EXPERTS * rows * cols // 64, 18), dtype=np.uint8)
    blocks[:, :2] = rng.uniform(-0.05, 0.05, (len(blocks), 1)).astype("<f2").view(np.uint8)
    down = B.BlockSwitchLinear(dev(blocks.reshape(-1)), "Q2_0", (EXPERTS, rows, cols))
    idx = dev(rng.integers(0, EXPERTS, pairs).astype(np.int32))
    gate = dev(rng.standard_normal((pairs, cols)).astype(np.float16))
    up = dev(rng.standard_normal((pairs, cols)).astype(np.float16))
    got = B.lookup_down_glu(down, idx, gate, up)
    assert got is not None and got.dtype == torch.float16
    assert torch.equal(got, B.lookup_matvec(down, idx, B.lookup_table_glu(gate, up), 1))


def test_a_bad_expert_id_is_recorded_not_trapped(cuda):
    data, w = stack("Q2_0", 1, EXPERTS, 4, 128)
    layer = B.BlockSwitchLinear(dev(data), "Q2_0", w.shape)
    _lib.check_device_errors()
    out = layer(torch.ones((2, 1, 1, 128), device="cuda"), dev(np.array([[0, 1], [7, 2]])))
    with pytest.raises(_lib.StrataError, match="SC_ERR_INDEX"):
        _lib.check_device_errors()
    good = out[0].cpu().numpy()[:, 0]
    np.testing.assert_allclose(good, w[[0, 1]].sum(-1), rtol=1e-5, atol=1e-6)
