"""Dense layers on the file's forms (strata_mlx_b200/dense.py, load.py) against the weights gguf-py's dequantizer
and the oracle give, ported from the reference's tests/test_dense.py: Q6_K as codes, scales and d (ScaledLinear:
a window through the CUDA kernel, a prompt chunk through floats made once and kept), and layers and embeddings
kept as blocks (BlockLinear, BlockEmbedding)."""

import gguf
import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import dense
from strata_mlx_b200.dense import MAX_TOKENS, BlockEmbedding, BlockLinear, ScaledLinear, as_blocks
from strata_mlx_b200.gguf import Tensor
from strata_mlx_b200.load import AS_BLOCKS, embedding, linear
from strata_mlx_b200.synthetic import blocks_numpy

pytestmark = pytest.mark.gpu

ROWS, COLS = 12, 1024
TOL = {torch.float32: 2e-5, torch.float16: 4e-3, torch.bfloat16: 8e-3}  # the half types: outputs rounded to them


def q6k(seed: int = 0) -> Tensor:
    rng = np.random.default_rng(seed)
    n = ROWS * COLS // 256
    blocks = rng.integers(0, 256, (n, 210), dtype=np.uint8)
    blocks[:, 208:210] = rng.uniform(-0.01, 0.01, (n, 1)).astype("<f2").view(np.uint8)
    return Tensor("q6k", (ROWS, COLS), "Q6_K", blocks.reshape(-1))


def reference(t: Tensor) -> np.ndarray:
    return gguf.quants.dequantize(t.data.reshape(ROWS, -1), gguf.GGMLQuantizationType.Q6_K).reshape(t.shape)


def randn(shape, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 5, 7, 8, MAX_TOKENS + 4])
def test_a_window_multiplies_as_the_weights_do(cuda, tokens, dtype):
    t = q6k(tokens)
    lin = linear(t)
    assert isinstance(lin, ScaledLinear)
    x = randn((1, tokens, COLS), dtype, tokens)
    got = lin(x)
    assert got.shape == (1, tokens, ROWS) and got.dtype == dtype
    want = x.float().cpu().numpy().astype(np.float64) @ reference(t).astype(np.float64).T
    assert np.abs(got.float().cpu().numpy() - want).max() <= TOL[dtype] * np.abs(want).max()


def test_activations_at_an_odd_offset(cuda):
    lin = linear(q6k(9))
    x = randn((3 * COLS + 1,), torch.bfloat16, 8)[1:].reshape(3, COLS)  # contiguous, 2 bytes past 16
    assert torch.equal(lin(x), lin(x.contiguous().clone()))


@pytest.mark.parametrize("tokens", [1, 4, MAX_TOKENS + 4])
def test_reordered_outputs_and_inputs(cuda, tokens):
    t = q6k(7)
    rng = np.random.default_rng(1)
    rows = rng.permutation(ROWS)
    cols = (rng.permutation(COLS // 128)[:, None] * 128 + np.arange(128)).reshape(-1)  # heads of 128 change places
    lin = linear(t, rows=rows, cols=cols)
    assert lin.d_step == 128
    x = randn((tokens, COLS), torch.float32, 3)
    want = x.cpu().numpy().astype(np.float64) @ reference(t).astype(np.float64)[rows][:, cols].T
    assert np.abs(lin(x).cpu().numpy() - want).max() <= 2e-5 * np.abs(want).max()
    with pytest.raises(ValueError, match="splits a run"):
        linear(t, cols=rng.permutation(COLS))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_the_weights_as_floats_are_the_weights(cuda, dtype):
    t = q6k(3)
    rng = np.random.default_rng(2)
    cols = (rng.permutation(COLS // 128)[:, None] * 128 + np.arange(128)).reshape(-1)
    for lin, want in ((linear(t), reference(t)), (linear(t, cols=cols), reference(t)[:, cols])):
        got = lin.floats(dtype).float().cpu().numpy()
        if dtype == torch.float32:
            assert np.abs(got - want).max() <= 1e-6 * np.abs(want).max()
        else:  # rounded once from the float32 weight
            np.testing.assert_array_equal(got, torch.from_numpy(want).to(dtype).float().numpy())


def test_floats_made_for_a_prompt_are_kept(cuda):
    lin = linear(q6k(5))
    x = randn((MAX_TOKENS + 2, COLS), torch.float32, 5)
    first = lin(x)
    held = lin._floats
    assert held is not None and lin in dense._holding
    assert lin(x) is not None and lin._floats is held  # the second piece of the prompt: not made again
    lin(x[:2])  # a window: the kernel, which needs no floats
    dense.release()
    assert lin._floats is None and not dense._holding
    assert torch.equal(lin(x), first)
    dense.release()


def test_floats_not_kept_are_made_for_each_piece_and_let_go(cuda):
    kept, made = linear(q6k(5)), linear(q6k(5))
    made.keep = False
    x = randn((MAX_TOKENS + 2, COLS), torch.float32, 6)
    assert torch.equal(made(x), kept(x))
    assert made._floats is None and made not in dense._holding
    dense.release()


def test_a_shape_the_kernel_does_not_take_stays_floats(cuda):
    blocks = np.zeros((6 * 2, 210), dtype=np.uint8)
    lin = linear(Tensor("odd", (6, 512), "Q6_K", blocks.reshape(-1)))  # six rows: not groups of four
    assert not isinstance(lin, ScaledLinear) and tuple(lin.weight.shape) == (6, 512)


# ---- layers kept as the file's blocks


def random_tensor(kind: str, seed: int = 0, shape=(16, 512)) -> Tensor:
    rng = np.random.default_rng(seed)
    return Tensor(kind, shape, kind, blocks_numpy(kind, 1, shape[0], shape[1], rng).reshape(-1))


def weights(t: Tensor) -> np.ndarray:
    return R.dequantize(t.data, t.type, t.shape)


@pytest.mark.parametrize("kind", AS_BLOCKS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 8, MAX_TOKENS + 1, 40])
def test_a_layer_of_blocks_multiplies_as_its_weights_do(cuda, kind, tokens, dtype):
    t = random_tensor(kind, seed=tokens)
    lin = linear(t, as_blocks=AS_BLOCKS)
    assert isinstance(lin, BlockLinear) and lin.nbytes == t.data.nbytes
    x = randn((1, tokens, t.shape[1]), dtype, tokens)
    got = lin(x)
    want = x.float().cpu().numpy().astype(np.float64) @ weights(t).astype(np.float64).T
    assert got.shape == (1, tokens, t.shape[0]) and got.dtype == dtype
    assert np.abs(got.float().cpu().numpy() - want).max() <= TOL[dtype] * np.abs(want).max()


@pytest.mark.parametrize("kind", AS_BLOCKS)
@pytest.mark.parametrize("tokens", [1, 4, MAX_TOKENS + 4])
def test_a_layer_of_blocks_with_outputs_and_inputs_reordered(cuda, kind, tokens):
    t = random_tensor(kind, seed=7)
    rng = np.random.default_rng(1)
    rows = rng.permutation(t.shape[0])
    cols = (rng.permutation(t.shape[1] // 128)[:, None] * 128 + np.arange(128)).reshape(-1)
    lin = linear(t, rows=rows, cols=cols, as_blocks=AS_BLOCKS)
    x = randn((tokens, t.shape[1]), torch.float32, 9)
    want = x.cpu().numpy().astype(np.float64) @ weights(t).astype(np.float64)[rows][:, cols].T
    assert np.abs(lin(x).cpu().numpy() - want).max() <= 2e-5 * np.abs(want).max()


@pytest.mark.parametrize("kind", AS_BLOCKS)
def test_a_window_over_blocks_gives_each_token_what_it_gets_alone(cuda, kind):
    t = random_tensor(kind, seed=3)
    lin = linear(t, as_blocks=AS_BLOCKS)
    x = randn((5, t.shape[1]), torch.float16, 4)
    together = lin(x)
    for i in range(5):
        assert torch.equal(lin(x[i : i + 1]), together[i : i + 1])


def test_a_type_not_asked_for_as_blocks_is_held_as_floats(cuda):
    t = random_tensor("Q3_K")
    assert not isinstance(linear(t), BlockLinear)
    lin = linear(t, as_blocks=("IQ4_XS",))
    assert not isinstance(lin, BlockLinear)
    x = randn((3, t.shape[1]), torch.float32, 2)
    want = x.cpu().numpy().astype(np.float64) @ weights(t).astype(np.float64).T
    assert np.abs(lin(x).cpu().numpy() - want).max() <= 2e-5 * np.abs(want).max()


def test_rows_that_do_not_end_on_a_block_are_held_as_before():
    odd = Tensor("odd", (2, 4, 320), "Q3_K", np.zeros(2 * 4 * 320 // 256 * 110, dtype=np.uint8))
    short = Tensor("short", (4, 320), "Q3_K", np.zeros(4 * 320 // 256 * 110, dtype=np.uint8))
    assert not as_blocks(odd) and not as_blocks(short) and as_blocks(random_tensor("Q3_K"))


@pytest.mark.parametrize("kind", AS_BLOCKS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_an_embedding_of_blocks_gives_the_rows_of_the_weights(cuda, kind, dtype):
    t = random_tensor(kind, seed=2)
    emb = embedding(t, dtype, AS_BLOCKS)
    assert isinstance(emb, BlockEmbedding) and emb.nbytes == t.data.nbytes
    ids = torch.tensor([[5, 0, 3, 3, 1]], device="cuda")
    got = emb(ids)
    want = weights(t)[ids.cpu().numpy()]
    assert got.shape == (1, 5, t.shape[1]) and got.dtype == dtype
    tol = 1e-6 if dtype == torch.float32 else 1e-3
    assert np.abs(got.float().cpu().numpy() - want).max() <= tol * np.abs(want).max()
    one = emb(torch.tensor([4], device="cuda"))
    assert one.shape == (1, t.shape[1])
    assert torch.equal(one, emb(torch.tensor([[4]], device="cuda"))[0])


# Q8_0 dense tensors (strata_mlx/gguf.py:203-206: a weight is d * int8 code, blocks of 32) -- the attention
# projections of the long-context configuration -- through the window kernel and BlockLinear.


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("tokens", [1, 2, 5, 8])
def test_q8_0_window_products_are_the_weights_products(cuda, tokens, dtype):
    from strata_mlx_b200.blocks import window_matvec

    rows, cols = 1024, 2048
    t = random_tensor("Q8_0", seed=80 + tokens, shape=(rows, cols))
    x = randn((tokens, cols), dtype, tokens)
    got = window_matvec(torch.from_numpy(t.data).cuda(), "Q8_0", rows, cols, x)
    torch.cuda.synchronize()
    from strata_mlx_b200 import _lib

    _lib.check_device_errors()
    want = x.float().cpu().numpy().astype(np.float64) @ weights(t).astype(np.float64).T
    assert got.shape == (tokens, rows) and got.dtype == dtype
    err = np.abs(got.float().cpu().numpy() - want).max() / np.abs(want).max()
    assert err <= (1e-5 if dtype == torch.float32 else 2e-3 if dtype == torch.float16 else 8e-3), err


@pytest.mark.parametrize("tokens", [1, 3, MAX_TOKENS + 4])
def test_a_q8_0_layer_of_blocks_multiplies_as_its_weights_do(cuda, tokens):
    t = random_tensor("Q8_0", seed=8, shape=(256, 1024))
    lin = linear(t, as_blocks=("Q8_0",))
    assert isinstance(lin, BlockLinear) and lin.nbytes == t.data.nbytes
    x = randn((tokens, t.shape[1]), torch.float32, tokens)
    want = x.cpu().numpy().astype(np.float64) @ weights(t).astype(np.float64).T
    assert np.abs(lin(x).cpu().numpy() - want).max() <= 2e-5 * np.abs(want).max()


def test_a_q8_0_window_gives_each_token_what_it_gets_alone(cuda):
    t = random_tensor("Q8_0", seed=5, shape=(512, 1024))
    lin = linear(t, as_blocks=("Q8_0",))
    x = randn((6, t.shape[1]), torch.bfloat16, 6)
    together = lin(x)
    for i in range(6):
        assert torch.equal(lin(x[i : i + 1]), together[i : i + 1])
