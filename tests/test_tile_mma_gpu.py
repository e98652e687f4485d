"""The tcgen05 tile product of prefill (tile_mma.cu) at shapes that give every block several items: groups of up to
8 tiles of one expert, an expert whose run of tiles spans three groups, tiles of no expert, and rings of stages that
wrap inside an item and across items. Checked against the oracle's product with the weights rounded to the
activations' type (strata_mlx/blocks.py:492, :516-536)."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200.synthetic import blocks_numpy

pytestmark = pytest.mark.gpu

# 256-, 64- and 32-weight blocks; rows of 1024 columns of IQ3_XXS, IQ3_S and IQ2_XXS start at two offsets
# modulo 16 bytes (two raw boxes a chunk)
KINDS = ["IQ3_XXS", "Q2_0", "IQ3_S", "IQ4_NL", "IQ2_XXS"]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def tile_list(rng, experts, picked):
    """Tiles sorted by expert as tiles_of lays them out: expert 5 holds 19 tiles (groups of 8, 8 and 3), `picked`
    other experts 1-3 tiles each, then two tiles of no expert."""
    counts = {5: 19}
    others = rng.choice([e for e in range(experts) if e != 5], size=picked, replace=False)
    counts.update({int(e): int(rng.integers(1, 4)) for e in others})
    runs = [np.full(c, e) for e, c in sorted(counts.items())]
    return np.concatenate(runs + [np.full(2, experts)]).astype(np.int32)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dt, nd", [(torch.bfloat16, "bfloat16"), (torch.float16, np.float16)])
def test_the_tensor_core_product_is_the_product_with_rounded_weights(cuda, kind, dt, nd):
    rng = np.random.default_rng(11)
    experts, rows, cols = 40, 1024, 1024  # 8 row blocks: ~330 items over the SMs
    data = blocks_numpy(kind, experts, rows, cols, rng, uniform=0.01)
    w = R.dequantize(data, kind, (experts, rows, cols))
    te = tile_list(rng, experts, 30)
    a = dev(rng.standard_normal((16 * len(te), cols)).astype(np.float32)).to(dt)
    blocks = dev(data)
    assert _lib.lib().sc_tile_matmul_path(_lib.KINDS[kind], experts, rows, cols, _lib.DTYPES[dt], a.shape[0],
                                          _lib.ptr(a), _lib.ptr(blocks)) == 1  # the tensor-core kernel takes it
    got = B.tile_matmul(blocks, kind, (experts, rows, cols), a, dev(te))
    torch.cuda.synchronize()
    _lib.check_device_errors()
    got = got.cpu().numpy()
    want = R.tile_matmul(w, a.float().cpu().numpy(), te, nd)
    ok = np.repeat(te < experts, 16)
    err = np.abs(got[ok] - want[ok]).max() / np.abs(want[ok]).max()
    assert err <= 1e-5, err  # float32 sums in the tensor cores' order


@pytest.mark.parametrize("kind, cols", [("IQ3_XXS", 512), ("IQ3_XXS", 256), ("IQ2_XXS", 512)])
def test_rows_whose_chunks_start_at_four_or_eight_offsets(cuda, kind, cols):
    """Rows of 196, 98 and 132 bytes: their chunks start at 4, 8 and 4 different offsets modulo 16 bytes."""
    rng = np.random.default_rng(5)
    experts, rows = 24, 256
    data = blocks_numpy(kind, experts, rows, cols, rng, uniform=0.01)
    w = R.dequantize(data, kind, (experts, rows, cols))
    te = tile_list(rng, experts, 12)
    a = dev(rng.standard_normal((16 * len(te), cols)).astype(np.float32)).to(torch.bfloat16)
    got = B.tile_matmul(dev(data), kind, (experts, rows, cols), a, dev(te))
    torch.cuda.synchronize()
    _lib.check_device_errors()
    want = R.tile_matmul(w, a.float().cpu().numpy(), te, "bfloat16")
    ok = np.repeat(te < experts, 16)
    got = got.cpu().numpy()
    assert np.abs(got[ok] - want[ok]).max() <= 1e-5 * np.abs(want[ok]).max()


def test_a_call_with_no_expert_tiles_writes_nothing(cuda):
    rng = np.random.default_rng(2)
    data = blocks_numpy("IQ3_XXS", 4, 128, 256, rng, uniform=0.01)
    te = np.full(3, 4, dtype=np.int32)
    a = torch.randn((48, 256), device="cuda").to(torch.bfloat16)
    out = torch.full((48, 128), 7.0, device="cuda")
    lib = _lib.lib()
    from strata_mlx_b200._lib import ptr, stream
    rc = lib.sc_tile_matmul(_lib.KINDS["IQ3_XXS"], ptr(dev(data)), 4, 128, 256, ptr(a), _lib.DTYPES[torch.bfloat16], 48,
                            ptr(dev(te)), ptr(out), ptr(_lib.error_word(a.device)), stream())
    assert rc == 0
    torch.cuda.synchronize()
    _lib.check_device_errors()
    assert bool((out == 7.0).all())


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_the_one_call_prompt_is_the_three_products(cuda, monkeypatch, dt):
    """_tiled_glu through sc_tile_glu (swiglu and the unsort in the epilogues) gives the bits of the composition of
    tile_matmul, swiglu and index_select (blocks.py:566-576)."""
    rng = np.random.default_rng(9)
    experts, hidden, inner, k, tokens = 12, 512, 256, 4, 300
    lins = {}
    for name, kind, (rows, cols) in (("gate", "IQ3_XXS", (inner, hidden)), ("up", "IQ3_XXS", (inner, hidden)),
                                     ("down", "IQ3_S", (hidden, inner))):
        data = blocks_numpy(kind, experts, rows, cols, rng, uniform=0.002)
        lins[name] = B.BlockSwitchLinear(dev(data), kind, (experts, rows, cols))
    x = dev(rng.standard_normal((1, tokens, hidden)).astype(np.float32)).to(dt)
    idx = dev(rng.integers(0, experts, (1, tokens, k)).astype(np.int32))
    one = B._tiled_glu(x, idx, lins["up"], lins["gate"], lins["down"])
    # the composition: tile_matmul x 3, swiglu, the unsort
    tiles, token, where = B.tiles_of(idx, experts)
    a = x.reshape(-1, hidden).index_select(0, token.to(torch.int64))
    prod = lambda lin, a: B.tile_matmul(lin.blocks, lin.kind, (experts, lin.output_dims, lin.input_dims), a, tiles)
    h = B.swiglu(prod(lins["gate"], a).to(dt), prod(lins["up"], a).to(dt))
    want = prod(lins["down"], h).index_select(0, where.to(torch.int64)).to(dt).reshape(1, tokens, k, hidden)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    assert one.shape == want.shape and torch.equal(one, want)
