"""The prefill tile products at configuration 3's own shapes: 2,048 tokens' top-10 of 512
experts with the benchmark's seeded Zipf-skewed routes (synthetic.prefill_routes: ~360 experts used, one expert
with ~1,845 pairs = 116 tiles), IQ3_XXS gate / up (512 x 2048) and down (2048 x 512), bfloat16 activations.

tile_matmul is checked against the oracle's product with the weights rounded to bfloat16 (strata_mlx/blocks.py:492,
:516-536) on every pair of a sample of experts (the most used one, whose tiles span many groups of the kernel's
work list, and 40 others: several thousand pairs), and sc_tile_glu (the three products, swiglu and the unsort in one
call) is checked bit for bit against the composition of three tile_matmul calls, a swiglu and the unsort, on every
pair."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200.synthetic import blocks_numpy, prefill_routes

pytestmark = pytest.mark.gpu

KIND, H, I, E, K = "IQ3_XXS", 2048, 512, 512, 10


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def config3(cuda):
    rng = np.random.default_rng(33)
    data = {name: blocks_numpy(KIND, E, r, c, rng, uniform=0.01) for name, r, c in
            (("gate", I, H), ("up", I, H), ("down", H, I))}
    lin = {name: B.BlockSwitchLinear(dev(data[name]), KIND, (E, r, c)) for name, r, c in
           (("gate", I, H), ("up", I, H), ("down", H, I))}
    idx = prefill_routes()
    x = dev(rng.standard_normal((idx.shape[0], H)).astype(np.float32)).to(torch.bfloat16)
    return data, lin, idx, x


def sample_experts(idx, n=40, seed=7):
    counts = np.bincount(idx.reshape(-1), minlength=E)
    used = np.nonzero(counts)[0]
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(used, size=min(n, len(used)), replace=False).tolist()) | {int(np.argmax(counts))}
    return sorted(pick), counts


def test_the_tiles_of_config3(config3):
    _, _, idx, _ = config3
    te, token, where = B.tiles_of(dev(idx), E)
    te = te.view(torch.int32).cpu().numpy()
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert len(te) == idx.size // 16 + E  # 1,792 tiles: the worst case for 20,480 pairs of 512 experts
    assert (te < E).sum() == sum(-(-c // 16) for c in counts)
    R.tiles_of_check(idx, E, te, token.view(torch.int32).cpu().numpy(), where.view(torch.int32).cpu().numpy())


@pytest.mark.parametrize("name", ["gate", "up", "down"])
def test_tile_products_at_config3_are_the_oracles(config3, name):
    data, lin, idx, x = config3
    te, token, where = B.tiles_of(dev(idx), E)
    a = x.index_select(0, token.to(torch.int64))
    if name == "down":  # the down product's input: inner activations of the pairs' slots (any bfloat16 values)
        g = torch.Generator(device="cuda")
        g.manual_seed(3)
        a = torch.randn((a.shape[0], I), generator=g, device="cuda").to(torch.bfloat16)
    rows, cols = (H, I) if name == "down" else (I, H)
    assert _lib.lib().sc_tile_matmul_path(_lib.KINDS[KIND], E, rows, cols, _lib.DTYPES[torch.bfloat16], a.shape[0],
                                          _lib.ptr(a), _lib.ptr(lin[name].blocks)) == 1
    got = B.tile_matmul(lin[name].blocks, KIND, (E, rows, cols), a, te)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    got = got.cpu().numpy()
    te_np = te.view(torch.int32).cpu().numpy()
    a_np = a.float().cpu().numpy()
    experts, counts = sample_experts(idx)
    checked = 0
    for e in experts:
        slots = np.nonzero(np.repeat(te_np == e, 16))[0]
        w = R.round_to(R.expert_rows(data[name], KIND, e, rows, cols), "bfloat16").astype(np.float64)
        want = a_np[slots].astype(np.float64) @ w.T
        err = np.abs(got[slots] - want).max() / np.abs(want).max()
        assert err <= 1e-5, (e, int(counts[e]), err)
        checked += len(slots)
    assert checked >= 2000, checked


def test_the_one_call_glu_at_config3_is_the_composition(config3):
    _, lin, idx, x = config3
    ii = dev(idx).reshape(1, -1, K)
    xx = x.reshape(1, -1, H)
    one = B._tiled_glu(xx, ii, lin["up"], lin["gate"], lin["down"])
    te, token, where = B.tiles_of(ii, E)
    a = x.index_select(0, token.to(torch.int64))

    def product(l, a):
        return B.tile_matmul(l.blocks, KIND, (E, l.output_dims, l.input_dims), a, te)

    h = B.swiglu(product(lin["gate"], a).to(torch.bfloat16), product(lin["up"], a).to(torch.bfloat16))
    comp = product(lin["down"], h).index_select(0, where.to(torch.int64)).to(torch.bfloat16)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    assert torch.equal(one.reshape(-1, H), comp)
