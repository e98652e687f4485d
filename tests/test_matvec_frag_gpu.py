"""The grouped fragment path of the unfused expert products (16-bit activations, Q2_0 / IQ3_S / IQ3_XXS, 32 pairs or
more) against float64 sums of the oracle's weights, and its forms against each other bit for bit."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200.synthetic import blocks_numpy

pytestmark = pytest.mark.gpu
KINDS = ["Q2_0", "IQ3_S", "IQ3_XXS"]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layer(kind, experts, rows, cols, seed):
    rng = np.random.default_rng(seed)
    data = blocks_numpy(kind, experts, rows, cols, rng)
    return B.BlockSwitchLinear(dev(data), kind, (experts, rows, cols)), R.dequantize(data, kind, (experts, rows, cols))


def skewed(rng, tokens, k, experts, s=0.8):
    """Each token's k distinct experts, drawn with Zipf-like weights (a few hot experts get many pairs)."""
    p = 1.0 / np.arange(1, experts + 1) ** s
    p = p / p.sum()
    perm = rng.permutation(experts)
    return np.stack([perm[rng.choice(experts, k, replace=False, p=p)] for _ in range(tokens)])


def products(w, idx, xs):
    """float64 W[idx[..]] . xs[..] an expert at a time: idx (...), xs (..., cols) -> (..., rows)"""
    out = np.zeros(idx.shape + (w.shape[1],))
    for e in np.unique(idx):
        at = np.nonzero(idx == e)
        out[at] = xs[at].astype(np.float64) @ w[e].T.astype(np.float64)
    return out


def check(got, want, w, cols, dt):
    """within the output type's rounding (half a unit in the last place: at most 2^-8 of the value in bfloat16,
    2^-11 in float16) plus 1e-5 max|w| sqrt(cols) for the sums' order"""
    rel = 2.0 ** -8 if dt == torch.bfloat16 else 2.0 ** -11
    err = np.abs(got.astype(np.float64) - want) - rel * np.abs(want)
    assert err.max() <= 1e-5 * np.abs(w).max() * np.sqrt(cols), err.max()


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows, cols", [(512, 2048), (2048, 512)])
def test_mid_batch_products_are_the_weights_products(cuda, kind, dt, rows, cols):
    """64 tokens x top-10 of 64 experts (share 10: gate/up; share 1: down), skewed routes so that hot experts get
    more than one group of eight pairs."""
    experts, tokens, k = 64, 64, 10
    lin, w = layer(kind, experts, rows, cols, rows + cols)
    rng = np.random.default_rng(7)
    idx = skewed(rng, tokens, k, experts)
    assert np.bincount(idx.reshape(-1)).max() > 8
    x = dev(rng.standard_normal((tokens, 1, 1, cols)).astype(np.float32)).to(dt)
    got = lin(x, dev(idx.astype(np.int32))).float().cpu().numpy()[:, :, 0]
    xf = x.float().cpu().numpy()[:, 0, 0]
    want = products(w, idx, np.broadcast_to(xf[:, None, :], (tokens, k, cols)))
    check(got, want, w, cols, dt)
    # one activation row a pair (the down product's form)
    xp = dev(rng.standard_normal((tokens * k, 1, cols)).astype(np.float32)).to(dt)
    flat = idx.reshape(-1)
    got = lin(xp, dev(flat.astype(np.int32))).float().cpu().numpy()[:, 0]
    want = products(w, flat, xp.float().cpu().numpy()[:, 0])
    check(got, want, w, cols, dt)
    _lib.check_device_errors()


@pytest.mark.parametrize("kind", KINDS)
def test_a_large_call_is_split_and_gives_the_bits_of_its_parts(cuda, kind):
    """More pairs than a launch takes (1,024): the host splits the call on whole tokens; each part's bits are those
    of the same pairs called alone (a pair's sums do not depend on the other pairs)."""
    experts, rows, cols = 64, 256, 1024
    lin, w = layer(kind, experts, rows, cols, 11)
    rng = np.random.default_rng(12)
    tokens, k = 130, 10  # 1,300 pairs
    idx = skewed(rng, tokens, k, experts)
    x = dev(rng.standard_normal((tokens, 1, 1, cols)).astype(np.float32)).to(torch.bfloat16)
    whole = lin(x, dev(idx.astype(np.int32)))
    for t0, t1 in ((0, 40), (40, 130)):
        part = lin(x[t0:t1], dev(idx[t0:t1].astype(np.int32)))
        assert torch.equal(whole[t0:t1], part)
    xf = x.float().cpu().numpy()[:, 0, 0]
    want = products(w, idx, np.broadcast_to(xf[:, None, :], (tokens, k, cols)))
    check(whole.float().cpu().numpy()[:, :, 0], want, w, cols, torch.bfloat16)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gate_up_and_glu_forms_give_the_bits_of_the_products_apart(cuda, kind, dt):
    experts, inner, hidden, tokens, k = 96, 256, 1024, 48, 8
    gate, _ = layer(kind, experts, inner, hidden, 21)
    up, _ = layer(kind, experts, inner, hidden, 22)
    down, _ = layer(kind, experts, hidden, inner, 23)
    rng = np.random.default_rng(24)
    idx = dev(skewed(rng, tokens, k, experts).astype(np.int32))
    x = dev((0.05 * rng.standard_normal((tokens, hidden))).astype(np.float32)).to(dt)
    h = B.gate_up(gate, up, x, idx)
    x5 = x.reshape(tokens, 1, 1, hidden)
    g, u = gate(x5, idx).reshape(tokens * k, inner), up(x5, idx).reshape(tokens * k, inner)
    assert torch.equal(h, B.swiglu(g, u))
    flat = idx.reshape(-1)
    y = B.matvec_glu(down, flat, g, u)
    assert torch.equal(y, down(B.swiglu(g, u).reshape(tokens * k, 1, inner), flat).reshape(tokens * k, hidden))
    _lib.check_device_errors()


def test_a_bad_expert_id_is_recorded_on_the_grouped_path(cuda):
    lin, w = layer("IQ3_S", 8, 64, 512, 31)
    idx = np.tile(np.arange(8), 5).astype(np.int32)  # 40 pairs
    idx[17] = 9
    x = torch.ones((40, 1, 512), device="cuda", dtype=torch.bfloat16)
    _lib.check_device_errors()
    out = lin(x, dev(idx))
    with pytest.raises(_lib.StrataError, match="SC_ERR_INDEX"):
        _lib.check_device_errors()
    good = out[:17, 0].float().cpu().numpy()
    want = w[idx[:17]].astype(np.float64).sum(-1)
    assert (np.abs(good - want) - 2.0 ** -8 * np.abs(want)).max() <= 1e-5 * np.abs(w).max() * np.sqrt(512)
