"""The persistent chain kernel (sc_moe_decode_chain, fused.DecodeChain): every layer of a stack in one launch, with
grid-wide barriers between a layer's phases. Checked bit for bit against the same layers called one by one
(sc_moe_decode_layer's three kernels) -- routes of every layer and the last output -- over windows of 1..8 tokens,
block-type mixes that change from layer to layer, with and without refeed, at 64 and 512 experts; against the oracle
at 512 experts; and replayed from a CUDA graph."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import blocks_numpy
from tests import decode_bar

pytestmark = pytest.mark.gpu

H, I, K, S = 2048, 512, 10, 512
# block scales that keep a chained layer's outputs O(1) for O(1) inputs (IQ3 layers amplify as sigma^3)
SIGMA = {"Q2_0": 0.025, "IQ3_S": 2.4e-4, "IQ3_XXS": 2.4e-4}
MIXES = [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "IQ3_S"), ("IQ3_XXS", "IQ3_XXS", "IQ3_XXS"),
         ("IQ3_S", "IQ3_S", "Q2_0"), ("Q2_0", "Q2_0", "IQ3_XXS")]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_layer(rng, E, kinds, shared=True):
    kg, ku, kd = kinds
    L = {"router": rng.normal(0, 0.02, (E, H)).astype(np.float16), "kinds": kinds,
         "gate": blocks_numpy(kg, E, I, H, rng, SIGMA[kg]), "up": blocks_numpy(ku, E, I, H, rng, SIGMA[ku]),
         "down": blocks_numpy(kd, E, H, I, rng, SIGMA[kd])}
    if shared:
        L.update(sgate=blocks_numpy(kg, 1, S, H, rng, SIGMA[kg]), sup=blocks_numpy(ku, 1, S, H, rng, SIGMA[ku]),
                 sdown=blocks_numpy(kd, 1, H, S, rng, SIGMA[kd]),
                 shared_gate=rng.normal(0, 0.02, (H,)).astype(np.float16), shared_kinds=kinds)
    lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
        ("gate", kg, (E, I, H)), ("up", ku, (E, I, H)), ("down", kd, (E, H, I)))}
    sh = None
    if shared:
        sh = tuple(B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
            ("sgate", kg, (1, S, H)), ("sup", ku, (1, S, H)), ("sdown", kd, (1, H, S))))
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], K, shared=sh,
                             shared_gate=dev(L["shared_gate"]) if shared else None)
    return L, layer


_stacks: dict = {}


def stack(E, n, shared=True):
    key = (E, n, shared)
    if key not in _stacks:
        rng = np.random.default_rng(1000 + E + n)
        _stacks[key] = [make_layer(rng, E, MIXES[i % len(MIXES)], shared) for i in range(n)]
    return _stacks[key]


def one_by_one(layers, x, refeed):
    y, routes = x, []
    for i, l in enumerate(layers):
        if refeed and i % refeed == 0:
            y = x
        y = l(y)
        routes.append(l.routes(x.shape[0], x.device)[0].clone())
    return y, routes


@pytest.mark.parametrize("E", [64, 512])
@pytest.mark.parametrize("tokens", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("refeed", [0, 2])
def test_the_chain_in_one_launch_is_the_layers_one_by_one(cuda, E, tokens, refeed):
    layers = [l for _, l in stack(E, 5)]
    if refeed:
        layers = layers[:4]
    chain = F.DecodeChain(layers, refeed)
    rng = np.random.default_rng(tokens)
    x = dev(rng.standard_normal((tokens, H)).astype(np.float32)).to(torch.bfloat16)
    got = chain(x)
    again = chain(x)  # the launch left the barrier count at zero: a second launch on the workspace is the same
    torch.cuda.synchronize()
    chain.check_errors()
    want, want_routes = one_by_one(layers, x, refeed)
    torch.cuda.synchronize()
    assert torch.isfinite(want.float()).all()
    idx, _ = chain.routes(tokens, x.device)
    for i, r in enumerate(want_routes):
        assert torch.equal(idx[i], r), f"layer {i}: other routes"
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()
    assert torch.equal(again, want)


def test_a_chain_without_a_shared_expert(cuda):
    layers = [l for _, l in stack(64, 3, shared=False)]
    chain = F.DecodeChain(layers, 0)
    x = torch.randn((3, H), device="cuda").to(torch.bfloat16)
    got = chain(x)
    want, _ = one_by_one(layers, x, 0)
    torch.cuda.synchronize()
    chain.check_errors()
    assert torch.equal(got, want)


@pytest.mark.parametrize("tokens", [1, 8])
def test_one_layer_of_the_chain_at_512_experts_is_the_oracles(cuda, tokens):
    L, layer = stack(512, 2)[1]
    chain = F.DecodeChain([layer])
    x = dev(np.random.default_rng(9).standard_normal((tokens, H)).astype(np.float32)).to(torch.bfloat16)
    got = chain(x)
    torch.cuda.synchronize()
    chain.check_errors()
    parts = R.moe_layer_blocks(x.float().cpu().numpy(), L, H, I, K, "bfloat16", shared_inter=S)
    idx, w = chain.routes(tokens, x.device)
    np.testing.assert_array_equal(idx[0].view(torch.int32).cpu().numpy(), parts["idx"].astype(np.int32))
    np.testing.assert_allclose(w[0].cpu().numpy(), parts["w"], rtol=1e-5, atol=1e-7)
    decode_bar.check(got.float().cpu().numpy(), parts, "bfloat16")


def test_the_chain_replayed_from_a_graph(cuda):
    layers = [l for _, l in stack(512, 5)][:4]
    g = F.DecodeGraph(layers, tokens=2, chain=True, refeed=2, persistent=True)
    x = torch.randn((2, H), device="cuda").to(torch.bfloat16)
    out = g(x.cpu()).cuda()
    want, _ = one_by_one(layers, x, 2)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    g.x.copy_(x)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(g.outs[-1], want)
