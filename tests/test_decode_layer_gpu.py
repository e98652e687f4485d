"""The three-kernel decode block (route, gate/up, down + combine on mma.sync fragments, chained by programmatic
dependent launch) against the CPU oracle and against the chain of single-purpose kernels."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import layer_numpy
from tests import decode_bar

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def build(kinds, seed, H=2048, I=512, E=24, S=512, K=10):
    rng = np.random.default_rng(seed)
    L = layer_numpy(rng, H, I, E, kinds, shared_inter=S)
    lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)))}
    shared = None
    if S:
        shared = tuple(B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
            ("sgate", kinds[0], (1, S, H)), ("sup", kinds[1], (1, S, H)), ("sdown", kinds[2], (1, H, S))))
    W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)))}
    if S:
        W.update({k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
            ("sgate", kinds[0], (S, H)), ("sup", kinds[1], (S, H)), ("sdown", kinds[2], (H, S)))})
    return L, lin, shared, W, rng


def nd_name(dt):
    return "bfloat16" if dt == torch.bfloat16 else "float16"


def oracle(L, W, x, K, dt, S):
    return R.moe_layer(x, L["router"], L.get("shared_gate"), W["gate"], W["up"], W["down"], W.get("sgate"),
                       W.get("sup"), W.get("sdown"), K, dt)


KINDS = [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "IQ3_S"), ("IQ3_XXS", "IQ3_XXS", "IQ3_XXS"),
         ("IQ3_S", "IQ3_S", "Q2_0"), ("Q2_0", "Q2_0", "IQ3_XXS")]


@pytest.mark.parametrize("kinds", KINDS)
@pytest.mark.parametrize("tokens", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_the_three_kernel_block_is_the_oracles(cuda, kinds, tokens, dt):
    L, lin, shared, W, rng = build(kinds, tokens)
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], 10, shared=shared,
                             shared_gate=dev(L["shared_gate"]), dtype=dt)
    # float16 holds 65504 at most: smaller activations keep the IQ3 layers' outputs (|w| up to ~9) in its range
    scale = 1.0 if dt == torch.bfloat16 else 0.02
    x = dev(scale * rng.standard_normal((tokens, 2048)).astype(np.float32)).to(dt)
    got = layer(x)
    again = layer(x)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    layer.check_errors()
    assert torch.equal(got, again), "two calls on the same window gave different bits"
    parts = R.moe_layer_blocks(x.float().cpu().numpy(), L, 2048, 512, 10, nd_name(dt), shared_inter=512)
    idx, w = layer.routes(tokens, x.device)
    np.testing.assert_array_equal(idx.view(torch.int32).cpu().numpy(), parts["idx"].astype(np.int32))
    np.testing.assert_allclose(w.cpu().numpy(), parts["w"], rtol=1e-5, atol=1e-7)
    # every output within two units of the combine's rounded terms (decode_bar.py), gate edges excepted and checked
    stats = decode_bar.check(got.float().cpu().numpy(), parts, nd_name(dt))
    assert stats["gate_exceptions"] <= 0.01 * stats["checked"], stats


@pytest.mark.parametrize("kinds", KINDS[:3])
@pytest.mark.parametrize("tokens", [1, 5])
def test_the_three_kernel_block_agrees_with_the_chain(cuda, monkeypatch, kinds, tokens):
    L, lin, shared, W, rng = build(kinds, 100 + tokens)
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], 10, shared=shared,
                             shared_gate=dev(L["shared_gate"]))
    x = dev(rng.standard_normal((tokens, 2048)).astype(np.float32)).to(torch.bfloat16)
    fused = layer(x).float()
    fidx = layer.routes(tokens, x.device)[0].clone()
    monkeypatch.setenv("SC_DECODE_CHAIN", "1")
    chain = layer(x).float()
    cidx = layer.routes(tokens, x.device)[0].clone()
    torch.cuda.synchronize()
    assert torch.equal(torch.sort(fidx.view(torch.int32), -1).values, torch.sort(cidx.view(torch.int32), -1).values)
    assert (fused - chain).abs().max().item() <= 2e-2 * chain.abs().max().item()


def test_a_block_without_a_shared_expert(cuda):
    L, lin, shared, W, rng = build(("IQ3_S", "IQ3_S", "Q2_0"), 7, S=0)
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], 10)
    x = dev(rng.standard_normal((3, 2048)).astype(np.float32)).to(torch.bfloat16)
    got = layer(x).float().cpu().numpy()
    want, _, _ = R.moe_layer(x.float().cpu().numpy(), L["router"], None, W["gate"], W["up"], W["down"], None, None,
                             None, 10, "bfloat16")
    assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()


def test_the_layers_replayed_as_a_graph_give_the_eager_bits(cuda):
    """DecodeGraph captures the layers' kernels (with their programmatic dependencies) in one CUDA graph."""
    layers = []
    for s, kinds in enumerate(KINDS[:3]):
        L, lin, shared, W, rng = build(kinds, 200 + s, E=32)
        layers.append(F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], 10, shared=shared,
                                       shared_gate=dev(L["shared_gate"])))
    x = torch.randn((1, 2048), device="cuda").to(torch.bfloat16)
    eager = x
    for l in layers:
        eager = l(eager)
    g = F.DecodeGraph(layers, tokens=1, chain=True)
    out = g(x.cpu()).cuda()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
