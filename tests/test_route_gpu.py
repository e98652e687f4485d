"""Router, top-k, combine and the decode block against the CPU oracle (ported from strata-mlx
tests/test_fused.py:90-138, plus the block of fused.py:487-497)."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import layer_numpy

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("tokens", [1, 3, 8, 20])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_a_router_product_in_float32_from_float16_weights(cuda, tokens, dt):
    torch.manual_seed(tokens)
    w = (torch.randn(48, 256) * 0.05).half().cuda()
    router = F.WindowLinear(w)
    x = torch.randn(1, tokens, 256).to(dt).cuda()
    got = router(x)
    want = x.double() @ w.double().T
    assert got.shape == (1, tokens, 48) and got.dtype == torch.float32
    assert (got.double() - want).abs().max().item() <= 1e-5 * want.abs().max().item()
    if tokens <= 8:
        alone = torch.cat([router(x[:, t : t + 1]) for t in range(tokens)], dim=1)
        assert torch.equal(alone, got)


@pytest.mark.parametrize("tokens", [1, 3, 8, 40])
@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("n", [512, 96, 2048])
def test_the_routers_choice_is_a_stable_sort(cuda, tokens, ties, n):
    torch.manual_seed(tokens + 10 * ties + n)
    for _ in range(5):
        logits = torch.randn(1, tokens, n)
        if ties:
            logits = torch.round(logits * 4) / 4
        want = R.top_k(logits.numpy(), 10)
        got = F.top_k(logits.cuda(), 10).view(torch.int32).cpu().numpy()
        np.testing.assert_array_equal(got, want)
        idx, w = F.top_k_softmax(logits.cuda(), 10)
        np.testing.assert_array_equal(idx.view(torch.int32).cpu().numpy(), want)
        np.testing.assert_allclose(w.cpu().numpy(), R.softmax_topk(logits.numpy(), want), rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("tokens", [1, 3, 8, 16])
@pytest.mark.parametrize("dt, nd", [(torch.float16, np.float16), (torch.bfloat16, "bfloat16")])
def test_the_end_of_the_moe_block_is_the_oracles_bits(cuda, tokens, dt, nd):
    torch.manual_seed(tokens)
    for _ in range(5):
        y = (torch.randn(1, tokens, 10, 2560) * 0.5).to(dt)
        w = torch.softmax(torch.randn(1, tokens, 10), dim=-1)
        g = (2 * torch.randn(1, tokens, 1)).to(dt)
        s = (0.5 * torch.randn(1, tokens, 2560)).to(dt)
        got = F.moe_combine(y.cuda(), w.cuda(), g.cuda(), s.cuda()).float().cpu().numpy()
        want = R.moe_combine(y.float().numpy(), w.numpy(), g.float().numpy(), s.float().numpy(), nd)
        # the gate's exp is CUDA's expf against numpy's: where they round the gate apart, a unit of the type
        assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
        exact = (got == want).mean()
        assert exact > 0.99, exact


def _layer(kinds, seed, hidden=2048, inter=512, experts=64, shared=512):
    kinds = tuple(kinds)
    rng = np.random.default_rng(seed)
    L = layer_numpy(rng, hidden, inter, experts, kinds, shared_inter=shared)
    W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (experts, inter, hidden)), ("up", kinds[1], (experts, inter, hidden)),
        ("down", kinds[2], (experts, hidden, inter)), ("sgate", kinds[0], (shared, hidden)),
        ("sup", kinds[1], (shared, hidden)), ("sdown", kinds[2], (hidden, shared)))}
    return L, W


@pytest.mark.parametrize("kinds", [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "IQ3_S"), ("IQ3_S", "IQ3_S", "Q2_0"),
                                   ("IQ4_NL", "IQ4_NL", "IQ2_S")])
@pytest.mark.parametrize("tokens", [1, 5])
def test_the_decode_block_is_the_oracles(cuda, monkeypatch, kinds, tokens):
    """Router, top-10, softmax, routed SwiGLU experts, shared expert, combine: config-2 shapes with 64 experts."""
    L, W = _layer(kinds, tokens)
    experts, hidden, inter = 64, 2048, 512
    rng = np.random.default_rng(100 + tokens)
    x32 = rng.standard_normal((tokens, hidden)).astype(np.float32)
    x = dev(x32).to(torch.bfloat16)
    want, widx, ww = R.moe_layer(x.float().cpu().numpy(), L["router"], L["shared_gate"], W["gate"], W["up"], W["down"],
                                 W["sgate"], W["sup"], W["sdown"], 10, "bfloat16")
    lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (experts, inter, hidden)), ("up", kinds[1], (experts, inter, hidden)),
        ("down", kinds[2], (experts, hidden, inter)), ("sgate", kinds[0], (1, 512, hidden)),
        ("sup", kinds[1], (1, 512, hidden)), ("sdown", kinds[2], (1, hidden, 512)))}
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], 10,
                             shared=(lin["sgate"], lin["sup"], lin["sdown"]), shared_gate=dev(L["shared_gate"]))
    fused = layer(x).float().cpu().numpy()  # the three-kernel path where the block types have fragment decoders
    assert np.abs(fused - want).max() <= 2e-2 * np.abs(want).max()
    monkeypatch.setenv("SC_DECODE_CHAIN", "1")  # the chain of single-purpose kernels
    got = layer(x).float().cpu().numpy()
    idx, w = layer.routes(tokens, x.device)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    np.testing.assert_array_equal(np.sort(idx.view(torch.int32).cpu().numpy(), -1), np.sort(widx, -1))
    assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()  # bfloat16 activations, rounded at every step
    routed = F.RoutedMoE(dev(L["router"]), B.BlockSwitchGLU(lin["gate"], lin["up"], lin["down"]),
                         F.SharedExpert(lin["sgate"], lin["sup"], lin["sdown"]), dev(L["shared_gate"]), 10)
    got2 = routed(x).float().cpu().numpy()
    assert np.abs(got2 - want).max() <= 2e-2 * np.abs(want).max()
    np.testing.assert_array_equal(got2, got)  # the Python block and the C chain give the same bits


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_swiglu_16_byte_and_scalar_paths_match_the_oracle(cuda, dt):
    """B.swiglu (sc_swiglu): the 16-byte path (aligned, n a multiple of 8) and the scalar one (an odd offset) give
    the same bits, and the oracle's swiglu (blocks.py:230-238) within a unit of the type (numpy's exp and CUDA's
    expf round apart now and then)."""
    torch.manual_seed(5)
    n = 8 * 12345
    g = (torch.randn(n + 1) * 4).to(dt).cuda()
    u = (torch.randn(n + 1) * 2).to(dt).cuda()
    vec = B.swiglu(g[:n], u[:n])
    odd = B.swiglu(g[1:], u[1:])
    assert torch.equal(B.swiglu(g[1 : n + 1].clone(), u[1 : n + 1].clone()), odd)
    assert torch.equal(vec[1:], B.swiglu(g[1:n].clone(), u[1:n].clone()))
    nd = "bfloat16" if dt == torch.bfloat16 else "float16"
    want = R.swiglu(g[:n].float().cpu().numpy(), u[:n].float().cpu().numpy(), nd)
    got = vec.float().cpu().numpy()
    same = got == want
    assert same.mean() > 0.99, same.mean()
    unit = np.abs(want) * (2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10) + 1e-30
    assert (np.abs(got - want) <= unit)[~same].all()
