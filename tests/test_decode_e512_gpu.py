"""The fused decode block at the benchmark's own configuration: 512 experts, hidden 2048,
SwiGLU inter 512, top-10, a shared expert of inter 512. At 512 experts the route kernel's plan is a bitmap of 16
words and its top-k ranks 512 logits per token in the last block: the paths the benchmark takes and smaller test
layers do not. Checked against the oracle (only the chosen experts dequantized) with the bar of decode_bar.py, on
1, 2, 5 and 8 tokens and three block-type mixes."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import layer_numpy
from tests import decode_bar

pytestmark = pytest.mark.gpu

H, I, E, K, S = 2048, 512, 512, 10, 512
MIXES = [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "IQ3_S"), ("IQ3_S", "IQ3_S", "Q2_0")]
_layers: dict = {}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layer_of(kinds):
    """The layer's blocks on the CPU (for the oracle) and the decode block on the GPU, made once per mix."""
    if kinds not in _layers:
        rng = np.random.default_rng(512 + len(_layers))
        L = layer_numpy(rng, H, I, E, kinds, shared_inter=S)
        lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
            ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)),
            ("sgate", kinds[0], (1, S, H)), ("sup", kinds[1], (1, S, H)), ("sdown", kinds[2], (1, H, S)))}
        layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], K,
                                 shared=(lin["sgate"], lin["sup"], lin["sdown"]), shared_gate=dev(L["shared_gate"]))
        _layers[kinds] = (L, layer, rng)
    return _layers[kinds]


@pytest.mark.parametrize("kinds", MIXES)
@pytest.mark.parametrize("tokens", [1, 2, 5, 8])
def test_the_decode_block_at_512_experts_is_the_oracles(cuda, kinds, tokens):
    L, layer, rng = layer_of(kinds)
    x = dev(rng.standard_normal((tokens, H)).astype(np.float32)).to(torch.bfloat16)
    got = layer(x)
    again = layer(x)
    torch.cuda.synchronize()
    layer.check_errors()
    assert torch.equal(got, again), "two calls on the same window gave different bits"
    parts = R.moe_layer_blocks(x.float().cpu().numpy(), L, H, I, K, "bfloat16", shared_inter=S)
    idx, w = layer.routes(tokens, x.device)
    # the same experts, in the same order (largest logit first, ties to the lower index)
    np.testing.assert_array_equal(idx.view(torch.int32).cpu().numpy(), parts["idx"].astype(np.int32))
    np.testing.assert_allclose(w.cpu().numpy(), parts["w"], rtol=1e-5, atol=1e-7)
    stats = decode_bar.check(got.float().cpu().numpy(), parts, "bfloat16")
    assert stats["gate_exceptions"] <= 0.01 * stats["checked"], stats
