"""The MoE block on a chunk of a prompt, on the library's kernels end to end (strata_mlx/fused.py:357-390, 467-497;
blocks.py:407-440): the router's tiled product for more than 8 tokens, the shared expert through the tile products,
the combine over every token in MLX's add order, and BlockSwitchLinear's many-pair product through tiles (no host
synchronization), each against the oracle or the pair-at-a-time kernels."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import blocks_numpy

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("tokens", [9, 100, 2048])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_router_of_a_prompt_chunk(cuda, tokens, dt):
    rng = np.random.default_rng(tokens)
    w = rng.normal(0, 0.02, (512, 2048)).astype(np.float16)
    x = dev(rng.standard_normal((tokens, 2048)).astype(np.float32)).to(dt)
    got = F.WindowLinear(dev(w))(x).cpu().numpy()
    want = R.router(w, x.float().cpu().numpy())
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max() * np.sqrt(2048)


def test_combine_of_many_tokens_keeps_the_add_order(cuda):
    rng = np.random.default_rng(3)
    T, K, Dd = 300, 10, 2048
    y = R.round_to(rng.standard_normal((T, K, Dd)).astype(np.float32), "bfloat16")
    w = rng.dirichlet(np.ones(K), T).astype(np.float32)
    g = R.round_to(rng.standard_normal((T, 1)).astype(np.float32), "bfloat16")
    s = R.round_to(rng.standard_normal((T, Dd)).astype(np.float32), "bfloat16")
    got = F._combine_rows(dev(y).to(torch.bfloat16), dev(w), dev(g).to(torch.bfloat16), dev(s).to(torch.bfloat16))
    want = R.moe_combine(y, w, g.reshape(-1), s, "bfloat16")
    same = (got.float().cpu().numpy() == want)
    assert same.mean() > 0.999, same.mean()  # all but the rare sigmoid that expf and numpy round apart


def test_shared_expert_of_a_prompt_chunk_goes_through_tiles(cuda):
    rng = np.random.default_rng(4)
    kind, H, S, T = "IQ3_XXS", 2048, 512, 2048
    data = {n: blocks_numpy(kind, 1, r, c, rng, uniform=0.01) for n, r, c in (("g", S, H), ("u", S, H), ("d", H, S))}
    lin = [B.BlockSwitchLinear(dev(data[n]), kind, (1, r, c)) for n, r, c in (("g", S, H), ("u", S, H), ("d", H, S))]
    sh = F.SharedExpert(*lin)
    x = dev(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16)
    got = sh(x)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    # the oracle of the tile path: weights rounded to bfloat16, float32 products rounded to bfloat16, swiglu
    wg, wu, wd = (R.round_to(R.dequantize(data[n], kind, (r, c)), "bfloat16").astype(np.float64)
                  for n, r, c in (("g", S, H), ("u", S, H), ("d", H, S)))
    sample = rng.choice(T, 64, replace=False)
    xs = x.float().cpu().numpy()[sample].astype(np.float64)
    h = R.swiglu(R.round_to((xs @ wg.T).astype(np.float32), "bfloat16"),
                 R.round_to((xs @ wu.T).astype(np.float32), "bfloat16"), "bfloat16")
    want = R.round_to((h.astype(np.float64) @ wd.T).astype(np.float32), "bfloat16")
    g = got.float().cpu().numpy()[sample]
    assert np.abs(g - want).max() <= 2e-2 * np.abs(want).max()


def test_many_pairs_of_a_stack_go_through_tiles_without_a_host_sync(cuda):
    rng = np.random.default_rng(5)
    kind, E, rows, cols = "Q2_0", 64, 512, 2048
    data = blocks_numpy(kind, E, rows, cols, rng, uniform=0.01)
    lin = B.BlockSwitchLinear(dev(data), kind, (E, rows, cols))
    idx = dev(rng.integers(0, E, (600, 10)).astype(np.int32))  # 6,000 pairs: past unpack_from
    x = dev(rng.standard_normal((600, 1, 1, cols)).astype(np.float32)).to(torch.bfloat16)
    got = lin(x, idx)
    assert got.shape == (600, 10, 1, rows)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    w = R.round_to(R.dequantize(data, kind, (E, rows, cols)), "bfloat16")
    flat = idx.cpu().numpy().reshape(-1)
    pick = rng.choice(flat.size, 200, replace=False)
    xs = x.float().cpu().numpy().reshape(600, cols)
    want = np.einsum("prc,pc->pr", w[flat[pick]].astype(np.float64), xs[pick // 10].astype(np.float64))
    g = got.float().cpu().numpy().reshape(-1, rows)[pick]
    assert np.abs(g - want).max() <= 8e-3 * np.abs(want).max()


def test_the_routed_block_on_a_prompt_chunk(cuda):
    """RoutedMoE over 2,048 tokens: router (tiled), top-k, switch_glu (tiles), shared expert (tiles), combine
    (every row): the output the composition of the oracle-checked parts gives."""
    rng = np.random.default_rng(6)
    kind, E, H, I, S, T, K = "IQ3_XXS", 64, 2048, 512, 512, 2048, 10
    st = {n: blocks_numpy(kind, e, r, c, rng, uniform=0.01) for n, e, r, c in
          (("g", E, I, H), ("u", E, I, H), ("d", E, H, I), ("sg", 1, S, H), ("su", 1, S, H), ("sd", 1, H, S))}
    lin = {n: B.BlockSwitchLinear(dev(st[n]), kind, (e, r, c)) for n, e, r, c in
           (("g", E, I, H), ("u", E, I, H), ("d", E, H, I), ("sg", 1, S, H), ("su", 1, S, H), ("sd", 1, H, S))}
    router = dev(rng.normal(0, 0.02, (E, H)).astype(np.float16))
    sgw = dev(rng.normal(0, 0.02, (1, H)).astype(np.float16))
    block = F.RoutedMoE(router, B.BlockSwitchGLU(lin["g"], lin["u"], lin["d"]),
                        F.SharedExpert(lin["sg"], lin["su"], lin["sd"]), sgw, top_k=K)
    x = dev(rng.standard_normal((1, T, H)).astype(np.float32)).to(torch.bfloat16)
    got = block(x)
    logits = F.WindowLinear(router)(x)
    idx, w = F.top_k_softmax(logits, K)
    y = B.switch_glu(x, idx, lin["u"], lin["g"], lin["d"])
    g = F.WindowLinear(sgw)(x).to(x.dtype)
    s = F.SharedExpert(lin["sg"], lin["su"], lin["sd"])(x)
    want = F._combine_rows(y, w, g, s)
    torch.cuda.synchronize()
    _lib.check_device_errors()
    assert torch.equal(got, want)
