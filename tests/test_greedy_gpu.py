"""Greedy decoding parity: 256 tokens from a fixed seed through a small synthetic MoE decoder, the CUDA decode block
(fused.MoEDecodeLayer) against the oracle's block, the same tokens chosen at every step. The decoder: a token's
embedding (bfloat16), L residual MoE blocks x <- bf16(x + moe(x)) (Q2_0 / IQ3_S / IQ3_XXS experts), logits = head . x
in float64 on the host for both paths (the head is not the path under test), the arg max (the lower index on a
tie). A step's activations are compared too: bit-equal in most steps (the gate's sigmoid rounds apart in CUDA and
numpy now and then, one bfloat16 unit), never more than a few units apart."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import blocks_numpy, layer_numpy

pytestmark = pytest.mark.gpu

V, H, I, E, K, S, LAYERS, STEPS = 512, 2048, 256, 32, 4, 256, 4, 256  # H 2048: rows of every type end on 16 bytes (the fused path)
SIGMA = {"Q2_0": 0.02, "IQ3_S": 2e-4, "IQ3_XXS": 2e-4}
KINDS = [("Q2_0", "Q2_0", "Q2_0"), ("IQ3_S", "IQ3_S", "IQ3_S"), ("IQ3_XXS", "IQ3_XXS", "IQ3_XXS"),
         ("IQ3_S", "IQ3_S", "Q2_0")]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def model(seed=7):
    rng = np.random.default_rng(seed)
    emb = R.round_to(rng.standard_normal((V, H)).astype(np.float32), "bfloat16")
    head = rng.standard_normal((V, H)).astype(np.float32)
    layers = []
    for l in range(LAYERS):
        kinds = KINDS[l % len(KINDS)]
        # expert scales by block type that make a block add O(1) to a residual stream of ~4 (an IQ3 block's output
        # grows as its scale cubed, Q2_0's as well, from different constants): without norms between the blocks,
        # larger scales make each block multiply the stream, and a one-unit rounding difference with it; the router
        # and shared gate keep 0.02
        L = layer_numpy(rng, H, I, E, kinds, shared_inter=S, sigma=0.02)
        for name, kind, mats, r, c in (("gate", kinds[0], E, I, H), ("up", kinds[1], E, I, H), ("down", kinds[2], E, H, I),
                                       ("sgate", kinds[0], 1, S, H), ("sup", kinds[1], 1, S, H), ("sdown", kinds[2], 1, H, S)):
            L[name] = blocks_numpy(kind, mats, r, c, rng, SIGMA[kind])
        W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
            ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)),
            ("sgate", kinds[0], (S, H)), ("sup", kinds[1], (S, H)), ("sdown", kinds[2], (H, S)))}
        lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
            ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)))}
        shared = tuple(B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
            ("sgate", kinds[0], (1, S, H)), ("sup", kinds[1], (1, S, H)), ("sdown", kinds[2], (1, H, S))))
        cuda = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], K, shared=shared,
                                shared_gate=dev(L["shared_gate"]))
        layers.append((L, W, cuda))
    return emb, head, layers


def next_token(head, x):
    logits = head.astype(np.float64) @ np.asarray(x, dtype=np.float64).reshape(-1)
    return int(np.argmax(logits))  # the first maximum: the lower index on a tie


def test_256_greedy_tokens_match_the_oracle(cuda):
    """Both paths decode 256 tokens greedily, each from its own previous choice. A layer is compared after every
    step; where a token's routes differ between the two (a one-unit difference of an activation upstream moves the
    10th and 11th router logits past each other), the oracle's gap between its K-th and (K+1)-th logit must be a
    near-tie (below 1e-3 of the logits' scale) and the oracle then continues from the GPU's activations (teacher
    forcing at that layer); such re-syncs must be rare. Every step's token must be the oracle's."""
    emb, head, layers = model()
    tok_gpu = tok_ref = 1
    same_x, resyncs = 0, 0
    for step in range(STEPS):
        xg = dev(emb[tok_gpu][None]).to(torch.bfloat16)
        xr = emb[tok_ref][None].astype(np.float32)
        for L, W, cuda in layers:
            xin = xg
            xg = (xg.float() + cuda(xg).float()).to(torch.bfloat16)
            y, idx, _ = R.moe_layer(xr, L["router"], L["shared_gate"], W["gate"], W["up"], W["down"], W["sgate"],
                                    W["sup"], W["sdown"], K, "bfloat16")
            xr_next = R.round_to(xr + y, "bfloat16")
            gidx = cuda.routes(1, xin.device)[0].view(torch.int32).cpu().numpy()
            if not np.array_equal(np.sort(gidx, -1), np.sort(idx.astype(np.int32), -1)):
                lg = np.sort(R.router(L["router"], R.round_to(xr, "bfloat16")).reshape(-1))[::-1]
                gap = lg[K - 1] - lg[K]
                assert gap <= 1e-3 * np.abs(lg).max(), f"step {step}: other routes without a near-tie ({gap})"
                resyncs += 1
                xr_next = xg.float().cpu().numpy()
            xr = xr_next
            xh = xg.float().cpu().numpy()
            assert np.isfinite(xh).all() and np.isfinite(xr).all()
            assert np.abs(xh - xr).max() <= 2.0 ** -5 * max(1.0, np.abs(xr).max()), f"step {step}"
        xg_host = xg.float().cpu().numpy()
        same_x += int(np.array_equal(xg_host, xr))
        tok_gpu, tok_ref = next_token(head, xg_host), next_token(head, xr)
        assert tok_gpu == tok_ref, f"step {step}: the CUDA path chose {tok_gpu}, the oracle {tok_ref}"
    assert resyncs <= 0.05 * STEPS * LAYERS, resyncs
    assert same_x >= 0.5 * STEPS, same_x
