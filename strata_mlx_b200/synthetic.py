"""Seeded synthetic GGUF blocks and MoE layers of the benchmark configurations (no model files exist here).

Blocks are uniform random bytes with a float16 scale written at each of the type's scale offsets (the
generator of strata-mlx's tests, tests/test_gguf.py:12-30), the scale drawn from N(0, sigma) as the benchmark
configurations ask (fp16 d ~ N(0, 0.02)). IQ1_M's scale is spread over the top nibbles of its four scale words.

`blocks_numpy` makes small stacks on the CPU (the tests feed the same bytes to the oracle); `blocks_cuda`
makes benchmark-sized stacks directly in HBM with torch's CUDA generator.
"""

from __future__ import annotations

import numpy as np
import torch

BLOCK = {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
         "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56), "Q2_0": (64, 18),
         "Q3_K": (256, 110), "Q8_0": (32, 34)}
# where each block keeps its float16 scale (strata-mlx tests/test_gguf.py:12-14)
SCALE_BYTES = {"Q2_0": [0], "Q8_0": [0], "IQ4_NL": [0], "IQ4_XS": [0], "Q3_K": [108], "IQ3_S": [0],
               "IQ3_XXS": [0], "IQ2_S": [0], "IQ2_XS": [0], "IQ2_XXS": [0], "IQ1_M": []}


def n_blocks(kind: str, mats: int, rows: int, cols: int) -> int:
    per_block, _ = BLOCK[kind]
    if cols % per_block:
        raise ValueError(f"{kind}: rows of {cols} weights do not end on a block of {per_block}")
    return mats * rows * cols // per_block


def blocks_numpy(kind: str, mats: int, rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02,
                 uniform: float | None = None) -> np.ndarray:
    """uint8 bytes of a (mats, rows, cols) stack; scales N(0, sigma), or U(-uniform, uniform) when given."""
    n = n_blocks(kind, mats, rows, cols)
    bb = BLOCK[kind][1]
    b = rng.integers(0, 256, (n, bb), dtype=np.uint8)

    def scales(size):
        v = rng.uniform(-uniform, uniform, size) if uniform else rng.normal(0.0, sigma, size)
        return v.astype("<f2")

    for at in SCALE_BYTES[kind]:
        b[:, at : at + 2] = scales((n, 1)).view(np.uint8)
    if kind == "IQ1_M":
        d = scales(n).view("<u2")
        words = b[:, 48:56].copy().view("<u2")
        for i in range(4):
            words[:, i] = (words[:, i] & 0x0FFF) | (((d >> (4 * i)) & 15) << 12)
        b[:, 48:56] = words.view(np.uint8)
    return b.reshape(-1)


def blocks_cuda(kind: str, mats: int, rows: int, cols: int, seed: int, device="cuda", sigma: float = 0.02) -> torch.Tensor:
    """The same distribution made in HBM: uniform bytes from torch's CUDA generator, then float16 N(0, sigma)
    scales written at the scale offsets."""
    n = n_blocks(kind, mats, rows, cols)
    bb = BLOCK[kind][1]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    b = torch.randint(0, 256, (n, bb), dtype=torch.uint8, device=device, generator=g)
    for at in SCALE_BYTES[kind]:
        d = (torch.randn((n,), generator=g, device=device) * sigma).to(torch.float16)
        b[:, at : at + 2] = d.view(torch.uint8).reshape(n, 2)
    if kind == "IQ1_M":
        d = (torch.randn((n,), generator=g, device=device) * sigma).to(torch.float16).view(torch.int16).to(torch.int32) & 0xFFFF
        words = b[:, 48:56].contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        for i in range(4):
            words[:, i] = (words[:, i] & 0x0FFF) | (((d >> (4 * i)) & 15) << 12)
        b[:, 48:56] = words.to(torch.int16).view(torch.uint8).reshape(n, 8)
    return b.reshape(-1)


def layer_numpy(rng: np.random.Generator, hidden: int, inter: int, experts: int, kinds=("Q2_0", "Q2_0", "Q2_0"),
                shared_inter: int = 0, shared_kinds=None, sigma: float = 0.02) -> dict:
    """A MoE layer's tensors on the CPU: router (E, H) float16 N(0, sigma), routed gate/up (E, I, H) and down
    (E, H, I) blocks, and optionally a shared expert and its float16 gate vector."""
    kg, ku, kd = kinds
    out = {"router": rng.normal(0, sigma, (experts, hidden)).astype(np.float16),
           "gate": blocks_numpy(kg, experts, inter, hidden, rng, sigma), "up": blocks_numpy(ku, experts, inter, hidden, rng, sigma),
           "down": blocks_numpy(kd, experts, hidden, inter, rng, sigma), "kinds": kinds}
    if shared_inter:
        sk = shared_kinds or kinds
        out.update(sgate=blocks_numpy(sk[0], 1, shared_inter, hidden, rng, sigma),
                   sup=blocks_numpy(sk[1], 1, shared_inter, hidden, rng, sigma),
                   sdown=blocks_numpy(sk[2], 1, hidden, shared_inter, rng, sigma),
                   shared_gate=rng.normal(0, sigma, (hidden,)).astype(np.float16), shared_kinds=sk)
    return out


# ---- configuration 3's routes: a prefill chunk's top-10 of 512 experts, Zipf-skewed

PREFILL_TOKENS, PREFILL_EXPERTS, PREFILL_TOP_K, ZIPF_S = 2048, 512, 10, 0.8


def prefill_routes(tokens: int = PREFILL_TOKENS, experts: int = PREFILL_EXPERTS, k: int = PREFILL_TOP_K,
                   s: float = ZIPF_S, seed: int = 2048) -> np.ndarray:
    """(tokens, k) int32 expert ids: the top-k of logits N(0, 1) - s ln(rank_e), the ranks a seeded permutation of the
    experts. s = 0.8 uses 364 of 512 experts at 2,048 tokens, as many as strata-mlx reports for its real layers
    (340-395); at s = 1 only ~220 are used."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((tokens, experts)) - s * np.log(rng.permutation(experts) + 1)
    return np.argsort(-logits, axis=1, kind="stable")[:, :k].astype(np.int32)
