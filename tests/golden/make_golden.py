"""Writes tests/golden/dequant_golden.npz: seeded random GGUF blocks of every block type and the float32
weights the reference's own test oracle gives for them (tests/test_blocks.py:13-19 of strata-mlx):

  * gguf-py 0.19.0 ``gguf.quants.dequantize`` (the version strata-mlx pins, uv.lock:135-136) for the nine types
    it has;
  * for Q2_0, which gguf-py 0.19.0 lacks, the numpy decoder of strata-mlx tests/test_gguf.py:33-38
    ((code - 1) * d, restated here).

The blocks are made as the reference's ``random_tensor`` makes them (tests/test_gguf.py:17-30): uniform bytes,
then a float16 scale drawn from U(-0.05, 0.05) written at each scale offset, IQ1_M's scale spread over the top
nibbles of its four scale words. Run:  python tests/golden/make_golden.py
"""

import os

import numpy as np

ROWS, COLS = 2, 1536
KINDS = {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
         "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56), "Q2_0": (64, 18),
         "Q3_K": (256, 110), "Q8_0": (32, 34)}
# strata-mlx tests/test_gguf.py:12-14: where each block keeps its float16 scales
SCALE_BYTES = {"Q2_0": [0], "Q8_0": [0], "IQ4_NL": [0], "IQ4_XS": [0], "Q3_K": [108], "IQ3_S": [0],
               "IQ3_XXS": [0], "IQ2_S": [0], "IQ2_XS": [0], "IQ2_XXS": [0], "IQ1_M": []}


def random_blocks(kind: str, seed: int, rows: int = ROWS, cols: int = COLS) -> np.ndarray:
    per_block, block_bytes = KINDS[kind]
    rng = np.random.default_rng(seed)
    n = rows * cols // per_block
    blocks = rng.integers(0, 256, (n, block_bytes), dtype=np.uint8)
    for at in SCALE_BYTES[kind]:
        blocks[:, at : at + 2] = rng.uniform(-0.05, 0.05, (n, 1)).astype("<f2").view(np.uint8)
    if kind == "IQ1_M":
        d = rng.uniform(-0.05, 0.05, n).astype("<f2").view("<u2")
        words = blocks[:, 48:56].copy().view("<u2")
        for i in range(4):
            words[:, i] = (words[:, i] & 0x0FFF) | (((d >> (4 * i)) & 15) << 12)
        blocks[:, 48:56] = words.view(np.uint8)
    return blocks.reshape(-1)


def gguf_reference(kind: str, data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    if kind == "Q2_0":
        b = data.reshape(-1, 18)
        d = b[:, :2].copy().view("<f2").astype(np.float32)
        code = np.stack([(b[:, 2:] >> s) & 3 for s in (0, 2, 4, 6)], axis=2).reshape(-1, 64)
        return ((code.astype(np.float32) - 1) * d).reshape(rows, cols)
    import gguf

    qtype = getattr(gguf.GGMLQuantizationType, kind)
    return gguf.quants.dequantize(data.reshape(rows, -1), qtype).reshape(rows, cols).astype(np.float32)


def main() -> None:
    out = {}
    for i, kind in enumerate(sorted(KINDS)):
        data = random_blocks(kind, seed=100 + i)
        out[f"{kind}_blocks"] = data
        out[f"{kind}_weights"] = gguf_reference(kind, data, ROWS, COLS)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_golden.npz")
    np.savez_compressed(path, rows=ROWS, cols=COLS, **out)
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
