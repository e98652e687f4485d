"""A small GGUF file of two MoE layers' expert stacks, written with gguf-py's writer, for the paged expert store's
tests (strata_mlx_b200/paged.py)."""

import gguf
import numpy as np
from gguf import GGMLQuantizationType as Q

from strata_mlx_b200 import gguf as G
from strata_mlx_b200.synthetic import blocks_numpy

E, H, I = 12, 512, 256
KINDS = {"up": "IQ3_S", "gate": "IQ3_S", "down": "IQ3_XXS"}
QTYPE = {"IQ3_S": Q.IQ3_S, "IQ3_XXS": Q.IQ3_XXS}


def write(path: str, layers: int = 2, sigma: float = 0.002) -> G.GGUF:
    rng = np.random.default_rng(3)
    w = gguf.GGUFWriter(path, "test")
    for layer in range(layers):
        for name, (rows, cols) in (("up", (I, H)), ("gate", (I, H)), ("down", (H, I))):
            kind = KINDS[name]
            a = blocks_numpy(kind, E, rows, cols, rng, sigma=sigma).reshape(E, rows, -1)
            w.add_tensor(f"blk.{layer}.ffn_{name}_exps.weight", a, raw_dtype=QTYPE[kind])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return G.GGUF(path)


def layer_tensors(f: G.GGUF, layer: int) -> tuple:
    """(gate, up, down) gguf.Tensor of a layer."""
    return tuple(f[f"blk.{layer}.ffn_{n}_exps.weight"] for n in ("gate", "up", "down"))
