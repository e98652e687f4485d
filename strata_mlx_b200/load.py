"""A GGUF tensor as the layer that holds it on a CUDA device (strata_mlx/load.py:215-273): the tensor-to-layer part of
the reference's loader. The rest of that loader (the model's assembly, shards in memory, the expert store) is the
engine's, outside the expert path.

    scaled     a Q6_K layer as codes, scales and d (dense.ScaledLinear), outputs and inputs optionally reordered
    linear     Q6_K -> ScaledLinear; a type asked for as blocks -> dense.BlockLinear (its kernels read the file's
               blocks); the rest -> FloatLinear (float32 weights)
    experts    a stack of experts -> blocks.BlockSwitchLinear
    embedding  an embedding of a type asked for as blocks -> dense.BlockEmbedding; else its rows as floats
"""

from __future__ import annotations

import numpy as np
import torch

from ._lib import KINDS
from .blocks import BlockSwitchLinear, dequantize
from .dense import AS_BLOCKS, BlockEmbedding, BlockLinear, ScaledLinear, fits
from .dense import as_blocks as as_blocks_
from .gguf import Tensor, q6k_parts, to_float

_FLOATS = ("F32", "F16", "BF16")


def _dev(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def scaled(t: Tensor, rows: np.ndarray | None = None, cols: np.ndarray | None = None, device="cuda") -> ScaledLinear:
    """A Q6_K layer as its codes, scales and d (load.py:215-232); `rows` and `cols` reorder its outputs and inputs.
    An input reorder must move whole runs of 16 weights (a scale's); d then goes to every `step` inputs, the
    longest run of up to 256 that the reorder keeps together."""
    step = 256
    if cols is not None:
        cols = np.asarray(cols)
        if (cols.reshape(-1, 16) - cols[::16, None] != np.arange(16)).any():
            raise ValueError(f"{t.name}: the input reorder splits a run of 16 weights")
        while (cols.reshape(-1, step) - cols[::step, None] != np.arange(step)).any():
            step //= 2
    codes, scales, d = q6k_parts(t)
    if rows is not None:
        codes, scales, d = codes[rows], scales[rows], d[rows]
    if cols is not None:
        codes, scales, d = codes[:, cols], scales[:, cols[::16] // 16], d[:, cols[::step] // 256]
    return ScaledLinear(_dev(codes, device), _dev(scales, device), _dev(d, device))


class FloatLinear:
    """A float layer: out = x . W^T with W (out, in) in the activations' type."""

    def __init__(self, weight: torch.Tensor):
        self.weight = weight
        self.output_dims, self.input_dims = (int(v) for v in weight.shape)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.weight.to(x.dtype).T


def linear(t: Tensor, rows: np.ndarray | None = None, cols: np.ndarray | None = None, as_blocks: tuple = (),
           device="cuda"):
    """A layer holding the tensor's weights, called like a Linear (load.py:235-256); `rows` and `cols` reorder its
    outputs and inputs. Q6_K that the kernel takes becomes a ScaledLinear; a tensor of a type in `as_blocks` stays
    the file's blocks (BlockLinear); the rest are held as float32 weights (FloatLinear), where the reference holds
    MLX's affine arrays: block types dequantized on the device, float types and other Q6_K as they are."""
    if t.type == "Q6_K" and fits(*t.shape):
        return scaled(t, rows, cols, device)
    if as_blocks_(t, as_blocks):
        raw = t.data.reshape(t.shape[0], -1)
        raw = raw if rows is None else raw[rows]
        return BlockLinear(_dev(raw.reshape(-1), device), t.type, (raw.shape[0], t.shape[1]), cols)
    if t.type in _FLOATS or t.type == "Q6_K":
        w = _dev(to_float(t).astype(np.float32), device)
    elif t.type in KINDS and len(t.shape) == 2:
        w = dequantize(_dev(t.data, device), t.type, t.shape)
    else:
        raise ValueError(f"{t.name}: {t.type} layers are not supported")
    if rows is not None:
        w = w[torch.as_tensor(np.asarray(rows), device=w.device)]
    if cols is not None:
        w = w[:, torch.as_tensor(np.asarray(cols), device=w.device)]
    return FloatLinear(w.contiguous())


def experts(t: Tensor, device="cuda") -> BlockSwitchLinear:
    """A stack of experts, kept as the file's blocks (load.py:259-263)."""
    if t.type not in KINDS:
        raise ValueError(f"{t.name}: {t.type} experts are not supported")
    return BlockSwitchLinear(_dev(t.data, device), t.type, t.shape)


def embedding(t: Tensor, dtype: torch.dtype = torch.float16, as_blocks: tuple = (), device="cuda"):
    """An embedding (load.py:266-273): of a type in `as_blocks`, its rows dequantized as tokens come
    (BlockEmbedding); otherwise its rows as floats of `dtype`, taken with `torch.nn.functional.embedding`."""
    if as_blocks_(t, as_blocks):
        return BlockEmbedding(_dev(t.data, device), t.type, t.shape, dtype)
    if t.type in _FLOATS:
        w = _dev(to_float(t), device).to(dtype)
    elif t.type in KINDS and len(t.shape) == 2:
        w = dequantize(_dev(t.data, device), t.type, t.shape, dtype)
    else:
        raise ValueError(f"{t.name}: {t.type} embeddings are not supported")
    return lambda ids: torch.nn.functional.embedding(ids.to(torch.int64), w)
