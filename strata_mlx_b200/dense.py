"""Dense layers on the file's own forms (strata_mlx/dense.py), on CUDA: the reference's names, arguments and errors,
torch CUDA tensors in place of mx.array.

    ScaledLinear    a Q6_K layer as its three parts (gguf.q6k_parts): a weight is code * scale * d, a signed byte
                    to a code, a signed byte scale to 16 weights, a float16 d to 256. A window of up to MAX_TOKENS
                    tokens goes through sc_scaled_matvec; a chunk of a prompt multiplies as floats, made by
                    sc_scaled_floats (each weight worked out in float32, rounded once) and kept for the next chunks
                    unless `keep` is False (dense.py:141-167).
    BlockLinear     a layer held as the file's blocks (Q3_K, IQ4_XS, Q8_0 and the other block types): a window
                    through sc_window_matvec, a chunk of a prompt through the weights dequantized for it and let
                    go (dense.py:197-228).
    BlockEmbedding  an embedding held as blocks: a token's row is dequantized when the token comes
                    (dense.py:231-244).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, stream
from .blocks import BLOCK, DTYPES, _contig, _dtype, dequantize, require_cuda, window_matvec

MAX_TOKENS = 8  # dense.py:33: more than a window is a chunk of a prompt, multiplied as floats
_ROWS, _WEIGHTS = 4, 8  # dense.py:34: the rows and columns a layer's shape must divide into

_holding = []  # layers that hold their weights as floats as well, since a prompt was read


def release():
    """Drops every float copy of a Q6_K layer's weights that a prompt chunk created (dense.py:88-95)."""
    for layer in _holding:
        layer._floats = None
    _holding.clear()


def fits(rows: int, cols: int) -> bool:
    """True when the window kernel can run a layer of rows x cols: rows by 4, cols by 256 (dense.py:97-99)."""
    return rows % _ROWS == 0 and cols % (32 * _WEIGHTS) == 0


def kept_floats(tensors: dict, itemsize: int = 2) -> int:
    """Device bytes that float copies (`itemsize` bytes a weight) of a file's Q6_K layers occupy after a prompt,
    when the copies are kept; output.weight is left out since prompt chunks never reach it (dense.py:102-106)."""
    return sum(itemsize * t.shape[0] * t.shape[1] for name, t in tensors.items()
               if t.type == "Q6_K" and len(t.shape) == 2 and fits(*t.shape) and name != "output.weight")


class ScaledLinear:
    """A Q6_K linear layer stored as its codes, scales and d, used like `nn.Linear` (dense.py:109-167)."""

    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, d: torch.Tensor):
        require_cuda(codes, scales, d)
        if codes.dtype != torch.int8 or scales.dtype != torch.int8 or d.dtype != torch.float16:
            raise ValueError("codes and scales int8, d float16")
        self.codes, self.scales, self.d = _contig(codes), _contig(scales), _contig(d)
        self.output_dims, self.input_dims = (int(v) for v in codes.shape)
        self.d_step = self.input_dims // int(d.shape[1])  # weights per d value: 256, less after an input reorder
        self._floats = None
        self.keep = True  # reuse the float copy built for one prompt chunk in the chunks after it
        if not fits(*codes.shape):
            raise ValueError(f"a layer of {tuple(codes.shape)} does not fit the kernel")
        if tuple(scales.shape) != (self.output_dims, self.input_dims // 16) or self.input_dims % int(d.shape[1]):
            raise ValueError("scales (rows, cols / 16) and d (rows, cols / d_step) expected")

    @property
    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel() + 2 * self.d.numel()

    def floats(self, dtype: torch.dtype) -> torch.Tensor:
        """All weights as an (out, in) tensor of `dtype`: d * scale * code in float32, one rounding (dense.py:125-139)."""
        out = torch.empty((self.output_dims, self.input_dims), dtype=dtype, device=self.codes.device)
        check(_lib.lib().sc_scaled_floats(ptr(self.codes), ptr(self.scales), ptr(self.d), self.output_dims,
                                          self.input_dims, self.d_step, DTYPES[dtype], ptr(out), stream()),
              "scaled_floats")
        return out

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        require_cuda(x)
        rows, cols = self.output_dims, self.input_dims
        lead = tuple(x.shape[:-1])
        tokens = int(np.prod(lead)) if lead else 1
        if tokens > MAX_TOKENS:
            if not self.keep:
                return x @ self.floats(x.dtype).T
            if self._floats is None or self._floats.dtype != x.dtype:
                self._floats = self.floats(x.dtype)
                _holding.append(self)
            return x @ self._floats.T
        xs = _contig(x.reshape(tokens, cols))
        if xs.data_ptr() % 16:  # a view at an odd offset: the kernels load the activations 16 bytes at a time
            xs = xs.clone()
        out = torch.empty((tokens, rows), dtype=x.dtype, device=x.device)
        check(_lib.lib().sc_scaled_matvec(ptr(self.codes), ptr(self.scales), ptr(self.d), rows, cols, self.d_step,
                                          ptr(xs), _dtype(xs), tokens, ptr(out), ptr(_lib.error_word(x.device)),
                                          stream()), "scaled_matvec")
        return out.reshape(*lead, rows)


# ---- layers kept as the file's blocks (dense.py:172-244)

AS_BLOCKS = ("Q3_K", "IQ4_XS")  # dense.py:182: dense types left as blocks when memory is short
ARRAY_BYTES = 1.125  # dense.py:183: bytes per weight of MLX's 8-bit affine form (code, f16 scale + bias per 32)


def as_blocks(t, kinds: tuple = AS_BLOCKS) -> bool:
    """True for a 2-D tensor of a type in `kinds` whose rows are whole blocks (dense.py:185-187)."""
    per_block = BLOCK[t.type][0] if t.type in BLOCK else 32 if t.type == "Q8_0" else 0
    return t.type in kinds and per_block > 0 and len(t.shape) == 2 and t.shape[1] % per_block == 0


def spared(tensors: dict) -> int:
    """Bytes saved by holding a file's eligible dense tensors as blocks rather than 8-bit affine arrays; expert
    stacks and output.weight are not counted (dense.py:190-194)."""
    return sum(int(ARRAY_BYTES * int(np.prod(t.shape))) - t.data.nbytes for name, t in tensors.items()
               if as_blocks(t) and not name.endswith("_exps.weight") and name != "output.weight")


class BlockLinear:
    """A linear layer whose weights stay the file's quantized blocks, used like `nn.Linear` (dense.py:197-228).

    Row i of `blocks` produces output i. When the loader permuted the layer's inputs, `inputs[j]` gives the file
    column of input j; a block cannot be split, so the activations are gathered into file order instead."""

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, inputs: np.ndarray | None = None):
        require_cuda(blocks)
        self.blocks, self.kind = _contig(blocks), kind
        self.output_dims, self.input_dims = (int(v) for v in shape)
        self.to_file = None if inputs is None else torch.from_numpy(
            np.argsort(np.asarray(inputs)).astype(np.int64)).to(blocks.device)

    @property
    def nbytes(self) -> int:
        return self.blocks.numel()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        require_cuda(x)
        rows, cols = self.output_dims, self.input_dims
        lead = tuple(x.shape[:-1])
        tokens = int(np.prod(lead)) if lead else 1
        xs = x.reshape(tokens, cols)
        if self.to_file is not None:
            xs = xs.index_select(1, self.to_file)
        if tokens <= MAX_TOKENS:
            out = window_matvec(self.blocks, self.kind, rows, cols, xs)
        else:  # a prompt chunk: dequantize to the activation type for this call only
            out = xs @ dequantize(self.blocks, self.kind, (rows, cols), xs.dtype).T
        return out.reshape(*lead, rows)


class BlockEmbedding:
    """An embedding table kept as blocks; each lookup dequantizes only the rows of the given ids (dense.py:231-244)."""

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, dtype: torch.dtype):
        require_cuda(blocks)
        self.num_embeddings, self.dims = (int(v) for v in shape)
        self.rows, self.kind, self.dtype = _contig(blocks).reshape(self.num_embeddings, -1), kind, dtype

    @property
    def nbytes(self) -> int:
        return self.rows.numel()

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        taken = self.rows.index_select(0, ids.reshape(-1).to(torch.int64))
        n = int(ids.numel())
        return dequantize(taken.reshape(-1), self.kind, (n, 1, self.dims), self.dtype).reshape(*ids.shape, self.dims)
