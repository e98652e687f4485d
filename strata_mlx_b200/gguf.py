"""GGUF files: each tensor as the file's bytes (strata_mlx/gguf.py), and onto a CUDA device unchanged.

The reader follows the GGUF layout (version 2 and 3): a header (magic "GGUF", version, tensor count, metadata
count), the metadata as typed key / value pairs, each tensor's name, dimensions (innermost first), type and offset,
then the data from the next multiple of `general.alignment` (32 by default). A tensor comes back as `Tensor` with
numpy-order shape (the last axis runs along a row) and `data`, a uint8 view into the mapped file: nothing is copied
or converted until `to_device` puts the bytes on the GPU, where the block kernels read them as they are.

The reference also turns tensors into MLX's affine arrays (`to_affine`, `pack`): that form is MLX's own, with no
use on CUDA, and is left out. `to_float` (float types and Q6_K) and `q6k_parts` (Q6_K as dense.ScaledLinear holds
it) are kept.
"""

from __future__ import annotations

import mmap
import os
import re
import struct
from dataclasses import dataclass

import numpy as np
import torch

# GGUF type id -> (type name, weights in a block, bytes in a block), for the formats strata-mlx reads
# (strata_mlx/gguf.py:25-33); the ids and block sizes are fixed by the file format
TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 30: ("BF16", 1, 2),
    2: ("Q4_0", 32, 18), 6: ("Q5_0", 32, 22), 8: ("Q8_0", 32, 34),
    11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210),
    20: ("IQ4_NL", 32, 18), 23: ("IQ4_XS", 256, 136), 42: ("Q2_0", 64, 18),
    16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98), 21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82), 29: ("IQ1_M", 256, 56),
}

# metadata value types: id -> struct format of a scalar (8 string, 9 array are read apart)
_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9


@dataclass
class Tensor:
    """One tensor of a GGUF file (the field set of strata_mlx/gguf.py:38-49, which load.py and the tests share)."""

    name: str
    shape: tuple  # dimensions outermost first; a row of blocks lies along shape[-1]
    type: str  # the type's name in TYPES, e.g. "IQ3_S"
    data: np.ndarray  # uint8 bytes mapped from the file, not copied
    path: str = ""  # the file that holds the tensor
    offset: int = 0  # byte offset of `data` inside that file

    @property
    def quantized(self) -> bool:
        """False for the plain float types, True for every block type."""
        return self.type not in ("F32", "F16", "BF16")


class GGUF:
    """A GGUF file: `metadata` (key -> value), `tensors` (name -> Tensor, in the file's order)."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self._map
        pos = 0

        def rd(fmt: str):
            nonlocal pos
            v = struct.unpack_from("<" + fmt, buf, pos)
            pos += struct.calcsize("<" + fmt)
            return v[0] if len(v) == 1 else v

        def string() -> str:
            nonlocal pos
            n = rd("Q")
            s = bytes(buf[pos : pos + n]).decode("utf-8", errors="replace")
            pos += n
            return s

        def value(t: int):
            if t == _STRING:
                return string()
            if t == _ARRAY:
                et, n = rd("I"), rd("Q")
                return [value(et) for _ in range(n)]
            if t not in _SCALAR:
                raise ValueError(f"{path}: metadata value type {t} unknown")
            return rd(_SCALAR[t])

        if bytes(buf[:4]) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        pos = 4
        self.version = rd("I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} not read")
        n_tensors, n_kv = rd("Q"), rd("Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = string()
            self.metadata[key] = value(rd("I"))
        infos = []
        for _ in range(n_tensors):
            name = string()
            dims = [rd("Q") for _ in range(rd("I"))]
            tid, off = rd("I"), rd("Q")
            infos.append((name, dims, tid, off))
        align = int(self.metadata.get("general.alignment", 32))
        start = (pos + align - 1) // align * align
        self.tensors = {}
        for name, dims, tid, off in infos:
            if tid not in TYPES:
                raise ValueError(f"{path}: tensor {name} has type {tid}, not one this reader knows")
            kind, per, nbytes = TYPES[tid]
            shape = tuple(int(v) for v in reversed(dims))
            count = int(np.prod(shape)) if shape else 1
            if shape and shape[-1] % per:
                raise ValueError(f"{path}: {name}'s rows of {shape[-1]} do not end on a {kind} block")
            size = count // per * nbytes
            data = np.frombuffer(buf, dtype=np.uint8, count=size, offset=start + off)
            self.tensors[name] = Tensor(name, shape, kind, data, path, start + off)

    def __getitem__(self, name: str) -> Tensor:
        return self.tensors[name]

    def __contains__(self, name: str) -> bool:
        return name in self.tensors


_SPLIT = re.compile(r"-(\d{5})-of-(\d{5})\.gguf$")


def shards(path: str) -> list:
    """Every file of a split model, first to last, given any of them (strata_mlx/gguf.py:125-132): names end in
    -00001-of-0000N.gguf. A single file is its own list."""
    m = _SPLIT.search(path)
    if not m:
        return [path]
    n = int(m.group(2))
    return [path[: m.start()] + f"-{i:05d}-of-{n:05d}.gguf" for i in range(1, n + 1)]


def to_float(t: Tensor) -> np.ndarray:
    """A float tensor, or a Q6_K one, as float32 (strata_mlx/gguf.py:135-147)."""
    if t.type == "F32":
        return t.data.view("<f4").reshape(t.shape)
    if t.type == "F16":
        return t.data.view("<f2").astype(np.float32).reshape(t.shape)
    if t.type == "BF16":
        return (t.data.view("<u2").astype(np.uint32) << 16).view(np.float32).reshape(t.shape)
    if t.type == "Q6_K":
        codes, scales, d = q6k_parts(t)
        rows = codes.shape[0]
        s = d.astype(np.float32).repeat(codes.shape[1] // d.shape[1] // 16, axis=1) * scales.astype(np.float32)
        return (codes.astype(np.float32).reshape(rows, -1, 16) * s[:, :, None]).reshape(t.shape)
    raise ValueError(f"{t.name}: {t.type} is read as its blocks (to_device), not as floats")


def q6k_parts(t: Tensor):
    """A Q6_K tensor of rows as its three parts, a weight being code * scale * d (strata_mlx/gguf.py:150-165):

    codes   int8 (rows, cols)          the block's six bits a weight, less 32
    scales  int8 (rows, cols / 16)
    d       float16 (rows, cols / 256)

    A Q6_K block of 256 weights: 128 bytes of low four bits, 64 of high two bits, 16 scales, a float16 d. Each half of
    the block (128 weights) has 64 low bytes L and 32 high bytes Hb; its weight 32 q + j (run q < 4, j < 32) is the low
    nibble (q < 2) or high nibble (q >= 2) of L[32 (q % 2) + j], with bits 2q, 2q + 1 of Hb[j] above them, less 32;
    the scales run in order, one to each 16 weights.
    """
    if t.type != "Q6_K":
        raise ValueError(f"{t.name}: {t.type}, not Q6_K")
    rows = t.shape[0] if len(t.shape) > 1 else 1
    b = t.data.reshape(-1, 210)
    n = b.shape[0]
    low = b[:, :128].reshape(n, 2, 64)
    high = b[:, 128:192].reshape(n, 2, 32)
    runs = []
    for q in range(4):
        nib = low[:, :, 32 * (q % 2) : 32 * (q % 2) + 32]
        nib = nib & 15 if q < 2 else nib >> 4
        hi = (high >> (2 * q)) & 3
        runs.append(nib | (hi << 4))
    codes = (np.stack(runs, axis=2).astype(np.int16) - 32).astype(np.int8)  # (n, 2 halves, 4 runs, 32)
    scales = np.ascontiguousarray(b[:, 192:208]).view(np.int8)
    d = np.ascontiguousarray(b[:, 208:210]).view("<f2")
    return codes.reshape(rows, -1), scales.reshape(rows, -1), d.reshape(rows, -1)


def to_device(t: Tensor, device="cuda") -> torch.Tensor:
    """The tensor's bytes on `device`, unchanged (uint8): what blocks.BlockSwitchLinear, dense.BlockLinear and the
    C entry points take."""
    return torch.from_numpy(np.array(t.data, copy=True)).to(device)
