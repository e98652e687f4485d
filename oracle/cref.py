"""ctypes binding of the C oracle (oracle/liboracle.so) -- TEST INFRASTRUCTURE ONLY: the CPU baseline of bench.py
and a cross-check of the numpy oracle."""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KINDS = {"Q2_0": 0, "IQ4_NL": 1, "IQ4_XS": 2, "IQ3_S": 3, "IQ3_XXS": 4, "IQ2_S": 5, "IQ2_XS": 6, "IQ2_XXS": 7,
         "IQ1_M": 8, "Q3_K": 9, "Q8_0": 10}
DT = {"float32": 0, "float16": 1, "bfloat16": 2}
_P, _I = ctypes.c_void_p, ctypes.c_int


class RefLayer(ctypes.Structure):
    _fields_ = [("hidden", _I), ("inter", _I), ("experts", _I), ("top_k", _I), ("dtype", _I),
                ("kind_gate", _I), ("kind_up", _I), ("kind_down", _I), ("gate", _P), ("up", _P), ("down", _P),
                ("router", _P), ("shared_inter", _I), ("kind_sgate", _I), ("kind_sup", _I), ("kind_sdown", _I),
                ("sgate", _P), ("sup", _P), ("sdown", _P), ("shared_gate", _P)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            from oracle.build import build

            build()
        _lib = ctypes.CDLL(path)
        _lib.ref_dequant.argtypes = [_I, _P, ctypes.c_int64, _I, _I, _P]
        _lib.ref_matvec.argtypes = [_I, _P, _I, _I, _P, _P]
        _lib.ref_moe_layer.argtypes = [_P, _P, _I, _P, _P, _P]
        _lib.ref_set_threads.argtypes = [_I]
    return _lib


def threads(n: int = 0) -> int:
    """Sets the OpenMP threads (n > 0) and returns the count in use."""
    return lib().ref_set_threads(n)


def dequantize(blocks: np.ndarray, kind: str, shape: tuple) -> np.ndarray:
    *lead, rows, cols = shape
    mats = int(np.prod(lead)) if lead else 1
    out = np.empty(shape, dtype=np.float32)
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    rc = lib().ref_dequant(KINDS[kind], b.ctypes.data, mats, rows, cols, out.ctypes.data)
    if rc:
        raise ValueError(f"ref_dequant {kind} {shape}: {rc}")
    return out


class Layer:
    """A MoE layer for the C oracle; keeps its numpy arrays alive."""

    def __init__(self, L: dict, hidden: int, inter: int, experts: int, top_k: int, dtype: str = "bfloat16",
                 shared_inter: int = 0):
        self.keep = {k: np.ascontiguousarray(v) for k, v in L.items() if isinstance(v, np.ndarray)}
        s = RefLayer()
        s.hidden, s.inter, s.experts, s.top_k, s.dtype = hidden, inter, experts, top_k, DT[dtype]
        s.kind_gate, s.kind_up, s.kind_down = (KINDS[k] for k in L["kinds"])
        s.gate, s.up, s.down = (self.keep[k].ctypes.data for k in ("gate", "up", "down"))
        s.router = self.keep["router"].ctypes.data
        if "sgate" in L:
            s.shared_inter = shared_inter
            s.kind_sgate, s.kind_sup, s.kind_sdown = (KINDS[k] for k in L["shared_kinds"])
            s.sgate, s.sup, s.sdown = (self.keep[k].ctypes.data for k in ("sgate", "sup", "sdown"))
            s.shared_gate = self.keep["shared_gate"].ctypes.data
        self.s, self.hidden, self.top_k = s, hidden, top_k

    def __call__(self, x: np.ndarray) -> tuple:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.hidden)
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.top_k), dtype=np.uint32)
        w = np.empty((T, self.top_k), dtype=np.float32)
        rc = lib().ref_moe_layer(ctypes.addressof(self.s), x.ctypes.data, T, out.ctypes.data, idx.ctypes.data,
                                 w.ctypes.data)
        if rc:
            raise ValueError(f"ref_moe_layer: {rc}")
        return out, idx, w
