"""ctypes binding of libstrata_cuda.so (include/strata_cuda.h).

The library is built in the package directory (``__graft_entry__.build()`` or
``python strata_mlx_b200/csrc/build.py``). There is no fallback: every product path calls these kernels, and
loading fails loudly when the library is missing or CUDA is not available.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libstrata_cuda.so")

# include/strata_cuda.h enums
KINDS = {"Q2_0": 0, "IQ4_NL": 1, "IQ4_XS": 2, "IQ3_S": 3, "IQ3_XXS": 4, "IQ2_S": 5, "IQ2_XS": 6, "IQ2_XXS": 7,
         "IQ1_M": 8, "Q3_K": 9, "Q8_0": 10}
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
IDX_DTYPES = {torch.int32: 0, torch.uint32: 1, torch.int64: 2}
ABI_VERSION = 1

ERRORS = {-1: "SC_ERR_KIND", -2: "SC_ERR_SHAPE", -3: "SC_ERR_DTYPE", -4: "SC_ERR_ALIGN", -5: "SC_ERR_ARG",
          -6: "SC_ERR_CUDA", -7: "SC_ERR_WORKSPACE", -8: "SC_ERR_UNSUPPORTED", -9: "SC_ERR_TIMEOUT",
          -10: "SC_ERR_INDEX", -11: "SC_ERR_SCRATCH"}

# every symbol include/strata_cuda.h declares, with its ctypes signature
_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "sc_version": (_I, []),
    "sc_error_string": (ctypes.c_char_p, [_I]),
    "sc_block_info": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "sc_dequant": (_I, [_I, _P, _I64, _I, _I, _I, _P, _P]),
    "sc_expert_matvec": (_I, [_I, _P, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P]),
    "sc_expert_matvec_ptrs": (_I, [_I, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P]),
    "sc_window_matvec": (_I, [_I, _P, _I, _I, _P, _I, _I, _P, _P, _P]),
    "sc_matvec_glu": (_I, [_I, _P, _I, _I, _I, _P, _I, _P, _P, _I, _I, _P, _P, _P]),
    "sc_expert_gate_up": (_I, [_I, _P, _P, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P]),
    "sc_swiglu": (_I, [_P, _P, _I64, _I, _P, _P]),
    "sc_router": (_I, [_P, _I, _I, _P, _I, _I, _P, _P]),
    "sc_top_k": (_I, [_P, _I, _I, _I, _P, _P]),
    "sc_top_k_softmax": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "sc_moe_combine": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "sc_tiles_of": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "sc_tiles_of_workspace": (_SZ, [_I]),
    "sc_tile_matmul": (_I, [_I, _P, _I, _I, _I, _P, _I, _I, _P, _P, _P, _P]),
    "sc_tile_matmul_path": (_I, [_I, _I, _I, _I, _I, _I, _P, _P]),
    "sc_tile_glu": (_I, [_I, _P, _I, _P, _I, _P, _I, _I, _I, _P, _I, _I, _P, _P, _I, _P, _P, _SZ, _P, _P]),
    "sc_tile_glu_workspace": (_SZ, [_I, _I, _I]),
    "sc_scaled_matvec": (_I, [_P, _P, _P, _I, _I, _I, _P, _I, _I, _P, _P, _P]),
    "sc_scaled_floats": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "sc_moe_decode_layer": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "sc_moe_decode_workspace": (_SZ, [_P, _I]),
    "sc_moe_decode_routes": (_I, [_P, _I, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "sc_moe_decode_stage": (_I, [_P, _P, _I, _P, _P, _SZ, _I, _P]),
    "sc_moe_decode_layer_ep": (_I, [_P, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "sc_moe_decode_combine": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "sc_ep_exchange_bytes": (_SZ, [_P, _I, _I]),
    "sc_ipc_handle": (_I, [_P, _P, _P]),
    "sc_ipc_open": (_I, [_P, _P]),
    "sc_ipc_close": (_I, [_P]),
    "sc_ep_feed": (_I, [_P, _P, _P, _P]),
    "sc_moe_decode_layer_ep_p2p": (_I, [_P, _P, _I, _I, _I, _P, _SZ, _P]),
    "sc_ep_combine": (_I, [_P, _P, _I, _I, _P, _P, _SZ, _P]),
    "sc_moe_decode_chain": (_I, [_P, _I, _P, _I, _I, _P, _P, _SZ, _P]),
    "sc_moe_decode_chain_workspace": (_SZ, [_P, _I, _I]),
    "sc_moe_decode_chain_routes": (_I, [_P, _I, _I, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "sc_paged_attention": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _P, _P, _SZ, _P]),
    "sc_paged_attention_workspace": (_SZ, [_I, _I]),
    "sc_add_rmsnorm": (_I, [_P, _P, _P, _I, _I, ctypes.c_float, _I, _P, _P]),
    "sc_rope_cache": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _I, _P]),
    "sc_moe_decode_layer_noalloc": (_I, [_P, _P, _I, _P, _P]),
    "sc_moe_decode_noalloc_error": (_I, [ctypes.POINTER(_I), _P]),
}


class SCExchange(ctypes.Structure):
    """sc_ep_exchange (include/strata_cuda.h): the ranks' exchange buffers for expert parallel over peer memory."""
    _fields_ = [("peers", ctypes.c_void_p), ("own", ctypes.c_uint64), ("ranks", ctypes.c_int), ("rank", ctypes.c_int),
                ("tokens_per_rank", ctypes.c_int)]


class SCLayer(ctypes.Structure):
    """include/strata_cuda.h sc_moe_layer"""

    _fields_ = [("hidden", _I), ("inter", _I), ("experts", _I), ("top_k", _I),
                ("kind_gate", _I), ("kind_up", _I), ("kind_down", _I),
                ("gate", _P), ("up", _P), ("down", _P), ("router", _P),
                ("shared_inter", _I), ("kind_sgate", _I), ("kind_sup", _I), ("kind_sdown", _I),
                ("sgate", _P), ("sup", _P), ("sdown", _P), ("shared_gate", _P), ("dtype", _I)]


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """The library, loaded once, with every declared symbol bound. Needs no GPU."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(f"{path} is not built: run __graft_entry__.build() "
                                   "(or python strata_mlx_b200/csrc/build.py) first")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            if lib.sc_version() != ABI_VERSION:
                raise RuntimeError(f"{path}: ABI version {lib.sc_version()}, expected {ABI_VERSION}")
            _lib = lib
    return _lib


def lib() -> ctypes.CDLL:
    if _lib is None:
        load()
    return _lib


class StrataError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc == 0:
        return
    msg = f"{what}: {ERRORS.get(rc, rc)} ({lib().sc_error_string(rc).decode()})"
    if rc in (-1, -2, -3, -4, -5, -7, -11):
        raise ValueError(msg)
    raise StrataError(msg)


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def require_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("strata_mlx_b200 computes on CUDA tensors only; got a tensor on " + str(t.device))


_err_words: dict = {}


def error_word(device=None) -> torch.Tensor:
    """The device int kernels record bad expert ids and given-up waits in (one per device)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    w = _err_words.get(dev)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=dev)
        _err_words[dev] = w
    return w


def check_device_errors(device=None) -> None:
    """Reads (synchronizing) and clears the device error word; raises if a kernel recorded an error."""
    w = error_word(device)
    v = int(w[0].item())
    if v:
        w.zero_()
        raise StrataError(f"a kernel recorded {ERRORS.get(v, v)}: {lib().sc_error_string(v).decode()}")
