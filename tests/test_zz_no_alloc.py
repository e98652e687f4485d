"""sc_moe_decode_layer_noalloc: the decode MoE block for callers that cannot allocate device memory.

Some hosts own all device memory from start-up (a serving process with a fixed memory plan) or bind the library
from a language without a CUDA allocator: they pass inputs and outputs only, so the block's scratch comes from a
static array inside the library. This file is collected last; it calls the entry point through the C ABI and
checks it against sc_moe_decode_layer (which takes a caller workspace), on two calls in a row.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import _lib
from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import fused as F
from strata_mlx_b200.synthetic import layer_numpy

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_the_block_without_a_workspace_gives_the_bits_of_the_block_with_one(cuda):
    lib = _lib.load()
    kinds = ("IQ3_S", "IQ3_S", "Q2_0")
    E, H, I, K, S = 64, 2048, 512, 10, 512
    rng = np.random.default_rng(42)
    L = layer_numpy(rng, H, I, E, kinds, shared_inter=S)
    lin = {k: B.BlockSwitchLinear(dev(L[k]), kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)),
        ("sgate", kinds[0], (1, S, H)), ("sup", kinds[1], (1, S, H)), ("sdown", kinds[2], (1, H, S)))}
    layer = F.MoEDecodeLayer(dev(L["router"]), lin["gate"], lin["up"], lin["down"], K,
                             shared=(lin["sgate"], lin["sup"], lin["sdown"]), shared_gate=dev(L["shared_gate"]))
    W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
        ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)),
        ("sgate", kinds[0], (S, H)), ("sup", kinds[1], (S, H)), ("sdown", kinds[2], (H, S)))}
    stream = torch.cuda.current_stream().cuda_stream
    for call, tokens in enumerate((5, 3)):  # two calls in a row: the second must not see the first's contents
        x = dev(rng.standard_normal((tokens, H)).astype(np.float32)).to(torch.bfloat16)
        want = layer(x)  # sc_moe_decode_layer with its own workspace
        got = torch.full_like(x, float("nan"))
        rc = lib.sc_moe_decode_layer_noalloc(ctypes.addressof(layer.layer), x.data_ptr(), tokens, got.data_ptr(), stream)
        assert rc == 0, lib.sc_error_string(rc).decode()
        code = ctypes.c_int(-1)
        assert lib.sc_moe_decode_noalloc_error(ctypes.byref(code), stream) == 0
        assert code.value == 0, f"call {call}: its kernels recorded {_lib.ERRORS.get(code.value, code.value)}"
        layer.check_errors()
        assert torch.equal(got, want), f"call {call}: the two entry points differ"
        ref, _, _ = R.moe_layer(x.float().cpu().numpy(), L["router"], L["shared_gate"], W["gate"], W["up"], W["down"],
                                W["sgate"], W["sup"], W["sdown"], K, "bfloat16")
        g = got.float().cpu().numpy()
        assert np.abs(g - ref).max() <= 2e-2 * np.abs(ref).max()


def test_a_layer_beyond_the_static_scratch_is_refused_with_a_clear_error(cuda):
    lib = _lib.load()
    big = _lib.SCLayer()
    big.hidden, big.inter, big.experts, big.top_k = 8192, 8192, 2048, 16
    big.kind_gate = big.kind_up = big.kind_down = _lib.KINDS["Q2_0"]
    fake = 0x1000  # never dereferenced: the size check refuses the call before anything is enqueued
    big.gate = big.up = big.down = big.router = fake
    big.dtype = _lib.DTYPES[torch.bfloat16]
    need = lib.sc_moe_decode_workspace(ctypes.addressof(big), 8)
    assert need > 4 << 20
    rc = lib.sc_moe_decode_layer_noalloc(ctypes.addressof(big), fake, 8, fake, None)
    assert rc == -11 and "static scratch" in lib.sc_error_string(rc).decode()
