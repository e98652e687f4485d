"""The C ABI without a GPU: the library loads, exports every symbol include/strata_cuda.h declares, and turns
bad arguments into error codes before touching CUDA. No kernel is launched here."""

import ctypes
import os
import re

import pytest
import torch

from strata_mlx_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "strata_cuda.h")


def declared() -> list:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^SC_API\s+[\w\s\*]+?\b(sc_\w+)\s*\(", text, flags=re.M)))


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_version_and_error_strings():
    lib = _lib.load()
    assert lib.sc_version() == _lib.ABI_VERSION
    for code in list(_lib.ERRORS) + [0]:
        s = lib.sc_error_string(code).decode()
        assert s and s != "unknown error code"
    assert lib.sc_error_string(12345).decode() == "unknown error code"


def test_block_info_is_the_reference_table():
    from strata_mlx_b200.blocks import BLOCK

    lib = _lib.load()
    for kind, want in list(BLOCK.items()) + [("Q8_0", (32, 34))]:
        pb, bb = ctypes.c_int(), ctypes.c_int()
        assert lib.sc_block_info(_lib.KINDS[kind], ctypes.byref(pb), ctypes.byref(bb)) == 0
        assert (pb.value, bb.value) == want
    assert lib.sc_block_info(99, None, None) == -1


def test_bad_arguments_are_rejected_before_any_launch():
    lib = _lib.load()
    fake = 0x1000  # never dereferenced: every call below fails its checks first
    assert lib.sc_dequant(99, fake, 1, 2, 256, 0, fake, None) == -1  # unknown kind
    assert lib.sc_dequant(_lib.KINDS["IQ3_S"], fake, 1, 2, 640, 0, fake, None) == -2  # 640 does not end on a block
    assert lib.sc_dequant(0, None, 1, 2, 64, 0, fake, None) == -5
    assert lib.sc_expert_matvec(0, fake, 4, 8, 100, fake, 1, 1, fake, 0, fake, None, None) == -2
    assert lib.sc_expert_matvec(0, fake, 4, 8, 128, fake, 1, 1, fake, 7, fake, None, None) == -3  # bad dtype
    assert lib.sc_router(fake, 8, 12, fake, 0, 1, fake, None) == -4  # cols not a multiple of 8
    assert lib.sc_top_k(fake, 1, 8, 17, fake, None) == -2  # k above 16
    assert lib.sc_tiles_of(fake, 0, 10, 2, 4, fake, fake, fake, None, 0, None) == -7
    assert lib.sc_tile_matmul(0, fake, 4, 100, 128, fake, 1, 16, fake, fake, None, None) == -2  # rows not by 64
    assert lib.sc_moe_decode_workspace(None, 1) == 0


def test_tiles_of_workspace_grows_with_experts():
    lib = _lib.load()
    assert lib.sc_tiles_of_workspace(512) > lib.sc_tiles_of_workspace(8) > 0


def test_products_refuse_tensors_off_the_gpu():
    """No CPU fallback: the drop-in raises rather than compute anywhere but on CUDA."""
    from strata_mlx_b200 import blocks

    b = torch.zeros(18 * 4, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        blocks.BlockSwitchLinear(b, "Q2_0", (1, 4, 64))
    with pytest.raises(ValueError, match="CUDA"):
        blocks.dequantize(b, "Q2_0", (4, 64))


def test_which_kernel_takes_a_tile_product():
    """bfloat16 / float16 at rows by 128 and columns by 256 go to the tcgen05 kernel; the rest to the CUDA cores."""
    lib = _lib.lib()
    k = _lib.KINDS["IQ3_XXS"]
    aligned = ctypes.c_void_p(1 << 20)
    assert lib.sc_tile_matmul_path(k, 512, 512, 2048, 2, 32768, aligned, aligned) == 1
    assert lib.sc_tile_matmul_path(k, 512, 2048, 512, 1, 32768, aligned, aligned) == 1
    assert lib.sc_tile_matmul_path(k, 512, 512, 2048, 0, 32768, aligned, aligned) == 0  # float32
    assert lib.sc_tile_matmul_path(k, 512, 64, 2048, 2, 32768, aligned, aligned) == 0  # rows not by 128
    assert lib.sc_tile_matmul_path(k, 512, 512, 2048, 2, 16 * 5000, aligned, aligned) == 0  # too many tiles
    assert lib.sc_tile_matmul_path(k, 512, 512, 2048, 2, 32768, ctypes.c_void_p((1 << 20) + 8), aligned) == 0


def _decode_layer(base: int, shift: dict) -> "_lib.SCLayer":
    """A decode block of the benchmark's shapes over fake, never dereferenced addresses; `shift` moves named
    pointers off their 16-byte boundary."""
    L = _lib.SCLayer()
    L.hidden, L.inter, L.experts, L.top_k, L.shared_inter = 2048, 512, 512, 10, 512
    L.kind_gate = L.kind_up = L.kind_down = L.kind_sgate = L.kind_sup = L.kind_sdown = _lib.KINDS["Q2_0"]
    for i, name in enumerate(("gate", "up", "down", "router", "sgate", "sup", "sdown", "shared_gate")):
        setattr(L, name, base + (i << 24) + shift.get(name, 0))
    L.dtype = _lib.DTYPES[torch.bfloat16]
    return L


def test_the_decode_block_refuses_pointers_off_16_bytes_before_any_launch():
    """The fused kernels bulk-copy expert rows and read router rows and the window 16 bytes at a time: a pointer at
    an odd offset is refused with SC_ERR_ALIGN on the host, before anything is enqueued (no GPU is used here)."""
    lib = _lib.load()
    base, x = 1 << 32, (1 << 32) - (1 << 24)
    ws = ctypes.c_void_p(1 << 30)
    for name in ("router", "shared_gate"):  # every path reads these 16 bytes at a time
        L = _decode_layer(base, {name: 2})
        n = lib.sc_moe_decode_workspace(ctypes.addressof(L), 1)
        assert n > 0  # the size does not depend on the pointers
        assert lib.sc_moe_decode_layer(ctypes.addressof(L), x, 1, x, ws, n, None) == -4, name
    for name in ("gate", "up", "down", "sgate", "sup", "sdown"):  # the fused kernels' bulk copies
        L = _decode_layer(base, {name: 8})
        n = lib.sc_moe_decode_workspace(ctypes.addressof(L), 1)
        assert lib.sc_moe_decode_stage(ctypes.addressof(L), x, 1, x, ws, n, 1, None) == -4, name
        assert lib.sc_moe_decode_layer_ep(ctypes.addressof(L), x, 1, 0, 256, x, ws, n, None) == -4, name
    L = _decode_layer(base, {})
    n = lib.sc_moe_decode_workspace(ctypes.addressof(L), 1)
    assert lib.sc_moe_decode_stage(ctypes.addressof(L), x + 4, 1, x, ws, n, 1, None) == -4  # the window


def test_paged_attention_workspace_and_refusals():
    """sc_paged_attention's workspace holds, per chunk of whole 16-token pages (about 296 chunks over the key/value
    heads), 64 rows of partial outputs (256 floats) with their maxima and sums, and 256 spare bytes; its argument
    checks answer before any launch."""
    lib = _lib.load()
    for ctx, kv in ((1, 2), (300, 2), (8192, 2), (131072 + 272, 2), (20000, 1), (65536, 4)):
        pages = -(-ctx // 16)
        want = -(-296 // kv)
        cpages = -(-pages // want)
        chunks = -(-pages // cpages)
        assert chunks <= want
        assert lib.sc_paged_attention_workspace(ctx, kv) == chunks * kv * 64 * (256 * 4 + 8) + 256
    assert lib.sc_paged_attention_workspace(0, 2) == 0 and lib.sc_paged_attention_workspace(8, 0) == 0
    fake = 0x1000  # never dereferenced
    ws = lib.sc_paged_attention_workspace(4096, 2)
    f = ctypes.c_float(1 / 16)

    def call(q=fake, ctx=4096, tokens=1, q_heads=16, kv_heads=2, head_dim=256, ws_bytes=ws, k=fake, table=fake):
        return lib.sc_paged_attention(q, k, fake, table, fake, ctx, tokens, q_heads, kv_heads, head_dim, f, fake,
                                      fake, ws_bytes, None)

    assert call(table=None) == -5
    assert call(head_dim=128) == -2
    assert call(q_heads=12) == -2  # eight query heads a key/value head
    assert call(tokens=0) == -2 and call(tokens=9) == -2
    assert call(ctx=3, tokens=4) == -2  # the window is part of the context
    assert call(q=fake + 8) == -4 and call(k=fake + 2) == -4
    assert call(ws_bytes=ws - 1) == -7
