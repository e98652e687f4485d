"""Experts computed on the GGUF file's own blocks, on a B200: the call surface of strata_mlx/blocks.py over
torch CUDA tensors, every product a kernel of libstrata_cuda.so.

    dequantize        every weight of a stack, bit for bit the reference's unpack32 (blocks.py:397-404)
    BlockSwitchLinear a stack of experts called like mlx-lm's QuantizedSwitchLinear (blocks.py:407-440)
    matvec_separate   each pair's expert a buffer of its own (blocks.py:331-346)
    window_matvec     one layer, a window of tokens (blocks.py:383-394)
    matvec_glu        down with silu(gate) * up worked out in the kernel (blocks.py:782-798)
    tiles_of          a prompt's pairs sorted into tiles of 16 by expert, on the GPU (blocks.py:539-563)
    tile_matmul       a tile's tokens times its expert's rows: tcgen05 tensor cores (blocks.py:516-536)
    switch_glu        the routed SwiGLU, choosing among the above (blocks.py:801-829)
    BlockSwitchGLU    a layer's routed experts, called like mlx-lm's SwitchGLU (blocks.py:832-839)

Q2_0's table-of-sums functions (blocks.py:579-771) answered an Apple GPU that was bound by arithmetic; the
B200's decode is bound by bytes, so their names are kept and they run the direct decode kernels: a "table" is
the activations themselves.

Tensors are torch CUDA tensors; `blocks` is a uint8 tensor of the file's bytes. Module constants keep the
reference's names so that tests can monkeypatch them as the reference's tests do.
"""

from __future__ import annotations


import torch

from . import _lib
from ._lib import KINDS, DTYPES, check, ptr, stream, require_cuda

# type -> (weights per block, bytes per block), strata_mlx/blocks.py:35-38
BLOCK = {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
         "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56), "Q2_0": (64, 18),
         "Q3_K": (256, 110)}

MAX_SEPARATE = 29  # the reference's Metal binding limit (blocks.py:328); the CUDA kernel takes any number
TILES_FROM = 1600  # (token, expert) pairs from which a prompt goes through tiles (blocks.py:462)
TOKENS_TILE, ROWS_TILE, COLS_TILE = 16, 64, 64  # blocks.py:463
LOOKUP_FROM = 1  # blocks.py:593
GLU_IN_DOWN = True  # blocks.py:701
BLOCK_GLU = True  # blocks.py:778
MATVEC_GLU_UPTO = 30  # blocks.py:779


def _kind(kind: str) -> int:
    if kind not in KINDS:
        raise ValueError(f"unknown block type {kind}")
    return KINDS[kind]


def _dtype(t: torch.Tensor) -> int:
    if t.dtype not in DTYPES:
        raise ValueError(f"activations of {t.dtype} are not taken (float32, float16, bfloat16)")
    return DTYPES[t.dtype]


def _row_bytes(kind: str, cols: int) -> int:
    per_block, block_bytes = BLOCK[kind] if kind in BLOCK else (32, 34)
    if cols % per_block:
        raise ValueError(f"{kind}: rows of {cols} weights do not end on a block of {per_block}")
    return cols // per_block * block_bytes


def _threads_per_row(runs: int) -> int:
    """blocks.py:303-308, kept for the `per_row` attribute; the CUDA kernel picks its own lanes per row."""
    p = 1
    while p < 32 and runs % (2 * p) == 0 and runs // (2 * p) >= 4:
        p *= 2
    return p


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def dequantize(blocks: torch.Tensor, kind: str, shape: tuple, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The weights of `blocks` (uint8, a tensor of `shape` as the file holds it) as floats (blocks.py:397-404)."""
    require_cuda(blocks)
    *lead, rows, cols = shape
    mats = 1
    for v in lead:
        mats *= int(v)
    out = torch.empty(tuple(shape), dtype=dtype, device=blocks.device)
    check(_lib.lib().sc_dequant(_kind(kind), ptr(_contig(blocks)), mats, rows, cols, DTYPES[dtype], ptr(out), stream()),
          f"dequantize {kind} {tuple(shape)}")
    return out


class BlockSwitchLinear:
    """A stack of linear layers kept as the file's blocks; called like mlx-lm's `QuantizedSwitchLinear`
    (blocks.py:407-440)."""

    # From this many pairs on the reference unpacks the stack once and multiplies floats (blocks.py:410-413).
    # Kept, with the same meaning: the stack is dequantized (sc_dequant) and multiplied expert by expert.
    unpack_from = 5000

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, per_row: int | None = None):
        require_cuda(blocks)
        self.blocks, self.kind = _contig(blocks), kind
        self.num_experts, self.output_dims, self.input_dims = (int(v) for v in shape)
        _row_bytes(kind, self.input_dims)
        self.per_row = per_row or _threads_per_row(self.input_dims // 32)

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False) -> torch.Tensor:
        """x (..., 1, in), one row to each index or to each run of the last axis of `indices`."""
        require_cuda(x, indices)
        batch, k = tuple(x.shape[:-2]), (indices.shape[-1] if indices.ndim else 1)
        if batch == tuple(indices.shape):
            share = 1
        elif batch == (*indices.shape[:-1], 1):
            share = k
        else:
            x, share = torch.broadcast_to(x, (*indices.shape, 1, self.input_dims)), 1
        if indices.numel() >= self.unpack_from:
            return self._as_floats(x, indices, share)
        return self._pairs(x, indices, share)

    def _pairs(self, x: torch.Tensor, indices: torch.Tensor, share: int) -> torch.Tensor:
        """Each pair's product straight from the blocks (sc_expert_matvec)."""
        pairs = indices.numel()
        idx = _contig(indices.reshape(-1).to(torch.int32)).view(torch.uint32)
        xs = _contig(x.reshape(-1, self.input_dims))
        out = torch.empty((pairs, self.output_dims), dtype=x.dtype, device=x.device)
        check(_lib.lib().sc_expert_matvec(_kind(self.kind), ptr(self.blocks), self.num_experts, self.output_dims,
                                          self.input_dims, ptr(idx), pairs, share, ptr(xs), _dtype(xs), ptr(out),
                                          ptr(_lib.error_word(x.device)), stream()),
              f"BlockSwitchLinear {self.kind}")
        return out.reshape(*indices.shape, 1, self.output_dims)

    def _as_floats(self, x: torch.Tensor, indices: torch.Tensor, share: int) -> torch.Tensor:
        """Many pairs at once (the reference unpacks the stack for MLX's gather_mm, blocks.py:438-440). For a stack
        the tile products take, the pairs go through tiles_of and tile_matmul on the GPU, weights rounded to the
        activations' type as gather_mm's are: no host synchronization. Other shapes and float32 activations stay on
        the pair-at-a-time kernel, the weights exact: no float copy of the stack, no host synchronization."""
        if x.dtype in (torch.float16, torch.bfloat16) and tileable(self.kind, self.output_dims, self.input_dims):
            flat = indices.reshape(-1, 1)
            tiles, token, where = tiles_of(flat, self.num_experts)
            xs = x.reshape(-1, self.input_dims)
            a = xs.index_select(0, token.to(torch.int64) // share)  # a slot's pair p reads input row p // share
            c = tile_matmul(self.blocks, self.kind, (self.num_experts, self.output_dims, self.input_dims), a, tiles)
            out = c.index_select(0, where.to(torch.int64)).to(x.dtype)
            return out.reshape(*indices.shape, 1, self.output_dims)
        return self._pairs(x, indices, share)


def matvec_separate(experts: list, kind: str, rows: int, cols: int, x: torch.Tensor, share: int) -> torch.Tensor:
    """out[pair] = W[pair] . x, every pair's expert a buffer of its own (blocks.py:331-346). x (pairs / share,
    cols). Returns (pairs, rows)."""
    require_cuda(x, *experts)
    n = len(experts)
    bases = torch.tensor([e.data_ptr() for e in experts], dtype=torch.int64, device=x.device)
    xs = _contig(x.reshape(-1, cols))
    out = torch.empty((n, rows), dtype=x.dtype, device=x.device)
    check(_lib.lib().sc_expert_matvec_ptrs(_kind(kind), ptr(bases), n, rows, cols, share, ptr(xs), _dtype(xs), ptr(out),
                                           ptr(_lib.error_word(x.device)), stream()), f"matvec_separate {kind}")
    return out


def window_matvec(blocks: torch.Tensor, kind: str, rows: int, cols: int, x: torch.Tensor,
                  per_row: int | None = None) -> torch.Tensor:
    """out[t] = W . x[t] for one layer `blocks` of (rows, cols) and x (tokens, cols) (blocks.py:383-394)."""
    require_cuda(blocks, x)
    xs = _contig(x.reshape(-1, cols))
    tokens = xs.shape[0]
    out = torch.empty((tokens, rows), dtype=x.dtype, device=x.device)
    check(_lib.lib().sc_window_matvec(_kind(kind), ptr(_contig(blocks)), rows, cols, ptr(xs), _dtype(xs), tokens,
                                      ptr(out), ptr(_lib.error_word(x.device)), stream()), f"window_matvec {kind}")
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """mlx-lm's swiglu as blocks.py:230-238 restates it: sigmoid in float32 rounded to the type, two products
    in the type."""
    require_cuda(gate, up)
    g, u = _contig(gate), _contig(up.to(gate.dtype))
    out = torch.empty_like(g)
    check(_lib.lib().sc_swiglu(ptr(g), ptr(u), g.numel(), _dtype(g), ptr(out), stream()), "swiglu")
    return out


def matvec_glu(lin, idx: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, glu: int = 0) -> torch.Tensor | None:
    """`lin(swiglu(gate, up), idx)` for a BlockSwitchLinear, one pair to each row of gate and up, (pairs, out)
    (blocks.py:782-798). The reference returns None where its threadgroup memory is too small; the CUDA kernel
    takes any size, so this never does."""
    require_cuda(idx, gate, up)
    pairs = idx.shape[0]
    g, u = _contig(gate.reshape(pairs, -1)), _contig(up.reshape(pairs, -1).to(gate.dtype))
    flat = _contig(idx.reshape(-1).to(torch.int32)).view(torch.uint32)
    out = torch.empty((pairs, lin.output_dims), dtype=gate.dtype, device=gate.device)
    check(_lib.lib().sc_matvec_glu(_kind(lin.kind), ptr(lin.blocks), lin.num_experts, lin.output_dims, lin.input_dims,
                                   ptr(flat), pairs, ptr(g), ptr(u), _dtype(g), glu, ptr(out),
                                   ptr(_lib.error_word(gate.device)), stream()), f"matvec_glu {lin.kind}")
    return out


def gate_up(gate, up, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """swiglu(gate(x, indices), up(x, indices)) in one kernel (blocks.py:808-818 fused): x (..., in), one row to
    each run of the last axis of `indices`. Returns (pairs, inner). Gate and up stacks of one block type."""
    require_cuda(x, indices)
    k = indices.shape[-1]
    xs = _contig(x.reshape(-1, gate.input_dims))
    flat = _contig(indices.reshape(-1).to(torch.int32)).view(torch.uint32)
    pairs = flat.numel()
    h = torch.empty((pairs, gate.output_dims), dtype=x.dtype, device=x.device)
    check(_lib.lib().sc_expert_gate_up(_kind(gate.kind), ptr(gate.blocks), ptr(up.blocks), gate.num_experts,
                                       gate.output_dims, gate.input_dims, ptr(flat), pairs, k, ptr(xs), _dtype(xs),
                                       ptr(h), ptr(_lib.error_word(x.device)), stream()), f"gate_up {gate.kind}")
    return h


# ---- prompts: an expert's blocks a tile at a time, under the tcgen05 tensor cores


def tileable(kind: str, rows: int, cols: int) -> bool:
    """Whether `tile_matmul` takes a stack of such layers (blocks.py:511-513)."""
    return rows % ROWS_TILE == 0 and cols % COLS_TILE == 0 and cols % BLOCK[kind][0] == 0


def tile_matmul(blocks: torch.Tensor, kind: str, shape: tuple, a: torch.Tensor, tile_expert: torch.Tensor) -> torch.Tensor:
    """out[p] = W[expert of p's tile] . a[p] (blocks.py:516-536). a (P, cols) float16/bfloat16/float32, P a
    multiple of TOKENS_TILE; tile_expert (P / TOKENS_TILE,) names each tile's expert, or none (>= experts) for a
    tile to leave out: its rows of the result are then whatever was in memory. The weights are rounded to the type
    of `a` before they multiply; sums are float32. Returns (P, rows) float32."""
    require_cuda(blocks, a, tile_expert)
    experts, rows, cols = (int(v) for v in shape)
    p = a.shape[0]
    te = _contig(tile_expert.reshape(-1).to(torch.int64).clamp(0, experts).to(torch.int32)).view(torch.uint32)
    aa = _contig(a)
    out = torch.empty((p, rows), dtype=torch.float32, device=a.device)
    check(_lib.lib().sc_tile_matmul(_kind(kind), ptr(_contig(blocks)), experts, rows, cols, ptr(aa), _dtype(aa), p,
                                    ptr(te), ptr(out), ptr(_lib.error_word(a.device)), stream()),
          f"tile_matmul {kind} {tuple(shape)}")
    return out


def tiles_of(indices: torch.Tensor, experts: int) -> tuple:
    """The pairs of `indices` (..., k) laid out in tiles of TOKENS_TILE, each tile one expert's
    (blocks.py:539-563): (the expert of each tile, or `experts` for a tile nothing fills; the token of each slot;
    the slot of each pair), all worked out on the GPU in a number of tiles that depends only on the number of pairs."""
    require_cuda(indices)
    k = indices.shape[-1]
    flat = _contig(indices.reshape(-1))
    if flat.dtype not in _lib.IDX_DTYPES:
        flat = flat.to(torch.int64)
    pairs = flat.numel()
    most = pairs // TOKENS_TILE + min(experts, pairs)
    dev = indices.device
    tile_expert = torch.empty(most, dtype=torch.uint32, device=dev)
    token = torch.empty(most * TOKENS_TILE, dtype=torch.uint32, device=dev)
    where = torch.empty(pairs, dtype=torch.uint32, device=dev)
    lib = _lib.lib()
    ws_bytes = lib.sc_tiles_of_workspace(experts)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    check(lib.sc_tiles_of(ptr(flat), _lib.IDX_DTYPES[flat.dtype], pairs, k, experts, ptr(tile_expert), ptr(token),
                          ptr(where), ptr(ws), ws_bytes, stream()), "tiles_of")
    return tile_expert, token, where


def _tiled_glu(x: torch.Tensor, indices: torch.Tensor, up, gate, down) -> torch.Tensor:
    """The three products of a prompt's pairs through `tile_matmul`, the pairs in tiles (blocks.py:566-576). For
    float16 / bfloat16 on the tensor-core kernel the three run as one call (sc_tile_glu: swiglu and the unsort in
    the products' epilogues), with the same bits."""
    tiles, token, where = tiles_of(indices, gate.num_experts)
    a = x.reshape(-1, x.shape[-1]).index_select(0, token.to(torch.int64))
    if a.dtype in (torch.float16, torch.bfloat16):
        lib = _lib.lib()
        p, pairs = a.shape[0], indices.numel()
        n = lib.sc_tile_glu_workspace(p, gate.output_dims, _dtype(a))
        ws = torch.empty(n, dtype=torch.uint8, device=a.device)
        out = torch.empty((pairs, down.output_dims), dtype=a.dtype, device=a.device)
        rc = lib.sc_tile_glu(_kind(gate.kind), ptr(gate.blocks), _kind(up.kind), ptr(up.blocks), _kind(down.kind),
                             ptr(down.blocks), gate.num_experts, gate.input_dims, gate.output_dims, ptr(a), _dtype(a), p,
                             ptr(tiles), ptr(where), pairs, ptr(out), ptr(ws), n, ptr(_lib.error_word(a.device)),
                             stream())
        if rc != -8:  # SC_ERR_UNSUPPORTED: a product the tensor-core kernel does not take; compose the three
            check(rc, "tile_glu")
            return out.reshape(*indices.shape, down.output_dims)

    def product(lin, a):
        return tile_matmul(lin.blocks, lin.kind, (lin.num_experts, lin.output_dims, lin.input_dims), a, tiles)

    h = swiglu(product(gate, a).to(x.dtype), product(up, a).to(x.dtype))
    out = product(down, h).index_select(0, where.to(torch.int64)).to(x.dtype)
    return out.reshape(*indices.shape, down.output_dims)


# ---- Q2_0's table-of-sums entry points: the same answers from the direct decode kernels


class _Table:
    """What `lookup_table` returns: the activations, which the direct kernel reads as they are."""

    def __init__(self, x: torch.Tensor):
        self.x = x
        self.dtype = x.dtype
        self.shape = (x.shape[0], x.shape[1] // 2, 16)


def lookable(lin, dtype: torch.dtype) -> bool:
    return lin.kind == "Q2_0" and dtype == torch.float16


def lookup_table(x: torch.Tensor) -> _Table:
    """x (n, cols) float16 -> its 'table' (blocks.py:650-659)."""
    return _Table(x)


def lookup_table_glu(gate: torch.Tensor, up: torch.Tensor) -> _Table:
    """The 'table' of silu(gate) * up, both (n, cols) float16 (blocks.py:662-671): kept as gate and up, so that
    lookup_matvec works silu(g) * u out in float32 (blocks.py:609-611) in the kernel, as lookup_down_glu does,
    and gives its bits."""
    return _GluTable(gate, up)


class _GluTable(_Table):
    def __init__(self, gate: torch.Tensor, up: torch.Tensor):
        self.gate, self.up, self.dtype = gate, up, gate.dtype
        self.shape = (gate.shape[0], gate.shape[1] // 2, 16)


def lookup_matvec(lin, idx: torch.Tensor, table, share: int) -> torch.Tensor:
    """out[pair] = W[idx[pair]] . x[pair / share], x given as its `lookup_table` (blocks.py:674-695)."""
    if isinstance(table, _GluTable):
        return matvec_glu(lin, idx, table.gate, table.up, glu=1)
    x = table.x
    pairs = idx.shape[0]
    out = lin(x.reshape(-1, 1, 1, x.shape[-1]) if share > 1 else x.reshape(pairs, 1, x.shape[-1]),
              idx.reshape(-1, share) if share > 1 else idx.reshape(pairs))
    return out.reshape(pairs, lin.output_dims)


def lookup_down_glu(lin, idx: torch.Tensor, gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor | None:
    """`lookup_matvec(lin, idx, lookup_table_glu(gate, up), 1)` in one kernel (blocks.py:740-760)."""
    return matvec_glu(lin, idx, gate, up, glu=1)


def _lookup_glu(x: torch.Tensor, indices: torch.Tensor, up, gate, down) -> torch.Tensor:
    k = indices.shape[-1]
    idx = indices.reshape(-1)
    table = lookup_table(x.reshape(-1, x.shape[-1]))  # one for gate and up: they read the same input
    g, u = lookup_matvec(gate, idx, table, k), lookup_matvec(up, idx, table, k)
    out = lookup_down_glu(down, idx, g, u) if GLU_IN_DOWN else None
    if out is None:
        out = lookup_matvec(down, idx, lookup_table_glu(g, u), 1)
    return out.reshape(*indices.shape, down.output_dims)


def switch_glu(x: torch.Tensor, indices: torch.Tensor, up, gate, down) -> torch.Tensor:
    """down(silu(gate(x)) * up(x)) through each token's experts: x (..., in), indices (..., experts per token)
    (blocks.py:801-829)."""
    require_cuda(x, indices)
    if (indices.numel() >= TILES_FROM and x.dtype in (torch.float16, torch.bfloat16, torch.float32)
            and all(tileable(lin.kind, lin.output_dims, lin.input_dims) for lin in (up, gate, down))):
        return _tiled_glu(x, indices, up, gate, down)
    if indices.numel() >= LOOKUP_FROM and all(lookable(lin, x.dtype) for lin in (up, gate, down)):
        return _lookup_glu(x, indices, up, gate, down)
    blocky = all(isinstance(lin, BlockSwitchLinear) for lin in (up, gate, down))
    if (BLOCK_GLU and x.dtype in (torch.float16, torch.bfloat16) and blocky
            and indices.numel() < min(lin.unpack_from for lin in (up, gate, down))):
        flat = indices.reshape(-1)
        if gate.kind == up.kind and gate.output_dims == up.output_dims:
            h = gate_up(gate, up, x, indices)  # gate, up and swiglu in one kernel: the same bits as apart
            out = down(h.reshape(*indices.shape, 1, -1), indices)
            return out.reshape(*indices.shape, down.output_dims)
        x5 = x.unsqueeze(-2).unsqueeze(-2)
        g, u = gate(x5, indices), up(x5, indices)
        out = (matvec_glu(down, flat, g.reshape(flat.numel(), -1), u.reshape(flat.numel(), -1))
               if flat.numel() <= MATVEC_GLU_UPTO else None)
        if out is not None:
            return out.reshape(*indices.shape, down.output_dims)
        return down(swiglu(g, u), indices).squeeze(-2)
    # as mlx-lm's SwitchGLU (sorting the pairs changes nothing for these kernels)
    x5 = x.unsqueeze(-2).unsqueeze(-2)
    h = swiglu(gate(x5, indices), up(x5, indices))
    return down(h, indices).squeeze(-2)


class BlockSwitchGLU:
    """A layer's routed experts, called like mlx-lm's `SwitchGLU` (blocks.py:832-839)."""

    def __init__(self, gate: BlockSwitchLinear, up: BlockSwitchLinear, down: BlockSwitchLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        return switch_glu(x, indices, self.up_proj, self.gate_proj, self.down_proj)
