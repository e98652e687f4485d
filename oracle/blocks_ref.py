"""CPU oracle for the quantized-expert hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy float32, the arithmetic of strata-mlx's block decoders and of the MoE
routing/combine kernels, so that the CUDA library can be checked against it. Nothing in the product imports
it: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may.

Pinning: the restated decoders are checked against gguf-py 0.19.0's ``gguf.quants.dequantize`` (the oracle of
the reference's own tests, tests/test_blocks.py:13-19) for the nine types gguf-py has, and against the numpy
Q2_0 decoder of tests/test_gguf.py:33-38 for Q2_0; tests/golden/ holds vectors made by those decoders.

Reference citations are paths inside the strata-mlx project.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

# strata_mlx/blocks.py:35-38 -- type -> (weights per block, bytes per block)
BLOCK = {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
         "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56), "Q2_0": (64, 18),
         "Q3_K": (256, 110)}
# strata_mlx/gguf.py:27 -- the dense type the synthetic decoder's attention projections use
DENSE = {"Q8_0": (32, 34)}

# strata_mlx/gguf.py:34
KVALUES_IQ4NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int16)

_tables: dict = {}


def table(name: str) -> np.ndarray:
    """ggml's codebooks as gguf-py builds them (strata_mlx/blocks.py:275-289): grids as uint8 rows, the IQ1 grid
    shifted by +1 so that its -1/0/1 are 0/1/2, ksigns as 128 bytes."""
    if name not in _tables:
        from gguf import quants
        if name == "ksigns":
            _tables[name] = np.frombuffer(quants.IQ2_XXS.ksigns, dtype=np.uint8).copy()
        elif name == "kvalues":
            _tables[name] = KVALUES_IQ4NL.copy()
        else:
            cls = {"iq3s_grid": quants.IQ3_S, "iq3xxs_grid": quants.IQ3_XXS, "iq2s_grid": quants.IQ2_S,
                   "iq2xs_grid": quants.IQ2_XS, "iq2xxs_grid": quants.IQ2_XXS, "iq1_grid": quants.IQ1_M}[name]
            cls.init_grid()
            g = cls.grid.reshape(cls.grid_shape) + (1 if name == "iq1_grid" else 0)
            _tables[name] = g.astype(np.int16).astype(np.uint8)
    return _tables[name]


def _half(b: np.ndarray) -> np.ndarray:
    """strata_mlx/blocks.py:41-43 half_at: two little-endian bytes as a float16, widened exactly to float32."""
    return np.ascontiguousarray(b[..., :2]).view("<f2")[..., 0].astype(F32)


def _u16(b: np.ndarray) -> np.ndarray:
    return b[..., 0].astype(np.uint32) | (b[..., 1].astype(np.uint32) << 8)


def _u32(b: np.ndarray) -> np.ndarray:
    return (b[..., 0].astype(np.uint32) | (b[..., 1].astype(np.uint32) << 8) | (b[..., 2].astype(np.uint32) << 16)
            | (b[..., 3].astype(np.uint32) << 24))


def _signed(v: np.ndarray, bits: np.ndarray) -> np.ndarray:
    """(sign >> j) & 1 ? -v : v -- negation is exact, so the bits are the reference's."""
    return np.where(bits.astype(bool), -v, v).astype(F32)


def _runs(kind: str, blocks: np.ndarray) -> np.ndarray:
    """Every run of 32 weights of `blocks` (n_blocks, block_bytes) -> (n_blocks, runs_per_block, 32) float32, each
    run computed as the reference's unpack32 computes it (strata_mlx/blocks.py:57-193)."""
    b = blocks
    n = b.shape[0]
    if kind == "Q2_0":  # blocks.py:58-67
        d = _half(b)[:, None, None]
        codes = b[:, 2:18].reshape(n, 2, 8)
        c = np.stack([(codes >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(n, 2, 32)
        return d * (c.astype(F32) - F32(1))
    if kind == "IQ4_NL":  # blocks.py:69-77
        d = _half(b)[:, None]
        kv = table("kvalues").astype(F32)
        q = b[:, 2:18]
        w = np.concatenate([d * kv[q & 15], d * kv[q >> 4]], axis=-1)
        return w.reshape(n, 1, 32)
    if kind == "IQ4_XS":  # blocks.py:78-88
        kv = table("kvalues").astype(F32)
        ib = np.arange(8)
        ls = ((b[:, 4 + ib // 2].astype(np.uint32) >> (4 * (ib % 2))) & 15) | (((_u16(b[:, 2:4])[:, None] >> (2 * ib)) & 3) << 4)
        d = _half(b)[:, None] * (ls.astype(F32) - F32(32))  # (n, 8)
        q = b[:, 8:136].reshape(n, 8, 16)
        return np.concatenate([d[..., None] * kv[q & 15], d[..., None] * kv[q >> 4]], axis=-1)
    if kind == "IQ3_S":  # blocks.py:89-101
        grid = table("iq3s_grid").astype(F32)
        ib = np.arange(8)
        sc = (b[:, 106 + ib // 2].astype(np.uint32) >> (4 * (ib % 2))) & 15
        d = _half(b)[:, None] * (F32(1) + F32(2) * sc.astype(F32))  # 1 + 2*s is an exact integer
        high = b[:, 66:74].astype(np.uint32)  # (n, 8)
        l = np.arange(8)
        qs = b[:, 2:66].reshape(n, 8, 8).astype(np.uint32)
        gidx = qs | (((high[:, :, None] >> l) & 1) << 8)  # (n, 8, 8)
        g = grid[gidx]  # (n, 8, 8, 4)
        sb = b[:, 74:106].reshape(n, 8, 4).astype(np.uint32)
        sign = sb[:, :, l // 2] >> (4 * (l % 2))  # (n, 8, 8)
        bits = (sign[..., None] >> np.arange(4)) & 1
        v = d[:, :, None, None] * g
        return _signed(v, bits).reshape(n, 8, 32)
    if kind == "IQ3_XXS":  # blocks.py:103-115
        grid = table("iq3xxs_grid").astype(F32)
        ks = table("ksigns").astype(np.uint32)
        aux = _u32(b[:, 66:98].reshape(n, 8, 4))  # (n, 8)
        d = _half(b)[:, None] * (F32(0.5) + (aux >> 28).astype(F32)) * F32(0.5)
        l = np.arange(8)
        g = grid[b[:, 2:66].reshape(n, 8, 8)]  # (n, 8, 8, 4)
        sign = ks[(aux[:, :, None] >> (7 * (l // 2))) & 127] >> (4 * (l % 2))
        bits = (sign[..., None] >> np.arange(4)) & 1
        return _signed(d[:, :, None, None] * g, bits).reshape(n, 8, 32)
    if kind == "IQ2_S":  # blocks.py:117-131
        grid = table("iq2s_grid").astype(F32)
        d = _half(b) * F32(0.25)
        high = b[:, 66:74].astype(np.uint32)
        scales = b[:, 74:82].astype(np.uint32)
        l = np.arange(4)
        qs = b[:, 2:34].reshape(n, 8, 4).astype(np.uint32)
        gidx = qs | (((high[:, :, None] >> (2 * l)) & 3) << 8)
        g = grid[gidx]  # (n, 8, 4, 8)
        sign = b[:, 34:66].reshape(n, 8, 4).astype(np.uint32)
        s = np.where(l < 2, scales[:, :, None] & 15, scales[:, :, None] >> 4)
        dl = d[:, None, None] * (F32(0.5) + s.astype(F32))
        bits = (sign[..., None] >> np.arange(8)) & 1
        return _signed(dl[..., None] * g, bits).reshape(n, 8, 32)
    if kind == "IQ2_XS":  # blocks.py:132-147
        grid = table("iq2xs_grid").astype(F32)
        ks = table("ksigns").astype(np.uint32)
        d = _half(b) * F32(0.25)
        scales = b[:, 66:74].astype(np.uint32)
        q = _u16(b[:, 2:66].reshape(n, 8, 4, 2))  # (n, 8, 4)
        g = grid[q & 511]
        sign = ks[q >> 9]
        l = np.arange(4)
        s = np.where(l < 2, scales[:, :, None] & 15, scales[:, :, None] >> 4)
        dl = d[:, None, None] * (F32(0.5) + s.astype(F32))
        bits = (sign[..., None] >> np.arange(8)) & 1
        return _signed(dl[..., None] * g, bits).reshape(n, 8, 32)
    if kind == "IQ2_XXS":  # blocks.py:148-161
        grid = table("iq2xxs_grid").astype(F32)
        ks = table("ksigns").astype(np.uint32)
        q = b[:, 2:66].reshape(n, 8, 8)
        aux = _u32(q[:, :, 4:8])  # (n, 8)
        d = _half(b)[:, None] * (F32(0.5) + (aux >> 28).astype(F32)) * F32(0.25)
        l = np.arange(4)
        g = grid[q[:, :, :4]]  # (n, 8, 4, 8)
        sign = ks[(aux[:, :, None] >> (7 * l)) & 127]
        bits = (sign[..., None] >> np.arange(8)) & 1
        return _signed(d[:, :, None, None] * g, bits).reshape(n, 8, 32)
    if kind == "Q3_K":  # blocks.py:48-53 (q3k_scale) and :164-175
        r = np.arange(8)
        s = b[:, 96:108].astype(np.uint32)

        def q3k_scale(k):
            p, word = k % 4, k // 4
            low = np.where(word < 2, s[:, 4 * (word % 2) + p] & 15, s[:, 4 * (word % 2) + p] >> 4)
            # word < 2: byte 4*word + p; else byte 4*(word-2) + p -- word % 2 covers both
            return ((low | (((s[:, 8 + p] >> (2 * word)) & 3) << 4)).astype(np.int32) - 32).astype(F32)

        d = _half(b[:, 108:110])
        s0 = np.stack([d * q3k_scale(2 * rr) for rr in r], axis=1)  # (n, 8)
        s1 = np.stack([d * q3k_scale(2 * rr + 1) for rr in r], axis=1)
        qb = b[:, 32:96].reshape(n, 2, 32).astype(np.int32)
        q = qb[:, r // 4, :] >> (2 * (r % 4))[None, :, None]  # (n, 8, 32)
        hm = (b[:, None, 0:32].astype(np.int32) >> r[None, :, None]) & 1
        v = (q & 3) - np.where(hm == 1, 0, 4)
        scale = np.where(np.arange(32) < 16, s0[..., None], s1[..., None])
        return scale * v.astype(F32)
    if kind == "IQ1_M":  # blocks.py:176-193
        grid = table("iq1_grid").astype(F32)
        w16 = _u16(b[:, 48:56].reshape(n, 4, 2))  # (n, 4)
        packed = (w16[:, 0] >> 12) | ((w16[:, 1] >> 8) & 0x00F0) | ((w16[:, 2] >> 4) & 0x0F00) | (w16[:, 3] & 0xF000)
        d = packed.astype(np.uint16).view(np.float16).astype(F32)
        ib = np.arange(8)
        scales = w16[:, ib // 2] >> (6 * (ib % 2))  # (n, 8)
        l = np.arange(4)
        qh = b[:, 32:48].reshape(n, 8, 2).astype(np.uint32)
        high = (qh[:, :, l // 2] >> (4 * (l % 2))) & 15  # (n, 8, 4)
        qs = b[:, 0:32].reshape(n, 8, 4).astype(np.uint32)
        g = grid[qs | ((high & 7) << 8)]  # (n, 8, 4, 8)
        dl = d[:, None, None] * (F32(2) * ((scales[:, :, None] >> (3 * (l // 2))) & 7).astype(F32) + F32(1))
        delta = np.where(high & 8, F32(-1.125), F32(-0.875)).astype(F32)
        return (dl[..., None] * (g + delta[..., None])).astype(F32).reshape(n, 8, 32)
    if kind == "Q8_0":  # strata_mlx/gguf.py:203-206: d * int8 code
        d = _half(b)[:, None]
        return (d * b[:, 2:34].view(np.int8).astype(F32)).reshape(n, 1, 32)
    raise ValueError(f"unknown block type {kind}")


def block_info(kind: str) -> tuple:
    if kind in BLOCK:
        return BLOCK[kind]
    if kind in DENSE:
        return DENSE[kind]
    raise ValueError(f"unknown block type {kind}")


def row_bytes(kind: str, cols: int) -> int:
    per_block, block_bytes = block_info(kind)
    if cols % per_block:
        raise ValueError(f"{kind}: rows of {cols} weights do not end on a block of {per_block}")
    return cols // per_block * block_bytes


def dequantize(blocks: np.ndarray, kind: str, shape: tuple) -> np.ndarray:
    """strata_mlx/blocks.py:397-404: every weight of a stack of `shape` as float32, bit for bit as unpack32."""
    per_block, block_bytes = block_info(kind)
    *lead, rows, cols = shape
    row_bytes(kind, cols)
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, block_bytes)
    return _runs(kind, b).reshape(shape)


# ---- products, in float64 unless stated: the tolerance of a float32 sum is asserted by the tests


def matvec(w: np.ndarray, idx: np.ndarray, x: np.ndarray, share: int) -> np.ndarray:
    """strata_mlx/blocks.py:196-220: out[pair, row] = W[idx[pair], row, :] . x[pair // share]; float64 sums."""
    idx = np.asarray(idx).reshape(-1)
    xs = np.asarray(x, dtype=np.float64).reshape(-1, w.shape[-1])
    return np.einsum("poi,pi->po", w[idx].astype(np.float64), xs[np.arange(len(idx)) // share])


def round_to(a: np.ndarray, dtype) -> np.ndarray:
    """Round float32 values to an activation type (numpy has float16; bfloat16 by round-to-nearest-even)."""
    a = np.asarray(a, dtype=F32)
    if dtype in ("float32", np.float32):
        return a
    if dtype in ("float16", np.float16):
        return a.astype(np.float16).astype(F32)
    if dtype == "bfloat16":
        u = a.view(np.uint32).astype(np.uint64)
        nan = np.isnan(a)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        out = r.astype(np.uint32).view(F32)
        return np.where(nan, a, out).astype(F32)
    raise ValueError(dtype)


def swiglu(g: np.ndarray, u: np.ndarray, dtype) -> np.ndarray:
    """mlx-lm's swiglu as strata_mlx/blocks.py:230-238 restates it: sigmoid in float32 rounded to the
    activations' type, then g * sig and (g * sig) * up, each product rounded to that type."""
    g = round_to(g, dtype)
    u = round_to(u, dtype)
    with np.errstate(over="ignore"):  # exp of a large |g| is inf: y is then 0, as in float32
        y = F32(1) / (F32(1) + np.exp(np.abs(g)).astype(F32))
    sig = round_to(np.where(g < 0, y, F32(1) - y), dtype)
    a = round_to(g * sig, dtype)
    return round_to(a * u, dtype)


def router(w16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """strata_mlx/fused.py:334-390 WindowLinear: float16 weights times x, float64 sums (asserted to 1e-5)."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(w16, dtype=np.float64).T


def top_k(logits: np.ndarray, k: int) -> np.ndarray:
    """strata_mlx/fused.py:400-436: the k largest of each row, largest first, ties to the lower index -- the
    order of a stable sort on -logits (argpartition's order in the reference's test, tests/test_fused.py:109-120)."""
    lg = np.asarray(logits, dtype=F32)
    order = np.argsort(-lg, axis=-1, kind="stable")
    return order[..., :k].astype(np.uint32)


def softmax_topk(logits: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """strata_mlx/fused.py:491: softmax over the chosen logits, float32 (precise)."""
    sel = np.take_along_axis(np.asarray(logits, dtype=np.float64), idx.astype(np.int64), axis=-1)
    e = np.exp(sel - sel.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True)).astype(F32)


def moe_combine(y: np.ndarray, w: np.ndarray, g: np.ndarray, s: np.ndarray, dtype) -> np.ndarray:
    """strata_mlx/fused.py:448-481: OutT(sum_k y_k*w_k) + OutT(OutT(sigmoid(g)) * s), the products of each token
    added in MLX's col_reduce order: 8 partial sums (partial j takes k = j, j+8, ...), then in order."""
    return moe_combine_parts(y, w, g, s, dtype)["out"]


def gate_of(g: np.ndarray, dtype) -> np.ndarray:
    """The shared expert's gate as the combine uses it (fused.py:493): sigmoid in float32, rounded to the type."""
    gg = np.asarray(g, dtype=F32)
    with np.errstate(over="ignore"):
        return round_to(F32(1) / (F32(1) + np.exp(-gg).astype(F32)), dtype)


def moe_combine_parts(y: np.ndarray, w: np.ndarray, g: np.ndarray, s: np.ndarray, dtype, gate=None) -> dict:
    """moe_combine with its two rounded terms: {"out", "routed" = OutT(sum_k y_k w_k), "shared" = OutT(gate * s),
    "gate" = OutT(sigmoid(g))}, each (tokens, D) (gate (tokens, 1)). `gate`, when given, replaces the sigmoid's
    rounded value (a test's alternative for a gate on a rounding edge)."""
    y = np.asarray(y, dtype=F32)
    w = np.asarray(w, dtype=F32)
    *lead, K, D = y.shape
    yy = y.reshape(-1, K, D)
    ww = w.reshape(-1, K)
    acc = np.zeros((yy.shape[0], D), dtype=F32)
    for j in range(min(8, K)):
        part = np.zeros((yy.shape[0], D), dtype=F32)
        for k in range(j, K, 8):
            part = (yy[:, k] * ww[:, k : k + 1]).astype(F32) + part  # contraction off: product rounded first
        acc = part if j == 0 else (part + acc).astype(F32)
    routed = round_to(acc, dtype)
    if gate is None:
        gate = gate_of(np.asarray(g, dtype=F32).reshape(-1, 1), dtype)
    gate = np.asarray(gate, dtype=F32).reshape(-1, 1)
    shared = round_to(gate * np.asarray(s, dtype=F32).reshape(-1, D), dtype)
    out = round_to(routed + shared, dtype)
    return {"out": out.reshape(*lead, D), "routed": routed.reshape(*lead, D), "shared": shared.reshape(*lead, D),
            "gate": gate}


TOKENS_TILE = 16  # strata_mlx/blocks.py:463


def tiles_of_check(indices: np.ndarray, experts: int, tile_expert, token, where) -> None:
    """The invariants of strata_mlx/blocks.py:539-563 as tests/test_blocks.py:177-195 states them."""
    k = indices.shape[-1]
    flat = np.asarray(indices).reshape(-1)
    pairs = len(flat)
    most = pairs // TOKENS_TILE + min(experts, pairs)
    assert len(tile_expert) == most and len(token) == most * TOKENS_TILE and len(where) == pairs
    assert len(set(where.tolist())) == pairs
    np.testing.assert_array_equal(tile_expert[where // TOKENS_TILE], flat)
    np.testing.assert_array_equal(token[where], np.arange(pairs) // k)
    used = np.zeros(len(tile_expert), dtype=bool)
    used[where // TOKENS_TILE] = True
    assert (tile_expert[~used] >= experts).all() and (tile_expert[used] < experts).all()
    assert used.sum() == sum(-(-c // TOKENS_TILE) for c in np.bincount(flat, minlength=experts))


def tile_matmul(w: np.ndarray, a: np.ndarray, tile_expert: np.ndarray, dtype) -> np.ndarray:
    """strata_mlx/blocks.py:516-536: C[p] = W[tile expert of p] . a[p] with the weights rounded to a's type
    (blocks.py:492); float64 sums. Rows of tiles that name no expert are returned as NaN (unspecified)."""
    wr = round_to(w, dtype).astype(np.float64)
    P = a.shape[0]
    out = np.full((P, w.shape[1]), np.nan)
    ad = np.asarray(a, dtype=np.float64)
    for t, e in enumerate(np.asarray(tile_expert).reshape(-1)):
        if e < w.shape[0]:
            out[16 * t : 16 * t + 16] = ad[16 * t : 16 * t + 16] @ wr[e].T
    return out


def moe_layer(x, router_w, shared_gate_w, gate, up, down, sgate, sup, sdown, k: int, dtype):
    """One MoE block as strata_mlx/fused.py:487-497 computes it: router (float32 logits), top-k, softmax over the
    chosen logits, the routed SwiGLU experts (blocks.py:801-829, each product rounded to the activations' type),
    the shared expert and its sigmoid gate, and moe_combine. Weights are float32 arrays (dequantized blocks);
    x is (T, H) float32 holding values of `dtype`. Returns (out (T, H) float32, idx, w)."""
    x = round_to(x, dtype)
    logits = router(router_w, x).astype(F32)
    idx = top_k(logits, k)
    wts = softmax_topk(logits, idx)
    T, H = x.shape
    flat = idx.reshape(-1)
    g = round_to(matvec(gate, flat, x, k), dtype)
    u = round_to(matvec(up, flat, x, k), dtype)
    h = swiglu(g, u, dtype)
    y = round_to(matvec(down, flat, h, 1), dtype).reshape(T, k, H)
    if sgate is not None:
        zero = np.zeros(T, dtype=np.int64)
        sg = round_to(matvec(sgate[None], zero, x, 1), dtype)
        su = round_to(matvec(sup[None], zero, x, 1), dtype)
        s = round_to(matvec(sdown[None], zero, swiglu(sg, su, dtype), 1), dtype)
        gs = round_to(router(shared_gate_w.reshape(1, -1), x), dtype).reshape(T)
    else:
        s = np.zeros((T, H), dtype=F32)
        gs = np.full(T, -np.inf, dtype=F32)
    return moe_combine(y, wts, gs, s, dtype), idx, wts


def expert_rows(blocks: np.ndarray, kind: str, e: int, rows: int, cols: int) -> np.ndarray:
    """Expert e of a (experts, rows, cols) stack of blocks, dequantized: (rows, cols) float32."""
    rb = row_bytes(kind, cols)
    return dequantize(np.asarray(blocks)[e * rows * rb : (e + 1) * rows * rb], kind, (rows, cols))


def moe_layer_blocks(x, L: dict, hidden: int, inter: int, k: int, dtype, shared_inter: int = 0) -> dict:
    """moe_layer on a layer given as blocks (synthetic.layer_numpy's dict), dequantizing only the experts the window
    chose: bounded work at benchmark sizes (512 experts). Returns {"out", "idx", "w", "routed", "shared", "gate",
    "s", "y", "gs"}: the output, the routes, and the combine's inputs and rounded terms (moe_combine_parts)."""
    kg, ku, kd = L["kinds"]
    x = round_to(x, dtype)
    T, H = x.shape
    logits = router(L["router"], x).astype(F32)
    idx = top_k(logits, k)
    wts = softmax_topk(logits, idx)
    y = np.zeros((T, k, H), dtype=F32)
    for e in np.unique(idx):
        wg, wu = expert_rows(L["gate"], kg, e, inter, H), expert_rows(L["up"], ku, e, inter, H)
        wd = expert_rows(L["down"], kd, e, H, inter)
        for t, j in zip(*np.nonzero(idx == e)):
            xt = x[t].astype(np.float64)
            g = round_to((wg.astype(np.float64) @ xt).astype(F32), dtype)
            u = round_to((wu.astype(np.float64) @ xt).astype(F32), dtype)
            h = swiglu(g, u, dtype)
            y[t, j] = round_to((wd.astype(np.float64) @ h.astype(np.float64)).astype(F32), dtype)
    if shared_inter:
        sk = L.get("shared_kinds", L["kinds"])
        sg = dequantize(L["sgate"], sk[0], (shared_inter, H))
        su = dequantize(L["sup"], sk[1], (shared_inter, H))
        sd = dequantize(L["sdown"], sk[2], (H, shared_inter))
        xd = x.astype(np.float64)
        h = swiglu(round_to((xd @ sg.T.astype(np.float64)).astype(F32), dtype),
                   round_to((xd @ su.T.astype(np.float64)).astype(F32), dtype), dtype)
        s = round_to((h.astype(np.float64) @ sd.T.astype(np.float64)).astype(F32), dtype)
        gs = round_to(router(L["shared_gate"].reshape(1, -1), x), dtype).reshape(T)
    else:
        s = np.zeros((T, H), dtype=F32)
        gs = np.full(T, -np.inf, dtype=F32)
    parts = moe_combine_parts(y, wts, gs, s, dtype)
    parts.update(idx=idx, w=wts, s=s, y=y, gs=gs)
    return parts
