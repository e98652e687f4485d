"""A synthetic MoE decoder around the library's MoE blocks: the stack BASELINE configurations 4 and 5 time (strata-mlx
runs a real model's trunk through its engine, strata_mlx/engine.py:276-279 and :710-749, with the MoE blocks of
fused.py:487-497 in every layer; no model file exists here, so the trunk is a synthetic stand-in of the same shape).

A layer is pre-norm attention then a pre-norm MoE block, each added to the residual stream:

    h = rmsnorm(x); q, k, v = h Wq, h Wk, h Wv; RoPE; k, v into the paged cache
    x = x + attention(q, cache) Wo                 grouped-query attention, sc_paged_attention
    x = x + moe(rmsnorm(x))                        the MoE block: router, top-10, experts from GGUF blocks, shared
                                                   expert, combine (MoEDecodeLayer, or expert parallel)

Attention is replicated on every rank and is not the path under test: the dense projections are bfloat16 matrices
multiplied by cuBLAS (configuration 4) or Q8_0 blocks through the library's window matvec (configuration 5), the
attention is the library's paged kernel. The MoE blocks are the library's decode kernels; expert parallel over the
ranks of a process group when one is given:

    replicated   every rank holds the same window (configuration 4: one sequence, a verify pass of 1 + 4 tokens):
                 each rank runs its experts' pairs, an NCCL all-reduce sums the pairs' outputs, every rank combines
    per rank     each rank holds its own sequence (configuration 5: batch = ranks): the window of the MoE block is
                 every rank's token (ep.EPMoEDecodeLayer: all-gather, all-reduce)

The cache's positions and the window's token ids live on the device, so that a pass replays from a CUDA graph: the
graph is captured once, and `advance` moves the position on the device between replays.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, stream

HEAD_DIM, PAGE = 256, 16


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor, out: torch.Tensor,
                eps: float = 1e-6) -> torch.Tensor:
    """x += delta (rounded to x's type; skipped for None), out = rmsnorm(x) w: one kernel (sc_add_rmsnorm)."""
    rows, cols = x.shape
    check(_lib.lib().sc_add_rmsnorm(ptr(x), ptr(delta), ptr(w), rows, cols, eps, _lib.DTYPES[x.dtype], ptr(out),
                                    stream()), "sc_add_rmsnorm")
    return out


class PagedCache:
    """Keys and values of one sequence for every layer, in pages of PAGE tokens: k, v (layers, pages, PAGE, kv_heads,
    HEAD_DIM) bfloat16; `table` the sequence's pages in order (a shuffled list: a sequence's pages need not be
    adjacent); `pos` (device int32) the tokens held."""

    def __init__(self, layers: int, kv_heads: int, max_tokens: int, device, seed: int = 0):
        self.pages = -(-max_tokens // PAGE)
        self.max_tokens = self.pages * PAGE
        shape = (layers, self.pages, PAGE, kv_heads, HEAD_DIM)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.table = torch.randperm(self.pages, generator=g).to(torch.int32).to(device)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.kv_heads = kv_heads

    def fill_random(self, tokens: int, seed: int = 1) -> None:
        """Stands in for the prefill of a prompt of random tokens: the first `tokens` positions of every layer get
        N(0, 1) keys and values (what random tokens' keys and values are like after the norm), without computing them."""
        g = torch.Generator(device=self.k.device).manual_seed(seed)
        n_pages = -(-tokens // PAGE)
        for buf in (self.k, self.v):
            if n_pages == self.pages:
                buf.normal_(generator=g)
                continue
            pages = self.table[:n_pages].long()
            for l in range(buf.shape[0]):
                buf[l, pages] = torch.randn(buf[l, pages].shape, generator=g, device=buf.device).to(torch.bfloat16)
        self.pos.fill_(tokens)

    def slots(self, t: int) -> torch.Tensor:
        """Flat slots (page * PAGE + offset) of the next t positions, from the device position."""
        p = self.pos.long() + torch.arange(t, device=self.pos.device)
        return self.table.long()[p // PAGE] * PAGE + p % PAGE


class Rope:
    """Rotary position embedding on the halves of each head (rotate_half form), base 10000."""

    def __init__(self, max_pos: int, device, base: float = 10000.0):
        inv = 1.0 / (base ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float64) / HEAD_DIM))
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos = ang.cos().float().to(device)
        self.sin = ang.sin().float().to(device)

    def __call__(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        c, s = self.cos[positions][:, None, :], self.sin[positions][:, None, :]  # (t, 1, D/2)
        xf = x.float()
        a, b = xf[..., : HEAD_DIM // 2], xf[..., HEAD_DIM // 2 :]
        return torch.cat([a * c - b * s, b * c + a * s], dim=-1).to(x.dtype)


class Dense:
    """A dense projection: bfloat16 weights (out, in) through cuBLAS, or Q8_0 blocks through sc_window_matvec."""

    def __init__(self, out_f: int, in_f: int, kind: str, gen: torch.Generator, device, sigma: float = 0.02):
        self.kind, self.out_f, self.in_f = kind, out_f, in_f
        w = torch.randn((out_f, in_f), generator=gen, device=device) * sigma
        if kind == "bf16":
            self.w = w.to(torch.bfloat16)
            self.nbytes = self.w.numel() * 2
        elif kind == "Q8_0":  # d = max|w| / 127 per 32 weights, codes round(w / d) (strata_mlx/gguf.py:203-206 form)
            blk = w.reshape(out_f, in_f // 32, 32)
            d = (blk.abs().amax(-1, keepdim=True) / 127.0).clamp_min(1e-12).to(torch.float16)
            q = torch.round(blk / d.float()).clamp(-127, 127).to(torch.int8)
            raw = torch.empty((out_f, in_f // 32, 34), dtype=torch.uint8, device=device)
            raw[..., :2] = d.view(torch.uint8).reshape(out_f, in_f // 32, 2)
            raw[..., 2:] = q.view(torch.uint8)
            self.w = raw.reshape(-1)
            self.nbytes = self.w.numel()
        else:
            raise ValueError(f"dense kind {kind}")

    @staticmethod
    def stacked(parts: list) -> "Dense":
        """One projection whose outputs are the parts' outputs in turn."""
        d = Dense.__new__(Dense)
        d.kind, d.in_f = parts[0].kind, parts[0].in_f
        d.out_f = sum(p.out_f for p in parts)
        d.w = torch.cat([p.w for p in parts], 0)
        d.nbytes = sum(p.nbytes for p in parts)
        return d

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.kind == "bf16":
            return x @ self.w.T
        from .blocks import window_matvec

        return window_matvec(self.w, "Q8_0", self.out_f, self.in_f, x)

    def floats(self) -> torch.Tensor:
        if self.kind == "bf16":
            return self.w.float()
        from .blocks import dequantize

        return dequantize(self.w, "Q8_0", (self.out_f, self.in_f))


class Attention:
    def __init__(self, hidden: int, q_heads: int, kv_heads: int, dense: str, gen, device):
        self.hq, self.hkv = q_heads, kv_heads
        self.wq = Dense(q_heads * HEAD_DIM, hidden, dense, gen, device)
        self.wk = Dense(kv_heads * HEAD_DIM, hidden, dense, gen, device)
        self.wv = Dense(kv_heads * HEAD_DIM, hidden, dense, gen, device)
        self.wo = Dense(hidden, q_heads * HEAD_DIM, dense, gen, device)
        # q, k and v in one product: their rows stacked (blocks stay whole rows, so the bytes are concatenated)
        self.wqkv = Dense.stacked([self.wq, self.wk, self.wv])
        self.nbytes = sum(d.nbytes for d in (self.wq, self.wk, self.wv, self.wo))

    def __call__(self, h: torch.Tensor, cache: PagedCache, layer: int, rope: Rope, ws: torch.Tensor,
                 ctx: torch.Tensor) -> torch.Tensor:
        t = h.shape[0]
        qkv = self.wqkv(h)
        nq, nk = self.hq * HEAD_DIM, self.hkv * HEAD_DIM
        q = qkv[:, :nq].contiguous()
        k = qkv[:, nq : nq + nk].contiguous()
        v = qkv[:, nq + nk :].contiguous()
        lib = _lib.lib()
        # RoPE on q (in place) and k, k and v into the cache at the positions pos .. pos + t - 1
        check(lib.sc_rope_cache(ptr(q), ptr(k), ptr(v), t, self.hq, self.hkv, HEAD_DIM, ptr(rope.cos), ptr(rope.sin),
                                ptr(cache.pos), ptr(cache.table), PAGE, ptr(cache.k[layer]), ptr(cache.v[layer]),
                                _lib.DTYPES[h.dtype], stream()), "sc_rope_cache")
        out = torch.empty((t, self.hq, HEAD_DIM), dtype=h.dtype, device=h.device)
        check(lib.sc_paged_attention(ptr(q), ptr(cache.k[layer]), ptr(cache.v[layer]), ptr(cache.table), ptr(ctx),
                                     cache.max_tokens, t, self.hq, self.hkv, HEAD_DIM, 1.0 / math.sqrt(HEAD_DIM),
                                     ptr(out), ptr(ws), ws.numel(), stream()), "sc_paged_attention")
        return self.wo(out.reshape(t, self.hq * HEAD_DIM))


class ReplicatedEPMoE:
    """The MoE block expert parallel over a window every rank holds (configuration 4): sc_moe_decode_layer_ep on the
    rank's experts, an NCCL all-reduce of the pairs' outputs (each non-zero on one rank), the combine on every rank.
    The same bits as the single-device block."""

    def __init__(self, base, e0: int, e1: int, group=None):
        self.base, self.e0, self.e1, self.group = base, e0, e1, group
        self._y: dict = {}

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        T = x.shape[0]
        ws = self.base.workspace(T, x.device)
        y = self._y.get(T)
        if y is None:
            y = torch.empty((T, self.base.top_k, self.base.hidden), dtype=x.dtype, device=x.device)
            self._y[T] = y
        lib = _lib.lib()
        check(lib.sc_moe_decode_layer_ep(self.base.layer_ref(), ptr(x), T, self.e0, self.e1, ptr(y), ptr(ws), ws.numel(),
                                         stream()), "sc_moe_decode_layer_ep")
        dist.all_reduce(y, group=self.group)
        out = torch.empty_like(x)
        check(lib.sc_moe_decode_combine(self.base.layer_ref(), ptr(y), T, ptr(out), ptr(ws), ws.numel(), stream()),
              "sc_moe_decode_combine")
        return out


class SyntheticDecoder:
    """`n_layers` layers of attention (16 query / 2 key-value heads of 256, RoPE, paged cache) and the MoE block of
    configuration 2 (512 experts, top-10, SwiGLU inner 512, shared expert 512), hidden 2048, a bfloat16 embedding and
    output head. kinds[l]: layer l's expert block type; dense: "bf16" or "Q8_0" projections. With `group` (a torch
    process group of G ranks) the experts are sharded over the ranks: mode "replicated" (every rank holds the same
    window) or "per_rank" (each rank its own sequence). Weights are seeded synthetic ones, the same on every rank."""

    def __init__(self, n_layers: int, kinds: list, dense: str = "bf16", hidden: int = 2048, experts: int = 512,
                 inter: int = 512, top_k: int = 10, shared_inter: int = 512, q_heads: int = 16, kv_heads: int = 2,
                 vocab: int = 32768, max_pos: int = 8192 + 64, device=None, group=None, mode: str = "replicated",
                 sigma: dict | None = None, seed: int = 0):
        from . import blocks as B
        from . import ep as EP
        from . import fused as F
        from .synthetic import blocks_cuda

        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device, self.hidden, self.vocab, self.n_layers, self.mode = device, hidden, vocab, n_layers, mode
        self.group = group
        world, rank = 1, 0
        if group is not None:
            import torch.distributed as dist

            world, rank = dist.get_world_size(group), dist.get_rank(group)
        sig = sigma or {"Q2_0": 0.025, "IQ3_S": 2.4e-4, "IQ3_XXS": 2.4e-4}
        e0, e1 = EP.expert_range(rank, world, experts)
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.embed = (torch.randn((vocab, hidden), generator=g, device=device)).to(torch.bfloat16)
        self.head = (torch.randn((vocab, hidden), generator=g, device=device) * 0.02).to(torch.bfloat16)
        self.head_f32 = self.head.float()  # logits in float32: bfloat16 logits of a large vocabulary tie too often
        self.final_norm = torch.ones(hidden, dtype=torch.bfloat16, device=device)
        self.layers = []
        self.expert_bytes = []
        for l in range(n_layers):
            kind = kinds[l % len(kinds)]
            s = sig.get(kind, 0.02)
            base_seed = seed * 1000 + 10 * l
            attn = Attention(hidden, q_heads, kv_heads, dense, g, device)
            lin = {}
            for name, shp, sd in (("gate", (experts, inter, hidden), 1), ("up", (experts, inter, hidden), 2),
                                  ("down", (experts, hidden, inter), 3)):
                full = blocks_cuda(kind, *shp, base_seed + sd, device, sigma=s)
                mine = EP.local_experts(full, experts, rank, world) if world > 1 else full
                lin[name] = B.BlockSwitchLinear(mine, kind, (e1 - e0,) + shp[1:])
                del full
            shared = tuple(B.BlockSwitchLinear(blocks_cuda(kind, 1, r, c, base_seed + sd, device, sigma=s), kind, (1, r, c))
                           for r, c, sd in ((shared_inter, hidden, 4), (shared_inter, hidden, 5), (hidden, shared_inter, 6)))
            gr = torch.Generator(device=device)
            gr.manual_seed(base_seed + 7)
            router = (torch.randn((experts, hidden), generator=gr, device=device) * 0.02).half()
            sgw = (torch.randn((hidden,), generator=gr, device=device) * 0.02).half()
            base = F.MoEDecodeLayer(router, lin["gate"], lin["up"], lin["down"], top_k, shared=shared, shared_gate=sgw)
            if world > 1 and mode == "replicated":
                base.layer.experts = experts  # the router's rows; the stacks hold this rank's share
                moe = ReplicatedEPMoE(base, e0, e1, group)
            elif world > 1:
                moe = EP.EPMoEDecodeLayer(router, lin["gate"], lin["up"], lin["down"], top_k, experts, shared=shared,
                                          shared_gate=sgw, group=group)
                base = moe.base
            else:
                moe = base
            self.layers.append({"attn": attn, "moe": moe, "base": base, "kind": kind,
                                "n1": torch.ones(hidden, dtype=torch.bfloat16, device=device),
                                "n2": torch.ones(hidden, dtype=torch.bfloat16, device=device)})
            rbh = B._row_bytes(kind, hidden)
            rbi = B._row_bytes(kind, inter)
            self.expert_bytes.append((2 * inter * rbh + hidden * rbi, 2 * shared_inter * rbh + hidden * B._row_bytes(kind, shared_inter)))
            torch.cuda.empty_cache()
        self.rope = Rope(max_pos, device)
        self.kv_heads, self.q_heads = kv_heads, q_heads
        self.dense_bytes = sum(l["attn"].nbytes for l in self.layers)
        self._ws = None

    def cache(self, max_tokens: int, seed: int = 0) -> PagedCache:
        return PagedCache(self.n_layers, self.kv_heads, max_tokens, self.device, seed)

    def workspace(self, cache: PagedCache) -> torch.Tensor:
        n = _lib.lib().sc_paged_attention_workspace(cache.max_tokens, self.kv_heads)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, tokens: torch.Tensor, cache: PagedCache, trace: list | None = None) -> torch.Tensor:
        """The window `tokens` (t,) int64 on the device at the cache's position: every layer (their keys and values
        written at positions pos .. pos + t - 1), then the output head. Returns logits (t, vocab) float32. Does not
        move the position (advance does), so that a verify pass can be replayed at the same place."""
        t = tokens.shape[0]
        ws = self.workspace(cache)
        ctx = cache.pos + t  # the window's keys are in the cache when attention reads it
        x = self.embed.index_select(0, tokens)  # the residual stream, added to in place
        h = torch.empty_like(x)
        delta = None
        for l, L in enumerate(self.layers):
            add_rmsnorm(x, delta, L["n1"], h)  # the previous layer's MoE output joins the stream here
            if trace is not None:
                trace.append(x.clone())  # each layer's input, for tests that check a layer at a time
            a = L["attn"](h, cache, l, self.rope, ws, ctx)
            add_rmsnorm(x, a, L["n2"], h)
            delta = L["moe"](h)
        add_rmsnorm(x, delta, self.final_norm, h)
        if trace is not None:
            trace.append(x.clone())
        return h.float() @ self.head_f32.T

    @staticmethod
    def advance(cache: PagedCache, t: int) -> None:
        cache.pos.add_(t)

    def check_errors(self) -> None:
        for L in self.layers:
            L["base"].check_errors()
        _lib.check_device_errors()


def _bf(a):
    from oracle import blocks_ref as R

    return R.round_to(np.asarray(a, dtype=np.float32), "bfloat16")


def _norm(a):
    a = np.asarray(a, dtype=np.float32)
    return _bf(a / np.sqrt((a * a).mean(-1, keepdims=True) + np.float32(1e-6)))


def oracle_layer(dec: SyntheticDecoder, l: int, x: np.ndarray, pos: int, cache_k: list, cache_v: list,
                 blocks: dict) -> tuple:
    """Layer l of the decoder in float32 numpy on the CPU with the GPU's bfloat16 rounding points, for the window x
    (t, hidden) (values of bfloat16) at positions pos .. pos + t - 1: dense products in float64 rounded to bfloat16,
    attention in float64 (the probabilities rounded to bfloat16 as the kernel rounds them), the MoE block by the
    oracle (oracle/blocks_ref.py moe_layer_blocks, on every expert of `blocks`, synthetic.layer_numpy's form). The
    layer's keys and values are appended to cache_k[l] / cache_v[l] ((positions, kv_heads, D) float32). Returns
    (output, the MoE block's parts). TEST INFRASTRUCTURE: used by tests only."""
    from oracle import blocks_ref as R

    t = x.shape[0]
    A = dec.layers[l]["attn"]
    cos, sin = dec.rope.cos.cpu().numpy(), dec.rope.sin.cpu().numpy()
    positions = np.arange(pos, pos + t)

    def rope(a):
        c, s = cos[positions][:, None, :], sin[positions][:, None, :]
        h1, h2 = a[..., : HEAD_DIM // 2], a[..., HEAD_DIM // 2 :]
        return _bf(np.concatenate([h1 * c - h2 * s, h2 * c + h1 * s], axis=-1))

    def mm(d, a):
        return _bf(a.astype(np.float64) @ d.floats().cpu().numpy().astype(np.float64).T)

    h = _norm(x)
    q = rope(mm(A.wq, h).reshape(t, A.hq, HEAD_DIM))
    k = rope(mm(A.wk, h).reshape(t, A.hkv, HEAD_DIM))
    v = mm(A.wv, h).reshape(t, A.hkv, HEAD_DIM)
    K = np.concatenate([cache_k[l], k], 0)
    V = np.concatenate([cache_v[l], v], 0)
    o = np.zeros((t, A.hq, HEAD_DIM), dtype=np.float32)
    for i in range(t):
        n = pos + i + 1
        for hh in range(A.hq):
            kv = hh // (A.hq // A.hkv)
            sc = (K[:n, kv].astype(np.float64) @ q[i, hh].astype(np.float64)) / math.sqrt(HEAD_DIM)
            p = np.exp(sc - sc.max())
            o[i, hh] = (_bf(p) @ V[:n, kv].astype(np.float64)) / p.sum()
    x = _bf(x + mm(A.wo, _bf(o).reshape(t, -1)))
    parts = R.moe_layer_blocks(_norm(x), blocks, dec.hidden, blocks["inter"], blocks["top_k"], "bfloat16",
                               shared_inter=blocks["shared_inter"])
    cache_k[l], cache_v[l] = K, V
    return _bf(x + parts["out"]), parts


def oracle_head(dec: SyntheticDecoder, x: np.ndarray) -> np.ndarray:
    """The output head on the last layer's output: float64 logits of the normed window. TEST INFRASTRUCTURE."""
    return _norm(x).astype(np.float64) @ dec.head.float().cpu().numpy().astype(np.float64).T
