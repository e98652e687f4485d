"""Expert parallelism for the decode MoE block: one process per GPU (torch.distributed over NCCL), rank r of G holding
experts [r E / G, (r + 1) E / G) of every layer; the router, the shared expert and its gate are replicated. The
reference (strata_mlx/fused.py:487-497, _Routed.__call__) runs every expert on one device; this is the same block
over G devices.

A layer runs over the window of every rank's tokens:
  1. all-gather: each rank's t tokens into the window X (G t tokens, rank r's at rows r t .. r t + t - 1);
  2. sc_moe_decode_layer_ep: route the whole window (the replicated router gives every rank the same routes), run
     this rank's experts on the pairs that chose them, and the shared expert on every token; y_pairs (G t, K, H)
     holds each pair's output on the rank that owns the pair's expert and zero on the others;
  3. all-reduce (sum) of y_pairs: each pair's output is non-zero on exactly one rank, so the sum is that output
     exactly;
  4. sc_moe_decode_combine: every token's combine, in the fixed order of moe_combine (fused.py:448-462).
Each token's result has the bits the single-device layer gives it. Per layer the exchange carries t H values per
rank in (all-gather) and G t K H values across ranks (all-reduce).

EPDecodeChain runs a chain of such layers with the exchange done by the kernels themselves over peer memory (NVLink):
each rank maps the others' exchange buffers (CUDA IPC, PeerExchange); a combine writes its tokens' outputs straight
into every rank's next window, the down kernel writes each pair's output straight to the rank of the pair's token,
and release / acquire counts mark the parts complete (layout in csrc/ep.cuh). No collective runs on the data path."""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, ptr, stream


def expert_range(rank: int, world: int, experts: int) -> tuple:
    """The experts [begin, end) that rank `rank` of `world` holds: equal contiguous shares."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return rank * per, (rank + 1) * per


def local_experts(blocks: torch.Tensor, experts: int, rank: int, world: int) -> torch.Tensor:
    """This rank's share of a stack of `experts` experts' blocks (expert-major bytes): a copy of its slice."""
    e0, e1 = expert_range(rank, world, experts)
    per = blocks.numel() // experts
    if per * experts != blocks.numel():
        raise ValueError("the blocks do not split into experts")
    return blocks.reshape(-1)[e0 * per : e1 * per].clone()


class EPMoEDecodeLayer:
    """One MoE block in decode, expert parallel over the ranks of `group`. gate, up and down are BlockSwitchLinear
    stacks of this rank's experts only (expert_range(rank, world, experts)); router is the full (experts, hidden)
    float16 router; shared / shared_gate as MoEDecodeLayer takes them. Calling it with this rank's tokens
    (t, hidden) returns their outputs; every rank of the group must call it with the same t."""

    def __init__(self, router: torch.Tensor, gate, up, down, top_k: int, experts: int, shared=None,
                 shared_gate=None, dtype: torch.dtype = torch.bfloat16, group=None):
        from .fused import MoEDecodeLayer

        self._setup(experts, top_k, gate.input_dims, dtype, group)
        if gate.num_experts != self.e1 - self.e0:
            raise ValueError(f"rank {self.rank} holds experts [{self.e0}, {self.e1}); the stacks hold {gate.num_experts}")
        self.base = MoEDecodeLayer(router, gate, up, down, top_k, shared=shared, shared_gate=shared_gate, dtype=dtype)
        self.base.layer.experts = experts  # the router's rows; the blocks hold this rank's share
        self._bufs: dict = {}

    def _setup(self, experts: int, top_k: int, hidden: int, dtype: torch.dtype, group) -> None:
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.experts, self.top_k, self.hidden, self.dtype = experts, top_k, hidden, dtype
        self.e0, self.e1 = expert_range(self.rank, self.world, experts)

    # ---- the four steps; the device ones are overridden by the CPU tests of the exchange

    def _gather(self, xs: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        t = xs.shape[0]
        X = self._buf("X", (self.world * t, self.hidden), xs)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(X, xs, group=self.group)
        else:
            dist.all_gather(list(X.split(t)), xs, group=self.group)
        return X

    def _local(self, X: torch.Tensor):
        T = X.shape[0]
        ws = self.base.workspace(T, X.device)
        Y = self._buf("Y", (T, self.top_k, self.hidden), X)
        check(_lib.lib().sc_moe_decode_layer_ep(self.base.layer_ref(), ptr(X), T, self.e0, self.e1, ptr(Y), ptr(ws),
                                                ws.numel(), stream()), "sc_moe_decode_layer_ep")
        return Y, ws

    def _sum(self, Y: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_reduce(Y, group=self.group)

    def _combine(self, Y: torch.Tensor, state) -> torch.Tensor:
        T = Y.shape[0]
        out = self._buf("out", (T, self.hidden), Y)
        check(_lib.lib().sc_moe_decode_combine(self.base.layer_ref(), ptr(Y), T, ptr(out), ptr(state), state.numel(),
                                               stream()), "sc_moe_decode_combine")
        return out

    def _buf(self, name: str, shape: tuple, like: torch.Tensor) -> torch.Tensor:
        b = self._bufs.get((name, shape))
        if b is None:
            b = torch.empty(shape, dtype=self.dtype, device=like.device)
            self._bufs[(name, shape)] = b
        return b

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        xs = x.reshape(-1, self.hidden)
        if xs.dtype != self.dtype:
            raise ValueError(f"activations of {xs.dtype}; the layer was built for {self.dtype}")
        xs = xs if xs.is_contiguous() else xs.contiguous()
        t = xs.shape[0]
        X = self._gather(xs)
        Y, state = self._local(X)
        self._sum(Y)
        out = self._combine(Y, state)
        return out[self.rank * t : (self.rank + 1) * t].reshape(x.shape)


class PeerExchange:
    """Every rank's exchange buffer (sc_ep_exchange_bytes for the layer's shape, zeroed) mapped into every other rank
    by CUDA IPC; `desc` is the sc_ep_exchange the kernels take. close() unmaps the peers' buffers."""

    def __init__(self, layer_struct, tokens_per_rank: int, device, group=None):
        import torch.distributed as dist

        lib = _lib.lib()
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        n = lib.sc_ep_exchange_bytes(ctypes.addressof(layer_struct), self.world, tokens_per_rank)
        if n == 0:
            raise ValueError("no exchange for this layer")
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)
        handle, off = ctypes.create_string_buffer(64), ctypes.c_size_t()
        check(lib.sc_ipc_handle(ptr(self.buf), handle, ctypes.byref(off)), "sc_ipc_handle")
        every = [None] * self.world
        dist.all_gather_object(every, (bytes(handle.raw), off.value), group=group)
        self._opened, bases = [], []
        for r, (h, o) in enumerate(every):
            if r == self.rank:
                bases.append(self.buf.data_ptr())
                continue
            base = ctypes.c_void_p()
            check(lib.sc_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(base)), "sc_ipc_open")
            self._opened.append(base.value)
            bases.append(base.value + o)
        self.peers = torch.tensor([b if b < 2 ** 63 else b - 2 ** 64 for b in bases], dtype=torch.int64, device=device)
        self.desc = _lib.SCExchange(self.peers.data_ptr(), self.buf.data_ptr(), self.world, self.rank, tokens_per_rank)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def close(self) -> None:
        for base in self._opened:
            _lib.lib().sc_ipc_close(ctypes.c_void_p(base))
        self._opened = []


class EPDecodeChain:
    """A chain of EPMoEDecodeLayer (an even number: the layers alternate the exchange's halves) run with the exchange
    in the kernels over peer memory. Calling it with this rank's tokens (t, hidden) runs every layer and returns the
    last layer's outputs for them; every rank of the group must call it with the same t. Bit-identical to the
    single-device chain."""

    def __init__(self, layers: list, tokens_per_rank: int, device, group=None):
        if not layers or len(layers) % 2:
            raise ValueError("the chain needs an even number of layers")
        self.layers, self.t, self.device = layers, tokens_per_rank, device
        first = layers[0]
        self.hidden, self.dtype = first.hidden, first.dtype
        self.ex = PeerExchange(first.base.layer, tokens_per_rank, device, group)
        self.T = self.ex.world * tokens_per_rank
        self.out = torch.empty((tokens_per_rank, self.hidden), dtype=self.dtype, device=device)
        for l in layers:
            l.base.workspace(self.T, device)

    def __call__(self, x: torch.Tensor, refeed: int = 0) -> torch.Tensor:
        """refeed: every `refeed` layers (an even number dividing the chain) the layer takes this rank's tokens x
        again, not the previous layer's outputs -- for a synthetic chain, which has none of the norms a model puts
        between its MoE blocks and would otherwise grow without bound."""
        lib = _lib.lib()
        xs = x.reshape(self.t, self.hidden)
        if xs.dtype != self.dtype:
            raise ValueError(f"activations of {xs.dtype}; the chain was built for {self.dtype}")
        xs = xs if xs.is_contiguous() else xs.contiguous()
        seg = refeed or len(self.layers)
        if seg % 2 or len(self.layers) % seg:
            raise ValueError(f"refeed {refeed}: an even number that divides the {len(self.layers)} layers")
        d = ctypes.byref(self.ex.desc)
        for s0 in range(0, len(self.layers), seg):
            # the segment's first window: this rank's tokens into every rank's window 0 (as a new call would)
            check(lib.sc_ep_feed(self.layers[s0].base.layer_ref(), d, ptr(xs), stream()), "sc_ep_feed")
            for i in range(s0, s0 + seg):
                l = self.layers[i]
                ws = l.base.workspace(self.T, self.device)
                ref = l.base.layer_ref()
                check(lib.sc_moe_decode_layer_ep_p2p(ref, d, l.e0, l.e1, i % 2, ptr(ws), ws.numel(), stream()),
                      "sc_moe_decode_layer_ep_p2p")
                last = int(i == s0 + seg - 1)
                check(lib.sc_ep_combine(ref, d, i % 2, last, ptr(self.out), ptr(ws), ws.numel(), stream()),
                      "sc_ep_combine")
        return self.out.reshape(x.shape)

    def check_errors(self) -> None:
        for l in self.layers:
            l.base.check_errors()

    def close(self) -> None:
        self.ex.close()
