"""The MoE block around the experts, on a B200: the call surface of strata_mlx/fused.py's router, top-k and
combine (fused.py:326-507) over torch CUDA tensors, plus the whole block in decode as one C call.

    WindowLinear   float16 router weights times a window of tokens, float32 logits (fused.py:357-390)
    top_k          the k largest logits, ties to the lower index (fused.py:393-436)
    moe_combine    sum_k y_k w_k in MLX's order + sigmoid(g) * shared (fused.py:439-481)
    RoutedMoE      the block: router, top_k, softmax, experts, shared expert, combine (fused.py:484-497)
    MoEDecodeLayer the block in decode through sc_moe_decode_layer, a chain of kernels with no host sync
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import DTYPES, KINDS, check, ptr, stream, require_cuda

ROUTER_TOPK = True  # fused.py:420
ROUTER_AS_IS = True  # fused.py:421
COMBINE_UPTO = 16  # fused.py:464: tokens the combine kernel takes; more go through torch's operations


def _device(device) -> torch.device:
    """A CUDA device with its index ("cuda" names the current one), so that workspaces are keyed alike."""
    d = torch.device(device)
    return torch.device(d.type, torch.cuda.current_device()) if d.type == "cuda" and d.index is None else d


class WindowLinear:
    """A float16 linear layer without bias whose products come back in float32; a window of up to `upto` tokens
    goes through the router kernel, which reads the weights once as they are (fused.py:357-390)."""

    upto, groups = 8, 16

    def __init__(self, linear):
        self.linear = linear  # an object with .weight (rows, cols), or a tensor
        w = self.weight
        self.rows, self.cols = w.shape

    @property
    def weight(self) -> torch.Tensor:
        return self.linear if isinstance(self.linear, torch.Tensor) else self.linear.weight

    def takes(self, x: torch.Tensor) -> bool:
        return x.numel() // self.cols <= self.upto and self.weight.dtype == torch.float16 and self.cols % 8 == 0

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        require_cuda(x)
        tokens = x.numel() // self.cols
        if not self.takes(x):
            w = self.weight
            if w.dtype == torch.float16 and self.cols % 8 == 0 and x.dtype in DTYPES:
                # a chunk of a prompt: the reference multiplies floats here (fused.py:386-388); sc_router's tiled
                # product takes the float16 weights as they are, float32 sums
                xs = x.reshape(tokens, self.cols)
                xs = xs if xs.is_contiguous() else xs.contiguous()
                w = w if w.is_contiguous() else w.contiguous()
                out = torch.empty((tokens, self.rows), dtype=torch.float32, device=x.device)
                check(_lib.lib().sc_router(ptr(w), self.rows, self.cols, ptr(xs), DTYPES[xs.dtype], tokens, ptr(out),
                                           stream()), "WindowLinear")
                return out.reshape(*x.shape[:-1], self.rows)
            if isinstance(self.linear, torch.Tensor):
                return x.float() @ self.linear.float().T
            return self.linear(x)
        xs = x.reshape(tokens, self.cols)
        xs = xs if xs.is_contiguous() else xs.contiguous()
        w = self.weight if self.weight.is_contiguous() else self.weight.contiguous()
        out = torch.empty((tokens, self.rows), dtype=torch.float32, device=x.device)
        check(_lib.lib().sc_router(ptr(w), self.rows, self.cols, ptr(xs), DTYPES[xs.dtype], tokens, ptr(out), stream()),
              "WindowLinear")
        return out.reshape(*x.shape[:-1], self.rows)


def top_k(logits: torch.Tensor, k: int) -> torch.Tensor:
    """The indices of the k largest logits (..., N) float32, largest first, ties to the lower index
    (fused.py:424-436); uint32 like the reference's kernel."""
    require_cuda(logits)
    n = logits.shape[-1]
    if not ROUTER_TOPK or n > 2048 or logits.dtype != torch.float32 or k > 16:
        order = torch.sort(-logits.float(), dim=-1, stable=True).indices[..., :k]
        return order.to(torch.int32).view(torch.uint32)
    rows = logits.numel() // n
    lg = logits.reshape(rows, n)
    lg = lg if lg.is_contiguous() else lg.contiguous()
    idx = torch.empty((rows, k), dtype=torch.uint32, device=logits.device)
    check(_lib.lib().sc_top_k(ptr(lg), rows, n, k, ptr(idx), stream()), "top_k")
    return idx.reshape(*logits.shape[:-1], k)


def top_k_softmax(logits: torch.Tensor, k: int) -> tuple:
    """top_k and the softmax over the chosen logits (fused.py:490-491) in one kernel."""
    require_cuda(logits)
    n = logits.shape[-1]
    rows = logits.numel() // n
    lg = logits.reshape(rows, n).contiguous()
    idx = torch.empty((rows, k), dtype=torch.uint32, device=logits.device)
    w = torch.empty((rows, k), dtype=torch.float32, device=logits.device)
    check(_lib.lib().sc_top_k_softmax(ptr(lg), rows, n, k, ptr(idx), ptr(w), stream()), "top_k_softmax")
    return idx.reshape(*logits.shape[:-1], k), w.reshape(*logits.shape[:-1], k)


def moe_combine(y: torch.Tensor, w: torch.Tensor, g: torch.Tensor, s: torch.Tensor) -> torch.Tensor | None:
    """y (..., K, D), w (..., K) float32, g (..., 1), s (..., D) -> (..., D) (fused.py:467-481); None where not
    taken (more than COMBINE_UPTO tokens, or activations other than float16/bfloat16)."""
    require_cuda(y, w, g, s)
    *lead, k, d = y.shape
    rows = y.numel() // (k * d)
    if rows > COMBINE_UPTO or y.dtype not in (torch.float16, torch.bfloat16) or w.dtype != torch.float32 or k > 16:
        return None
    out = torch.empty((rows, d), dtype=y.dtype, device=y.device)
    yy, ww = y.reshape(rows, k, d).contiguous(), w.reshape(rows, k).contiguous()
    gg, ss = g.reshape(rows).to(y.dtype).contiguous(), s.reshape(rows, d).to(y.dtype).contiguous()
    check(_lib.lib().sc_moe_combine(ptr(yy), ptr(ww), ptr(gg), ptr(ss), rows, k, d, DTYPES[y.dtype], ptr(out), stream()),
          "moe_combine")
    return out.reshape(*lead, d)


def _combine_rows(y: torch.Tensor, w: torch.Tensor, g: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """sc_moe_combine over any number of rows (the combine of a prompt chunk's tokens), MLX's add order of
    fused.py:448-462 kept for every row."""
    *lead, k, d = y.shape
    rows = y.numel() // (k * d)
    out = torch.empty((rows, d), dtype=y.dtype, device=y.device)
    yy, ww = y.reshape(rows, k, d).contiguous(), w.reshape(rows, k).float().contiguous()
    gg, ss = g.reshape(rows).to(y.dtype).contiguous(), s.reshape(rows, d).to(y.dtype).contiguous()
    check(_lib.lib().sc_moe_combine(ptr(yy), ptr(ww), ptr(gg), ptr(ss), rows, k, d, DTYPES[y.dtype], ptr(out), stream()),
          "moe_combine")
    return out.reshape(*lead, d)


class SharedExpert:
    """The block's shared expert, an MLP on block weights (mlx-lm's MLP with gate_proj, up_proj, down_proj): each
    projection is a BlockSwitchLinear of one expert."""

    def __init__(self, gate_proj, up_proj, down_proj):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        from .blocks import BlockSwitchLinear, TILES_FROM, switch_glu, tileable, window_matvec

        lead = x.shape[:-1]
        xs = x.reshape(-1, x.shape[-1])
        lins = (self.gate_proj, self.up_proj, self.down_proj)
        if (xs.shape[0] >= TILES_FROM and all(isinstance(l, BlockSwitchLinear) for l in lins)
                and all(tileable(l.kind, l.output_dims, l.input_dims) for l in lins)):
            # a chunk of a prompt: the expert as a stack of one through the tile products (the tcgen05 kernel)
            idx = torch.zeros((xs.shape[0], 1), dtype=torch.int32, device=x.device)
            out = switch_glu(xs, idx, self.up_proj, self.gate_proj, self.down_proj)
            return out.reshape(*lead, -1)
        g = window_matvec(self.gate_proj.blocks, self.gate_proj.kind, self.gate_proj.output_dims, self.gate_proj.input_dims, xs)
        u = window_matvec(self.up_proj.blocks, self.up_proj.kind, self.up_proj.output_dims, self.up_proj.input_dims, xs)
        from .blocks import swiglu

        h = swiglu(g, u)
        out = window_matvec(self.down_proj.blocks, self.down_proj.kind, self.down_proj.output_dims,
                            self.down_proj.input_dims, h)
        return out.reshape(*lead, -1)


class RoutedMoE:
    """The model's MoE block with the router's choice made by `top_k` and its end by `moe_combine`
    (fused.py:484-497): router logits in float32, top_k, softmax over the chosen logits, the routed experts
    (`switch_mlp`, a BlockSwitchGLU), the shared expert and its gate, and the combine."""

    def __init__(self, gate, switch_mlp, shared_expert=None, shared_expert_gate=None, top_k: int = 10):
        self.gate = gate if isinstance(gate, WindowLinear) else WindowLinear(gate)
        self.switch_mlp, self.shared_expert = switch_mlp, shared_expert
        self.shared_expert_gate = shared_expert_gate  # (H,) float16 weights of a product with x
        self.top_k = top_k

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        gate = self.gate
        logits = gate(x if ROUTER_AS_IS and gate.takes(x) else x.float())
        if ROUTER_TOPK and logits.shape[-1] <= 2048 and self.top_k <= 16:
            idx, w = top_k_softmax(logits, self.top_k)  # the softmax over the chosen logits in the same kernel
        else:
            idx = top_k(logits, self.top_k)
            w = torch.softmax(torch.gather(logits.float(), -1, idx.to(torch.int64)), dim=-1)
        y = self.switch_mlp(x, idx)
        if self.shared_expert is not None:
            g = WindowLinear(self.shared_expert_gate.reshape(1, -1))(x).to(x.dtype)
            s = self.shared_expert(x)
        else:
            g = torch.full((*x.shape[:-1], 1), float("-inf"), dtype=x.dtype, device=x.device)
            s = torch.zeros_like(x)
        out = moe_combine(y, w, g, s) if COMBINE_UPTO else None
        if out is None and COMBINE_UPTO and y.dtype in (torch.float16, torch.bfloat16) and y.shape[-2] <= 16:
            out = _combine_rows(y, w, g, s)  # a chunk of a prompt: the same kernel and add order for every row
        if out is None:
            out = (y.float() * w[..., None]).sum(dim=-2).to(x.dtype) + torch.sigmoid(g) * s
        return out


class MoEDecodeLayer:
    """One MoE block in decode (1..8 tokens) through the single C call sc_moe_decode_layer: the same answer as
    RoutedMoE, with the routing, experts, shared expert and combine enqueued by the library on the current stream
    and no host synchronization. Holds its workspace (sc_moe_decode_workspace bytes) per token count."""

    def __init__(self, router: torch.Tensor, gate, up, down, top_k: int, shared=None, shared_gate=None,
                 dtype: torch.dtype = torch.bfloat16):
        require_cuda(router)
        self._keep = [router, gate.blocks, up.blocks, down.blocks]
        L = _lib.SCLayer()
        L.hidden, L.inter, L.experts, L.top_k = gate.input_dims, gate.output_dims, gate.num_experts, top_k
        L.kind_gate, L.kind_up, L.kind_down = KINDS[gate.kind], KINDS[up.kind], KINDS[down.kind]
        L.gate, L.up, L.down, L.router = gate.blocks.data_ptr(), up.blocks.data_ptr(), down.blocks.data_ptr(), router.data_ptr()
        if shared is not None:
            sg, su, sd = shared
            self._keep += [sg.blocks, su.blocks, sd.blocks, shared_gate]
            L.shared_inter = sg.output_dims
            L.kind_sgate, L.kind_sup, L.kind_sdown = KINDS[sg.kind], KINDS[su.kind], KINDS[sd.kind]
            L.sgate, L.sup, L.sdown = sg.blocks.data_ptr(), su.blocks.data_ptr(), sd.blocks.data_ptr()
            L.shared_gate = shared_gate.data_ptr()
        L.dtype = DTYPES[dtype]
        self.layer, self.dtype, self.hidden, self.top_k = L, dtype, gate.input_dims, top_k
        self._ws: dict = {}

    def workspace(self, tokens: int, device) -> torch.Tensor:
        device = _device(device)
        ws = self._ws.get((tokens, device))
        if ws is None:
            n = _lib.lib().sc_moe_decode_workspace(self.layer_ref(), tokens)
            if n == 0:
                raise ValueError(f"sc_moe_decode_layer does not take {tokens} tokens for this layer")
            ws = torch.zeros(n, dtype=torch.uint8, device=device)
            self._ws[(tokens, device)] = ws
        return ws

    def layer_ref(self) -> int:
        import ctypes

        return ctypes.addressof(self.layer)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        require_cuda(x)
        xs = x.reshape(-1, self.hidden)
        if xs.dtype != self.dtype:
            raise ValueError(f"activations of {xs.dtype}; the layer was built for {self.dtype}")
        xs = xs if xs.is_contiguous() else xs.contiguous()
        tokens = xs.shape[0]
        ws = self.workspace(tokens, x.device)
        if out is None:
            out = torch.empty_like(xs)
        check(_lib.lib().sc_moe_decode_layer(self.layer_ref(), ptr(xs), tokens, ptr(out), ptr(ws), ws.numel(), stream()),
              "sc_moe_decode_layer")
        return out.reshape(x.shape)

    def stage(self, x: torch.Tensor, out: torch.Tensor, stage: int) -> None:
        """One of the fused path's three kernels (0 route, 1 gate/up, 2 down + combine) on the workspace a
        previous call with this token count filled: for timing and profiling the kernels one at a time."""
        xs = x.reshape(-1, self.hidden)
        tokens = xs.shape[0]
        ws = self.workspace(tokens, x.device)
        check(_lib.lib().sc_moe_decode_stage(self.layer_ref(), ptr(xs), tokens, ptr(out), ptr(ws), ws.numel(), stage,
                                             stream()), "sc_moe_decode_stage")

    def check_errors(self) -> None:
        """Reads (synchronizing) and clears the error words of this layer's workspaces; raises when a kernel
        recorded one (a bad expert id, or a bounded wait that gave up)."""
        for ws in self._ws.values():
            v = int(ws[:4].view(torch.int32).item())
            if v:
                ws[:4].zero_()
                raise _lib.StrataError(f"a kernel recorded {_lib.ERRORS.get(v, v)}: "
                                       f"{_lib.lib().sc_error_string(v).decode()}")

    def routes(self, tokens: int, device) -> tuple:
        """(idx (tokens, K) uint32, weights (tokens, K) float32) of the last call with `tokens` tokens."""
        import ctypes

        io, wo = ctypes.c_size_t(), ctypes.c_size_t()
        check(_lib.lib().sc_moe_decode_routes(self.layer_ref(), tokens, ctypes.byref(io), ctypes.byref(wo)), "routes")
        ws = self.workspace(tokens, device)
        k = self.top_k
        idx = ws[io.value : io.value + tokens * k * 4].view(torch.int32).view(torch.uint32).reshape(tokens, k)
        w = ws[wo.value : wo.value + tokens * k * 4].view(torch.float32).reshape(tokens, k)
        return idx, w


class DecodeChain:
    """A stack of decode layers (MoEDecodeLayer, one shape) run by one launch of sc_moe_decode_chain: the persistent
    kernel routes and multiplies every layer in turn, grid-wide barriers between its phases, so that no launch
    separates the layers. __call__(x) applies the layers to the window x (tokens, hidden) -- each layer taking the
    previous one's output, or x again every `refeed` layers -- and returns the last layer's output. The same bits as
    calling the layers one by one."""

    def __init__(self, layers: list, refeed: int = 0):
        import ctypes

        if not layers:
            raise ValueError("a chain needs a layer")
        self.layers, self.refeed = layers, refeed
        self.hidden, self.dtype, self.top_k = layers[0].hidden, layers[0].dtype, layers[0].top_k
        self._structs = (_lib.SCLayer * len(layers))(*[l.layer for l in layers])
        self._ws: dict = {}
        self._out: dict = {}

    def _ref(self) -> int:
        import ctypes

        return ctypes.addressof(self._structs)

    def workspace(self, tokens: int, device) -> torch.Tensor:
        device = _device(device)
        ws = self._ws.get((tokens, device))
        if ws is None:
            n = _lib.lib().sc_moe_decode_chain_workspace(self._ref(), len(self.layers), tokens)
            if n == 0:
                raise ValueError(f"sc_moe_decode_chain does not take these layers at {tokens} tokens")
            ws = torch.zeros(n, dtype=torch.uint8, device=device)  # zeroed once: the kernel's barrier count
            self._ws[(tokens, device)] = ws
        return ws

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        require_cuda(x)
        xs = x.reshape(-1, self.hidden)
        if xs.dtype != self.dtype:
            raise ValueError(f"activations of {xs.dtype}; the chain was built for {self.dtype}")
        xs = xs if xs.is_contiguous() else xs.contiguous()
        tokens = xs.shape[0]
        ws = self.workspace(tokens, x.device)
        if out is None:
            out = torch.empty_like(xs)
        check(_lib.lib().sc_moe_decode_chain(self._ref(), len(self.layers), ptr(xs), tokens, self.refeed, ptr(out),
                                             ptr(ws), ws.numel(), stream()), "sc_moe_decode_chain")
        return out.reshape(x.shape)

    def routes(self, tokens: int, device) -> tuple:
        """(idx (layers, tokens, K) uint32, weights (layers, tokens, K) float32) of the last call."""
        import ctypes

        io, wo = ctypes.c_size_t(), ctypes.c_size_t()
        check(_lib.lib().sc_moe_decode_chain_routes(self._ref(), len(self.layers), tokens, ctypes.byref(io),
                                                    ctypes.byref(wo)), "routes")
        ws = self.workspace(tokens, device)
        n, k = len(self.layers), self.top_k
        idx = ws[io.value : io.value + n * tokens * k * 4].view(torch.int32).view(torch.uint32).reshape(n, tokens, k)
        w = ws[wo.value : wo.value + n * tokens * k * 4].view(torch.float32).reshape(n, tokens, k)
        return idx, w

    def check_errors(self) -> None:
        """Reads (synchronizing) the error words of the chain's workspaces; on an error zeroes the workspace (its
        barrier count may be left mid-way) and raises."""
        for ws in self._ws.values():
            v = int(ws[:4].view(torch.int32).item())
            if v:
                ws.zero_()
                raise _lib.StrataError(f"a kernel recorded {_lib.ERRORS.get(v, v)}: "
                                       f"{_lib.lib().sc_error_string(v).decode()}")


class DecodeGraph:
    """A stack of decode layers (MoEDecodeLayer) replayed as one CUDA graph: the call a serving loop makes per
    decoded window. __call__ takes the window's activations on the host (pinned, or any CPU tensor), copies them
    in, runs every layer, and returns the last layer's output on the host. `layers` each take the window itself
    when `chain` is False, or the previous layer's output when True; with `refeed` = n > 0 (and `chain`), every
    n-th layer takes the window again -- for a synthetic chain, which has none of the norms a model puts between
    its MoE blocks and would otherwise grow without bound."""

    def __init__(self, layers: list, tokens: int, device=None, chain: bool = False, capture: bool = True,
                 refeed: int = 0, persistent: bool = False):
        self.layers, self.tokens, self.chain, self.capture, self.refeed = layers, tokens, chain, capture, refeed
        # persistent: every layer in one launch of the chain kernel (DecodeChain); only the last output is kept
        self.persistent = DecodeChain(layers, refeed if chain else 1) if persistent else None
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        H, dt = layers[0].hidden, layers[0].dtype
        self.x = torch.zeros((tokens, H), dtype=dt, device=dev)
        self.outs = [torch.zeros((tokens, H), dtype=dt, device=dev) for _ in layers]
        self.host_in = torch.zeros((tokens, H), dtype=dt).pin_memory()
        self.host_out = torch.zeros((tokens, H), dtype=dt).pin_memory()
        for l in layers:
            l.workspace(tokens, dev)
        if self.persistent is not None:
            self.persistent.workspace(tokens, dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = torch.cuda.CUDAGraph() if capture else None
        with torch.cuda.stream(self.stream):
            self.run_layers()  # warm: kernel attributes are set outside the capture
        self.stream.synchronize()
        if capture:
            with torch.cuda.graph(self.graph, stream=self.stream):
                self.run_layers()

    def run_layers(self) -> None:
        if self.persistent is not None:
            self.persistent(self.x, out=self.outs[-1])
            return
        x = self.x
        for i, (l, o) in enumerate(zip(self.layers, self.outs)):
            if self.refeed and i % self.refeed == 0:
                x = self.x
            l(x, out=o)
            if self.chain:
                x = o

    def replay(self) -> torch.Tensor:
        """Runs the graph on the activations already in self.x (device-resident); returns the last output. Without
        capture (for profilers that cannot follow a stream capture) the layers are launched one by one."""
        if self.graph is None:
            self.run_layers()
        else:
            self.graph.replay()
        return self.outs[-1]

    def __call__(self, x_host: torch.Tensor) -> torch.Tensor:
        s = torch.cuda.current_stream()
        self.host_in.copy_(x_host.reshape(self.host_in.shape))
        self.x.copy_(self.host_in, non_blocking=True)
        self.replay()
        self.host_out.copy_(self.outs[-1], non_blocking=True)
        s.synchronize()
        return self.host_out
