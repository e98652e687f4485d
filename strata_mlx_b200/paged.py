"""Experts held within a budget of device memory and read from the model's files as routes ask for them: the paged
expert store of strata_mlx/paged.py:105-441 (ExpertStore, PagedSwitchGLU, load_profile, save_profile) on CUDA.

The decode path of this library keeps every expert resident, since a B200 (180 GB a GPU) holds these models whole.
The store serves the hosts where that does not hold: a smaller GPU, several models sharing one, or a budget the
caller chooses. Its rules are the reference's, and so are its thresholds:

  * a resident expert is its three tensors (up, gate, down) exactly as the file holds them, device uint8 tensors
    of their own; all layers share one store, and past the budget the least recently used experts leave first;
  * a layer waits on the host for its routes and reads the experts it lacks. Consecutive experts go to the file as
    one run, and a thread pool reads the runs into pinned host memory; each expert is then copied to the device on
    the current stream;
  * up to SEPARATE_UPTO (token, expert) pairs, each pair's expert goes to the kernel where it lies (the kernel takes
    a device array of expert pointers: `blocks.matvec_separate`); a larger window runs `blocks.switch_glu` over a
    stack of the experts it uses, and only an answer's window (up to KEEP_UPTO pairs) keeps what it read; a prompt
    that uses WHOLE_FROM or more of a layer's experts takes the layer's tensors whole (resident experts copied on
    the device, the gaps read) and keeps none of it;
  * `hold` / `ahead` / `release` let a prompt's chunks read a layer once, the next layer read ahead on a thread;
  * `preload` fills the free budget with the most used experts of a count table, `profile` returns this run's
    counts plus half of earlier ones, and `load_profile` / `save_profile` keep them between runs.

Bookkeeping: every resident expert has a record (its tensors, its bytes, the tick of its last use). Each use takes
the next tick of a counter; eviction drops the smallest ticks first, never an expert of the call in progress.
`lru` iterates the residents least recently used first.

Memory is the device's: `fit` sets the budget from what the device has free now. All device work goes on the current
CUDA stream. A dropped expert's memory returns to torch's caching allocator, which hands it out again only in that
stream's order, after the kernels that read it.
"""

from __future__ import annotations

import contextlib
import os
import tempfile
import threading
import time
from collections.abc import Mapping
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np
import torch

from .blocks import BLOCK, BlockSwitchLinear, matvec_separate, swiglu, switch_glu

WHOLE_FROM = 384  # strata_mlx/paged.py:36: a layer's experts used by one call from which its tensors are taken whole
KEEP_UPTO = 640  # :37: pairs in one call up to which what was read stays in the store (an answer, not a prompt)
SEPARATE_UPTO = 80  # :39: pairs up to which each pair's expert goes to the kernel where it lies
LEAST = int(0.5e9)  # :62: the smallest budget `fit` sets
WORKING = int(2e9)  # device bytes `fit` leaves for everything but the experts: activations, workspaces, graphs


class _Residents(Mapping):
    """(layer, expert) -> (its (up, gate, down) device tensors, bytes), iterated least recently used first."""

    def __init__(self):
        self._rec = {}  # key -> [tick of the last use, tensors, bytes]

    def __getitem__(self, key):
        _, tensors, nbytes = self._rec[key]
        return tensors, nbytes

    def __iter__(self):
        return iter(sorted(self._rec, key=lambda k: self._rec[k][0]))

    def __len__(self):
        return len(self._rec)

    def __contains__(self, key):
        return key in self._rec

    def put(self, key, tensors: tuple, nbytes: int, tick: int):
        self._rec[key] = [tick, tensors, nbytes]

    def stamp(self, key, tick: int):
        self._rec[key][0] = tick

    def drop(self, key) -> int:
        """Forgets `key`; returns the bytes it held."""
        return self._rec.pop(key)[2]

    def clear(self):
        self._rec.clear()


@dataclass
class _Held:
    """A layer that a prompt's chunks go through: its tensors whole (when read so), or the experts read so far."""

    layer: int
    stacks: list | None = None
    loose: dict = field(default_factory=dict)


def _runs(mask: np.ndarray) -> list:
    """Maximal runs of equal values of a boolean mask, as (first, count, value)."""
    if mask.size == 0:
        return []
    edges = np.flatnonzero(mask[1:] != mask[:-1]) + 1
    starts = np.concatenate(([0], edges))
    ends = np.concatenate((edges, [mask.size]))
    return [(int(a), int(b - a), bool(mask[a])) for a, b in zip(starts, ends)]


def _stacked(parts: list) -> torch.Tensor:
    return parts[0] if len(parts) == 1 else torch.cat(parts)


class ExpertStore:
    """Experts in device memory within `budget` bytes (strata_mlx/paged.py:105-370). `threads`: parallel file reads."""

    def __init__(self, budget: int, threads: int = 8, device=None):
        self.budget, self.held = int(budget), 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.lru = _Residents()
        self.layers = {}  # layer -> its (up, gate, down) gguf.Tensor, registered by PagedSwitchGLU
        self.use = {}  # layer -> an answer's uses of each expert (np.ndarray)
        self.kept = None  # the _Held layer between `hold` and `release`
        self.coming = None  # a read ahead: (layer, its runs, the future of its host buffers)
        self._clock = 0
        self._files = {}
        self._readers = ThreadPoolExecutor(threads)
        self._ahead = ThreadPoolExecutor(1)
        self._stats = threading.Lock()
        self.reset_stats()

    # ---- budget and statistics

    def fit(self, reserve: int = WORKING) -> int:
        """Sets the budget to the device memory free now, plus what the store holds, less `reserve`; at least LEAST."""
        free, _ = torch.cuda.mem_get_info(self.device)
        self.budget = max(LEAST, int(free) + self.held - int(reserve))
        return self.budget

    def reset_stats(self):
        self.hits = self.misses = self.bytes_read = 0
        self.read_s = 0.0  # seconds spent reading files
        self.waited_s = 0.0  # of the reads ahead, what a prompt still waited for

    def _tick(self) -> int:
        self._clock += 1
        return self._clock

    @staticmethod
    def _per_expert(t) -> int:
        return t.data.nbytes // t.shape[0]

    # ---- the files

    def _descriptor(self, path: str) -> int:
        fd = self._files.get(path)
        if fd is None:
            fd = self._files[path] = os.open(path, os.O_RDONLY)
        return fd

    def _pread(self, t, first: int, count: int) -> torch.Tensor:
        """Experts [first, first + count) of tensor t as the file holds them, in (pinned, for a GPU) host memory."""
        one = self._per_expert(t)
        buf = torch.empty(count * one, dtype=torch.uint8, pin_memory=self.device.type == "cuda")
        n = os.preadv(self._descriptor(t.path), [memoryview(buf.numpy())], t.offset + first * one)
        if n != buf.numel():
            raise OSError(f"{t.name}: short read ({n} of {buf.numel()} bytes)")
        return buf

    def _read_all(self, jobs: list) -> list:
        """(tensor, first, count) jobs read on the pool, in order (files only: safe on any thread)."""
        t0 = time.perf_counter()
        host = list(self._readers.map(lambda job: self._pread(*job), jobs))
        with self._stats:
            self.read_s += time.perf_counter() - t0
            self.bytes_read += sum(h.numel() for h in host)
        return host

    def _read_experts(self, tensors: tuple, experts: list) -> dict:
        """expert -> its (up, gate, down) on the device, consecutive experts read from the files as one run."""
        if not experts:
            return {}
        order = np.unique(np.asarray(experts, dtype=np.int64))
        cuts = np.flatnonzero(np.diff(order) != 1) + 1
        spans = [(int(s[0]), int(s.size)) for s in np.split(order, cuts)]
        host = self._read_all([(t, first, count) for t in tensors for first, count in spans])
        out = {int(e): [] for e in order}
        for j, t in enumerate(tensors):
            one = self._per_expert(t)
            for (first, count), buf in zip(spans, host[j * len(spans) : (j + 1) * len(spans)]):
                for i in range(count):
                    out[first + i].append(buf[i * one : (i + 1) * one].to(self.device, non_blocking=True))
        return {e: tuple(v) for e, v in out.items()}

    # ---- experts one by one

    def get(self, layer: int, tensors: tuple, experts: list, keep: bool = True) -> list:
        """The (up, gate, down) device tensors of each of `experts`, read where the store lacks them
        (strata_mlx/paged.py:330-370). `keep`: an answer's experts, counted and kept; a prompt's, neither."""
        if not keep and self.kept is not None and self.kept.layer == layer:
            return self._from_held(layer, tensors, experts)
        return self._fetch(layer, tensors, experts, keep)

    def _count(self, layer: int, experts: list, n_experts: int):
        counts = self.use.get(layer)
        if counts is None:
            counts = self.use[layer] = np.zeros(n_experts, dtype=np.int64)
        np.add.at(counts, np.asarray(experts, dtype=np.int64), 1)

    def _fetch(self, layer: int, tensors: tuple, experts: list, keep: bool) -> list:
        if keep:
            self._count(layer, experts, tensors[0].shape[0])
        distinct = list(dict.fromkeys(experts))
        absent = [e for e in distinct if (layer, e) not in self.lru]
        self.misses += len(absent)
        self.hits += len(experts) - len(absent)
        fresh = self._read_experts(tensors, absent)
        for e in distinct:  # this call's experts become the most recent, in the order the call names them
            if e not in fresh:
                self.lru.stamp((layer, e), self._tick())
            elif keep:
                nbytes = sum(a.numel() for a in fresh[e])
                self.lru.put((layer, e), fresh[e], nbytes, self._tick())
                self.held += nbytes
        if self.held > self.budget:
            self._evict(mine={(layer, e) for e in distinct})
        return [fresh[e] if e in fresh else self.lru[(layer, e)][0] for e in experts]

    def _evict(self, mine: set):
        """Drops the least recently used residents until the budget holds, none of `mine` (the call in progress)."""
        for key in list(self.lru):
            if self.held <= self.budget:
                break
            if key not in mine:
                self.held -= self.lru.drop(key)

    def _from_held(self, layer: int, tensors: tuple, experts: list) -> list:
        """A held layer's experts: views of its whole tensors, or each read once while the layer is held."""
        held = self.kept
        if held.stacks is not None:
            sizes = [self._per_expert(t) for t in tensors]
            return [tuple(s.narrow(0, e * n, n) for s, n in zip(held.stacks, sizes)) for e in experts]
        need = [e for e in dict.fromkeys(experts) if e not in held.loose]
        if need:
            held.loose.update(zip(need, self._fetch(layer, tensors, need, False)))
        return [held.loose[e] for e in experts]

    # ---- a layer whole

    def _gaps(self, layer: int, tensors: tuple) -> list:
        """The layer's experts in file order as runs (first, count, resident)."""
        resident = np.fromiter(((layer, e) in self.lru for e in range(tensors[0].shape[0])), dtype=bool)
        return _runs(resident)

    def _read_gaps(self, tensors: tuple, runs: list) -> list:
        """Per tensor, the host buffers of the runs not resident (files only: safe on the read-ahead thread)."""
        gaps = [(first, count) for first, count, resident in runs if not resident]
        host = self._read_all([(t, first, count) for t in tensors for first, count in gaps])
        return [host[j * len(gaps) : (j + 1) * len(gaps)] for j in range(len(tensors))]

    def _assemble(self, layer: int, tensors: tuple, runs: list, host: list) -> list:
        """Each tensor whole on the device, in file order: resident experts copied, the read gaps uploaded."""
        out = []
        for j, t in enumerate(tensors):
            one = self._per_expert(t)
            whole = torch.empty(t.shape[0] * one, dtype=torch.uint8, device=self.device)
            gaps = iter(host[j])
            for first, count, resident in runs:
                span = whole.narrow(0, first * one, count * one)
                if resident:
                    for i in range(count):
                        span.narrow(0, i * one, one).copy_(self.lru[(layer, first + i)][0][j])
                else:
                    span.copy_(next(gaps), non_blocking=True)
            out.append(whole)
        return out

    def _whole_now(self, layer: int, tensors: tuple) -> list:
        runs = self._gaps(layer, tensors)
        return self._assemble(layer, tensors, runs, self._read_gaps(tensors, runs))

    def whole(self, tensors: tuple, layer: int | None = None) -> list:
        """A layer's three tensors with every expert, resident ones copied on the device and the rest read
        (strata_mlx/paged.py:199-206); kept only while the layer is held."""
        held = self.kept
        if held is None or held.layer != layer:
            return self._whole_now(layer, tensors)
        if held.stacks is None:
            held.stacks = self._whole_now(layer, tensors)
            held.loose = {}  # the stacks hold whatever was read one by one
        return held.stacks

    # ---- a prompt's layers

    def hold(self, layer: int):
        """Until `release` or the next `hold`, the prompt's chunks read each of this layer's experts once: the layer
        whole if it was read ahead, else each expert the first time a chunk uses it (strata_mlx/paged.py:162-197)."""
        stacks = None
        if self.coming is not None:
            ahead, runs, future = self.coming
            self.coming = None
            t0 = time.perf_counter()
            if ahead == layer:
                stacks = self._assemble(layer, self.layers[layer], runs, future.result())
            else:
                future.exception()  # another layer's reads: finished, not used
            self.waited_s += time.perf_counter() - t0
        self.kept = _Held(layer, stacks)

    def ahead(self, layer: int):
        """Starts reading the gaps of `layer` on a thread of its own, for that layer's `hold`."""
        if self.coming is not None and self.coming[0] == layer:
            return
        self.release_ahead()
        tensors = self.layers[layer]
        runs = self._gaps(layer, tensors)
        self.coming = (layer, runs, self._ahead.submit(self._read_gaps, tensors, runs))

    def release_ahead(self):
        if self.coming is not None:
            self.coming[2].exception()
            self.coming = None

    def release(self):
        self.kept = None
        self.release_ahead()

    # ---- filling and counting

    def clear(self):
        """Lets go of every expert and of the counts of their use."""
        self.lru.clear()
        self.use.clear()
        self.held = 0
        self.release()

    def preload(self, counts: np.ndarray, group: int = 512) -> int:
        """Fills the free budget with the experts that `counts` (layers, experts) says are used most, in order of
        use until one does not fit; the least used of them are the oldest residents, the first to leave
        (strata_mlx/paged.py:292-315). Returns how many were read."""
        if not self.layers or counts.ndim != 2 or counts.shape[0] <= max(self.layers):
            return 0
        n_experts = counts.shape[1]
        if any(ts[0].shape[0] != n_experts for ts in self.layers.values()):
            return 0
        layers = np.array(sorted(self.layers), dtype=np.int64)
        lay = np.repeat(layers, n_experts)
        exp = np.tile(np.arange(n_experts, dtype=np.int64), layers.size)
        uses = counts[layers].reshape(-1).astype(np.int64)
        resident = np.fromiter(((int(l), int(e)) in self.lru for l, e in zip(lay, exp)), dtype=bool, count=lay.size)
        pick = np.flatnonzero((uses > 0) & ~resident)
        pick = pick[np.argsort(-uses[pick], kind="stable")]  # most used first; ties by layer, then expert
        size = {int(l): sum(self._per_expert(t) for t in self.layers[int(l)]) for l in layers}
        bytes_each = np.array([size[int(l)] for l in lay[pick]], dtype=np.int64)
        pick = pick[np.cumsum(bytes_each) <= self.budget - self.held]
        chosen = [(int(lay[i]), int(exp[i])) for i in pick[::-1]]  # least used first: the oldest ticks
        for a in range(0, len(chosen), group):
            part = chosen[a : a + group]
            got = {}
            for layer in dict.fromkeys(l for l, _ in part):
                got[layer] = self._read_experts(self.layers[layer], [e for l, e in part if l == layer])
            for layer, e in part:
                self.lru.put((layer, e), got[layer][e], size[layer], self._tick())
                self.held += size[layer]
        return len(chosen)

    def profile(self, before: np.ndarray | None = None) -> np.ndarray | None:
        """Uses of each expert, (layers, experts): this run's count plus half of `before` when it has that shape,
        so that recent use weighs more than old (strata_mlx/paged.py:317-328)."""
        if not self.layers:
            return None
        shape = (max(self.layers) + 1, next(iter(self.layers.values()))[0].shape[0])
        out = np.zeros(shape, dtype=np.uint32)
        if before is not None and before.shape == shape:
            out += np.right_shift(before.astype(np.uint32), 1)
        for layer, counts in self.use.items():
            out[layer, : counts.size] += counts.astype(np.uint32)
        return out


class PagedSwitchGLU:
    """A layer's routed experts kept in an ExpertStore, called like mlx-lm's SwitchGLU (and blocks.BlockSwitchGLU):
    (x, indices) -> down(silu(gate x) * up x) per pair (strata_mlx/paged.py:373-419). gate, up, down: the layer's
    gguf.Tensor expert stacks."""

    def __init__(self, layer: int, store: ExpertStore, gate, up, down):
        for t in (gate, up, down):
            if t.type not in BLOCK:
                raise ValueError(f"{t.name}: {t.type} experts are not supported")
        self.layer, self.store, self.tensors = layer, store, (up, gate, down)
        store.layers[layer] = self.tensors

    @staticmethod
    def _stack_linear(blocks: torch.Tensor, t, experts: int) -> BlockSwitchLinear:
        lin = BlockSwitchLinear(blocks, t.type, (experts, *t.shape[1:]))
        lin.unpack_from = 1 << 62  # never a float copy of the stack: the store exists because memory is short
        return lin

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        routes = indices.cpu().numpy()  # the layer waits here for its router
        if routes.size <= SEPARATE_UPTO:
            return self._pairwise(x, routes)
        distinct, local = np.unique(routes, return_inverse=True)
        if distinct.size >= WHOLE_FROM:
            stacks = self.store.whole(self.tensors, self.layer)
            experts = self.tensors[0].shape[0]
        else:
            got = self.store.get(self.layer, self.tensors, distinct.tolist(), keep=routes.size <= KEEP_UPTO)
            stacks = [_stacked([g[j] for g in got]) for j in range(3)]
            experts = distinct.size
            indices = torch.from_numpy(local.reshape(routes.shape).astype(np.int32)).to(x.device)
        up, gate, down = (self._stack_linear(s, t, experts) for s, t in zip(stacks, self.tensors))
        return switch_glu(x, indices, up, gate, down)

    def _pairwise(self, x: torch.Tensor, routes: np.ndarray) -> torch.Tensor:
        """A few pairs: no stack; the kernels read each pair's expert where it lies."""
        k = routes.shape[-1] if routes.ndim else 1
        distinct = list(dict.fromkeys(routes.reshape(-1).tolist()))
        where = dict(zip(distinct, self.store.get(self.layer, self.tensors, distinct)))
        per_pair = [where[e] for e in routes.reshape(-1).tolist()]
        up_t, gate_t, down_t = self.tensors
        inner, width = up_t.shape[1], up_t.shape[2]
        rows = x.reshape(-1, width)
        g = matvec_separate([p[1] for p in per_pair], gate_t.type, inner, width, rows, k)
        u = matvec_separate([p[0] for p in per_pair], up_t.type, inner, width, rows, k)
        y = matvec_separate([p[2] for p in per_pair], down_t.type, width, inner, swiglu(g, u), 1)
        return y.reshape(*routes.shape, width)


def load_profile(path: str | None) -> np.ndarray | None:
    """The use counts saved at `path`; None when there is no path, no file, or the file cannot be read."""
    if not path:
        return None
    try:
        return np.load(path)
    except (OSError, ValueError):
        return None


def save_profile(path: str, counts: np.ndarray) -> None:
    """Writes `counts` to a temporary file in the same folder and renames it over `path`: a reader finds the old
    file or the new one, never a part."""
    folder = os.path.dirname(os.path.abspath(path))
    os.makedirs(folder, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=folder, prefix=".profile-", suffix=".npy")
    try:
        with os.fdopen(fd, "wb") as f:
            np.save(f, counts)
        os.replace(tmp, path)
    except BaseException:
        with contextlib.suppress(OSError):
            os.unlink(tmp)
        raise
