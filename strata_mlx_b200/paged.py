"""Experts kept within a budget of device memory and read from the model's files as the routes ask for them: the
paged expert store of strata_mlx/paged.py:105-419 (ExpertStore, PagedSwitchGLU) on CUDA.

The decode path of this library keeps every expert resident, as a B200 (180 GB a GPU) holds these models whole; the
store is for the hosts where that does not hold -- a smaller GPU, several models sharing one, or a budget the caller
chooses -- and keeps the reference's rules:

  * an expert in memory is its three tensors (up, gate, down) as the file's blocks, device uint8 tensors of their
    own, in one store for every layer; past the budget the least recently used go first;
  * a layer waits on the host for its routes, reads the experts it lacks (parallel reads of the file into pinned
    host memory, copied to the device on the current stream), and hands each pair's expert to the kernels where it
    lies (`blocks.matvec_separate`, the CUDA kernel taking a device array of expert pointers) for up to SEPARATE_UPTO
    pairs; a larger window goes through `blocks.switch_glu` on a stack of the experts it uses, kept only for an
    answer's sizes (KEEP_UPTO pairs); a prompt using WHOLE_FROM or more of a layer's experts takes the layer's
    tensors whole, those held copied on the device and the rest read, and keeps none of what it read;
  * `hold` / `ahead` / `release` let a prompt's chunks read a layer once, the next one read ahead on a thread;
  * `preload` fills the free budget with the most used experts of a count table, `profile` gives this run's counts
    with earlier ones halved, `load_profile` / `save_profile` keep them between runs.

Memory is the device's: `fit` sets the budget from what the device has free now, not from a laptop's RAM rules. All
work goes on the current CUDA stream: a dropped expert's memory returns to torch's caching allocator, which hands it
out again only in that stream's order, after the kernels that read it.
"""

from __future__ import annotations

import os
import threading
import time
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from .blocks import BLOCK, BlockSwitchLinear, matvec_separate, swiglu, switch_glu

WHOLE_FROM = 384  # strata_mlx/paged.py:44: a layer's experts used by one call from which its tensors are taken whole
KEEP_UPTO = 640  # :45: pairs in one call up to which what was read stays in the store (an answer, not a prompt)
SEPARATE_UPTO = 80  # :47: pairs up to which each pair's expert goes to the kernels where it lies
WORKING = int(2e9)  # device bytes `fit` leaves for everything but the experts: activations, workspaces, the graph
LEAST = int(0.5e9)  # the smallest budget `fit` sets


class ExpertStore:
    """The experts in device memory, within `budget` bytes."""

    def __init__(self, budget: int, threads: int = 8, device=None):
        self.budget, self.held = int(budget), 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.lru = OrderedDict()  # (layer, expert) -> ((up, gate, down) device tensors, bytes)
        self.layers = {}  # layer -> its three gguf.Tensor (up, gate, down)
        self.use = {}  # (layer, expert) -> times an answer asked for it
        self.fds = {}
        self.pool = ThreadPoolExecutor(threads)
        # while a prompt's chunks go through a layer: [layer, its tensors whole or None, {expert: its tensors}]
        self.kept = None
        # a read ahead: (layer, what _join needs, the future of its reads); the thread only reads files
        self.reader, self.coming = ThreadPoolExecutor(1), None
        self.counting = threading.Lock()
        self.reset_stats()

    # ---- budget and statistics

    def fit(self, reserve: int = WORKING) -> int:
        """Sets the budget to the device memory free now, plus what the store holds, less `reserve`; at least LEAST."""
        free, _ = torch.cuda.mem_get_info(self.device)
        self.budget = max(LEAST, int(free) + self.held - int(reserve))
        return self.budget

    def reset_stats(self):
        self.hits = self.misses = self.bytes_read = 0
        self.read_s = 0.0
        self.waited_s = 0.0  # of the reads ahead, what a prompt still waited for

    # ---- reading the file

    def _fd(self, path: str) -> int:
        if path not in self.fds:
            self.fds[path] = os.open(path, os.O_RDONLY)
        return self.fds[path]

    @staticmethod
    def _one(t) -> int:
        return t.data.nbytes // t.shape[0]

    def _read_host(self, t, first: int, count: int) -> torch.Tensor:
        """Experts [first, first + count) of tensor t, as the file holds them, in pinned host memory."""
        n = count * self._one(t)
        buf = torch.empty(n, dtype=torch.uint8, pin_memory=self.device.type == "cuda")
        got = os.preadv(self._fd(t.path), [memoryview(buf.numpy())], t.offset + first * self._one(t))
        if got != n:
            raise OSError(f"{t.name}: short read ({got} of {n} bytes)")
        return buf

    def _upload(self, host: torch.Tensor) -> torch.Tensor:
        return host.to(self.device, non_blocking=True)

    def _read_experts(self, tensors: tuple, experts: list) -> dict:
        """Each expert's three tensors read from the files in parallel and put on the device."""
        t0 = time.perf_counter()
        jobs = [(e, t) for e in experts for t in tensors]
        host = list(self.pool.map(lambda job: self._read_host(job[1], job[0], 1), jobs))
        n = len(tensors)
        got = {e: tuple(self._upload(h) for h in host[i * n : (i + 1) * n]) for i, e in enumerate(experts)}
        with self.counting:
            self.read_s += time.perf_counter() - t0
            self.bytes_read += sum(h.numel() for h in host)
        return got

    # ---- experts one by one

    def get(self, layer: int, tensors: tuple, experts: list, keep: bool = True) -> list:
        """The (up, gate, down) device tensors of each of `experts`, read if the store lacks them. `keep`: an
        answer's experts, counted and kept; a prompt's, not (strata_mlx/paged.py:330-370)."""
        if not keep and self.kept is not None and self.kept[0] == layer:
            return self._held(layer, tensors, experts)
        return self._get(layer, tensors, experts, keep)

    def _get(self, layer: int, tensors: tuple, experts: list, keep: bool) -> list:
        if keep:
            for e in experts:
                self.use[(layer, e)] = self.use.get((layer, e), 0) + 1
        missing = [e for e in dict.fromkeys(experts) if (layer, e) not in self.lru]
        self.hits += len(experts) - len(missing)
        self.misses += len(missing)
        got = self._read_experts(tensors, missing) if missing else {}
        if keep:
            for e, arrays in got.items():
                size = sum(a.numel() for a in arrays)
                self.lru[(layer, e)] = (arrays, size)
                self.held += size
        out = []
        for e in experts:
            if e in got:
                out.append(got[e])
                if keep:
                    self.lru.move_to_end((layer, e))
            else:
                self.lru.move_to_end((layer, e))
                out.append(self.lru[(layer, e)][0])
        # this call's experts are the most recent; drop from the other end, never one this call uses
        while self.held > self.budget and len(self.lru) > len(set(experts)):
            _, (_, size) = self.lru.popitem(last=False)
            self.held -= size
        return out

    def _held(self, layer: int, tensors: tuple, experts: list) -> list:
        _, stacks, each = self.kept
        if stacks is not None:
            ones = [self._one(t) for t in tensors]
            return [tuple(s[e * one : (e + 1) * one] for s, one in zip(stacks, ones)) for e in experts]
        missing = [e for e in dict.fromkeys(experts) if e not in each]
        if missing:
            each.update(zip(missing, self._get(layer, tensors, missing, False)))
        return [each[e] for e in experts]

    # ---- a layer whole

    def whole(self, tensors: tuple, layer: int | None = None) -> list:
        """A layer's three tensors with every expert: those in the store copied on the device, the rest read; kept
        only while the layer is held."""
        if self.kept is None or self.kept[0] != layer:
            return self._layer(layer, tensors)
        if self.kept[1] is None:
            self.kept[1] = self._layer(layer, tensors)
            self.kept[2] = {}  # what was read one by one is all in there
        return self.kept[1]

    def _runs(self, layer, tensors: tuple) -> list:
        """The layer's experts in file order as runs (first, count, held)."""
        runs = []
        for e in range(tensors[0].shape[0]):
            held = (layer, e) in self.lru
            if runs and runs[-1][2] == held:
                runs[-1][1] += 1
            else:
                runs.append([e, 1, held])
        return [tuple(r) for r in runs]

    def _read_runs(self, tensors: tuple, runs: list) -> list:
        """The bytes of the runs the store lacks, per tensor, in pinned host memory (files only: safe on a thread)."""
        t0 = time.perf_counter()
        jobs = [(t, first, count) for t in tensors for first, count, held in runs if not held]
        host = list(self.pool.map(lambda job: self._read_host(*job), jobs))
        with self.counting:
            self.read_s += time.perf_counter() - t0
            self.bytes_read += sum(h.numel() for h in host)
        per = len(jobs) // len(tensors) if tensors else 0
        return [host[i * per : (i + 1) * per] for i in range(len(tensors))]

    def _join(self, layer, tensors: tuple, runs: list, host: list) -> list:
        """Each tensor whole on the device: held experts copied, read runs uploaded, in file order."""
        out = []
        for j, t in enumerate(tensors):
            one = self._one(t)
            dst = torch.empty(t.shape[0] * one, dtype=torch.uint8, device=self.device)
            reads = iter(host[j])
            for first, count, held in runs:
                if held:
                    for e in range(first, first + count):
                        dst[e * one : (e + 1) * one].copy_(self.lru[(layer, e)][0][j])
                else:
                    dst[first * one : (first + count) * one].copy_(next(reads), non_blocking=True)
            out.append(dst)
        return out

    def _layer(self, layer, tensors: tuple) -> list:
        runs = self._runs(layer, tensors)
        return self._join(layer, tensors, runs, self._read_runs(tensors, runs))

    def hold(self, layer: int):
        """From here to `release` or the next `hold`, what a prompt's chunks read of this layer is read once: the
        layer whole if it was read ahead, else each expert the first time a chunk uses it."""
        stacks = None
        if self.coming is not None:
            ahead, runs, read = self.coming
            self.coming = None
            t0 = time.perf_counter()
            if ahead == layer:
                stacks = self._join(layer, self.layers[layer], runs, read.result())
            else:
                read.exception()  # waited for; nothing of it is used
            self.waited_s += time.perf_counter() - t0
        self.kept = [layer, stacks, {}]

    def ahead(self, layer: int):
        """Starts reading, on a thread of its own, the experts of `layer` the store lacks, for that layer's `hold`."""
        if self.coming is not None and self.coming[0] == layer:
            return
        self.release_ahead()
        tensors = self.layers[layer]
        runs = self._runs(layer, tensors)
        self.coming = (layer, runs, self.reader.submit(self._read_runs, tensors, runs))

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
        """Fills the free budget with the experts `counts` (layers, experts) says are used most, the least used of
        them first in the store's order (the first to be dropped). Returns how many were read."""
        if not self.layers or counts.ndim != 2 or counts.shape[0] <= max(self.layers) \
                or any(t[0].shape[0] != counts.shape[1] for t in self.layers.values()):
            return 0
        size = {layer: sum(self._one(t) for t in tensors) for layer, tensors in self.layers.items()}
        order = sorted(((int(counts[layer, e]), layer, e) for layer in self.layers for e in range(counts.shape[1])
                        if counts[layer, e] > 0 and (layer, e) not in self.lru), reverse=True)
        chosen, room = [], self.budget - self.held
        for _, layer, e in order:
            if size[layer] > room:
                break
            chosen.append((layer, e))
            room -= size[layer]
        chosen.reverse()
        for a in range(0, len(chosen), group):
            part = chosen[a : a + group]
            for layer in dict.fromkeys(layer for layer, _ in part):
                mine = [e for l2, e in part if l2 == layer]
                for e, arrays in self._read_experts(self.layers[layer], mine).items():
                    self.lru[(layer, e)] = (arrays, size[layer])
                    self.held += size[layer]
            # keep the least-used-first order across layers of one group
            for key in part:
                self.lru.move_to_end(key)
        return len(chosen)

    def profile(self, before: np.ndarray | None = None) -> np.ndarray | None:
        """How often each expert was used, (layers, experts): this run's counts plus half of `before`, so that what
        the store is used for now weighs more than what it was used for once."""
        if not self.layers:
            return None
        shape = (max(self.layers) + 1, next(iter(self.layers.values()))[0].shape[0])
        out = np.zeros(shape, dtype=np.uint32)
        if before is not None and before.shape == shape:
            out += before.astype(np.uint32) // 2
        for (layer, e), n in self.use.items():
            out[layer, e] += n
        return out


class PagedSwitchGLU:
    """A layer's routed experts, called like mlx-lm's SwitchGLU (and blocks.BlockSwitchGLU), their blocks in an
    ExpertStore (strata_mlx/paged.py:373-419). gate, up, down: the layer's gguf.Tensor expert stacks."""

    def __init__(self, layer: int, store: ExpertStore, gate, up, down):
        for t in (gate, up, down):
            if t.type not in BLOCK:
                raise ValueError(f"{t.name}: {t.type} experts are not supported")
        self.layer, self.store, self.tensors = layer, store, (up, gate, down)
        store.layers[layer] = self.tensors

    @staticmethod
    def _linear(blocks: torch.Tensor, t, experts: int) -> BlockSwitchLinear:
        lin = BlockSwitchLinear(blocks, t.type, (experts, *t.shape[1:]))
        lin.unpack_from = 1 << 62  # never a float copy of the stack: the store is for memory that is short
        return lin

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        idx = indices.cpu().numpy()  # the layer waits here for its router
        used, local = np.unique(idx, return_inverse=True)
        if idx.size <= SEPARATE_UPTO:
            return self._separately(x, idx, used)
        if len(used) >= WHOLE_FROM:
            stacks, n = self.store.whole(self.tensors, self.layer), self.tensors[0].shape[0]
        else:
            each = self.store.get(self.layer, self.tensors, used.tolist(), keep=idx.size <= KEEP_UPTO)
            stacks = [torch.cat(col) if len(col) > 1 else col[0] for col in zip(*each)]
            n = len(used)
            indices = torch.from_numpy(local.reshape(idx.shape).astype(np.int32)).to(x.device)
        up, gate, down = (self._linear(b, t, n) for b, t in zip(stacks, self.tensors))
        return switch_glu(x, indices, up, gate, down)

    def _separately(self, x: torch.Tensor, idx: np.ndarray, used: np.ndarray) -> torch.Tensor:
        """A few pairs: no stack is built; each pair's expert goes to the kernel where it lies."""
        k = idx.shape[-1] if idx.ndim else 1
        by = dict(zip(used.tolist(), self.store.get(self.layer, self.tensors, used.tolist())))
        pairs = [by[e] for e in idx.reshape(-1).tolist()]
        up_t, gate_t, down_t = self.tensors
        inner, wide = up_t.shape[1], up_t.shape[2]
        xs = x.reshape(-1, wide)
        ups, gates, downs = zip(*pairs)
        h = swiglu(matvec_separate(list(gates), gate_t.type, inner, wide, xs, k),
                   matvec_separate(list(ups), up_t.type, inner, wide, xs, k))
        out = matvec_separate(list(downs), down_t.type, wide, inner, h, 1)
        return out.reshape(*idx.shape, wide)


def load_profile(path: str | None) -> np.ndarray | None:
    """The use counts saved at `path`, or None when there is no such file or it cannot be read."""
    try:
        if path and os.path.exists(path):
            return np.load(path)
    except (OSError, ValueError):
        pass
    return None


def save_profile(path: str, counts: np.ndarray) -> None:
    """Writes beside `path` and renames over it, so that a reader never finds half a file."""
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = f"{path}.{os.getpid()}.tmp"
    with open(tmp, "wb") as f:
        np.save(f, counts)
    os.replace(tmp, path)
