"""The paged expert store's rules on the host (strata_mlx_b200/paged.py, the reference's strata_mlx/paged.py:105-419):
the bytes it holds are the file's, the least recently used go first within the budget, a call keeps its own experts,
a layer whole and a layer read ahead, preloading by counts and the counts it keeps, and the layer's three ways to its
products. No GPU: the store on the CPU, the kernels stood in for by the oracle."""

import numpy as np
import pytest
import torch

from oracle import blocks_ref as R
from strata_mlx_b200 import paged as P

from .paged_model import E, layer_tensors, write


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return write(str(tmp_path_factory.mktemp("paged") / "experts.gguf"))


def tensors(model, layer=0):
    gate, up, down = layer_tensors(model, layer)
    return (up, gate, down)


def file_bytes(t, e):
    one = t.data.nbytes // t.shape[0]
    return t.data[e * one : (e + 1) * one]


def expert_size(ts):
    return sum(t.data.nbytes // t.shape[0] for t in ts)


def store_for(model, experts_held):
    s = P.ExpertStore(experts_held * expert_size(tensors(model)), threads=4, device="cpu")
    for layer in (0, 1):
        s.layers[layer] = tensors(model, layer)
    return s


def test_the_store_holds_the_files_bytes(model):
    s = store_for(model, 100)
    ts = tensors(model)
    got = s.get(0, ts, [3, 1, 3])
    for e, arrays in zip([3, 1, 3], got):
        for t, a in zip(ts, arrays):
            assert np.array_equal(a.numpy(), file_bytes(t, e))
    assert (s.misses, s.hits) == (2, 1)  # expert 3 read once
    assert s.bytes_read == 2 * expert_size(ts)
    assert set(s.lru) == {(0, 3), (0, 1)} and s.held == 2 * expert_size(ts)


def test_the_least_recently_used_go_first_within_the_budget(model):
    s = store_for(model, 2)
    ts = tensors(model)
    for e in (0, 1, 0, 2):
        s.get(0, ts, [e])
    assert list(s.lru) == [(0, 0), (0, 2)]  # 1 was the least recent when 2 came
    assert s.held <= s.budget


def test_a_call_keeps_every_expert_it_uses(model):
    s = store_for(model, 1)
    ts = tensors(model)
    got = s.get(0, ts, [4, 5, 6])
    assert len(got) == 3 and set(s.lru) == {(0, 4), (0, 5), (0, 6)}  # over budget, but none of them goes
    s.get(0, ts, [7])
    assert list(s.lru) == [(0, 7)]


def test_a_prompts_experts_are_not_kept_or_counted(model):
    s = store_for(model, 100)
    ts = tensors(model)
    s.get(0, ts, [2, 3], keep=False)
    assert not s.lru and not s.use


def test_a_layer_whole_is_the_file_and_keeps_nothing(model):
    s = store_for(model, 100)
    ts = tensors(model)
    s.get(0, ts, [2, 9])
    whole = s.whole(ts, 0)
    for t, a in zip(ts, whole):
        assert np.array_equal(a.numpy(), t.data.reshape(-1))
    assert set(s.lru) == {(0, 2), (0, 9)}


def test_a_layer_read_ahead_is_what_its_hold_takes(model):
    s = store_for(model, 100)
    ts = tensors(model, 1)
    s.get(1, ts, [5])
    s.ahead(1)
    s.hold(1)
    stacks = s.kept.stacks
    for t, a in zip(ts, stacks):
        assert np.array_equal(a.numpy(), t.data.reshape(-1))
    got = s.get(1, ts, [0, 11], keep=False)  # slices of the held layer
    for e, arrays in zip([0, 11], got):
        for t, a in zip(ts, arrays):
            assert np.array_equal(a.numpy(), file_bytes(t, e))
    s.release()
    assert s.kept is None and s.coming is None


def test_preload_takes_the_most_used_and_profile_halves_the_past(model):
    s = store_for(model, 3)
    counts = np.zeros((2, E), dtype=np.uint32)
    counts[0, [1, 4, 7, 8]] = [5, 9, 1, 7]
    counts[1, 2] = 6
    assert s.preload(counts) == 3
    assert list(s.lru) == [(1, 2), (0, 8), (0, 4)]  # the least used first: the first to go
    s.get(0, tensors(model), [4, 4, 1])
    prof = s.profile(counts)
    assert prof[0, 4] == 9 // 2 + 2 and prof[0, 1] == 5 // 2 + 1 and prof[1, 2] == 3


def test_profiles_are_saved_and_loaded(tmp_path):
    counts = np.arange(24, dtype=np.uint32).reshape(2, 12)
    path = str(tmp_path / "use" / "counts.npy")
    P.save_profile(path, counts)
    assert np.array_equal(P.load_profile(path), counts)
    assert P.load_profile(str(tmp_path / "none.npy")) is None


def test_reads_of_consecutive_experts_are_runs(model, monkeypatch):
    s = store_for(model, 100)
    ts = tensors(model)
    calls = []
    real = s._pread
    monkeypatch.setattr(s, "_pread", lambda t, first, count: calls.append((first, count)) or real(t, first, count))
    got = s.get(0, ts, [6, 2, 3, 4, 9])
    assert sorted(set(calls)) == [(2, 3), (6, 1), (9, 1)] and len(calls) == 3 * len(ts)
    for e, arrays in zip([6, 2, 3, 4, 9], got):
        for t, a in zip(ts, arrays):
            assert np.array_equal(a.numpy(), file_bytes(t, e))
    assert s.bytes_read == 5 * expert_size(ts)


class _Weights:
    """Stands in for BlockSwitchLinear: the stack's weights through the oracle's decoder."""

    def __init__(self, blocks, kind, shape):
        self.w = R.dequantize(blocks.numpy(), kind, tuple(shape)).astype(np.float64)
        self.unpack_from = 0


def _silu_glu(g, u):
    return g / (1.0 + np.exp(-g)) * u


def _fake_switch_glu(x, indices, up, gate, down):
    idx = indices.numpy().reshape(x.shape[0], -1)
    xs = x.numpy()
    out = np.zeros((*idx.shape, down.w.shape[1]))
    for t in range(idx.shape[0]):
        for j, e in enumerate(idx[t]):
            out[t, j] = down.w[e] @ _silu_glu(gate.w[e] @ xs[t], up.w[e] @ xs[t])
    return torch.from_numpy(out)


def _fake_matvec_separate(experts, kind, rows, cols, x, share):
    xs = x.numpy().reshape(-1, cols)
    return torch.from_numpy(np.stack([R.dequantize(b.numpy(), kind, (1, rows, cols))[0].astype(np.float64)
                                      @ xs[p // share] for p, b in enumerate(experts)]))


def test_the_layer_takes_pairs_stacks_and_whole_layers_to_the_same_products(model, monkeypatch):
    """PagedSwitchGLU on the host: a few pairs (each expert where it lies), a larger window (a stack of the experts it
    uses, routes renumbered into it) and a prompt using most experts (the layer whole) give the products of the
    file's own experts."""
    monkeypatch.setattr(P, "BlockSwitchLinear", _Weights)
    monkeypatch.setattr(P, "switch_glu", _fake_switch_glu)
    monkeypatch.setattr(P, "matvec_separate", _fake_matvec_separate)
    monkeypatch.setattr(P, "swiglu", lambda g, u: torch.from_numpy(_silu_glu(g.numpy(), u.numpy())))
    gate, up, down = layer_tensors(model, 1)
    wg, wu, wd = (R.dequantize(t.data, t.type, t.shape).astype(np.float64) for t in (gate, up, down))
    s = P.ExpertStore(100 * expert_size((up, gate, down)), threads=4, device="cpu")
    glu = P.PagedSwitchGLU(1, s, gate, up, down)
    rng = np.random.default_rng(8)
    width = up.shape[2]
    for tokens, whole_from in ((5, P.WHOLE_FROM), (40, P.WHOLE_FROM), (40, 6)):
        monkeypatch.setattr(P, "WHOLE_FROM", whole_from)
        idx = np.stack([rng.choice(E, 4, replace=False) for _ in range(tokens)]).astype(np.int32)
        idx[:, 0] = np.arange(tokens) % 7  # at most 10 distinct experts a window before the last case
        x = rng.standard_normal((tokens, width)) * 0.1
        got = glu(torch.from_numpy(x), torch.from_numpy(idx)).numpy()
        want = np.stack([[wd[e] @ _silu_glu(wg[e] @ x[t], wu[e] @ x[t]) for e in idx[t]] for t in range(tokens)])
        assert got.shape == (tokens, 4, width)
        np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-12)
    assert s.misses > 0 and s.hits > 0 and s.lru
