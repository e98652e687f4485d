"""Expert parallelism's exchange (strata_mlx_b200/ep.py) on CPU ranks over gloo: the all-gather of the window, the
sum of the pairs' outputs over ranks and the combine give every rank's token the bits the single-device block
gives it. The device steps (sc_moe_decode_layer_ep, sc_moe_decode_combine) are played by the oracle here, on the
experts of each rank only; their CUDA form is checked against the single-device layer on two GPUs in
test_ep_gpu.py."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import blocks_ref as R
from strata_mlx_b200 import ep as EP
from strata_mlx_b200.synthetic import layer_numpy

H, I, E, K, S = 256, 64, 8, 3, 64
KINDS = ("IQ3_S", "IQ3_S", "Q2_0")
ND = "bfloat16"


def layer_weights():
    rng = np.random.default_rng(3)
    L = layer_numpy(rng, H, I, E, KINDS, shared_inter=S)
    W = {k: R.dequantize(L[k], kind, shp) for k, kind, shp in (
        ("gate", KINDS[0], (E, I, H)), ("up", KINDS[1], (E, I, H)), ("down", KINDS[2], (E, H, I)),
        ("sgate", KINDS[0], (1, S, H)), ("sup", KINDS[1], (1, S, H)), ("sdown", KINDS[2], (1, H, S)))}
    return L, W


def token(rank):
    return np.random.default_rng(100 + rank).standard_normal((1, H)).astype(np.float32)


class OracleEP(EP.EPMoEDecodeLayer):
    """The exchange of EPMoEDecodeLayer with the oracle in the device steps' place, on this rank's experts only."""

    def __init__(self, L, W):
        self._setup(E, K, H, torch.float32, None)
        self.L, self.W, self._bufs = L, W, {}

    def _local(self, X):
        x = R.round_to(X.numpy(), ND)
        logits = R.router(self.L["router"], x).astype(np.float32)
        idx = R.top_k(logits, K)
        wts = R.softmax_topk(logits, idx)
        T = x.shape[0]
        y = np.zeros((T, K, H), dtype=np.float32)
        for t in range(T):
            for k in range(K):
                e = int(idx[t, k])
                if not self.e0 <= e < self.e1:
                    continue  # another rank's expert: its owner fills this pair
                g = R.round_to(R.matvec(self.W["gate"], [e], x[t : t + 1], 1), ND)
                u = R.round_to(R.matvec(self.W["up"], [e], x[t : t + 1], 1), ND)
                h = R.swiglu(g, u, ND)
                y[t, k] = R.round_to(R.matvec(self.W["down"], [e], h, 1), ND)[0]
        zero = np.zeros(T, dtype=np.int64)
        sg = R.round_to(R.matvec(self.W["sgate"], zero, x, 1), ND)
        su = R.round_to(R.matvec(self.W["sup"], zero, x, 1), ND)
        s = R.round_to(R.matvec(self.W["sdown"], zero, R.swiglu(sg, su, ND), 1), ND)
        gs = R.round_to(R.router(self.L["shared_gate"].reshape(1, -1), x), ND).reshape(T)
        return torch.from_numpy(y), (wts, gs, s)

    def _combine(self, Y, state):
        wts, gs, s = state
        return torch.from_numpy(R.moe_combine(Y.numpy(), wts, gs, s, ND))


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L, W = layer_weights()
        layer = OracleEP(L, W)
        assert (layer.e0, layer.e1) == EP.expert_range(rank, world, E)
        got = layer(torch.from_numpy(token(rank))).numpy()
        want, _, _ = R.moe_layer(token(rank), L["router"], L["shared_gate"], W["gate"], W["up"], W["down"],
                                 W["sgate"][0], W["sup"][0], W["sdown"][0], K, ND)
        out[rank] = bool(np.array_equal(got, want))
    finally:
        torch.distributed.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_every_rank_gets_the_single_device_bits(world):
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_rank, args=(world, free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert dict(out) == {r: True for r in range(world)}


def test_expert_ranges_cover_the_experts_once():
    for world in (1, 2, 4, 8):
        got = [EP.expert_range(r, world, 512) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == 512
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    with pytest.raises(ValueError):
        EP.expert_range(0, 3, 512)


def test_a_rank_keeps_its_experts_bytes():
    blocks = torch.arange(8 * 6, dtype=torch.uint8)  # 8 experts of 6 bytes
    assert torch.equal(EP.local_experts(blocks, 8, 1, 4), torch.arange(12, 24, dtype=torch.uint8))
