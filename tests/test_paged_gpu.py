"""The paged expert store's layer (strata_mlx_b200/paged.PagedSwitchGLU) against the same layer with every expert
resident (blocks.BlockSwitchGLU), in a budget of a few experts so that the store reads and drops them between calls:
a few pairs through each pair's own expert buffer (the kernel taking a device array of expert pointers), a larger
window through a stack of the experts it uses, a prompt through the layer whole (strata_mlx/paged.py:388-419)."""

import numpy as np
import pytest
import torch

from strata_mlx_b200 import blocks as B
from strata_mlx_b200 import gguf as G
from strata_mlx_b200 import paged as P

from .paged_model import E, H, layer_tensors, write

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return write(str(tmp_path_factory.mktemp("paged_gpu") / "experts.gguf"))


def resident(model, layer):
    gate, up, down = layer_tensors(model, layer)
    lin = [B.BlockSwitchLinear(G.to_device(t), t.type, t.shape) for t in (gate, up, down)]
    return B.BlockSwitchGLU(*lin)


def routes(tokens, k, seed, pool=None):
    rng = np.random.default_rng(seed)
    pool = np.arange(E) if pool is None else np.asarray(pool)
    return np.stack([rng.choice(pool, k, replace=False) for _ in range(tokens)]).astype(np.int32)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_the_paged_layer_gives_the_resident_layers_results(cuda, model, monkeypatch, dt):
    dev = torch.device("cuda", 0)
    size = sum(t.data.nbytes // t.shape[0] for t in layer_tensors(model, 0))
    store = P.ExpertStore(5 * size, threads=4, device=dev)
    layers = [P.PagedSwitchGLU(l, store, *layer_tensors(model, l)) for l in (0, 1)]
    full = [resident(model, l) for l in (0, 1)]
    rng = np.random.default_rng(7)
    for step, tokens in enumerate((1, 2, 40, 1, 40)):  # separate, separate, a stack, and again after drops
        for l in (0, 1):
            # a window's experts a subset, so that the stack's local indices are not the layer's
            pool = [2, 3, 5, 7, 8, 10, 11] if tokens > 2 else None
            idx = torch.from_numpy(routes(tokens, 4, 10 * step + l, pool)).to(dev)
            x = torch.from_numpy(rng.standard_normal((tokens, H)).astype(np.float32)).to(dev).to(dt)
            got, want = layers[l](x, idx), full[l](x, idx)
            torch.cuda.synchronize()
            assert got.shape == want.shape == (tokens, 4, H)
            if tokens * 4 > P.SEPARATE_UPTO:  # the same kernels on a stack of the used experts: the same bits
                assert torch.equal(got, want)
            else:  # each pair's expert where it lies: the exact kernel, within the products' bar
                err = (got.float() - want.float()).abs().max().item()
                assert err <= 2e-2 * want.float().abs().max().item(), err
    assert store.misses > 0 and store.hits > 0
    # a prompt that uses most of a layer's experts takes the layer whole and keeps none of it
    monkeypatch.setattr(P, "WHOLE_FROM", 8)
    held = dict(store.lru)
    idx = torch.from_numpy(routes(40, 4, 99)).to(dev)
    x = torch.from_numpy(rng.standard_normal((40, H)).astype(np.float32)).to(dev).to(dt)
    got, want = layers[0](x, idx), full[0](x, idx)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert dict(store.lru).keys() == held.keys()
    from strata_mlx_b200 import _lib

    _lib.check_device_errors(dev)
