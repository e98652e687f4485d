"""The synthetic decoder of configurations 4 and 5 (decoder.SyntheticDecoder: attention over a paged cache and the
library's MoE blocks, layer after layer) against the CPU oracle (decoder.oracle_layer: a layer in float32 with the
GPU's bfloat16 rounding points and the MoE block of oracle/blocks_ref.py), teacher-forced on a shortened stack: a
prompt read in windows of 8 tokens, then a verify pass of 1 + 4 tokens.

Each layer is checked on the GPU's own input for it (the tokens, and every layer's activations, forced on both): a
one-unit difference of a bfloat16 activation upstream can move a token's 10th and 11th router logits past each other
(on random weights such near-ties are common), and a different expert is a different output; so a layer's outputs are
compared for the tokens whose routes the oracle and the GPU share, and those must be most of them. The top-1 token of
the output head must be the oracle's wherever the oracle's best two logits are apart by more than the logits' error."""

import numpy as np
import pytest
import torch

from strata_mlx_b200 import decoder as D

pytestmark = pytest.mark.gpu

E, I, S, K, VOCAB = 64, 512, 512, 10, 512


def blocks_of(L):
    router, gate, up, down, sg, su, sd, sgw = L["base"]._keep
    kind = L["kind"]
    return {"router": router.cpu().numpy(), "gate": gate.cpu().numpy(), "up": up.cpu().numpy(),
            "down": down.cpu().numpy(), "sgate": sg.cpu().numpy(), "sup": su.cpu().numpy(), "sdown": sd.cpu().numpy(),
            "shared_gate": sgw.cpu().numpy(), "kinds": (kind,) * 3, "shared_kinds": (kind,) * 3, "inter": I,
            "top_k": K, "shared_inter": S}


@pytest.mark.parametrize("dense", ["bf16", "Q8_0"])
def test_teacher_forced_passes_match_the_oracle(cuda, dense):
    kinds = ["Q2_0", "IQ3_S"] if dense == "bf16" else ["IQ3_XXS", "Q2_0"]
    dec = D.SyntheticDecoder(2, kinds, dense=dense, experts=E, vocab=VOCAB, max_pos=256, seed=3)
    cache = dec.cache(64)
    blocks = [blocks_of(L) for L in dec.layers]
    ck = [np.zeros((0, dec.kv_heads, D.HEAD_DIM), np.float32) for _ in dec.layers]
    cv = [np.zeros((0, dec.kv_heads, D.HEAD_DIM), np.float32) for _ in dec.layers]
    rng = np.random.default_rng(5)
    tokens = rng.integers(0, VOCAB, 29)
    pos, compared, same_routes, top1_checked, top1_same = 0, 0, 0, 0, 0
    for w in (8, 8, 8, 5):  # three windows of a prompt, then a verify pass of 1 + 4 tokens
        win = tokens[pos : pos + w]
        trace = []
        got = dec.forward(torch.from_numpy(win).cuda(), cache, trace=trace).cpu().numpy()
        torch.cuda.synchronize()
        dec.check_errors()
        xs = [t.float().cpu().numpy() for t in trace]
        for l in range(dec.n_layers):
            gpu_idx = dec.layers[l]["base"].routes(w, "cuda")[0].view(torch.int32).cpu().numpy()
            want, parts = D.oracle_layer(dec, l, xs[l], pos, ck, cv, blocks[l])
            same = (np.sort(gpu_idx, -1) == np.sort(parts["idx"].astype(np.int32), -1)).all(-1)
            compared += w
            same_routes += int(same.sum())
            d = np.abs(xs[l + 1] - want)[same]
            # two units of bfloat16 at the residual stream's magnitude, and a little for the window's sums
            assert d.max(initial=0.0) <= 2 ** -6 * np.abs(want).max() + 1e-6, (pos, l, d.max())
        want = D.oracle_head(dec, xs[-1])
        diff = np.abs(got - want).max()
        assert diff <= 1e-3 * np.abs(want).max(), diff
        for i in range(w):
            top2 = np.sort(want[i])[-2:]
            if top2[1] - top2[0] > 2 * diff:
                top1_checked += 1
                top1_same += int(np.argmax(got[i]) == np.argmax(want[i]))
        dec.advance(cache, w)
        pos += w
    assert int(cache.pos.item()) == 29
    assert same_routes >= 0.9 * compared, (same_routes, compared)
    assert top1_checked >= 25 and top1_same == top1_checked, (top1_checked, top1_same)
