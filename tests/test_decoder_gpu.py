"""The synthetic decoder of configurations 4 and 5 (decoder.SyntheticDecoder: attention over a paged cache and the
library's MoE blocks, layer after layer) against the CPU oracle (decoder.oracle_forward: the same pass in float32 with
the GPU's bfloat16 rounding points and the MoE blocks of oracle/blocks_ref.py), teacher-forced on a shortened stack:
a prompt read in windows of 8 tokens, then a verify pass of 1 + 4 tokens; the logits close to the oracle's and the
top-1 token the oracle's wherever the oracle's best two logits are apart by more than the logits' error."""

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
    pos, checked, matched = 0, 0, 0
    for w in (8, 8, 8, 5):  # three windows of a prompt, then a verify pass of 1 + 4 tokens
        win = tokens[pos : pos + w]
        got = dec.forward(torch.from_numpy(win).cuda(), cache).cpu().numpy()
        dec.advance(cache, w)
        torch.cuda.synchronize()
        dec.check_errors()
        want = D.oracle_forward(dec, win, ck, cv, pos, blocks)
        diff = np.abs(got - want).max()
        assert diff <= 0.05 * np.abs(want).max(), (pos, diff)
        for i in range(w):
            top2 = np.sort(want[i])[-2:]
            if top2[1] - top2[0] > 2 * diff:
                checked += 1
                matched += int(np.argmax(got[i]) == np.argmax(want[i]))
        pos += w
    assert int(cache.pos.item()) == 29
    assert checked >= 20 and matched == checked, (checked, matched)
